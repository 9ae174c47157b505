// Expert residency and admission for layers whose experts do not all fit on the device: a bank of
// `slots` device slots, and the reference's admission rules for which routed expert earns a slot
// (llama_moe_cache in third_party/patches/llama-b11669-hybrid-experts.patch:2174-2294, the admission
// step :3086-3160).  Host-only logic; the device side (uploads, slot remapping) is in umsx_api.cu.
//
//   LFU ("Avalon's rule", hybrid patch :2188-2201, :3091-3101, :3121-3137): per-expert demand counts
//     capped at 15 and halved whenever the demands since the last halving reach `window` slots' worth
//     (window ramps from 2 to 5 as demands accumulate, :3095-3096); an expert enters a free slot after
//     `fill_after` demands, replaces the least recently used resident expert (one not selected by this
//     dispatch) only after `admit_after` demands and with a strictly higher count; at most four
//     admissions per layer per dispatch.
//   LRU (:3138-3145): a missing expert takes a free slot or the least recently used resident expert's
//     slot (one not selected by this dispatch).
// Admission runs on single-token dispatches only; a dispatch of several tokens looks its experts up
// and changes no residency (no slot may be evicted while a position of the block still needs it,
// hybrid patch :3251-3256).  A missing expert that is not admitted is still computed on the device:
// it is uploaded into a transient slot for this call only (the reference computes it on the CPU).
#pragma once

#include <stdint.h>

#include <algorithm>
#include <vector>

namespace umsx {

enum { kBankLfu = 0, kBankLru = 1 };

struct BankStats {
    uint64_t dispatches = 0, demands = 0, hits = 0, misses = 0, admissions = 0, evictions = 0, transient = 0,
             halvings = 0;
};

class BankPolicy {
public:
    BankPolicy(int experts, int slots, int policy, int fill_after = 1, int admit_after = 6)
        : policy_(policy), fill_after_(fill_after), admit_after_(admit_after), slot_of_(experts, -1),
          key_of_(slots, -1), last_seen_(experts, 0), count_(experts, 0) {}

    // One dispatch of one layer.  `selected` are the experts its tokens chose: for one token its
    // top-k in rank order (admit = true), for several tokens the distinct experts in first-use order
    // (admit = false: a lookup).  Returns, for every selected expert, its bank slot after admission or
    // -1 if it stays non-resident (computed from a transient slot); `admitted` lists the (expert, slot)
    // uploads, `evicted` the experts that left the bank.
    std::vector<int> dispatch(const std::vector<int> &selected, std::vector<std::pair<int, int>> &admitted,
                              std::vector<int> &evicted, bool admit = true) {
        admitted.clear();
        evicted.clear();
        ++dispatch_calls_;
        ++stats_.dispatches;
        stats_.demands += selected.size();
        if (!admit) {
            std::vector<int> out(selected.size());
            for (size_t i = 0; i < selected.size(); ++i) {
                out[i] = slot_of_[selected[i]];
                if (out[i] >= 0) ++stats_.hits;
                else { ++stats_.misses; ++stats_.transient; }
            }
            return out;
        }
        for (int key : selected) last_seen_[key] = dispatch_calls_;
        if (policy_ == kBankLfu) {
            for (int key : selected) count_[key] += count_[key] < kCap;
            demands_ += selected.size();
            renewed_ += selected.size();
            const double entries = (double)std::max<size_t>(key_of_.size(), 1);
            const double window = std::min(5.0, 2.0 + 3.0 * (double)renewed_ / (20.0 * entries));
            if ((double)demands_ >= window * entries) {
                demands_ = 0;
                ++stats_.halvings;
                for (auto &c : count_) c >>= 1;
            }
        }
        int inserts = 0;
        for (int key : selected) {
            if (slot_of_[key] >= 0) { ++stats_.hits; continue; }
            ++stats_.misses;
            if (policy_ == kBankLfu && (count_[key] < std::min(fill_after_, admit_after_) || inserts >= kInsertsPerLayer))
                continue;
            int victim_slot = -1;
            uint64_t oldest = UINT64_MAX;
            for (int slot = 0; slot < (int)key_of_.size(); ++slot) {
                const int victim = key_of_[slot];
                if (victim < 0) { victim_slot = slot; break; }
                if (last_seen_[victim] >= dispatch_calls_) continue;  // selected by this dispatch
                if (last_seen_[victim] < oldest) { oldest = last_seen_[victim]; victim_slot = slot; }
            }
            if (victim_slot < 0) continue;
            const int victim = key_of_[victim_slot];
            if (policy_ == kBankLfu) {
                if (count_[key] < (victim < 0 ? fill_after_ : admit_after_)) continue;
                if (victim >= 0 && count_[victim] >= count_[key]) continue;
                ++inserts;
            }
            if (victim >= 0) {
                slot_of_[victim] = -1;
                evicted.push_back(victim);
                ++stats_.evictions;
            }
            key_of_[victim_slot] = key;
            slot_of_[key] = victim_slot;
            admitted.emplace_back(key, victim_slot);
            ++stats_.admissions;
        }
        std::vector<int> out(selected.size());
        for (size_t i = 0; i < selected.size(); ++i) {
            out[i] = slot_of_[selected[i]];
            stats_.transient += out[i] < 0;
        }
        return out;
    }

    const BankStats &stats() const { return stats_; }
    int slot_of(int expert) const { return slot_of_[expert]; }
    int slots() const { return (int)key_of_.size(); }

private:
    static constexpr uint16_t kCap = 15;
    static constexpr int kInsertsPerLayer = 4;
    int policy_, fill_after_, admit_after_;
    std::vector<int> slot_of_, key_of_;
    std::vector<uint64_t> last_seen_;
    std::vector<uint16_t> count_;
    uint64_t dispatch_calls_ = 0, demands_ = 0, renewed_ = 0;
    BankStats stats_;
};

}  // namespace umsx
