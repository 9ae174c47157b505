"""Restatement of the reference's expert-residency admission rules -- TEST INFRASTRUCTURE ONLY.

Only tests/ import this module; the product's policy is unified-memory-scheduler_b200/csrc/umsx_bank.h.

Follows llama_moe_cache in third_party/patches/llama-b11669-hybrid-experts.patch:
  state and constants           :2186-2203 (lfu_cap 15, lfu_admit_after 6, lfu_fill_after 1,
                                 lfu_inserts_per_layer 4; the "lru" policy sets admission_margin 1, :2388)
  single-token dispatch         :3258-3265 (selected = the token's top-k in rank order, then admit)
  batch dispatch                :3251-3256 (dispatch_calls advances; nothing is admitted or evicted)
  admit                         :3087-3160 (last_seen, LFU counts / halving window, victim search,
                                 LFU count rules, insert cap; LRU takes the victim without count rules)
One instance models one layer's bank (the reference's lfu_entries, the admissible slots over all
groups, is that bank's slot count when one layer is banked).  Parity is pinned by this
restatement and the known-answer cases in tests/test_bank_policy.py (the reference engine is a
llama.cpp patch that is not built here; its own tests cover the offline trace simulator, a
different tool).
"""
from __future__ import annotations

LFU, LRU = 0, 1
STAT_NAMES = ("dispatches", "demands", "hits", "misses", "admissions", "evictions", "transient", "halvings",
              "upload_bytes")


class RefBank:
    CAP = 15
    INSERTS_PER_LAYER = 4

    def __init__(self, experts: int, slots: int, policy: int, fill_after: int = 1, admit_after: int = 6):
        self.policy = policy
        self.fill_after, self.admit_after = fill_after, admit_after
        self.slot_map = [-1] * experts    # expert -> slot
        self.key_of = [-1] * slots        # slot -> expert
        self.last_seen = [0] * experts
        self.count = [0] * experts
        self.dispatch_calls = 0
        self.lfu_demands = 0
        self.lfu_renewed = 0
        self.stats = dict.fromkeys(STAT_NAMES, 0)

    def _victim(self):
        victim_slot, oldest = -1, None
        for slot, victim in enumerate(self.key_of):
            if victim < 0:
                return slot
            if self.last_seen[victim] >= self.dispatch_calls:
                continue
            if oldest is None or self.last_seen[victim] < oldest:
                oldest, victim_slot = self.last_seen[victim], slot
        return victim_slot

    def dispatch(self, selected: list[int], admit: bool) -> list[int]:
        self.dispatch_calls += 1
        st = self.stats
        st["dispatches"] += 1
        st["demands"] += len(selected)
        if admit:
            for key in selected:
                self.last_seen[key] = self.dispatch_calls
            if self.policy == LFU:
                for key in selected:
                    if self.count[key] < self.CAP:
                        self.count[key] += 1
                self.lfu_demands += len(selected)
                self.lfu_renewed += len(selected)
                entries = float(max(len(self.key_of), 1))
                window = min(5.0, 2.0 + 3.0 * self.lfu_renewed / (20.0 * entries))
                if self.lfu_demands >= window * entries:
                    self.lfu_demands = 0
                    st["halvings"] += 1
                    self.count = [c >> 1 for c in self.count]
            inserts = 0
            for key in selected:
                if self.slot_map[key] >= 0:
                    st["hits"] += 1
                    continue
                st["misses"] += 1
                if self.policy == LFU and (self.count[key] < min(self.fill_after, self.admit_after)
                                           or inserts >= self.INSERTS_PER_LAYER):
                    continue
                slot = self._victim()
                if slot < 0:
                    continue
                victim = self.key_of[slot]
                if self.policy == LFU:
                    if self.count[key] < (self.fill_after if victim < 0 else self.admit_after):
                        continue
                    if victim >= 0 and self.count[victim] >= self.count[key]:
                        continue
                    inserts += 1
                if victim >= 0:
                    self.slot_map[victim] = -1
                    st["evictions"] += 1
                self.key_of[slot] = key
                self.slot_map[key] = slot
                st["admissions"] += 1
        out = [self.slot_map[k] for k in selected]
        if not admit:
            st["hits"] += sum(s >= 0 for s in out)
            st["misses"] += sum(s < 0 for s in out)
        st["transient"] += sum(s < 0 for s in out)
        return out
