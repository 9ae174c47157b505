// C ABI of libumsx: handle lifecycle, weight upload / repack, and the entry
// points declared in include/umsx.h.  No exception crosses the ABI; failures
// set a thread-local message and return a umsx_status.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "umsx_bank.h"
#include "umsx_internal.h"

using namespace umsx;

namespace {

thread_local std::string g_error;
thread_local uint64_t g_launches = 0;

umsx_status fail(umsx_status s, const std::string &msg) {
    g_error = msg;
    return s;
}

#define UMSX_CUDA(call)                                                                        \
    do {                                                                                       \
        cudaError_t err_ = (call);                                                             \
        if (err_ != cudaSuccess) return fail(UMSX_EDEVICE, std::string(#call) + ": " + cudaGetErrorString(err_)); \
    } while (0)

#define UMSX_LAUNCHED(n)                                                                       \
    do {                                                                                       \
        g_launches += (uint64_t)(n);                                                           \
        cudaError_t err_ = cudaGetLastError();                                                 \
        if (err_ != cudaSuccess) return fail(UMSX_EDEVICE, std::string("kernel launch: ") + cudaGetErrorString(err_)); \
    } while (0)

constexpr size_t kAlign = 256;
inline size_t align_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

// Bump allocator over one device allocation.
struct Arena {
    uint8_t *base = nullptr;
    size_t used = 0, size = 0;
    template <class T>
    T *take(size_t count) {
        const size_t off = used;
        used = align_up(used + count * sizeof(T));
        return base ? reinterpret_cast<T *>(base + off) : nullptr;
    }
};

float normal_scale(double sigma) { return (float)(sigma * std::sqrt(3.0) / 16777216.0); }

uint64_t stream_id(uint32_t layer, int kind) { return (uint64_t)layer * 16u + (uint64_t)kind; }

size_t block_bytes(int quant) { return quant == UMSX_QUANT_MXFP4 ? 17 : 34; }

}  // namespace

namespace umsx {
void record_error(const char *msg) { g_error = msg; }
void record_launches(uint64_t kernels) { g_launches += kernels; }
}  // namespace umsx

// Per-call scratch: the router's dispatch state, the quantized activations,
// the per-job expert outputs and forward_host staging.  A layer owns one; a
// stack owns one shared by all of its layers (they run one after another).
struct Workspace {
    Dispatch disp{};
    uint8_t *act_codes = nullptr;
    float *act_scales = nullptr;
    float *act_f32 = nullptr;
    uint8_t *act_rec = nullptr;
    float *act_sc = nullptr;
    uint32_t *act_done = nullptr;
    float *y = nullptr;
    void *x_dev = nullptr;
    float *out_dev = nullptr;
    unsigned *bar = nullptr;  // grid barrier counter of the persistent decode kernel
    uint16_t *a16 = nullptr;    // prefill: x rows in job order as f16 Q8_0 values, hi then lo [2][T*K][H]
    uint16_t *act16 = nullptr;  // prefill: activations as f16 Q8_0 values, hi then lo [2][T*K][I]
    int32_t *inv = nullptr;   // prefill: (token, rank) -> job row
    uint8_t *mem = nullptr;
    int max_tokens = 0;
};

struct umsx_moe {
    umsx_moe_desc d{};
    int device = 0;
    int e_lo = 0, e_local = 0;
    float *router_w = nullptr, *router_b = nullptr;
    Matrix gate_up, gate, up, down;
    float *gu_bias = nullptr, *down_bias = nullptr;
    uint8_t *weights_mem = nullptr;
    Workspace ws;
    std::mutex mu;
    // Residency bank (umsx_moe_create_banked): the device planes hold bank_slots experts admitted by
    // the policy plus bank_total - bank_slots transient slots for the misses of one call; every expert
    // stays in pinned host memory (ggml blocks) and is uploaded on admission or on demand.
    bool banked = false;
    int bank_slots = 0, bank_total = 0;
    umsx::BankPolicy *policy = nullptr;
    uint8_t *host_blocks[3] = {};  // [E][per] ggml blocks: gate_up or gate, up (separate), down
    size_t host_per[3] = {};
    float *host_gu_bias = nullptr, *host_dn_bias = nullptr;  // [E][2I], [E][H] fp32
    int32_t *d_map = nullptr;       // [E] expert -> device slot for the current call
    uint8_t *bank_staging = nullptr;
    uint64_t upload_bytes = 0;
};

namespace {

umsx_status validate_desc(const umsx_moe_desc *d) {
    if (!d) return fail(UMSX_EINVAL, "null descriptor");
    if (d->hidden <= 0 || d->hidden % 64 || d->intermediate <= 0 || d->intermediate % 64)
        return fail(UMSX_EINVAL, "hidden and intermediate must be positive multiples of 64");
    if (d->experts <= 0 || d->experts > 1024 || d->top_k <= 0 || d->top_k > 32 || d->top_k > d->experts)
        return fail(UMSX_EINVAL, "need 1 <= top_k <= min(32, experts) and experts <= 1024");
    if (d->quant != UMSX_QUANT_MXFP4 && d->quant != UMSX_QUANT_Q8_0) return fail(UMSX_EUNSUPPORTED, "quant must be MXFP4 or Q8_0");
    if (d->routing < 0 || d->routing > 2) return fail(UMSX_EINVAL, "unknown routing mode");
    if (d->activation != UMSX_ACT_SILU && d->activation != UMSX_ACT_SWIGLU_OAI) return fail(UMSX_EINVAL, "unknown activation");
    if (d->max_tokens <= 0 || d->max_tokens > 65536) return fail(UMSX_EINVAL, "max_tokens must be in [1, 65536]");
    const int world = d->ep_world <= 0 ? 1 : d->ep_world;
    if (d->experts % world || d->ep_rank < 0 || d->ep_rank >= world)
        return fail(UMSX_EINVAL, "experts must split evenly over ep_world and 0 <= ep_rank < ep_world");
    return UMSX_OK;
}

size_t weight_bytes(const umsx_moe *m, Arena &a) {
    const auto &d = m->d;
    const int H = d.hidden, I = d.intermediate, E = d.experts, EL = m->banked ? m->bank_total : m->e_local;
    a.take<float>((size_t)E * H);
    if (d.has_router_bias) a.take<float>(E);
    auto mat = [&](Matrix &mm, int rows, int cols) {
        mm.rows = rows;
        mm.cols = cols;
        mm.quant = d.quant;
        mm.codes = a.take<uint8_t>(mm.code_bytes_per_expert() * EL);
        mm.scales = a.take<uint8_t>(mm.scale_bytes_per_expert() * EL);
        mm.emax = d.quant == UMSX_QUANT_MXFP4 ? a.take<uint8_t>((size_t)rows * EL) : nullptr;
    };
    Matrix tmp;
    if (d.fused_gate_up) mat(tmp, 2 * I, H);
    else { mat(tmp, I, H); mat(tmp, I, H); }
    mat(tmp, H, I);
    if (d.has_bias) { a.take<float>((size_t)EL * 2 * I); a.take<float>((size_t)EL * H); }
    return a.used;
}

void carve_weights(umsx_moe *m, Arena &a) {
    const auto &d = m->d;
    const int H = d.hidden, I = d.intermediate, E = d.experts, EL = m->banked ? m->bank_total : m->e_local;
    m->router_w = a.take<float>((size_t)E * H);
    if (d.has_router_bias) m->router_b = a.take<float>(E);
    auto mat = [&](Matrix &mm, int rows, int cols) {
        mm.rows = rows;
        mm.cols = cols;
        mm.quant = d.quant;
        mm.codes = a.take<uint8_t>(mm.code_bytes_per_expert() * EL);
        mm.scales = a.take<uint8_t>(mm.scale_bytes_per_expert() * EL);
        mm.emax = d.quant == UMSX_QUANT_MXFP4 ? a.take<uint8_t>((size_t)rows * EL) : nullptr;
    };
    if (d.fused_gate_up) mat(m->gate_up, 2 * I, H);
    else { mat(m->gate, I, H); mat(m->up, I, H); }
    mat(m->down, H, I);
    if (d.has_bias) {
        m->gu_bias = a.take<float>((size_t)EL * 2 * I);
        m->down_bias = a.take<float>((size_t)EL * H);
    }
}

void carve_workspace(Workspace &w, const umsx_moe_desc &d, int e_local, int max_tokens, Arena &a) {
    const size_t T = max_tokens, K = d.top_k, E = d.experts, EL = e_local, H = d.hidden, I = d.intermediate;
    Dispatch &p = w.disp;
    p.logits = a.take<float>(T * E);
    p.ids = a.take<int32_t>(T * K);
    p.weights = a.take<float>(T * K);
    p.token_done = a.take<uint32_t>(T);
    p.all_done = a.take<uint32_t>(1);
    p.counts = a.take<int32_t>(EL);
    p.offsets = a.take<int32_t>(EL + 1);
    p.active = a.take<int32_t>(EL);
    p.n_active = a.take<int32_t>(1);
    p.job_token = a.take<int32_t>(T * K);
    p.job_rank = a.take<int32_t>(T * K);
    p.xq_codes = a.take<uint8_t>(T * H);
    p.xq_scales = a.take<float>(T * (H / 32));
    p.slots = a.take<int4>(EL);
    p.tile_done = a.take<uint32_t>(T * (H / 32));
    w.act_codes = a.take<uint8_t>(T * K * I);
    w.act_scales = a.take<float>(T * K * (I / 32));
    const bool mx = d.quant == UMSX_QUANT_MXFP4;
    const size_t nbH = H / 32, nbI = I / 32;
    w.act_f32 = mx ? a.take<float>(T * K * I) : nullptr;
    w.act_rec = mx ? a.take<uint8_t>(T * K * nbI * 64) : nullptr;
    w.act_sc = mx ? a.take<float>(T * K * ((nbI + 3) & ~size_t(3))) : nullptr;
    w.act_done = mx ? a.take<uint32_t>(T * K * nbI) : nullptr;
    p.xr = mx ? a.take<uint8_t>(T * nbH * 64) : nullptr;
    p.xr_sc = mx ? a.take<float>(T * ((nbH + 3) & ~size_t(3))) : nullptr;
    p.err = a.take<uint32_t>(1);
    w.y = a.take<float>(T * K * H);
    w.x_dev = a.take<float>(T * H);
    w.out_dev = a.take<float>(T * H);
    w.bar = a.take<unsigned>(1);
    if (max_tokens >= kPrefillMinTokens) {  // tensor-core prefill operands
        w.a16 = a.take<uint16_t>(2 * T * K * H);
        w.act16 = a.take<uint16_t>(2 * T * K * I);
        w.inv = a.take<int32_t>(T * K);
    }
    w.max_tokens = max_tokens;
}

// Allocates and zeroes a workspace (the router's completion counters must start at zero).
umsx_status alloc_workspace(Workspace &w, const umsx_moe_desc &d, int e_local, int max_tokens, size_t reserve) {
    Arena probe;
    carve_workspace(w, d, e_local, max_tokens, probe);
    size_t free_b = 0, total_b = 0;
    UMSX_CUDA(cudaMemGetInfo(&free_b, &total_b));
    if (free_b < reserve || probe.used + (64u << 20) > free_b - reserve)
        return fail(UMSX_EOOM, "workspace of " + std::to_string(probe.used) + " bytes would violate the free-memory reserve");
    UMSX_CUDA(cudaMalloc(&w.mem, probe.used));
    Arena a{w.mem, 0, probe.used};
    carve_workspace(w, d, e_local, max_tokens, a);
    UMSX_CUDA(cudaMemset(w.mem, 0, probe.used));
    return UMSX_OK;
}

umsx_status allocate(umsx_moe *m, size_t reserve) {
    Arena wa;
    const size_t wbytes = weight_bytes(m, wa);
    size_t free_b = 0, total_b = 0;
    UMSX_CUDA(cudaMemGetInfo(&free_b, &total_b));
    if (free_b < reserve || wbytes + (64u << 20) > free_b - reserve)
        return fail(UMSX_EOOM, "allocation of " + std::to_string(wbytes) + " weight bytes would violate the " +
                                   std::to_string(reserve) + "-byte free-memory reserve");
    UMSX_CUDA(cudaMalloc(&m->weights_mem, wbytes));
    UMSX_CUDA(cudaMemset(m->weights_mem, 0, wbytes));  // defined padding bytes
    Arena w2{m->weights_mem, 0, wbytes};
    carve_weights(m, w2);
    return alloc_workspace(m->ws, m->d, m->e_local, m->d.max_tokens, reserve);
}

umsx_status make_handle(const umsx_moe_desc *desc, int device, size_t reserve, umsx_moe **out, int bank_slots = 0) {
    if (!out) return fail(UMSX_EINVAL, "null output handle pointer");
    *out = nullptr;
    if (umsx_status s = validate_desc(desc)) return s;
    int count = 0;
    UMSX_CUDA(cudaGetDeviceCount(&count));
    if (device < 0 || device >= count) return fail(UMSX_EINVAL, "device index out of range");
    UMSX_CUDA(cudaSetDevice(device));
    auto *m = new umsx_moe();
    m->d = *desc;
    if (bank_slots > 0) {
        m->banked = true;
        m->bank_slots = bank_slots;
        m->bank_total = bank_slots + std::min(desc->experts, desc->max_tokens * desc->top_k);
    }
    if (m->d.ep_world <= 0) m->d.ep_world = 1;
    m->device = device;
    m->e_local = desc->experts / m->d.ep_world;
    m->e_lo = m->d.ep_rank * m->e_local;
    if (umsx_status s = allocate(m, reserve)) {
        umsx_moe_destroy(m);
        return s;
    }
    *out = m;
    return UMSX_OK;
}

// Upload expert `le` of a matrix from ggml-layout host bytes through a device staging buffer.
umsx_status upload_matrix(Matrix &mm, const void *host_all, int e_global_lo, int e_local, uint8_t *staging) {
    const size_t per = (size_t)mm.rows * (mm.cols / 32) * block_bytes(mm.quant);
    for (int le = 0; le < e_local; ++le) {
        const uint8_t *src = static_cast<const uint8_t *>(host_all) + (size_t)(e_global_lo + le) * per;
        UMSX_CUDA(cudaMemcpy(staging, src, per, cudaMemcpyHostToDevice));
        UMSX_LAUNCHED(launch_repack(mm, le, staging, 0));
    }
    return UMSX_OK;
}

umsx_status generate_matrix(Matrix &mm, uint64_t seed, uint64_t stream, int e_global_lo, int e_local, uint8_t *staging) {
    const uint64_t nblk = (uint64_t)mm.rows * (mm.cols / 32);
    for (int le = 0; le < e_local; ++le) {
        UMSX_LAUNCHED(launch_gen_blocks(mm.quant, seed, stream, (uint64_t)(e_global_lo + le) * nblk, nblk, staging, 0));
        UMSX_LAUNCHED(launch_repack(mm, le, staging, 0));
    }
    return UMSX_OK;
}

// Row exponent maxima of the MXFP4 matrices (the prefill path's f16 rebase), and whether every block
// exponent of a matrix is >= 2 (Matrix::exp_ge2: the decode kernels then take the normal-scale form).
umsx_status compute_row_emax(umsx_moe *m) {
    if (m->d.quant != UMSX_QUANT_MXFP4) return UMSX_OK;
    uint32_t *low = nullptr;
    UMSX_CUDA(cudaMalloc(&low, 4 * 4));
    auto run = [&]() -> umsx_status {
        UMSX_CUDA(cudaMemset(low, 0, 4 * 4));
        Matrix *mats[4] = {&m->gate_up, &m->gate, &m->up, &m->down};
        for (int i = 0; i < 4; ++i)
            if (mats[i]->codes) UMSX_LAUNCHED(launch_row_emax(*mats[i], m->e_local, mats[i]->emax, low + i, 0));
        uint32_t h[4] = {1, 1, 1, 1};
        UMSX_CUDA(cudaMemcpy(h, low, sizeof(h), cudaMemcpyDeviceToHost));
        for (int i = 0; i < 4; ++i) mats[i]->exp_ge2 = mats[i]->codes && h[i] == 0;
        return UMSX_OK;
    };
    const umsx_status st = run();
    cudaFree(low);
    return st;
}

size_t max_expert_bytes(const umsx_moe *m) {
    const auto &d = m->d;
    const size_t bb = block_bytes(d.quant);
    const size_t gu = (size_t)(d.fused_gate_up ? 2 : 1) * d.intermediate * (d.hidden / 32) * bb;
    const size_t dn = (size_t)d.hidden * (d.intermediate / 32) * bb;
    return std::max(gu, dn);
}

bool resident(const umsx_moe *m, int e) { return e >= m->e_lo && e < m->e_lo + m->e_local; }

umsx_status create_from_host(const umsx_moe_desc *desc, const umsx_moe_weights *w, const float *gu_bias,
                             const float *down_bias, int device, size_t reserve_bytes, umsx_moe **out);

}  // namespace

extern "C" {

int umsx_version(void) { return UMSX_VERSION; }

const char *umsx_last_error(void) { return g_error.c_str(); }

uint64_t umsx_kernel_launches(void) { return g_launches; }

umsx_status umsx_moe_create(const umsx_moe_desc *desc, const umsx_moe_weights *w, int device, size_t reserve_bytes,
                            umsx_moe **out) {
    if (!w || !w->router_w || !w->down || (desc && desc->fused_gate_up ? !w->gate_up : (!w->gate || !w->up)))
        return fail(UMSX_EINVAL, "missing router, gate/up or down weights");
    if (desc && desc->has_router_bias && !w->router_b) return fail(UMSX_EINVAL, "has_router_bias set but router_b is null");
    if (desc && desc->has_bias && (!w->gate_up_bias || !w->down_bias)) return fail(UMSX_EINVAL, "has_bias set but biases are null");
    std::vector<float> gb, db;  // bf16 biases widened (exact)
    if (desc && desc->has_bias && desc->experts > 0 && desc->intermediate > 0 && desc->hidden > 0) {
        gb.resize((size_t)desc->experts * 2 * desc->intermediate);
        db.resize((size_t)desc->experts * desc->hidden);
        for (size_t i = 0; i < gb.size(); ++i) {
            const uint32_t bits = (uint32_t)w->gate_up_bias[i] << 16;
            std::memcpy(&gb[i], &bits, 4);
        }
        for (size_t i = 0; i < db.size(); ++i) {
            const uint32_t bits = (uint32_t)w->down_bias[i] << 16;
            std::memcpy(&db[i], &bits, 4);
        }
    }
    return create_from_host(desc, w, gb.data(), db.data(), device, reserve_bytes, out);
}

umsx_status umsx_moe_create_banked(const umsx_moe_desc *desc, const umsx_moe_weights *w, int slots, int policy,
                                   int device, size_t reserve_bytes, umsx_moe **out) {
    if (out) *out = nullptr;
    if (!w || !w->router_w || !w->down || (desc && desc->fused_gate_up ? !w->gate_up : (!w->gate || !w->up)))
        return fail(UMSX_EINVAL, "missing router, gate/up or down weights");
    if (desc && desc->has_router_bias && !w->router_b) return fail(UMSX_EINVAL, "has_router_bias set but router_b is null");
    if (desc && desc->has_bias && (!w->gate_up_bias || !w->down_bias)) return fail(UMSX_EINVAL, "has_bias set but biases are null");
    if (policy != UMSX_BANK_LFU && policy != UMSX_BANK_LRU) return fail(UMSX_EINVAL, "unknown bank policy");
    if (desc && desc->ep_world > 1) return fail(UMSX_EINVAL, "a banked layer holds every expert of its layer (ep_world 1)");
    if (!desc || slots < 1 || slots > desc->experts) return fail(UMSX_EINVAL, "bank slots must be in [1, experts]");
    umsx_moe *m = nullptr;
    if (umsx_status s = make_handle(desc, device, reserve_bytes, &m, slots)) return s;
    const auto &d = m->d;
    const size_t H = d.hidden, I = d.intermediate, E = d.experts;
    auto run = [&]() -> umsx_status {
        UMSX_CUDA(cudaMemcpy(m->router_w, w->router_w, E * H * sizeof(float), cudaMemcpyHostToDevice));
        if (d.has_router_bias) UMSX_CUDA(cudaMemcpy(m->router_b, w->router_b, E * sizeof(float), cudaMemcpyHostToDevice));
        const void *src[3] = {d.fused_gate_up ? w->gate_up : w->gate, d.fused_gate_up ? nullptr : w->up, w->down};
        const Matrix *mats[3] = {d.fused_gate_up ? &m->gate_up : &m->gate, &m->up, &m->down};
        for (int i = 0; i < 3; ++i) {
            if (!src[i]) continue;
            m->host_per[i] = (size_t)mats[i]->rows * (mats[i]->cols / 32) * block_bytes(d.quant);
            UMSX_CUDA(cudaMallocHost(&m->host_blocks[i], E * m->host_per[i]));
            std::memcpy(m->host_blocks[i], src[i], E * m->host_per[i]);
        }
        if (d.has_bias) {  // bf16 biases widened (exact)
            UMSX_CUDA(cudaMallocHost(&m->host_gu_bias, E * 2 * I * 4));
            UMSX_CUDA(cudaMallocHost(&m->host_dn_bias, E * H * 4));
            for (size_t i = 0; i < E * 2 * I; ++i) {
                const uint32_t bits = (uint32_t)w->gate_up_bias[i] << 16;
                std::memcpy(&m->host_gu_bias[i], &bits, 4);
            }
            for (size_t i = 0; i < E * H; ++i) {
                const uint32_t bits = (uint32_t)w->down_bias[i] << 16;
                std::memcpy(&m->host_dn_bias[i], &bits, 4);
            }
        }
        UMSX_CUDA(cudaMalloc(&m->bank_staging, max_expert_bytes(m)));
        UMSX_CUDA(cudaMalloc(&m->d_map, E * sizeof(int32_t)));
        m->policy = new BankPolicy((int)E, slots, policy == UMSX_BANK_LFU ? kBankLfu : kBankLru);
        UMSX_CUDA(cudaDeviceSynchronize());
        return UMSX_OK;
    };
    if (umsx_status st = run()) { umsx_moe_destroy(m); return st; }
    *out = m;
    return UMSX_OK;
}

umsx_status umsx_moe_bank_stats(umsx_moe *m, uint64_t *stats, int n, int32_t *slot_of_expert, int n_experts) {
    if (!m || !m->banked) return fail(UMSX_EINVAL, "not a banked layer");
    if ((stats && n < UMSX_BANK_STATS) || (slot_of_expert && n_experts < m->d.experts))
        return fail(UMSX_EINVAL, "output arrays too small");
    std::lock_guard<std::mutex> lock(m->mu);
    if (stats) {
        const BankStats &b = m->policy->stats();
        const uint64_t v[UMSX_BANK_STATS] = {b.dispatches, b.demands, b.hits, b.misses, b.admissions,
                                             b.evictions, b.transient, b.halvings, m->upload_bytes};
        std::memcpy(stats, v, sizeof(v));
    }
    if (slot_of_expert)
        for (int e = 0; e < m->d.experts; ++e) slot_of_expert[e] = m->policy->slot_of(e);
    return UMSX_OK;
}

umsx_status umsx_bank_simulate(int experts, int slots, int policy, int n_dispatches, const int32_t *counts,
                               const int32_t *selected, int32_t *slot_out, uint64_t *stats) {
    if (experts < 1 || slots < 1 || slots > experts || n_dispatches < 0 || (n_dispatches && (!counts || !selected)))
        return fail(UMSX_EINVAL, "bad bank simulation arguments");
    if (policy != UMSX_BANK_LFU && policy != UMSX_BANK_LRU) return fail(UMSX_EINVAL, "unknown bank policy");
    BankPolicy bank(experts, slots, policy == UMSX_BANK_LFU ? kBankLfu : kBankLru);
    std::vector<std::pair<int, int>> admitted;
    std::vector<int> evicted;
    size_t at = 0;
    for (int i = 0; i < n_dispatches; ++i) {
        if (counts[i] == 0) return fail(UMSX_EINVAL, "empty dispatch");
        // counts[i] > 0: one token's top-k (admission); counts[i] < 0: the distinct experts of a batch
        const int c = counts[i] < 0 ? -counts[i] : counts[i];
        std::vector<int> sel(selected + at, selected + at + c);
        for (int e : sel)
            if (e < 0 || e >= experts) return fail(UMSX_EINVAL, "expert index out of range");
        const std::vector<int> sl = bank.dispatch(sel, admitted, evicted, counts[i] > 0);
        if (slot_out) std::copy(sl.begin(), sl.end(), slot_out + at);
        at += c;
    }
    if (stats) {
        const BankStats &b = bank.stats();
        const uint64_t v[UMSX_BANK_STATS] = {b.dispatches, b.demands, b.hits, b.misses, b.admissions,
                                             b.evictions, b.transient, b.halvings, 0};
        std::memcpy(stats, v, sizeof(v));
    }
    return UMSX_OK;
}

}  // extern "C"

namespace {
// Creates a layer from host weights with fp32 biases (gu_bias [E][2I]: gate then up; down_bias [E][H]).
umsx_status create_from_host(const umsx_moe_desc *desc, const umsx_moe_weights *w, const float *gu_bias,
                             const float *down_bias, int device, size_t reserve_bytes, umsx_moe **out) {
    umsx_moe *m = nullptr;
    if (umsx_status s = make_handle(desc, device, reserve_bytes, &m)) return s;
    const auto &d = m->d;
    const int H = d.hidden, I = d.intermediate, E = d.experts;
    uint8_t *staging = nullptr;
    umsx_status st = UMSX_OK;
    auto run = [&]() -> umsx_status {
        UMSX_CUDA(cudaMemcpy(m->router_w, w->router_w, (size_t)E * H * sizeof(float), cudaMemcpyHostToDevice));
        if (d.has_router_bias) UMSX_CUDA(cudaMemcpy(m->router_b, w->router_b, (size_t)E * sizeof(float), cudaMemcpyHostToDevice));
        UMSX_CUDA(cudaMalloc(&staging, max_expert_bytes(m)));
        if (d.fused_gate_up) {
            if (umsx_status s = upload_matrix(m->gate_up, w->gate_up, m->e_lo, m->e_local, staging)) return s;
        } else {
            if (umsx_status s = upload_matrix(m->gate, w->gate, m->e_lo, m->e_local, staging)) return s;
            if (umsx_status s = upload_matrix(m->up, w->up, m->e_lo, m->e_local, staging)) return s;
        }
        if (umsx_status s = upload_matrix(m->down, w->down, m->e_lo, m->e_local, staging)) return s;
        if (d.has_bias) {
            UMSX_CUDA(cudaMemcpy(m->gu_bias, gu_bias + (size_t)m->e_lo * 2 * I, (size_t)m->e_local * 2 * I * 4,
                                 cudaMemcpyHostToDevice));
            UMSX_CUDA(cudaMemcpy(m->down_bias, down_bias + (size_t)m->e_lo * H, (size_t)m->e_local * H * 4,
                                 cudaMemcpyHostToDevice));
        }
        if (umsx_status s = compute_row_emax(m)) return s;
        UMSX_CUDA(cudaDeviceSynchronize());
        return UMSX_OK;
    };
    st = run();
    if (staging) cudaFree(staging);
    if (st) { umsx_moe_destroy(m); return st; }
    *out = m;
    return UMSX_OK;
}
}  // namespace

extern "C" {

umsx_status umsx_moe_create_synthetic(const umsx_moe_desc *desc, uint64_t seed, uint32_t layer, float router_sigma,
                                      float router_bias_sigma, float bias_sigma, int device, size_t reserve_bytes,
                                      umsx_moe **out) {
    umsx_moe *m = nullptr;
    if (umsx_status s = make_handle(desc, device, reserve_bytes, &m)) return s;
    const auto &d = m->d;
    const int H = d.hidden, I = d.intermediate, E = d.experts;
    uint8_t *staging = nullptr;
    auto run = [&]() -> umsx_status {
        UMSX_LAUNCHED(launch_gen_normal_f32(seed, stream_id(layer, 0), 0, (uint64_t)E * H, normal_scale(router_sigma), m->router_w, 0));
        if (d.has_router_bias)
            UMSX_LAUNCHED(launch_gen_normal_f32(seed, stream_id(layer, 1), 0, (uint64_t)E, normal_scale(router_bias_sigma), m->router_b, 0));
        UMSX_CUDA(cudaMalloc(&staging, max_expert_bytes(m)));
        if (d.fused_gate_up) {
            if (umsx_status s = generate_matrix(m->gate_up, seed, stream_id(layer, 2), m->e_lo, m->e_local, staging)) return s;
        } else {
            if (umsx_status s = generate_matrix(m->gate, seed, stream_id(layer, 2), m->e_lo, m->e_local, staging)) return s;
            if (umsx_status s = generate_matrix(m->up, seed, stream_id(layer, 3), m->e_lo, m->e_local, staging)) return s;
        }
        if (umsx_status s = generate_matrix(m->down, seed, stream_id(layer, 4), m->e_lo, m->e_local, staging)) return s;
        if (d.has_bias) {
            UMSX_LAUNCHED(launch_gen_normal_bf16_to_f32(seed, stream_id(layer, 5), (uint64_t)m->e_lo * 2 * I,
                                                        (uint64_t)m->e_local * 2 * I, normal_scale(bias_sigma), m->gu_bias, 0));
            UMSX_LAUNCHED(launch_gen_normal_bf16_to_f32(seed, stream_id(layer, 6), (uint64_t)m->e_lo * H,
                                                        (uint64_t)m->e_local * H, normal_scale(bias_sigma), m->down_bias, 0));
        }
        if (umsx_status s = compute_row_emax(m)) return s;
        UMSX_CUDA(cudaDeviceSynchronize());
        return UMSX_OK;
    };
    const umsx_status st = run();
    if (staging) cudaFree(staging);
    if (st) { umsx_moe_destroy(m); return st; }
    *out = m;
    return UMSX_OK;
}

void umsx_moe_destroy(umsx_moe *m) {
    if (!m) return;
    cudaSetDevice(m->device);
    cudaDeviceSynchronize();
    if (m->weights_mem) cudaFree(m->weights_mem);
    if (m->ws.mem) cudaFree(m->ws.mem);
    for (uint8_t *p : m->host_blocks)
        if (p) cudaFreeHost(p);
    if (m->host_gu_bias) cudaFreeHost(m->host_gu_bias);
    if (m->host_dn_bias) cudaFreeHost(m->host_dn_bias);
    if (m->d_map) cudaFree(m->d_map);
    if (m->bank_staging) cudaFree(m->bank_staging);
    delete m->policy;
    delete m;
}

}  // extern "C"

namespace {

umsx_status check_call(umsx_moe *m, const void *x, int x_dtype, int tokens, int max_tokens) {
    if (!m) return fail(UMSX_EINVAL, "null handle");
    if (!x) return fail(UMSX_EINVAL, "null input");
    if (x_dtype != UMSX_DTYPE_F32 && x_dtype != UMSX_DTYPE_BF16) return fail(UMSX_EINVAL, "x_dtype must be F32 or BF16");
    if (tokens <= 0 || tokens > max_tokens) return fail(UMSX_EINVAL, "tokens must be in [1, max_tokens]");
    if (reinterpret_cast<uintptr_t>(x) % 16) return fail(UMSX_EINVAL, "x must be 16-byte aligned");
    return UMSX_OK;
}

umsx_status run_router(umsx_moe *m, Workspace &ws, const void *x, int x_dtype, int tokens, int rmsnorm, float eps,
                       cudaStream_t s, int skip_counts = 0, int records = -1) {
    RouterParams p{};
    p.x = x;
    p.x_dtype = x_dtype;
    p.tokens = tokens;
    p.hidden = m->d.hidden;
    p.experts = m->d.experts;
    p.top_k = m->d.top_k;
    p.routing = m->d.routing;
    p.routed_scale = m->d.routed_scale;
    p.w = m->router_w;
    p.b = m->router_b;
    p.e_lo = m->e_lo;
    p.e_local = m->e_local;
    p.rmsnorm = rmsnorm;
    p.eps = eps;
    p.skip_counts = skip_counts;
    p.mx_records = records >= 0 ? records : m->d.quant == UMSX_QUANT_MXFP4;
    UMSX_LAUNCHED(launch_router(p, ws.disp, s));
    return UMSX_OK;
}

// Records an optional timing event; inside stream capture it becomes an external
// event-record node, so a replayed graph still timestamps the stage boundary.
umsx_status mark(cudaEvent_t ev, cudaStream_t s) {
    if (!ev) return UMSX_OK;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    UMSX_CUDA(cudaStreamIsCapturing(s, &cs));
    if (cs == cudaStreamCaptureStatusActive) UMSX_CUDA(cudaEventRecordWithFlags(ev, s, cudaEventRecordExternal));
    else UMSX_CUDA(cudaEventRecord(ev, s));
    return UMSX_OK;
}

// The persistent decode kernel serves a call when every layer is an MXFP4
// fused-gate_up layer with all experts local and the token count is small.
bool decode_eligible(const umsx_moe *m, int tokens, int n_layers) {
    const auto &d = m->d;
    return !m->banked && d.quant == UMSX_QUANT_MXFP4 && d.fused_gate_up && m->e_local == d.experts &&
           decode_supported(tokens, d.hidden, d.intermediate, d.experts, d.top_k, n_layers);
}

DecodeLayer decode_layer(const umsx_moe *m) {
    DecodeLayer L{};
    L.router_w = m->router_w;
    L.router_b = m->router_b;
    L.gu_codes = m->gate_up.codes;
    L.gu_scales = m->gate_up.scales;
    L.gu_bias = m->gu_bias;
    L.dn_codes = m->down.codes;
    L.dn_scales = m->down.scales;
    L.dn_bias = m->down_bias;
    L.gu_ge2 = m->gate_up.exp_ge2;
    L.dn_ge2 = m->down.exp_ge2;
    return L;
}

// Layer l of the persistent kernel's stack.
void set_decode_layer(DecodeParams &p, int l, const umsx_moe *m) { p.layer[l] = decode_layer(m); }

DecodeParams decode_params(const umsx_moe *m, Workspace &ws, const void *x, int x_dtype, int tokens, float *out) {
    const auto &d = m->d;
    DecodeParams p{};
    p.n_layers = 1;
    set_decode_layer(p, 0, m);
    p.tokens = tokens;
    p.hidden = d.hidden;
    p.inter = d.intermediate;
    p.experts = d.experts;
    p.top_k = d.top_k;
    p.routing = d.routing;
    p.activation = d.activation;
    p.routed_scale = d.routed_scale;
    p.alpha = d.swiglu_alpha;
    p.limit = d.swiglu_limit;
    p.x = x;
    p.x_dtype = x_dtype;
    p.out = out;
    p.logits = ws.disp.logits;
    p.act = ws.act_f32;
    p.y = ws.y;
    p.xr = ws.disp.xr;
    p.xr_sc = ws.disp.xr_sc;
    p.bar = ws.bar;
    p.err = ws.disp.err;
    p.fault_cta = -1;
    return p;
}

// Launches a persistent kernel: 1 launched; 0 this device cannot hold it resident (the caller
// then takes the per-stage path).
int try_decode(const DecodeParams &p, cudaStream_t s) {
    if (launch_decode(p, s) < 0) {
        (void)cudaGetLastError();
        return 0;
    }
    g_launches += 1;
    return 1;
}

// Reads and clears the device status word after the stream's work: a bounded wait that gave up
// (UMSX_ETIMEOUT) outranks a non-finite result (UMSX_ENONFINITE, the reference's rejection of
// non-finite combined outputs, tools/engine/expert_dispatch.cpp:14-18, :84-85).
umsx_status check_device_flag(Workspace &ws, cudaStream_t s) {
    uint32_t flag = 0;
    UMSX_CUDA(cudaMemcpyAsync(&flag, ws.disp.err, 4, cudaMemcpyDeviceToHost, s));
    UMSX_CUDA(cudaStreamSynchronize(s));
    if (!flag) return UMSX_OK;
    UMSX_CUDA(cudaMemsetAsync(ws.disp.err, 0, 4, s));
    UMSX_CUDA(cudaStreamSynchronize(s));
    if (flag & ~kErrNonFinite)
        return fail(UMSX_ETIMEOUT, "a bounded device wait gave up (flag " + std::to_string(flag) + ")");
    return fail(UMSX_ENONFINITE, "a combined expert output is not finite");
}

// One layer, out = MoE(x): the persistent kernel for small T, else the per-stage kernels.
umsx_status forward_layer(umsx_moe *m, const void *x, int x_dtype, int tokens, float *out, cudaStream_t s);

// router -> gate_up (+act, +Q8_0) -> down -> combine (+ optional residual).
// ev: null or 5 events bracketing the four stages.
// Many tokens (MXFP4 or Q8_0, fused or separate gate/up): router + dispatch, then the tensor-core
// grouped GEMMs.
bool prefill_eligible(const umsx_moe *m, const Workspace &ws, int tokens) {
    return tokens >= kPrefillMinTokens && ws.a16 && m->e_local <= 256;
}

// y_jobs (expert parallelism): instead of combining, write each resident job's output to
// y_jobs[t][r][:] and leave the other rows alone.
// extra: [T][H] added to each token's routed sum before the residual (shared experts), or null.
// The tiled router over `tokens` rows (RMSNorm fused when rmsnorm): ids, weights, the Q8_0 rows
// and this handle's expert dispatch.
umsx_status run_router_tiled(umsx_moe *m, Workspace &ws, const void *x, int x_dtype, int tokens, int rmsnorm, float eps,
                             cudaStream_t s) {
    const auto &d = m->d;
    RouterParams rp{};
    rp.x = x;
    rp.x_dtype = x_dtype;
    rp.tokens = tokens;
    rp.hidden = d.hidden;
    rp.experts = d.experts;
    rp.top_k = d.top_k;
    rp.routing = d.routing;
    rp.routed_scale = d.routed_scale;
    rp.w = m->router_w;
    rp.b = m->router_b;
    rp.e_lo = m->e_lo;
    rp.e_local = m->e_local;
    rp.rmsnorm = rmsnorm;
    rp.eps = eps;
    const int n = launch_router_tiled(rp, ws.disp, s);
    if (n < 0) return fail(UMSX_EDEVICE, "prefill router: shared-memory attribute refused");
    UMSX_LAUNCHED(n);
    return UMSX_OK;
}

// The grouped GEMMs of the tensor-core path over `jobs` packed job rows (an upper bound: the
// experts' segments come from disp.offsets): gate_up + activation into act16, down into ws.y.
umsx_status run_prefill_gemms(umsx_moe *m, Workspace &ws, const Dispatch &disp, int jobs, cudaStream_t s,
                              cudaEvent_t const *ev) {
    const auto &d = m->d;
    const int H = d.hidden, I = d.intermediate;
    MoeGemmParams g{};
    g.quant = d.quant;
    if (d.fused_gate_up) {
        g.codes = m->gate_up.codes;
        g.scales = m->gate_up.scales;
        g.emax = m->gate_up.emax;
        g.plane_rows = 2 * I;
    } else {
        g.codes = m->gate.codes;
        g.scales = m->gate.scales;
        g.emax = m->gate.emax;
        g.codes2 = m->up.codes;
        g.scales2 = m->up.scales;
        g.emax2 = m->up.emax;
        g.plane_rows = I;
    }
    g.rows = 2 * I;
    g.cols = H;
    g.fused = 1;
    g.inter = I;
    g.bias = m->gu_bias;
    g.offsets = disp.offsets;
    g.experts = m->e_local;
    g.m_tiles = I / 64;
    g.mode = 0;
    g.activation = d.activation;
    g.alpha = d.swiglu_alpha;
    g.limit = d.swiglu_limit;
    g.act_hi = ws.act16;
    g.act_lo = ws.act16 + (size_t)jobs * I;
    g.err = disp.err;
    int n = launch_moe_gemm(g, ws.a16, ws.a16 + (size_t)jobs * H, jobs, s);
    if (n < 0) return fail(UMSX_EDEVICE, "prefill gate_up: tensor map or launch setup failed");
    UMSX_LAUNCHED(n);
    if (ev) if (umsx_status st = mark(ev[2], s)) return st;
    MoeGemmParams dn{};
    dn.quant = d.quant;
    dn.codes = m->down.codes;
    dn.scales = m->down.scales;
    dn.emax = d.quant == UMSX_QUANT_MXFP4 ? m->down.emax : nullptr;
    dn.plane_rows = H;
    dn.rows = H;
    dn.cols = I;
    dn.fused = 0;
    dn.bias = m->down_bias;
    dn.offsets = disp.offsets;
    dn.experts = m->e_local;
    dn.m_tiles = (H + 127) / 128;
    dn.mode = 1;
    dn.y_out = ws.y;
    dn.err = disp.err;
    n = launch_moe_gemm(dn, ws.act16, ws.act16 + (size_t)jobs * I, jobs, s);
    if (n < 0) return fail(UMSX_EDEVICE, "prefill down: tensor map or launch setup failed");
    UMSX_LAUNCHED(n);
    return UMSX_OK;
}

umsx_status run_prefill(umsx_moe *m, Workspace &ws, const void *x, int x_dtype, int tokens, float *out,
                        const float *residual, int rmsnorm, float eps, cudaStream_t s, cudaEvent_t const *ev,
                        float *y_jobs = nullptr, const float *extra = nullptr) {
    const auto &d = m->d;
    const int K = d.top_k, H = d.hidden, jobs = tokens * K;
    if (ev) if (umsx_status st = mark(ev[0], s)) return st;
    if (umsx_status st = run_router_tiled(m, ws, x, x_dtype, tokens, rmsnorm, eps, s)) return st;
    UMSX_LAUNCHED(launch_prefill_pack(ws.disp, jobs, m->e_local == d.experts ? nullptr : ws.disp.offsets + m->e_local, K, H,
                                      ws.a16, ws.a16 + (size_t)jobs * H, ws.inv, s));
    if (ev) if (umsx_status st = mark(ev[1], s)) return st;
    if (umsx_status st = run_prefill_gemms(m, ws, ws.disp, jobs, s, ev)) return st;
    if (ev) if (umsx_status st = mark(ev[3], s)) return st;
    if (y_jobs) {
        UMSX_LAUNCHED(launch_prefill_scatter(ws.y, ws.inv, ws.disp.ids, m->e_lo, m->e_local, tokens, K, H, y_jobs, s));
        return UMSX_OK;
    }
    UMSX_LAUNCHED(launch_prefill_combine(ws.y, ws.disp.weights, ws.inv, tokens, K, H, extra, residual, out, ws.disp.err, s));
    if (ev) if (umsx_status st = mark(ev[4], s)) return st;
    return UMSX_OK;
}

// y_jobs: as run_prefill.
// Jobs per pass of the per-stage expert kernels.  A CTA holds one expert's jobs in
// registers and staging, MT at a time, and loops over the rest (re-reading its weights,
// mostly from L2).  With lambda = T * k / E jobs per expert on average, MT covers
// lambda + sqrt(lambda): large enough that few experts need a second pass, small enough
// that more CTAs fit on an SM and more weight bytes are in flight.
static int per_stage_chunk(int tokens, int top_k, int experts) {
    if (tokens <= 1) return 1;
    const double lam = (double)tokens * top_k / experts;
    const int want = std::max(2, (int)std::ceil(lam + std::sqrt(lam)));
    return std::min(tokens, want);
}

umsx_status run_layer(umsx_moe *m, Workspace &ws, const void *x, int x_dtype, int tokens, float *out,
                      const float *residual, int rmsnorm, float eps, cudaStream_t s, cudaEvent_t const *ev,
                      float *y_jobs = nullptr, const float *extra = nullptr, bool router_done = false) {
    const auto &d = m->d;
    if (!m->banked && prefill_eligible(m, ws, tokens))
        return run_prefill(m, ws, x, x_dtype, tokens, out, residual, rmsnorm, eps, s, ev, y_jobs, extra);
    if (ev) if (umsx_status st = mark(ev[0], s)) return st;
    if (!router_done)
        if (umsx_status st = run_router(m, ws, x, x_dtype, tokens, rmsnorm, eps, s, 1)) return st;
    if (ev) if (umsx_status st = mark(ev[1], s)) return st;
    const int slots = std::min(m->e_local, tokens * d.top_k);
    GateUpParams g{};
    g.gate_up = m->gate_up;
    g.gate = m->gate;
    g.up = m->up;
    g.fused = d.fused_gate_up;
    g.bias = m->gu_bias;
    g.intermediate = d.intermediate;
    g.hidden = d.hidden;
    g.activation = d.activation;
    g.alpha = d.swiglu_alpha;
    g.limit = d.swiglu_limit;
    g.act_codes = ws.act_codes;
    g.act_scales = ws.act_scales;
    g.act_f32 = ws.act_f32;
    g.act_rec = ws.act_rec;
    g.act_sc = ws.act_sc;
    g.act_done = ws.act_done;
    const int chunk = per_stage_chunk(tokens, d.top_k, d.experts);
    UMSX_LAUNCHED(launch_gate_up(g, ws.disp, slots, chunk, s));
    if (ev) if (umsx_status st = mark(ev[2], s)) return st;
    GemvParams p{};
    p.m = m->down;
    p.bias = m->down_bias;
    p.a_by_job = 1;
    p.out = y_jobs ? y_jobs : ws.y;
    p.o_ts = d.top_k;
    if (!ev && !y_jobs) {
        // down + fused rank-order combine (+ residual); the down weights follow from the
        // router's slot records, so their loads start before gate_up has finished
        p.tile_done = ws.disp.tile_done;
        p.route_w = ws.disp.weights;
        p.residual = residual;
        p.combine_out = out;
        p.top_k = d.top_k;
        p.prefetch_early = 1;
        p.extra = extra;
    }
    if (d.quant == UMSX_QUANT_MXFP4) { p.a_rec = ws.act_rec; p.a_rsc = ws.act_sc; }  // bulk-copied records
    else { p.a_codes = ws.act_codes; p.a_scales = ws.act_scales; }
    UMSX_LAUNCHED(launch_gemv(p, ws.disp, slots, chunk, s));
    if (y_jobs) return UMSX_OK;
    if (ev) {  // timed stages keep the combine a kernel of its own so that every stage has a boundary
        if (umsx_status st = mark(ev[3], s)) return st;
        UMSX_LAUNCHED(launch_combine(ws.y, ws.disp.weights, tokens, d.top_k, d.hidden, extra, residual, out, ws.disp.err, s));
        if (umsx_status st = mark(ev[4], s)) return st;
    }
    return UMSX_OK;
}

// Uploads expert e's ggml blocks (through the staging buffer, repacked in place) and biases into
// device slot `slot`, ordered on s.
umsx_status bank_upload(umsx_moe *m, int e, int slot, cudaStream_t s) {
    Matrix *mats[3] = {m->d.fused_gate_up ? &m->gate_up : &m->gate, m->d.fused_gate_up ? nullptr : &m->up, &m->down};
    for (int i = 0; i < 3; ++i) {
        if (!mats[i]) continue;
        UMSX_CUDA(cudaMemcpyAsync(m->bank_staging, m->host_blocks[i] + (size_t)e * m->host_per[i], m->host_per[i],
                                  cudaMemcpyHostToDevice, s));
        UMSX_LAUNCHED(launch_repack(*mats[i], slot, m->bank_staging, s));
        m->upload_bytes += m->host_per[i];
    }
    const size_t I = m->d.intermediate, H = m->d.hidden;
    if (m->d.has_bias) {
        UMSX_CUDA(cudaMemcpyAsync(m->gu_bias + (size_t)slot * 2 * I, m->host_gu_bias + (size_t)e * 2 * I, 2 * I * 4,
                                  cudaMemcpyHostToDevice, s));
        UMSX_CUDA(cudaMemcpyAsync(m->down_bias + (size_t)slot * H, m->host_dn_bias + (size_t)e * H, H * 4,
                                  cudaMemcpyHostToDevice, s));
    }
    return UMSX_OK;
}

// A banked layer's call: route on the device, read the routing back, let the policy admit experts
// into the bank (one-token calls) or look them up (several tokens), upload the admitted experts into
// their slots and the other missing ones into transient slots, point the dispatch's slot records at
// the device slots, then run the expert kernels.  The call synchronises with the host twice (after
// routing, and before its host vectors go out of scope).
umsx_status run_banked(umsx_moe *m, const void *x, int x_dtype, int tokens, float *out, cudaStream_t s) {
    const int K = m->d.top_k, E = m->d.experts;
    Workspace &ws = m->ws;
    if (umsx_status st = run_router(m, ws, x, x_dtype, tokens, 0, 0.0f, s, 1)) return st;
    std::vector<int32_t> ids((size_t)tokens * K);
    UMSX_CUDA(cudaMemcpyAsync(ids.data(), ws.disp.ids, ids.size() * 4, cudaMemcpyDeviceToHost, s));
    UMSX_CUDA(cudaStreamSynchronize(s));
    std::vector<int> selected;
    std::vector<char> seen(E, 0);
    for (int32_t e : ids) {
        if (e < 0 || e >= E) return fail(UMSX_EDEVICE, "routing produced an expert index out of range");
        if (!seen[e]) { seen[e] = 1; selected.push_back(e); }
    }
    std::vector<std::pair<int, int>> admitted;
    std::vector<int> evicted;
    const std::vector<int> slot = m->policy->dispatch(selected, admitted, evicted, tokens == 1);
    for (const auto &a : admitted)
        if (umsx_status st = bank_upload(m, a.first, a.second, s)) return st;
    std::vector<int32_t> map(E, -1);
    int transient = m->bank_slots;
    for (size_t i = 0; i < selected.size(); ++i) {
        if (slot[i] >= 0) { map[selected[i]] = slot[i]; continue; }
        map[selected[i]] = transient;
        if (umsx_status st = bank_upload(m, selected[i], transient++, s)) return st;
    }
    UMSX_CUDA(cudaMemcpyAsync(m->d_map, map.data(), (size_t)E * 4, cudaMemcpyHostToDevice, s));
    UMSX_LAUNCHED(launch_bank_remap(ws.disp.slots, m->d_map, std::min(E, tokens * K), s));
    UMSX_CUDA(cudaStreamSynchronize(s));  // the pageable sources above are read before they go out of scope
    return run_layer(m, ws, x, x_dtype, tokens, out, nullptr, 0, 0.0f, s, nullptr, nullptr, nullptr, true);
}

umsx_status forward_layer(umsx_moe *m, const void *x, int x_dtype, int tokens, float *out, cudaStream_t s) {
    if (m->banked) return run_banked(m, x, x_dtype, tokens, out, s);
    if (decode_eligible(m, tokens, 1)) {
        DecodeParams p = decode_params(m, m->ws, x, x_dtype, tokens, out);
        p.ids_out = m->ws.disp.ids;
        p.w_out = m->ws.disp.weights;
        if (try_decode(p, s) > 0) return UMSX_OK;
    }
    return run_layer(m, m->ws, x, x_dtype, tokens, out, nullptr, 0, 0.0f, s, nullptr);
}

}  // namespace

extern "C" {

umsx_status umsx_moe_forward(umsx_moe *m, const void *x, int x_dtype, int tokens, float *out, int32_t *ids,
                             float *weights, umsx_stream stream) {
    if (umsx_status st = check_call(m, x, x_dtype, tokens, m ? m->d.max_tokens : 0)) return st;
    if (!out) return fail(UMSX_EINVAL, "null output");
    if (m->e_local != m->d.experts)
        return fail(UMSX_EUNSUPPORTED, "expert-parallel handle: use umsx_moe_forward_jobs and combine on the token's rank");
    std::lock_guard<std::mutex> lock(m->mu);
    UMSX_CUDA(cudaSetDevice(m->device));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (umsx_status st = forward_layer(m, x, x_dtype, tokens, out, s)) return st;
    const size_t n = (size_t)tokens * m->d.top_k;
    if (ids) UMSX_CUDA(cudaMemcpyAsync(ids, m->ws.disp.ids, n * 4, cudaMemcpyDeviceToDevice, s));
    if (weights) UMSX_CUDA(cudaMemcpyAsync(weights, m->ws.disp.weights, n * 4, cudaMemcpyDeviceToDevice, s));
    return UMSX_OK;
}

umsx_status umsx_moe_forward_jobs(umsx_moe *m, const void *x, int x_dtype, int tokens, int32_t *ids, float *weights,
                                  float *y, umsx_stream stream) {
    if (umsx_status st = check_call(m, x, x_dtype, tokens, m ? m->d.max_tokens : 0)) return st;
    if (m->banked) return fail(UMSX_EUNSUPPORTED, "banked layer: call umsx_moe_forward or umsx_moe_forward_host");
    if (!y || reinterpret_cast<uintptr_t>(y) % 16) return fail(UMSX_EINVAL, "y must be a 16-byte aligned device buffer");
    std::lock_guard<std::mutex> lock(m->mu);
    UMSX_CUDA(cudaSetDevice(m->device));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (umsx_status st = run_layer(m, m->ws, x, x_dtype, tokens, nullptr, nullptr, 0, 0.0f, s, nullptr, y)) return st;
    const size_t n = (size_t)tokens * m->d.top_k;
    if (ids) UMSX_CUDA(cudaMemcpyAsync(ids, m->ws.disp.ids, n * 4, cudaMemcpyDeviceToDevice, s));
    if (weights) UMSX_CUDA(cudaMemcpyAsync(weights, m->ws.disp.weights, n * 4, cudaMemcpyDeviceToDevice, s));
    return UMSX_OK;
}

umsx_status umsx_moe_forward_host(umsx_moe *m, const void *x, int x_dtype, int tokens, float *out, umsx_stream stream) {
    if (umsx_status st = check_call(m, x, x_dtype, tokens, m ? m->d.max_tokens : 0)) return st;
    if (!out) return fail(UMSX_EINVAL, "null output");
    if (m->e_local != m->d.experts)
        return fail(UMSX_EUNSUPPORTED, "expert-parallel handle: use umsx_moe_forward_jobs and combine on the token's rank");
    std::lock_guard<std::mutex> lock(m->mu);
    UMSX_CUDA(cudaSetDevice(m->device));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t in_bytes = (size_t)tokens * m->d.hidden * (x_dtype == UMSX_DTYPE_BF16 ? 2 : 4);
    const size_t out_bytes = (size_t)tokens * m->d.hidden * 4;
    UMSX_CUDA(cudaMemcpyAsync(m->ws.x_dev, x, in_bytes, cudaMemcpyHostToDevice, s));
    if (umsx_status st = forward_layer(m, m->ws.x_dev, x_dtype, tokens, m->ws.out_dev, s)) return st;
    UMSX_CUDA(cudaMemcpyAsync(out, m->ws.out_dev, out_bytes, cudaMemcpyDeviceToHost, s));
    return check_device_flag(m->ws, s);
}

umsx_status umsx_moe_set_router(umsx_moe *m, const float *router_w, const float *router_b) {
    if (!m || !router_w) return fail(UMSX_EINVAL, "null handle or router weights");
    if ((router_b != nullptr) != (m->d.has_router_bias != 0))
        return fail(UMSX_EINVAL, "router_b must be given exactly when the layer has a router bias");
    std::lock_guard<std::mutex> lock(m->mu);
    UMSX_CUDA(cudaSetDevice(m->device));
    UMSX_CUDA(cudaDeviceSynchronize());  // no call of this handle reads the router meanwhile
    UMSX_CUDA(cudaMemcpy(m->router_w, router_w, (size_t)m->d.experts * m->d.hidden * 4, cudaMemcpyHostToDevice));
    if (router_b) UMSX_CUDA(cudaMemcpy(m->router_b, router_b, (size_t)m->d.experts * 4, cudaMemcpyHostToDevice));
    return UMSX_OK;
}

umsx_status umsx_moe_status(umsx_moe *m, umsx_stream stream) {
    if (!m) return fail(UMSX_EINVAL, "null handle");
    std::lock_guard<std::mutex> lock(m->mu);
    UMSX_CUDA(cudaSetDevice(m->device));
    return check_device_flag(m->ws, static_cast<cudaStream_t>(stream));
}

umsx_status umsx_route(umsx_moe *m, const void *x, int x_dtype, int tokens, int32_t *ids, float *weights,
                       int32_t *counts, umsx_stream stream) {
    if (umsx_status st = check_call(m, x, x_dtype, tokens, m ? m->d.max_tokens : 0)) return st;
    std::lock_guard<std::mutex> lock(m->mu);
    UMSX_CUDA(cudaSetDevice(m->device));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (umsx_status st = run_router(m, m->ws, x, x_dtype, tokens, 0, 0.0f, s)) return st;
    const Dispatch &d = m->ws.disp;
    const size_t n = (size_t)tokens * m->d.top_k;
    if (ids) UMSX_CUDA(cudaMemcpyAsync(ids, d.ids, n * 4, cudaMemcpyDeviceToDevice, s));
    if (weights) UMSX_CUDA(cudaMemcpyAsync(weights, d.weights, n * 4, cudaMemcpyDeviceToDevice, s));
    if (counts) UMSX_CUDA(cudaMemcpyAsync(counts, d.counts, (size_t)m->e_local * 4, cudaMemcpyDeviceToDevice, s));
    return UMSX_OK;
}

umsx_status umsx_expert_down_q8(umsx_moe *m, const void *packed_q8, const int32_t *experts, int jobs, float *out,
                                umsx_stream stream) {
    if (!m) return fail(UMSX_EINVAL, "null handle");
    if (m->banked) return fail(UMSX_EUNSUPPORTED, "banked layer: call umsx_moe_forward or umsx_moe_forward_host");
    if (jobs < 0 || jobs > m->d.max_tokens * m->d.top_k) return fail(UMSX_EINVAL, "invalid packed Q8 input shape");
    if (jobs == 0) return UMSX_OK;
    if (!packed_q8 || !experts || !out) return fail(UMSX_EINVAL, "null buffer");
    std::vector<int32_t> counts(m->e_local, 0), offsets(m->e_local + 1, 0), active, token(jobs), rank(jobs, 0);
    for (int j = 0; j < jobs; ++j) {
        if (!resident(m, experts[j])) return fail(UMSX_ENOTRESIDENT, "MXFP4 GPU expert is out of range or not resident");
        counts[experts[j] - m->e_lo]++;
    }
    int maxc = 0;
    for (int e = 0; e < m->e_local; ++e) {
        offsets[e + 1] = offsets[e] + counts[e];
        if (counts[e]) active.push_back(e);
        maxc = std::max(maxc, counts[e]);
    }
    std::vector<int32_t> fill(offsets.begin(), offsets.end() - 1);
    for (int j = 0; j < jobs; ++j) token[fill[experts[j] - m->e_lo]++] = j;
    const int n_active = (int)active.size();
    std::vector<int4> slot_rec(n_active);
    for (int a = 0; a < n_active; ++a) slot_rec[a] = make_int4(active[a], offsets[active[a]], counts[active[a]], 0);
    std::lock_guard<std::mutex> lock(m->mu);
    UMSX_CUDA(cudaSetDevice(m->device));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const Dispatch &d = m->ws.disp;
    // pageable sources: each copy is staged before cudaMemcpyAsync returns
    UMSX_CUDA(cudaMemcpyAsync(d.counts, counts.data(), counts.size() * 4, cudaMemcpyHostToDevice, s));
    UMSX_CUDA(cudaMemcpyAsync(d.offsets, offsets.data(), offsets.size() * 4, cudaMemcpyHostToDevice, s));
    UMSX_CUDA(cudaMemcpyAsync(d.active, active.data(), active.size() * 4, cudaMemcpyHostToDevice, s));
    UMSX_CUDA(cudaMemcpyAsync(d.n_active, &n_active, 4, cudaMemcpyHostToDevice, s));
    UMSX_CUDA(cudaMemcpyAsync(d.job_token, token.data(), token.size() * 4, cudaMemcpyHostToDevice, s));
    UMSX_CUDA(cudaMemcpyAsync(d.job_rank, rank.data(), rank.size() * 4, cudaMemcpyHostToDevice, s));
    UMSX_CUDA(cudaMemcpyAsync(d.slots, slot_rec.data(), slot_rec.size() * sizeof(int4), cudaMemcpyHostToDevice, s));
    GemvParams p{};
    p.m = m->down;
    p.bias = m->down_bias;
    p.a_q8 = static_cast<const uint8_t *>(packed_q8);
    p.a_ts = 1;
    p.a_rs = 0;
    p.out = out;
    p.o_ts = 1;
    UMSX_LAUNCHED(launch_gemv(p, d, n_active, maxc, s));
    return UMSX_OK;
}

static const Matrix *projection(umsx_moe *m, int proj) {
    switch (proj) {
        case UMSX_PROJ_GATE_UP: return m->d.fused_gate_up ? &m->gate_up : nullptr;
        case UMSX_PROJ_GATE: return m->d.fused_gate_up ? nullptr : &m->gate;
        case UMSX_PROJ_UP: return m->d.fused_gate_up ? nullptr : &m->up;
        case UMSX_PROJ_DOWN: return &m->down;
        default: return nullptr;
    }
}

umsx_status umsx_mul_mat_id(umsx_moe *m, int proj, const float *b, int n_b, const int32_t *ids, int n_ids, int tokens,
                            float *dst, umsx_stream stream) {
    if (!m || !b || !ids || !dst) return fail(UMSX_EINVAL, "null argument");
    if (m->banked) return fail(UMSX_EUNSUPPORTED, "banked layer: call umsx_moe_forward or umsx_moe_forward_host");
    if (tokens <= 0 || n_ids <= 0 || n_ids > m->d.experts || (n_b != 1 && n_b != n_ids) ||
        (size_t)tokens * n_ids > (size_t)m->d.max_tokens * m->d.top_k)
        return fail(UMSX_EINVAL, "invalid MUL_MAT_ID shape");
    const Matrix *mat = projection(m, proj);
    if (!mat) return fail(UMSX_EINVAL, "projection not present in this layer");
    std::lock_guard<std::mutex> lock(m->mu);
    UMSX_CUDA(cudaSetDevice(m->device));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    Dispatch d = m->ws.disp;
    d.ids = const_cast<int32_t *>(ids);
    UMSX_CUDA(cudaMemsetAsync(dst, 0, (size_t)tokens * n_ids * mat->rows * sizeof(float), s));
    UMSX_LAUNCHED(launch_dispatch(d, tokens * n_ids, n_ids, m->e_lo, m->e_local, s));
    GemvParams p{};
    p.m = *mat;
    p.a_f32 = b;
    p.a_ts = n_b;
    p.a_rs = n_b == 1 ? 0 : 1;
    p.out = dst;
    p.o_ts = n_ids;
    UMSX_LAUNCHED(launch_gemv(p, d, std::min(m->e_local, tokens * n_ids), tokens, s));
    return UMSX_OK;
}

umsx_status umsx_combine(const float *y, const float *weights, int tokens, int top_k, int width, float *out,
                         umsx_stream stream) {
    if (!y || !weights || !out || tokens <= 0 || top_k <= 0 || width <= 0 || width % 4)
        return fail(UMSX_EINVAL, "invalid combine arguments (width must be a multiple of 4)");
    UMSX_LAUNCHED(launch_combine(y, weights, tokens, top_k, width, nullptr, nullptr, out, nullptr, static_cast<cudaStream_t>(stream)));
    return UMSX_OK;
}

umsx_status umsx_moe_export_expert(umsx_moe *m, int proj, int expert, void *host_out, size_t size) {
    if (!m || !host_out) return fail(UMSX_EINVAL, "null argument");
    if (m->banked) return fail(UMSX_EUNSUPPORTED, "banked layer: call umsx_moe_forward or umsx_moe_forward_host");
    const Matrix *mat = projection(m, proj);
    if (!mat) return fail(UMSX_EINVAL, "projection not present in this layer");
    if (!resident(m, expert)) return fail(UMSX_ENOTRESIDENT, "expert out of range or not resident");
    const size_t per = (size_t)mat->rows * (mat->cols / 32) * block_bytes(mat->quant);
    if (size != per) return fail(UMSX_EINVAL, "export buffer size mismatch");
    std::lock_guard<std::mutex> lock(m->mu);
    UMSX_CUDA(cudaSetDevice(m->device));
    uint8_t *tmp = nullptr;
    UMSX_CUDA(cudaMalloc(&tmp, per));
    umsx_status st = UMSX_OK;
    g_launches += (uint64_t)launch_export(*mat, expert - m->e_lo, tmp, 0);
    cudaError_t err = cudaGetLastError();
    if (err == cudaSuccess) err = cudaMemcpy(host_out, tmp, per, cudaMemcpyDeviceToHost);
    if (err != cudaSuccess) st = fail(UMSX_EDEVICE, std::string("export: ") + cudaGetErrorString(err));
    cudaFree(tmp);
    return st;
}

}  // extern "C"

// ============================================================================
// Layer stack: h <- h + MoE_l(RMSNorm(h)) for l = 0..L-1, replayed as one CUDA
// graph per (token count, input dtype) on a library-owned stream.
// ============================================================================

struct umsx_stack {
    std::vector<umsx_moe *> layers;
    std::vector<umsx_moe *> shared;  // per layer: a one-expert shared-FFN handle added to the routed sum, or null
    float *y_sh = nullptr;           // [T][H] the current layer's shared-FFN output
    bool uniform = true;             // every layer has layer 0's shape and no shared FFN
    float eps = 1e-5f;
    int device = 0;
    int max_tokens = 0;
    int hidden = 0;
    Workspace ws;
    float *h = nullptr;
    cudaStream_t stream = nullptr;
    cudaEvent_t ev_in = nullptr, ev_out = nullptr;
    std::vector<cudaEvent_t> stage;  // 5 per layer while timing is on
    bool timing = false;
    int fault_cta = -1;                   // one-shot fault injection (umsx_stack_inject_fault)
    long long fault_wait_cycles = 0;
    struct Graph { int tokens, dtype; bool timing; cudaGraphExec_t exec; uint64_t kernels; };
    std::vector<Graph> graphs;
    std::mutex mu;
};

namespace {

void drop_graphs(umsx_stack *st) {
    for (auto &g : st->graphs) cudaGraphExecDestroy(g.exec);
    st->graphs.clear();
}

umsx_status record_stack(umsx_stack *st, int tokens, int dtype, cudaStream_t s) {
    const int H = st->hidden;
    if (dtype == UMSX_DTYPE_BF16)
        UMSX_LAUNCHED(launch_bf16_to_f32(static_cast<const uint16_t *>(st->ws.x_dev), st->h, (size_t)tokens * H, s));
    else
        UMSX_CUDA(cudaMemcpyAsync(st->h, st->ws.x_dev, (size_t)tokens * H * 4, cudaMemcpyDeviceToDevice, s));
    for (size_t l = 0; l < st->layers.size(); ++l) {
        const cudaEvent_t *ev = st->timing ? &st->stage[5 * l] : nullptr;
        umsx_moe *sh = st->shared.empty() ? nullptr : st->shared[l];
        // the shared FFN first (its output rows land in y_sh), then the routed layer, whose combine
        // adds them as the term after the k routed ones: h + ((sum_r w_r y_r) + y_shared)
        if (sh)
            if (umsx_status r = run_layer(sh, st->ws, st->h, UMSX_DTYPE_F32, tokens, nullptr, nullptr, 1, st->eps, s,
                                          nullptr, st->y_sh))
                return r;
        if (umsx_status r = run_layer(st->layers[l], st->ws, st->h, UMSX_DTYPE_F32, tokens, st->h, st->h, 1, st->eps, s,
                                      ev, nullptr, sh ? st->y_sh : nullptr))
            return r;
    }
    return UMSX_OK;
}

umsx_status stack_graph(umsx_stack *st, int tokens, int dtype, umsx_stack::Graph **out) {
    for (auto &g : st->graphs)
        if (g.tokens == tokens && g.dtype == dtype && g.timing == st->timing) { *out = &g; return UMSX_OK; }
    const uint64_t before = g_launches;
    UMSX_CUDA(cudaStreamBeginCapture(st->stream, cudaStreamCaptureModeThreadLocal));
    umsx_status r = record_stack(st, tokens, dtype, st->stream);
    cudaGraph_t graph = nullptr;
    const cudaError_t e = cudaStreamEndCapture(st->stream, &graph);
    if (r) { if (graph) cudaGraphDestroy(graph); return r; }
    if (e != cudaSuccess) return fail(UMSX_EDEVICE, std::string("stack capture: ") + cudaGetErrorString(e));
    cudaGraphExec_t exec = nullptr;
    const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ie != cudaSuccess) return fail(UMSX_EDEVICE, std::string("stack instantiate: ") + cudaGetErrorString(ie));
    const uint64_t kernels = g_launches - before;
    g_launches = before;  // counted per replay instead
    st->graphs.push_back({tokens, dtype, st->timing, exec, kernels});
    *out = &st->graphs.back();
    return UMSX_OK;
}

umsx_status stack_run(umsx_stack *st, const void *x, int dtype, int tokens, void *out, cudaMemcpyKind in_kind,
                      cudaMemcpyKind out_kind, cudaStream_t caller) {
    const size_t in_bytes = (size_t)tokens * st->hidden * (dtype == UMSX_DTYPE_BF16 ? 2 : 4);
    const size_t out_bytes = (size_t)tokens * st->hidden * 4;
    const int L = (int)st->layers.size();
    bool eligible = !st->timing && st->uniform;
    for (int l = 0; l < L && eligible; ++l) eligible = decode_eligible(st->layers[l], tokens, L);
    if (eligible) {
        // one persistent launch on the caller's stream, reading x and writing out in place when they are device memory
        const bool dev_in = in_kind == cudaMemcpyDeviceToDevice;
        const bool dev_out = out_kind == cudaMemcpyDeviceToDevice && reinterpret_cast<uintptr_t>(out) % 16 == 0;
        if (!dev_in) UMSX_CUDA(cudaMemcpyAsync(st->ws.x_dev, x, in_bytes, in_kind, caller));
        DecodeParams p = decode_params(st->layers[0], st->ws, dev_in ? x : st->ws.x_dev, dtype, tokens,
                                       dev_out ? static_cast<float *>(out) : st->h);
        p.n_layers = L;
        for (int l = 0; l < L; ++l) set_decode_layer(p, l, st->layers[l]);
        p.rmsnorm = 1;
        p.residual = 1;
        p.eps = st->eps;
        p.fault_cta = st->fault_cta;
        p.wait_cycles = st->fault_wait_cycles;
        st->fault_cta = -1;  // one forward only
        st->fault_wait_cycles = 0;
        if (try_decode(p, caller) > 0) {
            if (!dev_out) UMSX_CUDA(cudaMemcpyAsync(out, st->h, out_bytes, out_kind, caller));
            return UMSX_OK;
        }
    }
    UMSX_CUDA(cudaEventRecord(st->ev_in, caller));
    UMSX_CUDA(cudaStreamWaitEvent(st->stream, st->ev_in, 0));
    UMSX_CUDA(cudaMemcpyAsync(st->ws.x_dev, x, in_bytes, in_kind, st->stream));
    umsx_stack::Graph *g = nullptr;
    if (umsx_status r = stack_graph(st, tokens, dtype, &g)) return r;
    UMSX_CUDA(cudaGraphLaunch(g->exec, st->stream));
    g_launches += g->kernels;
    UMSX_CUDA(cudaMemcpyAsync(out, st->h, out_bytes, out_kind, st->stream));
    UMSX_CUDA(cudaEventRecord(st->ev_out, st->stream));
    UMSX_CUDA(cudaStreamWaitEvent(caller, st->ev_out, 0));
    return UMSX_OK;
}

}  // namespace

extern "C" {

}  // extern "C"

namespace {
umsx_status stack_create(umsx_moe *const *layers, umsx_moe *const *shared, int n_layers, int max_tokens, float rms_eps,
                         bool same_shape, umsx_stack **out) {
    if (!out || !layers || n_layers <= 0) return fail(UMSX_EINVAL, "need at least one layer");
    *out = nullptr;
    const umsx_moe *l0 = layers[0];
    if (!l0) return fail(UMSX_EINVAL, "null layer");
    // the workspace serves every layer: it is carved for the largest of each dimension
    umsx_moe_desc big = l0->d;
    int e_local = l0->e_local;
    bool uniform = true;
    auto widen = [&](const umsx_moe *m) {
        big.top_k = std::max(big.top_k, m->d.top_k);
        big.experts = std::max(big.experts, m->d.experts);
        big.intermediate = std::max(big.intermediate, m->d.intermediate);
        if (m->d.quant == UMSX_QUANT_MXFP4) big.quant = UMSX_QUANT_MXFP4;
        e_local = std::max(e_local, m->e_local);
    };
    for (int l = 0; l < n_layers; ++l) {
        const umsx_moe *m = layers[l];
        if (!m || m->device != l0->device || m->d.hidden != l0->d.hidden)
            return fail(UMSX_EINVAL, "stack layers must share device and width");
        const bool same = m->d.top_k == l0->d.top_k && m->d.experts == l0->d.experts &&
                          m->d.intermediate == l0->d.intermediate && m->e_local == l0->e_local;
        if (same_shape && !same) return fail(UMSX_EINVAL, "stack layers must share device and shape");
        uniform = uniform && same;
        if (m->e_local != m->d.experts)
            return fail(UMSX_EUNSUPPORTED, "a stack runs whole layers; expert-parallel handles use umsx_moe_forward_jobs");
        widen(m);
        const umsx_moe *sh = shared ? shared[l] : nullptr;
        if (m->banked || (sh && sh->banked)) return fail(UMSX_EUNSUPPORTED, "banked layer: call umsx_moe_forward or umsx_moe_forward_host");
        if (sh) {
            if (sh->device != l0->device || sh->d.hidden != l0->d.hidden || sh->d.experts != 1 || sh->d.top_k != 1)
                return fail(UMSX_EINVAL, "a shared-expert handle is a one-expert top-1 layer of the stack's width and device");
            uniform = false;
            widen(sh);
        }
    }
    if (max_tokens <= 0 || max_tokens > 65535) return fail(UMSX_EINVAL, "max_tokens must be in [1, 65535]");
    UMSX_CUDA(cudaSetDevice(l0->device));
    auto *st = new umsx_stack();
    st->layers.assign(layers, layers + n_layers);
    if (shared) st->shared.assign(shared, shared + n_layers);
    st->uniform = uniform;
    st->eps = rms_eps;
    st->device = l0->device;
    st->max_tokens = max_tokens;
    st->hidden = l0->d.hidden;
    auto run = [&]() -> umsx_status {
        if (umsx_status r = alloc_workspace(st->ws, big, e_local, max_tokens, 0)) return r;
        UMSX_CUDA(cudaMalloc(&st->h, (size_t)max_tokens * st->hidden * 4));
        if (!st->shared.empty()) UMSX_CUDA(cudaMalloc(&st->y_sh, (size_t)max_tokens * st->hidden * 4));
        UMSX_CUDA(cudaStreamCreateWithFlags(&st->stream, cudaStreamNonBlocking));
        UMSX_CUDA(cudaEventCreateWithFlags(&st->ev_in, cudaEventDisableTiming));
        UMSX_CUDA(cudaEventCreateWithFlags(&st->ev_out, cudaEventDisableTiming));
        return UMSX_OK;
    };
    if (umsx_status r = run()) { umsx_stack_destroy(st); return r; }
    *out = st;
    return UMSX_OK;
}
}  // namespace

extern "C" {

umsx_status umsx_stack_create(umsx_moe *const *layers, int n_layers, int max_tokens, float rms_eps, umsx_stack **out) {
    return stack_create(layers, nullptr, n_layers, max_tokens, rms_eps, true, out);
}

umsx_status umsx_stack_create_mixed(umsx_moe *const *layers, umsx_moe *const *shared, int n_layers, int max_tokens,
                                    float rms_eps, umsx_stack **out) {
    return stack_create(layers, shared, n_layers, max_tokens, rms_eps, false, out);
}

void umsx_stack_destroy(umsx_stack *st) {
    if (!st) return;
    cudaSetDevice(st->device);
    if (st->stream) cudaStreamSynchronize(st->stream);
    drop_graphs(st);
    for (auto e : st->stage) cudaEventDestroy(e);
    if (st->ev_in) cudaEventDestroy(st->ev_in);
    if (st->ev_out) cudaEventDestroy(st->ev_out);
    if (st->stream) cudaStreamDestroy(st->stream);
    if (st->h) cudaFree(st->h);
    if (st->y_sh) cudaFree(st->y_sh);
    if (st->ws.mem) cudaFree(st->ws.mem);
    delete st;
}

umsx_status umsx_stack_forward(umsx_stack *st, const void *x, int x_dtype, int tokens, float *out, umsx_stream stream) {
    if (!st) return fail(UMSX_EINVAL, "null stack");
    if (umsx_status r = check_call(st->layers[0], x, x_dtype, tokens, st->max_tokens)) return r;
    if (!out) return fail(UMSX_EINVAL, "null output");
    std::lock_guard<std::mutex> lock(st->mu);
    UMSX_CUDA(cudaSetDevice(st->device));
    return stack_run(st, x, x_dtype, tokens, out, cudaMemcpyDeviceToDevice, cudaMemcpyDeviceToDevice,
                     static_cast<cudaStream_t>(stream));
}

umsx_status umsx_stack_forward_host(umsx_stack *st, const void *x, int x_dtype, int tokens, float *out,
                                    umsx_stream stream) {
    if (!st) return fail(UMSX_EINVAL, "null stack");
    if (umsx_status r = check_call(st->layers[0], x, x_dtype, tokens, st->max_tokens)) return r;
    if (!out) return fail(UMSX_EINVAL, "null output");
    std::lock_guard<std::mutex> lock(st->mu);
    UMSX_CUDA(cudaSetDevice(st->device));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (umsx_status r = stack_run(st, x, x_dtype, tokens, out, cudaMemcpyHostToDevice, cudaMemcpyDeviceToHost, s))
        return r;
    return check_device_flag(st->ws, s);
}

umsx_status umsx_stack_status(umsx_stack *st, umsx_stream stream) {
    if (!st) return fail(UMSX_EINVAL, "null stack");
    std::lock_guard<std::mutex> lock(st->mu);
    UMSX_CUDA(cudaSetDevice(st->device));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    UMSX_CUDA(cudaStreamSynchronize(st->stream));  // graph replays run on the stack's own stream
    return check_device_flag(st->ws, s);
}

umsx_status umsx_stack_set_timing(umsx_stack *st, int enable) {
    if (!st) return fail(UMSX_EINVAL, "null stack");
    std::lock_guard<std::mutex> lock(st->mu);
    UMSX_CUDA(cudaSetDevice(st->device));
    st->timing = enable != 0;
    if (st->timing && st->stage.empty()) {
        st->stage.resize(5 * st->layers.size());
        for (auto &e : st->stage) UMSX_CUDA(cudaEventCreate(&e));
    }
    return UMSX_OK;
}

umsx_status umsx_stack_inject_fault(umsx_stack *st, int cta, int64_t wait_limit_cycles) {
    if (!st) return fail(UMSX_EINVAL, "null stack");
    if (cta < 0 || wait_limit_cycles <= 0 || wait_limit_cycles > 4000000000LL)
        return fail(UMSX_EINVAL, "need cta >= 0 and 0 < wait_limit_cycles <= 4e9");
    std::lock_guard<std::mutex> lock(st->mu);
    st->fault_cta = cta;
    st->fault_wait_cycles = wait_limit_cycles;
    return UMSX_OK;
}

umsx_status umsx_stack_stage_times(umsx_stack *st, float *ms, int n_stages) {
    if (!st || !ms || n_stages != 4) return fail(UMSX_EINVAL, "need a stack and room for 4 stage times");
    if (!st->timing) return fail(UMSX_EINVAL, "timing is not enabled on this stack");
    std::lock_guard<std::mutex> lock(st->mu);
    UMSX_CUDA(cudaSetDevice(st->device));
    UMSX_CUDA(cudaStreamSynchronize(st->stream));
    for (int k = 0; k < 4; ++k) ms[k] = 0.0f;
    for (size_t l = 0; l < st->layers.size(); ++l) {
        for (int k = 0; k < 4; ++k) {
            float t = 0.0f;
            UMSX_CUDA(cudaEventElapsedTime(&t, st->stage[5 * l + k], st->stage[5 * l + k + 1]));
            ms[k] += t;
        }
    }
    return UMSX_OK;
}

// ---- GGUF --------------------------------------------------------------------

namespace {
struct GgufOwner {
    umsx::GgufExperts e;
};
}  // namespace

umsx_status umsx_gguf_load_experts(const char *first_shard, int layer, const uint32_t *ids, int n_ids, int dequantize,
                                   umsx_gguf_experts *out) {
    if (!first_shard || !ids || !out || n_ids <= 0) return fail(UMSX_EINVAL, "invalid layer or selected expert IDs");
    std::memset(out, 0, sizeof(*out));
    auto *own = new (std::nothrow) GgufOwner;
    if (!own) return fail(UMSX_EOOM, "host allocation failed");
    std::string err;
    try {
        err = umsx::gguf_load_experts(first_shard, layer, std::vector<uint32_t>(ids, ids + n_ids), dequantize != 0, true,
                                      own->e);
    } catch (const std::bad_alloc &) {
        err = "host allocation failed";
    }
    if (!err.empty()) {
        delete own;
        return fail(err == "host allocation failed" ? UMSX_EOOM : UMSX_EINVAL, err);
    }
    const umsx::GgufExperts &e = own->e;
    out->hidden = e.hidden;
    out->intermediate = e.intermediate;
    out->experts = e.count;
    out->n_ids = e.n_ids;
    for (int p = 0; p < 3; ++p) {
        out->quant[p] = e.type[p];
        out->stride[p] = e.stride[p];
        out->packed[p] = e.packed[p].data();
        out->values[p] = e.values[p].empty() ? nullptr : e.values[p].data();
        out->bias[p] = e.has_bias[p] ? e.bias[p].data() : nullptr;
    }
    out->owner = own;
    return UMSX_OK;
}

void umsx_gguf_experts_free(umsx_gguf_experts *e) {
    if (!e) return;
    delete static_cast<GgufOwner *>(e->owner);
    std::memset(e, 0, sizeof(*e));
}

umsx_status umsx_moe_create_gguf(const umsx_moe_desc *desc, const char *first_shard, int layer, int device,
                                 size_t reserve_bytes, umsx_moe **out) {
    if (!desc || !first_shard || !out) return fail(UMSX_EINVAL, "null argument");
    if (desc->experts <= 0 || desc->experts > 65536) return fail(UMSX_EINVAL, "experts must be in [1, 65536]");
    try {
        std::vector<float> rw, rb;
        int64_t rshape[2] = {0, 0};
        bool has_rb = false;
        std::string err = umsx::gguf_load_router(first_shard, layer, rw, rshape, rb, has_rb);
        if (!err.empty()) return fail(UMSX_EINVAL, err);
        if (rshape[0] != desc->hidden || rshape[1] != desc->experts)
            return fail(UMSX_EINVAL, "GGUF router shape does not match the layer descriptor");
        if (has_rb != (desc->has_router_bias != 0))
            return fail(UMSX_EINVAL, "GGUF router bias presence does not match has_router_bias");
        std::vector<uint32_t> all((size_t)desc->experts);
        for (int i = 0; i < desc->experts; ++i) all[i] = (uint32_t)i;
        umsx::GgufExperts e;
        err = umsx::gguf_load_experts(first_shard, layer, all, false, false, e);
        if (!err.empty()) return fail(UMSX_EINVAL, err);
        if (e.hidden != desc->hidden || e.intermediate != desc->intermediate || e.count != desc->experts)
            return fail(UMSX_EINVAL, "GGUF expert shapes do not match the layer descriptor");
        for (int p = 0; p < 3; ++p)
            if (e.type[p] != desc->quant) return fail(UMSX_EINVAL, "GGUF expert quantization does not match desc->quant");
        const bool all_bias = e.has_bias[0] && e.has_bias[1] && e.has_bias[2];
        const bool any_bias = e.has_bias[0] || e.has_bias[1] || e.has_bias[2];
        if (any_bias != all_bias || all_bias != (desc->has_bias != 0))
            return fail(UMSX_EINVAL, "GGUF expert biases do not match has_bias (gate, up and down all or none)");
        const size_t E = (size_t)desc->experts, I = (size_t)desc->intermediate, H = (size_t)desc->hidden;
        umsx_moe_weights w{};
        w.router_w = rw.data();
        w.router_b = has_rb ? rb.data() : nullptr;
        std::vector<uint8_t> fused;
        if (desc->fused_gate_up) {  // per expert: the I gate rows, then the I up rows
            const size_t sg = e.stride[0], su = e.stride[1];
            fused.resize(E * (sg + su));
            for (size_t x = 0; x < E; ++x) {
                std::memcpy(fused.data() + x * (sg + su), e.packed[0].data() + x * sg, sg);
                std::memcpy(fused.data() + x * (sg + su) + sg, e.packed[1].data() + x * su, su);
            }
            w.gate_up = fused.data();
        } else {
            w.gate = e.packed[0].data();
            w.up = e.packed[1].data();
        }
        w.down = e.packed[2].data();
        std::vector<float> gb, db;
        if (all_bias) {
            gb.resize(E * 2 * I);
            for (size_t x = 0; x < E; ++x) {
                std::memcpy(gb.data() + x * 2 * I, e.bias[0].data() + x * I, I * 4);
                std::memcpy(gb.data() + x * 2 * I + I, e.bias[1].data() + x * I, I * 4);
            }
            db = e.bias[2];
        }
        return create_from_host(desc, &w, gb.data(), db.data(), device, reserve_bytes, out);
    } catch (const std::bad_alloc &) {
        return fail(UMSX_EOOM, "host allocation failed");
    }
}

}  // extern "C"

// ============================================================================
// Expert parallelism over NVLink: exchange buffers mapped between the ranks' processes with CUDA
// IPC, and a stack of expert-parallel layers whose decode step exchanges hidden rows and job
// outputs by P2P stores from inside its kernels (umsx_ep.cu).
// ============================================================================

struct umsx_ep {
    int rank = 0, world = 1, device = 0, hidden = 0, top_k = 0;
    // h_all [world][H] f32 | y_recv [K][H] f32 | flags [world] u32 | epoch u32 | y_all [world*K][H] f32
    uint8_t *buf = nullptr;
    size_t bytes = 0, off_y = 0, off_flags = 0, off_epoch = 0, off_yall = 0;
    cudaIpcMemHandle_t handle{};
    std::vector<uint8_t *> peers;  // each rank's buffer as mapped here (own entry = buf)
    bool connected = false;
    long long wait_cycles = 2000000000LL;  // about a second at 2 GHz
};

struct umsx_ep_stack {
    umsx_ep *ep = nullptr;
    std::vector<umsx_moe *> layers;
    float eps = 1e-5f;
    Workspace ws;
    float *h_own = nullptr, *y_jobs = nullptr, *out_dev = nullptr;
    void *x_dev = nullptr;
    cudaStream_t stream = nullptr;
    cudaEvent_t ev_in = nullptr, ev_out = nullptr;
    struct Graph { int dtype; cudaGraphExec_t exec; uint64_t kernels; };
    std::vector<Graph> graphs;
    bool persistent = false;  // the one-launch expert-parallel decode kernel serves every step
    std::mutex mu;
};

namespace {

// The persistent decode kernel in its expert-parallel form serves a stack when every layer is a
// resident MXFP4 fused-gate_up layer and the step's G tokens (one per rank) fit the kernel.
bool ep_persistent_eligible(const umsx_ep_stack *st) {
    const int G = st->ep->world, L = (int)st->layers.size();
    if (G < 2 || G > kDecodeMaxTokens) return false;
    for (const umsx_moe *m : st->layers) {
        const auto &d = m->d;
        if (m->banked || d.quant != UMSX_QUANT_MXFP4 || !d.fused_gate_up || m->e_local * G != d.experts ||
            m->e_lo != st->ep->rank * m->e_local || !decode_supported(G, d.hidden, d.intermediate, d.experts, d.top_k, L))
            return false;
    }
    return true;
}

// One step as a single launch: this rank's token goes to every rank, every rank routes all G tokens
// and runs its own experts' units, each job row goes to every rank, and every layer ends with a
// cross-rank flag exchange inside the kernel (k_decode, DecodeParams::ep_world).  Row `rank` of the
// kernel's [G][H] output is this rank's token.  Returns 1 launched, 0 not resident on this device.
int record_ep_persistent(umsx_ep_stack *st, int dtype, cudaStream_t s) {
    const umsx_ep *ep = st->ep;
    const int G = ep->world, H = ep->hidden, L = (int)st->layers.size();
    const umsx_moe *m0 = st->layers[0];
    DecodeParams p = decode_params(m0, st->ws, st->x_dev, dtype, G, st->ws.out_dev);
    p.n_layers = L;
    for (int l = 0; l < L; ++l) set_decode_layer(p, l, st->layers[l]);
    p.rmsnorm = 1;
    p.residual = 1;
    p.eps = st->eps;
    p.ep_world = G;
    p.ep_rank = ep->rank;
    p.e_lo = m0->e_lo;
    p.e_local = m0->e_local;
    p.y = reinterpret_cast<float *>(ep->buf + ep->off_yall);
    for (int q = 0; q < G; ++q) {
        p.peer_y[q] = reinterpret_cast<float *>(ep->peers[q] + ep->off_yall);
        p.peer_x[q] = reinterpret_cast<float *>(ep->peers[q]);
        p.peer_flags[q] = reinterpret_cast<unsigned *>(ep->peers[q] + ep->off_flags);
    }
    p.x_all = reinterpret_cast<const float *>(ep->buf);
    p.flags = reinterpret_cast<unsigned *>(ep->buf + ep->off_flags);
    p.epoch = reinterpret_cast<unsigned *>(ep->buf + ep->off_epoch);
    p.ep_wait_cycles = ep->wait_cycles;
    if (try_decode(p, s) <= 0) return 0;
    if (cudaMemcpyAsync(st->out_dev, st->ws.out_dev + (size_t)ep->rank * H, (size_t)H * 4, cudaMemcpyDeviceToDevice, s) !=
        cudaSuccess)
        return -1;
    return 1;
}

EpParams ep_params(umsx_ep_stack *st, const umsx_moe *m) {
    const umsx_ep *ep = st->ep;
    EpParams p{};
    p.rank = ep->rank;
    p.world = ep->world;
    p.hidden = ep->hidden;
    p.top_k = ep->top_k;
    p.e_lo = m->e_lo;
    p.e_local = m->e_local;
    p.h_own = st->h_own;
    for (int q = 0; q < ep->world; ++q) {
        p.peer_h_all[q] = reinterpret_cast<float *>(ep->peers[q]);
        p.peer_y_recv[q] = reinterpret_cast<float *>(ep->peers[q] + ep->off_y);
        p.peer_flags[q] = reinterpret_cast<unsigned *>(ep->peers[q] + ep->off_flags);
    }
    p.flags = reinterpret_cast<unsigned *>(ep->buf + ep->off_flags);
    p.epoch = reinterpret_cast<unsigned *>(ep->buf + ep->off_epoch);
    p.y_recv = reinterpret_cast<const float *>(ep->buf + ep->off_y);
    p.y_jobs = st->y_jobs;
    p.ids = st->ws.disp.ids;
    p.weights = st->ws.disp.weights;
    p.err = st->ws.disp.err;
    p.wait_cycles = ep->wait_cycles;
    return p;
}

umsx_status record_ep_step(umsx_ep_stack *st, int dtype, cudaStream_t s) {
    const int H = st->ep->hidden, G = st->ep->world;
    if (st->persistent) {
        const int r = record_ep_persistent(st, dtype, s);
        if (r < 0) return fail(UMSX_EDEVICE, "expert-parallel decode: copying the output row failed");
        if (r > 0) return UMSX_OK;
    }
    if (dtype == UMSX_DTYPE_BF16)
        UMSX_LAUNCHED(launch_bf16_to_f32(static_cast<const uint16_t *>(st->x_dev), st->h_own, (size_t)H, s));
    else
        UMSX_CUDA(cudaMemcpyAsync(st->h_own, st->x_dev, (size_t)H * 4, cudaMemcpyDeviceToDevice, s));
    const float *h_all = reinterpret_cast<const float *>(st->ep->buf);
    for (umsx_moe *m : st->layers) {
        const EpParams p = ep_params(st, m);
        UMSX_LAUNCHED(launch_ep_share(p, s));
        // the replicated router (RMSNorm fused) and this rank's experts for all G tokens
        if (umsx_status r = run_layer(m, st->ws, h_all, UMSX_DTYPE_F32, G, nullptr, nullptr, 1, st->eps, s, nullptr,
                                      st->y_jobs))
            return r;
        UMSX_LAUNCHED(launch_ep_combine(p, s));
    }
    UMSX_CUDA(cudaMemcpyAsync(st->out_dev, st->h_own, (size_t)H * 4, cudaMemcpyDeviceToDevice, s));
    return UMSX_OK;
}

}  // namespace

extern "C" {

umsx_status umsx_ep_create(int rank, int world, int device, int hidden, int top_k, umsx_ep **out) {
    if (!out) return fail(UMSX_EINVAL, "null output");
    *out = nullptr;
    if (world < 1 || world > kEpMaxRanks || rank < 0 || rank >= world)
        return fail(UMSX_EINVAL, "need 1 <= world <= 8 and 0 <= rank < world");
    if (hidden <= 0 || hidden % 64 || top_k < 1 || top_k > 32) return fail(UMSX_EINVAL, "invalid hidden or top_k");
    UMSX_CUDA(cudaSetDevice(device));
    auto *ep = new umsx_ep();
    ep->rank = rank;
    ep->world = world;
    ep->device = device;
    ep->hidden = hidden;
    ep->top_k = top_k;
    ep->off_y = align_up((size_t)world * hidden * 4);
    ep->off_flags = align_up(ep->off_y + (size_t)top_k * hidden * 4);
    ep->off_epoch = ep->off_flags + (size_t)world * 4;
    ep->off_yall = align_up(ep->off_epoch + 4);
    ep->bytes = align_up(ep->off_yall + (size_t)world * top_k * hidden * 4);
    auto run = [&]() -> umsx_status {
        UMSX_CUDA(cudaMalloc(&ep->buf, ep->bytes));
        UMSX_CUDA(cudaMemset(ep->buf, 0, ep->bytes));
        UMSX_CUDA(cudaIpcGetMemHandle(&ep->handle, ep->buf));
        UMSX_CUDA(cudaDeviceSynchronize());
        return UMSX_OK;
    };
    if (umsx_status r = run()) { umsx_ep_destroy(ep); return r; }
    ep->peers.assign(world, nullptr);
    ep->peers[rank] = ep->buf;
    *out = ep;
    return UMSX_OK;
}

umsx_status umsx_ep_handle(umsx_ep *ep, void *handle_out, size_t size) {
    if (!ep || !handle_out || size != sizeof(cudaIpcMemHandle_t))
        return fail(UMSX_EINVAL, "need the group and a buffer of the IPC handle size (64 bytes)");
    std::memcpy(handle_out, &ep->handle, sizeof(cudaIpcMemHandle_t));
    return UMSX_OK;
}

umsx_status umsx_ep_connect(umsx_ep *ep, const void *handles, size_t size) {
    if (!ep || !handles || size != (size_t)ep->world * sizeof(cudaIpcMemHandle_t))
        return fail(UMSX_EINVAL, "need every rank's IPC handle (world x 64 bytes, rank order)");
    if (ep->connected) return fail(UMSX_EINVAL, "already connected");
    UMSX_CUDA(cudaSetDevice(ep->device));
    for (int q = 0; q < ep->world; ++q) {
        if (q == ep->rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const uint8_t *>(handles) + (size_t)q * sizeof(h), sizeof(h));
        void *p = nullptr;
        UMSX_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
        ep->peers[q] = static_cast<uint8_t *>(p);
    }
    ep->connected = true;
    return UMSX_OK;
}

umsx_status umsx_ep_set_wait(umsx_ep *ep, int64_t wait_limit_cycles) {
    if (!ep || wait_limit_cycles <= 0) return fail(UMSX_EINVAL, "need the group and a positive bound");
    ep->wait_cycles = wait_limit_cycles;
    return UMSX_OK;
}

void umsx_ep_destroy(umsx_ep *ep) {
    if (!ep) return;
    cudaSetDevice(ep->device);
    cudaDeviceSynchronize();
    for (int q = 0; q < (int)ep->peers.size(); ++q)
        if (q != ep->rank && ep->peers[q]) cudaIpcCloseMemHandle(ep->peers[q]);
    if (ep->buf) cudaFree(ep->buf);
    delete ep;
}

umsx_status umsx_ep_stack_create(umsx_ep *ep, umsx_moe *const *layers, int n_layers, float rms_eps,
                                 umsx_ep_stack **out) {
    if (!out || !ep || !layers || n_layers <= 0) return fail(UMSX_EINVAL, "need a group and at least one layer");
    *out = nullptr;
    if (!ep->connected) return fail(UMSX_EINVAL, "connect the group first (umsx_ep_connect)");
    const umsx_moe *l0 = layers[0];
    for (int l = 0; l < n_layers; ++l) {
        const umsx_moe *m = layers[l];
        if (!m || m->device != ep->device || m->d.hidden != ep->hidden || m->d.top_k != ep->top_k ||
            m->d.experts != l0->d.experts || m->d.intermediate != l0->d.intermediate)
            return fail(UMSX_EINVAL, "layers must share the group's device, width and top_k, and one shape");
        if (m->d.ep_world != ep->world || m->d.ep_rank != ep->rank)
            return fail(UMSX_EINVAL, "layers must be created with the group's ep_rank and ep_world");
        if (m->banked) return fail(UMSX_EUNSUPPORTED, "banked layer: call umsx_moe_forward or umsx_moe_forward_host");
    }
    UMSX_CUDA(cudaSetDevice(ep->device));
    auto *st = new umsx_ep_stack();
    st->ep = ep;
    st->layers.assign(layers, layers + n_layers);
    st->eps = rms_eps;
    const int G = ep->world, H = ep->hidden, K = ep->top_k;
    auto run = [&]() -> umsx_status {
        if (umsx_status r = alloc_workspace(st->ws, l0->d, l0->e_local, G, 0)) return r;
        UMSX_CUDA(cudaMalloc(&st->h_own, (size_t)H * 4));
        UMSX_CUDA(cudaMalloc(&st->out_dev, (size_t)H * 4));
        UMSX_CUDA(cudaMalloc(&st->x_dev, (size_t)H * 4));
        UMSX_CUDA(cudaMalloc(&st->y_jobs, (size_t)G * K * H * 4));
        UMSX_CUDA(cudaMemset(st->y_jobs, 0, (size_t)G * K * H * 4));
        UMSX_CUDA(cudaStreamCreateWithFlags(&st->stream, cudaStreamNonBlocking));
        UMSX_CUDA(cudaEventCreateWithFlags(&st->ev_in, cudaEventDisableTiming));
        UMSX_CUDA(cudaEventCreateWithFlags(&st->ev_out, cudaEventDisableTiming));
        return UMSX_OK;
    };
    if (umsx_status r = run()) { umsx_ep_stack_destroy(st); return r; }
    st->persistent = ep_persistent_eligible(st);
    *out = st;
    return UMSX_OK;
}

void umsx_ep_stack_destroy(umsx_ep_stack *st) {
    if (!st) return;
    cudaSetDevice(st->ep->device);
    if (st->stream) cudaStreamSynchronize(st->stream);
    for (auto &g : st->graphs) cudaGraphExecDestroy(g.exec);
    if (st->ev_in) cudaEventDestroy(st->ev_in);
    if (st->ev_out) cudaEventDestroy(st->ev_out);
    if (st->stream) cudaStreamDestroy(st->stream);
    for (void *p : {(void *)st->h_own, (void *)st->out_dev, st->x_dev, (void *)st->y_jobs, (void *)st->ws.mem})
        if (p) cudaFree(p);
    delete st;
}

}  // extern "C"

namespace {
umsx_status ep_stack_run(umsx_ep_stack *st, const void *x, int x_dtype, float *out, cudaMemcpyKind in_kind,
                         cudaMemcpyKind out_kind, cudaStream_t caller) {
    if (!st) return fail(UMSX_EINVAL, "null stack");
    if (!x || !out) return fail(UMSX_EINVAL, "null buffer");
    if (x_dtype != UMSX_DTYPE_F32 && x_dtype != UMSX_DTYPE_BF16) return fail(UMSX_EINVAL, "x_dtype must be F32 or BF16");
    std::lock_guard<std::mutex> lock(st->mu);
    UMSX_CUDA(cudaSetDevice(st->ep->device));
    const int H = st->ep->hidden;
    UMSX_CUDA(cudaEventRecord(st->ev_in, caller));
    UMSX_CUDA(cudaStreamWaitEvent(st->stream, st->ev_in, 0));
    UMSX_CUDA(cudaMemcpyAsync(st->x_dev, x, (size_t)H * (x_dtype == UMSX_DTYPE_BF16 ? 2 : 4), in_kind, st->stream));
    umsx_ep_stack::Graph *g = nullptr;
    for (auto &gg : st->graphs)
        if (gg.dtype == x_dtype) g = &gg;
    if (!g) {
        const uint64_t before = g_launches;
        UMSX_CUDA(cudaStreamBeginCapture(st->stream, cudaStreamCaptureModeThreadLocal));
        umsx_status r = record_ep_step(st, x_dtype, st->stream);
        cudaGraph_t graph = nullptr;
        const cudaError_t e = cudaStreamEndCapture(st->stream, &graph);
        if (r) { if (graph) cudaGraphDestroy(graph); return r; }
        if (e != cudaSuccess) return fail(UMSX_EDEVICE, std::string("ep capture: ") + cudaGetErrorString(e));
        cudaGraphExec_t exec = nullptr;
        const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        if (ie != cudaSuccess) return fail(UMSX_EDEVICE, std::string("ep instantiate: ") + cudaGetErrorString(ie));
        const uint64_t kernels = g_launches - before;
        g_launches = before;
        st->graphs.push_back({x_dtype, exec, kernels});
        g = &st->graphs.back();
    }
    UMSX_CUDA(cudaGraphLaunch(g->exec, st->stream));
    g_launches += g->kernels;
    UMSX_CUDA(cudaMemcpyAsync(out, st->out_dev, (size_t)H * 4, out_kind, st->stream));
    UMSX_CUDA(cudaEventRecord(st->ev_out, st->stream));
    UMSX_CUDA(cudaStreamWaitEvent(caller, st->ev_out, 0));
    return UMSX_OK;
}
}  // namespace

extern "C" {

umsx_status umsx_ep_stack_forward(umsx_ep_stack *st, const void *x, int x_dtype, float *out, umsx_stream stream) {
    return ep_stack_run(st, x, x_dtype, out, cudaMemcpyDeviceToDevice, cudaMemcpyDeviceToDevice,
                        static_cast<cudaStream_t>(stream));
}

umsx_status umsx_ep_stack_forward_host(umsx_ep_stack *st, const void *x, int x_dtype, float *out, umsx_stream stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (umsx_status r = ep_stack_run(st, x, x_dtype, out, cudaMemcpyHostToDevice, cudaMemcpyDeviceToHost, s)) return r;
    return check_device_flag(st->ws, s);
}

umsx_status umsx_ep_stack_status(umsx_ep_stack *st, umsx_stream stream) {
    if (!st) return fail(UMSX_EINVAL, "null stack");
    UMSX_CUDA(cudaSetDevice(st->ep->device));
    UMSX_CUDA(cudaStreamSynchronize(st->stream));
    return check_device_flag(st->ws, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ============================================================================
// Expert-parallel prefill stack: tokens sharded over the ranks, each rank's experts run over the
// rows the other ranks send it (umsx_ep.cu has the exchange kernels).
// ============================================================================

struct umsx_ep_prefill {
    umsx_ep *ep = nullptr;
    std::vector<umsx_moe *> layers;
    float eps = 1e-5f;
    int tokens_max = 0, rows_max = 0;
    Workspace ws;
    // exported receive buffers: counts [G][G] | codes [rows][H] | scales [rows][H/32] | ids [rows][K] |
    // src [rows] int2 | y_back [tokens_max][K][H] f32
    uint8_t *buf = nullptr;
    size_t bytes = 0, off_codes = 0, off_scales = 0, off_ids = 0, off_src = 0, off_y = 0;
    cudaIpcMemHandle_t handle{};
    std::vector<uint8_t *> peers;
    bool connected = false;
    int32_t *pos = nullptr;
    unsigned *done = nullptr;
    int2 *loads = nullptr;  // [layers]
    float *h = nullptr;     // [tokens_max][H] residual stream
    void *x_stage = nullptr;
    cudaStream_t stream = nullptr;
    cudaEvent_t ev_in = nullptr, ev_out = nullptr;
    std::mutex mu;
};

namespace {

EpPrefillParams ep_prefill_params(umsx_ep_prefill *st, const umsx_moe *m, int tokens) {
    const umsx_ep *ep = st->ep;
    EpPrefillParams p{};
    p.rank = ep->rank;
    p.world = ep->world;
    p.hidden = ep->hidden;
    p.top_k = ep->top_k;
    p.e_per_rank = m->e_local;
    p.tokens = tokens;
    p.tokens_max = st->tokens_max;
    p.rows_max = st->rows_max;
    p.ids = st->ws.disp.ids;
    p.xq_codes = st->ws.disp.xq_codes;
    p.xq_scales = st->ws.disp.xq_scales;
    p.pos = st->pos;
    p.counts = reinterpret_cast<int32_t *>(st->buf);
    p.done = st->done;
    for (int q = 0; q < ep->world; ++q) {
        uint8_t *b = st->peers[q];
        p.peer_counts[q] = reinterpret_cast<int32_t *>(b);
        p.peer_codes[q] = b + st->off_codes;
        p.peer_scales[q] = reinterpret_cast<float *>(b + st->off_scales);
        p.peer_ids[q] = reinterpret_cast<int32_t *>(b + st->off_ids);
        p.peer_src[q] = reinterpret_cast<int2 *>(b + st->off_src);
        p.peer_y_back[q] = reinterpret_cast<float *>(b + st->off_y);
        p.peer_flags[q] = reinterpret_cast<unsigned *>(ep->peers[q] + ep->off_flags);
    }
    p.recv_ids = reinterpret_cast<const int32_t *>(st->buf + st->off_ids);
    p.recv_src = reinterpret_cast<const int2 *>(st->buf + st->off_src);
    p.inv = st->ws.inv;
    p.y_jobs = st->ws.y;
    p.n_jobs = st->ws.disp.offsets + m->e_local;
    p.loads = st->loads;
    p.flags = reinterpret_cast<unsigned *>(ep->buf + ep->off_flags);
    p.epoch = reinterpret_cast<unsigned *>(ep->buf + ep->off_epoch);
    p.err = st->ws.disp.err;
    p.wait_cycles = ep->wait_cycles;
    return p;
}

// One layer: route this rank's tokens, send their rows to the experts' ranks, run this rank's
// experts over the rows received, send the outputs back, combine in rank order with the residual.
umsx_status record_ep_prefill_layer(umsx_ep_prefill *st, umsx_moe *m, int layer, int tokens, cudaStream_t s) {
    const int K = m->d.top_k, H = m->d.hidden, jobs = st->rows_max * K;
    const EpPrefillParams p = ep_prefill_params(st, m, tokens);
    Workspace &ws = st->ws;
    // rows past the ones received this layer must read as "no local expert" for the dispatch scan
    UMSX_CUDA(cudaMemsetAsync(st->buf + st->off_ids, 0xFF, (size_t)jobs * 4, s));
    if (umsx_status r = run_router_tiled(m, ws, st->h, UMSX_DTYPE_F32, tokens, 1, st->eps, s)) return r;
    UMSX_LAUNCHED(launch_ep_count(p, s));
    UMSX_LAUNCHED(launch_ep_wait(p, s));
    UMSX_LAUNCHED(launch_ep_dispatch(p, s));
    UMSX_LAUNCHED(launch_ep_wait(p, s));
    Dispatch dd = ws.disp;  // the received rows take the place of tokens
    dd.ids = reinterpret_cast<int32_t *>(st->buf + st->off_ids);
    dd.xq_codes = st->buf + st->off_codes;
    dd.xq_scales = reinterpret_cast<float *>(st->buf + st->off_scales);
    UMSX_LAUNCHED(launch_dispatch(dd, jobs, K, m->e_lo, m->e_local, s));
    UMSX_LAUNCHED(launch_prefill_pack(dd, jobs, dd.offsets + m->e_local, K, H, ws.a16, ws.a16 + (size_t)jobs * H, ws.inv, s));
    if (umsx_status r = run_prefill_gemms(m, ws, dd, jobs, s, nullptr)) return r;
    UMSX_LAUNCHED(launch_ep_return(p, layer, s));
    UMSX_LAUNCHED(launch_ep_wait(p, s));
    UMSX_LAUNCHED(launch_combine(reinterpret_cast<const float *>(st->buf + st->off_y), ws.disp.weights, tokens, K, H,
                                 nullptr, st->h, st->h, ws.disp.err, s));
    return UMSX_OK;
}

umsx_status ep_prefill_run(umsx_ep_prefill *st, const void *x, int x_dtype, int tokens, float *out,
                           cudaMemcpyKind in_kind, cudaMemcpyKind out_kind, cudaStream_t caller) {
    if (!st) return fail(UMSX_EINVAL, "null stack");
    if (!st->connected) return fail(UMSX_EINVAL, "connect the stack first (umsx_ep_prefill_connect)");
    if (!x || !out) return fail(UMSX_EINVAL, "null buffer");
    if (x_dtype != UMSX_DTYPE_F32 && x_dtype != UMSX_DTYPE_BF16) return fail(UMSX_EINVAL, "x_dtype must be F32 or BF16");
    if (tokens < 1 || tokens > st->tokens_max) return fail(UMSX_EINVAL, "tokens must be in [1, max_tokens]");
    std::lock_guard<std::mutex> lock(st->mu);
    UMSX_CUDA(cudaSetDevice(st->ep->device));
    const size_t n = (size_t)tokens * st->ep->hidden;
    cudaStream_t s = st->stream;
    UMSX_CUDA(cudaEventRecord(st->ev_in, caller));
    UMSX_CUDA(cudaStreamWaitEvent(s, st->ev_in, 0));
    if (x_dtype == UMSX_DTYPE_BF16) {
        UMSX_CUDA(cudaMemcpyAsync(st->x_stage, x, n * 2, in_kind, s));
        UMSX_LAUNCHED(launch_bf16_to_f32(static_cast<const uint16_t *>(st->x_stage), st->h, n, s));
    } else {
        UMSX_CUDA(cudaMemcpyAsync(st->h, x, n * 4, in_kind, s));
    }
    for (size_t l = 0; l < st->layers.size(); ++l)
        if (umsx_status r = record_ep_prefill_layer(st, st->layers[l], (int)l, tokens, s)) return r;
    UMSX_CUDA(cudaMemcpyAsync(out, st->h, n * 4, out_kind, s));
    UMSX_CUDA(cudaEventRecord(st->ev_out, s));
    UMSX_CUDA(cudaStreamWaitEvent(caller, st->ev_out, 0));
    return UMSX_OK;
}

}  // namespace

extern "C" {

umsx_status umsx_ep_prefill_create(umsx_ep *ep, umsx_moe *const *layers, int n_layers, int max_tokens, float rms_eps,
                                   umsx_ep_prefill **out) {
    if (!out || !ep || !layers || n_layers <= 0) return fail(UMSX_EINVAL, "need a group and at least one layer");
    *out = nullptr;
    const umsx_moe *l0 = layers[0];
    for (int l = 0; l < n_layers; ++l) {
        const umsx_moe *m = layers[l];
        if (!m || m->device != ep->device || m->d.hidden != ep->hidden || m->d.top_k != ep->top_k ||
            m->d.experts != l0->d.experts || m->d.intermediate != l0->d.intermediate || m->d.quant != l0->d.quant)
            return fail(UMSX_EINVAL, "layers must share the group's device, width and top_k, and one shape");
        if (m->d.ep_world != ep->world || m->d.ep_rank != ep->rank)
            return fail(UMSX_EINVAL, "layers must be created with the group's ep_rank and ep_world");
        if (m->banked) return fail(UMSX_EUNSUPPORTED, "banked layer: call umsx_moe_forward or umsx_moe_forward_host");
        if (m->e_local > 256) return fail(UMSX_EUNSUPPORTED, "more than 256 experts per rank");
    }
    if (max_tokens < 1 || (size_t)max_tokens * ep->world > 65535 || max_tokens * ep->world < kPrefillMinTokens)
        return fail(UMSX_EINVAL, "max_tokens x world must be in [65, 65535]");
    UMSX_CUDA(cudaSetDevice(ep->device));
    auto *st = new umsx_ep_prefill();
    st->ep = ep;
    st->layers.assign(layers, layers + n_layers);
    st->eps = rms_eps;
    st->tokens_max = max_tokens;
    st->rows_max = max_tokens * ep->world;
    const size_t G = ep->world, H = ep->hidden, K = ep->top_k, R = st->rows_max, T = max_tokens;
    st->off_codes = align_up(G * G * 4);
    st->off_scales = align_up(st->off_codes + R * H);
    st->off_ids = align_up(st->off_scales + R * (H / 32) * 4);
    st->off_src = align_up(st->off_ids + R * K * 4);
    st->off_y = align_up(st->off_src + R * 8);
    st->bytes = align_up(st->off_y + T * K * H * 4);
    auto run = [&]() -> umsx_status {
        if (umsx_status r = alloc_workspace(st->ws, l0->d, l0->e_local, st->rows_max, 1u << 30)) return r;
        UMSX_CUDA(cudaMalloc(&st->buf, st->bytes));
        UMSX_CUDA(cudaMemset(st->buf, 0, st->bytes));
        UMSX_CUDA(cudaIpcGetMemHandle(&st->handle, st->buf));
        UMSX_CUDA(cudaMalloc(&st->pos, T * G * 4));
        UMSX_CUDA(cudaMalloc(&st->done, 4));
        UMSX_CUDA(cudaMemset(st->done, 0, 4));
        UMSX_CUDA(cudaMalloc(&st->loads, (size_t)n_layers * sizeof(int2)));
        UMSX_CUDA(cudaMemset(st->loads, 0, (size_t)n_layers * sizeof(int2)));
        UMSX_CUDA(cudaMalloc(&st->h, T * H * 4));
        UMSX_CUDA(cudaMalloc(&st->x_stage, T * H * 2));
        UMSX_CUDA(cudaStreamCreateWithFlags(&st->stream, cudaStreamNonBlocking));
        UMSX_CUDA(cudaEventCreateWithFlags(&st->ev_in, cudaEventDisableTiming));
        UMSX_CUDA(cudaEventCreateWithFlags(&st->ev_out, cudaEventDisableTiming));
        UMSX_CUDA(cudaDeviceSynchronize());
        return UMSX_OK;
    };
    if (umsx_status r = run()) { umsx_ep_prefill_destroy(st); return r; }
    st->peers.assign(G, nullptr);
    st->peers[ep->rank] = st->buf;
    *out = st;
    return UMSX_OK;
}

umsx_status umsx_ep_prefill_handle(umsx_ep_prefill *st, void *handle_out, size_t size) {
    if (!st || !handle_out || size != sizeof(cudaIpcMemHandle_t))
        return fail(UMSX_EINVAL, "need the stack and a buffer of the IPC handle size (64 bytes)");
    std::memcpy(handle_out, &st->handle, sizeof(cudaIpcMemHandle_t));
    return UMSX_OK;
}

umsx_status umsx_ep_prefill_connect(umsx_ep_prefill *st, const void *handles, size_t size) {
    if (!st || !handles || size != (size_t)st->ep->world * sizeof(cudaIpcMemHandle_t))
        return fail(UMSX_EINVAL, "need every rank's IPC handle (world x 64 bytes, rank order)");
    if (st->connected) return fail(UMSX_EINVAL, "already connected");
    if (!st->ep->connected) return fail(UMSX_EINVAL, "connect the group first (umsx_ep_connect)");
    UMSX_CUDA(cudaSetDevice(st->ep->device));
    for (int q = 0; q < st->ep->world; ++q) {
        if (q == st->ep->rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const uint8_t *>(handles) + (size_t)q * sizeof(h), sizeof(h));
        void *p = nullptr;
        UMSX_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
        st->peers[q] = static_cast<uint8_t *>(p);
    }
    st->connected = true;
    return UMSX_OK;
}

umsx_status umsx_ep_prefill_forward(umsx_ep_prefill *st, const void *x, int x_dtype, int tokens, float *out,
                                    umsx_stream stream) {
    return ep_prefill_run(st, x, x_dtype, tokens, out, cudaMemcpyDeviceToDevice, cudaMemcpyDeviceToDevice,
                          static_cast<cudaStream_t>(stream));
}

umsx_status umsx_ep_prefill_forward_host(umsx_ep_prefill *st, const void *x, int x_dtype, int tokens, float *out,
                                         umsx_stream stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (umsx_status r = ep_prefill_run(st, x, x_dtype, tokens, out, cudaMemcpyHostToDevice, cudaMemcpyDeviceToHost, s))
        return r;
    return check_device_flag(st->ws, s);
}

umsx_status umsx_ep_prefill_loads(umsx_ep_prefill *st, int32_t *rows_jobs, int n) {
    if (!st || !rows_jobs || n < 2 * (int)st->layers.size()) return fail(UMSX_EINVAL, "need room for 2 x layers values");
    std::lock_guard<std::mutex> lock(st->mu);
    UMSX_CUDA(cudaSetDevice(st->ep->device));
    UMSX_CUDA(cudaStreamSynchronize(st->stream));
    UMSX_CUDA(cudaMemcpy(rows_jobs, st->loads, st->layers.size() * sizeof(int2), cudaMemcpyDeviceToHost));
    return UMSX_OK;
}

umsx_status umsx_ep_prefill_status(umsx_ep_prefill *st, umsx_stream stream) {
    if (!st) return fail(UMSX_EINVAL, "null stack");
    UMSX_CUDA(cudaSetDevice(st->ep->device));
    UMSX_CUDA(cudaStreamSynchronize(st->stream));
    return check_device_flag(st->ws, static_cast<cudaStream_t>(stream));
}

void umsx_ep_prefill_destroy(umsx_ep_prefill *st) {
    if (!st) return;
    cudaSetDevice(st->ep->device);
    if (st->stream) cudaStreamSynchronize(st->stream);
    for (int q = 0; q < (int)st->peers.size(); ++q)
        if (q != st->ep->rank && st->peers[q]) cudaIpcCloseMemHandle(st->peers[q]);
    if (st->ev_in) cudaEventDestroy(st->ev_in);
    if (st->ev_out) cudaEventDestroy(st->ev_out);
    if (st->stream) cudaStreamDestroy(st->stream);
    for (void *p : {(void *)st->buf, (void *)st->pos, (void *)st->done, (void *)st->loads, (void *)st->h, st->x_stage,
                    (void *)st->ws.mem})
        if (p) cudaFree(p);
    delete st;
}

}  // extern "C"
