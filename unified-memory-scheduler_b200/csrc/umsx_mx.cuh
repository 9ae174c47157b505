// Exact MXFP4 x Q8_0 dot primitives shared by the per-stage kernels
// (umsx_kernels.cu) and the persistent decode kernel (umsx_decode.cu).
#pragma once

#include <stdint.h>

#include "umsx_device.cuh"
#include "umsx_internal.h"

namespace umsx {

constexpr int kMaxExperts = 1024;

__device__ __forceinline__ bool better(float a, int ia, float b, int ib) { return a > b || (a == b && ia < ib); }

// An unsigned key in the order of the float (no NaN): -0 and +0 share a key, as they compare equal.
__device__ __forceinline__ uint32_t order_key(float f) {
    const uint32_t b = __float_as_uint(f == 0.0f ? 0.0f : f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Warp-wide routing of one token from its E logits (all 32 lanes take part;
// `lg` was written by other CTAs, so it is read through L2).  Lane r < K ends
// with the expert of rank r in `sel` and its weight in `w`.  Ties go to the lower
// expert index; a NaN logit counts as -inf (orc_route does the same).  routing: UMSX_ROUTE_TOPK_SOFTMAX (top-k of the logits, softmax
// over those k), UMSX_ROUTE_SOFTMAX_TOPK_NORM (softmax, top-k, renormalise), or
// softmax, top-k, times routed_scale.
template <int NV = kMaxExperts / 32>  // E <= 32 * NV
__device__ __forceinline__ void select_topk(const float *lg, int E, int K, int routing, float routed_scale, int lane,
                                            int &sel, float &w_out) {
    float v[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        const int e = lane + 32 * j;
        const float l = e < E ? __ldcg(lg + e) : 0.0f;
        v[j] = l != l ? -__uint_as_float(0x7f800000u) : l;  // NaN ranks lowest, so every pick is a valid expert
    }
    if (routing != UMSX_ROUTE_TOPK_SOFTMAX) {
        float m = -__uint_as_float(0x7f800000u);
#pragma unroll
        for (int j = 0; j < NV; ++j)
            if (lane + 32 * j < E) m = fmaxf(m, v[j]);
        m = warp_max(m);
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            if (lane + 32 * j < E) {
                v[j] = exp_shared(__fadd_rn(v[j], -m));
                s = __fadd_rn(s, v[j]);
            }
        }
        const float total = warp_tree_sum(s);
#pragma unroll
        for (int j = 0; j < NV; ++j)
            if (lane + 32 * j < E) v[j] = __fdiv_rn(v[j], total);
    }
    uint32_t taken = 0;
    int my_sel = -1;
    float my_val = 0.0f;
    for (int r = 0; r < K; ++r) {
        float bv = -__uint_as_float(0x7f800000u);
        int be = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int e = lane + 32 * j;
            if (e < E && !((taken >> j) & 1u) && better(v[j], e, bv, be)) { bv = v[j]; be = e; }
        }
        // warp-wide best by (value, lower index): the largest key, then the lowest index holding
        // it (a lane with no candidate offers key 0, below every value's key), then its value
        const uint32_t key = be == 0x7fffffff ? 0u : order_key(bv);
        const uint32_t top = __reduce_max_sync(kFull, key);
        const int win = (int)__reduce_min_sync(kFull, key == top ? (uint32_t)be : 0xffffffffu);
        bv = __shfl_sync(kFull, bv, win & 31);
        be = win;
        if ((be & 31) == lane) taken |= 1u << (be >> 5);
        if (lane == r) { my_sel = be; my_val = bv; }
    }
    // weights: lane r < K holds rank r
    float w = 0.0f;
    if (routing == UMSX_ROUTE_TOPK_SOFTMAX) {
        const float m = __shfl_sync(kFull, my_val, 0);
        const float ex = lane < K ? exp_shared(__fadd_rn(my_val, -m)) : 0.0f;
        float sum = 0.0f;
        for (int r = 0; r < K; ++r) sum = __fadd_rn(sum, __shfl_sync(kFull, ex, r));
        w = __fdiv_rn(ex, sum);
    } else if (routing == UMSX_ROUTE_SOFTMAX_TOPK_NORM) {
        float sum = 0.0f;
        for (int r = 0; r < K; ++r) sum = __fadd_rn(sum, __shfl_sync(kFull, my_val, r));
        w = __fdiv_rn(my_val, sum);
    } else {
        w = __fmul_rn(my_val, routed_scale);
    }
    sel = my_sel;
    w_out = w;
}

// select_topk with the per-lane value count fitted to E: with 32 values per lane for a
// 128-expert router the one selecting warp of a token runs a long serial compare chain
// over slots that hold no expert.
__device__ __forceinline__ void select_topk_fit(const float *lg, int E, int K, int routing, float routed_scale,
                                                int lane, int &sel, float &w_out) {
    if (E <= 128) select_topk<4>(lg, E, K, routing, routed_scale, lane, sel, w_out);
    else if (E <= 256) select_topk<8>(lg, E, K, routing, routed_scale, lane, sel, w_out);
    else select_topk<kMaxExperts / 32>(lg, E, K, routing, routed_scale, lane, sel, w_out);
}

constexpr long long kWaitLimitCycles = 4000000;  // ~2 ms: bounded waits on mbarriers
__host__ __device__ constexpr int pad4(int n) { return (n + 3) & ~3; }

// One warp holds the 32 Q8_0 codes of a block (code of element `lane`); writes the
// block's MXFP4 staging record: for lane half lh and lane p, at
// ((lh*2 + p/2)*16 + (p%2)*8) the code word a(lh, p) and its byte negation.
__device__ __forceinline__ void write_mx_record(int code, uint8_t *rec, int lane) {
    const uint32_t c = (uint32_t)code & 0xffu;
    const uint32_t w = c | (__shfl_down_sync(kFull, c, 1) << 8) | (__shfl_down_sync(kFull, c, 2) << 16) |
                       (__shfl_down_sync(kFull, c, 3) << 24);
    if ((lane & 3) == 0) {
        const int lh = lane >> 4, p = (lane & 15) >> 2;
        *reinterpret_cast<uint2 *>(rec + (lh * 2 + (p >> 1)) * 16 + (p & 1) * 8) = make_uint2(w, neg8x4(w));
    }
}

constexpr uint32_t kMagicI = 0x4B400000u;
constexpr float kMagicF = 12582912.0f;
__device__ __forceinline__ float lane_sum(int biased) { return __fsub_rn(__int_as_float(biased), kMagicF); }

// Staged activations of up to MT jobs: per (job, block) 4 x uint4 =
// {a(4p..4p+3), a(16+4p..), -a(4p..), -a(16+4p..)} for p = 0..3, one fp32 scale
// (the fp16 value widened) and, for Q8_0 weights, a "holds -128" flag.
struct Staged {
    const uint4 *q;
    const float *sc;
    const int *flag;
    int scs;  // scale stride per job
};

// Byte offsets of the planes of row group `rg` of local expert `e`.
__device__ __forceinline__ size_t code_offset(int quant, int e, int nrg, int rg, int nb) {
    return ((size_t)e * nrg + rg) * (size_t)nb * (quant == UMSX_QUANT_MXFP4 ? 256 : 1024);
}
__device__ __forceinline__ size_t scale_offset(int quant, int e, int nrg, int rg, int nb) {
    const int chunks = quant == UMSX_QUANT_MXFP4 ? ((nb / 2) + 3) / 4 : nb / 2;
    return ((size_t)e * nrg + rg) * (size_t)chunks * 128;
}

// Block scale 2^(e-128) of exponent byte i of a lane's quad word.  GE2: every exponent of the
// matrix is >= 2 (checked at create time), where the scale is the normal float (e - 1) << 23,
// taken from ew - 0x01010101 (no byte borrows then) with one shift and one mask; otherwise the
// general rule, subnormal for e < 2.  Both give the same bits where GE2 holds.
template <bool GE2, int I>
__device__ __forceinline__ float quad_scale(uint32_t ew, uint32_t ewm) {
    if (!GE2) return e8m0_half((ew >> (8 * I)) & 0xffu);
    constexpr int sh = 23 - 8 * I;
    return __uint_as_float((sh >= 0 ? ewm << (sh >= 0 ? sh : 0) : ewm >> (sh >= 0 ? 0 : -sh)) & 0x7f800000u);
}

template <int MT>
__device__ __forceinline__ void mx_half(uint2 wq, float eh, const uint4 *aq, const float *sc, int nb, int scs,
                                        int m, float (&acc)[MT][4], const int (&trow)[MT]) {
    uint32_t pos[4], neg[4];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        const uint32_t w = q ? wq.y : wq.x, n = w ^ 0x88888888u;
        pos[2 * q] = prmt(kMagLo, kMagHi, w);
        neg[2 * q] = prmt(kMagLo, kMagHi, n);
        pos[2 * q + 1] = prmt(kMagLo, kMagHi, w >> 16);
        neg[2 * q + 1] = prmt(kMagLo, kMagHi, n >> 16);
    }
#pragma unroll
    for (int t = 0; t < MT; ++t) {
        if (t < m) {
            const float d = __fmul_rn(sc[trow[t] * scs], eh);
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const uint4 av = aq[(size_t)trow[t] * nb * 4 + q];
                const int l0 = dp4a_ss(neg[2 * q], av.y, dp4a_ss(pos[2 * q], av.x, (int)kMagicI));
                const int l1 = dp4a_ss(neg[2 * q + 1], av.w, dp4a_ss(pos[2 * q + 1], av.z, (int)kMagicI));
                acc[t][2 * q] = __fmaf_rn(d, lane_sum(l0), acc[t][2 * q]);
                acc[t][2 * q + 1] = __fmaf_rn(d, lane_sum(l1), acc[t][2 * q + 1]);
            }
        }
    }
}

// ---- per-warp cp.async ring for the weight stream --------------------------
// A warp streams its rows (one lane half of a 16-row group: per block pair 256
// contiguous bytes, pairs 512 bytes apart) through S stages of 4 block pairs in
// shared memory, S - 1 stages in flight, so that the bytes in flight per SM do not
// depend on registers.  Stage layout: [4 pairs][32 lanes] uint2 codes, then the
// quad's 32 exponent words.  Lanes read bytes copied by other lanes, hence the
// __syncwarp after each wait.

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

constexpr int kRingStageBytes = 4 * 256 + 128;

struct MxRing {
    const uint8_t *codes;   // this warp's lane half of the row group: pair s at codes + s*512
    const uint8_t *scales;  // the row group's exponent quads: quad j at scales + j*128
    uint8_t *ring;          // S stages of kRingStageBytes
    int steps;              // block pairs
    __device__ __forceinline__ void init(const uint8_t *c, const uint8_t *sc, int nb, int lh, uint8_t *r) {
        codes = c + lh * 256;
        scales = sc;
        ring = r;
        steps = nb / 2;
    }
    // Copies stage j (pairs 4j..4j+3, exponent quad j) into slot j % S, then commits.
    template <int S>
    __device__ __forceinline__ void issue(int j, int lane) const {
        uint8_t *st = ring + (j % S) * kRingStageBytes;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int seg = 2 * k + (lane >> 4), s = 4 * j + seg;
            if (s < steps) cp_async16(st + seg * 256 + (lane & 15) * 16, codes + (size_t)s * 512 + (lane & 15) * 16);
        }
        if (lane < 8 && 4 * j < steps) cp_async16(st + 1024 + lane * 16, scales + (size_t)j * 128 + lane * 16);
        cp_async_commit();
    }
};

// mx_warp_dot over a cp.async ring of S stages.
// primed: the caller has already issued the ring's first S - 1 stages (mx_ring_prime).
// GE2: every block exponent of the matrix is >= 2 (quad_scale).
template <int MT, int S, bool GE2 = false>
__device__ __forceinline__ void mx_warp_dot_ring(const MxRing &ws, int lh, const Staged &a, int nb, int m, int lane,
                                                 float (&acc)[MT][4], const int (&trow)[MT], bool primed = false) {
#pragma unroll
    for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int l = 0; l < 4; ++l) acc[t][l] = 0.0f;
    const int half = lane >> 4;
    const uint4 *aq = a.q + half * 4 + lh * 2;
    const float *sc = a.sc + half;
    const int nst = (ws.steps + 3) / 4;
    if (!primed)
#pragma unroll
        for (int j = 0; j < S - 1; ++j) ws.issue<S>(j, lane);
    for (int j = 0; j < nst; ++j) {
        cp_async_wait<S - 2>();
        __syncwarp();
        ws.issue<S>(j + S - 1, lane);
        const uint8_t *st = ws.ring + (j % S) * kRingStageBytes;
        const uint32_t ew = *reinterpret_cast<const uint32_t *>(st + 1024 + lane * 4);
        const uint32_t ewm = ew - 0x01010101u;  // GE2 only (padding bytes past the last pair may borrow upward)
        float eh[4];
        eh[0] = quad_scale<GE2, 0>(ew, ewm);
        eh[1] = quad_scale<GE2, 1>(ew, ewm);
        eh[2] = quad_scale<GE2, 2>(ew, ewm);
        eh[3] = quad_scale<GE2, 3>(ew, ewm);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int s = 4 * j + i;
            if (s < ws.steps) {
                const uint2 wq = *reinterpret_cast<const uint2 *>(st + i * 256 + lane * 8);
                mx_half<MT>(wq, eh[i], aq + (size_t)s * 8, sc + 2 * s, nb, a.scs, m, acc, trow);
            }
        }
    }
    cp_async_wait<0>();
    __syncwarp();  // the ring is free for the next row group
}

// Issues the first S - 1 stages of a ring ahead of its mx_warp_dot_ring(..., primed = true).
template <int S>
__device__ __forceinline__ void mx_ring_prime(const MxRing &ws, int lane) {
#pragma unroll
    for (int j = 0; j < S - 1; ++j) ws.issue<S>(j, lane);
}

// Staging by bulk copy of precomputed records: job t's records (nb * 64 bytes) and
// scales (pad4(nb) floats) land at smem + t*nb*64 and at the scale area + t*pad4(nb).
// Returns false (after flagging `err`) if the copies did not complete in time.
__device__ __forceinline__ bool stage_mx_bulk(const uint8_t *rec, const float *rsc, const int *rows_s, int m, int nb,
                                              uint8_t *smem, int mt, uint64_t *bar, uint32_t &phase, uint32_t *err) {
    const int nbp = pad4(nb);
    if (threadIdx.x == 0) {
        mbar_expect_tx(bar, (uint32_t)m * (uint32_t)(nb * 64 + nbp * 4));
        for (int t = 0; t < m; ++t) {
            bulk_g2s(smem + (size_t)t * nb * 64, rec + (size_t)rows_s[t] * nb * 64, nb * 64, bar);
            bulk_g2s(smem + (size_t)mt * nb * 64 + (size_t)t * nbp * 4, rsc + (size_t)rows_s[t] * nbp, nbp * 4, bar);
        }
    }
    const bool ok = mbar_wait_bounded(bar, phase, kWaitLimitCycles);
    // one decision for the whole CTA, so that no thread leaves while others wait at a barrier
    const bool failed = __syncthreads_or(!ok) != 0;
    if (failed) {
        if (threadIdx.x == 0) atomicOr(err, 1u);
        mbar_wait_bounded(bar, phase, kWaitLimitCycles);  // let copies in flight land before leaving
    }
    phase ^= 1u;
    return !failed;
}

__device__ __forceinline__ Staged staged_bulk_view(uint8_t *smem, int mt, int nb) {
    Staged s;
    s.q = reinterpret_cast<const uint4 *>(smem);
    s.sc = reinterpret_cast<const float *>(smem + (size_t)mt * nb * 64);
    s.flag = nullptr;
    s.scs = pad4(nb);
    return s;
}

__host__ __device__ constexpr size_t bulk_staged_bytes(int mt, int nb) { return (size_t)mt * nb * 64 + (size_t)mt * pad4(nb) * 4; }

// Completes rows from the four partial lane sets: v = chain-combined lanes of this
// thread's half.  Returns the row dot on lanes < 16 of the lh = 0 warp.
template <int MT>
__device__ __forceinline__ void mx_chain_combine(float (&acc)[MT][4]) {
#pragma unroll
    for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int p = 0; p < 4; ++p) acc[t][p] = __fadd_rn(acc[t][p], __shfl_xor_sync(kFull, acc[t][p], 16));
}

__device__ __forceinline__ float mx_row_total(const float (&lo)[4], const float *hi) {
    const float t0 = __fadd_rn(hi[0], lo[0]), t1 = __fadd_rn(hi[1], lo[1]);
    const float t2 = __fadd_rn(hi[2], lo[2]), t3 = __fadd_rn(hi[3], lo[3]);
    return __fadd_rn(__fadd_rn(t0, t2), __fadd_rn(t1, t3));
}

// Thread 0: bulk-copies the router rows of experts c, c + nC, ... (n_rows of them) into smem, and
// for each the 16-byte aligned group of four router biases that holds its bias.
__device__ __forceinline__ void load_router_rows(const float *router_w, const float *router_b, int c, int nC,
                                                 int n_rows, int H, float *wrow, float (*wbias)[4], uint64_t *bar) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // earlier generic reads of wrow come first
    mbar_expect_tx(bar, (uint32_t)(n_rows * (H * 4 + (router_b ? 16 : 0))));
    for (int j = 0; j < n_rows; ++j) {
        const int e = c + j * nC;
        bulk_g2s(wrow + (size_t)j * H, router_w + (size_t)e * H, H * 4, bar);
        if (router_b) bulk_g2s(wbias[j], router_b + (e & ~3), 16, bar);
    }
}

}  // namespace umsx
