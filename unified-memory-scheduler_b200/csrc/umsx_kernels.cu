// umsx kernels for sm_100a: router, dispatch, exact quantized expert GEMVs,
// combine, and the weight layout / generator kernels.
//
// Exactness contract (reference paths inside appatalks/unified-memory-scheduler):
// an MXFP4 x Q8_0 row dot splits each 32-weight block into eight int lanes of
// four products (VPSIGNB semantics, tools/engine/quantized_cuda.cu:145-157),
// accumulates lane l of block b as fma(d_b, float(L), acc) in an even-block and
// an odd-block chain, and sums lanes as ((l0+l4)+(l2+l6))+((l1+l5)+(l3+l7))
// (tools/trace/compatible_down.cu:95-99, tools/trace/cpu_mxfp4_vnni.cpp:57-67).
// Here a lane owns one row (Q8_0) or one of the two block chains of a row (MXFP4)
// with all eight int lanes, so the chain order is the reference's and the final
// order is computed in registers after one shuffle.
#include <stdint.h>

#include "umsx_device.cuh"
#include "umsx_internal.h"
#include "umsx_mx.cuh"

namespace umsx {

// ============================================================================
// Router: logits + softmax / top-k / weights + x -> Q8_0, and (small T*K) the
// dispatch build, all in one launch.  grid = (ceil(E/4), T), block = 128.
// ============================================================================

constexpr int kRouterWarps = 4;
constexpr int kFusedDispatchMax = 512;
constexpr int kRouterRegs = 96;  // router-weight chain values a lane holds in registers (H <= 3072)

// Programmatic dependent launch: the next kernel in the stream may start once
// every CTA of this one has signalled; `pdl_wait` blocks until the previous
// kernel has completed and its writes are visible.  Both are no-ops for
// kernels launched without the PDL attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// Warp-wide selection for one token (all 32 lanes participate).
__device__ int select_token(const RouterParams &p, const Dispatch &d, int t, int lane) {
    const int K = p.top_k;
    int sel;
    float w;
    select_topk_fit(d.logits + (size_t)t * p.experts, p.experts, K, p.routing, p.routed_scale, lane, sel, w);
    if (lane < K) {
        d.ids[(size_t)t * K + lane] = sel;
        d.weights[(size_t)t * K + lane] = w;
    }
    return sel;  // lane r < K: the expert of rank r
}

// One CTA builds counts / offsets / active list / slot records / job lists for
// N = T*K entries.
__device__ void build_dispatch_cta(const Dispatch &d, int entries, int K, int e_lo, int e_local) {
    __shared__ int cnt[kMaxExperts];
    __shared__ int off[kMaxExperts];
    __shared__ int ids_s[kFusedDispatchMax];
    __shared__ int n_act_s;
    const int tid = threadIdx.x, nth = blockDim.x;
    for (int e = tid; e < e_local; e += nth) cnt[e] = 0;
    for (int j = tid; j < entries; j += nth) ids_s[j] = __ldcg(d.ids + j) - e_lo;
    __syncthreads();
    for (int j = tid; j < entries; j += nth) {
        const int e = ids_s[j];
        if (e >= 0 && e < e_local) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    if (tid < 32) {
        // exclusive scans of counts and of (count > 0), lanes own contiguous chunks
        const int chunk = (e_local + 31) / 32;
        const int lo = min(tid * chunk, e_local), hi = min(lo + chunk, e_local);
        int s = 0, a = 0;
        for (int e = lo; e < hi; ++e) { s += cnt[e]; a += cnt[e] > 0; }
        int ps = s, pa = a;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int ys = __shfl_up_sync(kFull, ps, o), ya = __shfl_up_sync(kFull, pa, o);
            if (tid >= o) { ps += ys; pa += ya; }
        }
        int base = ps - s, abase = pa - a;
        for (int e = lo; e < hi; ++e) {
            off[e] = base;
            d.offsets[e] = base;
            d.counts[e] = cnt[e];
            if (cnt[e] > 0) {
                d.active[abase] = e;
                d.slots[abase] = make_int4(e, base, cnt[e], 0);
                ++abase;
            }
            base += cnt[e];
        }
        if (tid == 31) { d.offsets[e_local] = ps; d.n_active[0] = pa; n_act_s = pa; }
    }
    __syncthreads();
    for (int sl = n_act_s + tid; sl < e_local; sl += nth) d.slots[sl] = make_int4(-1, 0, 0, 0);
    for (int e = tid; e < e_local; e += nth) cnt[e] = 0;  // reused: jobs placed so far per expert
    __syncthreads();
    // Job lists in (token, rank) order: one warp walks the entries 32 at a time; an entry's
    // place among the earlier entries of its expert = the count placed by earlier chunks +
    // the lower lanes of this chunk with the same expert (a match mask).
    if (tid < 32) {
        const unsigned below = (1u << tid) - 1u;
        for (int j0 = 0; j0 < entries; j0 += 32) {
            const int j = j0 + tid;
            const int e = j < entries ? ids_s[j] : -1;
            const bool mine = e >= 0 && e < e_local;
            const unsigned grp = __match_any_sync(kFull, mine ? e : -1);
            if (mine) {
                const int pos = off[e] + cnt[e] + __popc(grp & below);
                d.job_token[pos] = j / K;
                d.job_rank[pos] = j % K;
            }
            __syncwarp();
            if (mine && 31 - __clz(grp) == tid) cnt[e] += __popc(grp);  // the group's highest lane
            __syncwarp();
        }
    }
}

// grid = (ceil(E/4), T), block = 128: one warp per expert logit.
template <bool REGS>
__global__ void __launch_bounds__(128) k_router(RouterParams p, Dispatch d) {
    extern __shared__ float xs[];
    __shared__ float inv_s;
    __shared__ int last;
    const int t = blockIdx.y, H = p.hidden;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e = blockIdx.x * kRouterWarps + warp;
    const bool has_e = e < p.experts;
    float wv[REGS ? kRouterRegs : 1];
    if constexpr (REGS) {
        // The router weights do not depend on the previous kernel: fetch this lane's
        // chain (k = lane, lane+32, ...) before waiting on it.
        const float *wr = p.w + (size_t)(has_e ? e : 0) * H;
#pragma unroll
        for (int i = 0; i < kRouterRegs; ++i) wv[i] = (lane + 32 * i < H) ? __ldg(wr + lane + 32 * i) : 0.0f;
    }
    pdl_wait();
    pdl_launch_dependents();
    if (p.x_dtype == UMSX_DTYPE_BF16) {
        const uint2 *xb = reinterpret_cast<const uint2 *>(static_cast<const uint16_t *>(p.x) + (size_t)t * H);
#pragma unroll 8
        for (int i = threadIdx.x; i < H / 4; i += blockDim.x) {
            const uint2 v = xb[i];
            xs[4 * i + 0] = bf16_bits_to_f32(v.x & 0xffffu);
            xs[4 * i + 1] = bf16_bits_to_f32(v.x >> 16);
            xs[4 * i + 2] = bf16_bits_to_f32(v.y & 0xffffu);
            xs[4 * i + 3] = bf16_bits_to_f32(v.y >> 16);
        }
    } else {
        const float4 *xf = reinterpret_cast<const float4 *>(static_cast<const float *>(p.x) + (size_t)t * H);
#pragma unroll 8
        for (int i = threadIdx.x; i < H / 4; i += blockDim.x) reinterpret_cast<float4 *>(xs)[i] = xf[i];
    }
    __syncthreads();
    float inv = 1.0f;  // x * 1 is exact: without RMSNorm the products below leave x unchanged
    if (p.rmsnorm) {
        // RMSNorm with unit weight: sum of squares in the shared strided order (orc_rmsnorm)
        if (warp == 0) {
            float acc = 0.0f;
            if constexpr (REGS) {
#pragma unroll
                for (int i = 0; i < kRouterRegs; ++i)
                    if (lane + 32 * i < H) acc = __fmaf_rn(xs[lane + 32 * i], xs[lane + 32 * i], acc);
            } else {
                for (int k = lane; k < H; k += 32) acc = __fmaf_rn(xs[k], xs[k], acc);
            }
            const float ss = warp_tree_sum(acc);
            if (lane == 0) inv_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)H), p.eps)));
        }
        __syncthreads();
        inv = inv_s;
    }
    // x -> Q8_0 (one warp per 32-element block), spread over this token's CTAs.
    const int nbH = H / 32;
    for (int b = blockIdx.x * kRouterWarps + warp; b < nbH; b += gridDim.x * kRouterWarps) {
        const float v = __fmul_rn(xs[b * 32 + lane], inv);
        const float amax = warp_max(fabsf(v));
        const float qinv = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
        const int code = q8_code(v, qinv);
        const float qs = f16_bits_to_f32(f32_to_f16_bits(__fdiv_rn(amax, 127.0f)));
        if (p.mx_records) {
            write_mx_record(code, d.xr + ((size_t)t * nbH + b) * 64, lane);
            if (lane == 0) d.xr_sc[(size_t)t * pad4(nbH) + b] = qs;
        } else {
            d.xq_codes[((size_t)t * nbH + b) * 32 + lane_pair_offset(lane)] = (uint8_t)(int8_t)code;
            if (lane == 0) d.xq_scales[(size_t)t * nbH + b] = qs;
        }
    }
    // logits: 32 strided FMA chains, then the xor tree (orc_logit)
    if (has_e) {
        float acc = 0.0f;
        if constexpr (REGS) {
#pragma unroll
            for (int i = 0; i < kRouterRegs; ++i)
                if (lane + 32 * i < H) acc = __fmaf_rn(wv[i], __fmul_rn(xs[lane + 32 * i], inv), acc);
        } else {
            const float *wr = p.w + (size_t)e * H;
            constexpr int kRB = 16;
            for (int k0 = lane; k0 < H; k0 += 32 * kRB) {
                float w[kRB];
#pragma unroll
                for (int i = 0; i < kRB; ++i) w[i] = (k0 + 32 * i < H) ? __ldg(wr + k0 + 32 * i) : 0.0f;
#pragma unroll
                for (int i = 0; i < kRB; ++i)
                    if (k0 + 32 * i < H) acc = __fmaf_rn(w[i], __fmul_rn(xs[k0 + 32 * i], inv), acc);
            }
        }
        float l = warp_tree_sum(acc);
        if (p.b) l = __fadd_rn(l, __ldg(p.b + e));
        if (lane == 0) d.logits[(size_t)t * p.experts + e] = l;
    }
    // the last CTA of this token selects; the last token to finish builds the dispatch
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(d.token_done + t, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    int sel = -1;
    if (warp == 0) sel = select_token(p, d, t, lane);
    if (threadIdx.x == 0) d.token_done[t] = 0;
    if (!p.fuse_dispatch) return;
    if (gridDim.y == 1 && p.skip_counts) {
        // One token: the slot records follow from the selection itself (experts in
        // ascending order, one job each); counts / offsets / active are not written.
        if (warp == 0) {
            const int K = p.top_k, e = sel - p.e_lo;
            const bool res = lane < K && e >= 0 && e < p.e_local;
            int pos = 0;
            for (int j = 0; j < K; ++j) {
                const int ej = __shfl_sync(kFull, e, j);
                const bool rj = __shfl_sync(kFull, (int)res, j) != 0;
                pos += rj && ej < e;
            }
            const int nres = __popc(__ballot_sync(kFull, res));
            if (res) {
                d.slots[pos] = make_int4(e, pos, 1, 0);
                d.job_token[pos] = 0;
                d.job_rank[pos] = lane;
            }
            if (lane >= nres && lane < min(p.e_local, K)) d.slots[lane] = make_int4(-1, 0, 0, 0);
            if (lane == 0) d.n_active[0] = nres;
        }
        return;
    }
    if (gridDim.y > 1) {
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) last = atomicAdd(d.all_done, 1u) == gridDim.y - 1;
        __syncthreads();
        if (!last) return;
        __threadfence();
        if (threadIdx.x == 0) d.all_done[0] = 0;
    } else {
        __syncthreads();  // one token: this CTA selected it
    }
    build_dispatch_cta(d, p.tokens * p.top_k, p.top_k, p.e_lo, p.e_local);
}

// Large T*K: one CTA per local expert.  Each CTA histograms every entry, scans,
// and compacts its own entries in order (ballot per warp, prefix across warps).
__global__ void __launch_bounds__(256) k_dispatch(Dispatch d, int entries, int K, int e_lo, int e_local) {
    __shared__ int cnt[kMaxExperts];
    __shared__ int warp_tot[8];
    __shared__ int base_s, off_s;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int me = blockIdx.x;
    pdl_wait();
    pdl_launch_dependents();
    for (int e = tid; e < e_local; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int j = tid; j < entries; j += blockDim.x) {
        const int e = __ldcg(d.ids + j) - e_lo;
        if (e >= 0 && e < e_local) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    if (tid == 0) {
        int s = 0, a = 0, z = 0, total = 0;
        for (int e = 0; e < e_local; ++e) {
            if (e < me) { s += cnt[e]; a += cnt[e] > 0; z += cnt[e] == 0; }
            total += cnt[e] > 0;
        }
        off_s = s;
        d.offsets[me] = s;
        d.counts[me] = cnt[me];
        if (cnt[me] > 0) {
            d.active[a] = me;
            d.slots[a] = make_int4(me, s, cnt[me], 0);
        } else {
            d.slots[total + z] = make_int4(-1, 0, 0, 0);
        }
        if (me == e_local - 1) {
            d.offsets[e_local] = s + cnt[me];
            d.n_active[0] = total;
        }
        base_s = 0;
    }
    __syncthreads();
    for (int j0 = 0; j0 < entries; j0 += blockDim.x) {
        const int j = j0 + tid;
        const bool mine = j < entries && __ldcg(d.ids + j) - e_lo == me;
        const unsigned bal = __ballot_sync(kFull, mine);
        if (lane == 0) warp_tot[warp] = __popc(bal);
        __syncthreads();
        int wbase = base_s;
        for (int w = 0; w < warp; ++w) wbase += warp_tot[w];
        if (mine) {
            const int pos = off_s + wbase + __popc(bal & ((1u << lane) - 1u));
            d.job_token[pos] = j / K;
            d.job_rank[pos] = j % K;
        }
        __syncthreads();
        if (tid == 0) {
            int s = 0;
            for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += warp_tot[w];
            base_s += s;
        }
        __syncthreads();
    }
}

// ============================================================================
// Exact quantized GEMV cores.
//
// MXFP4: a warp covers 16 rows; lane L owns row L&15 and the even (L<16) or odd
// (L>=16) block chain of that row, i.e. one of the reference's two FMA chains,
// holding all eight int-lane accumulators of it.  Each block it reads 16 bytes
// (32 codes) and forms the eight 4-product lane sums with prmt (magnitudes of
// positive and of negative codes) and dp4a against staged activations and their
// byte negations (VPSIGNB semantics).  The two chains meet in one xor-16 shuffle.
// Q8_0: a warp covers 32 rows, one lane per row and one chain (the reference's
// Q8_0 dot has no even/odd split); signed dp4a, with the exact VPSIGNB path only
// for activation blocks that hold a -128 code.
// The int lane sum becomes a float exactly by starting dp4a at 0x4B400000
// (1.5*2^23) and subtracting 1.5*2^23: |sum| < 2^22 keeps it in one binade.
// ============================================================================

template <int QUANT>
struct Geo;
template <>
struct Geo<UMSX_QUANT_MXFP4> {
    static constexpr int kRowsPerWarp = 16;
    static constexpr int kChains = 2;
    static constexpr int kBatch = 8;  // block pairs per load batch
};
template <>
struct Geo<UMSX_QUANT_Q8_0> {
    static constexpr int kRowsPerWarp = 32;
    static constexpr int kChains = 1;
    static constexpr int kBatch = 4;  // blocks per load batch
};

template <int MT>
__device__ __forceinline__ void mx_block(uint4 wq, uint32_t e8, int b, const Staged &a, int nb, int m,
                                         float (&acc)[MT][8]) {
    const uint32_t wv[4] = {wq.x, wq.y, wq.z, wq.w};
    uint32_t pl[4], nl[4], ph[4], nh[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const uint32_t nw = wv[p] ^ 0x88888888u;
        pl[p] = prmt(kMagLo, kMagHi, wv[p]);
        nl[p] = prmt(kMagLo, kMagHi, nw);
        ph[p] = prmt(kMagLo, kMagHi, wv[p] >> 16);
        nh[p] = prmt(kMagLo, kMagHi, nw >> 16);
    }
    const float eh = e8m0_half(e8);
#pragma unroll
    for (int t = 0; t < MT; ++t) {
        if (t < m) {
            const uint4 *aq = a.q + ((size_t)t * nb + b) * 4;
            const float d = __fmul_rn(a.sc[t * nb + b], eh);
#pragma unroll
            for (int p = 0; p < 4; ++p) {
                const uint4 av = aq[p];
                const int lo = dp4a_ss(nl[p], av.z, dp4a_ss(pl[p], av.x, (int)kMagicI));
                const int hi = dp4a_ss(nh[p], av.w, dp4a_ss(ph[p], av.y, (int)kMagicI));
                acc[t][p] = __fmaf_rn(d, lane_sum(lo), acc[t][p]);
                acc[t][p + 4] = __fmaf_rn(d, lane_sum(hi), acc[t][p + 4]);
            }
        }
    }
}

template <int MT>
__device__ __forceinline__ void q8_block(uint4 w01, uint4 w23, uint32_t ws16, int b, const Staged &a, int nb, int m,
                                         float (&acc)[MT][8]) {
    const uint32_t lo[4] = {w01.x, w01.z, w23.x, w23.z}, hi[4] = {w01.y, w01.w, w23.y, w23.w};
    const float wd = f16_bits_to_f32(ws16);
#pragma unroll
    for (int t = 0; t < MT; ++t) {
        if (t < m) {
            const uint4 *aq = a.q + ((size_t)t * nb + b) * 4;
            const float d = __fmul_rn(wd, a.sc[t * nb + b]);
            if (!a.flag[t * nb + b]) {
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    const uint4 av = aq[p];
                    acc[t][p] = __fmaf_rn(d, lane_sum(dp4a_ss(lo[p], av.x, (int)kMagicI)), acc[t][p]);
                    acc[t][p + 4] = __fmaf_rn(d, lane_sum(dp4a_ss(hi[p], av.y, (int)kMagicI)), acc[t][p + 4]);
                }
            } else {  // |w| * (w<0 ? -a : a) with -(-128) = -128, as VPSIGNB computes it
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    const uint4 av = aq[p];
                    const uint32_t ml = __vcmplts4(lo[p], 0u), mh = __vcmplts4(hi[p], 0u);
                    const int sl = dp4a_us(neg8x4(lo[p]) & ml, av.z, dp4a_us(lo[p] & ~ml, av.x, (int)kMagicI));
                    const int sh = dp4a_us(neg8x4(hi[p]) & mh, av.w, dp4a_us(hi[p] & ~mh, av.y, (int)kMagicI));
                    acc[t][p] = __fmaf_rn(d, lane_sum(sl), acc[t][p]);
                    acc[t][p + 4] = __fmaf_rn(d, lane_sum(sh), acc[t][p + 4]);
                }
            }
        }
    }
}

// Steps per load batch.  Q8_0 by jobs per pass: Qwen3-30B-A3B / DeepSeek-V2-Lite-shaped
// layers measured best with 8 blocks at one job per pass (T = 1: 33.2 / 35.4 us against
// 35.0 / 38.5 us with 4), 4 at two to four (T = 16), 2 at eight (T = 64: 490 against 572 us).
template <int QUANT>
__host__ __device__ constexpr int stream_batch(int mt) {
    return QUANT == UMSX_QUANT_MXFP4 ? Geo<QUANT>::kBatch : (mt <= 1 ? 8 : (mt <= 4 ? 4 : 2));
}

// One warp's weight stream: batches of B steps (a step is a block pair for MXFP4,
// 16 bytes per lane; a block for Q8_0, 32 bytes per lane), each batch loaded with
// every load in flight at once.
template <int QUANT, int B_ = Geo<QUANT>::kBatch>
struct WBatch {
    static constexpr int B = B_;
    uint4 w[B][QUANT == UMSX_QUANT_MXFP4 ? 1 : 2];
    uint32_t s[QUANT == UMSX_QUANT_MXFP4 ? B / 4 : B / 2];
};

template <int QUANT, int B_ = Geo<QUANT>::kBatch>
struct WStream {
    static constexpr int B = B_;
    const uint4 *cp;
    const uint32_t *sp;
    int steps;
    __device__ __forceinline__ void init(const uint8_t *codes, const uint8_t *scales, int nb, int lane) {
        cp = reinterpret_cast<const uint4 *>(codes) + (QUANT == UMSX_QUANT_MXFP4 ? lane : 2 * lane);
        sp = reinterpret_cast<const uint32_t *>(scales) + lane;
        steps = QUANT == UMSX_QUANT_MXFP4 ? nb / 2 : nb;
    }
    __device__ __forceinline__ void load(int s0, WBatch<QUANT, B> &b) const {
        if constexpr (QUANT == UMSX_QUANT_MXFP4) {
#pragma unroll
            for (int i = 0; i < B; ++i)
                if (s0 + i < steps) b.w[i][0] = __ldg(cp + (size_t)(s0 + i) * 32);
#pragma unroll
            for (int i = 0; i < B / 4; ++i)
                if (s0 + 4 * i < steps) b.s[i] = __ldg(sp + (size_t)((s0 >> 2) + i) * 32);
        } else {
#pragma unroll
            for (int i = 0; i < B; ++i)
                if (s0 + i < steps) {
                    b.w[i][0] = __ldg(cp + (size_t)(s0 + i) * 64);
                    b.w[i][1] = __ldg(cp + (size_t)(s0 + i) * 64 + 1);
                }
#pragma unroll
            for (int i = 0; i < B / 2; ++i)
                if (s0 + 2 * i < steps) b.s[i] = __ldg(sp + (size_t)((s0 >> 1) + i) * 32);
        }
    }
};

// Dot products of one warp's rows against the staged activations.  `cur` holds
// batch 0 already in flight; the next batch is loaded before the current one is
// consumed.  Blocks are consumed strictly in order, as the FMA chains require.
template <int QUANT, int MT, int B>
__device__ __forceinline__ void warp_dot(const WStream<QUANT, B> &ws, WBatch<QUANT, B> cur, int nb, const Staged &a,
                                         int m, int lane, float (&acc)[MT][8]) {
#pragma unroll
    for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int l = 0; l < 8; ++l) acc[t][l] = 0.0f;
    const int half = lane >> 4;
    for (int s0 = 0; s0 < ws.steps; s0 += B) {
        WBatch<QUANT, B> nxt;
        if (s0 + B < ws.steps) ws.load(s0 + B, nxt);
#pragma unroll
        for (int i = 0; i < B; ++i) {
            if (s0 + i < ws.steps) {
                if constexpr (QUANT == UMSX_QUANT_MXFP4)
                    mx_block<MT>(cur.w[i][0], (cur.s[i >> 2] >> (8 * (i & 3))) & 0xffu, 2 * (s0 + i) + half, a, nb, m, acc);
                else
                    q8_block<MT>(cur.w[i][0], cur.w[i][1], (cur.s[i >> 1] >> (16 * (i & 1))) & 0xffffu, s0 + i, a, nb, m, acc);
            }
        }
        cur = nxt;
    }
}

// The reference's final order: lanes = even + odd (MXFP4), t_i = l(i+4) + l(i),
// result = (t0 + t2) + (t1 + t3).  For MXFP4 both lanes of a row end equal.
template <int QUANT>
__device__ __forceinline__ float finish_row(const float (&a)[8]) {
    float l[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        if constexpr (QUANT == UMSX_QUANT_MXFP4) l[i] = __fadd_rn(a[i], __shfl_xor_sync(kFull, a[i], 16));
        else l[i] = a[i];
    }
    const float t0 = __fadd_rn(l[4], l[0]), t1 = __fadd_rn(l[5], l[1]);
    const float t2 = __fadd_rn(l[6], l[2]), t3 = __fadd_rn(l[7], l[3]);
    return __fadd_rn(__fadd_rn(t0, t2), __fadd_rn(t1, t3));
}

// Shared-memory bytes for MT staged jobs of nb blocks.
__host__ __device__ constexpr size_t staged_bytes(int mt, int nb) { return (size_t)mt * nb * (64 + 4 + 4); }

__device__ __forceinline__ Staged staged_view(uint8_t *smem, int mt, int nb) {
    Staged s;
    s.q = reinterpret_cast<const uint4 *>(smem);
    s.sc = reinterpret_cast<const float *>(smem + (size_t)mt * nb * 64);
    s.flag = reinterpret_cast<const int *>(smem + (size_t)mt * nb * 68);
    s.scs = nb;
    return s;
}

// Stage internal-layout Q8 rows (lane-pair order codes + fp32 scales) of the given jobs.
__device__ __forceinline__ void stage_internal(const uint8_t *codes, const float *scales, const int *rows_s, int m,
                                               int nb, uint8_t *smem, int mt, bool flags) {
    uint4 *q = reinterpret_cast<uint4 *>(smem);
    float *sc = reinterpret_cast<float *>(smem + (size_t)mt * nb * 64);
    int *fl = reinterpret_cast<int *>(smem + (size_t)mt * nb * 68);
#pragma unroll 4
    for (int i = threadIdx.x; i < m * nb * 4; i += blockDim.x) {
        const int t = i / (nb * 4), r = i - t * nb * 4, b = r >> 2, p = r & 3;
        const uint2 v = __ldcg(reinterpret_cast<const uint2 *>(codes + ((size_t)rows_s[t] * nb + b) * 32 + p * 8));
        q[((size_t)t * nb + b) * 4 + p] = make_uint4(v.x, v.y, neg8x4(v.x), neg8x4(v.y));
    }
#pragma unroll 2
    for (int i = threadIdx.x; i < m * nb; i += blockDim.x) {
        const int t = i / nb, b = i - t * nb;
        sc[i] = __ldcg(scales + (size_t)rows_s[t] * nb + b);
        if (flags) {
            const uint4 *c = reinterpret_cast<const uint4 *>(codes + ((size_t)rows_s[t] * nb + b) * 32);
            const uint4 c0 = __ldcg(c), c1 = __ldcg(c + 1);
            const uint32_t any = __vcmpeq4(c0.x, 0x80808080u) | __vcmpeq4(c0.y, 0x80808080u) |
                                 __vcmpeq4(c0.z, 0x80808080u) | __vcmpeq4(c0.w, 0x80808080u) |
                                 __vcmpeq4(c1.x, 0x80808080u) | __vcmpeq4(c1.y, 0x80808080u) |
                                 __vcmpeq4(c1.z, 0x80808080u) | __vcmpeq4(c1.w, 0x80808080u);
            fl[i] = any != 0;
        }
    }
}

// ============================================================================
// gate_up (+bias, +activation, +Q8_0 of the activation): a CTA computes 32
// intermediate values (their gate rows and up rows) for every job of one
// expert, then quantizes that 32-value block.  grid = (I/32, slots).
// ============================================================================

template <int QUANT, int MT>
__global__ void __launch_bounds__(64 * Geo<QUANT>::kChains) k_gate_up(GateUpParams p, Dispatch d) {
    constexpr int RPW = Geo<QUANT>::kRowsPerWarp, GW = 32 / RPW;  // warps per half (gate or up)
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ float res[MT][2][32];
    __shared__ int rows_s[MT];
    pdl_wait();
    pdl_launch_dependents();
    const int4 rec = __ldcg(d.slots + blockIdx.y);
    const int e = rec.x;
    if (e < 0) return;
    const int seg = rec.y, cnt = rec.z;
    const int H = p.hidden, I = p.intermediate, nb = H / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int half = warp / GW, wi = warp % GW;
    const Matrix &mat = p.fused ? p.gate_up : (half ? p.up : p.gate);
    const int nrg = mat.rows / RPW;
    const int rg_half = blockIdx.x * GW + wi;  // row group within the gate (or up) rows
    const int rg = p.fused ? half * (I / RPW) + rg_half : rg_half;
    WStream<QUANT, stream_batch<QUANT>(MT)> ws;
    ws.init(mat.codes + code_offset(QUANT, e, nrg, rg, nb), mat.scales + scale_offset(QUANT, e, nrg, rg, nb), nb, lane);
    WBatch<QUANT, stream_batch<QUANT>(MT)> first;
    ws.load(0, first);  // weights stream while the activations are staged
    const int rrow = lane % RPW;            // row within this warp
    const int row = rg_half * RPW + rrow;   // intermediate index
    const float bias = p.bias ? __ldg(p.bias + (size_t)e * 2 * I + half * I + row) : 0.0f;
    const Staged st = staged_view(smem, MT, nb);
    const int nbI = I / 32;
    for (int c0 = 0; c0 < cnt; c0 += MT) {
        const int m = min(MT, cnt - c0);
        if (c0 > 0) ws.load(0, first);
        __syncthreads();
        if (threadIdx.x < m) rows_s[threadIdx.x] = __ldcg(d.job_token + seg + c0 + threadIdx.x);
        __syncthreads();
        stage_internal(d.xq_codes, d.xq_scales, rows_s, m, nb, smem, MT, QUANT == UMSX_QUANT_Q8_0);
        __syncthreads();
        float acc[MT][8];
        warp_dot<QUANT, MT, stream_batch<QUANT>(MT)>(ws, first, nb, st, m, lane, acc);
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            if (t < m) {
                const float v = __fadd_rn(finish_row<QUANT>(acc[t]), bias);
                if (lane < RPW) res[t][half][wi * RPW + rrow] = v;
            }
        }
        __syncthreads();
        // activation + Q8_0: warp w quantizes the 32 values of jobs w, w + nwarps, ...
        for (int t = warp; t < m; t += 2 * GW) {
            const float g = res[t][0][lane], u = res[t][1][lane];
            const float a = p.activation == UMSX_ACT_SWIGLU_OAI ? swiglu_oai(g, u, p.alpha, p.limit) : silu_mul(g, u);
            const float amax = warp_max(fabsf(a));
            const float inv = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
            const size_t jrow = (size_t)(seg + c0 + t);
            p.act_codes[(jrow * nbI + blockIdx.x) * 32 + lane_pair_offset(lane)] = (uint8_t)(int8_t)q8_code(a, inv);
            if (lane == 0)
                p.act_scales[jrow * nbI + blockIdx.x] = f16_bits_to_f32(f32_to_f16_bits(__fdiv_rn(amax, 127.0f)));
        }
    }
}

// ============================================================================
// Generic expert GEMV: out[row(job)][n] = dot(W_e[n], act(job)) (+ bias).
// One CTA = W warps of one expert; grid = (N / (W*rows-per-warp), slots).
// Activation sources: 0 = internal Q8 (codes + fp32 scales), 1 = ggml block_q8_0
// rows, 2 = fp32 rows quantized here with the x86 Q8_0 rule.
// ============================================================================

struct GemvSrc {
    const uint8_t *q8_codes;
    const float *q8_scales;
    const uint8_t *ggml;
    const float *f32;
};

template <int QUANT, int W, int MT, int SRC, int COMBINE>
__global__ void __launch_bounds__(W * 32) k_gemv(GemvParams p, GemvSrc src, Dispatch d) {
    constexpr int RPW = Geo<QUANT>::kRowsPerWarp;
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ int rows_s[MT], outs_s[MT], last_s[MT];
    if (!p.prefetch_early) {
        pdl_wait();
        pdl_launch_dependents();
    }
    const int4 rec = __ldcg(d.slots + blockIdx.y);
    const int e = rec.x;
    if (e < 0) return;
    const int seg = rec.y, cnt = rec.z;
    const int N = p.m.rows, nb = p.m.cols / 32, nrg = N / RPW;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rg = blockIdx.x * W + warp;
    const bool active_warp = rg < nrg;
    WStream<QUANT, stream_batch<QUANT>(MT)> ws;
    ws.init(p.m.codes + code_offset(QUANT, e, nrg, active_warp ? rg : 0, nb),
            p.m.scales + scale_offset(QUANT, e, nrg, active_warp ? rg : 0, nb), nb, lane);
    WBatch<QUANT, stream_batch<QUANT>(MT)> first;
    if (active_warp) ws.load(0, first);
    if (p.prefetch_early) {  // the weights were chosen two kernels back; the activations come from the last one
        pdl_wait();
        pdl_launch_dependents();
    }
    const int n = rg * RPW + lane % RPW;
    const float bias = (p.bias && active_warp) ? __ldg(p.bias + (size_t)e * N + n) : 0.0f;
    const Staged st = staged_view(smem, MT, nb);
    uint4 *sq = reinterpret_cast<uint4 *>(smem);
    float *ssc = reinterpret_cast<float *>(smem + (size_t)MT * nb * 64);
    int *sfl = reinterpret_cast<int *>(smem + (size_t)MT * nb * 68);
    for (int c0 = 0; c0 < cnt; c0 += MT) {
        const int m = min(MT, cnt - c0);
        if (c0 > 0 && active_warp) ws.load(0, first);
        __syncthreads();
        if (threadIdx.x < m) {
            const int j = seg + c0 + threadIdx.x;
            const int tok = __ldcg(d.job_token + j), rank = __ldcg(d.job_rank + j);
            rows_s[threadIdx.x] = p.a_by_job ? j : tok * p.a_ts + rank * p.a_rs;
            outs_s[threadIdx.x] = tok * p.o_ts + rank;
        }
        __syncthreads();
        if constexpr (SRC == 0) {
            stage_internal(src.q8_codes, src.q8_scales, rows_s, m, nb, smem, MT, QUANT == UMSX_QUANT_Q8_0);
        } else if constexpr (SRC == 1) {
            for (int i = threadIdx.x; i < m * nb * 4; i += blockDim.x) {
                const int t = i / (nb * 4), r = i - t * nb * 4, b = r >> 2, pp = r & 3;
                const uint8_t *blk = src.ggml + ((size_t)rows_s[t] * nb + b) * 34 + 2;
                uint32_t lo = 0, hi = 0;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    lo |= (uint32_t)blk[4 * pp + k] << (8 * k);
                    hi |= (uint32_t)blk[16 + 4 * pp + k] << (8 * k);
                }
                sq[((size_t)t * nb + b) * 4 + pp] = make_uint4(lo, hi, neg8x4(lo), neg8x4(hi));
            }
            for (int i = threadIdx.x; i < m * nb; i += blockDim.x) {
                const int t = i / nb, b = i - t * nb;
                const uint8_t *blk = src.ggml + ((size_t)rows_s[t] * nb + b) * 34;
                ssc[i] = f16_bits_to_f32((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
                if (QUANT == UMSX_QUANT_Q8_0) {
                    int any = 0;
                    for (int k = 0; k < 32; ++k) any |= blk[2 + k] == 0x80;
                    sfl[i] = any;
                }
            }
        } else {
            uint8_t *sb = smem;
            for (int i = warp; i < m * nb; i += W) {
                const int t = i / nb, b = i - t * nb;
                const float v = __ldg(src.f32 + (size_t)rows_s[t] * p.m.cols + b * 32 + lane);
                const float amax = warp_max(fabsf(v));
                const float inv = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
                const int q = q8_code(v, inv);
                // code byte of element `lane` into the a(...) words of lane pair (lane%16)/4
                sb[((size_t)i * 4 + ((lane & 15) >> 2)) * 16 + (lane >> 4) * 4 + (lane & 3)] = (uint8_t)(int8_t)q;
                __syncwarp();
                if (lane < 4) {
                    uint4 *slot4 = sq + (size_t)i * 4 + lane;
                    const uint4 cur = *slot4;
                    *slot4 = make_uint4(cur.x, cur.y, neg8x4(cur.x), neg8x4(cur.y));
                }
                const unsigned has = __ballot_sync(kFull, q == -128);
                if (lane == 0) {
                    ssc[i] = f16_bits_to_f32(f32_to_f16_bits(__fdiv_rn(amax, 127.0f)));
                    sfl[i] = has != 0;
                }
            }
        }
        __syncthreads();
        if (active_warp) {
            float acc[MT][8];
            warp_dot<QUANT, MT, stream_batch<QUANT>(MT)>(ws, first, nb, st, m, lane, acc);
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                if (t < m) {
                    float v = finish_row<QUANT>(acc[t]);
                    if (p.bias) v = __fadd_rn(v, bias);
                    if (lane < RPW) p.out[(size_t)outs_s[t] * N + n] = v;
                }
            }
        }
        if constexpr (COMBINE) {
            // Rank-order combine (+ residual) of this CTA's rows, done by whichever of the
            // K expert CTAs of a token finishes last: no CTA waits for another.
            __threadfence();  // every writer of this CTA's rows publishes them at device scope
            __syncthreads();
            if (threadIdx.x < m) {
                const int tok = outs_s[threadIdx.x] / p.top_k;
                const unsigned prev = atomicAdd(p.tile_done + (size_t)tok * gridDim.x + blockIdx.x, 1u);
                last_s[threadIdx.x] = prev == (unsigned)(p.top_k - 1) ? tok : -1;
            }
            __syncthreads();
            for (int t = 0; t < m; ++t) {
                const int tok = last_s[t];
                if (tok < 0) continue;
                __threadfence();
                const int K = p.top_k, n0 = blockIdx.x * W * RPW;
                for (int i = threadIdx.x; i < W * RPW && n0 + i < N; i += blockDim.x) {
                    float acc = 0.0f;
                    for (int r = 0; r < K; ++r)
                        acc = __fadd_rn(acc, __fmul_rn(__ldcg(p.route_w + (size_t)tok * K + r),
                                                       __ldcg(p.out + ((size_t)tok * K + r) * N + n0 + i)));
                    if (p.extra) acc = __fadd_rn(acc, __ldcg(p.extra + (size_t)tok * N + n0 + i));
                    if (p.residual) acc = __fadd_rn(p.residual[(size_t)tok * N + n0 + i], acc);
                    flag_nonfinite(acc, d.err);
                    p.combine_out[(size_t)tok * N + n0 + i] = acc;
                }
                if (threadIdx.x == 0) p.tile_done[(size_t)tok * gridDim.x + blockIdx.x] = 0;
            }
        }
    }
}

// ============================================================================
// MXFP4 expert GEMVs (4 threads per row).
//
// A row is shared by four threads: block chain h (even / odd blocks, the
// reference's two FMA chains) x lane half lh (int lanes 0-3 = the low-nibble
// elements 4p..4p+3, or lanes 4-7 = the high-nibble elements 16+4p..16+4p+3).
// A warp holds 16 rows x 2 chains of one lane half; a row group of 16 rows is a
// warp pair.  Per block a thread loads 8 bytes (two words, each the selectors
// of two of its lanes) and forms 4 lane sums with prmt + dp4a.  Chains meet by an
// xor-16 shuffle, lane halves through shared memory, then the reference's
// order t_i = l(i+4) + l(i), (t0 + t2) + (t1 + t3).
// Code-plane chunk (row group, block pair) = 512 bytes: [lh][L = 16h + r][word0, word1],
// word0 = sel(p0) | sel(p1) << 16, word1 = sel(p2) | sel(p3) << 16, sel(p) = the
// four 4-bit codes of lane p of this lane half.
// Staged activations per (job, block): 4 uint4 [lh*2 + q] =
// {a(lh, 2q), -a(lh, 2q), a(lh, 2q+1), -a(lh, 2q+1)}, a(lh, p) = its 4 code bytes.
// ============================================================================

// Staging into the MXFP4 record layout from internal Q8 rows (lane-pair order).
__device__ __forceinline__ void stage_mx_internal(const uint8_t *codes, const float *scales, const int *rows_s, int m,
                                                  int nb, uint8_t *smem, int mt) {
    uint4 *q = reinterpret_cast<uint4 *>(smem);
    float *sc = reinterpret_cast<float *>(smem + (size_t)mt * nb * 64);
#pragma unroll 4
    for (int i = threadIdx.x; i < m * nb * 4; i += blockDim.x) {
        const int t = i / (nb * 4), r = i - t * nb * 4, b = r >> 2, lh = (r >> 1) & 1, qq = r & 1;
        const uint32_t *src = reinterpret_cast<const uint32_t *>(codes + ((size_t)rows_s[t] * nb + b) * 32);
        const uint32_t a0 = __ldcg(src + (2 * qq) * 2 + lh), a1 = __ldcg(src + (2 * qq + 1) * 2 + lh);
        q[((size_t)t * nb + b) * 4 + lh * 2 + qq] = make_uint4(a0, neg8x4(a0), a1, neg8x4(a1));
    }
#pragma unroll 2
    for (int i = threadIdx.x; i < m * nb; i += blockDim.x) {
        const int t = i / nb, b = i - t * nb;
        sc[i] = __ldcg(scales + (size_t)rows_s[t] * nb + b);
    }
}

// From ggml block_q8_0 rows (34-byte blocks).
__device__ __forceinline__ void stage_mx_ggml(const uint8_t *ggml, const int *rows_s, int m, int nb, uint8_t *smem,
                                              int mt) {
    uint4 *q = reinterpret_cast<uint4 *>(smem);
    float *sc = reinterpret_cast<float *>(smem + (size_t)mt * nb * 64);
    for (int i = threadIdx.x; i < m * nb * 4; i += blockDim.x) {
        const int t = i / (nb * 4), r = i - t * nb * 4, b = r >> 2, lh = (r >> 1) & 1, qq = r & 1;
        const uint8_t *blk = ggml + ((size_t)rows_s[t] * nb + b) * 34 + 2 + lh * 16;
        uint32_t a0 = 0, a1 = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            a0 |= (uint32_t)blk[4 * (2 * qq) + k] << (8 * k);
            a1 |= (uint32_t)blk[4 * (2 * qq + 1) + k] << (8 * k);
        }
        q[((size_t)t * nb + b) * 4 + lh * 2 + qq] = make_uint4(a0, neg8x4(a0), a1, neg8x4(a1));
    }
    for (int i = threadIdx.x; i < m * nb; i += blockDim.x) {
        const int t = i / nb, b = i - t * nb;
        const uint8_t *blk = ggml + ((size_t)rows_s[t] * nb + b) * 34;
        sc[i] = f16_bits_to_f32((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
    }
}

// From fp32 rows, quantized here with the x86 Q8_0 rule (one warp per 32-value block).
__device__ __forceinline__ void stage_mx_f32(const float *f32, int cols, const int *rows_s, int m, int nb,
                                             uint8_t *smem, int mt) {
    constexpr int U = 8;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    float *sc = reinterpret_cast<float *>(smem + (size_t)mt * nb * 64);
    // element `lane` of a block: lane half lh = lane/16, lane p = (lane%16)/4, byte j = lane%4
    const int off = ((lane >> 4) * 2 + ((lane & 15) >> 3)) * 16 + (((lane & 15) >> 2) & 1) * 8 + (lane & 3);
    for (int i0 = warp; i0 < m * nb; i0 += nw * U) {
        float v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = i0 + u * nw;
            if (i < m * nb) {
                const int t = i / nb, b = i - t * nb;
                v[u] = __ldcg(f32 + (size_t)rows_s[t] * cols + b * 32 + lane);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = i0 + u * nw;
            if (i < m * nb) {
                const float amax = warp_max(fabsf(v[u]));
                const float inv = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
                uint8_t *rec = smem + (size_t)i * 64;
                rec[off] = (uint8_t)(int8_t)q8_code(v[u], inv);
                __syncwarp();
                if (lane < 8) {  // word k: lane half k/4, lane p = k%4
                    uint32_t *wa = reinterpret_cast<uint32_t *>(rec + ((lane >> 2) * 2 + ((lane & 3) >> 1)) * 16 + (lane & 1) * 8);
                    wa[1] = neg8x4(wa[0]);
                }
                if (lane == 0) sc[i] = f16_bits_to_f32(f32_to_f16_bits(__fdiv_rn(amax, 127.0f)));
                __syncwarp();
            }
        }
    }
}

// gate_up for MXFP4: a CTA computes 16 intermediate values (warps: gate lh0, gate
// lh1, up lh0, up lh1) for every job of one expert and writes the activated fp32
// values; the down kernel quantizes them.  grid = (I/16, slots).  Each warp streams
// its weights through an S-stage cp.async ring placed after the staged activations;
// the ring's first S - 1 stages are in flight while the activations are copied in.
template <int MT, int S>
__global__ void __launch_bounds__(128) k_gate_up_mx(GateUpParams p, Dispatch d) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ float xch[MT][2][16][4];
    __shared__ float res[MT][2][16];
    __shared__ int rows_s[MT], last_s[MT];
    __shared__ __align__(8) uint64_t bar;
    pdl_wait();
    pdl_launch_dependents();
    const int4 rec = __ldcg(d.slots + blockIdx.y);
    const int e = rec.x;
    if (e < 0) return;
    const int seg = rec.y, cnt = rec.z;
    const int H = p.hidden, I = p.intermediate, nb = H / 32, nbI = I / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int half = warp >> 1, lh = warp & 1;
    const Matrix &mat = p.fused ? p.gate_up : (half ? p.up : p.gate);
    const int nrg = mat.rows / 16;
    const int rg = p.fused ? half * (I / 16) + blockIdx.x : blockIdx.x;
    MxRing ws;
    ws.init(mat.codes + code_offset(UMSX_QUANT_MXFP4, e, nrg, rg, nb),
            mat.scales + scale_offset(UMSX_QUANT_MXFP4, e, nrg, rg, nb), nb, lh,
            smem + bulk_staged_bytes(MT, nb) + (size_t)warp * S * kRingStageBytes);
    mx_ring_prime<S>(ws, lane);  // weights stream while the activations are copied in
    if (threadIdx.x == 0) mbar_init(&bar, 1);
    int trow[MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) trow[t] = t;
    uint32_t phase = 0;
    const int r = lane & 15;
    const float bias = p.bias ? __ldg(p.bias + (size_t)e * 2 * I + half * I + blockIdx.x * 16 + r) : 0.0f;
    const Staged st = staged_bulk_view(smem, MT, nb);
    for (int c0 = 0; c0 < cnt; c0 += MT) {
        const int m = min(MT, cnt - c0);
        __syncthreads();
        if (threadIdx.x < m) rows_s[threadIdx.x] = __ldcg(d.job_token + seg + c0 + threadIdx.x);
        __syncthreads();
        if (!stage_mx_bulk(d.xr, d.xr_sc, rows_s, m, nb, smem, MT, &bar, phase, d.err)) {
            cp_async_wait<0>();  // the ring's copies land before the CTA leaves
            return;
        }
        float acc[MT][4];
        if (mat.exp_ge2) mx_warp_dot_ring<MT, S, true>(ws, lh, st, nb, m, lane, acc, trow, c0 == 0);
        else mx_warp_dot_ring<MT, S, false>(ws, lh, st, nb, m, lane, acc, trow, c0 == 0);
        mx_chain_combine<MT>(acc);
        if (lh == 1 && lane < 16)
#pragma unroll
            for (int t = 0; t < MT; ++t)
                if (t < m)
#pragma unroll
                    for (int q = 0; q < 4; ++q) xch[t][half][r][q] = acc[t][q];
        __syncthreads();
        if (lh == 0 && lane < 16)
#pragma unroll
            for (int t = 0; t < MT; ++t)
                if (t < m) res[t][half][r] = __fadd_rn(mx_row_total(acc[t], xch[t][half][r]), bias);
        __syncthreads();
        for (int i = threadIdx.x; i < m * 16; i += blockDim.x) {
            const int t = i >> 4, k = i & 15;
            const float g = res[t][0][k], u = res[t][1][k];
            const float a = p.activation == UMSX_ACT_SWIGLU_OAI ? swiglu_oai(g, u, p.alpha, p.limit) : silu_mul(g, u);
            p.act_f32[(size_t)(seg + c0 + t) * I + blockIdx.x * 16 + k] = a;
        }
        // The two CTAs of a 32-value block: the one finishing second quantizes it
        // into the down kernel's staging record.  No CTA waits for the other.
        __threadfence();
        __syncthreads();
        if (threadIdx.x < m) {
            const unsigned prev = atomicAdd(p.act_done + (size_t)(seg + c0 + threadIdx.x) * nbI + (blockIdx.x >> 1), 1u);
            last_s[threadIdx.x] = prev == 1u;
        }
        __syncthreads();
        for (int t = warp; t < m; t += 4) {
            if (!last_s[t]) continue;
            __threadfence();
            const size_t job = (size_t)(seg + c0 + t), blk = blockIdx.x >> 1;
            const float a = __ldcg(p.act_f32 + job * I + blk * 32 + lane);
            const float amax = warp_max(fabsf(a));
            const float qinv = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
            write_mx_record(q8_code(a, qinv), p.act_rec + (job * nbI + blk) * 64, lane);
            if (lane == 0) {
                p.act_sc[job * pad4(nbI) + blk] = f16_bits_to_f32(f32_to_f16_bits(__fdiv_rn(amax, 127.0f)));
                p.act_done[job * nbI + blk] = 0;
            }
        }
    }
}

// Generic MXFP4 GEMV: W row groups (2W warps) of one expert; grid = (N/(16W), slots).
// Sources as k_gemv: 0 internal Q8, 1 ggml block_q8_0, 2 fp32 (quantized here), 3 bulk-copied
// records.  Weights stream through one S-stage cp.async ring per warp, after the staging area.
template <int W, int MT, int SRC, int COMBINE, int S>
__global__ void __launch_bounds__(W * 64) k_gemv_mx(GemvParams p, GemvSrc src, Dispatch d) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ float xch[MT][W][16][4];
    __shared__ int rows_s[MT], outs_s[MT], last_s[MT];
    __shared__ __align__(8) uint64_t bar;
    if (!p.prefetch_early) {
        pdl_wait();
        pdl_launch_dependents();
    }
    const int4 rec = __ldcg(d.slots + blockIdx.y);
    const int e = rec.x;
    if (e < 0) return;
    const int seg = rec.y, cnt = rec.z;
    const int N = p.m.rows, nb = p.m.cols / 32, nrg = N / 16;
    uint32_t phase = 0;
    if (SRC == 3 && threadIdx.x == 0) mbar_init(&bar, 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rgl = warp >> 1, lh = warp & 1;
    const int rg = blockIdx.x * W + rgl;
    const bool active_rg = rg < nrg;
    MxRing ws;
    ws.init(p.m.codes + code_offset(UMSX_QUANT_MXFP4, e, nrg, active_rg ? rg : 0, nb),
            p.m.scales + scale_offset(UMSX_QUANT_MXFP4, e, nrg, active_rg ? rg : 0, nb), nb, lh,
            smem + (SRC == 3 ? bulk_staged_bytes(MT, nb) : staged_bytes(MT, nb)) + (size_t)warp * S * kRingStageBytes);
    if (active_rg) mx_ring_prime<S>(ws, lane);
    int trow[MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) trow[t] = t;
    if (p.prefetch_early) {  // the weights were chosen two kernels back; the activations come from the last one
        pdl_wait();
        pdl_launch_dependents();
    }
    const int r = lane & 15;
    const int n = rg * 16 + r;
    const float bias = (p.bias && active_rg) ? __ldg(p.bias + (size_t)e * N + n) : 0.0f;
    const Staged st = SRC == 3 ? staged_bulk_view(smem, MT, nb) : staged_view(smem, MT, nb);
    for (int c0 = 0; c0 < cnt; c0 += MT) {
        const int m = min(MT, cnt - c0);
        __syncthreads();
        if (threadIdx.x < m) {
            const int j = seg + c0 + threadIdx.x;
            const int tok = __ldcg(d.job_token + j), rank = __ldcg(d.job_rank + j);
            rows_s[threadIdx.x] = p.a_by_job ? j : tok * p.a_ts + rank * p.a_rs;
            outs_s[threadIdx.x] = tok * p.o_ts + rank;
        }
        __syncthreads();
        if constexpr (SRC == 0) stage_mx_internal(src.q8_codes, src.q8_scales, rows_s, m, nb, smem, MT);
        else if constexpr (SRC == 1) stage_mx_ggml(src.ggml, rows_s, m, nb, smem, MT);
        else if constexpr (SRC == 2) stage_mx_f32(src.f32, p.m.cols, rows_s, m, nb, smem, MT);
        else if (!stage_mx_bulk(p.a_rec, p.a_rsc, rows_s, m, nb, smem, MT, &bar, phase, d.err)) {
            cp_async_wait<0>();  // the ring's copies land before the CTA leaves
            return;
        }
        __syncthreads();
        float acc[MT][4];
        if (active_rg) {
            if (p.m.exp_ge2) mx_warp_dot_ring<MT, S, true>(ws, lh, st, nb, m, lane, acc, trow, c0 == 0);
            else mx_warp_dot_ring<MT, S, false>(ws, lh, st, nb, m, lane, acc, trow, c0 == 0);
            mx_chain_combine<MT>(acc);
            if (lh == 1 && lane < 16)
#pragma unroll
                for (int t = 0; t < MT; ++t)
                    if (t < m)
#pragma unroll
                        for (int q = 0; q < 4; ++q) xch[t][rgl][r][q] = acc[t][q];
        }
        __syncthreads();
        if (active_rg && lh == 0 && lane < 16) {
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                if (t < m) {
                    float v = mx_row_total(acc[t], xch[t][rgl][r]);
                    if (p.bias) v = __fadd_rn(v, bias);
                    p.out[(size_t)outs_s[t] * N + n] = v;
                }
            }
        }
        if constexpr (COMBINE) {
            // Rank-order combine (+ residual) of this CTA's rows, done by whichever of the
            // K expert CTAs of a token finishes last: no CTA waits for another.
            __threadfence();
            __syncthreads();
            if (threadIdx.x < m) {
                const int tok = outs_s[threadIdx.x] / p.top_k;
                const unsigned prev = atomicAdd(p.tile_done + (size_t)tok * gridDim.x + blockIdx.x, 1u);
                last_s[threadIdx.x] = prev == (unsigned)(p.top_k - 1) ? tok : -1;
            }
            __syncthreads();
            for (int t = 0; t < m; ++t) {
                const int tok = last_s[t];
                if (tok < 0) continue;
                __threadfence();
                const int K = p.top_k, n0 = blockIdx.x * W * 16;
                for (int i = threadIdx.x; i < W * 16 && n0 + i < N; i += blockDim.x) {
                    float acc2 = 0.0f;
                    for (int rr = 0; rr < K; ++rr)
                        acc2 = __fadd_rn(acc2, __fmul_rn(__ldcg(p.route_w + (size_t)tok * K + rr),
                                                         __ldcg(p.out + ((size_t)tok * K + rr) * N + n0 + i)));
                    if (p.extra) acc2 = __fadd_rn(acc2, __ldcg(p.extra + (size_t)tok * N + n0 + i));
                    if (p.residual) acc2 = __fadd_rn(p.residual[(size_t)tok * N + n0 + i], acc2);
                    flag_nonfinite(acc2, d.err);
                    p.combine_out[(size_t)tok * N + n0 + i] = acc2;
                }
                if (threadIdx.x == 0) p.tile_done[(size_t)tok * gridDim.x + blockIdx.x] = 0;
            }
        }
    }
}

// ============================================================================
// Combine: out[t][i] = ((0 + w0*y0) + w1*y1) + ... (expert_dispatch.cpp:77-87).
// ============================================================================

__global__ void k_combine(const float *__restrict__ y, const float *__restrict__ w, int tokens, int K, int width,
                          const float *extra, const float *residual, float *out, uint32_t *err) {
    const int v4 = width / 4;
    const size_t total = (size_t)tokens * v4;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t t = i / v4, c = i - t * v4;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r = 0; r < K; ++r) {
            const float wr = __ldg(w + t * K + r);
            const float4 v = __ldcs(reinterpret_cast<const float4 *>(y + (t * K + r) * width) + c);
            acc.x = __fadd_rn(acc.x, __fmul_rn(wr, v.x));
            acc.y = __fadd_rn(acc.y, __fmul_rn(wr, v.y));
            acc.z = __fadd_rn(acc.z, __fmul_rn(wr, v.z));
            acc.w = __fadd_rn(acc.w, __fmul_rn(wr, v.w));
        }
        if (extra) {  // the shared experts' output, the (K+1)-th term
            const float4 v = reinterpret_cast<const float4 *>(extra + t * width)[c];
            acc.x = __fadd_rn(acc.x, v.x);
            acc.y = __fadd_rn(acc.y, v.y);
            acc.z = __fadd_rn(acc.z, v.z);
            acc.w = __fadd_rn(acc.w, v.w);
        }
        if (residual) {  // h + moe, the residual stream of the layer stack (may alias out)
            const float4 r = reinterpret_cast<const float4 *>(residual + t * width)[c];
            acc.x = __fadd_rn(r.x, acc.x);
            acc.y = __fadd_rn(r.y, acc.y);
            acc.z = __fadd_rn(r.z, acc.z);
            acc.w = __fadd_rn(r.w, acc.w);
        }
        flag_nonfinite4(acc, err);
        reinterpret_cast<float4 *>(out + t * width)[c] = acc;
    }
}

// ============================================================================
// Layout kernels: ggml blocks <-> tile planes, one thread per (row, block).
// ============================================================================

template <bool TO_TILE>
__global__ void k_layout(Matrix m, int expert, uint8_t *ggml) {
    const int nb = m.cols / 32;
    const size_t total = (size_t)m.rows * nb;
    const bool mx = m.quant == UMSX_QUANT_MXFP4;
    const size_t bb = mx ? 17 : 34;
    const int rpw = mx ? 16 : 32, nrg = m.rows / rpw;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int row = (int)(i / nb), b = (int)(i - (size_t)row * nb);
        const int rg = row / rpw, r = row % rpw;
        uint8_t *blk = ggml + i * bb;
        if (mx) {
            const int np = nb / 2, nq = (np + 3) / 4, bp = b >> 1, h = b & 1, L = h * 16 + r;
            uint8_t *chunk = m.codes + (((size_t)expert * nrg + rg) * np + bp) * 512;
            uint8_t *ex = m.scales + (((size_t)expert * nrg + rg) * nq + (bp >> 2)) * 128 + L * 4 + (bp & 3);
            if (TO_TILE) *ex = blk[0]; else blk[0] = *ex;
            for (int lh = 0; lh < 2; ++lh) {
                uint32_t *words = reinterpret_cast<uint32_t *>(chunk + lh * 256 + L * 8);
                for (int w = 0; w < 2; ++w) {
                    if (TO_TILE) {
                        uint32_t v = 0;
                        for (int pp = 0; pp < 2; ++pp)
                            for (int q = 0; q < 4; ++q) {
                                const uint32_t byte = blk[1 + 4 * (2 * w + pp) + q];
                                v |= (lh ? (byte >> 4) : (byte & 15u)) << (16 * pp + 4 * q);
                            }
                        words[w] = v;
                    } else {
                        const uint32_t v = words[w];
                        for (int pp = 0; pp < 2; ++pp)
                            for (int q = 0; q < 4; ++q) {
                                const uint32_t code = (v >> (16 * pp + 4 * q)) & 15u;
                                uint8_t &byte = blk[1 + 4 * (2 * w + pp) + q];
                                byte = lh ? (uint8_t)((byte & 15u) | (code << 4)) : (uint8_t)((byte & 0xf0u) | code);
                            }
                    }
                }
            }
        } else {
            uint8_t *dst = m.codes + (((size_t)expert * nrg + rg) * nb + b) * 1024 + r * 32;
            uint8_t *sc = m.scales + (((size_t)expert * nrg + rg) * (nb / 2) + (b >> 1)) * 128 + r * 4 + (b & 1) * 2;
            if (TO_TILE) { sc[0] = blk[0]; sc[1] = blk[1]; } else { blk[0] = sc[0]; blk[1] = sc[1]; }
            for (int pp = 0; pp < 4; ++pp) {
                for (int q = 0; q < 4; ++q) {
                    if (TO_TILE) { dst[pp * 8 + q] = blk[2 + 4 * pp + q]; dst[pp * 8 + 4 + q] = blk[2 + 16 + 4 * pp + q]; }
                    else { blk[2 + 4 * pp + q] = dst[pp * 8 + q]; blk[2 + 16 + 4 * pp + q] = dst[pp * 8 + 4 + q]; }
                }
            }
        }
    }
}

// ============================================================================
// Generator kernels (bitwise twins of orc_gen_*).
// ============================================================================

__global__ void k_gen_blocks(int quant, uint64_t seed, uint64_t stream, uint64_t first, uint64_t n, uint8_t *out) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t b = first + i;
        if (quant == UMSX_QUANT_MXFP4) {
            const uint64_t r0 = rng(seed, stream, 3 * b), r1 = rng(seed, stream, 3 * b + 1), r2 = rng(seed, stream, 3 * b + 2);
            uint8_t *blk = out + i * 17;
            blk[0] = (uint8_t)(119 + (uint32_t)(r0 >> 32) % 5u);
            for (int j = 0; j < 8; ++j) { blk[1 + j] = (uint8_t)(r1 >> (8 * j)); blk[9 + j] = (uint8_t)(r2 >> (8 * j)); }
        } else {
            // 34-byte blocks start on even addresses: write 17 aligned 16-bit halves.
            uint16_t *blk = reinterpret_cast<uint16_t *>(out + i * 34);
            const uint64_t r0 = rng(seed, stream, 9 * b);
            const float f = __fadd_rn(__fmul_rn((float)(uint32_t)(r0 >> 40), 0x1.f212d8p-34f), 0x1.a36e2ep-14f);
            blk[0] = (uint16_t)f32_to_f16_bits(f);
            for (int q = 0; q < 8; ++q) {
                const uint64_t r = rng(seed, stream, 9 * b + 1 + q);
                uint32_t codes[4];
                for (int c = 0; c < 4; ++c) {
                    const uint32_t chunk = (uint32_t)(r >> (16 * c)) & 0xffffu;
                    codes[c] = (uint32_t)((int)(chunk % 255u) - 127) & 0xffu;
                }
                blk[1 + 2 * q] = (uint16_t)(codes[0] | (codes[1] << 8));
                blk[2 + 2 * q] = (uint16_t)(codes[2] | (codes[3] << 8));
            }
        }
    }
}

__global__ void k_gen_normal(uint64_t seed, uint64_t stream, uint64_t first, uint64_t n, float scale, float *out,
                             int round_bf16) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        float v = gen_normal(seed, stream, first + i, scale);
        if (round_bf16) v = bf16_bits_to_f32(f32_to_bf16_bits(v));
        out[i] = v;
    }
}

__global__ void k_bf16_to_f32(const uint16_t *in, float *out, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = bf16_bits_to_f32(in[i]);
}

// ============================================================================
// Launchers
// ============================================================================

// Dynamic shared memory plus a kernel's static shared memory (at most this much here) above
// 48 KiB needs the per-kernel opt-in.
constexpr size_t kStaticSmemMargin = 8192;

static inline int grid_for(size_t n, int threads, int cap = 148 * 16) {
    size_t g = (n + threads - 1) / threads;
    if (g < 1) g = 1;
    return (int)(g > (size_t)cap ? cap : g);
}

// Launch with the programmatic-stream-serialization attribute (PDL).
template <class... KArgs, class... Args>
static void launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kern, args...);
}

int launch_router(const RouterParams &p, const Dispatch &d, cudaStream_t s) {
    dim3 grid((p.experts + kRouterWarps - 1) / kRouterWarps, p.tokens);
    RouterParams q = p;
    q.fuse_dispatch = p.tokens * p.top_k <= kFusedDispatchMax;
    const size_t smem = (size_t)p.hidden * sizeof(float);
    if (p.hidden <= 32 * kRouterRegs) launch_pdl(k_router<true>, grid, dim3(kRouterWarps * 32), smem, s, q, d);
    else launch_pdl(k_router<false>, grid, dim3(kRouterWarps * 32), smem, s, q, d);
    int launched = 1;
    if (!q.fuse_dispatch) {
        launch_pdl(k_dispatch, dim3(p.e_local), dim3(256), 0, s, d, p.tokens * p.top_k, p.top_k, p.e_lo, p.e_local);
        ++launched;
    }
    return launched;
}

int launch_dispatch(const Dispatch &d, int entries, int top_k, int e_lo, int e_local, cudaStream_t s) {
    launch_pdl(k_dispatch, dim3(e_local), dim3(256), 0, s, d, entries, top_k, e_lo, e_local);
    return 1;
}

template <int QUANT, int MT>
static void gate_up_mt(const GateUpParams &p, const Dispatch &d, int slots, cudaStream_t s) {
    const int nb = p.hidden / 32;
    const size_t smem = staged_bytes(MT, nb);
    auto kern = k_gate_up<QUANT, MT>;
    if (smem + kStaticSmemMargin > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    launch_pdl(kern, dim3(p.intermediate / 32, slots), dim3(64 * Geo<QUANT>::kChains), smem, s, p, d);
}

// cp.async ring depth of the per-stage MXFP4 kernels: S - 1 stages of 4 block pairs
// (1 KB of codes) in flight per warp.  Measured on GPT-OSS-120B-shaped layers at
// T = 8 / 16 / 64, depths 2, 3, 4, 6, 8 gave 164 / 173 / 167 / 183 / 200 us at T = 8:
// these short CTAs are bound by their serial phases (slot and job reads, activation
// copy, epilogue), not by the bytes in flight, and a small ring leaves shared memory
// to more resident CTAs.
constexpr int kPerStageRing = 2;

template <int MT>
static void gate_up_mx_mt(const GateUpParams &p, const Dispatch &d, int slots, cudaStream_t s) {
    const int nb = p.hidden / 32;
    const size_t smem = bulk_staged_bytes(MT, nb) + (size_t)4 * kPerStageRing * kRingStageBytes;
    auto kern = k_gate_up_mx<MT, kPerStageRing>;
    if (smem + kStaticSmemMargin > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    launch_pdl(kern, dim3(p.intermediate / 16, slots), dim3(128), smem, s, p, d);
}

int launch_gate_up(const GateUpParams &p, const Dispatch &d, int slots, int max_per_expert, cudaStream_t s) {
    const int q = p.fused ? p.gate_up.quant : p.gate.quant;
    if (q == UMSX_QUANT_MXFP4) {
        if (max_per_expert <= 1) gate_up_mx_mt<1>(p, d, slots, s);
        else if (max_per_expert <= 2) gate_up_mx_mt<2>(p, d, slots, s);
        else if (max_per_expert <= 4) gate_up_mx_mt<4>(p, d, slots, s);
        else gate_up_mx_mt<8>(p, d, slots, s);
        return 1;
    }
#define UMSX_GU(QQ)                                                          \
    if (max_per_expert <= 1) gate_up_mt<QQ, 1>(p, d, slots, s);             \
    else if (max_per_expert <= 2) gate_up_mt<QQ, 2>(p, d, slots, s);        \
    else if (max_per_expert <= 4) gate_up_mt<QQ, 4>(p, d, slots, s);        \
    else gate_up_mt<QQ, 8>(p, d, slots, s);
    UMSX_GU(UMSX_QUANT_Q8_0)
#undef UMSX_GU
    return 1;
}

template <int QUANT, int MT, int SRC, int COMBINE>
static void gemv_mt(const GemvParams &p, const GemvSrc &src, const Dispatch &d, int slots, cudaStream_t s) {
    constexpr int W = 4;
    const int nb = p.m.cols / 32;
    const size_t smem = staged_bytes(MT, nb);
    auto kern = k_gemv<QUANT, W, MT, SRC, COMBINE>;
    if (smem + kStaticSmemMargin > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const int tiles = (p.m.rows / Geo<QUANT>::kRowsPerWarp + W - 1) / W;
    launch_pdl(kern, dim3(tiles, slots), dim3(W * 32), smem, s, p, src, d);
}

template <int MT, int SRC, int COMBINE>
static void gemv_mx_mt(const GemvParams &p, const GemvSrc &src, const Dispatch &d, int slots, cudaStream_t s) {
    constexpr int W = 2;
    const int nb = p.m.cols / 32;
    const size_t smem = (SRC == 3 ? bulk_staged_bytes(MT, nb) : staged_bytes(MT, nb)) +
                        (size_t)2 * W * kPerStageRing * kRingStageBytes;
    auto kern = k_gemv_mx<W, MT, SRC, COMBINE, kPerStageRing>;
    if (smem + kStaticSmemMargin > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const int tiles = (p.m.rows / 16 + W - 1) / W;
    launch_pdl(kern, dim3(tiles, slots), dim3(W * 64), smem, s, p, src, d);
}

template <int QUANT, int SRC, int COMBINE>
static void gemv_src(const GemvParams &p, const GemvSrc &src, const Dispatch &d, int slots, int mpe, cudaStream_t s) {
    if constexpr (QUANT == UMSX_QUANT_MXFP4) {
        if (mpe <= 1) gemv_mx_mt<1, SRC, COMBINE>(p, src, d, slots, s);
        else if (mpe <= 2) gemv_mx_mt<2, SRC, COMBINE>(p, src, d, slots, s);
        else if (mpe <= 4) gemv_mx_mt<4, SRC, COMBINE>(p, src, d, slots, s);
        else gemv_mx_mt<8, SRC, COMBINE>(p, src, d, slots, s);
        return;
    }
    if constexpr (SRC == 3) return;  // records exist for MXFP4 only
    if (mpe <= 1) gemv_mt<QUANT, 1, SRC, COMBINE>(p, src, d, slots, s);
    else if (mpe <= 2) gemv_mt<QUANT, 2, SRC, COMBINE>(p, src, d, slots, s);
    else if (mpe <= 4) gemv_mt<QUANT, 4, SRC, COMBINE>(p, src, d, slots, s);
    else gemv_mt<QUANT, 8, SRC, COMBINE>(p, src, d, slots, s);
}

int launch_gemv(const GemvParams &p, const Dispatch &d, int slots, int max_per_expert, cudaStream_t s) {
    GemvSrc src{};
    src.q8_codes = p.a_codes;
    src.q8_scales = p.a_scales;
    src.ggml = p.a_q8;
    src.f32 = p.a_f32;
    const int mode = p.a_q8 ? 1 : (p.a_f32 ? 2 : (p.a_rec ? 3 : 0));
    const bool comb = p.tile_done != nullptr;
#define UMSX_GV(QQ)                                                                          \
    if (mode == 0) { if (comb) gemv_src<QQ, 0, 1>(p, src, d, slots, max_per_expert, s);        \
                     else gemv_src<QQ, 0, 0>(p, src, d, slots, max_per_expert, s); }          \
    else if (mode == 1) gemv_src<QQ, 1, 0>(p, src, d, slots, max_per_expert, s);              \
    else { if (comb) gemv_src<QQ, 2, 1>(p, src, d, slots, max_per_expert, s);                  \
           else gemv_src<QQ, 2, 0>(p, src, d, slots, max_per_expert, s); }
    if (p.m.quant == UMSX_QUANT_MXFP4) {
        if (mode == 3) {  // staging records, only the MXFP4 layer path produces them
            if (comb) gemv_src<UMSX_QUANT_MXFP4, 3, 1>(p, src, d, slots, max_per_expert, s);
            else gemv_src<UMSX_QUANT_MXFP4, 3, 0>(p, src, d, slots, max_per_expert, s);
        } else { UMSX_GV(UMSX_QUANT_MXFP4) }
    } else { UMSX_GV(UMSX_QUANT_Q8_0) }
#undef UMSX_GV
    return 1;
}

int launch_combine(const float *y, const float *w, int tokens, int top_k, int width, const float *extra,
                   const float *residual, float *out, uint32_t *err, cudaStream_t s) {
    const size_t n = (size_t)tokens * (width / 4);
    k_combine<<<grid_for(n, 256), 256, 0, s>>>(y, w, tokens, top_k, width, extra, residual, out, err);
    return 1;
}

int launch_repack(const Matrix &m, int expert, const uint8_t *ggml, cudaStream_t s) {
    const size_t n = (size_t)m.rows * (m.cols / 32);
    k_layout<true><<<grid_for(n, 256), 256, 0, s>>>(m, expert, const_cast<uint8_t *>(ggml));
    return 1;
}

int launch_export(const Matrix &m, int expert, uint8_t *ggml, cudaStream_t s) {
    const size_t n = (size_t)m.rows * (m.cols / 32);
    k_layout<false><<<grid_for(n, 256), 256, 0, s>>>(m, expert, ggml);
    return 1;
}

int launch_gen_blocks(int quant, uint64_t seed, uint64_t stream, uint64_t first_block, uint64_t nblocks, uint8_t *out,
                      cudaStream_t s) {
    k_gen_blocks<<<grid_for(nblocks, 256), 256, 0, s>>>(quant, seed, stream, first_block, nblocks, out);
    return 1;
}

int launch_gen_normal_f32(uint64_t seed, uint64_t stream, uint64_t first, uint64_t n, float scale, float *out,
                          cudaStream_t s) {
    k_gen_normal<<<grid_for(n, 256), 256, 0, s>>>(seed, stream, first, n, scale, out, 0);
    return 1;
}

int launch_gen_normal_bf16_to_f32(uint64_t seed, uint64_t stream, uint64_t first, uint64_t n, float scale, float *out,
                                  cudaStream_t s) {
    k_gen_normal<<<grid_for(n, 256), 256, 0, s>>>(seed, stream, first, n, scale, out, 1);
    return 1;
}

int launch_bf16_to_f32(const uint16_t *in, float *out, size_t n, cudaStream_t s) {
    k_bf16_to_f32<<<grid_for(n, 256), 256, 0, s>>>(in, out, n);
    return 1;
}

// Points the slot records of a banked layer's dispatch at device bank slots: rec.x (an expert index)
// becomes map[rec.x]; records past the last active one (rec.x < 0) stay as they are.
__global__ void k_bank_remap(int4 *slots, const int32_t *map, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    int4 rec = slots[i];
    if (rec.x >= 0) {
        rec.x = map[rec.x];
        slots[i] = rec;
    }
}

int launch_bank_remap(int4 *slots, const int32_t *map, int n, cudaStream_t s) {
    k_bank_remap<<<(n + 127) / 128, 128, 0, s>>>(slots, map, n);
    return 1;
}

}  // namespace umsx
