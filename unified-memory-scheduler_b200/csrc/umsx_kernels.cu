// umsx kernels for sm_100a: router, dispatch, exact quantized expert GEMVs,
// combine, and the weight layout / generator kernels.
//
// Exactness contract (reference paths inside appatalks/unified-memory-scheduler):
// an MXFP4 x Q8_0 row dot splits each 32-weight block into eight int lanes of
// four products (VPSIGNB semantics, tools/engine/quantized_cuda.cu:145-157),
// accumulates lane l of block b as fma(d_b, float(L), acc) in an even-block and
// an odd-block chain, and sums lanes as ((l0+l4)+(l2+l6))+((l1+l5)+(l3+l7))
// (tools/trace/compatible_down.cu:95-99, tools/trace/cpu_mxfp4_vnni.cpp:57-67).
// Here one lane of a warp owns the lane pair (p, p+4) of one row, so the chain
// order is the reference's and the final order is two xor shuffles.
#include <stdint.h>

#include "umsx_device.cuh"
#include "umsx_internal.h"

namespace umsx {

// ============================================================================
// Router: logits + softmax / top-k / weights + x -> Q8_0, and (small T*K) the
// dispatch build, all in one launch.  grid = (ceil(E/8), T), block = 256.
// ============================================================================

constexpr int kRouterWarps = 8;
constexpr int kMaxExperts = 1024;
constexpr int kFusedDispatchMax = 512;

__device__ __forceinline__ bool better(float a, int ia, float b, int ib) { return a > b || (a == b && ia < ib); }

// Warp-wide selection for one token (all 32 lanes participate).
__device__ void select_token(const RouterParams &p, const Dispatch &d, int t, int lane) {
    const int E = p.experts, K = p.top_k;
    float v[kMaxExperts / 32];
    const float *lg = d.logits + (size_t)t * E;
#pragma unroll
    for (int j = 0; j < kMaxExperts / 32; ++j) {
        const int e = lane + 32 * j;
        v[j] = e < E ? __ldcg(lg + e) : 0.0f;
    }
    if (p.routing != UMSX_ROUTE_TOPK_SOFTMAX) {
        float m = -__uint_as_float(0x7f800000u);
#pragma unroll
        for (int j = 0; j < kMaxExperts / 32; ++j)
            if (lane + 32 * j < E) m = fmaxf(m, v[j]);
        m = warp_max(m);
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < kMaxExperts / 32; ++j) {
            if (lane + 32 * j < E) {
                v[j] = exp_shared(__fadd_rn(v[j], -m));
                s = __fadd_rn(s, v[j]);
            }
        }
        const float total = warp_tree_sum(s);
#pragma unroll
        for (int j = 0; j < kMaxExperts / 32; ++j)
            if (lane + 32 * j < E) v[j] = __fdiv_rn(v[j], total);
    }
    uint32_t taken = 0;
    int my_sel = -1;
    float my_val = 0.0f;
    for (int r = 0; r < K; ++r) {
        float bv = -__uint_as_float(0x7f800000u);
        int be = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < kMaxExperts / 32; ++j) {
            const int e = lane + 32 * j;
            if (e < E && !((taken >> j) & 1u) && better(v[j], e, bv, be)) { bv = v[j]; be = e; }
        }
#pragma unroll
        for (int s = 16; s >= 1; s >>= 1) {
            const float ov = __shfl_xor_sync(kFull, bv, s);
            const int oe = __shfl_xor_sync(kFull, be, s);
            if (better(ov, oe, bv, be)) { bv = ov; be = oe; }
        }
        if ((be & 31) == lane) taken |= 1u << (be >> 5);
        if (lane == r) { my_sel = be; my_val = bv; }
    }
    // weights: lane r < K holds rank r
    float w = 0.0f;
    if (p.routing == UMSX_ROUTE_TOPK_SOFTMAX) {
        const float m = __shfl_sync(kFull, my_val, 0);
        const float ex = lane < K ? exp_shared(__fadd_rn(my_val, -m)) : 0.0f;
        float sum = 0.0f;
        for (int r = 0; r < K; ++r) sum = __fadd_rn(sum, __shfl_sync(kFull, ex, r));
        w = __fdiv_rn(ex, sum);
    } else if (p.routing == UMSX_ROUTE_SOFTMAX_TOPK_NORM) {
        float sum = 0.0f;
        for (int r = 0; r < K; ++r) sum = __fadd_rn(sum, __shfl_sync(kFull, my_val, r));
        w = __fdiv_rn(my_val, sum);
    } else {
        w = __fmul_rn(my_val, p.routed_scale);
    }
    if (lane < K) {
        d.ids[(size_t)t * K + lane] = my_sel;
        d.weights[(size_t)t * K + lane] = w;
    }
}

// One CTA builds counts / offsets / active list / job lists for N = T*K entries.
__device__ void build_dispatch_cta(const Dispatch &d, int entries, int K, int e_lo, int e_local) {
    __shared__ int cnt[kMaxExperts];
    __shared__ int off[kMaxExperts];
    __shared__ int ids_s[kFusedDispatchMax];
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
            if (cnt[e] > 0) d.active[abase++] = e;
            base += cnt[e];
        }
        if (tid == 31) { d.offsets[e_local] = ps; d.n_active[0] = pa; }
    }
    __syncthreads();
    for (int j = tid; j < entries; j += nth) {
        const int e = ids_s[j];
        if (e < 0 || e >= e_local) continue;
        int before = 0;
        for (int i = 0; i < j; ++i) before += ids_s[i] == e;
        const int pos = off[e] + before;
        d.job_token[pos] = j / K;
        d.job_rank[pos] = j % K;
    }
}

__global__ void __launch_bounds__(256) k_router(RouterParams p, Dispatch d) {
    extern __shared__ float xs[];
    const int t = blockIdx.y, H = p.hidden;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (p.x_dtype == UMSX_DTYPE_BF16) {
        const uint16_t *xb = static_cast<const uint16_t *>(p.x) + (size_t)t * H;
        for (int i = threadIdx.x; i < H; i += blockDim.x) xs[i] = bf16_bits_to_f32(xb[i]);
    } else {
        const float *xf = static_cast<const float *>(p.x) + (size_t)t * H;
        for (int i = threadIdx.x; i < H; i += blockDim.x) xs[i] = xf[i];
    }
    __syncthreads();
    if (p.rmsnorm) {
        // RMSNorm with unit weight: sum of squares in the shared strided order (orc_rmsnorm)
        __shared__ float inv_s;
        if (warp == 0) {
            float acc = 0.0f;
            for (int k = lane; k < H; k += 32) acc = __fmaf_rn(xs[k], xs[k], acc);
            const float ss = warp_tree_sum(acc);
            if (lane == 0) inv_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)H), p.eps)));
        }
        __syncthreads();
        const float inv = inv_s;
        for (int i = threadIdx.x; i < H; i += blockDim.x) xs[i] = __fmul_rn(xs[i], inv);
        __syncthreads();
    }
    // x -> Q8_0 (one warp per 32-element block), spread over this token's CTAs.
    const int nbH = H / 32;
    for (int b = blockIdx.x * kRouterWarps + warp; b < nbH; b += gridDim.x * kRouterWarps) {
        const float v = xs[b * 32 + lane];
        const float amax = warp_max(fabsf(v));
        const float inv = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
        d.xq_codes[((size_t)t * nbH + b) * 32 + lane_pair_offset(lane)] = (uint8_t)(int8_t)q8_code(v, inv);
        if (lane == 0) d.xq_scales[(size_t)t * nbH + b] = f16_bits_to_f32(f32_to_f16_bits(__fdiv_rn(amax, 127.0f)));
    }
    // logits: 32 strided FMA chains, then the xor tree (orc_logit)
    const int e = blockIdx.x * kRouterWarps + warp;
    if (e < p.experts) {
        const float *wr = p.w + (size_t)e * H;
        float acc = 0.0f;
        for (int k = lane; k < H; k += 32) acc = __fmaf_rn(__ldg(wr + k), xs[k], acc);
        float l = warp_tree_sum(acc);
        if (p.b) l = __fadd_rn(l, __ldg(p.b + e));
        if (lane == 0) d.logits[(size_t)t * p.experts + e] = l;
    }
    // the last CTA of this token selects; the last token to finish builds the dispatch
    __shared__ int last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(d.token_done + t, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (warp == 0) select_token(p, d, t, lane);
    if (threadIdx.x == 0) d.token_done[t] = 0;
    if (!p.fuse_dispatch) return;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(d.all_done, 1u) == gridDim.y - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    build_dispatch_cta(d, p.tokens * p.top_k, p.top_k, p.e_lo, p.e_local);
    if (threadIdx.x == 0) d.all_done[0] = 0;
}

// Large T*K: one CTA per local expert.  Each CTA histograms every entry, scans,
// and compacts its own entries in order (ballot per warp, prefix across warps).
__global__ void __launch_bounds__(256) k_dispatch(Dispatch d, int entries, int K, int e_lo, int e_local) {
    __shared__ int cnt[kMaxExperts];
    __shared__ int warp_tot[8];
    __shared__ int base_s, off_s;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int me = blockIdx.x;
    for (int e = tid; e < e_local; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int j = tid; j < entries; j += blockDim.x) {
        const int e = __ldg(d.ids + j) - e_lo;
        if (e >= 0 && e < e_local) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    if (tid == 0) {
        int s = 0, a = 0;
        for (int e = 0; e < me; ++e) { s += cnt[e]; a += cnt[e] > 0; }
        off_s = s;
        d.offsets[me] = s;
        d.counts[me] = cnt[me];
        if (cnt[me] > 0) d.active[a] = me;
        if (me == e_local - 1) {
            d.offsets[e_local] = s + cnt[me];
            d.n_active[0] = a + (cnt[me] > 0);
        }
        base_s = 0;
    }
    __syncthreads();
    for (int j0 = 0; j0 < entries; j0 += blockDim.x) {
        const int j = j0 + tid;
        const bool mine = j < entries && __ldg(d.ids + j) - e_lo == me;
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
// Exact quantized GEMV cores.  One warp = one row group (8 rows x 4 lanes).
// Activations for up to MT jobs sit in shared memory as 32-byte lane-pair
// blocks (lane p reads 8 bytes: elements 4p..4p+3 and 16+4p..16+4p+3) plus one
// fp32 scale per block (the fp16 value, exactly widened).
// ============================================================================

template <int MT>
__device__ __forceinline__ void mx_block(uint32_t word, uint32_t e8, int b, int parity, const uint8_t *act_s,
                                         const float *sc_s, int nb, int m, int p, float (&acc)[MT][4]) {
    const uint32_t nword = word ^ 0x88888888u;
    const uint32_t posL = prmt(kMagLo, kMagHi, word), negL = prmt(kMagLo, kMagHi, nword);
    const uint32_t posH = prmt(kMagLo, kMagHi, word >> 16), negH = prmt(kMagLo, kMagHi, nword >> 16);
    const float eh = e8m0_half(e8);
#pragma unroll
    for (int t = 0; t < MT; ++t) {
        if (t < m) {
            const uint2 av = *reinterpret_cast<const uint2 *>(act_s + ((size_t)t * nb + b) * 32 + p * 8);
            const float d = __fmul_rn(sc_s[t * nb + b], eh);
            const int lo = dp4a_ss(negL, neg8x4(av.x), dp4a_ss(posL, av.x, 0));
            const int hi = dp4a_ss(negH, neg8x4(av.y), dp4a_ss(posH, av.y, 0));
            acc[t][parity * 2 + 0] = __fmaf_rn(d, (float)lo, acc[t][parity * 2 + 0]);
            acc[t][parity * 2 + 1] = __fmaf_rn(d, (float)hi, acc[t][parity * 2 + 1]);
        }
    }
}

template <int MT>
__device__ __forceinline__ void q8_block(uint2 wq, uint32_t wsc, int b, const uint8_t *act_s, const float *sc_s,
                                         int nb, int m, int p, float (&acc)[MT][4]) {
    const uint32_t mL = __vcmplts4(wq.x, 0u), mH = __vcmplts4(wq.y, 0u);
    const uint32_t posL = wq.x & ~mL, negL = neg8x4(wq.x) & mL;
    const uint32_t posH = wq.y & ~mH, negH = neg8x4(wq.y) & mH;
    const float wd = f16_bits_to_f32(wsc);
#pragma unroll
    for (int t = 0; t < MT; ++t) {
        if (t < m) {
            const uint2 av = *reinterpret_cast<const uint2 *>(act_s + ((size_t)t * nb + b) * 32 + p * 8);
            const float d = __fmul_rn(wd, sc_s[t * nb + b]);
            const int lo = dp4a_us(negL, neg8x4(av.x), dp4a_us(posL, av.x, 0));
            const int hi = dp4a_us(negH, neg8x4(av.y), dp4a_us(posH, av.y, 0));
            acc[t][0] = __fmaf_rn(d, (float)lo, acc[t][0]);
            acc[t][1] = __fmaf_rn(d, (float)hi, acc[t][1]);
        }
    }
}

// Dot products of one row group against the staged activations.
template <int QUANT, int MT>
__device__ __forceinline__ void rowgroup_dot(const uint8_t *__restrict__ codes, const uint8_t *__restrict__ scales,
                                             int nb, const uint8_t *act_s, const float *sc_s, int m, int lane,
                                             float (&acc)[MT][4]) {
    const int w = lane >> 2, p = lane & 3;
#pragma unroll
    for (int t = 0; t < MT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.0f;
    if constexpr (QUANT == UMSX_QUANT_MXFP4) {
        const int ng = nb >> 2;
        int g = 0;
        for (; g + 2 <= ng; g += 2) {
            const uint4 w0 = __ldg(reinterpret_cast<const uint4 *>(codes + (size_t)g * 512) + lane);
            const uint4 w1 = __ldg(reinterpret_cast<const uint4 *>(codes + (size_t)(g + 1) * 512) + lane);
            const uint32_t e0 = __ldg(reinterpret_cast<const uint32_t *>(scales + (size_t)g * 32) + w);
            const uint32_t e1 = __ldg(reinterpret_cast<const uint32_t *>(scales + (size_t)(g + 1) * 32) + w);
            mx_block<MT>(w0.x, e0 & 0xffu, 4 * g + 0, 0, act_s, sc_s, nb, m, p, acc);
            mx_block<MT>(w0.y, (e0 >> 8) & 0xffu, 4 * g + 1, 1, act_s, sc_s, nb, m, p, acc);
            mx_block<MT>(w0.z, (e0 >> 16) & 0xffu, 4 * g + 2, 0, act_s, sc_s, nb, m, p, acc);
            mx_block<MT>(w0.w, e0 >> 24, 4 * g + 3, 1, act_s, sc_s, nb, m, p, acc);
            mx_block<MT>(w1.x, e1 & 0xffu, 4 * g + 4, 0, act_s, sc_s, nb, m, p, acc);
            mx_block<MT>(w1.y, (e1 >> 8) & 0xffu, 4 * g + 5, 1, act_s, sc_s, nb, m, p, acc);
            mx_block<MT>(w1.z, (e1 >> 16) & 0xffu, 4 * g + 6, 0, act_s, sc_s, nb, m, p, acc);
            mx_block<MT>(w1.w, e1 >> 24, 4 * g + 7, 1, act_s, sc_s, nb, m, p, acc);
        }
        if (g < ng) {
            const uint4 w0 = __ldg(reinterpret_cast<const uint4 *>(codes + (size_t)g * 512) + lane);
            const uint32_t e0 = __ldg(reinterpret_cast<const uint32_t *>(scales + (size_t)g * 32) + w);
            mx_block<MT>(w0.x, e0 & 0xffu, 4 * g + 0, 0, act_s, sc_s, nb, m, p, acc);
            mx_block<MT>(w0.y, (e0 >> 8) & 0xffu, 4 * g + 1, 1, act_s, sc_s, nb, m, p, acc);
            mx_block<MT>(w0.z, (e0 >> 16) & 0xffu, 4 * g + 2, 0, act_s, sc_s, nb, m, p, acc);
            mx_block<MT>(w0.w, e0 >> 24, 4 * g + 3, 1, act_s, sc_s, nb, m, p, acc);
            ++g;
        }
        if (nb & 2) {  // tail group of two blocks: 8 bytes per lane, 2 exponent bytes per row
            const uint2 w0 = __ldg(reinterpret_cast<const uint2 *>(codes + (size_t)ng * 512) + lane);
            const uint32_t e0 = __ldg(reinterpret_cast<const uint16_t *>(scales + (size_t)ng * 32) + w);
            mx_block<MT>(w0.x, e0 & 0xffu, 4 * ng + 0, 0, act_s, sc_s, nb, m, p, acc);
            mx_block<MT>(w0.y, e0 >> 8, 4 * ng + 1, 1, act_s, sc_s, nb, m, p, acc);
        }
    } else {
        const int ng = nb >> 1;
        int g = 0;
        for (; g + 2 <= ng; g += 2) {
            const uint4 w0 = __ldg(reinterpret_cast<const uint4 *>(codes + (size_t)g * 512) + lane);
            const uint4 w1 = __ldg(reinterpret_cast<const uint4 *>(codes + (size_t)(g + 1) * 512) + lane);
            const uint32_t s0 = __ldg(reinterpret_cast<const uint32_t *>(scales + (size_t)g * 32) + w);
            const uint32_t s1 = __ldg(reinterpret_cast<const uint32_t *>(scales + (size_t)(g + 1) * 32) + w);
            q8_block<MT>(make_uint2(w0.x, w0.y), s0 & 0xffffu, 2 * g + 0, act_s, sc_s, nb, m, p, acc);
            q8_block<MT>(make_uint2(w0.z, w0.w), s0 >> 16, 2 * g + 1, act_s, sc_s, nb, m, p, acc);
            q8_block<MT>(make_uint2(w1.x, w1.y), s1 & 0xffffu, 2 * g + 2, act_s, sc_s, nb, m, p, acc);
            q8_block<MT>(make_uint2(w1.z, w1.w), s1 >> 16, 2 * g + 3, act_s, sc_s, nb, m, p, acc);
        }
        if (g < ng) {
            const uint4 w0 = __ldg(reinterpret_cast<const uint4 *>(codes + (size_t)g * 512) + lane);
            const uint32_t s0 = __ldg(reinterpret_cast<const uint32_t *>(scales + (size_t)g * 32) + w);
            q8_block<MT>(make_uint2(w0.x, w0.y), s0 & 0xffffu, 2 * g + 0, act_s, sc_s, nb, m, p, acc);
            q8_block<MT>(make_uint2(w0.z, w0.w), s0 >> 16, 2 * g + 1, act_s, sc_s, nb, m, p, acc);
        }
    }
}

// Final lane order of the reference: per lane pair t = l(p+4) + l(p); then
// (t0+t2) and (t1+t3) by xor 2; then their sum by xor 1.  All four lanes of a
// row end with the same bits.
template <int QUANT>
__device__ __forceinline__ float finish_row(const float (&a)[4]) {
    float lp, lp4;
    if constexpr (QUANT == UMSX_QUANT_MXFP4) {
        lp = __fadd_rn(a[0], a[2]);   // even + odd, lane p
        lp4 = __fadd_rn(a[1], a[3]);  // even + odd, lane p+4
    } else {
        lp = a[0];
        lp4 = a[1];
    }
    float t = __fadd_rn(lp4, lp);
    t = __fadd_rn(t, __shfl_xor_sync(kFull, t, 2));
    return __fadd_rn(t, __shfl_xor_sync(kFull, t, 1));
}

__device__ __forceinline__ size_t plane_code_stride(int quant, int nb) { return (size_t)nb * (quant == UMSX_QUANT_MXFP4 ? 128 : 256); }
__device__ __forceinline__ size_t plane_scale_stride(int quant, int nb) { return (size_t)nb * (quant == UMSX_QUANT_MXFP4 ? 8 : 16); }

// Copy the internal-layout Q8 rows of the given jobs into shared memory.
__device__ __forceinline__ void stage_q8_internal(const uint8_t *codes, const float *scales, const int *rows_s, int m,
                                                  int nb, uint8_t *act_s, float *sc_s) {
    const int per = nb * 2;  // uint4 per row
    for (int i = threadIdx.x; i < m * per; i += blockDim.x) {
        const int t = i / per, c = i - t * per;
        reinterpret_cast<uint4 *>(act_s)[(size_t)t * per + c] =
            __ldcg(reinterpret_cast<const uint4 *>(codes + (size_t)rows_s[t] * nb * 32) + c);
    }
    for (int i = threadIdx.x; i < m * nb; i += blockDim.x) {
        const int t = i / nb, b = i - t * nb;
        sc_s[i] = __ldcg(scales + (size_t)rows_s[t] * nb + b);
    }
}

// ============================================================================
// gate_up (+bias, +activation, +Q8_0 of the activation): a CTA computes 32
// intermediate values (4 gate row groups + 4 up row groups = 8 warps) for every
// job of one expert, then quantizes that 32-value block.  grid = (I/32, slots).
// ============================================================================

template <int QUANT, int MT>
__global__ void __launch_bounds__(256) k_gate_up(GateUpParams p, Dispatch d) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int slot = blockIdx.y;
    if (slot >= __ldg(d.n_active)) return;
    const int e = __ldg(d.active + slot);
    const int seg = __ldg(d.offsets + e), cnt = __ldg(d.counts + e);
    const int H = p.hidden, I = p.intermediate, nb = H / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t *act_s = smem;
    float *sc_s = reinterpret_cast<float *>(smem + (size_t)MT * nb * 32);
    float *res = sc_s + MT * nb;              // [MT][2][32]
    int *rows_s = reinterpret_cast<int *>(res + MT * 64);
    const int half = warp >> 2, rgi = warp & 3;
    const int rg_half = blockIdx.x * 4 + rgi;  // row group within gate (or up) rows
    const Matrix &mat = p.fused ? p.gate_up : (half ? p.up : p.gate);
    const int rg = p.fused ? (half * (I / 8) + rg_half) : rg_half;
    const int nrg = mat.rows / 8;
    const uint8_t *codes = mat.codes + ((size_t)e * nrg + rg) * plane_code_stride(QUANT, nb);
    const uint8_t *scales = mat.scales + ((size_t)e * nrg + rg) * plane_scale_stride(QUANT, nb);
    const int row = rg_half * 8 + (lane >> 2);  // intermediate index of this lane's row
    float bias = 0.0f;
    if (p.bias) bias = __ldg(p.bias + (size_t)e * 2 * I + half * I + row);
    const int nbI = I / 32;
    for (int c0 = 0; c0 < cnt; c0 += MT) {
        const int m = min(MT, cnt - c0);
        __syncthreads();
        if (threadIdx.x < m) rows_s[threadIdx.x] = __ldg(d.job_token + seg + c0 + threadIdx.x);
        __syncthreads();
        stage_q8_internal(d.xq_codes, d.xq_scales, rows_s, m, nb, act_s, sc_s);
        __syncthreads();
        float acc[MT][4];
        rowgroup_dot<QUANT, MT>(codes, scales, nb, act_s, sc_s, m, lane, acc);
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            if (t < m) {
                const float v = __fadd_rn(finish_row<QUANT>(acc[t]), bias);
                if ((lane & 3) == 0) res[(t * 2 + half) * 32 + rgi * 8 + (lane >> 2)] = v;
            }
        }
        __syncthreads();
        // activation + Q8_0: warp t quantizes the 32 values of job t
        for (int t = warp; t < m; t += 8) {
            const float g = res[(t * 2 + 0) * 32 + lane], u = res[(t * 2 + 1) * 32 + lane];
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
// One CTA = W row groups of one expert; grid = (N / (8W), slots).
// Activation sources: 0 = internal Q8 (codes + fp32 scales), 1 = ggml block_q8_0
// rows, 2 = fp32 rows quantized here with the x86 Q8_0 rule.
// ============================================================================

struct GemvSrc {
    const uint8_t *q8_codes;
    const float *q8_scales;
    const uint8_t *ggml;
    const float *f32;
};

template <int QUANT, int W, int MT, int SRC>
__global__ void __launch_bounds__(W * 32) k_gemv(GemvParams p, GemvSrc src, Dispatch d) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int slot = blockIdx.y;
    if (slot >= __ldg(d.n_active)) return;
    const int e = __ldg(d.active + slot);
    const int seg = __ldg(d.offsets + e), cnt = __ldg(d.counts + e);
    const int N = p.m.rows, nb = p.m.cols / 32, nrg = N / 8;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t *act_s = smem;
    float *sc_s = reinterpret_cast<float *>(smem + (size_t)MT * nb * 32);
    int *rows_s = reinterpret_cast<int *>(sc_s + MT * nb);
    int *outs_s = rows_s + MT;
    const int rg = blockIdx.x * W + warp;
    const bool active_warp = rg < nrg;
    const uint8_t *codes = p.m.codes + ((size_t)e * nrg + (active_warp ? rg : 0)) * plane_code_stride(QUANT, nb);
    const uint8_t *scales = p.m.scales + ((size_t)e * nrg + (active_warp ? rg : 0)) * plane_scale_stride(QUANT, nb);
    const int n = rg * 8 + (lane >> 2);
    const float bias = (p.bias && active_warp) ? __ldg(p.bias + (size_t)e * N + n) : 0.0f;
    for (int c0 = 0; c0 < cnt; c0 += MT) {
        const int m = min(MT, cnt - c0);
        __syncthreads();
        if (threadIdx.x < m) {
            const int j = seg + c0 + threadIdx.x;
            const int tok = __ldg(d.job_token + j), rank = __ldg(d.job_rank + j);
            rows_s[threadIdx.x] = p.a_by_job ? j : tok * p.a_ts + rank * p.a_rs;
            outs_s[threadIdx.x] = tok * p.o_ts + rank;
        }
        __syncthreads();
        if constexpr (SRC == 0) {
            stage_q8_internal(src.q8_codes, src.q8_scales, rows_s, m, nb, act_s, sc_s);
        } else if constexpr (SRC == 1) {
            for (int i = threadIdx.x; i < m * nb * 32; i += blockDim.x) {
                const int t = i / (nb * 32), r = i - t * nb * 32, b = r >> 5, k = r & 31;
                act_s[((size_t)t * nb + b) * 32 + lane_pair_offset(k)] = src.ggml[((size_t)rows_s[t] * nb + b) * 34 + 2 + k];
            }
            for (int i = threadIdx.x; i < m * nb; i += blockDim.x) {
                const int t = i / nb, b = i - t * nb;
                const uint8_t *blk = src.ggml + ((size_t)rows_s[t] * nb + b) * 34;
                sc_s[i] = f16_bits_to_f32((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
            }
        } else {
            for (int i = warp; i < m * nb; i += W) {
                const int t = i / nb, b = i - t * nb;
                const float v = __ldg(src.f32 + (size_t)rows_s[t] * p.m.cols + b * 32 + lane);
                const float amax = warp_max(fabsf(v));
                const float inv = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
                act_s[((size_t)t * nb + b) * 32 + lane_pair_offset(lane)] = (uint8_t)(int8_t)q8_code(v, inv);
                if (lane == 0) sc_s[i] = f16_bits_to_f32(f32_to_f16_bits(__fdiv_rn(amax, 127.0f)));
            }
        }
        __syncthreads();
        if (active_warp) {
            float acc[MT][4];
            rowgroup_dot<QUANT, MT>(codes, scales, nb, act_s, sc_s, m, lane, acc);
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                if (t < m) {
                    float v = finish_row<QUANT>(acc[t]);
                    if (p.bias) v = __fadd_rn(v, bias);
                    if ((lane & 3) == 0) p.out[(size_t)outs_s[t] * N + n] = v;
                }
            }
        }
    }
}

// ============================================================================
// Combine: out[t][i] = ((0 + w0*y0) + w1*y1) + ... (expert_dispatch.cpp:77-87).
// ============================================================================

__global__ void k_combine(const float *__restrict__ y, const float *__restrict__ w, int tokens, int K, int width,
                          const float *residual, float *out) {
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
        if (residual) {  // h + moe, the residual stream of the layer stack (may alias out)
            const float4 r = reinterpret_cast<const float4 *>(residual + t * width)[c];
            acc.x = __fadd_rn(r.x, acc.x);
            acc.y = __fadd_rn(r.y, acc.y);
            acc.z = __fadd_rn(r.z, acc.z);
            acc.w = __fadd_rn(r.w, acc.w);
        }
        reinterpret_cast<float4 *>(out + t * width)[c] = acc;
    }
}

// ============================================================================
// Layout kernels: ggml blocks <-> tile planes, one thread per (row, block).
// ============================================================================

template <bool TO_TILE>
__global__ void k_layout(Matrix m, int expert, uint8_t *ggml) {
    const int nb = m.cols / 32, nrg = m.rows / 8;
    const size_t total = (size_t)m.rows * nb;
    const bool mx = m.quant == UMSX_QUANT_MXFP4;
    const size_t bb = mx ? 17 : 34;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int row = (int)(i / nb), b = (int)(i - (size_t)row * nb);
        const int rg = row >> 3, w = row & 7;
        uint8_t *blk = ggml + i * bb;
        uint8_t *cbase = m.codes + ((size_t)expert * nrg + rg) * (size_t)nb * (mx ? 128 : 256);
        uint8_t *sbase = m.scales + ((size_t)expert * nrg + rg) * (size_t)nb * (mx ? 8 : 16);
        if (mx) {
            const int g = b >> 2, j = b & 3, nblk = (g < (nb >> 2)) ? 4 : 2;
            uint8_t *chunk = cbase + (size_t)g * 512;
            uint8_t *sc = sbase + (size_t)g * 32 + w * nblk + j;
            if (TO_TILE) *sc = blk[0]; else blk[0] = *sc;
            for (int pp = 0; pp < 4; ++pp) {
                uint32_t *word = reinterpret_cast<uint32_t *>(chunk + ((w * 4 + pp) * nblk + j) * 4);
                if (TO_TILE) {
                    uint32_t v = 0;
                    for (int q = 0; q < 4; ++q) {
                        const uint32_t byte = blk[1 + 4 * pp + q];
                        v |= (byte & 15u) << (4 * q);
                        v |= (byte >> 4) << (16 + 4 * q);
                    }
                    *word = v;
                } else {
                    const uint32_t v = *word;
                    for (int q = 0; q < 4; ++q)
                        blk[1 + 4 * pp + q] = (uint8_t)(((v >> (4 * q)) & 15u) | (((v >> (16 + 4 * q)) & 15u) << 4));
                }
            }
        } else {
            const int g = b >> 1, j = b & 1;
            uint8_t *chunk = cbase + (size_t)g * 512;
            uint8_t *sc = sbase + (size_t)g * 32 + (w * 2 + j) * 2;
            if (TO_TILE) { sc[0] = blk[0]; sc[1] = blk[1]; } else { blk[0] = sc[0]; blk[1] = sc[1]; }
            for (int pp = 0; pp < 4; ++pp) {
                uint8_t *dst = chunk + ((w * 4 + pp) * 2 + j) * 8;
                for (int q = 0; q < 4; ++q) {
                    if (TO_TILE) { dst[q] = blk[2 + 4 * pp + q]; dst[4 + q] = blk[2 + 16 + 4 * pp + q]; }
                    else { blk[2 + 4 * pp + q] = dst[q]; blk[2 + 16 + 4 * pp + q] = dst[4 + q]; }
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

static inline int grid_for(size_t n, int threads, int cap = 148 * 16) {
    size_t g = (n + threads - 1) / threads;
    if (g < 1) g = 1;
    return (int)(g > (size_t)cap ? cap : g);
}

int launch_router(const RouterParams &p, const Dispatch &d, cudaStream_t s) {
    dim3 grid((p.experts + kRouterWarps - 1) / kRouterWarps, p.tokens);
    RouterParams q = p;
    q.fuse_dispatch = p.tokens * p.top_k <= kFusedDispatchMax;
    k_router<<<grid, 256, (size_t)p.hidden * sizeof(float), s>>>(q, d);
    int launched = 1;
    if (!q.fuse_dispatch) {
        k_dispatch<<<p.e_local, 256, 0, s>>>(d, p.tokens * p.top_k, p.top_k, p.e_lo, p.e_local);
        ++launched;
    }
    return launched;
}

int launch_dispatch(const Dispatch &d, int entries, int top_k, int e_lo, int e_local, cudaStream_t s) {
    k_dispatch<<<e_local, 256, 0, s>>>(d, entries, top_k, e_lo, e_local);
    return 1;
}

template <int QUANT, int MT>
static void gate_up_mt(const GateUpParams &p, const Dispatch &d, int slots, cudaStream_t s) {
    const int nb = p.hidden / 32;
    const size_t smem = (size_t)MT * nb * 36 + MT * 64 * sizeof(float) + 64;
    auto kern = k_gate_up<QUANT, MT>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kern<<<dim3(p.intermediate / 32, slots), 256, smem, s>>>(p, d);
}

int launch_gate_up(const GateUpParams &p, const Dispatch &d, int slots, int max_per_expert, cudaStream_t s) {
    const int q = p.fused ? p.gate_up.quant : p.gate.quant;
#define UMSX_GU(QQ)                                                          \
    if (max_per_expert <= 1) gate_up_mt<QQ, 1>(p, d, slots, s);             \
    else if (max_per_expert <= 2) gate_up_mt<QQ, 2>(p, d, slots, s);        \
    else if (max_per_expert <= 4) gate_up_mt<QQ, 4>(p, d, slots, s);        \
    else gate_up_mt<QQ, 8>(p, d, slots, s);
    if (q == UMSX_QUANT_MXFP4) { UMSX_GU(UMSX_QUANT_MXFP4) } else { UMSX_GU(UMSX_QUANT_Q8_0) }
#undef UMSX_GU
    return 1;
}

template <int QUANT, int MT, int SRC>
static void gemv_mt(const GemvParams &p, const GemvSrc &src, const Dispatch &d, int slots, cudaStream_t s) {
    constexpr int W = 4;
    const int nb = p.m.cols / 32;
    const size_t smem = (size_t)MT * nb * 36 + 2 * MT * sizeof(int) + 16;
    auto kern = k_gemv<QUANT, W, MT, SRC>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const int tiles = (p.m.rows / 8 + W - 1) / W;
    kern<<<dim3(tiles, slots), W * 32, smem, s>>>(p, src, d);
}

template <int QUANT, int SRC>
static void gemv_src(const GemvParams &p, const GemvSrc &src, const Dispatch &d, int slots, int mpe, cudaStream_t s) {
    if (mpe <= 1) gemv_mt<QUANT, 1, SRC>(p, src, d, slots, s);
    else if (mpe <= 2) gemv_mt<QUANT, 2, SRC>(p, src, d, slots, s);
    else if (mpe <= 4) gemv_mt<QUANT, 4, SRC>(p, src, d, slots, s);
    else gemv_mt<QUANT, 8, SRC>(p, src, d, slots, s);
}

int launch_gemv(const GemvParams &p, const Dispatch &d, int slots, int max_per_expert, cudaStream_t s) {
    GemvSrc src{};
    src.ggml = p.a_q8;
    src.f32 = p.a_f32;
    const bool ggml = p.a_q8 != nullptr;
    if (p.m.quant == UMSX_QUANT_MXFP4) {
        if (ggml) gemv_src<UMSX_QUANT_MXFP4, 1>(p, src, d, slots, max_per_expert, s);
        else gemv_src<UMSX_QUANT_MXFP4, 2>(p, src, d, slots, max_per_expert, s);
    } else {
        if (ggml) gemv_src<UMSX_QUANT_Q8_0, 1>(p, src, d, slots, max_per_expert, s);
        else gemv_src<UMSX_QUANT_Q8_0, 2>(p, src, d, slots, max_per_expert, s);
    }
    return 1;
}

int launch_gemv_internal(const GemvParams &p, const uint8_t *codes, const float *scales, const Dispatch &d,
                         int slots, int max_per_expert, cudaStream_t s) {
    GemvSrc src{};
    src.q8_codes = codes;
    src.q8_scales = scales;
    if (p.m.quant == UMSX_QUANT_MXFP4) gemv_src<UMSX_QUANT_MXFP4, 0>(p, src, d, slots, max_per_expert, s);
    else gemv_src<UMSX_QUANT_Q8_0, 0>(p, src, d, slots, max_per_expert, s);
    return 1;
}

int launch_combine(const float *y, const float *w, int tokens, int top_k, int width, const float *residual, float *out,
                   cudaStream_t s) {
    const size_t n = (size_t)tokens * (width / 4);
    k_combine<<<grid_for(n, 256), 256, 0, s>>>(y, w, tokens, top_k, width, residual, out);
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

}  // namespace umsx
