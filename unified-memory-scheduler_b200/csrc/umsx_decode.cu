// Persistent decode kernel: a whole stack of MoE layers (or one layer) for a few
// tokens in ONE cooperative launch with one CTA per SM.
//
// Per layer, between grid-wide barriers:
//   R  every CTA folds the previous layer's expert outputs into its own copy of
//      the residual stream h (rank order, tools/engine/expert_dispatch.cpp:77-87),
//      normalises it (RMSNorm, unit weight) and quantizes it to Q8_0 records;
//      CTA c computes the router logits of experts c, c + #CTAs, ...
//   S  every CTA selects the top-k experts of every token from the logits itself
//      (identical inputs and code, so identical choices) and builds the slot list
//      (distinct experts, ascending) and the per-slot job lists.
//   G  gate_up units = (slot, 16 rows of gate + the matching 16 rows of up), a
//      contiguous share per CTA, five units at a time (4 warps each): exact
//      MXFP4 x Q8_0 row dots, bias, SwiGLU-OAI / SiLU -> fp32 activations.
//   D  every CTA quantizes the activation rows its down units read into Q8_0
//      records in shared memory; down units = (slot, 16 rows of down), ten at a
//      time (2 warps each), over those records -> per-job outputs y.
// Every warp streams its weight rows through its own cp.async ring in shared
// memory, several stages ahead, so that enough bytes are in flight per SM.
// The arithmetic of every value is the per-stage path's (umsx_kernels.cu), so
// both paths produce the same bits; this one only removes the kernel boundaries,
// the single-CTA selection and the second wave of CTAs.
//
// Grid barriers are a monotonic counter with bounded spins: a CTA that waits
// longer than kGridWaitCycles (or sees another CTA's error bit) sets `err` and
// returns, so a fault elsewhere cannot keep the kernel alive.  Tests shorten the
// bound and withhold one CTA's first arrival (DecodeParams::fault_cta) to see the
// waits run out.  One token (MT = 1) takes its slot list straight from the ranking
// (k distinct experts: slot r = rank r with the one job r).  The final output is
// checked for inf / NaN (kErrNonFinite).
#include <stdint.h>

#include "umsx_device.cuh"
#include "umsx_internal.h"
#include "umsx_mx.cuh"

namespace umsx {

namespace {

constexpr int kDecThreads = 640;                 // 20 warps
constexpr int kGuGroups = kDecThreads / 128;     // concurrent gate_up units (4 warps each)
constexpr int kDnGroups = kDecThreads / 64;      // concurrent down units (2 warps each)
constexpr int kDecWarps = kDecThreads / 32;
constexpr long long kGridWaitCycles = 40000000;  // ~20 ms at 2 GHz
constexpr int kMaxEntries = kDecodeMaxTokens * kDecodeMaxTopK;
constexpr int kDecodeMaxExperts = 256;
constexpr int kLogitBar = 11;  // named barrier of the logit warps (1..10 are the unit groups')

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void group_bar(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// The arrival half of a grid barrier, by thread 0 after a CTA-level barrier that orders the
// writes other CTAs need: release, so those writes become visible with the arrival.
__device__ __forceinline__ void grid_arrive(unsigned *bar) {
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
}

// One thread waits until the counter reaches target; false if the wait ran out (it then sets bit 2
// of err) or another CTA reported an error (any bit of err; a non-finite output is not an error).
__device__ __forceinline__ bool grid_spin(unsigned *bar, unsigned target, uint32_t *err, long long limit) {
    const long long t0 = clock64();
    for (unsigned it = 0; ld_acquire_gpu(bar) < target; ++it) {
        if ((it & 63u) == 63u) {
            if (*reinterpret_cast<volatile uint32_t *>(err) & ~kErrNonFinite) return false;
            if (clock64() - t0 > limit) { atomicOr(err, 2u); return false; }
        }
    }
    return true;
}

__device__ __forceinline__ long long wait_limit(const DecodeParams &p) { return p.wait_cycles > 0 ? p.wait_cycles : kGridWaitCycles; }

// The waiting half: returns false (uniformly within the CTA) if the wait ran out or another
// CTA reported an error.
__device__ bool grid_wait(const DecodeParams &p, unsigned target, int *ok_s) {
    if (threadIdx.x == 0) *ok_s = grid_spin(p.bar, target, p.err, wait_limit(p));
    __syncthreads();
    return *ok_s != 0;
}

// All CTAs arrive, then wait.
__device__ bool grid_sync(const DecodeParams &p, unsigned target, int *ok_s) {
    __syncthreads();
    if (threadIdx.x == 0) grid_arrive(p.bar);
    return grid_wait(p, target, ok_s);
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Cross-rank end of a phase (expert parallelism): every thread's earlier stores, this GPU's and the
// peers', are fenced system-wide; the CTAs of this rank meet at the grid barrier; CTA 0 then publishes
// exchange number e into this rank's slot of every rank's flag array (release), and every CTA waits,
// bounded, until every rank has published e here (acquire).  A rank that never arrives costs one wait
// bound and sets bit 2 of err.  Returns the CTA-uniform outcome.
__device__ bool ep_sync(const DecodeParams &p, unsigned &target, unsigned e, int *ok_s) {
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) grid_arrive(p.bar);
    target += gridDim.x;
    if (!grid_wait(p, target, ok_s)) return false;
    if (threadIdx.x == 0) {
        if (blockIdx.x == 0)
            for (int q = 0; q < p.ep_world; ++q) st_release_sys(p.peer_flags[q] + p.ep_rank, e);
        int ok = 1;
        const long long t0 = clock64();
        for (int src = 0; src < p.ep_world && ok; ++src) {
            for (unsigned it = 0; ld_acquire_sys(p.flags + src) < e; ++it) {
                if ((it & 63u) != 63u) continue;
                if ((*reinterpret_cast<volatile uint32_t *>(p.err) & ~kErrNonFinite) || clock64() - t0 > p.ep_wait_cycles) {
                    atomicOr(p.err, 2u);
                    ok = 0;
                    break;
                }
            }
        }
        *ok_s = ok;
    }
    __syncthreads();
    return *ok_s != 0;
}

struct DecSmem {
    float *wrow;    // [kDecRouterRows][H] router rows of this CTA's experts (bulk-copied a layer ahead)
    float *hs;      // [T][H] residual stream (this CTA's copy)
    uint8_t *xrec;  // [T][nb][64] Q8_0 records of the normalised h
    float *xsc;     // [T][pad4(nb)]
    uint8_t *arec;  // [2T][nbI][64] Q8_0 records of the activations this CTA's down units read
    float *asc;     // [2T][pad4(nbI)]
    uint8_t *ring;  // [warps][S][kRingStageBytes] weight stream rings
};

constexpr int kDecRouterRows = 2;  // experts <= 2 * #CTAs

// Ring stages per warp.  One token, 36 GPT-OSS-120B-shaped layers: depths 3 / 4 / 5 / 6 / 7
// measured 800 / 786 / 771 / 743 / 714 tok/s (more bytes in flight per SM did not pay, less
// shared memory did); more tokens need the staging room.
__host__ __device__ constexpr int ring_stages(int T) { return T == 1 ? 3 : 2; }

// stages: the ring depth of the kernel instantiation (ring_stages(MT)).
__host__ __device__ inline size_t decode_smem_layout(int T, int H, int I, int stages, size_t off[7]) {
    const size_t nb = H / 32, nbI = I / 32;
    size_t o = 0;
    off[0] = o; o += (size_t)kDecRouterRows * H * 4;
    off[1] = o; o += (size_t)T * H * 4;
    off[2] = o; o += (size_t)T * nb * 64;
    off[3] = o; o += (size_t)T * pad4((int)nb) * 4;
    off[4] = o; o += (size_t)2 * T * nbI * 64;
    off[5] = o; o += (size_t)2 * T * pad4((int)nbI) * 4;
    off[6] = o; o += (size_t)kDecWarps * stages * kRingStageBytes;
    return o;
}

// Q8_0 records of n_blk 32-value blocks of src (block i = row i / nb, block i % nb, rows of width
// H, each scaled by inv[row] first), eight threads per block with four values each, so a
// block's scale takes three shuffles: thread j of a block holds elements 4j..4j+3, i.e. one code
// word of the record.  Same codes and scales as quantize_record.  Called by whole warps
// (first_warp .. first_warp + n_warps - 1, warp = this thread's warp).
__device__ __forceinline__ void quantize_records4(const float *src, const float *inv, int n_blk, int nb, int H,
                                                  uint8_t *rec, float *scale, int scale_stride, int warp, int lane,
                                                  int first_warp, int n_warps) {
    const int total = n_blk * 8;
    for (int base = (warp - first_warp) * 32; base < total; base += n_warps * 32) {
        const int it = base + lane;
        const bool on = it < total;  // groups of 8 are all on or all off (total is a multiple of 8)
        const int blk = on ? it >> 3 : 0, j = it & 7;
        const int t = blk / nb, b = blk - t * nb;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (on) {
            const float4 h = *reinterpret_cast<const float4 *>(src + (size_t)t * H + b * 32 + 4 * j);
            const float sc = inv[t];
            v = make_float4(__fmul_rn(h.x, sc), __fmul_rn(h.y, sc), __fmul_rn(h.z, sc), __fmul_rn(h.w, sc));
        }
        float am = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
        am = fmaxf(am, __shfl_xor_sync(kFull, am, 1));
        am = fmaxf(am, __shfl_xor_sync(kFull, am, 2));
        am = fmaxf(am, __shfl_xor_sync(kFull, am, 4));
        if (on) {
            const float qinv = am != 0.0f ? __fdiv_rn(127.0f, am) : 0.0f;
            const uint32_t w = ((uint32_t)q8_code(v.x, qinv) & 0xffu) | (((uint32_t)q8_code(v.y, qinv) & 0xffu) << 8) |
                               (((uint32_t)q8_code(v.z, qinv) & 0xffu) << 16) | ((uint32_t)q8_code(v.w, qinv) << 24);
            const int lh = j >> 2, pp = j & 3;
            *reinterpret_cast<uint2 *>(rec + (size_t)blk * 64 + (lh * 2 + (pp >> 1)) * 16 + (pp & 1) * 8) =
                make_uint2(w, neg8x4(w));
            if (j == 0) scale[(size_t)t * scale_stride + b] = f16_bits_to_f32(f32_to_f16_bits(__fdiv_rn(am, 127.0f)));
        }
    }
}

// Q8_0 records (the codes and scales of quantize_records4) of nar activation rows of width I, row a
// being row jobs[a] of act in global memory, by every thread of the CTA with four items each in
// flight (an item: four values of a 32-value block).
__device__ __forceinline__ void quantize_act_rows(const float *act, const int *jobs, int nar, int nbI, int I,
                                                  uint8_t *rec, float *scale, int scale_stride, int warp, int lane) {
    const int total = nar * nbI * 8;
    for (int b0 = warp * 32; b0 < total; b0 += 4 * kDecThreads) {
        float4 v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int it = b0 + k * kDecThreads + lane;
            v[k] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (it < total) {
                const int blk = it >> 3, a = blk / nbI, b = blk - a * nbI;
                v[k] = __ldcg(reinterpret_cast<const float4 *>(act + (size_t)jobs[a] * I + b * 32 + 4 * (it & 7)));
            }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int it = b0 + k * kDecThreads + lane;
            const bool on = it < total;  // groups of 8 are all on or all off
            float am = fmaxf(fmaxf(fabsf(v[k].x), fabsf(v[k].y)), fmaxf(fabsf(v[k].z), fabsf(v[k].w)));
            am = fmaxf(am, __shfl_xor_sync(kFull, am, 1));
            am = fmaxf(am, __shfl_xor_sync(kFull, am, 2));
            am = fmaxf(am, __shfl_xor_sync(kFull, am, 4));
            if (on) {
                const int blk = it >> 3, j = it & 7, a = blk / nbI, b = blk - a * nbI;
                const float qinv = am != 0.0f ? __fdiv_rn(127.0f, am) : 0.0f;
                const uint32_t w = ((uint32_t)q8_code(v[k].x, qinv) & 0xffu) |
                                   (((uint32_t)q8_code(v[k].y, qinv) & 0xffu) << 8) |
                                   (((uint32_t)q8_code(v[k].z, qinv) & 0xffu) << 16) |
                                   ((uint32_t)q8_code(v[k].w, qinv) << 24);
                const int lh = j >> 2, pp = j & 3;
                *reinterpret_cast<uint2 *>(rec + (size_t)blk * 64 + (lh * 2 + (pp >> 1)) * 16 + (pp & 1) * 8) =
                    make_uint2(w, neg8x4(w));
                if (j == 0) scale[(size_t)a * scale_stride + b] = f16_bits_to_f32(f32_to_f16_bits(__fdiv_rn(am, 127.0f)));
            }
        }
    }
}

// out4[i] = (residual ? h4[i] : 0) + sum_r w[t][r] * y[t*K + r] over float4 columns, rank order;
// the loads of four ranks are in flight together.
__device__ __forceinline__ float4 fold4(const float4 *y4, const float *w, int t, int K, int H4, int n4, float4 h,
                                        int residual) {
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int r0 = 0; r0 < K; r0 += 4) {
        float4 yv[4];
#pragma unroll
        for (int r = 0; r < 4; ++r)
            if (r0 + r < K) yv[r] = __ldcg(y4 + (size_t)(t * K + r0 + r) * H4 + n4);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            if (r0 + r < K) {
                const float wr = w[t * K + r0 + r];
                acc.x = __fadd_rn(acc.x, __fmul_rn(wr, yv[r].x));
                acc.y = __fadd_rn(acc.y, __fmul_rn(wr, yv[r].y));
                acc.z = __fadd_rn(acc.z, __fmul_rn(wr, yv[r].z));
                acc.w = __fadd_rn(acc.w, __fmul_rn(wr, yv[r].w));
            }
        }
    }
    if (!residual) return acc;
    return make_float4(__fadd_rn(h.x, acc.x), __fadd_rn(h.y, acc.y), __fadd_rn(h.z, acc.z), __fadd_rn(h.w, acc.w));
}

// EP: the expert-parallel form (DecodeParams::ep_world > 1), a separate instantiation so that the
// single-GPU kernels carry none of its code.
template <int MT, bool EP>
__global__ void __launch_bounds__(kDecThreads, 1) k_decode(const __grid_constant__ DecodeParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ float inv_s[kDecodeMaxTokens];
    __shared__ int sel_e[kMaxEntries];
    __shared__ float sel_w[kMaxEntries];
    __shared__ int n_slots_s;
    __shared__ int slot_e[kMaxEntries], slot_cnt[kMaxEntries], slot_first[kMaxEntries];
    __shared__ int job_j[kMaxEntries];  // entries t*K + r grouped by slot, ascending within a slot
    __shared__ float xch_g[kGuGroups][MT][2][16][4];
    __shared__ float res_g[kGuGroups][MT][2][16];
    __shared__ float xch_d[kDnGroups][MT][16][4];
    __shared__ int ok_s, late_s;
    __shared__ __align__(8) uint64_t wbar;
    __shared__ __align__(16) float wbias[kDecRouterRows][4];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nC = gridDim.x, c = blockIdx.x;
    const int T = p.tokens, H = p.hidden, I = p.inter, E = p.experts, K = p.top_k;
    const int nb = H / 32, nbI = I / 32, N = T * K, H4 = H / 4;
    const int G1 = I / 16, G2 = H / 16;
    const int my_e = c < E ? (E - 1 - c) / nC + 1 : 0;  // router rows of this CTA (<= kDecRouterRows)
    const int n_lw = my_e * T;                          // warps computing logits; the others quantize h
    constexpr int S = ring_stages(MT);
    size_t off[7];
    decode_smem_layout(T, H, I, S, off);
    DecSmem sm{reinterpret_cast<float *>(smem + off[0]), reinterpret_cast<float *>(smem + off[1]), smem + off[2],
               reinterpret_cast<float *>(smem + off[3]), smem + off[4], reinterpret_cast<float *>(smem + off[5]),
               smem + off[6]};
    uint8_t *my_ring = sm.ring + (size_t)warp * S * kRingStageBytes;
    unsigned target = 0;
    uint32_t wphase = 0;

    if (tid == 0) {
        mbar_init(&wbar, 1);
        late_s = 0;
        if (my_e > 0) load_router_rows(p.layer[0].router_w, p.layer[0].router_b, c, nC, my_e, H, sm.wrow, wbias, &wbar);
    }
    constexpr bool ep = EP;
    __shared__ unsigned ep_base_s;
    if (ep) {
        // this rank's token into row ep_rank of every rank's x_all (a slice per CTA), the first exchange,
        // then h <- x_all: every rank holds all ranks' tokens
        if (tid == 0) ep_base_s = *reinterpret_cast<volatile unsigned *>(p.epoch);
        const int lo4 = (int)((long long)c * H4 / nC), hi4 = (int)((long long)(c + 1) * H4 / nC);
        for (int i = lo4 + tid; i < hi4; i += kDecThreads) {
            float4 v;
            if (p.x_dtype == UMSX_DTYPE_BF16) {
                const uint2 b = reinterpret_cast<const uint2 *>(p.x)[i];
                v = make_float4(bf16_bits_to_f32(b.x & 0xffffu), bf16_bits_to_f32(b.x >> 16), bf16_bits_to_f32(b.y & 0xffffu),
                                bf16_bits_to_f32(b.y >> 16));
            } else {
                v = reinterpret_cast<const float4 *>(p.x)[i];
            }
            for (int q = 0; q < p.ep_world; ++q) reinterpret_cast<float4 *>(p.peer_x[q])[(size_t)p.ep_rank * H4 + i] = v;
        }
        if (!ep_sync(p, target, ep_base_s + 1u, &ok_s)) return;
        for (int i = tid; i < T * H4; i += kDecThreads)
            reinterpret_cast<float4 *>(sm.hs)[i] = __ldcg(reinterpret_cast<const float4 *>(p.x_all) + i);
    } else if (p.x_dtype == UMSX_DTYPE_BF16) {
        const uint16_t *xb = static_cast<const uint16_t *>(p.x);
        for (int i = tid; i < T * H; i += kDecThreads) sm.hs[i] = bf16_bits_to_f32(xb[i]);
    } else {
        const float4 *xf = static_cast<const float4 *>(p.x);
        for (int i = tid; i < T * H4; i += kDecThreads) reinterpret_cast<float4 *>(sm.hs)[i] = xf[i];
    }

    for (int l = 0; l < p.n_layers; ++l) {
        const DecodeLayer &Ld = p.layer[l];
        // ---- R: fold in the previous layer, normalise, logits, x records ----------
        if (l > 0) {
            float4 *h4 = reinterpret_cast<float4 *>(sm.hs);
            const float4 *y4 = reinterpret_cast<const float4 *>(p.y);
            for (int i = tid; i < T * H4; i += kDecThreads) {
                const int t = i / H4;
                h4[i] = fold4(y4, sel_w, t, K, H4, i - t * H4, h4[i], p.residual);
            }
        }
        __syncthreads();
        if (warp < T) {
            float inv = 1.0f;  // x * 1 is exact: without RMSNorm the products below leave h unchanged
            if (p.rmsnorm) {
                const float *ht = sm.hs + (size_t)warp * H;
                float a = 0.0f;
#pragma unroll 2  // the next chunk's shared-memory loads in flight during this chunk's chain
                for (int k0 = lane; k0 < H; k0 += 32 * 8) {
                    float v[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) v[j] = k0 + 32 * j < H ? ht[k0 + 32 * j] : 0.0f;
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        if (k0 + 32 * j < H) a = __fmaf_rn(v[j], v[j], a);
                }
                const float ss = warp_tree_sum(a);
                inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)H), p.eps)));
            }
            if (lane == 0) inv_s[warp] = inv;
        }
        __syncthreads();
        if (warp < n_lw) {
            // logits of (expert, token) pairs: 32 strided FMA chains, then the xor tree
            if (!mbar_wait_bounded(&wbar, wphase, kWaitLimitCycles) && lane == 0) late_s = 1;
            for (int q = warp; q < n_lw; q += kDecWarps) {
                const int j = q / T, t = q - j * T, e = c + nC * j;
                const float *wr = sm.wrow + (size_t)j * H;
                const float *ht = sm.hs + (size_t)t * H;
                const float inv = inv_s[t];
                float acc = 0.0f;
#pragma unroll 2  // the next chunk's shared-memory loads in flight during this chunk's chain
                for (int k0 = lane; k0 < H; k0 += 32 * 8) {
                    float w[8], x[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        w[i] = k0 + 32 * i < H ? wr[k0 + 32 * i] : 0.0f;
                        x[i] = k0 + 32 * i < H ? ht[k0 + 32 * i] : 0.0f;
                    }
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        if (k0 + 32 * i < H) acc = __fmaf_rn(w[i], __fmul_rn(x[i], inv), acc);
                }
                float lg = warp_tree_sum(acc);
                if (Ld.router_b) lg = __fadd_rn(lg, wbias[j][e & 3]);
                if (lane == 0) __stcg(p.logits + (size_t)t * E + e, lg);
            }
            // this CTA's logits are out: it arrives at the grid barrier now and quantizes x (a
            // CTA-local job) while the other CTAs finish
            group_bar(kLogitBar, n_lw * 32);
            if (tid == 0 && !(l == 0 && c == p.fault_cta)) grid_arrive(p.bar);
        } else {
            if (n_lw == 0 && tid == 0 && !(l == 0 && c == p.fault_cta)) grid_arrive(p.bar);  // no logits here
            // Q8_0 records of the normalised rows (the gate_up activations), every CTA its own copy,
            // made by the warps that have no logit to compute
            quantize_records4(sm.hs, inv_s, T * nb, nb, H, sm.xrec, sm.xsc, pad4(nb), warp, lane, n_lw, kDecWarps - n_lw);
        }
        wphase ^= 1u;
        __syncthreads();
        if (late_s) {  // the router rows never arrived: report, let the copy land, stop
            if (tid == 0) atomicOr(p.err, 4u);
            mbar_wait_bounded(&wbar, wphase ^ 1u, kWaitLimitCycles);
            return;
        }
        target += nC;
        if (!grid_wait(p, target, &ok_s)) return;

        // ---- S: selection and slots (every CTA) -----------------------------------
        if (warp < T) {
            int sel;
            float w;
            // as many candidates per lane as the router has experts (the same picks, a shorter chain)
            if (E <= 128)
                select_topk<4>(p.logits + (size_t)warp * E, E, K, p.routing, p.routed_scale, lane, sel, w);
            else
                select_topk<kDecodeMaxExperts / 32>(p.logits + (size_t)warp * E, E, K, p.routing, p.routed_scale, lane, sel, w);
            if (lane < K) { sel_e[warp * K + lane] = sel; sel_w[warp * K + lane] = w; }
        }
        __syncthreads();
        if (MT == 1 && T == 1 && warp == 0) {
            // one token: its k picks are distinct experts, so slot r is rank r with the one job r
            const bool has = lane < K;
            int ej = has ? sel_e[lane] : 0;
            if (has && (ej < 0 || ej >= E)) {  // cannot happen (selection always picks a valid expert); never index with it
                atomicOr(p.err, 8u);
                ej = 0;
            }
            if (has) { slot_e[lane] = ej; slot_cnt[lane] = 1; slot_first[lane] = lane; job_j[lane] = lane; }
            if (lane == 0) n_slots_s = K;
            if (c == 0 && l == p.n_layers - 1 && p.ids_out && has) {
                p.ids_out[lane] = ej;
                p.w_out[lane] = sel_w[lane];
            }
        } else if (warp == 0) {
            bool has = lane < N;
            int ej = has ? sel_e[lane] : 0x7fffffff;
            if (has && (ej < 0 || ej >= E)) {  // cannot happen (selection always picks a valid expert); never index with it
                atomicOr(p.err, 8u);
                ej = 0;
            }
            if (c == 0 && l == p.n_layers - 1 && p.ids_out && has) {
                p.ids_out[lane] = ej;
                p.w_out[lane] = sel_w[lane];
            }
            if (ep && has) {  // this rank runs the jobs of its own experts only, indexed locally
                if (ej >= p.e_lo && ej < p.e_lo + p.e_local) {
                    ej -= p.e_lo;
                } else {
                    has = false;
                    ej = 0x7fffffff;
                }
            }
            int same_before = 0, cnt = 0, less = 0;
            for (int j = 0; j < N; ++j) {
                const int o = __shfl_sync(kFull, ej, j);
                same_before += (o == ej && j < lane);
                cnt += o == ej;
                less += o < ej;
            }
            const bool first = has && same_before == 0;
            const unsigned firsts = __ballot_sync(kFull, first);
            int slot = 0;
            for (int j = 0; j < N; ++j) {
                const int o = __shfl_sync(kFull, ej, j);
                slot += ((firsts >> j) & 1u) && o < ej;
            }
            if (first) { slot_e[slot] = ej; slot_cnt[slot] = cnt; slot_first[slot] = less; }
            if (has) job_j[less + same_before] = lane;
            if (lane == 0) n_slots_s = __popc(firsts);
        }
        __syncthreads();
        const int n_slots = n_slots_s;
        const int U1 = n_slots * G1, U2 = n_slots * G2;
        const int u_lo = c * U1 / nC, u_hi = (c + 1) * U1 / nC;  // c * U1 < 2^31 at every supported shape
        const int v_lo = c * U2 / nC, v_hi = (c + 1) * U2 / nC;
        // ---- G: gate_up units ------------------------------------------------------
        {
            const int gi = warp >> 2, wg = warp & 3, half = wg >> 1, lh = wg & 1, gt = tid & 127;
            const int r = lane & 15;
            Staged xs;
            xs.q = reinterpret_cast<const uint4 *>(sm.xrec);
            xs.sc = sm.xsc;
            xs.flag = nullptr;
            xs.scs = pad4(nb);
            for (int u = u_lo + gi; u < u_hi; u += kGuGroups) {
                const int s = u / G1, g = u - s * G1;
                const int e = slot_e[s], cnt = slot_cnt[s], jf = slot_first[s];
                const int rg = half * G1 + g;
                MxRing ws;
                ws.init(Ld.gu_codes + code_offset(UMSX_QUANT_MXFP4, e, 2 * G1, rg, nb),
                        Ld.gu_scales + scale_offset(UMSX_QUANT_MXFP4, e, 2 * G1, rg, nb), nb, lh, my_ring);
                const float bias = Ld.gu_bias ? __ldg(Ld.gu_bias + (size_t)e * 2 * I + half * I + g * 16 + r) : 0.0f;
                for (int c0 = 0; c0 < cnt; c0 += MT) {
                    const int m = min(MT, cnt - c0);
                    int trow[MT];
#pragma unroll
                    for (int t = 0; t < MT; ++t) trow[t] = t < m ? job_j[jf + c0 + t] / K : 0;
                    float acc[MT][4];
                    if (Ld.gu_ge2) mx_warp_dot_ring<MT, S, true>(ws, lh, xs, nb, m, lane, acc, trow);
                    else mx_warp_dot_ring<MT, S, false>(ws, lh, xs, nb, m, lane, acc, trow);
                    mx_chain_combine<MT>(acc);
                    if (lh == 1 && lane < 16)
#pragma unroll
                        for (int t = 0; t < MT; ++t)
                            if (t < m)
#pragma unroll
                                for (int q = 0; q < 4; ++q) xch_g[gi][t][half][r][q] = acc[t][q];
                    group_bar(1 + gi, 128);
                    if (lh == 0 && lane < 16)
#pragma unroll
                        for (int t = 0; t < MT; ++t)
                            if (t < m) res_g[gi][t][half][r] = __fadd_rn(mx_row_total(acc[t], xch_g[gi][t][half][r]), bias);
                    group_bar(1 + gi, 128);
                    for (int i = gt; i < m * 16; i += 128) {
                        const int t = i >> 4, k = i & 15;
                        const float gv = res_g[gi][t][0][k], uv = res_g[gi][t][1][k];
                        const float a = p.activation == UMSX_ACT_SWIGLU_OAI ? swiglu_oai(gv, uv, p.alpha, p.limit) : silu_mul(gv, uv);
                        __stcg(p.act + (size_t)job_j[jf + c0 + t] * I + g * 16 + k, a);
                    }
                    // (the down phase quantizes the activations: each CTA the rows its units read)
                    group_bar(1 + gi, 128);
                }
            }
        }
        // arrive, then start each warp's first down weights streaming while the others finish
        __syncthreads();
        if (tid == 0) grid_arrive(p.bar);
        target += nC;
        const int di0 = warp >> 1, lh0 = warp & 1;
        const bool primed = v_lo + di0 < v_hi;
        if (primed) {
            const int s = (v_lo + di0) / G2, g = v_lo + di0 - s * G2, e = slot_e[s];
            MxRing ws;
            ws.init(Ld.dn_codes + code_offset(UMSX_QUANT_MXFP4, e, G2, g, nbI),
                    Ld.dn_scales + scale_offset(UMSX_QUANT_MXFP4, e, G2, g, nbI), nbI, lh0, my_ring);
            mx_ring_prime<S>(ws, lane);
        }
        if (!grid_wait(p, target, &ok_s)) {
            cp_async_wait<0>();  // the primed copies land before the CTA leaves
            return;
        }

        // ---- D: down units -----------------------------------------------------------
        if (tid == 0 && my_e > 0 && l + 1 < p.n_layers)
            load_router_rows(p.layer[l + 1].router_w, p.layer[l + 1].router_b, c, nC, my_e, H, sm.wrow, wbias, &wbar);
        int jb = 0;
        if (v_lo < v_hi) {
            const int s_lo = v_lo / G2, s_hi = (v_hi - 1) / G2;
            jb = slot_first[s_lo];
            const int nar = slot_first[s_hi] + slot_cnt[s_hi] - jb;  // <= 2T: a CTA spans at most two slots
            quantize_act_rows(p.act, job_j + jb, nar, nbI, I, sm.arec, sm.asc, pad4(nbI), warp, lane);
        }
        __syncthreads();
        {
            const int di = warp >> 1, lh = warp & 1, r = lane & 15;
            Staged as;
            as.q = reinterpret_cast<const uint4 *>(sm.arec);
            as.sc = sm.asc;
            as.flag = nullptr;
            as.scs = pad4(nbI);
            for (int v = v_lo + di; v < v_hi; v += kDnGroups) {
                const int s = v / G2, g = v - s * G2;
                const int e = slot_e[s], cnt = slot_cnt[s], jf = slot_first[s];
                MxRing ws;
                ws.init(Ld.dn_codes + code_offset(UMSX_QUANT_MXFP4, e, G2, g, nbI),
                        Ld.dn_scales + scale_offset(UMSX_QUANT_MXFP4, e, G2, g, nbI), nbI, lh, my_ring);
                const float bias = Ld.dn_bias ? __ldg(Ld.dn_bias + (size_t)e * H + g * 16 + r) : 0.0f;
                for (int c0 = 0; c0 < cnt; c0 += MT) {
                    const int m = min(MT, cnt - c0);
                    int trow[MT];
#pragma unroll
                    for (int t = 0; t < MT; ++t) trow[t] = t < m ? jf + c0 + t - jb : 0;
                    float acc[MT][4];
                    if (Ld.dn_ge2) mx_warp_dot_ring<MT, S, true>(ws, lh, as, nbI, m, lane, acc, trow, primed && v == v_lo + di && c0 == 0);
                    else mx_warp_dot_ring<MT, S, false>(ws, lh, as, nbI, m, lane, acc, trow, primed && v == v_lo + di && c0 == 0);
                    mx_chain_combine<MT>(acc);
                    if (lh == 1 && lane < 16)
#pragma unroll
                        for (int t = 0; t < MT; ++t)
                            if (t < m)
#pragma unroll
                                for (int q = 0; q < 4; ++q) xch_d[di][t][r][q] = acc[t][q];
                    group_bar(1 + di, 64);
                    if (lh == 0 && lane < 16)
#pragma unroll
                        for (int t = 0; t < MT; ++t)
                            if (t < m) {
                                float y = mx_row_total(acc[t], xch_d[di][t][r]);
                                if (Ld.dn_bias) y = __fadd_rn(y, bias);
                                const size_t o = (size_t)job_j[jf + c0 + t] * H + g * 16 + r;
                                if (ep) {  // every rank folds every token: the row goes to all of them
                                    for (int q = 0; q < p.ep_world; ++q) __stcg(p.peer_y[q] + o, y);
                                } else {
                                    __stcg(p.y + o, y);
                                }
                            }
                    group_bar(1 + di, 64);
                }
            }
        }
        if (ep) {
            if (!ep_sync(p, target, ep_base_s + 2u + (unsigned)l, &ok_s)) return;
        } else {
            target += nC;
            if (!grid_sync(p, target, &ok_s)) return;
        }
    }
    if (ep && c == 0 && tid == 0) *p.epoch = ep_base_s + 1u + (unsigned)p.n_layers;  // every CTA read the base
    // final fold: each CTA writes its share of the output rows, and records a non-finite value (checking
    // the last layer suffices: an inf or NaN in h turns the next layer's RMSNorm, and so its output, NaN)
    const int total4 = T * H4;
    const int lo = (int)((long long)c * total4 / nC), hi = (int)((long long)(c + 1) * total4 / nC);
    const float4 *y4 = reinterpret_cast<const float4 *>(p.y);
    for (int i = lo + tid; i < hi; i += kDecThreads) {
        const int t = i / H4;
        const float4 v = fold4(y4, sel_w, t, K, H4, i - t * H4, reinterpret_cast<const float4 *>(sm.hs)[i], p.residual);
        flag_nonfinite4(v, p.err);
        reinterpret_cast<float4 *>(p.out)[i] = v;
    }
}

template <int MT, bool EP>
int launch_decode_mt(const DecodeParams &p, cudaStream_t s) {
    size_t off[7];
    const size_t dyn = decode_smem_layout(p.tokens, p.hidden, p.inter, ring_stages(MT), off);
    auto kern = k_decode<MT, EP>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn) != cudaSuccess) return -1;
    // shared memory as small as the kernel needs: the rest of the 256 KB stays L1
    if (cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxL1) != cudaSuccess) return -1;
    int dev = 0, sms = 0, per_sm = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return -1;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kDecThreads, dyn) != cudaSuccess || per_sm < 1)
        return -1;
    // a CTA's down units then span at most two slots, whose jobs fit the 2T staged rows
    if (min(p.experts, p.tokens * p.top_k) > sms || p.experts > kDecRouterRows * sms) return -1;
    if (cudaMemsetAsync(p.bar, 0, sizeof(unsigned), s) != cudaSuccess) return -1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(sms);
    cfg.blockDim = dim3(kDecThreads);
    cfg.dynamicSmemBytes = dyn;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, p) != cudaSuccess) return -1;
    return 1;
}

}  // namespace

bool decode_supported(int tokens, int hidden, int inter, int experts, int top_k, int n_layers) {
    return tokens >= 1 && tokens <= kDecodeMaxTokens && top_k >= 1 && top_k <= kDecodeMaxTopK && experts >= top_k &&
           experts <= kDecodeMaxExperts && n_layers >= 1 && n_layers <= kDecodeMaxLayers && hidden % 64 == 0 && inter % 64 == 0;
}

int launch_decode(const DecodeParams &p, cudaStream_t s) {
    // Expert parallelism: each rank's share of the G tokens' jobs mostly has one job per expert slot, so
    // the one-job-per-pass kernel (deeper rings; a slot with more jobs streams its rows once per job) serves it.
    if (p.ep_world > 1) return launch_decode_mt<1, true>(p, s);
    return p.tokens == 1 ? launch_decode_mt<1, false>(p, s) : launch_decode_mt<kDecodeMaxTokens, false>(p, s);
}

}  // namespace umsx
