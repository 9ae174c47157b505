// Expert-parallel exchange kernels: the dispatch / combine all-to-all of a decode step as plain P2P
// stores into the peers' exchange buffers over NVLink, from inside the two kernels below.
//
// Every rank g of G holds experts [g*E/G, (g+1)*E/G) of every layer and one token of the step
// (token g).  Per layer:
//   k_ep_share    writes this rank's hidden row into every peer's h_all[g] (the router is replicated:
//                 each rank routes all G tokens), publishes a flag in every peer, and waits until every
//                 peer's flag for this exchange has arrived;
//   (router + the local experts' jobs of all G tokens: the per-stage kernels, job rows y[t][r])
//   k_ep_combine  writes each local job's output row into the token owner's y_recv[r], flags, waits,
//                 then folds its own token: h <- h + sum_r w[g][r] * y_recv[r] in rank order, the
//                 reference's combine (tools/engine/expert_dispatch.cpp:77-87).
// The peers' buffers are reached through CUDA IPC mappings; stores are plain st.global, flags
// st.release.sys after a system-scope fence, waits ld.acquire.sys with a bounded spin (a rank that
// never arrives costs the others one wait bound and an error bit, not a hang).  Exchange numbers
// (epochs) count the exchanges of this rank's buffer; every rank runs the same sequence.
#include <stdint.h>

#include "umsx_device.cuh"
#include "umsx_internal.h"

namespace umsx {

namespace {

constexpr int kEpThreads = 512;

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Publishes epoch e to every peer's flag slot of this rank, then waits (thread 0, bounded) until every
// peer has published e here.  All threads' earlier stores are fenced system-wide first.  Returns the
// CTA-uniform outcome.
__device__ bool ep_exchange(const EpParams &p, unsigned e, int *ok_s) {
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int q = 0; q < p.world; ++q) st_release_sys(p.peer_flags[q] + p.rank, e);
        int ok = 1;
        const long long t0 = clock64();
        for (int src = 0; src < p.world && ok; ++src) {
            for (unsigned it = 0; ld_acquire_sys(p.flags + src) < e; ++it) {
                if ((it & 63u) != 63u) continue;
                // an exchange that already gave up in this call (its error bit is set) ends this one at once
                if ((*reinterpret_cast<volatile uint32_t *>(p.err) & ~kErrNonFinite) || clock64() - t0 > p.wait_cycles) {
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

__global__ void __launch_bounds__(kEpThreads) k_ep_share(EpParams p) {
    __shared__ unsigned e_s;
    __shared__ int ok_s;
    if (threadIdx.x == 0) e_s = ++*p.epoch;
    __syncthreads();
    const int H4 = p.hidden / 4;
    const float4 *h = reinterpret_cast<const float4 *>(p.h_own);
    for (int q = 0; q < p.world; ++q) {
        float4 *dst = reinterpret_cast<float4 *>(p.peer_h_all[q]) + (size_t)p.rank * H4;
        for (int i = threadIdx.x; i < H4; i += blockDim.x) dst[i] = h[i];
    }
    ep_exchange(p, e_s, &ok_s);
}

__global__ void __launch_bounds__(kEpThreads) k_ep_combine(EpParams p) {
    __shared__ unsigned e_s;
    __shared__ int ok_s;
    if (threadIdx.x == 0) e_s = ++*p.epoch;
    __syncthreads();
    const int K = p.top_k, H4 = p.hidden / 4;
    // dispatch back: the rows of this rank's jobs go to the rank that owns the token
    for (int j = 0; j < p.world * K; ++j) {
        const int e = __ldg(p.ids + j) - p.e_lo;
        if (e < 0 || e >= p.e_local) continue;
        const int t = j / K, r = j - t * K;
        const float4 *src = reinterpret_cast<const float4 *>(p.y_jobs) + (size_t)j * H4;
        float4 *dst = reinterpret_cast<float4 *>(p.peer_y_recv[t]) + (size_t)r * H4;
        for (int i = threadIdx.x; i < H4; i += blockDim.x) dst[i] = __ldcg(src + i);
    }
    if (!ep_exchange(p, e_s, &ok_s)) return;
    // combine this rank's token in rank order, then the residual
    const float *w = p.weights + (size_t)p.rank * K;
    float4 *h = reinterpret_cast<float4 *>(p.h_own);
    const float4 *y = reinterpret_cast<const float4 *>(p.y_recv);
    for (int i = threadIdx.x; i < H4; i += blockDim.x) {
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (int r = 0; r < K; ++r) {
            const float wr = __ldg(w + r);
            const float4 v = __ldcg(y + (size_t)r * H4 + i);
            acc.x = __fadd_rn(acc.x, __fmul_rn(wr, v.x));
            acc.y = __fadd_rn(acc.y, __fmul_rn(wr, v.y));
            acc.z = __fadd_rn(acc.z, __fmul_rn(wr, v.z));
            acc.w = __fadd_rn(acc.w, __fmul_rn(wr, v.w));
        }
        const float4 hv = h[i];
        const float4 o = make_float4(__fadd_rn(hv.x, acc.x), __fadd_rn(hv.y, acc.y), __fadd_rn(hv.z, acc.z),
                                     __fadd_rn(hv.w, acc.w));
        flag_nonfinite4(o, p.err);
        h[i] = o;
    }
}

// ---------------------------------------------------------------------------------------------
// Expert-parallel prefill.  Per layer, on every rank (after the router over its own T tokens):
//   k_ep_count     which ranks each token's experts live on, the token's row in each of those ranks'
//                  receive buffers (tokens ascending), and this rank's row of the G x G count matrix,
//                  stored into every rank's copy;                                   exchange 1
//   k_ep_dispatch  the Q8_0 row of every token (codes + scales: the experts' exact input), its ids on
//                  that rank (-1 elsewhere) and its origin, stored into each destination;  exchange 2
//   (the destination runs its experts over the received rows: dispatch, pack, grouped GEMMs)
//   k_ep_return    every job's output row stored into its token owner's y_back[t][r];     exchange 3
//   (the owner combines y_back in rank order with the residual)
// A producer kernel's CTAs fence their stores system-wide; the last CTA to finish publishes the
// exchange number to every peer (release), and k_ep_wait waits (acquire, bounded) for every peer's.
// Rank g's rows for layer l+1 are written only after g has published its return of layer l, which it
// does after its own experts finished reading the rows of layer l, so no buffer is overwritten
// while it is read.

// The last CTA of a producer kernel publishes the next exchange number to every peer.
__device__ void ep_publish(const EpPrefillParams &p) {
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(p.done, 1u);
        if (prev == gridDim.x - 1) {
            *p.done = 0;
            __threadfence_system();
            const unsigned e = ++*p.epoch;
            for (int q = 0; q < p.world; ++q) st_release_sys(p.peer_flags[q] + p.rank, e);
        }
    }
}

__global__ void __launch_bounds__(1024) k_ep_count(EpPrefillParams p) {
    __shared__ int base[kEpMaxRanks];
    __shared__ int warp_cnt[32][kEpMaxRanks];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    const int G = p.world, K = p.top_k;
    if (tid < kEpMaxRanks) base[tid] = 0;
    __syncthreads();
    for (int t0 = 0; t0 < p.tokens; t0 += blockDim.x) {
        const int t = t0 + tid;
        unsigned mask = 0;
        if (t < p.tokens)
            for (int r = 0; r < K; ++r) {
                const int e = __ldcg(p.ids + (size_t)t * K + r);
                const int g = e / p.e_per_rank;
                if (e >= 0 && g < G) mask |= 1u << g;
            }
        int pre[kEpMaxRanks];
#pragma unroll
        for (int g = 0; g < kEpMaxRanks; ++g) {
            const unsigned b = __ballot_sync(0xffffffffu, (mask >> g) & 1u);
            if (lane == 0) warp_cnt[warp][g] = __popc(b);
            pre[g] = __popc(b & ((1u << lane) - 1u));
        }
        __syncthreads();
#pragma unroll
        for (int g = 0; g < kEpMaxRanks; ++g) {
            if (g >= G) break;
            int off = base[g];
            for (int w = 0; w < warp; ++w) off += warp_cnt[w][g];
            if (t < p.tokens) p.pos[(size_t)t * G + g] = ((mask >> g) & 1u) ? off + pre[g] : -1;
        }
        __syncthreads();
        if (tid < G) {
            int tot = 0;
            for (int w = 0; w < nw; ++w) tot += warp_cnt[w][tid];
            base[tid] += tot;
        }
        __syncthreads();
    }
    if (tid < G * G) {  // this rank's row of the count matrix, in every rank's copy
        const int q = tid / G, g = tid - q * G;
        p.peer_counts[q][p.rank * G + g] = base[g];
    }
    ep_publish(p);
}

__global__ void __launch_bounds__(256) k_ep_dispatch(EpPrefillParams p) {
    __shared__ int off_s[kEpMaxRanks];
    const int G = p.world, K = p.top_k, H = p.hidden, nb = H / 32;
    if (threadIdx.x < G) {  // where this rank's rows start in rank g's buffer
        int o = 0;
        for (int src = 0; src < p.rank; ++src) o += __ldcg(p.counts + src * G + threadIdx.x);
        off_s[threadIdx.x] = o;
    }
    __syncthreads();
    for (int t = blockIdx.x; t < p.tokens; t += gridDim.x) {
        for (int g = 0; g < G; ++g) {
            const int pos = __ldcg(p.pos + (size_t)t * G + g);
            if (pos < 0) continue;
            const int row = off_s[g] + pos;
            if (row >= p.rows_max) {  // a count matrix from a failed exchange
                if (threadIdx.x == 0) atomicOr(p.err, 2u);
                continue;
            }
            const uint4 *cs = reinterpret_cast<const uint4 *>(p.xq_codes + (size_t)t * H);
            uint4 *cd = reinterpret_cast<uint4 *>(p.peer_codes[g] + (size_t)row * H);
            for (int i = threadIdx.x; i < H / 16; i += blockDim.x) cd[i] = __ldcg(cs + i);
            const float *ss = p.xq_scales + (size_t)t * nb;
            float *sd = p.peer_scales[g] + (size_t)row * nb;
            for (int i = threadIdx.x; i < nb; i += blockDim.x) sd[i] = __ldcg(ss + i);
            if (threadIdx.x < K) {
                const int e = __ldcg(p.ids + (size_t)t * K + threadIdx.x);
                p.peer_ids[g][(size_t)row * K + threadIdx.x] = e / p.e_per_rank == g ? e : -1;
            }
            if (threadIdx.x == 0) p.peer_src[g][row] = make_int2(p.rank, t);
        }
    }
    ep_publish(p);
}

__global__ void __launch_bounds__(256) k_ep_return(EpPrefillParams p, int layer) {
    __shared__ int rows_s;
    const int G = p.world, K = p.top_k, H4 = p.hidden / 4;
    if (threadIdx.x == 0) {
        int r = 0;
        for (int src = 0; src < G; ++src) r += __ldcg(p.counts + src * G + p.rank);
        rows_s = min(r, p.rows_max);
        if (blockIdx.x == 0 && p.loads) p.loads[layer] = make_int2(r, __ldcg(p.n_jobs));
    }
    __syncthreads();
    const int R = rows_s, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int j = blockIdx.x * nw + warp; j < R * K; j += gridDim.x * nw) {
        if (__ldcg(p.recv_ids + j) < 0) continue;
        const int2 src = __ldcg(p.recv_src + j / K);
        if (src.x < 0 || src.x >= G || src.y < 0 || src.y >= p.tokens_max) {
            if (lane == 0) atomicOr(p.err, 2u);
            continue;
        }
        const float4 *y = reinterpret_cast<const float4 *>(p.y_jobs) + (size_t)__ldcg(p.inv + j) * H4;
        float4 *dst = reinterpret_cast<float4 *>(p.peer_y_back[src.x]) + ((size_t)src.y * K + j % K) * H4;
        for (int i = lane; i < H4; i += 32) dst[i] = __ldcg(y + i);
    }
    ep_publish(p);
}

// Waits (thread 0, bounded) until every peer has published this rank's latest exchange number.
__global__ void k_ep_wait(EpPrefillParams p) {
    if (threadIdx.x != 0) return;
    const unsigned e = *reinterpret_cast<volatile unsigned *>(p.epoch);
    const long long t0 = clock64();
    for (int src = 0; src < p.world; ++src)
        for (unsigned it = 0; ld_acquire_sys(p.flags + src) < e; ++it) {
            if ((it & 63u) != 63u) continue;
            if ((*reinterpret_cast<volatile uint32_t *>(p.err) & ~kErrNonFinite) || clock64() - t0 > p.wait_cycles) {
                atomicOr(p.err, 2u);
                return;
            }
        }
}

}  // namespace

int launch_ep_count(const EpPrefillParams &p, cudaStream_t s) {
    k_ep_count<<<1, 1024, 0, s>>>(p);
    return 1;
}

int launch_ep_dispatch(const EpPrefillParams &p, cudaStream_t s) {
    k_ep_dispatch<<<p.tokens < 148 * 8 ? p.tokens : 148 * 8, 256, 0, s>>>(p);
    return 1;
}

int launch_ep_return(const EpPrefillParams &p, int layer, cudaStream_t s) {
    k_ep_return<<<148 * 4, 256, 0, s>>>(p, layer);
    return 1;
}

int launch_ep_wait(const EpPrefillParams &p, cudaStream_t s) {
    k_ep_wait<<<1, 32, 0, s>>>(p);
    return 1;
}

int launch_ep_share(const EpParams &p, cudaStream_t s) {
    k_ep_share<<<1, kEpThreads, 0, s>>>(p);
    return 1;
}

int launch_ep_combine(const EpParams &p, cudaStream_t s) {
    k_ep_combine<<<1, kEpThreads, 0, s>>>(p);
    return 1;
}

}  // namespace umsx
