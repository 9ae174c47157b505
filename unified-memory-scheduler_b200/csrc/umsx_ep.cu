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

}  // namespace

int launch_ep_share(const EpParams &p, cudaStream_t s) {
    k_ep_share<<<1, kEpThreads, 0, s>>>(p);
    return 1;
}

int launch_ep_combine(const EpParams &p, cudaStream_t s) {
    k_ep_combine<<<1, kEpThreads, 0, s>>>(p);
    return 1;
}

}  // namespace umsx
