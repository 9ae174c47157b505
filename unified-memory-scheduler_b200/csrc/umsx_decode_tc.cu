// Persistent decode kernel, tensor-core variant (one token): the exact MXFP4 x Q8_0 row
// dots of gate_up and down run on the 5th-generation tensor cores and give the same bits
// as the SIMT kernels and the reference.
//
// The reference's dot (tools/trace/cpu_mxfp4_vnni.cpp:22-68) forms, per 32-value block b,
// eight int lanes L_l = sum of four products (lane l = elements 4l..4l+3) and accumulates
// fma(d_b, L_l, acc_l) in an even-block and an odd-block chain.  Here one
// tcgen05.mma kind::mxf4.block_scale per block pair (K = 64) produces every L exactly:
//   A = 128 weight rows as e2m1, bulk-copied from a copy stored as ready operand tiles
//       (Matrix::tc_codes: stage-major, 32-byte swizzled; no decode at all);
//   B = the token's Q8_0 codes in balanced base 8 (q = d0 + 8 d1 + 64 d2, digits in
//       [-4, 4], each an exact e2m1 value): N = 48 rows n = 24h + 8j + l, row n holding
//       digit plane j of the four elements of int lane l of block h (zeros elsewhere);
//   the per-column B scale 2 * 8^j (and A scale 1) turn D[row][24h + 8j + l] into plane j's
//       share of L, so L = D[.., 24h + l] + D[.., 24h + 8 + l] + D[.., 24h + 16 + l] exactly
//       (every product and partial sum is a small integer).
// D goes to a two-stage ring of TMEM columns; eight epilogue warps (two per TMEM lane group:
// one per chain) run the reference's fp32 chains fma(d_b, L, acc), then its final lane order,
// the bias, and SwiGLU + Q8_0 (gate_up) or the output rows (down).  Activations never hold
// -128 (the quantizer's codes stay within +-127 here), so VPSIGNB and plain products agree.
//
// Routing, the residual fold and the phase structure (R, S, G, D between grid barriers)
// are those of k_decode (umsx_decode.cu).  Work is split into contiguous shares per CTA:
// gate_up in units of (slot, 32 gate rows + the matching 32 up rows), tiled two units at a
// time (gate rows at TMEM lanes 0-63, up rows at 64-127); down in groups of 16 rows, eight
// per tile.  Warp 0 lane 0 issues the bulk copies, lane 0 of warps 1 and 2 the MMAs (alternate
// stages), warps 4-11 are the
// epilogue; every warp builds the digit planes and takes part in the other phases.  Block
// exponents come from the tiled scale plane.
#include <stdint.h>

#include "umsx_device.cuh"
#include "umsx_internal.h"
#include "umsx_mx.cuh"
#include "umsx_tc.cuh"

namespace umsx {
namespace {

constexpr int kTcThreads = 512;
constexpr int kTcWarps = kTcThreads / 32;
constexpr int kAStages = 6;             // weight stages in flight
constexpr int kATile = 128 * 128;       // one stage: 128 weight rows x 128 bytes (4 block pairs)
constexpr int kBoxBytes = 16 * 128;     // one row group's share of a stage (16 rows x 128 bytes)
constexpr int kPlanes = 3;              // base-8 digit planes of the activation codes
constexpr int kBN = 48;                 // B rows = MMA N: 24h + 8j + l
constexpr int kBStages = 12;            // K extent of B: 12 x 256 values
constexpr int kBStage = kBN / 8 * 1024;  // one stage of B: 6 atoms of [4 pairs][8 rows][32 B]
constexpr int kDPair = kBN;             // TMEM result columns per block pair
constexpr int kDStages = 2;             // TMEM ring of stage results (4 pairs each)
constexpr int kSfCol = kDStages * 4 * kDPair;  // 384: A scales (8 columns), then B scales (2)
constexpr int kTmemCols = 512;
constexpr int kMaxKTc = kBStages * 256;
constexpr long long kTcWait = 40000000;  // ~20 ms
constexpr int kMaxEntriesTc = 8;
constexpr int kGuTileUnits = 2;   // gate_up tile: up to two units of 32 + 32 rows
constexpr int kDnTileGroups = 8;  // down tile: up to eight groups of 16 rows
constexpr int kEpiWarps = 8;      // warps 4..11: lane group (warp & 3), chain (warp - 4) >> 2

static_assert(kSfCol + 10 <= kTmemCols, "TMEM columns");
static_assert(kDStages == 2, "the two MMA issuers own one TMEM ring stage each");

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ bool err_set(const uint32_t *err) {
    return *reinterpret_cast<const volatile uint32_t *>(err) != 0u;
}

// All CTAs arrive; false (uniformly within the CTA) if the wait ran out or an error was flagged.
__device__ bool grid_sync_tc(unsigned *bar, unsigned target, uint32_t *err, int *ok_s) {
    __syncthreads();
    if (threadIdx.x == 0) {
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
        int ok = 1;
        const long long t0 = clock64();
        for (unsigned it = 0; ld_acquire(bar) < target; ++it) {
            if ((it & 63u) == 63u) {
                if (err_set(err)) { ok = 0; break; }
                if (clock64() - t0 > kTcWait) { atomicOr(err, 2u); ok = 0; break; }
            }
        }
        *ok_s = ok;
    }
    __syncthreads();
    return *ok_s != 0;
}

__device__ __forceinline__ bool mbar_test_now(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{ .reg .pred p; mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded mbarrier wait that also gives up as soon as any CTA has flagged an error; a phase
// that has completed already costs one non-blocking test.
__device__ __forceinline__ bool wait_tc(uint64_t *bar, uint32_t parity, uint32_t *err) {
    if (mbar_test_now(bar, parity)) return true;
    const long long t0 = clock64();
    for (unsigned it = 0; !mbar_test(bar, parity); ++it) {
        if ((it & 255u) == 255u) {
            if (err_set(err)) return false;
            if (clock64() - t0 > kTcWait) { atomicOr(err, 64u); return false; }
        }
    }
    return true;
}

// Block-scaled MXF4 MMA, K = 64 (two 32-value blocks), scale factors in TMEM.
__device__ __forceinline__ void mma_mxf4(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc,
                                         uint32_t sfa, uint32_t sfb) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb)
        : "memory");
}

__device__ __forceinline__ void tmem_st4(uint32_t taddr, uint32_t v) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(v), "r"(v), "r"(v),
                 "r"(v)
                 : "memory");
}

// Shared-memory descriptor, K-major with the 32-byte swizzle: one block pair (32 bytes) per row,
// 8-row atoms of 256 bytes, `sbo` bytes from one atom to the next along M / N.
__device__ __forceinline__ uint64_t smem_desc_sw32(const void *p, uint32_t sbo) {
    const uint64_t addr = smem_u32(p);
    return ((addr & 0x3FFFFull) >> 4) | (1ull << 16) | ((uint64_t)(sbo >> 4) << 32) | (1ull << 46) | (6ull << 61);
}

__device__ __forceinline__ void tmem_st2(uint32_t taddr, uint32_t v0, uint32_t v1) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x2.b32 [%0], {%1, %2};" ::"r"(taddr), "r"(v0), "r"(v1) : "memory");
}

// Instruction descriptor: A, B e2m1 (K-major), ue8m0 scales, M = 128, N = 48, dense K = 64.
constexpr uint32_t kIdescMxf4 = (1u << 7) | (1u << 10) | ((uint32_t)(kBN >> 3) << 17) | (1u << 23) | ((128u >> 4) << 24);

// Balanced base-8 digits of q (|q| <= 128) as e2m1 codes, plane j in bits 4j..4j+3.
__device__ __forceinline__ uint32_t digit_codes(int q) {
    uint32_t out = 0;
    int x = q;
#pragma unroll
    for (int j = 0; j < kPlanes; ++j) {
        const int r = x & 7;
        const int d = x >= 0 ? (r <= 4 ? r : r - 8) : (r >= 4 ? r - 8 : r);
        x = (x - d) >> 3;
        const uint32_t m = d < 0 ? (uint32_t)(-d) : (uint32_t)d;                 // 0..4
        const uint32_t code = (d < 0 ? 8u : 0u) | (m <= 1u ? 2u * m : m + 2u);  // 0, 1.0, 2.0, 3.0, 4.0
        out |= code << (4 * j);
    }
    return out;
}

// Writes the digit planes of `codes` (npairs block pairs) into B: row n = 24h + 8j + l of pair p
// holds digit plane j of the four values of int lane l of block 2p + h; all other bytes stay
// zero.  Layout per stage (6 KB): [atom n / 8][pair in stage][8 rows][32 B], 32-byte swizzle.
// Threads t0 .. t0 + nt - 1 of the caller share the work.
__device__ void build_planes(const int8_t *codes, int npairs, uint8_t *sB, int t0, int nt) {
    for (int item = t0; item < npairs * 16; item += nt) {
        const int pr = item >> 4, h = (item >> 3) & 1, l = item & 7;
        const int e0 = 64 * pr + 32 * h + 4 * l;  // first element of the lane
        const uint32_t c4 = *reinterpret_cast<const uint32_t *>(codes + e0);
        uint32_t dg[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) dg[i] = digit_codes((int)(int8_t)(c4 >> (8 * i)));
        uint8_t *base = sB + (size_t)(pr >> 2) * kBStage + (pr & 3) * 256 + l * 32 + ((h ^ ((l >> 2) & 1)) << 4) + 2 * l;
#pragma unroll
        for (int j = 0; j < kPlanes; ++j) {
            uint32_t v = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) v |= ((dg[i] >> (4 * j)) & 15u) << (4 * i);
            *reinterpret_cast<uint16_t *>(base + (3 * h + j) * 1024) = (uint16_t)v;
        }
    }
}

__host__ __device__ inline size_t tc_smem_layout(int H, int I, size_t off[8]) {
    const int KM = H > I ? H : I;
    size_t o = 0;
    off[0] = o; o += (size_t)kAStages * kATile;  // A ring
    off[1] = o; o += (size_t)kBStages * kBStage;  // B digit planes
    off[2] = o; o += (size_t)2 * H * 4;          // router rows
    off[3] = o; o += (size_t)H * 4;              // residual stream h
    off[4] = o; o += (size_t)((KM + 15) & ~15);  // Q8_0 codes (x, then a job's activation)
    off[5] = o; o += (size_t)(KM / 32) * 4;      // their scales
    off[6] = o; o += 64 * 4;                     // up-row totals of a gate_up tile
    off[7] = o; o += 128 * 8 * 4;                // odd-chain lanes of a tile's rows
    return o;
}

struct TileSpan {
    int s, first, n;  // slot, first unit within the slot, units in the tile
};
__device__ __forceinline__ TileSpan tile_at(int u, int u_hi, int per_slot, int max_n) {
    TileSpan t;
    t.s = u / per_slot;
    t.first = u - t.s * per_slot;
    t.n = min(max_n, min(u_hi - u, per_slot - t.first));
    return t;
}

// The 24 result columns of this warp's chain for two block pairs (pair 0 at taddr, pair 1 at
// taddr + kDPair), loaded and waited for in one block so that no use can move above the wait.
// Volatile asm keeps its place among the barrier waits and tcgen05 fences; no memory clobber, so
// that shared-memory loads may overlap it.
__device__ __forceinline__ void tmem_ld_two_pairs(uint32_t taddr, uint32_t (&a)[24], uint32_t (&b)[24]) {
    asm volatile(
        "{\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%48];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%16, %17, %18, %19, %20, %21, %22, %23}, [%49];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39}, [%50];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%40, %41, %42, %43, %44, %45, %46, %47}, [%51];\n\t"
        "tcgen05.wait::ld.sync.aligned;\n\t}"
        : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]), "=r"(a[4]), "=r"(a[5]), "=r"(a[6]), "=r"(a[7]), "=r"(a[8]), "=r"(a[9]), "=r"(a[10]), "=r"(a[11]), "=r"(a[12]), "=r"(a[13]), "=r"(a[14]), "=r"(a[15]), "=r"(a[16]), "=r"(a[17]), "=r"(a[18]), "=r"(a[19]), "=r"(a[20]), "=r"(a[21]), "=r"(a[22]), "=r"(a[23]), "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3]), "=r"(b[4]), "=r"(b[5]), "=r"(b[6]), "=r"(b[7]), "=r"(b[8]), "=r"(b[9]), "=r"(b[10]), "=r"(b[11]), "=r"(b[12]), "=r"(b[13]), "=r"(b[14]), "=r"(b[15]), "=r"(b[16]), "=r"(b[17]), "=r"(b[18]), "=r"(b[19]), "=r"(b[20]), "=r"(b[21]), "=r"(b[22]), "=r"(b[23])
        : "r"(taddr), "r"(taddr + 16), "r"(taddr + kDPair), "r"(taddr + kDPair + 16)
        );
}

// One fp32 chain (block parity h) of one row over `npairs` block pairs, read stage by stage
// (4 pairs) from the TMEM ring: acc[l] = fma(d_b, L_l, acc[l]) over the blocks b = 2p + h.
// tcol: this warp's lanes and chain columns; ex: the row's exponent words of parity h in the
// tiled scale plane (quad qd at ex[32 qd], byte = pair in the quad), all loaded at the start so
// that one memory latency covers the tile; sc: the activation's block scales.  A warp with no
// row in the tile (live = false) still waits for and releases every ring stage, which keeps the
// ring's phases in step.
__device__ __forceinline__ void chain8(uint32_t tcol, uint64_t *dfull, uint64_t *dfree, uint32_t &gd, int npairs,
                                       const uint32_t *ex, const float *sc, int h, bool live, uint32_t *err,
                                       float (&acc)[8]) {
#pragma unroll
    for (int l = 0; l < 8; ++l) acc[l] = 0.0f;
    const int nq = (npairs + 3) / 4;
    uint32_t w[kBStages];
#pragma unroll
    for (int k = 0; k < kBStages; ++k) w[k] = live && k < nq ? __ldg(ex + 32 * k) : 0u;
#pragma unroll
    for (int qd = 0; qd < kBStages; ++qd) {
        if (qd < nq) {
            const uint32_t we = w[qd];
            const int ds = (int)(gd % kDStages);
            if ((threadIdx.x & 31) == 0) wait_tc(&dfull[ds], (gd / kDStages) & 1u, err);  // one poller per warp
            __syncwarp();
            tc::fence_after_sync();
            if (live) {
                float dq[4];  // block factors of the stage's pairs, ready before the loads land
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int pr = min(4 * qd + i, npairs - 1);
                    dq[i] = __fmul_rn(sc[2 * pr + h], e8m0_half((we >> (8 * i)) & 0xffu));
                }
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    uint32_t v[2][24];
                    tmem_ld_two_pairs(tcol + ds * 4 * kDPair + 2 * hf * kDPair, v[0], v[1]);
#pragma unroll
                    for (int i2 = 0; i2 < 2; ++i2) {
                        const int i = 2 * hf + i2, pr = 4 * qd + i;
                        if (pr < npairs) {
                            const float d = dq[i];
#pragma unroll
                            for (int l = 0; l < 8; ++l) {
                                const float L = __fadd_rn(__fadd_rn(__uint_as_float(v[i2][l]), __uint_as_float(v[i2][8 + l])),
                                                          __uint_as_float(v[i2][16 + l]));
                                acc[l] = __fmaf_rn(d, L, acc[l]);
                            }
                        }
                    }
                }
            }
            tc::fence_before_sync();
            __syncwarp();
            if ((threadIdx.x & 31) == 0) tc::mbar_arrive(&dfree[ds]);
            ++gd;
        }
    }
}

__global__ void __launch_bounds__(kTcThreads, 1) k_decode_tc(const __grid_constant__ DecodeParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ float inv_s;
    __shared__ float sel_w[kMaxEntriesTc];
    __shared__ int n_slots_s, slot_e[kMaxEntriesTc], slot_job[kMaxEntriesTc];
    __shared__ int ok_s, late_s;
    __shared__ __align__(8) uint64_t wbar, fin_bar, full_a[kAStages], empty_a[kAStages], dfull[kDStages], dfree[kDStages];
    __shared__ __align__(16) float wbias[2][4];
    __shared__ uint32_t tmem_s;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nC = gridDim.x, c = blockIdx.x;
    const int H = p.hidden, I = p.inter, E = p.experts, K = p.top_k;
    const int nb = H / 32, nbI = I / 32, H4 = H / 4;
    const int my_e = c < E ? (E - 1 - c) / nC + 1 : 0;  // router rows of this CTA (<= 2)
    size_t off[8];
    tc_smem_layout(H, I, off);
    uint8_t *sA = smem + off[0], *sB = smem + off[1];
    float *wrow = reinterpret_cast<float *>(smem + off[2]), *hs = reinterpret_cast<float *>(smem + off[3]);
    int8_t *xq = reinterpret_cast<int8_t *>(smem + off[4]);
    float *xqs = reinterpret_cast<float *>(smem + off[5]), *xch = reinterpret_cast<float *>(smem + off[6]);
    float *xacc = reinterpret_cast<float *>(smem + off[7]);
    unsigned target = 0;
    uint32_t wphase = 0;
    bool wpending = false;    // a router-row copy is in flight
    uint32_t ga = 0, gd = 0;  // weight stages / TMEM result stages this thread's role has passed

    if (tid == 0) {
        for (int s = 0; s < kAStages; ++s) {
            mbar_init(&full_a[s], 1);
            mbar_init(&empty_a[s], 1);
        }
        for (int s = 0; s < kDStages; ++s) {
            mbar_init(&dfull[s], 1);
            mbar_init(&dfree[s], kEpiWarps);
        }
        mbar_init(&wbar, 1);
        mbar_init(&fin_bar, 2);
        late_s = 0;
    }
    if (warp == 1) {
        tc::tmem_alloc(&tmem_s, kTmemCols);
        tc::tmem_relinquish();
    }
    for (int i = tid; i < kBStages * kBStage / 16; i += kTcThreads)
        reinterpret_cast<uint4 *>(sB)[i] = make_uint4(0u, 0u, 0u, 0u);
    if (p.x_dtype == UMSX_DTYPE_BF16) {
        const uint16_t *xb = static_cast<const uint16_t *>(p.x);
        for (int i = tid; i < H; i += kTcThreads) hs[i] = bf16_bits_to_f32(xb[i]);
    } else {
        const float *xf = static_cast<const float *>(p.x);
        for (int i = tid; i < H; i += kTcThreads) hs[i] = xf[i];
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = tmem_s;
    if (tid == 0 && my_e > 0)
        load_router_rows(p.layer[0].router_w, p.layer[0].router_b, c, nC, my_e, H, wrow, wbias, &wbar);
    wpending = my_e > 0;
    if (warp >= 4 && warp < 8) {
        // scale factors, every byte: A = 2^0 (8 columns); B column n at TMEM lane n % 32 and column
        // n / 32 of its region: 2 * 8^j for the digit plane j = (n % 24) / 8 of the column
        const uint32_t lf = (uint32_t)(32 * (warp - 4)) << 16;
        tmem_st4(tmem + lf + kSfCol, 0x7F7F7F7Fu);
        tmem_st4(tmem + lf + kSfCol + 4, 0x7F7F7F7Fu);
        const uint32_t j0 = (uint32_t)((lane % 24) / 8), j1 = (uint32_t)(((32 + lane) % 24) / 8);
        tmem_st2(tmem + lf + kSfCol + 8, (128u + 3u * j0) * 0x01010101u, (128u + 3u * j1) * 0x01010101u);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tsfa = tmem + kSfCol, tsfb = tmem + kSfCol + 8;

    bool alive = true;
    for (int l = 0; l < p.n_layers && alive; ++l) {
        const DecodeLayer &Ld = p.layer[l];
        // ---- R: fold, RMSNorm, logits (warps < my_e), x -> Q8_0 codes (the other warps) ----
        if (l > 0) {
            float4 *h4 = reinterpret_cast<float4 *>(hs);
            const float4 *y4 = reinterpret_cast<const float4 *>(p.y);
            for (int i = tid; i < H4; i += kTcThreads) {
                float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                for (int r0 = 0; r0 < K; r0 += 4) {  // rank order, four loads in flight
                    float4 yv[4];
#pragma unroll
                    for (int r = 0; r < 4; ++r)
                        if (r0 + r < K) yv[r] = __ldcg(y4 + (size_t)(r0 + r) * H4 + i);
#pragma unroll
                    for (int r = 0; r < 4; ++r)
                        if (r0 + r < K) {
                            const float wr = sel_w[r0 + r];
                            acc.x = __fadd_rn(acc.x, __fmul_rn(wr, yv[r].x));
                            acc.y = __fadd_rn(acc.y, __fmul_rn(wr, yv[r].y));
                            acc.z = __fadd_rn(acc.z, __fmul_rn(wr, yv[r].z));
                            acc.w = __fadd_rn(acc.w, __fmul_rn(wr, yv[r].w));
                        }
                }
                const float4 h = h4[i];
                h4[i] = p.residual ? make_float4(__fadd_rn(h.x, acc.x), __fadd_rn(h.y, acc.y), __fadd_rn(h.z, acc.z),
                                                 __fadd_rn(h.w, acc.w))
                                   : acc;
            }
        }
        __syncthreads();
        if (warp == 0) {
            float inv = 1.0f;  // x * 1 is exact: without RMSNorm the products below leave h unchanged
            if (p.rmsnorm) {
                float a = 0.0f;
                for (int k0 = lane; k0 < H; k0 += 32 * 8) {
                    float v[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) v[j] = k0 + 32 * j < H ? hs[k0 + 32 * j] : 0.0f;
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        if (k0 + 32 * j < H) a = __fmaf_rn(v[j], v[j], a);
                }
                const float ss = warp_tree_sum(a);
                inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)H), p.eps)));
            }
            if (lane == 0) inv_s = inv;
        }
        __syncthreads();
        const float inv = inv_s;
        if (warp < my_e) {
            if (!mbar_wait_bounded(&wbar, wphase, kWaitLimitCycles) && lane == 0) late_s = 1;
            const int e = c + nC * warp;
            const float *wr = wrow + (size_t)warp * H;
            float acc = 0.0f;
            for (int k0 = lane; k0 < H; k0 += 32 * 8) {
                float w[8], x[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    w[i] = k0 + 32 * i < H ? wr[k0 + 32 * i] : 0.0f;
                    x[i] = k0 + 32 * i < H ? hs[k0 + 32 * i] : 0.0f;
                }
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    if (k0 + 32 * i < H) acc = __fmaf_rn(w[i], __fmul_rn(x[i], inv), acc);
            }
            float lg = warp_tree_sum(acc);
            if (Ld.router_b) lg = __fadd_rn(lg, wbias[warp][e & 3]);
            if (lane == 0) __stcg(p.logits + e, lg);
        } else {
            for (int b = warp - my_e; b < nb; b += kTcWarps - my_e) {
                const float v = __fmul_rn(hs[b * 32 + lane], inv);
                const float amax = warp_max(fabsf(v));
                const float qinv = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
                xq[b * 32 + lane] = (int8_t)q8_code(v, qinv);
                if (lane == 0) xqs[b] = f16_bits_to_f32(f32_to_f16_bits(__fdiv_rn(amax, 127.0f)));
            }
        }
        if (my_e > 0) wphase ^= 1u;
        wpending = false;
        __syncthreads();
        if (late_s) {  // the router rows never arrived: report, let the copy land, stop
            if (tid == 0) {
                atomicOr(p.err, 4u);
                mbar_wait_bounded(&wbar, wphase ^ 1u, kWaitLimitCycles);
            }
            alive = false;
            break;
        }
        target += nC;
        if (!grid_sync_tc(p.bar, target, p.err, &ok_s)) { alive = false; break; }

        // ---- S: selection and slots (every CTA) ---------------------------------------
        if (warp == 0) {
            int sel;
            float w;
            select_topk<8>(p.logits, E, K, p.routing, p.routed_scale, lane, sel, w);
            const bool has = lane < K;
            if (has && (sel < 0 || sel >= E)) {  // cannot happen (selection always picks a valid expert)
                atomicOr(p.err, 8u);
                sel = 0;
            }
            int less = 0;
            for (int j = 0; j < K; ++j) less += __shfl_sync(kFull, sel, j) < sel;
            if (has) {
                sel_w[lane] = w;
                slot_e[less] = sel;  // one token: K distinct experts, slot = rank of the expert id
                slot_job[less] = lane;
            }
            if (lane == 0) n_slots_s = K;
            if (c == 0 && l == p.n_layers - 1 && p.ids_out && has) {
                p.ids_out[lane] = sel;
                p.w_out[lane] = w;
            }
        } else {
            // meanwhile the gate_up digit planes of x (B is idle: the previous layer's MMAs all
            // completed before the last grid barrier)
            build_planes(xq, H / 64, sB, tid - 32, kTcThreads - 32);
            tc::fence_proxy_async();
        }
        __syncthreads();
        const int n_slots = n_slots_s;

        // ---- G then D --------------------------------------------------------------------
        for (int ph = 0; ph < 2 && alive; ++ph) {
            const bool gu = ph == 0;
            const int rows = gu ? 2 * I : H, Kd = gu ? H : I, npairs = Kd / 64, nst = (npairs + 3) / 4;
            const int per_slot = gu ? I / 32 : H / 16, max_n = gu ? kGuTileUnits : kDnTileGroups;
            const int U = n_slots * per_slot;
            const int u_lo = (int)((long long)c * U / nC), u_hi = (int)((long long)(c + 1) * U / nC);
            const uint8_t *scales = gu ? Ld.gu_scales : Ld.dn_scales;
            const int nrg = rows / 16;
            int built = gu ? -2 : -1;  // job whose digit planes B holds (gate_up: x)
            for (int u = u_lo; u < u_hi;) {
                const TileSpan t = tile_at(u, u_hi, per_slot, max_n);
                u += t.n;
                const int e = slot_e[t.s], job = slot_job[t.s];
                if (!gu && job != built) {
                    // down: the digit planes of this job's activation (every earlier MMA is done:
                    // the epilogue warps consumed all its results before this barrier)
                    __syncthreads();
                    for (int i = tid; i < I / 16; i += kTcThreads)
                        reinterpret_cast<uint4 *>(xq)[i] =
                            __ldcg(reinterpret_cast<const uint4 *>(p.act_q8 + (size_t)job * I) + i);
                    for (int i = tid; i < nbI; i += kTcThreads) xqs[i] = __ldcg(p.act_q8_sc + (size_t)job * nbI + i);
                    __syncthreads();
                    build_planes(xq, npairs, sB, tid, kTcThreads);
                    tc::fence_proxy_async();
                    __syncthreads();
                    built = job;
                }
                if (warp == 0) {
                    if (lane == 0) {
                        // per stage: the tile's gate groups and its up groups (gate_up), or its row groups
                        // (down), each a contiguous run of 2 KB pre-swizzled tiles
                        const uint8_t *wt = gu ? Ld.gu_tc : Ld.dn_tc;
                        const int g0 = gu ? 2 * t.first : t.first, ng = gu ? 2 * t.n : t.n;
                        const uint32_t bytes = (uint32_t)ng * kBoxBytes;
                        for (int st = 0; st < nst; ++st) {
                            const int slot = (int)(ga % kAStages);
                            if (!wait_tc(&empty_a[slot], ((ga / kAStages) & 1u) ^ 1u, p.err)) break;
                            mbar_expect_tx(&full_a[slot], gu ? 2 * bytes : bytes);
                            uint8_t *dst = sA + (size_t)slot * kATile;
                            const uint8_t *src = wt + (((size_t)e * nst + st) * nrg + g0) * kBoxBytes;
                            bulk_g2s(dst, src, bytes, &full_a[slot]);
                            if (gu) bulk_g2s(dst + 64 * 128, src + (size_t)(I / 16) * kBoxBytes, bytes, &full_a[slot]);
                            ++ga;
                        }
                    }
                } else if (warp == 1 || warp == 2) {
                    if (lane == 0) {  // two issuers, alternate stages (stage g uses TMEM ring stage g % 2)
                        for (int st = 0; st < nst; ++st) {
                            if ((int)(ga & 1u) != warp - 1) {
                                ++ga;
                                ++gd;
                                continue;
                            }
                            const int slot = (int)(ga % kAStages);
                            if (!wait_tc(&full_a[slot], (ga / kAStages) & 1u, p.err)) break;
                            tc::fence_after_sync();
                            const int np = min(4, npairs - 4 * st);
                            const int ds = (int)(gd % kDStages);
                            if (!wait_tc(&dfree[ds], ((gd / kDStages) & 1u) ^ 1u, p.err)) break;
                            tc::fence_after_sync();
                            const uint64_t da = smem_desc_sw32(sA + (size_t)slot * kATile, 1024);
                            const uint64_t db = smem_desc_sw32(sB + (size_t)st * kBStage, 1024);
                            for (int q = 0; q < np; ++q)  // block pair q: 256 bytes further in A and B
                                mma_mxf4(tmem + ds * 4 * kDPair + q * kDPair, da + 16 * q, db + 16 * q, kIdescMxf4, 0u, tsfa,
                                         tsfb);
                            tc::mma_commit(&dfull[ds]);
                            tc::mma_commit(&empty_a[slot]);
                            ++ga;
                            ++gd;
                        }
                    }
                } else if (warp >= 4 && warp < 4 + kEpiWarps) {
                    const int ew = warp - 4, g = ew & 3, h = ew >> 2, r = 32 * g + lane;
                    const uint32_t tcol = tmem + ((uint32_t)(32 * g) << 16) + 24 * h;
                    // gate_up: the rows of lane group g are unit (g & 1) of the tile, gate (g < 2) or up;
                    // down: rows 32 g .. 32 g + 31 of the tile
                    const bool live = gu ? (g & 1) < t.n : 32 * g < 16 * t.n;
                    const bool valid = gu ? live : r < 16 * t.n;
                    const int mrow = gu ? (r < 64 ? t.first * 32 + r : I + t.first * 32 + (r - 64))
                                        : min(t.first * 16 + r, rows - 1);
                    const uint32_t *ex = reinterpret_cast<const uint32_t *>(
                                             scales + ((size_t)e * nrg + (mrow >> 4)) * (size_t)nst * 128) +
                                         16 * h + (mrow & 15);
                    float acc[8];
                    chain8(tcol, dfull, dfree, gd, npairs, ex, xqs, h, live, p.err, acc);
                    // lanes = even + odd chain, then the reference's horizontal order
                    if (h == 1)
#pragma unroll
                        for (int k = 0; k < 8; ++k) xacc[r * 8 + k] = acc[k];
                    asm volatile("bar.sync 1, 256;" ::: "memory");
                    float tot = 0.0f;
                    if (h == 0) {
                        float s8[8];
#pragma unroll
                        for (int k = 0; k < 8; ++k) s8[k] = __fadd_rn(acc[k], xacc[r * 8 + k]);
                        const float t0 = __fadd_rn(s8[4], s8[0]), t1 = __fadd_rn(s8[5], s8[1]);
                        const float t2 = __fadd_rn(s8[6], s8[2]), t3 = __fadd_rn(s8[7], s8[3]);
                        tot = __fadd_rn(__fadd_rn(t0, t2), __fadd_rn(t1, t3));
                    }
                    asm volatile("bar.sync 1, 256;" ::: "memory");
                    if (h == 0 && gu) {
                        const float v =
                            live ? __fadd_rn(tot, Ld.gu_bias ? __ldg(Ld.gu_bias + (size_t)e * rows + mrow) : 0.0f) : 0.0f;
                        if (g >= 2) xch[r - 64] = v;
                        asm volatile("bar.sync 2, 128;" ::: "memory");
                        if (g < 2 && live) {
                            const float uv = xch[r];
                            const float a = p.activation == UMSX_ACT_SWIGLU_OAI ? swiglu_oai(v, uv, p.alpha, p.limit)
                                                                                : silu_mul(v, uv);
                            const float amax = warp_max(fabsf(a));
                            const float qinv = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
                            const int blk = t.first + g;  // this warp's 32 activations are one Q8_0 block
                            p.act_q8[(size_t)job * I + blk * 32 + lane] = (int8_t)q8_code(a, qinv);
                            if (lane == 0)
                                p.act_q8_sc[(size_t)job * nbI + blk] =
                                    f16_bits_to_f32(f32_to_f16_bits(__fdiv_rn(amax, 127.0f)));
                        }
                        asm volatile("bar.sync 2, 128;" ::: "memory");
                    } else if (h == 0 && valid) {
                        float y = tot;
                        if (Ld.dn_bias) y = __fadd_rn(y, __ldg(Ld.dn_bias + (size_t)e * H + mrow));
                        __stcg(p.y + (size_t)job * H + mrow, y);
                    }
                }
            }
            if (gu && tid == 0 && my_e > 0 && l + 1 < p.n_layers)
                load_router_rows(p.layer[l + 1].router_w, p.layer[l + 1].router_b, c, nC, my_e, H, wrow, wbias, &wbar);
            if (gu) wpending = my_e > 0 && l + 1 < p.n_layers;
            target += nC;
            if (!grid_sync_tc(p.bar, target, p.err, &ok_s)) { alive = false; break; }
        }
    }
    if (alive) {
        // final fold: each CTA writes its share of the output
        const int lo = (int)((long long)c * H4 / nC), hi = (int)((long long)(c + 1) * H4 / nC);
        const float4 *y4 = reinterpret_cast<const float4 *>(p.y);
        for (int i = lo + tid; i < hi; i += kTcThreads) {
            float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            for (int r = 0; r < K; ++r) {
                const float4 yv = __ldcg(y4 + (size_t)r * H4 + i);
                const float wr = sel_w[r];
                acc.x = __fadd_rn(acc.x, __fmul_rn(wr, yv.x));
                acc.y = __fadd_rn(acc.y, __fmul_rn(wr, yv.y));
                acc.z = __fadd_rn(acc.z, __fmul_rn(wr, yv.z));
                acc.w = __fadd_rn(acc.w, __fmul_rn(wr, yv.w));
            }
            const float4 h = reinterpret_cast<const float4 *>(hs)[i];
            reinterpret_cast<float4 *>(p.out)[i] =
                p.residual ? make_float4(__fadd_rn(h.x, acc.x), __fadd_rn(h.y, acc.y), __fadd_rn(h.z, acc.z),
                                         __fadd_rn(h.w, acc.w))
                           : acc;
        }
    }
    // drain: copies and MMAs still in flight (only after an error) land before the CTA exits
    if (tid == 0) {
        for (uint32_t g = ga > (uint32_t)kAStages ? ga - kAStages : 0u; g < ga; ++g)
            mbar_wait_bounded(&full_a[g % kAStages], (g / kAStages) & 1u, kWaitLimitCycles);
        if (wpending) mbar_wait_bounded(&wbar, wphase, kWaitLimitCycles);
    }
    if (tid == 32 || tid == 64) {  // both MMA issuers
        tc::mma_commit(&fin_bar);
        mbar_wait_bounded(&fin_bar, 0u, kWaitLimitCycles);
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace

bool decode_tc_supported(int tokens, int hidden, int inter, int experts, int top_k) {
    return tokens == 1 && top_k >= 1 && top_k <= kMaxEntriesTc && experts >= top_k && experts <= 256 &&
           hidden % 64 == 0 && inter % 64 == 0 && hidden <= kMaxKTc && inter <= kMaxKTc;
}

int launch_decode_tc(const DecodeParams &p, cudaStream_t s) {
    if (!decode_tc_supported(p.tokens, p.hidden, p.inter, p.experts, p.top_k) || !p.act_q8 || !p.act_q8_sc ||
        p.n_layers < 1 || p.n_layers > kDecodeMaxLayers)
        return -1;
    size_t off[8];
    const size_t dyn = 1024 + tc_smem_layout(p.hidden, p.inter, off);
    if (cudaFuncSetAttribute(k_decode_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn) != cudaSuccess)
        return -1;
    int dev = 0, sms = 0, per_sm = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return -1;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode_tc, kTcThreads, dyn) != cudaSuccess ||
        per_sm < 1)
        return -1;
    if (p.experts > 2 * sms) return -1;  // two router rows per CTA
    if (cudaMemsetAsync(p.bar, 0, sizeof(unsigned), s) != cudaSuccess) return -1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(sms);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = dyn;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, k_decode_tc, p) != cudaSuccess) return -1;
    return 1;
}

}  // namespace umsx
