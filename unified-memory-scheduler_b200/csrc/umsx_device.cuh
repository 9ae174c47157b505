// Device helpers shared by the umsx kernels (sm_100a).
//
// Every floating-point step that the CPU oracle must reproduce bit for bit is
// written with an explicit-rounding intrinsic (__fmul_rn, __fadd_rn, __fmaf_rn,
// __fdiv_rn), so nvcc's default FMA contraction cannot change it.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace umsx {

constexpr unsigned kFull = 0xffffffffu;

// ---- byte/integer primitives ------------------------------------------------

// prmt.b32 in its generic mode: selector nibble bits 0-2 pick one of the eight
// bytes of {b, a}; bit 3 replicates the picked byte's sign bit instead.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// sum of four unsigned(a) x signed(b) byte products plus c.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) { return __dp4a((int)a, (int)b, c); }

// Byte-wise two's-complement negation that wraps -128 to -128 (VPSIGNB's behaviour).
__device__ __forceinline__ uint32_t neg8x4(uint32_t a) { return __vsub4(0u, a); }

// MXFP4 magnitudes {0,1,2,3,4,6,8,12} (doubled e2m1) as a prmt table.
constexpr uint32_t kMagLo = 0x03020100u, kMagHi = 0x0C080604u;

// 2^(e-128), subnormal for e < 2 (tools/engine/quantized_cuda.cu:159-163).
__device__ __forceinline__ float e8m0_half(uint32_t e) {
    return __uint_as_float(e < 2 ? (0x00200000u << e) : ((e - 1u) << 23));
}

__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) { return __half2float(__ushort_as_half((unsigned short)h)); }
__device__ __forceinline__ uint32_t f32_to_f16_bits(float f) { return __half_as_ushort(__float2half_rn(f)); }
__device__ __forceinline__ float bf16_bits_to_f32(uint32_t h) { return __uint_as_float(h << 16); }
__device__ __forceinline__ uint32_t f32_to_bf16_bits(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (u >> 16) | 0x40u;
    u += 0x7fffu + ((u >> 16) & 1u);
    return u >> 16;
}

// ---- the shared exp --------------------------------------------------------
// Cody-Waite reduction by ln 2 split into a short high part and a low part, a
// degree-7 Taylor polynomial in Horner form, and scaling by 2^n in two exact
// steps.  The oracle (orc_exp) performs the same fp32 operations in the same
// order, so both produce identical bits.
__device__ __forceinline__ float exp_shared(float x) {
    if (x != x) return x;
    if (x > 88.72283935546875f) return __uint_as_float(0x7f800000u);
    if (x < -103.97208404541015625f) return 0.0f;
    const float n = rintf(__fmul_rn(x, 0x1.715476p+0f));
    float r = __fmaf_rn(-n, 0x1.62e4p-1f, x);
    r = __fmaf_rn(-n, 0x1.7f7d1cp-20f, r);
    float p = 0x1.a01a02p-13f;
    p = __fmaf_rn(p, r, 0x1.6c16c2p-10f);
    p = __fmaf_rn(p, r, 0x1.111112p-7f);
    p = __fmaf_rn(p, r, 0x1.555556p-5f);
    p = __fmaf_rn(p, r, 0x1.555556p-3f);
    p = __fmaf_rn(p, r, 0x1p-1f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int ni = (int)n, n1 = ni / 2, n2 = ni - n1;
    const float s1 = __uint_as_float((uint32_t)(n1 + 127) << 23), s2 = __uint_as_float((uint32_t)(n2 + 127) << 23);
    return __fmul_rn(__fmul_rn(p, s1), s2);
}

// SwiGLU-OAI (tools/engine/native_cpu.cpp:123-127): std::min / std::clamp semantics.
__device__ __forceinline__ float swiglu_oai(float g, float u, float alpha, float limit) {
    g = (limit < g) ? limit : g;
    u = (u < -limit) ? -limit : ((limit < u) ? limit : u);
    const float den = __fadd_rn(1.0f, exp_shared(__fmul_rn(alpha, -g)));
    return __fmul_rn(__fdiv_rn(g, den), __fadd_rn(u, 1.0f));
}

// silu(g) * u (tools/engine/f32_experts.cpp:73).
__device__ __forceinline__ float silu_mul(float g, float u) {
    const float den = __fadd_rn(1.0f, exp_shared(-g));
    return __fmul_rn(__fdiv_rn(g, den), u);
}

// Records a non-finite combined output in the status word (the reference rejects those,
// tools/engine/expert_dispatch.cpp:84-85); a no-op for finite values or a null word.
__device__ __forceinline__ void flag_nonfinite(float v, uint32_t *err) {
    if ((__float_as_uint(v) & 0x7f800000u) == 0x7f800000u && err) atomicOr(err, 16u);
}
__device__ __forceinline__ void flag_nonfinite4(float4 v, uint32_t *err) {
    flag_nonfinite(v.x, err);
    flag_nonfinite(v.y, err);
    flag_nonfinite(v.z, err);
    flag_nonfinite(v.w, err);
}

// ---- warp reductions --------------------------------------------------------

// The oracle's tree32: v[c] = v[c] + v[c^s] for s = 16..1 (fp add is commutative,
// so every lane ends with the same bits).
__device__ __forceinline__ float warp_tree_sum(float v) {
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) v = __fadd_rn(v, __shfl_xor_sync(kFull, v, s));
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, s));
    return v;
}

// Q8_0 code for one value with the x86 rule (parity patch :41-44): rn_even(x * rn(127/amax)).
__device__ __forceinline__ int q8_code(float v, float inv) {
    int q = __float2int_rn(__fmul_rn(v, inv));
    return q > 127 ? 127 : (q < -128 ? -128 : q);
}

// Byte offset of element i (0..31) of a Q8 block inside the "lane-pair" order the
// GEMV kernels use: [p = (i%16)/4][half = i/16][i%4].
__device__ __forceinline__ int lane_pair_offset(int i) { return ((i & 15) >> 2) * 8 + (i >> 4) * 4 + (i & 3); }

// ---- bulk copies into shared memory, completed on an mbarrier ----------------

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// cp.async.bulk global -> shared; src, dst 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Waits for the phase with the given parity, giving up after `limit_cycles`
// (clock64); returns false on time-out so the caller can report and stop.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, long long limit_cycles) {
    const long long t0 = clock64();
    while (!mbar_test(bar, parity))
        if (clock64() - t0 > limit_cycles) return false;
    return true;
}

// ---- counter-based generator (identical to the oracle's orc_rng) -------------

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ uint64_t rng(uint64_t seed, uint64_t stream, uint64_t index) {
    return mix64(mix64(seed ^ (stream * 0xD6E8FEB86659FD93ull)) + index);
}

__device__ __forceinline__ float gen_normal(uint64_t seed, uint64_t stream, uint64_t idx, float scale) {
    uint32_t s = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) s += (uint32_t)(rng(seed, stream, 4 * idx + i) >> 40);
    return __fmul_rn((float)((int32_t)s - (1 << 25)), scale);
}

}  // namespace umsx
