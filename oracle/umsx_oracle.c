/*
 * umsx CPU oracle -- TEST INFRASTRUCTURE ONLY (see umsx_oracle.h for the
 * provenance of every function and who may call this library).
 *
 * Build: gcc -O2 -std=c11 -ffp-contract=off -fopenmp -fPIC -shared (oracle/Makefile).
 * -ffp-contract=off matters: every multiply-add below that is not written as
 * fmaf() must round twice, as the reference's C++ (CMakeLists.txt:112-119) does.
 */
#include "umsx_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static inline uint32_t fbits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bitsf(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* ------------------------------------------------------------------------ */
/* fp16 / bf16 conversions (IEEE round-to-nearest-even), e8m0 half scale      */
/* ------------------------------------------------------------------------ */

float orc_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000) << 16;
    const uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ff;
    if (exp == 0) {
        /* zero or subnormal: man * 2^-24 is exact in fp32 */
        float v = (float)man * 0x1p-24f;
        return sign ? -v : v;
    }
    if (exp == 31) return bitsf(sign | 0x7f800000u | (man << 13));
    return bitsf(sign | ((exp + 112) << 23) | (man << 13));
}

uint16_t orc_f32_to_f16(float f) {
    const uint32_t x = fbits(f);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000);
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return sign | (ax > 0x7f800000u ? 0x7e00 : 0x7c00);
    const int e = (int)(ax >> 23) - 127;
    if (e >= 16) return sign | 0x7c00;
    if (e >= -14) {
        const uint32_t m = ax & 0x7fffff;
        uint32_t h = ((uint32_t)(e + 15) << 10) | (m >> 13);
        const uint32_t rem = m & 0x1fff;
        if (rem > 0x1000 || (rem == 0x1000 && (h & 1))) h++;
        return sign | (uint16_t)h; /* a carry into exponent 31 correctly yields inf */
    }
    if (e < -25) return sign;
    const uint32_t m = (ax & 0x7fffff) | 0x800000;
    const int s = -(e + 1); /* 14..24 bits dropped; unit is 2^-24 */
    uint32_t h = m >> s;
    const uint32_t rem = m & ((1u << s) - 1), half = 1u << (s - 1);
    if (rem > half || (rem == half && (h & 1))) h++;
    return sign | (uint16_t)h;
}

float orc_bf16_to_f32(uint16_t h) { return bitsf((uint32_t)h << 16); }

uint16_t orc_f32_to_bf16(float f) {
    uint32_t u = fbits(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7fffu + ((u >> 16) & 1);
    return (uint16_t)(u >> 16);
}

/* 2^(e-128): the MXFP4 code table holds doubled e2m1 values, so the block
 * scale is halved.  e < 2 lands in the fp32 subnormal range
 * (tools/trace/cpu_mxfp4_vnni.cpp:22-24, tools/engine/quantized_cuda.cu:159-163). */
float orc_e8m0_half(uint8_t e) {
    return bitsf(e < 2 ? (0x00200000u << e) : ((uint32_t)(e - 1) << 23));
}

/* ------------------------------------------------------------------------ */
/* exp: Cody-Waite reduction by ln 2 (hi/lo split) + degree-7 Taylor          */
/* polynomial in Horner form, scaled by 2^n in two exact steps.  Shared       */
/* bit-for-bit with the CUDA kernels (same fp32 operations, same order).      */
/* ------------------------------------------------------------------------ */

float orc_exp(float x) {
    if (x != x) return x;
    if (x > 88.72283935546875f) return INFINITY;
    if (x < -103.97208404541015625f) return 0.0f;
    const float n = rintf(x * 0x1.715476p+0f);
    float r = fmaf(-n, 0x1.62e4p-1f, x);
    r = fmaf(-n, 0x1.7f7d1cp-20f, r);
    float p = 0x1.a01a02p-13f;
    p = fmaf(p, r, 0x1.6c16c2p-10f);
    p = fmaf(p, r, 0x1.111112p-7f);
    p = fmaf(p, r, 0x1.555556p-5f);
    p = fmaf(p, r, 0x1.555556p-3f);
    p = fmaf(p, r, 0x1p-1f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int ni = (int)n, n1 = ni / 2, n2 = ni - n1;
    const float s1 = bitsf((uint32_t)(n1 + 127) << 23), s2 = bitsf((uint32_t)(n2 + 127) << 23);
    return (p * s1) * s2;
}

/* SwiGLU-OAI, tools/engine/native_cpu.cpp:123-127 (std::min / std::clamp semantics). */
float orc_swiglu_oai(float g, float u, float alpha, float limit) {
    g = (limit < g) ? limit : g;
    u = (u < -limit) ? -limit : ((limit < u) ? limit : u);
    const float t = alpha * (-g);
    const float den = 1.0f + orc_exp(t);
    const float q = g / den;
    return q * (u + 1.0f);
}

/* SiLU-gated: silu(g) * u (ggml_vec_swiglu_f32; tools/engine/f32_experts.cpp:73). */
float orc_silu_mul(float g, float u) {
    const float den = 1.0f + orc_exp(-g);
    return (g / den) * u;
}

/* ------------------------------------------------------------------------ */
/* Q8_0 activation quantization (x86 rule; parity patch :41-44, :96)          */
/* ------------------------------------------------------------------------ */

void orc_quantize_q8_0(const float *x, uint8_t *out, int n) {
    for (int b = 0; b < n / ORC_QK; ++b) {
        const float *v = x + b * ORC_QK;
        uint8_t *blk = out + (size_t)b * ORC_Q8_0_BYTES;
        float amax = 0.0f;
        for (int j = 0; j < ORC_QK; ++j) {
            const float a = fabsf(v[j]);
            if (a > amax) amax = a;
        }
        const float d = amax / 127.0f;
        const uint16_t dh = orc_f32_to_f16(d);
        blk[0] = (uint8_t)(dh & 0xff);
        blk[1] = (uint8_t)(dh >> 8);
        const float id = amax != 0.0f ? 127.0f / amax : 0.0f;
        for (int j = 0; j < ORC_QK; ++j) {
            float q = rintf(v[j] * id);
            if (q > 127.0f) q = 127.0f;
            if (q < -128.0f) q = -128.0f;
            blk[2 + j] = (uint8_t)(int8_t)(int)q;
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Dots                                                                       */
/* ------------------------------------------------------------------------ */

static const int kMxfp4Codes[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};

/* VPSIGNB product |w| * sign(w)(a), where negating -128 wraps to -128. */
static inline int signed_product(int w, int a) {
    if (w == 0) return 0;
    const int mag = w < 0 ? -w : w;
    const int sa = w > 0 ? a : (a == -128 ? -128 : -a);
    return mag * sa;
}

static inline float horizontal(const float lanes[8]) {
    /* (l0+l4)+(l2+l6) + (l1+l5)+(l3+l7), exact_packed_cpu.h:72-76, cpu_mxfp4_vnni.cpp:64-67 */
    const float t0 = lanes[4] + lanes[0], t1 = lanes[5] + lanes[1];
    const float t2 = lanes[6] + lanes[2], t3 = lanes[7] + lanes[3];
    return (t0 + t2) + (t1 + t3);
}

float orc_dot_mxfp4_q8_0(int n, const uint8_t *w, const uint8_t *a) {
    float even[8] = {0}, odd[8] = {0};
    const int nb = n / ORC_QK;
    for (int b = 0; b < nb; ++b) {
        const uint8_t *wb = w + (size_t)b * ORC_MXFP4_BYTES;
        const uint8_t *ab = a + (size_t)b * ORC_Q8_0_BYTES;
        const float d = orc_f16_to_f32((uint16_t)(ab[0] | (ab[1] << 8))) * orc_e8m0_half(wb[0]);
        float *acc = (b & 1) ? odd : even;
        for (int l = 0; l < 8; ++l) {
            int sum = 0;
            for (int j = 0; j < 4; ++j) {
                const int idx = 4 * l + j;
                const int code = idx < 16 ? (wb[1 + idx] & 15) : (wb[1 + idx - 16] >> 4);
                sum += signed_product(kMxfp4Codes[code], (int)(int8_t)ab[2 + idx]);
            }
            acc[l] = fmaf(d, (float)sum, acc[l]);
        }
    }
    float lanes[8];
    for (int l = 0; l < 8; ++l) lanes[l] = even[l] + odd[l];
    return horizontal(lanes);
}

/* Q8_0 x Q8_0: 8 lanes of 4 bytes, one FMA chain per lane, same horizontal order.
 * x = weight, y = activation; |x| is taken as an unsigned byte (|-128| = 128). */
float orc_dot_q8_0_q8_0(int n, const uint8_t *w, const uint8_t *a) {
    float acc[8] = {0};
    const int nb = n / ORC_QK;
    for (int b = 0; b < nb; ++b) {
        const uint8_t *wb = w + (size_t)b * ORC_Q8_0_BYTES;
        const uint8_t *ab = a + (size_t)b * ORC_Q8_0_BYTES;
        const float d = orc_f16_to_f32((uint16_t)(wb[0] | (wb[1] << 8))) *
                        orc_f16_to_f32((uint16_t)(ab[0] | (ab[1] << 8)));
        for (int l = 0; l < 8; ++l) {
            int sum = 0;
            for (int j = 0; j < 4; ++j) {
                const int idx = 4 * l + j;
                const int x = (int)(int8_t)wb[2 + idx], y = (int)(int8_t)ab[2 + idx];
                const int mag = x < 0 ? -x : x;
                const int sy = x > 0 ? y : (x == 0 ? 0 : (y == -128 ? -128 : -y));
                sum += mag * sy;
            }
            acc[l] = fmaf(d, (float)sum, acc[l]);
        }
    }
    return horizontal(acc);
}

void orc_dequant_mxfp4(const uint8_t *blocks, float *out, int64_t n) {
    for (int64_t b = 0; b < n / ORC_QK; ++b) {
        const uint8_t *blk = blocks + b * ORC_MXFP4_BYTES;
        const float s = orc_e8m0_half(blk[0]);
        for (int j = 0; j < ORC_QK; ++j) {
            const int code = j < 16 ? (blk[1 + j] & 15) : (blk[1 + j - 16] >> 4);
            out[b * ORC_QK + j] = (float)kMxfp4Codes[code] * s;
        }
    }
}

void orc_dequant_q8_0(const uint8_t *blocks, float *out, int64_t n) {
    for (int64_t b = 0; b < n / ORC_QK; ++b) {
        const uint8_t *blk = blocks + b * ORC_Q8_0_BYTES;
        const float d = orc_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
        for (int j = 0; j < ORC_QK; ++j) out[b * ORC_QK + j] = (float)(int8_t)blk[2 + j] * d;
    }
}

static inline size_t block_bytes(int quant) {
    return quant == ORC_QUANT_MXFP4 ? ORC_MXFP4_BYTES : ORC_Q8_0_BYTES;
}

static inline float row_dot(int quant, int n, const uint8_t *w, const uint8_t *a) {
    return quant == ORC_QUANT_MXFP4 ? orc_dot_mxfp4_q8_0(n, w, a) : orc_dot_q8_0_q8_0(n, w, a);
}

void orc_gemv(int quant, int n, int rows, const uint8_t *W, const uint8_t *a, float *out, int nthreads) {
    const size_t row_bytes = (size_t)(n / ORC_QK) * block_bytes(quant);
    if (nthreads < 1) nthreads = 1;
#pragma omp parallel for schedule(static) num_threads(nthreads)
    for (int r = 0; r < rows; ++r) out[r] = row_dot(quant, n, W + (size_t)r * row_bytes, a);
}

/* ------------------------------------------------------------------------ */
/* Router                                                                     */
/* ------------------------------------------------------------------------ */

/* 32 strided chains (chain c covers k = c, c+32, ...), then the xor butterfly
 * v[c] = v[c] + v[c^s] for s = 16, 8, 4, 2, 1 -- the order one warp computes. */
static float tree32(float v[32]) {
    for (int s = 16; s >= 1; s >>= 1) {
        float nv[32];
        for (int c = 0; c < 32; ++c) nv[c] = v[c] + v[c ^ s];
        memcpy(v, nv, sizeof(nv));
    }
    return v[0];
}

float orc_logit(const float *w_row, const float *x, int h) {
    float v[32] = {0};
    for (int c = 0; c < 32; ++c)
        for (int k = c; k < h; k += 32) v[c] = fmaf(w_row[k], x[k], v[c]);
    return tree32(v);
}

float orc_sum_strided(const float *p, int n) {
    float v[32] = {0};
    for (int c = 0; c < 32; ++c)
        for (int k = c; k < n; k += 32) v[c] = v[c] + p[k];
    return tree32(v);
}

/* k largest, value descending, lower index wins ties (topk-tie-probe.cpp:111-113). */
static void topk(const float *v, int n, int k, int32_t *sel) {
    unsigned char taken[1024];
    memset(taken, 0, (size_t)n);
    for (int r = 0; r < k; ++r) {
        int best = -1;
        for (int e = 0; e < n; ++e) {
            if (taken[e]) continue;
            if (best < 0 || v[e] > v[best]) best = e;
        }
        taken[best] = 1;
        sel[r] = best;
    }
}

void orc_route(int routing, int experts, int top_k, int hidden, float routed_scale,
               const float *router_w, const float *router_b, const float *x, int tokens,
               int32_t *ids, float *weights, float *logits_out) {
    float logits[1024], probs[1024];
    for (int t = 0; t < tokens; ++t) {
        const float *xt = x + (size_t)t * hidden;
        for (int e = 0; e < experts; ++e) {
            float l = orc_logit(router_w + (size_t)e * hidden, xt, hidden);
            if (router_b) l = l + router_b[e];
            if (logits_out) logits_out[(size_t)t * experts + e] = l;
            logits[e] = l != l ? -INFINITY : l;  /* NaN ranks lowest: every pick is a valid expert */
        }
        int32_t *sel = ids + (size_t)t * top_k;
        float *wt = weights + (size_t)t * top_k;
        if (routing == ORC_ROUTE_TOPK_SOFTMAX) {
            topk(logits, experts, top_k, sel);
            const float m = logits[sel[0]];
            float ex[64], sum = 0.0f;
            for (int r = 0; r < top_k; ++r) {
                ex[r] = orc_exp(logits[sel[r]] - m);
                sum = sum + ex[r];
            }
            for (int r = 0; r < top_k; ++r) wt[r] = ex[r] / sum;
        } else {
            float m = logits[0];
            for (int e = 1; e < experts; ++e) if (logits[e] > m) m = logits[e];
            for (int e = 0; e < experts; ++e) probs[e] = orc_exp(logits[e] - m);
            const float sum = orc_sum_strided(probs, experts);
            for (int e = 0; e < experts; ++e) probs[e] = probs[e] / sum;
            topk(probs, experts, top_k, sel);
            if (routing == ORC_ROUTE_SOFTMAX_TOPK_NORM) {
                float s = 0.0f;
                for (int r = 0; r < top_k; ++r) s = s + probs[sel[r]];
                for (int r = 0; r < top_k; ++r) wt[r] = probs[sel[r]] / s;
            } else {
                for (int r = 0; r < top_k; ++r) wt[r] = probs[sel[r]] * routed_scale;
            }
        }
    }
}

void orc_rmsnorm(const float *x, float *out, int n, float eps) {
    float v[32] = {0};
    for (int c = 0; c < 32; ++c)
        for (int k = c; k < n; k += 32) v[c] = fmaf(x[k], x[k], v[c]);
    const float ss = tree32(v);
    const float mean = ss / (float)n;
    const float inv = 1.0f / sqrtf(mean + eps);
    for (int k = 0; k < n; ++k) out[k] = x[k] * inv;
}

/* ------------------------------------------------------------------------ */
/* MoE layer                                                                  */
/* ------------------------------------------------------------------------ */

int orc_moe_experts(const orc_desc *d, const orc_weights *w, const float *x, int tokens,
                    const int32_t *ids, const float *weights, float *out, uint8_t *act_q8, float *y,
                    int nthreads) {
    const int H = d->hidden, I = d->intermediate, K = d->top_k, E = d->experts;
    if (H % 64 || I % 64 || tokens <= 0 || K <= 0) return 1;
    const size_t bb = block_bytes(d->quant);
    const size_t rowH = (size_t)(H / ORC_QK) * bb, rowI = (size_t)(I / ORC_QK) * bb;
    const size_t q8H = (size_t)(H / ORC_QK) * ORC_Q8_0_BYTES, q8I = (size_t)(I / ORC_QK) * ORC_Q8_0_BYTES;
    const int jobs = tokens * K;
    if (nthreads < 1) nthreads = 1;
    uint8_t *xq = (uint8_t *)malloc((size_t)tokens * q8H);
    float *gu = (float *)malloc((size_t)jobs * 2 * I * sizeof(float));
    uint8_t *aq = act_q8 ? act_q8 : (uint8_t *)malloc((size_t)jobs * q8I);
    float *yy = y ? y : (float *)malloc((size_t)jobs * H * sizeof(float));
    float *act = (float *)malloc((size_t)jobs * I * sizeof(float));
    for (int t = 0; t < tokens; ++t) orc_quantize_q8_0(x + (size_t)t * H, xq + (size_t)t * q8H, H);

#pragma omp parallel for collapse(2) schedule(static) num_threads(nthreads)
    for (int j = 0; j < jobs; ++j) {
        for (int r = 0; r < 2 * I; ++r) {
            const int e = ids[j];
            if (e < 0 || e >= E) { gu[(size_t)j * 2 * I + r] = 0.0f; continue; }
            const uint8_t *row;
            if (d->fused_gate_up) row = w->gate_up + ((size_t)e * 2 * I + r) * rowH;
            else row = r < I ? w->gate + ((size_t)e * I + r) * rowH : w->up + ((size_t)e * I + (r - I)) * rowH;
            float v = row_dot(d->quant, H, row, xq + (size_t)(j / K) * q8H);
            if (d->has_bias && w->gate_up_bias) v = v + orc_bf16_to_f32(w->gate_up_bias[(size_t)e * 2 * I + r]);
            gu[(size_t)j * 2 * I + r] = v;
        }
    }
    for (int j = 0; j < jobs; ++j) {
        const float *g = gu + (size_t)j * 2 * I, *u = g + I;
        float *a = act + (size_t)j * I;
        for (int i = 0; i < I; ++i)
            a[i] = d->activation == ORC_ACT_SWIGLU_OAI ? orc_swiglu_oai(g[i], u[i], d->swiglu_alpha, d->swiglu_limit)
                                                       : orc_silu_mul(g[i], u[i]);
        orc_quantize_q8_0(a, aq + (size_t)j * q8I, I);
    }
#pragma omp parallel for collapse(2) schedule(static) num_threads(nthreads)
    for (int j = 0; j < jobs; ++j) {
        for (int h = 0; h < H; ++h) {
            const int e = ids[j];
            if (e < 0 || e >= E) { yy[(size_t)j * H + h] = 0.0f; continue; }
            float v = row_dot(d->quant, I, w->down + ((size_t)e * H + h) * rowI, aq + (size_t)j * q8I);
            if (d->has_bias && w->down_bias) v = v + orc_bf16_to_f32(w->down_bias[(size_t)e * H + h]);
            yy[(size_t)j * H + h] = v;
        }
    }
    if (out) {
#pragma omp parallel for schedule(static) num_threads(nthreads)
        for (int t = 0; t < tokens; ++t) {
            for (int h = 0; h < H; ++h) {
                float acc = 0.0f;
                for (int r = 0; r < K; ++r) {
                    const float p = weights[(size_t)t * K + r] * yy[((size_t)t * K + r) * H + h];
                    acc = acc + p;
                }
                out[(size_t)t * H + h] = acc;
            }
        }
    }
    free(xq); free(gu); free(act);
    if (!act_q8) free(aq);
    if (!y) free(yy);
    return 0;
}

int orc_moe_layer(const orc_desc *d, const orc_weights *w, const float *x, int tokens, float *out,
                  int32_t *ids, float *weights, int32_t *counts, uint8_t *act_q8, float *y, int nthreads) {
    const int K = d->top_k, E = d->experts;
    if (E > 1024 || K > 64 || K > E) return 1;
    int32_t *sel = ids ? ids : (int32_t *)malloc((size_t)tokens * K * sizeof(int32_t));
    float *wt = weights ? weights : (float *)malloc((size_t)tokens * K * sizeof(float));
    orc_route(d->routing, E, K, d->hidden, d->routed_scale, w->router_w, w->router_b, x, tokens, sel, wt, NULL);
    if (counts) {
        memset(counts, 0, (size_t)E * sizeof(int32_t));
        for (int j = 0; j < tokens * K; ++j) counts[sel[j]]++;
    }
    const int rc = orc_moe_experts(d, w, x, tokens, sel, wt, out, act_q8, y, nthreads);
    if (!ids) free(sel);
    if (!weights) free(wt);
    return rc;
}

/* ------------------------------------------------------------------------ */
/* Deterministic synthetic generator: splitmix64 finaliser over               */
/* (seed, stream, index).  The CUDA generator performs the identical integer  */
/* and fp32 steps, so a weight generated on the device equals the oracle's.   */
/* ------------------------------------------------------------------------ */

static inline uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t orc_rng(uint64_t seed, uint64_t stream, uint64_t index) {
    return mix64(mix64(seed ^ (stream * 0xD6E8FEB86659FD93ull)) + index);
}

void orc_gen_mxfp4(uint64_t seed, uint64_t stream, uint64_t first_block, uint64_t nblocks,
                   int e_lo, int e_span, uint8_t *out) {
    for (uint64_t i = 0; i < nblocks; ++i) {
        const uint64_t b = first_block + i;
        const uint64_t r0 = orc_rng(seed, stream, 3 * b), r1 = orc_rng(seed, stream, 3 * b + 1),
                       r2 = orc_rng(seed, stream, 3 * b + 2);
        uint8_t *blk = out + i * ORC_MXFP4_BYTES;
        blk[0] = (uint8_t)(e_lo + (int)((uint32_t)(r0 >> 32) % (uint32_t)e_span));
        for (int j = 0; j < 8; ++j) {
            blk[1 + j] = (uint8_t)(r1 >> (8 * j));
            blk[9 + j] = (uint8_t)(r2 >> (8 * j));
        }
    }
}

void orc_gen_q8_0(uint64_t seed, uint64_t stream, uint64_t first_block, uint64_t nblocks, uint8_t *out) {
    for (uint64_t i = 0; i < nblocks; ++i) {
        const uint64_t b = first_block + i;
        uint8_t *blk = out + i * ORC_Q8_0_BYTES;
        const uint64_t r0 = orc_rng(seed, stream, 9 * b);
        const float f = (float)(uint32_t)(r0 >> 40) * 0x1.f212d8p-34f + 0x1.a36e2ep-14f;
        const uint16_t h = orc_f32_to_f16(f);
        blk[0] = (uint8_t)(h & 0xff);
        blk[1] = (uint8_t)(h >> 8);
        for (int q = 0; q < 8; ++q) {
            const uint64_t r = orc_rng(seed, stream, 9 * b + 1 + q);
            for (int c = 0; c < 4; ++c) {
                const uint32_t chunk = (uint32_t)(r >> (16 * c)) & 0xffffu;
                blk[2 + 4 * q + c] = (uint8_t)(int8_t)((int)(chunk % 255u) - 127);
            }
        }
    }
}

static inline float gen_normal(uint64_t seed, uint64_t stream, uint64_t idx, float scale) {
    uint32_t s = 0;
    for (int i = 0; i < 4; ++i) s += (uint32_t)(orc_rng(seed, stream, 4 * idx + i) >> 40);
    return (float)((int32_t)s - (1 << 25)) * scale;
}

void orc_gen_normal_f32(uint64_t seed, uint64_t stream, uint64_t first, uint64_t n, float scale, float *out) {
    for (uint64_t i = 0; i < n; ++i) out[i] = gen_normal(seed, stream, first + i, scale);
}

void orc_gen_normal_bf16(uint64_t seed, uint64_t stream, uint64_t first, uint64_t n, float scale, uint16_t *out) {
    for (uint64_t i = 0; i < n; ++i) out[i] = orc_f32_to_bf16(gen_normal(seed, stream, first + i, scale));
}

/* Sum of four U[0, 2^24) draws has mean 2^25 and sd 2^24 / sqrt(3). */
float orc_normal_scale(double sigma) { return (float)(sigma * sqrt(3.0) / 16777216.0); }
