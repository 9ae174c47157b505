/*
 * C entry points around the reference's own CPU kernels, compiled from the
 * reference sources where they lie (oracle/Makefile, target `ref`):
 *   tools/trace/cpu_mxfp4_vnni.cpp  -> ggml_vec_dot_mxfp4_q8_0 (AVX-512 VNNI)
 *   tools/trace/exact_packed_cpu.h  -> exact_packed_cpu::{gemv, gemm, pack_activation}
 * TEST INFRASTRUCTURE ONLY: used to pin the C oracle bit-for-bit and as the
 * timed CPU baseline (`bench.py --impl reference`).  Output goes to oracle/_ref/.
 *
 * The layer driver ref_layer_* runs the MoE layer with the reference's exact
 * packed MXFP4 GEMV for every expert product (weights repacked to
 * block_mxfp4x8 once, as ggml's CPU repack does), and the oracle's quantizer,
 * router, activation and rank-order combine around it.
 */
#include "exact_packed_cpu.h"

extern "C" {
#include "umsx_oracle.h"
}

#include <cstdlib>
#include <cstring>
#include <exception>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

extern "C" void ggml_vec_dot_mxfp4_q8_0(int n, float *result, size_t, const void *vx, size_t,
                                        const void *vy, size_t, int nrc);

namespace {

void quantize_adapter(const float *input, void *output, int64_t k) {
    orc_quantize_q8_0(input, static_cast<uint8_t *>(output), static_cast<int>(k));
}

/* Eight raw rows -> block_mxfp4x8, the interleave the reference test uses
 * (tests/test_exact_packed_cpu.cpp:19-35): e[row], then 8-byte halves. */
void pack_rows(const uint8_t *raw, int n, int rows, block_mxfp4x8 *out) {
    const int blocks = n / 32;
    for (int column = 0; column < rows; column += 8) {
        for (int block = 0; block < blocks; ++block) {
            auto &dst = out[column / 8 * blocks + block];
            for (int row = 0; row < 8; ++row) {
                const uint8_t *src = raw + ((size_t)(column + row) * blocks + block) * 17;
                dst.e[row] = src[0];
                for (int part = 0; part < 2; ++part) std::memcpy(dst.qs + (part * 8 + row) * 8, src + 1 + part * 8, 8);
            }
        }
    }
}

struct RefLayer {
    orc_desc desc;
    std::vector<float> router_w, router_b;
    std::vector<block_mxfp4x8> gate_up, down; /* per expert, contiguous */
    std::vector<uint16_t> gate_up_bias, down_bias;
};

} // namespace

extern "C" {

int ref_cpu_supported(void) {
    return __builtin_cpu_supports("avx512vnni") && __builtin_cpu_supports("avx512bw") &&
           __builtin_cpu_supports("avx512vl") && __builtin_cpu_supports("f16c");
}

void ref_vec_dot_mxfp4_q8_0(int n, float *s, const void *vx, const void *vy) {
    ggml_vec_dot_mxfp4_q8_0(n, s, 0, vx, 0, vy, 0, 1);
}

void ref_pack_mxfp4x8(const uint8_t *raw, int n, int rows, uint8_t *out) {
    pack_rows(raw, n, rows, reinterpret_cast<block_mxfp4x8 *>(out));
}

int ref_packed_gemv(int n, float *out, const void *packed_w, const void *act_q8, int nc) {
    try {
        exact_packed_cpu::gemv(n, out, 0, packed_w, act_q8, 1, nc);
        return 0;
    } catch (const std::exception &) {
        return 1;
    }
}

int ref_pack_activation(const float *x, void *out, int64_t k) {
    try {
        exact_packed_cpu::pack_activation(x, out, k, quantize_adapter);
        return 0;
    } catch (const std::exception &) {
        return 1;
    }
}

int ref_packed_gemm(int n, float *out, size_t stride, const void *packed_w, const void *packed_act, int nr, int nc) {
    try {
        exact_packed_cpu::gemm(n, out, stride, packed_w, packed_act, nr, nc);
        return 0;
    } catch (const std::exception &) {
        return 1;
    }
}

/* MXFP4, fused gate_up only (the configs that use MXFP4). */
void *ref_layer_create(const orc_desc *d, const orc_weights *w) {
    if (d->quant != ORC_QUANT_MXFP4 || !d->fused_gate_up || d->hidden % 64 || d->intermediate % 64) return nullptr;
    auto *layer = new RefLayer();
    layer->desc = *d;
    const int H = d->hidden, I = d->intermediate, E = d->experts;
    layer->router_w.assign(w->router_w, w->router_w + (size_t)E * H);
    if (w->router_b) layer->router_b.assign(w->router_b, w->router_b + E);
    layer->gate_up.resize((size_t)E * (2 * I / 8) * (H / 32));
    layer->down.resize((size_t)E * (H / 8) * (I / 32));
    for (int e = 0; e < E; ++e) {
        pack_rows(w->gate_up + (size_t)e * 2 * I * (H / 32) * 17, H, 2 * I,
                  layer->gate_up.data() + (size_t)e * (2 * I / 8) * (H / 32));
        pack_rows(w->down + (size_t)e * H * (I / 32) * 17, I, H, layer->down.data() + (size_t)e * (H / 8) * (I / 32));
    }
    if (d->has_bias && w->gate_up_bias) layer->gate_up_bias.assign(w->gate_up_bias, w->gate_up_bias + (size_t)E * 2 * I);
    if (d->has_bias && w->down_bias) layer->down_bias.assign(w->down_bias, w->down_bias + (size_t)E * H);
    return layer;
}

void ref_layer_destroy(void *handle) { delete static_cast<RefLayer *>(handle); }

int ref_layer_forward(void *handle, const float *x, int tokens, float *out, int nthreads) {
    auto *L = static_cast<RefLayer *>(handle);
    const orc_desc &d = L->desc;
    const int H = d.hidden, I = d.intermediate, K = d.top_k;
    const int jobs = tokens * K;
    const size_t q8H = (size_t)(H / 32) * 34, q8I = (size_t)(I / 32) * 34;
    std::vector<int32_t> ids((size_t)jobs);
    std::vector<float> weights((size_t)jobs);
    orc_route(d.routing, d.experts, K, H, d.routed_scale, L->router_w.data(),
              L->router_b.empty() ? nullptr : L->router_b.data(), x, tokens, ids.data(), weights.data(), nullptr);
    std::vector<uint8_t> xq((size_t)tokens * q8H), aq((size_t)jobs * q8I);
    std::vector<float> gu((size_t)jobs * 2 * I), y((size_t)jobs * H);
    for (int t = 0; t < tokens; ++t) orc_quantize_q8_0(x + (size_t)t * H, xq.data() + (size_t)t * q8H, H);
    const int tilesGU = 2 * I / 8, tilesD = H / 8;
    if (nthreads < 1) nthreads = 1;
#pragma omp parallel for collapse(2) schedule(static) num_threads(nthreads)
    for (int j = 0; j < jobs; ++j) {
        for (int tile = 0; tile < tilesGU; ++tile) {
            const int e = ids[(size_t)j];
            const auto *W = L->gate_up.data() + ((size_t)e * tilesGU + tile) * (H / 32);
            exact_packed_cpu::gemv(H, gu.data() + (size_t)j * 2 * I + tile * 8, 0, W, xq.data() + (size_t)(j / K) * q8H, 1, 8);
        }
    }
    for (int j = 0; j < jobs; ++j) {
        const int e = ids[(size_t)j];
        float *g = gu.data() + (size_t)j * 2 * I;
        if (!L->gate_up_bias.empty())
            for (int r = 0; r < 2 * I; ++r) g[r] = g[r] + orc_bf16_to_f32(L->gate_up_bias[(size_t)e * 2 * I + r]);
        std::vector<float> a((size_t)I);
        for (int i = 0; i < I; ++i)
            a[(size_t)i] = d.activation == ORC_ACT_SWIGLU_OAI ? orc_swiglu_oai(g[i], g[I + i], d.swiglu_alpha, d.swiglu_limit)
                                                              : orc_silu_mul(g[i], g[I + i]);
        orc_quantize_q8_0(a.data(), aq.data() + (size_t)j * q8I, I);
    }
#pragma omp parallel for collapse(2) schedule(static) num_threads(nthreads)
    for (int j = 0; j < jobs; ++j) {
        for (int tile = 0; tile < tilesD; ++tile) {
            const int e = ids[(size_t)j];
            const auto *W = L->down.data() + ((size_t)e * tilesD + tile) * (I / 32);
            exact_packed_cpu::gemv(I, y.data() + (size_t)j * H + tile * 8, 0, W, aq.data() + (size_t)j * q8I, 1, 8);
        }
    }
    for (int j = 0; j < jobs && !L->down_bias.empty(); ++j) {
        const int e = ids[(size_t)j];
        for (int h = 0; h < H; ++h) y[(size_t)j * H + h] = y[(size_t)j * H + h] + orc_bf16_to_f32(L->down_bias[(size_t)e * H + h]);
    }
    for (int t = 0; t < tokens; ++t) {
        for (int h = 0; h < H; ++h) {
            float acc = 0.0f;
            for (int r = 0; r < K; ++r) acc = acc + weights[(size_t)t * K + r] * y[((size_t)t * K + r) * H + h];
            out[(size_t)t * H + h] = acc;
        }
    }
    return 0;
}

} // extern "C"
