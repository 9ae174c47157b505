/*
 * umsx CPU oracle -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's exact packed CPU MoE-layer path
 * (appatalks/unified-memory-scheduler, "VRAMBridge").  Only tests/, the
 * smoke() check in __graft_entry__.py and bench.py's cpu_baseline /
 * --impl reference legs may load this library, and only as the checker or the
 * timed CPU baseline.  The product path (libumsx.so) never links or calls it.
 *
 * What each function restates (paths are inside the reference project):
 *   - MXFP4 x Q8_0 dot: tools/trace/cpu_mxfp4_vnni.cpp:22-68 and
 *     tools/trace/exact_packed_cpu.h:14-77 (8 int lanes of 4 elements, even/odd
 *     block FMA chains, horizontal order ((l0+l4)+(l2+l6))+((l1+l5)+(l3+l7))),
 *     VPSIGNB -128 semantics (tools/engine/quantized_cuda.cu:145-163).
 *   - Q8_0 activation quantizer: rule stated in
 *     third_party/patches/llama-b11669-mxfp4-q8-parity-experimental.patch:41-44,96
 *     (d = fp16_rn(amax/127), q = rn_even(x * rn(127/amax))).
 *   - Q8_0 x Q8_0 dot: the reference has no restatement (ggml is not vendored);
 *     restated from ggml's published 8-lane VNNI algorithm (one FMA chain per
 *     lane, same horizontal order).  Parity for this dot is UNPINNED.
 *   - FFN sequence, biases, activations: tools/engine/native_cpu.cpp:106-166,
 *     tools/engine/f32_experts.cpp:34-99 (SwiGLU-OAI at :68-71, SiLU at :73).
 *   - Weighted combine in rank order from 0.0f, no contraction:
 *     tools/engine/expert_dispatch.cpp:77-87 (test: tests/test_expert_dispatch.cpp:65-73).
 *   - Top-k tie rule (value desc, lower index wins): tools/trace/topk-tie-probe.cpp:111-113.
 *   - Router modes (gpt-oss / qwen3 / deepseek): BASELINE configs; the router
 *     code is upstream llama.cpp (absent), so the order of the logit reduction,
 *     the exp and the softmax sums are defined HERE and shared bit-for-bit with
 *     the CUDA kernels.  Parity of those pieces is UNPINNED against ggml.
 *
 * Pinned: the MXFP4 x Q8_0 dot and the exact packed GEMV/GEMM are checked
 * bit-for-bit against the reference's own sources compiled here (oracle/Makefile
 * builds tools/trace/cpu_mxfp4_vnni.cpp and tools/trace/exact_packed_cpu.h into
 * oracle/_ref/), on the reference test's seeds and edge cases.
 */
#ifndef UMSX_ORACLE_H
#define UMSX_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml block sizes: block_mxfp4 = {uint8 e; uint8 qs[16]}, block_q8_0 = {fp16 d; int8 qs[32]} */
#define ORC_QK 32
#define ORC_MXFP4_BYTES 17
#define ORC_Q8_0_BYTES 34
#define ORC_QUANT_Q8_0 8   /* ggml type ids */
#define ORC_QUANT_MXFP4 39

#define ORC_ROUTE_TOPK_SOFTMAX 0      /* gpt-oss: top-k of logits, softmax over the k */
#define ORC_ROUTE_SOFTMAX_TOPK_NORM 1 /* qwen3: softmax over E, top-k, renormalise    */
#define ORC_ROUTE_SOFTMAX_TOPK 2      /* deepseek: softmax over E, top-k, x scale     */

#define ORC_ACT_SILU 0
#define ORC_ACT_SWIGLU_OAI 1

/* ---- scalar primitives ---- */
float orc_f16_to_f32(uint16_t h);
uint16_t orc_f32_to_f16(float f);
float orc_bf16_to_f32(uint16_t h);
uint16_t orc_f32_to_bf16(float f);
float orc_e8m0_half(uint8_t e);
float orc_exp(float x);
float orc_swiglu_oai(float g, float u, float alpha, float limit);
float orc_silu_mul(float g, float u);

/* ---- quantized rows ---- */
void orc_quantize_q8_0(const float *x, uint8_t *out, int n);
float orc_dot_mxfp4_q8_0(int n, const uint8_t *w, const uint8_t *a);
float orc_dot_q8_0_q8_0(int n, const uint8_t *w, const uint8_t *a);
void orc_dequant_mxfp4(const uint8_t *blocks, float *out, int64_t n);
void orc_dequant_q8_0(const uint8_t *blocks, float *out, int64_t n);
/* out[r] = dot(W row r, a) for r in [0, rows); W is [rows][n/32] ggml blocks. */
void orc_gemv(int quant, int n, int rows, const uint8_t *W, const uint8_t *a, float *out, int nthreads);

/* ---- router ---- */
float orc_logit(const float *w_row, const float *x, int h);
float orc_sum_strided(const float *v, int n);
void orc_route(int routing, int experts, int top_k, int hidden, float routed_scale,
               const float *router_w, const float *router_b, const float *x, int tokens,
               int32_t *ids, float *weights, float *logits);

/* ---- MoE layer ---- */
typedef struct {
    int hidden, intermediate, experts, top_k;
    int quant, routing, activation, fused_gate_up, has_bias;
    float swiglu_alpha, swiglu_limit, routed_scale;
} orc_desc;

typedef struct {
    const float *router_w;      /* [E][H] */
    const float *router_b;      /* [E] or NULL */
    const uint8_t *gate_up;     /* fused: [E][2I][H/32] blocks (gate rows first) */
    const uint8_t *gate;        /* separate: [E][I][H/32] */
    const uint8_t *up;          /* separate: [E][I][H/32] */
    const uint8_t *down;        /* [E][H][I/32] */
    const uint16_t *gate_up_bias; /* bf16 [E][2I] (gate then up) or NULL */
    const uint16_t *down_bias;    /* bf16 [E][H] or NULL */
} orc_weights;

/* x fp32 [T][H] -> out fp32 [T][H].  Optional outputs may be NULL.
 * act_q8: [T*k][I/32*34] Q8_0 down inputs, y: [T*k][H] expert outputs. */
int orc_moe_layer(const orc_desc *d, const orc_weights *w, const float *x, int tokens, float *out,
                  int32_t *ids, float *weights, int32_t *counts, uint8_t *act_q8, float *y, int nthreads);

/* Experts only, for a given routing (used by the MUL_MAT_ID / ExpertPlan checks). */
int orc_moe_experts(const orc_desc *d, const orc_weights *w, const float *x, int tokens,
                    const int32_t *ids, const float *weights, float *out, uint8_t *act_q8, float *y,
                    int nthreads);

/* RMSNorm with unit weight, the sum of squares in the shared strided order. */
void orc_rmsnorm(const float *x, float *out, int n, float eps);

/* ---- deterministic synthetic generator (shared with the CUDA generator) ---- */
uint64_t orc_rng(uint64_t seed, uint64_t stream, uint64_t index);
void orc_gen_mxfp4(uint64_t seed, uint64_t stream, uint64_t first_block, uint64_t nblocks,
                   int e_lo, int e_span, uint8_t *out);
void orc_gen_q8_0(uint64_t seed, uint64_t stream, uint64_t first_block, uint64_t nblocks, uint8_t *out);
void orc_gen_normal_f32(uint64_t seed, uint64_t stream, uint64_t first, uint64_t n, float scale, float *out);
void orc_gen_normal_bf16(uint64_t seed, uint64_t stream, uint64_t first, uint64_t n, float scale, uint16_t *out);
float orc_normal_scale(double sigma);

#ifdef __cplusplus
}
#endif
#endif
