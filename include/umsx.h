/*
 * umsx -- B200-native (sm_100a) MoE-layer hot path behind a C ABI.
 *
 * The ABI carries plain pointers and sizes only.  Device pointers are
 * caller-owned; calls are stream-ordered and asynchronous unless the name
 * says `_host`.  No exception crosses it: every call returns a umsx_status and
 * umsx_last_error() holds the message of the last failure on this thread.
 * One handle per host thread, or the caller serialises (the reference guards
 * its CUDA runner with a mutex, tools/engine/quantized_cuda.cu:415).
 *
 * Reference interfaces replaced (paths inside appatalks/unified-memory-scheduler):
 *   ExpertPlan + ExpertRunner           tools/engine/expert_dispatch.hpp:21-48, .cpp:22-89
 *   Mxfp4NativeCudaDown                 tools/engine/quantized_cuda.hpp:38-50, .cu:367-453
 *   ggml MUL_MAT_ID -> ADD_ID -> SWIGLU_OAI -> MUL -> rank sum
 *                                       third_party/patches/llama-b11669-hybrid-experts.patch:1394-1683, :1911-1916
 *   router build_lora_mm(gate_inp, cur) hybrid patch :1361-1384 (softmax/top-k upstream)
 *   Q8_0 activation quantizer (x86 rule) llama-b11669-mxfp4-q8-parity-experimental.patch:41-44, :96
 */
#ifndef UMSX_H
#define UMSX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define UMSX_VERSION 1

typedef enum umsx_status {
    UMSX_OK = 0,
    UMSX_EINVAL = 1,        /* invalid argument / shape (std::invalid_argument in the reference) */
    UMSX_ENOTRESIDENT = 2,  /* expert out of range or not resident on this handle */
    UMSX_EOOM = 3,          /* allocation would violate the configured free-memory reserve */
    UMSX_ETIMEOUT = 4,      /* a bounded device wait (expert-parallel exchange) gave up */
    UMSX_EDEVICE = 5,       /* CUDA runtime error */
    UMSX_EUNSUPPORTED = 6,  /* shape or mode this build does not implement */
    UMSX_ENONFINITE = 7     /* non-finite result (the reference rejects these, expert_dispatch.cpp:14-18) */
} umsx_status;

/* A cudaStream_t, passed as void* so this header needs no CUDA include.  NULL = legacy default stream. */
typedef void *umsx_stream;

enum { UMSX_QUANT_Q8_0 = 8, UMSX_QUANT_MXFP4 = 39 }; /* ggml type ids */

enum {
    UMSX_ROUTE_TOPK_SOFTMAX = 0,      /* gpt-oss: top-k of logits, softmax over the k selected */
    UMSX_ROUTE_SOFTMAX_TOPK_NORM = 1, /* qwen3: softmax over all experts, top-k, renormalise */
    UMSX_ROUTE_SOFTMAX_TOPK = 2       /* deepseek: softmax over all experts, top-k, times routed_scale */
};

enum { UMSX_ACT_SILU = 0, UMSX_ACT_SWIGLU_OAI = 1 }; /* F32Activation, tools/engine/f32_experts.hpp:11 */

enum { UMSX_DTYPE_F32 = 0, UMSX_DTYPE_BF16 = 1 };

enum { UMSX_PROJ_GATE_UP = 0, UMSX_PROJ_GATE = 1, UMSX_PROJ_UP = 2, UMSX_PROJ_DOWN = 3 };

typedef struct umsx_moe_desc {
    int32_t hidden;          /* H: model width (K of gate/up, N of down); multiple of 64 */
    int32_t intermediate;    /* I: expert FFN width; multiple of 64 */
    int32_t experts;         /* E: routed experts in the whole layer */
    int32_t top_k;           /* k <= 32 */
    int32_t quant;           /* UMSX_QUANT_MXFP4 or UMSX_QUANT_Q8_0 */
    int32_t routing;         /* UMSX_ROUTE_* */
    int32_t activation;      /* UMSX_ACT_* */
    int32_t fused_gate_up;   /* 1: one [E][2I][H] matrix, gate rows [0,I) then up rows [I,2I) */
    int32_t has_bias;        /* expert biases present (bf16) */
    int32_t has_router_bias; /* router bias present (fp32) */
    float swiglu_alpha;      /* 1.702 for GPT-OSS */
    float swiglu_limit;      /* 7.0 for GPT-OSS */
    float routed_scale;      /* weight multiplier for UMSX_ROUTE_SOFTMAX_TOPK (1.0 for DeepSeek-V2-Lite) */
    int32_t max_tokens;      /* largest T a forward call passes; sizes the handle's workspace */
    int32_t ep_rank;         /* expert-parallel rank: experts [ep_rank*E/ep_world, ...) are resident */
    int32_t ep_world;        /* 1 for a single GPU; > 1: see umsx_moe_forward_jobs */
} umsx_moe_desc;

/* HOST pointers in ggml layouts (what a GGUF holds); create() copies the
 * resident experts to the device and repacks them.  NULL for absent tensors. */
typedef struct umsx_moe_weights {
    const float *router_w;         /* [E][H] fp32 */
    const float *router_b;         /* [E] fp32 */
    const void *gate_up;           /* fused: [E][2I][H/32] blocks */
    const void *gate;              /* separate: [E][I][H/32] blocks */
    const void *up;                /* separate: [E][I][H/32] blocks */
    const void *down;              /* [E][H][I/32] blocks */
    const uint16_t *gate_up_bias;  /* bf16 [E][2I]: gate bias then up bias */
    const uint16_t *down_bias;     /* bf16 [E][H] */
} umsx_moe_weights;

typedef struct umsx_moe umsx_moe;

/* Replaces Mxfp4NativeCudaDown(const LoadedExperts&, resident, device) (quantized_cuda.cu:377-407)
 * and the graph's expert tensors: uploads, repacks into the sm_100a tile layout, keeps
 * `reserve_bytes` of device memory free (the reference keeps 1 GiB, quantized_cuda.cu:18,25-30). */
umsx_status umsx_moe_create(const umsx_moe_desc *desc, const umsx_moe_weights *weights, int device,
                            size_t reserve_bytes, umsx_moe **out);

/* Same, with every tensor generated on the device from (seed, layer) by the
 * counter-based generator (router and bias normal sigmas as given). */
umsx_status umsx_moe_create_synthetic(const umsx_moe_desc *desc, uint64_t seed, uint32_t layer,
                                      float router_sigma, float router_bias_sigma, float bias_sigma,
                                      int device, size_t reserve_bytes, umsx_moe **out);

void umsx_moe_destroy(umsx_moe *moe);

/* Replaces the router of a resident layer from HOST buffers (router_w [E][H] fp32, router_b [E] fp32,
 * given exactly when desc.has_router_bias); synchronous.  The expert tensors stay as they are.  Used
 * for the load-skew configuration, whose router bias follows a Zipf law over the experts (no
 * counterpart in the reference, which loads its router with the model). */
umsx_status umsx_moe_set_router(umsx_moe *moe, const float *router_w, const float *router_b);

/* Residency bank policies: the reference's VRAMBRIDGE_HYBRID_POLICY "lfu" and "lru"
 * (hybrid patch :2384-2388). */
enum { UMSX_BANK_LFU = 0, UMSX_BANK_LRU = 1 };
#define UMSX_BANK_STATS 9

/* A layer whose experts do not all stay on the device.  Replaces the reference's hybrid expert cache
 * (llama_moe_cache, hybrid patch :2174-2294; admission :3086-3160; dispatch :3244-3266): every expert
 * is kept in pinned HOST memory (copied from `weights`, which the caller may free afterwards); the
 * device holds `slots` bank slots (1..E) plus min(E, max_tokens*k) transient slots.  Each
 * umsx_moe_forward / umsx_moe_forward_host call routes on the device, reads the top-k back (one
 * host synchronisation), lets the policy admit experts into the bank (one-token calls only, as the
 * reference; batches look up), uploads admitted experts into their slots and the remaining misses
 * into transient slots, and runs the same expert kernels as a resident layer: the output is
 * bit-identical to umsx_moe_create's layer on the same weights (the reference computes misses on
 * the CPU instead).  Policies:
 *   UMSX_BANK_LFU  demand counts capped at 15, halved every window (2..5 bank-fulls of demands); an
 *                  expert fills a free slot after 1 demand, replaces the least recently used resident
 *                  (not selected by this dispatch) after 6 demands and with a strictly higher count;
 *                  at most 4 admissions per dispatch;
 *   UMSX_BANK_LRU  a miss takes a free slot or the least recently used resident's slot.
 * ep_world must be 1.  Banked layers run through umsx_moe_forward(_host) only: stacks, EP stacks,
 * forward_jobs, mul_mat_id, expert_down_q8 and export_expert return UMSX_EUNSUPPORTED. */
umsx_status umsx_moe_create_banked(const umsx_moe_desc *desc, const umsx_moe_weights *weights, int slots,
                                   int policy, int device, size_t reserve_bytes, umsx_moe **out);

/* Counters of a banked layer (stats[UMSX_BANK_STATS], may be NULL): dispatches, demands (selected
 * experts), hits, misses, admissions, evictions, transient uploads, LFU halvings, bytes uploaded
 * (expert blocks).  slot_of_expert[E] (may be NULL): the bank slot of every expert, -1 if not
 * resident.  Host-side state: no device synchronisation. */
umsx_status umsx_moe_bank_stats(umsx_moe *moe, uint64_t *stats, int n, int32_t *slot_of_expert, int n_experts);

/* The bank policy alone, on the host (no device): runs n_dispatches dispatches of `selected`
 * (concatenated; counts[i] > 0 entries of a one-token dispatch in rank order, admission on;
 * counts[i] < 0 for -counts[i] distinct experts of a batch, lookup only) and writes each selected
 * expert's slot after its dispatch to slot_out (-1 = transient), and stats[UMSX_BANK_STATS]
 * (bytes uploaded 0).  Used to test the policy against a restatement of the reference's rules. */
umsx_status umsx_bank_simulate(int experts, int slots, int policy, int n_dispatches, const int32_t *counts,
                               const int32_t *selected, int32_t *slot_out, uint64_t *stats);

/* Whole layer, device buffers: out[T][H] = sum_r w[t,r] * expert(ids[t,r], x[t]) in rank order.
 * Replaces build_moe_ffn's expert branch + rank sum (hybrid patch :1394-1683, :1911-1916).
 * x is [T][H] fp32 or bf16 (x_dtype).  Optional ids/weights outputs may be NULL. */
umsx_status umsx_moe_forward(umsx_moe *moe, const void *x, int x_dtype, int tokens, float *out,
                             int32_t *ids, float *weights, umsx_stream stream);

/* Same with HOST buffers: copies in, runs, copies out, synchronises (the reference's
 * synchronous host-vector contract, quantized_cuda.cu:413-453). */
umsx_status umsx_moe_forward_host(umsx_moe *moe, const void *x, int x_dtype, int tokens, float *out,
                                  umsx_stream stream);

/* Expert parallelism, one rank's share of a layer (no counterpart in the reference, which runs
 * on one GPU): routes all `tokens` rows (the router is replicated on every rank), runs the
 * experts this handle holds (desc.ep_rank of desc.ep_world: experts [ep_rank*E/ep_world, ...))
 * for the (token, rank) jobs that chose them, and writes their outputs to y[t][r][:] (fp32
 * [T][k][H], expert bias included, 16-byte aligned device buffer); rows of jobs whose expert
 * lives on another rank are left untouched.  ids/weights [T][k] (may be NULL) as umsx_route.
 * The caller moves every row to the token's rank and combines there in rank order with
 * umsx_combine, which gives the single-GPU layer's bits (each row is computed by the same
 * kernels from the same inputs).  umsx_moe_forward and stacks refuse expert-parallel handles. */
umsx_status umsx_moe_forward_jobs(umsx_moe *moe, const void *x, int x_dtype, int tokens, int32_t *ids,
                                  float *weights, float *y, umsx_stream stream);

/* Status of the handle's earlier calls on `stream`: synchronises the stream, then reads and clears
 * the handle's device status word.  UMSX_ENONFINITE if a combined output (the layer's result) was
 * inf or NaN -- the reference rejects those (ExpertPlan, tools/engine/expert_dispatch.cpp:14-18,
 * :84-85) -- UMSX_ETIMEOUT if a bounded device wait gave up, else UMSX_OK.  The word is sticky
 * until read here or by a _host call, which return the same statuses. */
umsx_status umsx_moe_status(umsx_moe *moe, umsx_stream stream);

/* Router only: logits (fixed fp32 reduction order), softmax/top-k/renormalise per
 * desc.routing, ties to the lowest expert index (topk-tie-probe.cpp:111-113),
 * per-expert counts.  ids [T][k] int32, weights [T][k] fp32, counts [E] int32 (may be NULL). */
umsx_status umsx_route(umsx_moe *moe, const void *x, int x_dtype, int tokens, int32_t *ids, float *weights,
                       int32_t *counts, umsx_stream stream);

/* Mxfp4NativeCudaDown::execute(packed_q8, jobs) (quantized_cuda.cu:413-453), device buffers:
 * packed_q8 is [jobs][I/32] ggml block_q8_0 rows, experts[j] the job's expert id, out [jobs][H] fp32
 * including the down bias.  Bit-exact with the reference CPU vec_dot.  Non-resident or
 * out-of-range experts give UMSX_ENOTRESIDENT (checked on the host copy of `experts`,
 * so `experts` is a HOST pointer here, as the reference's job vector is). */
umsx_status umsx_expert_down_q8(umsx_moe *moe, const void *packed_q8, const int32_t *experts, int jobs,
                                float *out, umsx_stream stream);

/* ggml MUL_MAT_ID shape (hybrid patch :1394-1683): as = the handle's projection `proj`
 * ([K][N][E] in ggml order), b = [T][n_b][K] fp32 rows (n_b = 1 broadcasts one row per token,
 * else n_b = n_ids), ids = [T][n_ids] int32 (-1 = masked: that output row is zero,
 * hybrid patch :617-621), dst = [T][n_ids][N] fp32.  The activation is quantized to Q8_0 with
 * the x86 rule and the dot is the reference's exact one; no bias is added (ADD_ID is separate). */
umsx_status umsx_mul_mat_id(umsx_moe *moe, int proj, const float *b, int n_b, const int32_t *ids, int n_ids,
                            int tokens, float *dst, umsx_stream stream);

/* Weighted combine in rank order from 0.0f without contraction
 * (ExpertPlan::execute, expert_dispatch.cpp:77-87): out[t][i] = sum_r w[t][r] * y[t][r][i].
 * Handle-free and asynchronous, so it does not check its output for non-finite values (the
 * layer entry points do, see umsx_moe_status). */
umsx_status umsx_combine(const float *y, const float *weights, int tokens, int top_k, int width, float *out,
                         umsx_stream stream);

/* Copies expert `expert` of projection `proj` back out of the device tile layout into
 * ggml blocks (host buffer of `size` bytes); the round trip must reproduce the original
 * bytes (the reference's repack export hook, tests/test_masked_matmul.cpp). */
umsx_status umsx_moe_export_expert(umsx_moe *moe, int proj, int expert, void *host_out, size_t size);

/* A stack of MoE layers with the residual stream of a transformer block, attention
 * omitted: h <- h + MoE_l(RMSNorm(h)) for every layer l in order (RMSNorm with unit
 * weight, eps rms_eps; the norm is fused into each layer's router and the residual add
 * into its combine).  The layers must share device and shape; the stack owns one
 * workspace for up to max_tokens tokens.  With T <= 4 tokens and MXFP4 fused gate_up
 * layers (all experts resident) a forward is ONE persistent cooperative kernel on the
 * caller's stream; otherwise the stack replays the per-stage kernels as one CUDA graph
 * per token count, on a stream of its own ordered after / before the caller's stream.
 * Both give identical bits.
 * Replaces the per-layer ffn_norm -> build_moe_ffn -> residual sequence of the
 * llama.cpp graph the hybrid patch modifies (llama-b11669-hybrid-experts.patch:1355-1930). */
typedef struct umsx_stack umsx_stack;
umsx_status umsx_stack_create(umsx_moe *const *layers, int n_layers, int max_tokens, float rms_eps, umsx_stack **out);
/* A stack whose layers may differ in shape (same width and device), each optionally with shared
 * experts: shared[l] (NULL for none) is a one-expert top-1 handle holding the always-on shared FFN
 * (the reference graph's ffn_{gate,up,down}_shexp, several shared experts as one FFN of their summed
 * width), and layer l becomes h <- h + ((sum_r w_r y_r) + y_shared): the shared FFN's output is the
 * term after the k routed ones in the same rank-order combine, as the graph's ggml_add of the shared
 * branch to the routed sum.  A dense FFN (DeepSeek's layer 0) is a one-expert top-1 layer (its
 * softmax over one logit is exactly 1.0).  Such stacks run the per-stage kernels (graph replay). */
umsx_status umsx_stack_create_mixed(umsx_moe *const *layers, umsx_moe *const *shared, int n_layers, int max_tokens,
                                    float rms_eps, umsx_stack **out);
void umsx_stack_destroy(umsx_stack *stack);
/* x [T][H] (device, fp32 or bf16) -> out [T][H] fp32 final hidden state. */
umsx_status umsx_stack_forward(umsx_stack *stack, const void *x, int x_dtype, int tokens, float *out, umsx_stream stream);
/* Same with host buffers (pinned for overlap); copies in and out and synchronises. */
umsx_status umsx_stack_forward_host(umsx_stack *stack, const void *x, int x_dtype, int tokens, float *out,
                                    umsx_stream stream);
/* umsx_moe_status for a stack: every layer's combined output is checked. */
umsx_status umsx_stack_status(umsx_stack *stack, umsx_stream stream);
/* With timing on, each replay timestamps the router, gate_up, down and combine stage of every
 * layer; stage_times returns the four per-stage sums (ms) over the layers of the last replay. */
umsx_status umsx_stack_set_timing(umsx_stack *stack, int enable);
umsx_status umsx_stack_stage_times(umsx_stack *stack, float *ms, int n_stages);
/* Fault injection for failure-detection tests (no counterpart in the reference): the next
 * one-launch decode forward of the stack runs with CTA `cta` withholding its first grid-barrier
 * arrival and every grid-barrier wait bounded by wait_limit_cycles SM cycles, so the waits run out,
 * the kernel ends, and the call reports UMSX_ETIMEOUT (a _host call, or umsx_stack_status).  One
 * forward only; a CTA index beyond the grid injects nothing. */
umsx_status umsx_stack_inject_fault(umsx_stack *stack, int cta, int64_t wait_limit_cycles);

/* The router of umsx_route without a handle and without allocating anything (no counterpart
 * in the reference).  For callers that cannot call cudaMalloc: an operator inside a framework
 * that plans every buffer ahead and hands it only its own tensors, or a process whose device
 * memory budget is spent.  The caller passes device buffers: x [T][H] (fp32 or bf16, 16-byte
 * aligned), router_w [E][H] fp32, router_b [E] fp32 or NULL, and receives ids [T][k] int32,
 * weights [T][k] fp32 and, if counts is not NULL, counts [E] int32; results equal umsx_route's.
 * The kernel's scratch (logits, completion counters, dispatch lists, quantized x) is a fixed
 * 512 KiB array inside this library that every GPU loading it holds until the process exits;
 * limits: T <= 64, E <= 256, k <= min(8, E), H a multiple of 64 up to 4096 (UMSX_EINVAL
 * beyond).  It runs on the calling thread's current device; the first call on a device looks
 * up the array's device address, so make that first call before any stream capture; a
 * cudaDeviceReset (or anything else that destroys the device's primary context) invalidates that
 * address, so a process that resets a device must not call this entry point on it again.  All calls
 * on a device share the array: calls that overlap on the GPU (other streams, other threads)
 * race and must be serialised by the caller.  Errors read back through umsx_last_error(). */
umsx_status umsx_route_static(const void *x, int x_dtype, int tokens, const float *router_w, const float *router_b,
                              int hidden, int experts, int top_k, int routing, float routed_scale, int32_t *ids,
                              float *weights, int32_t *counts, umsx_stream stream);

/* ---- Expert parallelism over NVLink (no counterpart in the reference, which refuses more than one
 * GPU backend: llama-b11669-hybrid-experts.patch:2617-2618) ---------------------------------------
 * One process per GPU.  A group is one exchange buffer per rank, mapped into every other rank's
 * process with CUDA IPC: create it on every rank, gather the ranks' handles (umsx_ep_handle) in rank
 * order with the caller's transport (torch.distributed in the Python binding), then connect.
 * An expert-parallel stack holds this rank's share of every layer (handles created with
 * desc.ep_rank / ep_world equal to the group's) and runs a decode step of one token per rank:
 * per layer, each rank stores its hidden row into every peer's buffer, all ranks route all the
 * group's tokens (the router is replicated), each runs the jobs of its own experts, stores each
 * job's output row into the buffer of the rank that owns the token, and that rank combines its
 * token in rank order with the residual.  With up to four ranks and MXFP4 layers with fused gate_up
 * the whole step is one kernel launch per rank: each rank's token goes to every rank once, every
 * rank folds every token, and each job's output row goes to every rank, with one flag exchange per
 * layer inside the kernel.  Stores are plain P2P stores from inside the kernels, flags
 * st.release.sys, waits ld.acquire.sys bounded by umsx_ep_set_wait (default about
 * one second): a rank that never arrives gives the others UMSX_ETIMEOUT from _host calls or
 * umsx_ep_stack_status, not a hang.  Each token's result has the single-GPU stack's bits.  All ranks
 * must call forward the same number of times, in step. */
typedef struct umsx_ep umsx_ep;
typedef struct umsx_ep_stack umsx_ep_stack;
umsx_status umsx_ep_create(int rank, int world, int device, int hidden, int top_k, umsx_ep **out);
/* The rank's IPC handle (size = 64 bytes). */
umsx_status umsx_ep_handle(umsx_ep *ep, void *handle_out, size_t size);
/* handles: every rank's handle in rank order (size = world * 64 bytes). */
umsx_status umsx_ep_connect(umsx_ep *ep, const void *handles, size_t size);
umsx_status umsx_ep_set_wait(umsx_ep *ep, int64_t wait_limit_cycles);
void umsx_ep_destroy(umsx_ep *ep);
umsx_status umsx_ep_stack_create(umsx_ep *ep, umsx_moe *const *layers, int n_layers, float rms_eps,
                                 umsx_ep_stack **out);
void umsx_ep_stack_destroy(umsx_ep_stack *stack);
/* x: this rank's token [1][H] (fp32 or bf16, device) -> out [1][H] fp32 (device). */
umsx_status umsx_ep_stack_forward(umsx_ep_stack *stack, const void *x, int x_dtype, float *out, umsx_stream stream);
umsx_status umsx_ep_stack_forward_host(umsx_ep_stack *stack, const void *x, int x_dtype, float *out,
                                       umsx_stream stream);
umsx_status umsx_ep_stack_status(umsx_ep_stack *stack, umsx_stream stream);

/* Expert-parallel prefill: every rank brings its own tokens (up to max_tokens; counts may differ
 * between ranks) and holds its share of the experts of every layer.  Per layer: each rank routes
 * its tokens (RMSNorm fused), counts the rows it sends each rank and stores its row of the G x G
 * count matrix into every rank (exchange 1), stores the Q8_0 row of each token (the experts' exact
 * input), its expert ids and its origin into the receive buffer of every rank that holds one of its
 * experts (exchange 2), runs its experts over the rows it received with the tensor-core grouped GEMM,
 * stores every job's output row into the owner's buffer (exchange 3), and combines its tokens in
 * rank order with the residual.  All three exchanges are P2P stores from inside the kernels that
 * compute the rows (umsx_ep.cu) with the group's flags and bounded waits.  Each token's result has
 * the single-GPU stack's bits on the same path (T >= 65 tokens: the tensor-core prefill).  The
 * receive buffers are per stack: gather and connect their handles like the group's, after
 * umsx_ep_connect.  Requires 65 <= max_tokens * world <= 65535 and <= 256 experts per rank. */
typedef struct umsx_ep_prefill umsx_ep_prefill;
umsx_status umsx_ep_prefill_create(umsx_ep *ep, umsx_moe *const *layers, int n_layers, int max_tokens,
                                   float rms_eps, umsx_ep_prefill **out);
umsx_status umsx_ep_prefill_handle(umsx_ep_prefill *stack, void *handle_out, size_t size);
umsx_status umsx_ep_prefill_connect(umsx_ep_prefill *stack, const void *handles, size_t size);
/* x: this rank's tokens [T][H] (fp32 or bf16, device) -> out [T][H] fp32 (device). */
umsx_status umsx_ep_prefill_forward(umsx_ep_prefill *stack, const void *x, int x_dtype, int tokens, float *out,
                                    umsx_stream stream);
umsx_status umsx_ep_prefill_forward_host(umsx_ep_prefill *stack, const void *x, int x_dtype, int tokens,
                                         float *out, umsx_stream stream);
/* Per layer of the last call: {rows this rank received, expert jobs it ran} (rows_jobs[2 * layers]);
 * synchronises the stack's stream.  The per-GPU load of expert parallelism (configs[3] skew). */
umsx_status umsx_ep_prefill_loads(umsx_ep_prefill *stack, int32_t *rows_jobs, int n);
umsx_status umsx_ep_prefill_status(umsx_ep_prefill *stack, umsx_stream stream);
void umsx_ep_prefill_destroy(umsx_ep_prefill *stack);

/* ---- GGUF checkpoints ------------------------------------------------------------------
 * The selected experts of one layer read from a GGUF file or a set of shards named
 * <stem>-00001-of-NNNNN.gguf (pass the first).  Replaces load_gguf_experts
 * (tools/engine/gguf_experts.cpp:45-140; LoadedExperts, gguf_experts.hpp:14-20): tensors
 * blk.L.ffn_{gate,up,down}_exps.weight (required, separate gate and up) and .bias (optional),
 * each in one shard; per tensor the byte slice of every selected expert (stride = tensor bytes /
 * experts) and, with dequantize != 0, its fp32 values; biases always as fp32.  Same limits as
 * the reference: layer in [0, 4096), 1..16 distinct ids, at most 32 Mi values per tensor
 * selection, experts per tensor <= 65536; types f32, f16, bf16, q8_0, mxfp4.  Errors:
 * UMSX_EINVAL with the reason in umsx_last_error().  Index p of each array: 0 gate, 1 up,
 * 2 down.  Host memory, released by umsx_gguf_experts_free. */
typedef struct umsx_gguf_experts {
    int32_t hidden, intermediate, experts, n_ids; /* experts: count in the file's tensors */
    int32_t quant[3];                             /* ggml type ids */
    uint64_t stride[3];                           /* bytes per expert */
    const uint8_t *packed[3];                     /* [n_ids][stride] ggml blocks */
    const float *values[3];                       /* [n_ids][rows * cols] fp32, or NULL */
    const float *bias[3];                         /* [n_ids][I, I, H] fp32, or NULL if absent */
    void *owner;
} umsx_gguf_experts;

umsx_status umsx_gguf_load_experts(const char *first_shard, int layer, const uint32_t *ids, int n_ids,
                                   int dequantize, umsx_gguf_experts *out);
void umsx_gguf_experts_free(umsx_gguf_experts *experts);

/* A resident layer straight from a GGUF checkpoint: the router blk.L.ffn_gate_inp.weight
 * ([E][H], f32/f16/bf16) and .bias, and every expert of blk.L.ffn_{gate,up,down}_exps (read
 * as umsx_gguf_load_experts does, without its 16-id limit), repacked as umsx_moe_create does.
 * desc must match the file: hidden, intermediate, experts, quant (all three projections),
 * has_bias (gate, up and down biases all present) and has_router_bias; fused_gate_up = 1
 * concatenates each expert's gate rows and up rows.  Biases keep their fp32 values.  No
 * counterpart in the reference beyond the loader above (the reference hands LoadedExperts to
 * Mxfp4NativeCudaDown's constructor, quantized_cuda.hpp:38-50). */
umsx_status umsx_moe_create_gguf(const umsx_moe_desc *desc, const char *first_shard, int layer, int device,
                                 size_t reserve_bytes, umsx_moe **out);

/* Number of this library's kernels launched by the calling thread since load (graph replays count
 * every kernel they contain). */
uint64_t umsx_kernel_launches(void);

const char *umsx_last_error(void);
int umsx_version(void);

#ifdef __cplusplus
}
#endif
#endif /* UMSX_H */
