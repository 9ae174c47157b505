// Internal structures of libumsx (not part of the C ABI).
//
// Device layout of an expert matrix (N rows x K columns, nb = K/32 blocks):
//   MXFP4 code plane: rows in groups of 16, blocks in pairs; chunk (group, pair) is
//     512 bytes = [lane half lh][L = 16*h + r][8 bytes] for row r and block 2*pair + h:
//     two 32-bit words, word w = sel(2w) | sel(2w+1) << 16, sel(p) = the four 4-bit
//     codes of elements 4p..4p+3 (lh 0) or 16+4p..16+4p+3 (lh 1).  A warp-wide 8-byte
//     load reads one lane half of a chunk.
//   MXFP4 exponent plane: chunk (group, pair quad) is 128 bytes, lane L holds the
//     exponents of its (row, block) for four consecutive pairs (padded to a quad).
//   Q8_0 code plane: rows in groups of 32; chunk (group, block) is 1 KB, lane r holds
//     the 32 codes of row r in lane-pair order [p][4p..4p+3, 16+4p..16+4p+3].
//   Q8_0 scale plane: chunk (group, block pair) is 128 bytes, lane r holds the two
//     fp16 scales of row r.
// The planes keep the ggml byte count (17 or 34 bytes per 32 weights), apart from
// the MXFP4 exponent padding.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "../../include/umsx.h"

namespace umsx {

struct Matrix {
    uint8_t *codes = nullptr;   // code plane, all local experts
    uint8_t *scales = nullptr;  // exponent / fp16-scale plane
    uint8_t *emax = nullptr;    // MXFP4: largest block exponent of every row [experts][rows] (prefill rebase)
    int rows = 0;               // N per expert
    int cols = 0;               // K
    int quant = 0;
    int exp_ge2 = 0;            // MXFP4: every block exponent is >= 2 (normal block scales; set at create time)
    size_t code_bytes_per_expert() const { return (size_t)rows * (cols / 32) * (quant == UMSX_QUANT_MXFP4 ? 16 : 32); }
    size_t scale_bytes_per_expert() const {
        if (quant == UMSX_QUANT_MXFP4) return (size_t)(rows / 16) * (((cols / 64) + 3) / 4) * 128;
        return (size_t)rows * (cols / 32) * 2;
    }
};

// Routing/dispatch state that the router writes and the expert kernels read.
struct Dispatch {
    float *logits;       // [T][E]
    int32_t *ids;        // [T][K]
    float *weights;      // [T][K]
    uint32_t *token_done;  // [T], zero between launches
    uint32_t *all_done;    // [1], zero between launches
    int32_t *counts;     // [E_local]
    int32_t *offsets;    // [E_local + 1]
    int32_t *active;     // [E_local] local expert index per active slot
    int32_t *n_active;   // [1]
    int32_t *job_token;  // [T*K] jobs grouped by expert, tokens ascending
    int32_t *job_rank;   // [T*K]
    uint8_t *xq_codes;   // [T][H/32][32] Q8_0 codes of x, lane-pair order
    float *xq_scales;    // [T][H/32] fp16-rounded Q8_0 scales of x
    int4 *slots;         // [E_local] per active slot {local expert, segment start, count, -}; expert -1 past the last
    uint32_t *tile_done; // [T][H/32] combine arrival counters, zero between launches
    uint8_t *xr;         // [T][H/32][64] x as MXFP4 staging records (MXFP4 layers)
    float *xr_sc;        // [T][pad4(H/32)] their scales
    uint32_t *err;       // [1] status bits set by kernels (never cleared by kernels): kErr*
};

// Bits of the device status word (Dispatch::err, DecodeParams::err).  The synchronous entry points
// turn kErrNonFinite into UMSX_ENONFINITE and every other bit into UMSX_ETIMEOUT.
constexpr uint32_t kErrNonFinite = 16u;  // a combined output (a layer's result) was inf or NaN

struct RouterParams {
    const void *x;
    int x_dtype;
    int tokens, hidden, experts, top_k, routing;
    float routed_scale;
    const float *w;   // [E][H]
    const float *b;   // [E] or null
    int e_lo, e_local;
    int fuse_dispatch;  // the last finishing CTA builds the dispatch (small T*K)
    int rmsnorm;        // normalise each input row (unit weight) before routing / quantizing
    float eps;
    int skip_counts;    // the caller needs only slot records and job lists (per-expert counts unwritten)
    int mx_records;     // write x as MXFP4 staging records (Dispatch::xr) instead of lane-pair Q8 rows
};

struct GateUpParams {
    Matrix gate_up;     // fused [2I][H] ...
    Matrix gate, up;    // ... or separate [I][H]
    int fused;
    const float *bias;  // [E_local][2I] fp32 (gate then up) or null
    int intermediate, hidden, activation;
    float alpha, limit;
    uint8_t *act_codes; // [T*K][I/32][32] Q8_0 codes of the activation, permuted job order, lane-pair order
    float *act_scales;  // [T*K][I/32] fp16-rounded Q8_0 scales
    float *act_f32;     // [T*K][I] activation values before quantization (MXFP4 path)
    uint8_t *act_rec;   // [T*K][I/32][64] quantized activations as MXFP4 staging records
    float *act_sc;      // [T*K][pad4(I/32)] their scales
    uint32_t *act_done; // [T*K][I/32] arrival counters of the two CTAs of each 32-value block
};

struct GemvParams {
    Matrix m;
    const float *bias;      // [E_local][N] or null
    const float *a_f32;     // activation rows to quantize, or null
    const uint8_t *a_q8;    // ggml block_q8_0 rows, or null
    const uint8_t *a_codes; // internal Q8 rows (lane-pair codes) when a_f32, a_q8 and a_rec are null
    const float *a_scales;
    const uint8_t *a_rec;   // MXFP4 staging records [row][nb][64] + scales [row][pad4(nb)], bulk-copied
    const float *a_rsc;
    int a_by_job;           // activation row = permuted job index
    int a_ts, a_rs;         // else activation row = token*a_ts + rank*a_rs
    float *out;             // output rows of N floats
    int o_ts;               // output row = token*o_ts + rank
    // fused rank-order combine (layer path): the last of a token's top_k expert CTAs
    // for a row tile writes combine_out[token] = residual + sum_r route_w[token][r] * out[token*top_k + r]
    uint32_t *tile_done;    // [T][N / rows-per-CTA] arrival counters, zero between launches; null = no combine
    const float *route_w;   // [T][top_k]
    const float *residual;  // [T][N] or null
    float *combine_out;     // [T][N]
    int top_k;
    int prefetch_early;     // the slot records were written two kernels back: prefetch weights before waiting
    const float *extra;     // [T][N] added after the top_k routed terms (the shared experts' output), or null
};

// Persistent decode kernel (umsx_decode.cu): every layer of a stack, or one layer,
// for at most kDecodeMaxTokens tokens in one cooperative launch.  MXFP4 weights with
// fused gate_up only; all experts local.
constexpr int kEpMaxRanks = 8;
constexpr int kDecodeMaxLayers = 48;
constexpr int kDecodeMaxTokens = 4;
constexpr int kDecodeMaxTopK = 8;

struct DecodeLayer {
    const float *router_w;    // [E][H]
    const float *router_b;    // [E] or null
    const uint8_t *gu_codes;  // fused gate_up planes [E][2I][H]
    const uint8_t *gu_scales;
    const float *gu_bias;     // [E][2I] or null
    const uint8_t *dn_codes;  // down planes [E][H][I]
    const uint8_t *dn_scales;
    const float *dn_bias;     // [E][H] or null
    int gu_ge2, dn_ge2;       // Matrix::exp_ge2 of the two matrices
};

struct DecodeParams {
    DecodeLayer layer[kDecodeMaxLayers];
    int n_layers;
    int tokens, hidden, inter, experts, top_k, routing, activation;
    float routed_scale, alpha, limit, eps;
    int rmsnorm;       // RMSNorm (unit weight) of h before each router
    int residual;      // h <- h + MoE(h) per layer; else out = MoE(x)
    const void *x;     // [T][H] F32 or BF16
    int x_dtype;
    float *out;        // [T][H]
    int32_t *ids_out;  // [T][K] routing of the last layer, or null
    float *w_out;      // [T][K]
    float *logits;     // [T][E] scratch
    float *act;        // [T*K][I] scratch
    float *y;          // [T*K][H] scratch
    uint8_t *xr;       // [T][H/32][64] Q8_0 records of the normalised rows
    float *xr_sc;      // [T][pad4(H/32)]
    unsigned *bar;     // grid barrier counter (zeroed by the launcher)
    uint32_t *err;     // status bits (kErr*): a grid barrier wait ran out, a non-finite output
    // fault injection for tests: CTA fault_cta withholds its first grid-barrier arrival (-1: none), so
    // every wait of that barrier runs out after wait_cycles (0: the default bound) and reports it
    int fault_cta;
    long long wait_cycles;
    // Expert parallelism over NVLink (ep_world > 1; 1 = all experts local): tokens = ep_world, token g
    // being rank g's (p.x holds this rank's one row); this rank holds experts [e_lo, e_lo + e_local) of
    // every layer and routes all tokens; each local job's output row is stored into every rank's y;
    // the token rows are exchanged first and every layer ends with a cross-rank flag exchange.
    int ep_world, ep_rank, e_lo, e_local;
    float *peer_y[kEpMaxRanks];         // each rank's y [T*K][H] (this rank's entry = y)
    float *peer_x[kEpMaxRanks];         // each rank's x_all [world][H]
    const float *x_all;                 // this rank's x_all
    unsigned *peer_flags[kEpMaxRanks];  // each rank's flag array [world] (slot = source rank)
    unsigned *flags;                    // this rank's flag array
    unsigned *epoch;                    // this rank's exchange counter (monotonic, never zeroed)
    long long ep_wait_cycles;           // bound of every cross-rank wait
};

bool decode_supported(int tokens, int hidden, int inter, int experts, int top_k, int n_layers);
// Returns 1 (kernels launched) or -1 if this device cannot hold the kernel resident on every SM.
int launch_decode(const DecodeParams &p, cudaStream_t s);

// Prefill grouped GEMM (umsx_prefill.cu): tcgen05 kind::f16 over the experts' job segments.
constexpr int kPrefillMinTokens = 65;  // from this many tokens an MXFP4 layer takes the tensor-core path

struct MoeGemmParams {
    int quant;            // UMSX_QUANT_MXFP4 or UMSX_QUANT_Q8_0
    const uint8_t *codes, *scales, *emax;  // the projection's planes (and, MXFP4, row exponents; null for Q8_0)
    const uint8_t *codes2, *scales2, *emax2;  // separate gate/up: the up planes (and MXFP4 row exponents), else null
    int plane_rows;       // rows per expert of the plane(s) `codes` points to
    int rows, cols;       // per expert: output rows N, reduction K
    int fused, inter;     // fused gate_up: tile rows 0-63 gate rows, 64-127 the matching up rows (offset inter)
    const float *bias;    // [E][rows] or null
    const int32_t *offsets;  // [E + 1] job segments (jobs in expert order)
    int experts, m_tiles;
    int mode;             // 0: gate_up -> act_hi + act_lo = f16 Q8_0 values [jobs][inter]; 1: down -> y_out [jobs][rows]
    int activation;
    float alpha, limit;
    uint16_t *act_hi, *act_lo;
    float *y_out;
    uint32_t *err;
};

// Router for many tokens: tiled logits (same arithmetic as launch_router), per-token selection and
// x -> Q8_0 (lane-pair order), then the dispatch build.
int launch_router_tiled(const RouterParams &p, const Dispatch &d, cudaStream_t s);
// Also ORs 1 into *low (if not null) when a block exponent of the matrix is below 2.
int launch_row_emax(const Matrix &m, int experts, uint8_t *emax, uint32_t *low, cudaStream_t s);
// n_jobs: device count of the resident experts' jobs (offsets[e_local]) bounding `jobs`, or null.
int launch_prefill_pack(const Dispatch &d, int jobs, const int32_t *n_jobs, int K, int hidden, void *a_hi, void *a_lo,
                        int32_t *inv, cudaStream_t s);
// y[t][r] = yj[inv[t][r]] for the (t, r) whose expert id lies in [e_lo, e_lo + e_local).
int launch_prefill_scatter(const float *yj, const int32_t *inv, const int32_t *ids, int e_lo, int e_local, int tokens,
                           int K, int width, float *y, cudaStream_t s);
// extra: [T][width] added after the K routed terms (shared experts), or null
int launch_prefill_combine(const float *y, const float *w, const int32_t *inv, int tokens, int K, int width,
                           const float *extra, const float *residual, float *out, uint32_t *err, cudaStream_t s);
int launch_moe_gemm(const MoeGemmParams &p, const void *act_hi, const void *act_lo, int rows_total, cudaStream_t s);

// Expert-parallel exchange of a decode step (umsx_ep.cu): one token per rank, peers reached through
// CUDA IPC mappings of their exchange buffers.

struct EpParams {
    int rank, world, hidden, top_k, e_lo, e_local;
    float *h_own;                     // [H] this rank's token (its residual stream)
    float *peer_h_all[kEpMaxRanks];   // each rank's h_all [world][H] (this rank's own entry included)
    float *peer_y_recv[kEpMaxRanks];  // each rank's y_recv [K][H]
    unsigned *peer_flags[kEpMaxRanks];  // each rank's flag array [world]
    unsigned *flags;                  // this rank's flag array
    unsigned *epoch;                  // this rank's exchange counter
    const float *y_recv;              // this rank's y_recv
    const float *y_jobs;              // [world][K][H] outputs of this rank's jobs
    const int32_t *ids;               // [world][K] routing (replicated)
    const float *weights;             // [world][K]
    uint32_t *err;
    long long wait_cycles;            // bound of every exchange wait
};

int launch_ep_share(const EpParams &p, cudaStream_t s);
int launch_ep_combine(const EpParams &p, cudaStream_t s);

// Expert-parallel prefill (umsx_ep.cu): tokens sharded over the ranks, experts split contiguously
// (rank g holds [g*E/G, (g+1)*E/G)); token rows go to the ranks that hold their experts and the
// expert outputs come back, both as P2P stores into the peers' receive buffers.
struct EpPrefillParams {
    int rank, world, hidden, top_k, e_per_rank, tokens, tokens_max, rows_max;
    const int32_t *ids;          // [T][K] routing of this rank's tokens
    const uint8_t *xq_codes;     // [T][H] Q8_0 codes of this rank's normalised tokens (lane-pair order)
    const float *xq_scales;      // [T][H/32]
    int32_t *pos;                // [T][world] row of token t in rank g's receive buffer, -1 if none
    int32_t *counts;             // [world][world] count matrix (row = source rank), this rank's copy
    unsigned *done;              // CTA arrival counter (zero between launches)
    int32_t *peer_counts[kEpMaxRanks];
    uint8_t *peer_codes[kEpMaxRanks];    // [rows_max][H]
    float *peer_scales[kEpMaxRanks];     // [rows_max][H/32]
    int32_t *peer_ids[kEpMaxRanks];      // [rows_max][K] expert ids held by that rank, -1 for the others
    int2 *peer_src[kEpMaxRanks];         // [rows_max] (source rank, source token)
    float *peer_y_back[kEpMaxRanks];     // [tokens_max][K][H]
    const int32_t *recv_ids;     // this rank's receive buffers (its own peer_* entries)
    const int2 *recv_src;
    const int32_t *inv;          // [rows_max][K] job row of (received row, rank slot) in y_jobs
    const float *y_jobs;         // [jobs][H] outputs of this rank's expert jobs (expert order)
    const int32_t *n_jobs;       // this rank's job count (device)
    int2 *loads;                 // per layer {rows received, jobs run}, or null
    unsigned *flags;
    unsigned *peer_flags[kEpMaxRanks];
    unsigned *epoch;
    uint32_t *err;
    long long wait_cycles;
};

int launch_ep_count(const EpPrefillParams &p, cudaStream_t s);
int launch_ep_dispatch(const EpPrefillParams &p, cudaStream_t s);
int launch_ep_return(const EpPrefillParams &p, int layer, cudaStream_t s);
int launch_ep_wait(const EpPrefillParams &p, cudaStream_t s);

// Thread-local status channel shared by every translation unit (umsx_api.cu).
void record_error(const char *msg);      // the message umsx_last_error() returns
void record_launches(uint64_t kernels);  // adds to umsx_kernel_launches()

// Launchers (umsx_kernels.cu).  Each returns the number of kernels launched.
int launch_router(const RouterParams &p, const Dispatch &d, cudaStream_t s);
int launch_dispatch(const Dispatch &d, int entries, int top_k, int e_lo, int e_local, cudaStream_t s);
// max_per_expert: jobs a CTA takes per pass (the kernels loop over an expert's other jobs).
int launch_gate_up(const GateUpParams &p, const Dispatch &d, int max_slots, int max_per_expert, cudaStream_t s);
int launch_gemv(const GemvParams &p, const Dispatch &d, int max_slots, int max_per_expert, cudaStream_t s);

// err: status word that records a non-finite output (kErrNonFinite), or null
int launch_combine(const float *y, const float *w, int tokens, int top_k, int width, const float *extra,
                   const float *residual, float *out, uint32_t *err, cudaStream_t s);
int launch_repack(const Matrix &m, int expert, const uint8_t *ggml, cudaStream_t s);
int launch_bank_remap(int4 *slots, const int32_t *map, int n, cudaStream_t s);
int launch_export(const Matrix &m, int expert, uint8_t *ggml, cudaStream_t s);
int launch_gen_blocks(int quant, uint64_t seed, uint64_t stream, uint64_t first_block, uint64_t nblocks,
                      uint8_t *out, cudaStream_t s);
int launch_gen_normal_f32(uint64_t seed, uint64_t stream, uint64_t first, uint64_t n, float scale, float *out,
                          cudaStream_t s);
int launch_gen_normal_bf16_to_f32(uint64_t seed, uint64_t stream, uint64_t first, uint64_t n, float scale,
                                  float *out, cudaStream_t s);
int launch_bf16_to_f32(const uint16_t *in, float *out, size_t n, cudaStream_t s);

// GGUF expert slices (umsx_gguf.cpp), the reference's LoadedExperts
// (tools/engine/gguf_experts.hpp:14-20).  Index p: 0 gate, 1 up, 2 down.
struct GgufExperts {
    int hidden = 0, intermediate = 0, count = 0, n_ids = 0;  // count: experts in the file's tensors
    int type[3] = {-1, -1, -1};                                // ggml type ids
    int64_t shape[3][3] = {};                                  // ne[0..2] of each weight tensor
    size_t stride[3] = {};                                     // bytes per expert
    std::vector<uint8_t> packed[3];                            // [n_ids][stride]
    std::vector<float> values[3];                              // [n_ids][rows * cols] when dequantized
    bool has_bias[3] = {};
    int64_t bias_len[3] = {};
    std::vector<float> bias[3];                                // [n_ids][bias_len]
};
// Reads the slices of experts `ids` of layer `layer`; "" or an error message.  bounded:
// the reference's limits for a selection (at most 16 ids, 32 Mi values per tensor).
std::string gguf_load_experts(const std::string &first_shard, int layer, const std::vector<uint32_t> &ids,
                              bool dequant, bool bounded, GgufExperts &out);
// The router weight blk.L.ffn_gate_inp.weight ([E][H] fp32; shape = {H, E}) and its bias if present.
std::string gguf_load_router(const std::string &first_shard, int layer, std::vector<float> &w, int64_t shape[2],
                             std::vector<float> &b, bool &has_b);

}  // namespace umsx
