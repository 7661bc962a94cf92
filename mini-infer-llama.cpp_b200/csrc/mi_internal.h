// Internal host/device interface of the backend (not part of the C-ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace mi {

// Device view of the expf exception hash (see mi_expf_core.h).
struct ExpTab {
  const uint4* buckets;
  uint32_t log2b, mul1, mul2;
  uint32_t filter;  // the table holds only results near a rounding boundary (mi_expf_near_tie)
};

// ---------------------------------------------------------------------------
// Q8_0 GEMV
// ---------------------------------------------------------------------------
enum GemvPrologue : int32_t {
  PRO_ACT = 0,         // activation given as Q8_0_ACT blocks
  PRO_QUANT = 1,       // quantize F32 x in the prologue
  PRO_NORM_QUANT = 2,  // rms_norm(x) * norm_w, then quantize
  PRO_EMBED_NORM = 3,  // x = dequantized embedding row tokens[*pos]; then as PRO_NORM_QUANT
};

enum GemvEpilogue : int32_t {
  EPI_STORE = 0,        // out[r] = dot
  EPI_BIAS = 1,         // out[r] = dot + bias[r]
  EPI_RESID = 2,        // out[r] = resid[r] + dot
  EPI_SILU_GATEUP = 3,  // packed rows 8q+t / 8q+4+t are gate / up row 4q+t:
                        // out[4q+t] = silu(gate) * up
  EPI_ARGMAX = 4,       // out[r] = dot, plus the greedy token over all rows
  EPI_SILU_GATEUP_Q = 5,  // as EPI_SILU_GATEUP, but each CTA owns 64 packed rows (one
                          // 32-element block of the result) and stores that block
                          // quantized to Q8_0_ACT at act_out (the down GEMV's input)
};

// Tensor parallelism: ranks (one per GPU) exchange vectors through buffers of
// 8-byte words, value bits | tag << 32, that producers store into every
// rank's copy over NVLink (peer pointers). A consumer waits, bounded, until a
// word carries the current step's tag; no separate flag or fence is needed
// because each word is written by one 64-bit store.
constexpr int kMaxRanks = 8;

struct GemvParams {
  const uint8_t* w;
  int64_t K, N, n_pad;
  int32_t rows_per_cta, stage_rows, n_stages, pro, epi;
  int32_t kc, n_chunks;  // set by the launcher: blocks per K-chunk of a stage, chunks per row pass
  int32_t tokens_len;  // entries of `tokens` / `tokens_rw` (bounds for pos)
  int32_t stage_x;     // set by the launcher: F32 input staged in shared memory
  // prologue inputs
  const float* x;
  const uint8_t* act;  // Q8_0_ACT, K/32 blocks of 36 B
  const float* norm_w;
  float eps;
  int32_t pad1;
  const uint8_t* embed;  // packed Q8_0 embedding table [K x embed_npad]
  int64_t embed_npad, embed_rows;
  const int32_t* tokens;
  const int32_t* pos;
  float* x_out;  // PRO_EMBED_NORM: CTA 0 stores the embedding row here
  // epilogue
  const float* bias;
  const float* resid;
  float* out;
  uint8_t* act_out;  // EPI_SILU_GATEUP_Q: Q8_0_ACT blocks of the result
  // EPI_ARGMAX
  float* part_val;
  int32_t* part_idx;
  uint32_t* counter;
  int32_t* next_token;
  int32_t* tokens_rw;  // with *feedback != 0 the winner is also stored at tokens[pos+1]
  int32_t* pos_rw;     // ... and pos is advanced
  const int32_t* feedback;
  ExpTab et;
  int32_t* err;
  uint64_t* trace;     // optional step trace (4 stamps per kernel slot)
  int32_t trace_slot;
  // Tensor parallelism (the TP kernel instantiation only): this GEMV computes
  // rows [row0, row0 + N) of the full output (Q8_0_ACT blocks: row0 / 64 for
  // the gate/up epilogue). _ll inputs are indexed by full-vector position.
  int32_t n_ranks, rank;
  int64_t row0;
  const uint32_t* epoch;        // the step's tag
  const uint64_t* x_ll;         // F32 input vector (PRO_QUANT / PRO_NORM_QUANT)
  const uint64_t* act_ll;       // Q8_0_ACT input, 9 words per block (PRO_ACT)
  const uint64_t* resid_ll;     // EPI_RESID residual
  uint64_t* out_ll[kMaxRanks];  // every rank's copy of the output (EPI_ARGMAX: candidates)
  uint32_t* epoch_rw;           // EPI_ARGMAX: advanced once the step's token is known
};

struct GemvPlan {
  int grid, threads, tpr;
  int32_t rows_per_cta, stage_rows, n_stages, stage_x;
  int32_t kc, n_chunks;  // K-chunk of a stage in 32-element blocks (kc == K/32: whole rows)
  size_t smem;
};

// Work split for an n-row, k-column packed matrix over the device's SMs.
// rows_per_cta > 0 fixes the rows per CTA (a multiple of 8; of 64 for the
// SiLU*up quantizing epilogue, at most 8 blocks).
GemvPlan plan_gemv(int64_t k, int64_t n, int num_sms, int pro, int32_t rows_per_cta = 0);
// Per-device kernel attributes (dynamic shared memory limit); called once per
// device at context creation, outside any stream capture.
cudaError_t prepare_kernels();
cudaError_t launch_gemv(const GemvParams& p, const GemvPlan& plan, cudaStream_t s, bool pdl,
                        bool tp = false);

// ---------------------------------------------------------------------------
// Decode attention (one query token per head)
// ---------------------------------------------------------------------------
struct AttnParams {
  const float* qkv;     // executor: q | k | v projections (pre-RoPE q and k)
  const float* q_rot;   // op: rotated queries [n_head][hd]
  float* cache_k;       // [n_ctx][n_head_kv][hd]
  float* cache_v;
  int32_t head_dim, n_head, n_head_kv, n_kv_fixed;  // n_kv_fixed: op mode
  const int32_t* pos;   // executor: current position (n_past)
  const float2* rope_cs;  // executor: [pos][head_dim/2] (cos, sin)
  float scale;
  int32_t n_ctx;         // executor: cache / RoPE table capacity (bounds for pos)
  float* scores;        // scratch [n_head][scores_stride] (used when the scores do not fit on chip)
  int64_t scores_stride;
  float* out;           // [n_head][hd]; may be null when act_out is set
  uint8_t* act_out;     // optional: the output quantized to Q8_0_ACT (head_dim % 32 == 0)
  ExpTab et;
  int32_t* err;
  int32_t kv_tile;         // set by the launcher: K/V positions per shared-memory chunk
  int32_t scores_in_smem;  // set by the launcher
  uint64_t* trace;         // optional step trace (4 stamps per kernel slot)
  int32_t trace_slot;
  const uint64_t* qkv_ll;  // tensor parallelism: q | k | v as exchange words (instead of qkv)
  const uint32_t* epoch;
  // Batched queries (op mode, gridDim.y = T): query t uses q_rot + t*n_head*hd,
  // n_kv = n_kv_fixed + t, and writes its outputs at row t.
  int8_t* act_qs;  // optional: output quantized to the split Q8_0_ACT layout (row n_head*hd bytes)
  float* act_d;
};
cudaError_t launch_attn_decode(const AttnParams& p, bool exec_mode, cudaStream_t s, bool pdl,
                               bool tp = false, int32_t n_queries = 1);
// Exact decode attention for one query past the on-chip score limit, spread
// over the GPU (attn_long.cu): scores, softmax (ordered denominator by
// spec_ordered_sum) and the ordered value chains as three kernels; uses
// p.scores [n_head][scores_stride] for the scores and then the probabilities.
bool attn_long_fits(int64_t head_dim, int64_t n_head, int64_t n_head_kv, int64_t n_kv, int optin);
cudaError_t prepare_attn_long_kernels(int optin);  // per device, at init
cudaError_t prepare_attn_split_kernels();          // per device, at init
cudaError_t launch_attn_decode_long(const AttnParams& p, cudaStream_t s);

// Decode attention split over positions (attn_split.cu): a fast mode that
// regroups the softmax and value sums (not bit-exact). part holds
// attn_split_scratch_bytes() bytes.
bool attn_split_fits(int64_t head_dim, int64_t n_head, int64_t n_head_kv);
void attn_split_shape(int64_t n_kv, int64_t n_head_kv, int32_t* n_splits, int32_t* per_split);
size_t attn_split_scratch_bytes(int64_t n_head, int64_t n_kv, int64_t n_head_kv, int64_t head_dim);
cudaError_t launch_attn_split(const float* q, const float* ck, const float* cv, int64_t D, int64_t H, int64_t HKV,
                              int64_t n_kv, float scale, const ExpTab& et, int32_t* err, float* part, float* out,
                              cudaStream_t s);

// ---------------------------------------------------------------------------
// Fused QKV projection + decode attention (executor, one GPU)
// ---------------------------------------------------------------------------
// One thread-block cluster of n_rep + 1 CTAs per KV head: CTA c < n_rep
// computes the q rows of query head kvh * n_rep + c, CTA n_rep the k and v
// rows of the KV head. Every CTA runs the rms_norm + quantize prologue; the
// k/v CTA applies RoPE, appends k and v to the cache and stores them into the
// query CTAs' shared memory; after the cluster barrier each query CTA runs the
// decode attention of its head. Removes the QKV -> attention kernel boundary.
struct QkvAttnParams {
  const uint8_t* w;  // packed Q | K | V rows
  int64_t K, n_pad;
  const float* bias;  // [n_head * hd + 2 * n_head_kv * hd]
  int32_t pro;        // PRO_NORM_QUANT, or PRO_EMBED_NORM (layer 0)
  int32_t tokens_len;
  const float* x;
  const float* norm_w;
  float eps;
  int32_t pad0;
  const uint8_t* embed;
  int64_t embed_npad, embed_rows;
  const int32_t* tokens;
  float* x_out;  // PRO_EMBED_NORM: CTA 0 stores the embedding row here
  float* cache_k;
  float* cache_v;
  int32_t head_dim, n_head, n_head_kv, n_ctx;
  const int32_t* pos;
  const float2* rope_cs;
  float scale;
  int32_t kv_tile, scores_in_smem;  // set from the plan
  int32_t pad1;
  float* scores;  // [n_head][scores_stride] when the scores do not fit on chip
  int64_t scores_stride;
  float* out;         // [n_head][hd]; null when act_out is set
  uint8_t* act_out;   // the O projection's Q8_0_ACT input (head_dim % 32 == 0)
  ExpTab et;
  int32_t* err;
  uint64_t* trace;
  int32_t trace_slot;
  // Detail slots: CTA 0 (query CTA of head 0) and CTA n_rep (the first k/v
  // CTA) store 0 entry, 1 dependency satisfied, 2 x loaded, 3 rms_norm sum
  // done, 4 prologue done, 5 rows done, 6 bias + RoPE done, 7 hand-over done
  // (query CTA: k / v received; k/v CTA: k / v sent).
  int32_t trace_slot_q, trace_slot_kv;
};
struct QkvAttnPlan {
  bool ok;
  int32_t cluster, kv_tile, scores_in_smem;
  size_t smem;
};
// The fused kernel's plan for a model shape, or ok == false when the shape
// does not fit it (head_dim, cluster size, shared memory within smem_budget
// bytes) or the device cannot run one of its clusters.
QkvAttnPlan plan_qkv_attn(int64_t K, int32_t head_dim, int32_t n_head, int32_t n_head_kv, int32_t n_ctx,
                          size_t smem_budget);
cudaError_t launch_qkv_attn(const QkvAttnParams& p, const QkvAttnPlan& plan, cudaStream_t s, bool pdl);
cudaError_t prepare_qkv_attn_kernel(int optin);

// ---------------------------------------------------------------------------
// Persistent decode step (decode_persist.cu): one launch per decode step on
// one GPU. CTAs stay resident for the whole step; phases hand over through
// device counters instead of kernel boundaries, and every CTA streams the
// weights of its coming work items into a shared-memory ring a layer ahead.
// ---------------------------------------------------------------------------
struct PersistLayer {
  const uint8_t* qkv;     // packed Q | K | V rows, n_pad qkv_npad
  const float* bqkv;
  const float* attn_norm;
  const uint8_t* o;       // packed, E rows
  const uint8_t* gateup;  // packed gate/up rows interleaved by groups of 4
  const float* ffn_norm;
  const uint8_t* down;    // packed, E rows of K = n_ff
};

struct PersistParams {
  int32_t n_layer, E, H, HKV, D, FF, V, n_ctx;
  int64_t qkv_npad, gu_npad, head_npad;
  float eps, scale;
  const PersistLayer* layers;  // device array of n_layer
  const uint8_t* embed;        // packed Q8_0 embedding [E x V]
  int64_t embed_npad;
  const uint8_t* head;         // packed LM head [E x V]
  const float* out_norm;
  float* cache;                // [layer][k|v][n_ctx][HKV][D]
  const float2* rope;          // [pos][D/2]
  float* x;                    // residual stream (layer input / down output)
  float* x2;                   // residual stream after attention
  uint8_t* act_q;              // Q8_0_ACT: the down projection's input
  float* logits;
  float* scores;               // [H][n_ctx] when the scores do not fit on chip
  float* part_val;             // per-CTA LM-head winners
  int32_t* part_idx;
  int32_t* tokens;
  int32_t tokens_len;
  int32_t with_head;           // 0: the step only writes the KV cache and advances pos
  int32_t* pos;
  int32_t* next_token;
  const int32_t* feedback;
  int32_t* err;
  uint32_t* ticket;            // CTAs finished with the step (the last one closes it)
  unsigned long long* epoch;   // steps completed since the counters were zeroed
  unsigned long long* ctr;     // [n_layer][4] hand-over counters (1: x2, 2: act, 3: x stored)
  // schedule: CTAs [0, n_attn) are one cluster (per KV head n_rep query
  // CTAs and one k/v CTA) running the attention and the O projection; the
  // other n_gemv CTAs the gate/up and down projections and the LM head
  int32_t n_attn, n_gemv;
  int32_t kv_tile, scores_in_smem;
  int32_t ring_gemv, ring_attn;  // weight-ring bytes of the two roles
  ExpTab et;
  uint64_t* trace;             // optional: 8 stamps per slot, 2 slots per layer + 1
  int32_t fast;                // 1: the labelled fast mode (regrouped sums, not bit-exact)
};

struct PersistPlan {
  bool ok;
  int32_t grid, cluster, n_attn, n_gemv, kv_tile, scores_in_smem, ring_gemv, ring_attn;
  size_t smem;
};
// The persistent kernel's plan for a model shape on this device, or ok ==
// false when the shape does not fit it (then the executor keeps the
// kernel-per-phase graph).
PersistPlan plan_persist(int64_t E, int32_t D, int32_t H, int32_t HKV, int64_t FF, int64_t V, int32_t n_layer,
                         int32_t n_ctx, int num_sms);
cudaError_t launch_persist(const PersistParams& p, const PersistPlan& plan, cudaStream_t s);
cudaError_t prepare_persist_kernel(int optin);

// ---------------------------------------------------------------------------
// Batched prefill (prefill.cu)
// ---------------------------------------------------------------------------
// Exact Q8_0 GEMM over M tokens: out[t * out_stride + r] = dot(W row r, act t)
// (+ bias[r] / + resid[t * out_stride + r]); EPI_SILU_GATEUP_Q writes the
// quantized silu(gate) * up activation instead. Activations in the split
// Q8_0_ACT layout: quants [M][act_stride] bytes, scales [M][act_stride / 32].
struct GemmParams {
  const uint8_t* w;
  int64_t K, N, n_pad;
  const int8_t* act_qs;
  const float* act_d;
  int64_t act_stride;
  int64_t M;
  int32_t epi;
  const float* bias;
  const float* resid;
  float* out;
  int64_t out_stride;
  int8_t* q_out;  // EPI_SILU_GATEUP_Q: split Q8_0_ACT rows of q_stride bytes
  float* d_out;
  int64_t q_stride;
  ExpTab et;
  // The tensor-core path (prefill_tc.cu): the weights' prefill copy made by
  // launch_pack_tc (nullptr: the CUDA-core kernel of prefill.cu), and the
  // error word for its bounded waits.
  const uint8_t* wt;
  const float* st;
  int32_t* err;
};
cudaError_t prepare_gemm_kernel();
cudaError_t launch_gemm(const GemmParams& p, cudaStream_t s);
// Tensor-core exact GEMM (prefill_tc.cu). tc_rows(npad) is the row count of
// the prefill copy (a multiple of 128); launch_pack_tc fills it
// (tc_weight_bytes of fp16 quants at wt, n_tc * K / 32 floats at st) from a
// packed matrix.
int64_t tc_rows(int64_t npad);
size_t tc_weight_bytes(int64_t n_tc, int64_t K);
cudaError_t launch_pack_tc(const uint8_t* w, int64_t K, int64_t npad, int64_t n_tc, uint8_t* wt, float* st,
                           cudaStream_t s);
cudaError_t prepare_gemm_tc_kernel();
cudaError_t launch_gemm_tc(const GemmParams& p, cudaStream_t s);

// Per token: [embedding lookup (x_out),] [rms_norm * norm_w,] Q8_0_ACT quantize
// into the split layout (q_out [t][K], d_out [t][K/32]).
struct NormQuantParams {
  int64_t K;
  const float* x;             // [T][K] when embed == nullptr
  const uint8_t* embed;       // packed Q8_0 embedding table
  int64_t embed_npad, embed_rows;
  const int32_t* tokens;      // [T]
  float* x_out;               // embedding rows [T][K]
  const float* norm_w;        // nullptr: quantize only
  float eps;
  int8_t* q_out;
  float* d_out;
  int32_t* err;
};
cudaError_t launch_norm_quant(const NormQuantParams& p, int64_t n_tokens, cudaStream_t s);
// Causal attention for T queries at positions n_past + t: one CTA per (KV
// head, query), n_rep query heads each; output quantized to the split
// Q8_0_ACT layout (act_qs / act_d, rows of `row` elements) or F32 rows (out).
struct PrefillAttnParams {
  const float* q_rot;    // [T][n_head][head_dim]
  const float* cache_k;  // [n_ctx][n_head_kv][head_dim]
  const float* cache_v;
  int32_t head_dim, n_head, n_head_kv, n_rep, n_past;
  float scale;
  int64_t row;  // output row length (n_head * head_dim)
  int8_t* act_qs;
  float* act_d;
  float* out;
  ExpTab et;
  int32_t sc_stride;  // set by the launcher
};
bool prefill_attn_fits(int32_t head_dim, int32_t n_rep, int64_t max_kv);
cudaError_t launch_attn_prefill(const PrefillAttnParams& p, int64_t n_tokens, cudaStream_t s);
cudaError_t launch_rope_kv(const float* qkv, int64_t row, int32_t head_dim, int32_t n_head,
                           int32_t n_head_kv, int32_t n_past, int64_t n_tokens, const float2* rope_cs,
                           float* q_rot, float* cache_k, float* cache_v, cudaStream_t s);

// ---------------------------------------------------------------------------
// Small ops
// ---------------------------------------------------------------------------
// Packs n GGUF rows (source rows src_row0 .. src_row0+n-1 of a matrix) into a
// packed matrix with dst_npad rows: source row i lands on packed row
// (i/4)*group_stride + row_offset + i%4.
cudaError_t launch_pack_q8_0(const uint8_t* raw, int64_t k, int64_t n, int64_t src_row0,
                             uint8_t* dst, int64_t dst_npad, int64_t row_offset,
                             int64_t group_stride, cudaStream_t s);
cudaError_t launch_expf_range(uint64_t first, int64_t count, float* dst, const ExpTab& et,
                              cudaStream_t s);
cudaError_t launch_zero_pad_rows(uint8_t* dst, int64_t k, int64_t n_pad, cudaStream_t s);
cudaError_t launch_quantize_act(const float* x, int64_t k, int64_t m, uint8_t* act,
                                cudaStream_t s);
cudaError_t launch_block_isums(const uint8_t* w, int64_t k, int64_t n, int64_t n_pad,
                               const uint8_t* act, int32_t* isums, cudaStream_t s);
// dst[j*n + i] = dot(W row i, act row j) in the reference's scalar order (one
// fma chain over the blocks' int32 sums).
cudaError_t launch_gemv_scalar_order(const uint8_t* w, int64_t k, int64_t n, int64_t n_pad,
                                     const uint8_t* act, int64_t m, float* dst, cudaStream_t s);
cudaError_t launch_get_rows(const uint8_t* table, int64_t ne0, int64_t n_pad,
                            const int32_t* ids, int64_t n_ids, float* dst, cudaStream_t s);
cudaError_t launch_rms_norm(const float* x, int64_t ne0, int64_t n_rows, float eps, float* dst,
                            cudaStream_t s);
cudaError_t launch_binop(int op, const float* a, const float* b, int64_t ne0, int64_t n_rows,
                         int64_t b_rows, float v, float* dst, cudaStream_t s);
cudaError_t launch_silu(const float* x, int64_t n, float* dst, const ExpTab& et, cudaStream_t s);
cudaError_t launch_expf(const float* x, int64_t n, float* dst, const ExpTab& et, cudaStream_t s);
cudaError_t launch_rope(const float* x, int64_t head_dim, int64_t n_head, int64_t n_tokens,
                        int32_t n_dims, const float2* cs, float* dst, cudaStream_t s);
cudaError_t launch_attn_qk(const float* q, const float* k, int64_t hd, int64_t nh, int64_t nhkv,
                           int64_t n_kv, int64_t nt, float* scores, cudaStream_t s);
cudaError_t launch_softmax(const float* x, int64_t n_kv, int64_t nt, int64_t nh, int32_t n_past,
                           float scale, float* dst, const ExpTab& et, cudaStream_t s);
cudaError_t launch_attn_kqv(const float* p, const float* v, int64_t hd, int64_t nh, int64_t nhkv,
                            int64_t n_kv, int64_t nt, float* dst, cudaStream_t s);
cudaError_t launch_argmax(const float* x, int64_t n, float* part_val, int32_t* part_idx,
                          uint32_t* counter, int32_t* out, cudaStream_t s);
// pos += 1 (and *epoch += 1 when given) after the preceding kernel.
cudaError_t launch_advance(int32_t* pos, cudaStream_t s, bool pdl, uint32_t* epoch = nullptr);
cudaError_t launch_set_pos(int32_t* pos, int32_t value, cudaStream_t s);

// ---------------------------------------------------------------------------
// Library state (ops_capi.cu)
// ---------------------------------------------------------------------------
struct DeviceCtx {
  int device = -1;
  int num_sms = 0;
  ExpTab et{};
  void* et_buf = nullptr;
  int32_t* err = nullptr;  // device error word
  // scratch for mi_cuda_argmax
  float* am_val = nullptr;
  int32_t* am_idx = nullptr;
  uint32_t* am_counter = nullptr;
  // RoPE table cache for the per-op entry point
  float2* rope = nullptr;
  int32_t rope_n_pos = 0, rope_n_dims = 0;
  float rope_base = 0.0f;
};

// Per-device context, initialized on first use (loads the expf table).
DeviceCtx* device_ctx(int device, std::string* err);
DeviceCtx* current_ctx(std::string* err);
// The context of `device` if mi_cuda_init (or any entry point) already created
// it, else nullptr; never creates one (creation allocates device memory).
const DeviceCtx* existing_device_ctx(int device);
void set_error(const std::string& msg);

// Host RoPE table (host_math.cpp): cs[(pos - pos0) * (n_dims/2) + p] for
// pos in [pos0, pos0 + n_pos), evaluated with the host libm exactly as the
// reference (src/ops_cpu.cpp:286-292).
void build_rope_table(int32_t pos0, int32_t n_pos, int32_t n_dims, float freq_base, float* cs);

// Host expf helpers (host_math.cpp).
void expf_fingerprints(uint32_t* core, uint32_t* libm);
// Counts floats with bits in [first, first+n) where libm expf != y[i - first].
uint64_t expf_count_mismatch(uint64_t first, int64_t n, const float* y);

}  // namespace mi
