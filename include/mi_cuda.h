/* mi_cuda.h -- C-ABI of the B200 (sm_100a) decode backend for mini-infer.
 *
 * Plain pointers, sizes and status codes only. Two layers:
 *
 *  1. Per-op entry points: device-pointer versions of the reference's CPU
 *     kernels on the decode path. Each replaces one `mi_compute_<op>(dst,
 *     ith, nth)` of the reference (src/ops_cpu.h:62-138): the inputs that
 *     kernel reads from dst->src[0..1] and dst->op_params become arguments,
 *     the output it writes to dst->data becomes `dst`. Results are bit-identical
 *     to the reference's AVX2 dispatch path on the same inputs.
 *
 *  2. The Qwen2 decode executor: device-resident replacements for the
 *     reference's model API (src/model_qwen2.h:83-189): weights uploaded to
 *     HBM once, KV cache in HBM, one CUDA graph per decode step.
 *
 * Every function returns MI_CUDA_OK (0) or an error code; the message of the
 * last error on the calling thread is in mi_cuda_last_error(). The reference
 * aborts or asserts in the same situations (src/gallocr.cpp:195-201,
 * src/context.cpp:23); a library must not.
 *
 * Streams are passed as `void*` holding a cudaStream_t (NULL = the legacy
 * default stream). Pointers named d_* are device pointers, h_* host pointers.
 */
#ifndef MI_CUDA_H
#define MI_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MI_CUDA_OK 0
#define MI_CUDA_ERR_ARG 1      /* bad argument (null pointer, bad shape) */
#define MI_CUDA_ERR_CUDA 2     /* a CUDA runtime call failed */
#define MI_CUDA_ERR_IO 3       /* file could not be opened or read */
#define MI_CUDA_ERR_FORMAT 4   /* GGUF content not usable (type, missing tensor) */
#define MI_CUDA_ERR_TIMEOUT 5  /* a bounded device-side wait gave up */
#define MI_CUDA_ERR_STATE 6    /* object used in the wrong state (e.g. n_past >= n_ctx) */

typedef void* mi_cuda_stream;

/* Message of the last error on this thread ("" if none). */
const char* mi_cuda_last_error(void);

/* Selects `device` for the calling thread and loads the device tables the
 * kernels need (the expf exception table, verified against this host's libm).
 * Idempotent per device; every other entry point calls it for the current
 * device on first use. */
int mi_cuda_init(int device);

/* Reads and clears the device error word that bounded waits set when they
 * give up (0 = none, else MI_CUDA_ERR_TIMEOUT). Synchronizes the device. */
int mi_cuda_device_error(int device, int32_t* code_out);

/* ---------------------------------------------------------------------------
 * Q8_0 weights in HBM.
 *
 * GGUF Q8_0 rows (34-byte blocks {fp16 d; int8 qs[32]}, reference
 * src/quant.h:22-28) are repacked once, on the device, into the layout the
 * GEMV streams: rows in groups of 4, for each 32-element block the group's
 * 4 x 32 quant bytes contiguous (128 B), and the fp16 scales in a second plane
 * (4 per group and block). The byte count per weight stays 34/32.
 * ------------------------------------------------------------------------- */

/* Bytes of a packed [k x n] Q8_0 matrix (n rounded up to a multiple of 8). */
size_t mi_cuda_q8_0_packed_bytes(int64_t k, int64_t n);

/* d_raw: n GGUF Q8_0 rows of k elements, in device memory. */
int mi_cuda_q8_0_pack(const void* d_raw, int64_t k, int64_t n, void* d_packed, mi_cuda_stream s);

/* ---------------------------------------------------------------------------
 * Per-op entry points
 * ------------------------------------------------------------------------- */

/* mi_compute_quantize_q8_0 (ref src/ops_cpu.cpp:462-479 ->
 * mi_quantize_row_q8_0_act, src/quant.cpp:199-218): m rows of k F32 -> m rows
 * of k/32 Q8_0_ACT blocks (36 B: float d, int8 qs[32]). */
int mi_cuda_quantize_q8_0_act(const float* d_x, int64_t k, int64_t m, void* d_act,
                              mi_cuda_stream s);

/* mi_compute_mul_mat, Q8_0 weight (ref src/ops_cpu.cpp:177-268, dot =
 * mi_vec_dot_q8_0_wact_avx2_f16c, src/quant_avx2.cpp:170-181):
 * d_dst[j*n + i] = dot(W row i, act row j), act already Q8_0_ACT. */
int mi_cuda_mul_mat_q8_0(const void* d_w_packed, int64_t k, int64_t n, const void* d_act,
                         int64_t m, float* d_dst, mi_cuda_stream s);

/* The pair the reference graph builds for a Q8_0 weight (quantize node +
 * mul_mat node, ref src/graph.cpp:130-144) as one launch: the activation
 * quantize runs in the GEMV's prologue. d_x: m rows of k F32. */
int mi_cuda_mul_mat_q8_0_f32(const void* d_w_packed, int64_t k, int64_t n, const float* d_x,
                             int64_t m, float* d_dst, mi_cuda_stream s);

/* mi_compute_mul_mat with the reference's scalar dot (MI_QUANT_FORCE_SCALAR,
 * ref src/quant.cpp:221-239): d_dst[j*n + i] = fma chain over the blocks of
 * (float)isum * (fp16(w.d) * a.d), one accumulator per row. For parity with a
 * reference run on the scalar path; the decode path uses the AVX2 order. */
int mi_cuda_mul_mat_q8_0_scalar(const void* d_w_packed, int64_t k, int64_t n, const void* d_act,
                                int64_t m, float* d_dst, mi_cuda_stream s);

/* Per-block int32 sums of W row i x act row 0 (sum of the 8 lane partials,
 * ref mi_q8_0_block_isum_avx2, src/quant_avx2.cpp:121-124), computed by the
 * GEMV's own dp4a path: d_isums[i*(k/32) + b]. */
int mi_cuda_q8_0_block_isums(const void* d_w_packed, int64_t k, int64_t n, const void* d_act,
                             int32_t* d_isums, mi_cuda_stream s);

/* mi_compute_get_rows on a Q8_0 table (ref src/ops_cpu.cpp:110-141): the table
 * is a packed [ne0 x n_rows] matrix. */
int mi_cuda_get_rows_q8_0(const void* d_table_packed, int64_t ne0, int64_t n_rows,
                          const int32_t* d_ids, int64_t n_ids, float* d_dst, mi_cuda_stream s);

/* mi_compute_rms_norm (ref src/ops_cpu.cpp:143-165), rows of ne0. */
int mi_cuda_rms_norm(const float* d_x, int64_t ne0, int64_t n_rows, float eps, float* d_dst,
                     mi_cuda_stream s);

/* mi_compute_mul / mi_compute_add (ref src/ops_cpu.cpp:56-80, 167-175):
 * b has b_rows rows of ne0 (1 = broadcast over all n_rows). */
int mi_cuda_mul(const float* d_a, const float* d_b, int64_t ne0, int64_t n_rows, int64_t b_rows,
                float* d_dst, mi_cuda_stream s);
int mi_cuda_add(const float* d_a, const float* d_b, int64_t ne0, int64_t n_rows, int64_t b_rows,
                float* d_dst, mi_cuda_stream s);

/* mi_compute_scale (ref src/ops_cpu.cpp:429-444). */
int mi_cuda_scale(const float* d_x, int64_t n, float v, float* d_dst, mi_cuda_stream s);

/* mi_compute_silu (ref src/ops_cpu.cpp:412-427), libm-exact expf. */
int mi_cuda_silu(const float* d_x, int64_t n, float* d_dst, mi_cuda_stream s);

/* mi_compute_rope, NEOX pairing (ref src/ops_cpu.cpp:270-302):
 * x [n_tokens][n_head][head_dim]. cos/sin come from a host table built with
 * the host libm's powf/cosf/sinf exactly as the reference evaluates them. */
int mi_cuda_rope_neox(const float* d_x, int64_t head_dim, int64_t n_head, int64_t n_tokens,
                      int32_t n_past, int32_t n_dims, float freq_base, float* d_dst,
                      mi_cuda_stream s);

/* mi_compute_attn_qk (ref src/ops_cpu.cpp:356-380): q [n_tokens][n_head][hd],
 * cache_k [n_ctx][n_head_kv][hd]; scores [n_head][n_tokens][n_kv]. */
int mi_cuda_attn_qk(const float* d_q, const float* d_cache_k, int64_t head_dim, int64_t n_head,
                    int64_t n_head_kv, int64_t n_kv, int64_t n_tokens, float* d_scores,
                    mi_cuda_stream s);

/* mi_compute_softmax (ref src/ops_cpu.cpp:304-346): causal, x [n_head][n_tokens][n_kv]. */
int mi_cuda_softmax(const float* d_x, int64_t n_kv, int64_t n_tokens, int64_t n_head,
                    int32_t n_past, float scale, float* d_dst, mi_cuda_stream s);

/* mi_compute_attn_kqv (ref src/ops_cpu.cpp:386-410): probs [n_head][n_tokens][n_kv],
 * cache_v [n_ctx][n_head_kv][hd]; dst [n_tokens][n_head][hd]. */
int mi_cuda_attn_kqv(const float* d_probs, const float* d_cache_v, int64_t head_dim,
                     int64_t n_head, int64_t n_head_kv, int64_t n_kv, int64_t n_tokens,
                     float* d_dst, mi_cuda_stream s);

/* The three attention nodes of one decode step (ref src/model_qwen2.cpp:170-172,
 * n_tokens = 1, n_past = n_kv - 1), every sum in the reference's order: q
 * [n_head][hd] already rotated, caches hold positions [0, n_kv). One launch;
 * from 512 positions (with 16-byte aligned caches and hd a multiple of 4)
 * three launches that spread the scores, the softmax and the ordered value
 * chains over the GPU -- same results. d_scratch holds
 * mi_cuda_attention_decode_scratch_bytes() bytes; dst [n_head][hd]. */
size_t mi_cuda_attention_decode_scratch_bytes(int64_t n_head, int64_t n_kv);
int mi_cuda_attention_decode(const float* d_q, const float* d_cache_k, const float* d_cache_v,
                             int64_t head_dim, int64_t n_head, int64_t n_head_kv, int64_t n_kv,
                             float scale, void* d_scratch, float* d_dst, mi_cuda_stream s);

/* No counterpart in the reference: a fast mode of mi_cuda_attention_decode
 * (same inputs and output layout) that splits the positions over many CTAs and
 * combines their partial softmax sums. The scores are fused dot products, the
 * exponentials CUDA's expf, the denominator and value sums regrouped, so
 * results differ from the reference's in the last bits (within max-abs 1e-5
 * on N(0,1) data). head_dim a power of two <= 128, n_head / n_head_kv <= 16,
 * caches and scratch 16-byte aligned. d_scratch holds
 * mi_cuda_attention_decode_split_scratch_bytes() bytes. */
size_t mi_cuda_attention_decode_split_scratch_bytes(int64_t n_head, int64_t n_head_kv, int64_t n_kv,
                                                    int64_t head_dim);
int mi_cuda_attention_decode_split(const float* d_q, const float* d_cache_k, const float* d_cache_v,
                                   int64_t head_dim, int64_t n_head, int64_t n_head_kv, int64_t n_kv,
                                   float scale, void* d_scratch, float* d_dst, mi_cuda_stream s);

/* No counterpart in the reference. mi_cuda_attention_decode for callers that
 * cannot allocate device memory on their call path (a zero-allocation runtime
 * after start-up, code running while the caller records a CUDA graph, a plugin
 * host that owns all device memory): same inputs, outputs and results, but the
 * score scratch is a 4 MiB array inside the library that every GPU loading the
 * library keeps until exit, so n_head * n_kv may be at most 1,048,576 (larger
 * sizes return MI_CUDA_ERR_ARG). It allocates nothing; mi_cuda_init(device) must
 * have run once before (it loads the expf table), else MI_CUDA_ERR_STATE. The
 * first call on a device looks up the array's device address and may load the
 * module, so make it before any stream capture. All calls on a device share the
 * array: calls that can overlap on the GPU race and must be serialized. */
int mi_cuda_attention_decode_noalloc(const float* d_q, const float* d_cache_k,
                                     const float* d_cache_v, int64_t head_dim, int64_t n_head,
                                     int64_t n_head_kv, int64_t n_kv, float scale, float* d_dst,
                                     mi_cuda_stream s);

/* mi_qwen2_sample_greedy on the device (ref src/model_qwen2.cpp:690-700):
 * first index of the maximum. */
int mi_cuda_argmax(const float* d_x, int64_t n, int32_t* d_out, mi_cuda_stream s);

/* The device expf (libm-exact) on n values; for verification. */
int mi_cuda_expf(const float* d_x, int64_t n, float* d_y, mi_cuda_stream s);

/* Compares the device expf with this host's libm expf on every float whose
 * bit pattern is in [first, first + count); returns the mismatch count. */
int mi_cuda_expf_verify(uint64_t first, uint64_t count, uint64_t* n_mismatch);

/* ---------------------------------------------------------------------------
 * Qwen2 decode executor (ref src/model_qwen2.h:83-189)
 * ------------------------------------------------------------------------- */

typedef struct mi_cuda_model mi_cuda_model;
typedef struct mi_cuda_kv_cache mi_cuda_kv_cache;

typedef struct {
  int32_t n_vocab, n_embd, n_layer, n_head, n_head_kv, n_ff, head_dim, n_ctx_train;
  float rms_eps, rope_freq_base;
} mi_cuda_qwen2_hparams;

/* mi_qwen2_model_load (ref src/model_qwen2.cpp:466-546): reads the GGUF (v3,
 * Q8_0 projection/embedding weights, F32 norms/biases), uploads every weight
 * to HBM once on `device`, and keeps nothing mapped afterwards. */
int mi_cuda_qwen2_model_load(const char* gguf_path, int device, mi_cuda_model** out);

/* Tensor parallelism over the GPUs of one node, one process per GPU
 * (world <= 8). No reference counterpart: the reference is one process on one
 * CPU. Each rank uploads its rows of every projection (stacked QKV, O, the
 * FFN in whole 32-element activation blocks, down, LM head); norms, RoPE and
 * attention are replicated. Row-sharding keeps every output row's arithmetic
 * that of the unsharded GEMV (ref src/ops_cpu.cpp:226-237), so results are
 * bit-identical to world == 1. */
int mi_cuda_qwen2_model_load_shard(const char* gguf_path, int device, int rank, int world,
                                   mi_cuda_model** out);
/* The split used for every matrix: rank r owns units [first, first + count)
 * of n_units (8-row groups; FFN activation blocks). Host-only arithmetic. */
int mi_cuda_tp_shard_range(int64_t n_units, int rank, int world, int64_t* first, int64_t* count);
/* Bytes of one exchange handle (a CUDA IPC memory handle). */
int32_t mi_cuda_ipc_handle_bytes(void);

void mi_cuda_qwen2_model_free(mi_cuda_model* model);
int mi_cuda_qwen2_get_hparams(const mi_cuda_model* model, mi_cuda_qwen2_hparams* out);
/* Bytes of weights resident in HBM. */
size_t mi_cuda_qwen2_weight_bytes(const mi_cuda_model* model);

/* mi_kv_cache_init (ref src/model_qwen2.cpp:557-596): F32 K/V caches
 * [n_ctx][n_head_kv][head_dim] per layer in HBM, the step workspace, and the
 * captured decode-step graphs. */
int mi_cuda_kv_cache_init(mi_cuda_model* model, int32_t n_ctx, mi_cuda_kv_cache** out);
void mi_cuda_kv_cache_free(mi_cuda_kv_cache* kv);

/* KV cache of a sharded model: mi_cuda_kv_cache_init allocates its exchange
 * buffer (words that every rank's GEMV epilogues store into over NVLink) but
 * captures no step graph. Send this rank's handle to every rank, then call
 * mi_cuda_tp_connect with all ranks' handles concatenated in rank order: it
 * maps the peers' buffers and captures the graphs. From then on every rank
 * must issue the same sequence of steps; a rank that stops makes the others'
 * bounded device waits expire (MI_CUDA_ERR_TIMEOUT). */
int mi_cuda_tp_exchange_handle(mi_cuda_kv_cache* kv, void* handle_out);
int mi_cuda_tp_connect(mi_cuda_kv_cache* kv, const void* handles);

/* mi_qwen2_forward (ref src/model_qwen2.cpp:609-688): runs n_tokens tokens
 * starting at position n_past, writes their K/V rows, and copies logits to
 * h_logits_out (n_tokens * n_vocab floats, or n_vocab if last_logits_only;
 * may be NULL). Like the reference, the caller tracks n_past. */
int mi_cuda_qwen2_forward(mi_cuda_model* model, mi_cuda_kv_cache* kv, const int32_t* h_tokens,
                          int32_t n_tokens, int32_t n_past, int32_t last_logits_only,
                          float* h_logits_out);

/* Greedy token of the last forward (device argmax of its last logits row), or
 * of the last device-resident step. Right after mi_cuda_qwen2_forward,
 * _generate or _read_tokens it comes from the state those calls already read
 * back (no device round trip); otherwise it waits for the stream. */
int mi_cuda_qwen2_last_token(mi_cuda_kv_cache* kv, int32_t* h_token_out);

/* mi_qwen2_sample_greedy (ref src/model_qwen2.cpp:690-700), on host logits. */
int32_t mi_cuda_qwen2_sample_greedy(const float* h_logits, int32_t n_vocab);

/* The reference CLI's --bench generation (ref src/main.cpp:372-424) with the
 * greedy token fed back on the device: prompt forward, then n_predict - 1
 * single-token decode steps. Writes n_predict tokens. Timings in ms. */
int mi_cuda_qwen2_generate(mi_cuda_model* model, mi_cuda_kv_cache* kv, const int32_t* h_prompt,
                           int32_t n_prompt, int32_t n_predict, int32_t* h_tokens_out,
                           double* prefill_ms, double* decode_ms);

/* Device-resident stepping, for timing without host round trips:
 * set_position uploads h_tokens to positions [0, n) of the token buffer and
 * sets the position to `pos`; decode_steps replays n_steps decode-step graphs
 * on the executor's stream, each embedding token[pos], writing the greedy
 * token to token[pos + 1] and advancing pos. With period > 0 the position is
 * reset to pos0 on the device after every `period` steps, so a long run
 * revisits the same positions (and regenerates the same tokens).
 * Asynchronous. */
int mi_cuda_qwen2_set_position(mi_cuda_kv_cache* kv, const int32_t* h_tokens, int32_t n,
                               int32_t pos);
int mi_cuda_qwen2_decode_steps(mi_cuda_kv_cache* kv, int32_t n_steps, int32_t pos0,
                               int32_t period);
int mi_cuda_qwen2_read_tokens(mi_cuda_kv_cache* kv, int32_t first, int32_t n, int32_t* h_out);
/* Step trace (the reference's barrier statistics, src/threadpool.cpp:78-81,
 * become device timestamps): for each kernel of the most recent decode step,
 * 8 globaltimer stamps (ns) from its first CTA -- entry, predecessor done
 * (dependency wait returned), prologue done, epilogue start, then up to four
 * kernel-specific phase marks (attention: scores, exp, sum, KV done; 0 when
 * unused). Copies up to max_slots kernels x 8 stamps into h_out; *n_slots =
 * slots copied. */
int mi_cuda_qwen2_step_trace(mi_cuda_kv_cache* kv, uint64_t* h_out, int32_t max_slots,
                             int32_t* n_slots);

/* The executor's CUDA stream (cudaStream_t) and its per-step kernel count. */
mi_cuda_stream mi_cuda_qwen2_stream(mi_cuda_kv_cache* kv);
int32_t mi_cuda_qwen2_kernels_per_step(mi_cuda_kv_cache* kv);

/* No counterpart in the reference: a labelled FAST MODE of the decode step
 * (on = 1), for measuring how close the step's design comes to the bandwidth
 * roofline without the reference's sequential sums. Same schedule and
 * kernel as the persistent step, but rms_norm's sum of squares and the
 * softmax denominator are block trees, the attention value sums and the
 * down projection's dot products are split over thread groups, and the
 * softmax uses CUDA's expf. Results are NOT bit-identical to the reference
 * (greedy tokens can differ where the top two logits are close); on = 0
 * restores the exact step. Applies to decode steps only (a batched prompt
 * stays exact). MI_CUDA_ERR_STATE where the persistent step is not in use
 * (tensor parallelism, shapes it does not support, MI_CUDA_PERSIST=0). */
int mi_cuda_qwen2_set_fast_mode(mi_cuda_kv_cache* kv, int32_t on);
int32_t mi_cuda_qwen2_fast_mode(mi_cuda_kv_cache* kv);

#ifdef __cplusplus
}
#endif

#endif /* MI_CUDA_H */
