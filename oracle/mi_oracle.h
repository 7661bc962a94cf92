/* TEST INFRASTRUCTURE ONLY -- the CPU oracle (checker), never the product.
 *
 * Plain-C restatement of the reference's single-request decode path
 * (GuoHaojiee/mini-infer-llama.cpp, src/ops_cpu.cpp, src/quant.cpp,
 * src/quant_avx2.cpp, src/model_qwen2.cpp). Every function reproduces the
 * reference's IEEE operation order so its outputs are bit-identical to the
 * reference's AVX2 dispatch path; tests/test_oracle_pin.py pins it against
 * the reference compiled from source (oracle/_ref/libmi_ref.so) and against
 * the reference tests' known-answer cases.
 *
 * Layouts (ne[0] innermost, as the reference's tensor.h:125-128):
 *   Q8_0 block      34 B: {uint16 fp16 d; int8 qs[32]}   (quant.h:22-28)
 *   Q8_0_ACT block  36 B: {float d; int8 qs[32]}         (quant.h:121-127)
 *   KV cache        F32 [head_dim, n_head_kv, n_ctx]      (model_qwen2.cpp:564-578)
 */
#ifndef MI_ORACLE_H
#define MI_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

float mio_fp16_to_fp32(uint16_t h);
uint16_t mio_fp32_to_fp16(float f);

void mio_quantize_row_q8_0_act(const float* x, uint8_t* y, int64_t n);
void mio_quantize_row_q8_0(const float* x, uint8_t* y, int64_t n);
void mio_dequantize_row_q8_0(const uint8_t* x, float* y, int64_t n);

int32_t mio_block_isum(const int8_t* x, const int8_t* y);
void mio_block_lanes(const int8_t* x, const int8_t* y, int32_t lanes[8]);
float mio_vec_dot_q8_0_wact(const uint8_t* w, const uint8_t* a, int64_t n);
float mio_vec_dot_q8_0_wact_scalar(const uint8_t* w, const uint8_t* a, int64_t n);

/* dst[n, m] = W[k, n]^T . act[k, m] with W Q8_0 rows and act Q8_0_ACT rows. */
void mio_mul_mat_q8_0(const uint8_t* w, int64_t k, int64_t n, const uint8_t* act, int64_t m,
                      float* dst);
void mio_get_rows_q8_0(const uint8_t* table, int64_t ne0, const int32_t* ids, int64_t n_ids,
                       float* dst);
void mio_rms_norm(const float* x, int64_t ne0, int64_t n_rows, float eps, float* dst);
void mio_mul_row(const float* a, const float* b, int64_t ne0, int64_t n_rows, int b_bcast,
                 float* dst);
void mio_add_row(const float* a, const float* b, int64_t ne0, int64_t n_rows, int b_bcast,
                 float* dst);
void mio_silu(const float* x, int64_t n, float* dst);
void mio_rope_neox(const float* x, int64_t head_dim, int64_t n_head, int64_t n_tokens,
                   int32_t n_past, int32_t n_dims, float freq_base, float* dst);
void mio_attn_qk(const float* q, const float* cache_k, int64_t head_dim, int64_t n_head,
                 int64_t n_head_kv, int64_t n_kv, int64_t n_tokens, float* scores);
void mio_softmax(const float* x, int64_t n_kv, int64_t n_tokens, int64_t n_head, int32_t n_past,
                 float scale, float* dst);
void mio_attn_kqv(const float* probs, const float* cache_v, int64_t head_dim, int64_t n_head,
                  int64_t n_head_kv, int64_t n_kv, int64_t n_tokens, float* dst);
float mio_expf(float x);

/* Whole-model restatement (model_qwen2.cpp:133-267, 609-700). */
typedef struct {
  int32_t n_vocab, n_embd, n_layer, n_head, n_head_kv, n_ff, head_dim;
  float rms_eps, rope_freq_base;
} mio_hparams;

typedef struct {
  const float* attn_norm;
  const uint8_t* wq;
  const float* bq;
  const uint8_t* wk;
  const float* bk;
  const uint8_t* wv;
  const float* bv;
  const uint8_t* wo;
  const float* ffn_norm;
  const uint8_t* wgate;
  const uint8_t* wup;
  const uint8_t* wdown;
} mio_layer;

typedef struct {
  const uint8_t* token_embd; /* Q8_0 [n_embd, n_vocab] */
  const float* output_norm;
  const uint8_t* output;     /* Q8_0 [n_embd, n_vocab]; == token_embd when tied */
  const mio_layer* layers;
} mio_weights;

/* cache_k/cache_v: n_layer pointers to F32 [head_dim, n_head_kv, n_ctx].
 * logits: n_tokens*n_vocab floats, or n_vocab when last_logits_only.
 * layer_out (optional): n_layer * n_embd * n_tokens floats. */
void mio_qwen2_forward(const mio_hparams* hp, const mio_weights* w, float* const* cache_k,
                       float* const* cache_v, int32_t n_ctx, const int32_t* tokens,
                       int32_t n_tokens, int32_t n_past, int32_t last_logits_only,
                       float* logits, float* layer_out);
int32_t mio_sample_greedy(const float* logits, int32_t n_vocab);

#ifdef __cplusplus
}
#endif

#endif
