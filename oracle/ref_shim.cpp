// TEST INFRASTRUCTURE ONLY -- part of the CPU oracle, never linked into the
// product library. Only tests/, __graft_entry__.smoke() and bench.py's
// cpu_baseline / --impl reference legs load the library this file is built
// into (oracle/_ref/libmi_ref.so).
//
// A flat extern "C" face over the reference's own, unmodified CPU code, which
// oracle/Makefile compiles from the reference sources with the reference's
// Release flags. Each wrapper builds eager mi_tensor values exactly the way
// the reference's own tests do (tests/test_ops_cpu.cpp:26-306) and calls the
// reference kernel, so the numbers that come back ARE the reference's.
//
// Reference entry points wrapped here (paths relative to the reference repo):
//   mi_quantize_row_q8_0_act ........ src/quant.cpp:199-218
//   mi_vec_dot_q8_0_wact[_scalar] ... src/quant.cpp:221-239, src/quant_avx2.cpp:170-200
//   mi_q8_0_block_isum_{scalar,avx2}  src/quant.cpp:165-171, src/quant_avx2.cpp:121-124
//   mi_compute_* ops ................ src/ops_cpu.cpp:110-479
//   mi_qwen2_model_load / mi_kv_cache_init / mi_qwen2_forward /
//   mi_qwen2_sample_greedy ......... src/model_qwen2.cpp:466-700
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "context.h"
#include "model_qwen2.h"
#include "ops_cpu.h"
#include "quant.h"
#include "tensor.h"
#include "threadpool.h"

namespace {

// A scratch eager context big enough for the tensors one wrapper needs. The
// data pointers of the tensors it hands out are replaced by caller buffers
// via from_data, so its own arena only holds metadata.
struct scratch_ctx {
  mi_context* ctx;
  explicit scratch_ctx(size_t n_tensors = 16) {
    mi_context_params p{};
    p.tensor_capacity = n_tensors;
    p.data_capacity = 0;
    p.no_alloc = true;
    ctx = mi_context_new(p);
  }
  ~scratch_ctx() { mi_context_free(ctx); }
  mi_tensor* wrap(mi_type type, int n_dims, const int64_t* ne, void* data) {
    return mi_context_new_tensor_from_data(ctx, type, n_dims, ne, data);
  }
};

thread_local std::string g_last_error;

}  // namespace

extern "C" {

const char* mi_ref_last_error() { return g_last_error.c_str(); }

// ---- quant.h -------------------------------------------------------------

void mi_ref_quantize_row_q8_0_act(const float* x, void* y, int64_t n) {
  mi_quantize_row_q8_0_act(x, (block_q8_0_act*)y, n);
}

void mi_ref_quantize_row_q8_0(const float* x, void* y, int64_t n) {
  mi_quantize_row_q8_0(x, (block_q8_0*)y, n);
}

float mi_ref_vec_dot_q8_0_wact(const void* w, const void* a, int64_t n) {
  return mi_vec_dot_q8_0_wact((const block_q8_0*)w, (const block_q8_0_act*)a, n);
}

float mi_ref_vec_dot_q8_0_wact_scalar(const void* w, const void* a, int64_t n) {
  return mi_vec_dot_q8_0_wact_scalar((const block_q8_0*)w, (const block_q8_0_act*)a, n);
}

int32_t mi_ref_block_isum_scalar(const int8_t* x, const int8_t* y) {
  return mi_q8_0_block_isum_scalar(x, y);
}

int32_t mi_ref_block_isum_avx2(const int8_t* x, const int8_t* y) {
  return mi_q8_0_block_isum_avx2(x, y);
}

float mi_ref_fp16_to_fp32(uint16_t h) { return mi_fp16_to_fp32(h); }

// ---- ops_cpu.h, through mi_compute_forward ---------------------------------

// dst[n, m] = W[k, n]^T . X[k, m]: the quantize node + mul_mat node pair that
// mi_graph_mul_mat builds for a Q8_0 weight (src/graph.cpp:130-144). act_out
// (m * k/32 * 36 bytes) receives the Q8_0_ACT bytes, out the F32 result.
void mi_ref_mul_mat_q8_0(const void* w, int64_t k, int64_t n, const float* x, int64_t m,
                         void* act_out, float* out) {
  scratch_ctx sc;
  int64_t ne_w[2] = {k, n};
  int64_t ne_x[2] = {k, m};
  int64_t ne_o[2] = {n, m};
  mi_tensor* tw = sc.wrap(MI_TYPE_Q8_0, 2, ne_w, (void*)w);
  mi_tensor* tx = sc.wrap(MI_TYPE_F32, 2, ne_x, (void*)x);
  mi_tensor* tq = sc.wrap(MI_TYPE_Q8_0_ACT, 2, ne_x, act_out);
  tq->op = MI_OP_QUANTIZE_Q8_0;
  tq->src[0] = tx;
  mi_compute_forward(tq, 0, 1);
  mi_tensor* to = sc.wrap(MI_TYPE_F32, 2, ne_o, out);
  to->op = MI_OP_MUL_MAT;
  to->src[0] = tw;
  to->src[1] = tq;
  mi_compute_forward(to, 0, 1);
}

// The three attention nodes of one layer (src/model_qwen2.cpp:170-172) on
// eager tensors: q [head_dim, n_head, n_tokens], caches [head_dim, n_head_kv,
// n_ctx]. scores/probs are [n_kv, n_tokens, n_head], out [head_dim, n_head,
// n_tokens]; n_kv = n_past + n_tokens.
void mi_ref_attention(const float* q, const float* cache_k, const float* cache_v, int64_t head_dim,
                      int64_t n_head, int64_t n_head_kv, int64_t n_ctx, int32_t n_past,
                      int64_t n_tokens, float scale, float* scores, float* probs, float* out) {
  scratch_ctx sc;
  int64_t n_kv = n_past + n_tokens;
  int32_t n_rep = (int32_t)(n_head / n_head_kv);
  int64_t ne_q[3] = {head_dim, n_head, n_tokens};
  int64_t ne_c[3] = {head_dim, n_head_kv, n_ctx};
  int64_t ne_s[3] = {n_kv, n_tokens, n_head};
  mi_tensor* tq = sc.wrap(MI_TYPE_F32, 3, ne_q, (void*)q);
  mi_tensor* tk = sc.wrap(MI_TYPE_F32, 3, ne_c, (void*)cache_k);
  mi_tensor* tv = sc.wrap(MI_TYPE_F32, 3, ne_c, (void*)cache_v);
  mi_tensor* ts = sc.wrap(MI_TYPE_F32, 3, ne_s, scores);
  ts->op = MI_OP_ATTN_QK;
  ts->src[0] = tq;
  ts->src[1] = tk;
  mi_op_params_set_i32(ts, 0, n_past);
  mi_op_params_set_i32(ts, 1, n_rep);
  mi_compute_forward(ts, 0, 1);
  mi_tensor* tp = sc.wrap(MI_TYPE_F32, 3, ne_s, probs);
  tp->op = MI_OP_SOFTMAX;
  tp->src[0] = ts;
  mi_op_params_set_i32(tp, 0, n_past);
  mi_op_params_set_f32(tp, 1, scale);
  mi_compute_forward(tp, 0, 1);
  mi_tensor* to = sc.wrap(MI_TYPE_F32, 3, ne_q, out);
  to->op = MI_OP_ATTN_KQV;
  to->src[0] = tp;
  to->src[1] = tv;
  mi_op_params_set_i32(to, 0, n_rep);
  mi_compute_forward(to, 0, 1);
}

// Generic single-op runner for the element-wise / row ops: op is an mi_op
// value, x is [ne0, ne1, ne2] F32, y (optional) is the second operand with its
// own shape, params are the op_params slots (up to 3 i32/f32 bit patterns).
void mi_ref_unary_op(int32_t op, const float* x, int64_t ne0, int64_t ne1, int64_t ne2,
                     const float* y, int64_t yne0, int64_t yne1, int64_t yne2,
                     const int32_t* params, int32_t n_params, float* out) {
  scratch_ctx sc;
  int64_t ne_x[3] = {ne0, ne1, ne2};
  int64_t ne_y[3] = {yne0, yne1, yne2};
  mi_tensor* tx = sc.wrap(MI_TYPE_F32, 3, ne_x, (void*)x);
  mi_tensor* to = sc.wrap(MI_TYPE_F32, 3, ne_x, out);
  to->op = (mi_op)op;
  to->src[0] = tx;
  if (y) to->src[1] = sc.wrap(MI_TYPE_F32, 3, ne_y, (void*)y);
  for (int i = 0; i < n_params && i < MI_MAX_OP_PARAMS; i++) to->op_params[i] = params[i];
  mi_compute_forward(to, 0, 1);
}

// get_rows on a Q8_0 table [ne0, n_rows] (src/ops_cpu.cpp:110-141).
void mi_ref_get_rows_q8_0(const void* table, int64_t ne0, int64_t n_rows, const int32_t* ids,
                          int64_t n_ids, float* out) {
  scratch_ctx sc;
  int64_t ne_t[2] = {ne0, n_rows};
  int64_t ne_i[1] = {n_ids};
  int64_t ne_o[2] = {ne0, n_ids};
  mi_tensor* tt = sc.wrap(MI_TYPE_Q8_0, 2, ne_t, (void*)table);
  mi_tensor* ti = sc.wrap(MI_TYPE_I32, 1, ne_i, (void*)ids);
  mi_tensor* to = sc.wrap(MI_TYPE_F32, 2, ne_o, out);
  to->op = MI_OP_GET_ROWS;
  to->src[0] = tt;
  to->src[1] = ti;
  mi_compute_forward(to, 0, 1);
}

// ---- model_qwen2.h ---------------------------------------------------------

struct mi_ref_session {
  mi_qwen2_model* model;
  mi_kv_cache* kv;
};

void* mi_ref_model_open(const char* gguf_path, int32_t n_ctx, int32_t n_threads) {
  std::string err;
  mi_qwen2_model* model = mi_qwen2_model_load(gguf_path, &err);
  if (!model) {
    g_last_error = err;
    return nullptr;
  }
  mi_threadpool_params tp{n_threads > 0 ? n_threads : 1, true, MI_MULMAT_STATIC, 8};
  mi_kv_cache* kv = mi_kv_cache_init(model->hparams, model->weights, n_ctx, tp);
  auto* s = new mi_ref_session{model, kv};
  return s;
}

void mi_ref_model_close(void* h) {
  auto* s = (mi_ref_session*)h;
  if (!s) return;
  mi_kv_cache_free(s->kv);
  mi_qwen2_model_free(s->model);
  delete s;
}

// hp[0..9] = n_vocab, n_embd, n_layer, n_head, n_head_kv, n_ff, head_dim,
// n_ctx_train, bits(rms_eps), bits(rope_freq_base)
void mi_ref_model_hparams(void* h, int32_t* hp) {
  auto* s = (mi_ref_session*)h;
  const mi_qwen2_hparams& p = s->model->hparams;
  hp[0] = p.n_vocab;
  hp[1] = p.n_embd;
  hp[2] = p.n_layer;
  hp[3] = p.n_head;
  hp[4] = p.n_head_kv;
  hp[5] = p.n_ff;
  hp[6] = p.head_dim;
  hp[7] = p.n_ctx_train;
  std::memcpy(&hp[8], &p.rms_eps, 4);
  std::memcpy(&hp[9], &p.rope_freq_base, 4);
}

// One mi_qwen2_forward call; logits_out gets n_tokens*n_vocab floats (or
// n_vocab with last_logits_only). kv->n_past is left for the caller, as in
// the reference (src/model_qwen2.h:181-187).
void mi_ref_forward(void* h, const int32_t* tokens, int32_t n_tokens, int32_t n_past,
                    int32_t last_logits_only, float* logits_out) {
  auto* s = (mi_ref_session*)h;
  mi_qwen2_forward_params fp{};
  fp.tokens = tokens;
  fp.n_tokens = n_tokens;
  fp.n_past = n_past;
  fp.last_logits_only = last_logits_only != 0;
  mi_qwen2_forward(s->model, s->kv, fp, logits_out);
}

int32_t mi_ref_sample_greedy(const float* logits, int32_t n_vocab) {
  return mi_qwen2_sample_greedy(logits, n_vocab);
}

// Dump hook: copies the "layer_{i}" checkpoint of one forward call into
// layer_out[i * n_embd * n_tokens ...] and "output_norm" into norm_out.
namespace {
struct dump_target {
  float* layers;
  float* norm;
  int64_t per;
};
void on_dump(void* ud, const char* name, const mi_tensor* t) {
  auto* d = (dump_target*)ud;
  int64_t n = mi_nelements(t);
  if (std::strncmp(name, "layer_", 6) == 0 && d->layers) {
    int l = std::atoi(name + 6);
    std::memcpy(d->layers + (int64_t)l * d->per, t->data, (size_t)n * 4);
  } else if (std::strcmp(name, "output_norm") == 0 && d->norm) {
    std::memcpy(d->norm, t->data, (size_t)n * 4);
  }
}
}  // namespace

void mi_ref_forward_dump(void* h, const int32_t* tokens, int32_t n_tokens, int32_t n_past,
                         float* layers_out, float* norm_out, float* logits_out) {
  auto* s = (mi_ref_session*)h;
  dump_target d{layers_out, norm_out, (int64_t)s->model->hparams.n_embd * n_tokens};
  mi_dump_sink sink{&on_dump, &d};
  mi_qwen2_forward_params fp{};
  fp.tokens = tokens;
  fp.n_tokens = n_tokens;
  fp.n_past = n_past;
  fp.dump = &sink;
  mi_qwen2_forward(s->model, s->kv, fp, logits_out);
}

// The reference CLI's --bench generation loop (src/main.cpp:372-424): one
// last_logits_only prefill over the prompt, then n_predict-1 decode forwards
// each fed the greedy token of the previous one. Writes the n_predict greedy
// tokens and the two timings (ms) the CLI prints.
int32_t mi_ref_generate(void* h, const int32_t* prompt, int32_t n_prompt, int32_t n_predict,
                        int32_t* tokens_out, double* prefill_ms, double* decode_ms) {
  auto* s = (mi_ref_session*)h;
  int n_vocab = s->model->hparams.n_vocab;
  std::vector<float> logits((size_t)n_vocab);
  mi_qwen2_forward_params fp{};
  fp.tokens = prompt;
  fp.n_tokens = n_prompt;
  fp.n_past = 0;
  fp.last_logits_only = true;
  auto t0 = std::chrono::steady_clock::now();
  mi_qwen2_forward(s->model, s->kv, fp, logits.data());
  auto t1 = std::chrono::steady_clock::now();
  *prefill_ms = std::chrono::duration<double, std::milli>(t1 - t0).count();
  s->kv->n_past = n_prompt;
  int32_t next_id = mi_qwen2_sample_greedy(logits.data(), n_vocab);
  double dms = 0.0;
  int produced = 0;
  for (int step = 0; step < n_predict; step++) {
    tokens_out[produced++] = next_id;
    if (step + 1 == n_predict) break;
    if (s->kv->n_past >= s->kv->n_ctx) break;
    mi_qwen2_forward_params sp{};
    sp.tokens = &next_id;
    sp.n_tokens = 1;
    sp.n_past = s->kv->n_past;
    auto d0 = std::chrono::steady_clock::now();
    mi_qwen2_forward(s->model, s->kv, sp, logits.data());
    auto d1 = std::chrono::steady_clock::now();
    dms += std::chrono::duration<double, std::milli>(d1 - d0).count();
    s->kv->n_past += 1;
    next_id = mi_qwen2_sample_greedy(logits.data(), n_vocab);
  }
  *decode_ms = dms;
  return produced;
}

void mi_ref_set_n_past(void* h, int32_t n_past) { ((mi_ref_session*)h)->kv->n_past = n_past; }

}  // extern "C"
