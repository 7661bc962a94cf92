// A flat extern "C" face over the reference's model API with the ops_cuda
// backend plugged in, for ctypes callers (the drop-in tests). It is the
// reference's own sequence -- mi_qwen2_model_load, mi_kv_cache_init (gallocr
// reserve), mi_qwen2_forward per step (graph build, gallocr plan, execute) --
// with mi_ops_cuda_attach between the KV-cache init and the first forward,
// which is the one call a host program adds to run on the GPU.
#include <cstdint>
#include <cstring>
#include <string>

#include "gallocr.h"
#include "model_qwen2.h"
#include "ops_cuda.h"
#include "threadpool.h"

namespace {

struct Session {
  mi_qwen2_model* model = nullptr;
  mi_kv_cache* kv = nullptr;
};

thread_local std::string g_err;

void set_err(char* buf, int len, const std::string& msg) {
  g_err = msg;
  if (buf && len > 0) {
    std::strncpy(buf, msg.c_str(), (size_t)len - 1);
    buf[len - 1] = 0;
  }
}

}  // namespace

extern "C" {

const char* mirc_last_error() { return g_err.c_str(); }

// device >= 0: attach the device backend on that GPU; device < 0: the
// reference's CPU threadpool with n_threads threads.
void* mirc_open(const char* gguf_path, int n_ctx, int n_threads, int device, char* err, int err_len) {
  std::string e;
  auto* s = new Session();
  s->model = mi_qwen2_model_load(gguf_path, &e);
  if (!s->model) {
    set_err(err, err_len, "model load: " + e);
    delete s;
    return nullptr;
  }
  mi_threadpool_params tp{n_threads > 0 ? n_threads : 1, false, MI_MULMAT_STATIC, 8};
  s->kv = mi_kv_cache_init(s->model->hparams, s->model->weights, n_ctx, tp);
  if (device >= 0 && !mi_ops_cuda_attach(s->model, s->kv, device, &e)) {
    set_err(err, err_len, "ops_cuda attach: " + e);
    mi_kv_cache_free(s->kv);
    mi_qwen2_model_free(s->model);
    delete s;
    return nullptr;
  }
  return s;
}

int mirc_n_vocab(void* h) { return ((Session*)h)->model->hparams.n_vocab; }

int64_t mirc_arena_size(void* h) { return (int64_t)((Session*)h)->kv->galloc->arena_size; }

void mirc_forward(void* h, const int32_t* tokens, int n_tokens, int n_past, int last_logits_only, float* logits) {
  auto* s = (Session*)h;
  mi_qwen2_forward_params p{};
  p.tokens = tokens;
  p.n_tokens = n_tokens;
  p.n_past = n_past;
  p.last_logits_only = last_logits_only != 0;
  mi_qwen2_forward(s->model, s->kv, p, logits);
  s->kv->n_past = n_past + n_tokens;
}

// out[0..7] = steps, nodes, views_skipped, arena_bytes, arena_tensors,
// instantiations, updates, weight_bytes (mi_ops_cuda_stats).
void mirc_stats(int64_t* out) {
  mi_ops_cuda_stats st = mi_ops_cuda_get_stats();
  const int64_t v[8] = {st.steps, st.nodes, st.views_skipped, st.arena_bytes, st.arena_tensors,
                        st.instantiations, st.updates, st.weight_bytes};
  std::memcpy(out, v, sizeof(v));
}

void mirc_close(void* h) {
  auto* s = (Session*)h;
  if (!s) return;
  if (mi_ops_cuda_attached()) mi_ops_cuda_detach();
  mi_kv_cache_free(s->kv);
  mi_qwen2_model_free(s->model);
  delete s;
}

}  // extern "C"
