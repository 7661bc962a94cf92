// ops_cuda: device executor under the reference's mi_graph_compute (see
// ops_cuda.h). Every compute node of the reference's scheduled graph maps to
// one call of the backend's per-op C-ABI (include/mi_cuda.h), each of which
// replaces one mi_compute_<op> (src/ops_cpu.cpp:481-530) bit for bit.
#include "ops_cuda.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <unordered_map>
#include <vector>

#include "gallocr.h"
#include "mi_cuda.h"
#include "ops_cpu.h"
#include "tensor.h"

namespace {

struct Staged {
  void* d = nullptr;
  size_t bytes = 0;
};

struct Backend {
  int device = 0;
  cudaStream_t stream = nullptr;
  mi_qwen2_model* model = nullptr;
  mi_kv_cache* kv = nullptr;
  const uint8_t* h_arena = nullptr;  // gallocr's host arena (the plan's base)
  uint8_t* d_arena = nullptr;        // its device twin
  size_t arena_bytes = 0;
  // WEIGHT and KV leaves: device copies (Q8_0 matrices packed for the GEMV)
  std::unordered_map<const mi_tensor*, void*> dev;
  std::vector<void*> owned;
  // INPUT / OUTPUT tensors live in host memory the graph context hands out
  // (the same bump-allocated addresses every step): device staging buffers
  // keyed by that host address, grown on demand outside the capture
  std::unordered_map<const void*, Staged> staged;
  cudaGraphExec_t exec = nullptr;
  mi_ops_cuda_stats st{};
};

Backend* g_be = nullptr;

[[noreturn]] void die(const char* what, const char* msg) {
  std::fprintf(stderr, "ops_cuda: %s: %s\n", what, msg);
  std::abort();
}
void ck(int rc, const char* what) {
  if (rc != MI_CUDA_OK) die(what, mi_cuda_last_error());
}
void ckc(cudaError_t e, const char* what) {
  if (e != cudaSuccess) die(what, cudaGetErrorString(e));
}

bool fail(std::string* err, const std::string& msg) {
  if (err) *err = msg;
  return false;
}

int64_t n_rows(const mi_tensor* t) { return t->ne[1] * t->ne[2] * t->ne[3]; }

// Dense layout in the reference's sense: nb[0] one element (block), every
// higher stride the product of the lower extents (dims of extent 1 free).
bool contiguous(const mi_tensor* t) {
  const size_t bs = mi_type_block_size(t->type);
  if (t->nb[0] != mi_type_block_bytes(t->type) || t->ne[0] % (int64_t)bs != 0) return false;
  size_t s = t->nb[0] * (size_t)(t->ne[0] / (int64_t)bs);
  for (int i = 1; i < MI_MAX_DIMS; i++) {
    if (t->ne[i] > 1 && t->nb[i] != s) return false;
    s *= (size_t)t->ne[i];
  }
  return true;
}

// Device address of a tensor's data: an uploaded leaf (plus a view's
// offset), the arena twin at gallocr's planned offset, or a staging buffer.
void* resolve(Backend& b, const mi_tensor* t) {
  const mi_tensor* base = t->view_src ? t->view_src : t;
  const size_t off = t->view_src ? t->view_offs : 0;
  auto it = b.dev.find(base);
  if (it != b.dev.end()) return (uint8_t*)it->second + off;
  const uint8_t* h = (const uint8_t*)t->data;
  if (h && h >= b.h_arena && h < b.h_arena + b.arena_bytes) {
    b.st.arena_tensors++;
    return b.d_arena + (h - b.h_arena);
  }
  auto s = b.staged.find(base->data);
  if (s != b.staged.end()) return (uint8_t*)s->second.d + off;
  die("resolve", t->name[0] ? t->name : "tensor outside the arena, the weights, the KV cache and the staged I/O");
}

void* stage(Backend& b, const mi_tensor* t) {
  Staged& s = b.staged[t->data];
  const size_t need = mi_nbytes(t);
  if (s.bytes < need) {
    if (s.d) ckc(cudaFree(s.d), "cudaFree");
    s.d = nullptr;
    ckc(cudaMalloc(&s.d, need), "cudaMalloc (staging)");
    s.bytes = need;
  }
  return s.d;
}

// One exec node -> one device call on `s`. Operand layouts are the
// reference's (ne[0] innermost, dense); anything else is refused loudly.
void dispatch(Backend& b, mi_tensor* n, cudaStream_t s) {
  mi_tensor* a = n->src[0];
  mi_tensor* c = n->src[1];
  if (!contiguous(n) || (a && !contiguous(a)) || (c && !contiguous(c)))
    die(mi_op_name(n->op), "strided operand (the device ops take dense tensors)");
  float* dst = (float*)resolve(b, n);
  const mi_cuda_stream st = (mi_cuda_stream)s;
  switch (n->op) {
    case MI_OP_GET_ROWS:
      if (a->type != MI_TYPE_Q8_0 || c->type != MI_TYPE_I32) die("get_rows", "table must be Q8_0, ids I32");
      ck(mi_cuda_get_rows_q8_0(resolve(b, a), a->ne[0], a->ne[1], (const int32_t*)resolve(b, c), c->ne[0], dst,
                               st),
         "get_rows");
      break;
    case MI_OP_RMS_NORM:
      ck(mi_cuda_rms_norm((const float*)resolve(b, a), a->ne[0], n_rows(a), mi_op_params_get_f32(n, 0), dst, st),
         "rms_norm");
      break;
    case MI_OP_MUL:
    case MI_OP_ADD: {
      const int64_t rows = n_rows(a), b_rows = n_rows(c);
      if (c->ne[0] != a->ne[0] || (b_rows != 1 && b_rows != rows)) die(mi_op_name(n->op), "broadcast shape");
      const float* pa = (const float*)resolve(b, a);
      const float* pb = (const float*)resolve(b, c);
      ck(n->op == MI_OP_MUL ? mi_cuda_mul(pa, pb, a->ne[0], rows, b_rows, dst, st)
                            : mi_cuda_add(pa, pb, a->ne[0], rows, b_rows, dst, st),
         mi_op_name(n->op));
      break;
    }
    case MI_OP_QUANTIZE_Q8_0:
      if (a->type != MI_TYPE_F32 || n->type != MI_TYPE_Q8_0_ACT) die("quantize", "F32 -> Q8_0_ACT only");
      ck(mi_cuda_quantize_q8_0_act((const float*)resolve(b, a), a->ne[0], n_rows(a), dst, st), "quantize");
      break;
    case MI_OP_MUL_MAT:
      if (a->type != MI_TYPE_Q8_0 || c->type != MI_TYPE_Q8_0_ACT)
        die("mul_mat", "the device GEMV takes Q8_0 weights times Q8_0_ACT activations");
      ck(mi_cuda_mul_mat_q8_0(resolve(b, a), a->ne[0], a->ne[1], resolve(b, c), c->ne[1], dst, st), "mul_mat");
      break;
    case MI_OP_ROPE:
      ck(mi_cuda_rope_neox((const float*)resolve(b, a), a->ne[0], a->ne[1], a->ne[2], mi_op_params_get_i32(n, 0),
                           mi_op_params_get_i32(n, 1), mi_op_params_get_f32(n, 2), dst, st),
         "rope");
      break;
    case MI_OP_SOFTMAX:
      ck(mi_cuda_softmax((const float*)resolve(b, a), a->ne[0], a->ne[1], a->ne[2], mi_op_params_get_i32(n, 0),
                         mi_op_params_get_f32(n, 1), dst, st),
         "softmax");
      break;
    case MI_OP_ATTN_QK:
      if (a->ne[1] != c->ne[1] * mi_op_params_get_i32(n, 1)) die("attn_qk", "n_head != n_head_kv * n_rep");
      ck(mi_cuda_attn_qk((const float*)resolve(b, a), (const float*)resolve(b, c), a->ne[0], a->ne[1], c->ne[1],
                         n->ne[0], a->ne[2], dst, st),
         "attn_qk");
      break;
    case MI_OP_ATTN_KQV:
      if (a->ne[2] != c->ne[1] * mi_op_params_get_i32(n, 0)) die("attn_kqv", "n_head != n_head_kv * n_rep");
      ck(mi_cuda_attn_kqv((const float*)resolve(b, a), (const float*)resolve(b, c), c->ne[0], a->ne[2], c->ne[1],
                          a->ne[0], a->ne[1], dst, st),
         "attn_kqv");
      break;
    case MI_OP_SILU:
      ck(mi_cuda_silu((const float*)resolve(b, a), mi_nelements(a), dst, st), "silu");
      break;
    case MI_OP_SCALE:
      ck(mi_cuda_scale((const float*)resolve(b, a), mi_nelements(a), mi_op_params_get_f32(n, 0), dst, st), "scale");
      break;
    case MI_OP_CPY:
      // the KV append: a dense [head_dim, n_head_kv, n_tokens] block into the
      // cache view at position n_past (src/model_qwen2.cpp:99-104)
      if (mi_nbytes(a) != mi_nbytes(n) || a->type != n->type) die("cpy", "shape or type mismatch");
      ckc(cudaMemcpyAsync(dst, resolve(b, a), mi_nbytes(n), cudaMemcpyDeviceToDevice, s), "cpy");
      break;
    default:
      die(mi_op_name(n->op), "op not covered by the device backend");
  }
  b.st.nodes++;
}

bool upload_weight(Backend& b, const mi_tensor* t, std::string* err) {
  if (!t || b.dev.count(t)) return true;  // tied output == token_embd
  const size_t bytes = mi_nbytes(t);
  void* d = nullptr;
  if (t->type == MI_TYPE_F32) {
    if (cudaMalloc(&d, bytes) != cudaSuccess) return fail(err, "cudaMalloc (weight)");
    b.owned.push_back(d);
    if (cudaMemcpy(d, t->data, bytes, cudaMemcpyHostToDevice) != cudaSuccess) return fail(err, "weight upload");
    b.st.weight_bytes += (int64_t)bytes;
  } else if (t->type == MI_TYPE_Q8_0) {
    const int64_t k = t->ne[0], n = t->ne[1];
    if (t->ne[2] != 1 || t->ne[3] != 1 || !contiguous(t)) return fail(err, std::string(t->name) + ": not a matrix");
    const size_t packed = mi_cuda_q8_0_packed_bytes(k, n);
    void* raw = nullptr;
    if (!packed || cudaMalloc(&raw, bytes) != cudaSuccess) return fail(err, "cudaMalloc (staging)");
    bool ok = cudaMemcpy(raw, t->data, bytes, cudaMemcpyHostToDevice) == cudaSuccess &&
              cudaMalloc(&d, packed) == cudaSuccess;
    if (ok) {
      b.owned.push_back(d);
      ok = mi_cuda_q8_0_pack(raw, k, n, d, (mi_cuda_stream)b.stream) == MI_CUDA_OK &&
           cudaStreamSynchronize(b.stream) == cudaSuccess;
    }
    cudaFree(raw);
    if (!ok) return fail(err, std::string(t->name) + ": Q8_0 upload / repack failed");
    b.st.weight_bytes += (int64_t)packed;
  } else {
    return fail(err, std::string(t->name) + ": weight type " + mi_type_name(t->type) +
                         " is not covered by the device kernels (Q8_0 projections, F32 norms and biases)");
  }
  b.dev[t] = d;
  return true;
}

void release(Backend* b) {
  if (!b) return;
  cudaSetDevice(b->device);
  if (b->stream) cudaStreamSynchronize(b->stream);
  if (b->exec) cudaGraphExecDestroy(b->exec);
  for (void* p : b->owned) cudaFree(p);
  for (auto& kv : b->staged) cudaFree(kv.second.d);
  if (b->d_arena) cudaFree(b->d_arena);
  if (b->stream) cudaStreamDestroy(b->stream);
  delete b;
}

}  // namespace

bool mi_ops_cuda_attach(mi_qwen2_model* model, mi_kv_cache* kv, int device, std::string* err) {
  mi_ops_cuda_detach();
  if (!model || !kv || !kv->galloc) return fail(err, "null model or KV cache");
  if (mi_cuda_init(device) != MI_CUDA_OK) return fail(err, mi_cuda_last_error());
  auto* b = new Backend();
  b->device = device;
  b->model = model;
  b->kv = kv;
  auto bail = [&](const std::string& msg) {
    release(b);
    return fail(err, msg);
  };
  if (cudaSetDevice(device) != cudaSuccess || cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking) != cudaSuccess)
    return bail("stream creation failed");
  std::string e;
  const mi_qwen2_weights& w = model->weights;
  bool ok = upload_weight(*b, w.token_embd, &e) && upload_weight(*b, w.output_norm, &e) &&
            upload_weight(*b, w.output, &e);
  for (int l = 0; ok && l < model->hparams.n_layer; l++) {
    const mi_qwen2_layer_weights& L = w.layers[l];
    for (const mi_tensor* t : {L.attn_norm, L.attn_q_w, L.attn_q_b, L.attn_k_w, L.attn_k_b, L.attn_v_w, L.attn_v_b,
                               L.attn_output_w, L.ffn_norm, L.ffn_gate_w, L.ffn_up_w, L.ffn_down_w})
      ok = ok && upload_weight(*b, t, &e);
  }
  if (!ok) return bail(e);
  // the KV cache in HBM, the reference's layout, zeroed like a fresh cache
  for (int l = 0; l < kv->n_layer; l++) {
    for (const mi_tensor* t : {(const mi_tensor*)kv->k[l], (const mi_tensor*)kv->v[l]}) {
      void* d = nullptr;
      if (cudaMalloc(&d, mi_nbytes(t)) != cudaSuccess) return bail("cudaMalloc (KV cache)");
      b->owned.push_back(d);
      if (cudaMemset(d, 0, mi_nbytes(t)) != cudaSuccess) return bail("cudaMemset (KV cache)");
      b->dev[t] = d;
    }
  }
  // gallocr's arena: one device allocation of the reserved size; the per-step
  // plans index into it at the offsets gallocr chose
  b->h_arena = kv->galloc->arena;
  b->arena_bytes = kv->galloc->arena_size;
  if (b->arena_bytes && cudaMalloc((void**)&b->d_arena, b->arena_bytes) != cudaSuccess)
    return bail("cudaMalloc (arena)");
  b->st.arena_bytes = (int64_t)b->arena_bytes;
  // The RoPE entry point keeps a host-built (cos, sin) table on the device
  // and rebuilds it when a position falls outside it: build it now for the
  // whole context, so no table upload happens inside a graph recording.
  {
    const mi_qwen2_hparams& hp = model->hparams;
    float* d = nullptr;
    if (cudaMalloc(&d, sizeof(float) * 2 * (size_t)hp.head_dim) != cudaSuccess) return bail("cudaMalloc");
    b->owned.push_back(d);
    cudaMemset(d, 0, sizeof(float) * 2 * (size_t)hp.head_dim);
    if (mi_cuda_rope_neox(d, hp.head_dim, 1, 1, kv->n_ctx - 1, hp.head_dim, hp.rope_freq_base,
                          d + hp.head_dim, (mi_cuda_stream)b->stream) != MI_CUDA_OK ||
        cudaStreamSynchronize(b->stream) != cudaSuccess)
      return bail(std::string("RoPE table: ") + mi_cuda_last_error());
  }
  g_be = b;
  return true;
}

void mi_ops_cuda_detach() {
  release(g_be);
  g_be = nullptr;
}

bool mi_ops_cuda_attached() { return g_be != nullptr; }

mi_ops_cuda_stats mi_ops_cuda_get_stats() { return g_be ? g_be->st : mi_ops_cuda_stats{}; }

void mi_ops_cuda_graph_compute(mi_cgraph* g) {
  Backend& b = *g_be;
  ckc(cudaSetDevice(b.device), "cudaSetDevice");
  // inputs in, output buffers ready -- before the recording (no allocation
  // or pageable copy may happen inside it)
  for (int i = 0; i < g->n_leafs; i++) {
    const mi_tensor* t = g->leafs[i];
    if ((t->flags & MI_TENSOR_FLAG_INPUT) && !b.dev.count(t))
      ckc(cudaMemcpyAsync(stage(b, t), t->data, mi_nbytes(t), cudaMemcpyHostToDevice, b.stream), "input upload");
  }
  for (int i = 0; i < g->n_nodes; i++) {
    const mi_tensor* t = g->nodes[i];
    if (t->flags & MI_TENSOR_FLAG_OUTPUT) stage(b, t);
    if (mi_op_is_view(t->op)) b.st.views_skipped++;
  }
  // the exec nodes (views already left out by the graph builder), recorded
  // into one CUDA graph in their topological order
  ckc(cudaStreamBeginCapture(b.stream, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
  for (int i = 0; i < g->n_exec_nodes; i++) dispatch(b, g->exec_nodes[i], b.stream);
  cudaGraph_t graph = nullptr;
  ckc(cudaStreamEndCapture(b.stream, &graph), "cudaStreamEndCapture");
  // Steps of one shape (every decode step) record the same kernels with new
  // arguments: update the executable graph in place, instantiate otherwise.
  if (b.exec) {
    cudaGraphExecUpdateResultInfo info{};
    if (cudaGraphExecUpdate(b.exec, graph, &info) == cudaSuccess) {
      b.st.updates++;
    } else {
      (void)cudaGetLastError();
      cudaGraphExecDestroy(b.exec);
      b.exec = nullptr;
    }
  }
  if (!b.exec) {
    ckc(cudaGraphInstantiate(&b.exec, graph, 0), "cudaGraphInstantiate");
    b.st.instantiations++;
  }
  cudaGraphDestroy(graph);
  ckc(cudaGraphLaunch(b.exec, b.stream), "cudaGraphLaunch");
  for (int i = 0; i < g->n_nodes; i++) {
    mi_tensor* t = g->nodes[i];
    if (t->flags & MI_TENSOR_FLAG_OUTPUT)
      ckc(cudaMemcpyAsync(t->data, b.staged[t->data].d, mi_nbytes(t), cudaMemcpyDeviceToHost, b.stream),
          "output download");
  }
  ckc(cudaStreamSynchronize(b.stream), "device step");
  int32_t code = 0;
  ck(mi_cuda_device_error(b.device, &code), "device error word");
  if (code) die("device step", "a bounded device wait gave up");
  b.st.steps++;
}

// The reference's executor entry, wrapped at link time (-Wl,--wrap for the
// C++ symbol of `void mi_graph_compute(mi_cgraph*, mi_threadpool*)`): the
// reference's forward calls this; without an attached backend it is the
// reference's own threadpool walk, unchanged.
extern "C" void __real__Z16mi_graph_computeP9mi_cgraphP13mi_threadpool(mi_cgraph* g, mi_threadpool* pool);
extern "C" void __wrap__Z16mi_graph_computeP9mi_cgraphP13mi_threadpool(mi_cgraph* g, mi_threadpool* pool) {
  if (g_be) {
    mi_ops_cuda_graph_compute(g);
    return;
  }
  __real__Z16mi_graph_computeP9mi_cgraphP13mi_threadpool(g, pool);
}
