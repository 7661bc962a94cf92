// Qwen2 decode executor: the device-resident replacement of the reference's
// model API (src/model_qwen2.h:83-189).
//
// The reference rebuilds and re-plans its graph every step and runs its ~700
// exec nodes one barrier at a time (src/model_qwen2.cpp:609-688,
// src/threadpool.cpp:171-180). Here the same computation is five fused
// kernels per layer plus one for the LM head, captured once into a CUDA graph
// and replayed every step:
//   1. QKV GEMV   prologue: [embedding lookup (layer 0)], rms_norm * attn_norm,
//                 quantize; epilogue: + [bq|bk|bv]
//   2. attention  RoPE(q, k), KV-cache append, QK, softmax, KV
//   3. O GEMV     prologue: quantize; epilogue: + residual
//   4. gate/up    prologue: rms_norm * ffn_norm, quantize; epilogue: silu(g)*u
//   5. down GEMV  prologue: quantize; epilogue: + residual
//   LM head      prologue: rms_norm * output_norm, quantize; epilogue: logits
//                 + greedy argmax (+ optional feedback into the token buffer)
// Kernels are chained with programmatic dependent launch: each GEMV starts
// streaming its weights into shared memory while its predecessor still runs.
// The step position lives on the device, so one graph serves every step.
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "gguf_reader.h"
#include "mi_cuda.h"
#include "mi_internal.h"

using namespace mi;

namespace {

struct Mat {
  uint8_t* w = nullptr;
  int64_t K = 0, N = 0, npad = 0;
  // the prefill copy for the tensor-core GEMM (launch_pack_tc), or nullptr
  uint8_t* wt = nullptr;
  float* st = nullptr;
};

struct Layer {
  Mat qkv, o, gateup, down;
  float* bqkv = nullptr;
  float* attn_norm = nullptr;
  float* ffn_norm = nullptr;
};

struct StepState {
  int32_t pos;
  int32_t next_token;
  int32_t feedback;
  uint32_t counter;
  int32_t err;
  int32_t pad[3];
};

int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

#define CK(expr)                                                                         \
  do {                                                                                   \
    cudaError_t _e = (expr);                                                             \
    if (_e != cudaSuccess)                                                               \
      return fail(MI_CUDA_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(_e)); \
  } while (0)

constexpr int kTraceStamps = 8;  // globaltimer stamps per kernel slot (mi_device.cuh)
// Shared memory of one fused QKV + attention CTA: with the ~48 KB of a 0.5B
// FFN-down GEMV CTA it still fits one SM, so the kernel's clusters can start
// (and stream their weights) while the previous layer's down projection runs.
constexpr size_t kFusedSmemBudget = 168 * 1024;

int64_t npad8(int64_t n) { return (n + 7) / 8 * 8; }
size_t packed_bytes(int64_t k, int64_t n) { return (size_t)(npad8(n) * k + npad8(n) * (k / 32) * 2); }
size_t a256(size_t v) { return (v + 255) / 256 * 256; }

}  // namespace

// Rows of every GEMV this rank computes (tensor parallelism; the full
// matrices when world == 1). Units: 8 rows, except the FFN whose unit is one
// 32-element block of its activation (64 packed gate/up rows).
struct Shard {
  int64_t qkv0 = 0, nqkv = 0;  // rows of the stacked [q | k | v] projection
  int64_t o0 = 0, no = 0;      // rows of n_embd outputs (O and down projections)
  int64_t ff0 = 0, nff = 0;    // FFN activation blocks
  int64_t v0 = 0, nv = 0;      // vocabulary rows of the LM head
};

struct mi_cuda_model {
  int device = 0;
  DeviceCtx* ctx = nullptr;
  mi_cuda_qwen2_hparams hp{};
  int rank = 0, world = 1;
  Shard sh;
  bool tied = true;
  uint8_t* buf = nullptr;
  size_t bytes = 0;
  uint8_t* tc_buf = nullptr;  // prefill copies of the GEMM weights (tensor-core layout)
  size_t tc_bytes = 0;
  bool tc_tried = false;      // pack_prefill_copies ran (once per model)
  Mat embed, lm_head;
  float* output_norm = nullptr;
  std::vector<Layer> layers;
};

struct mi_cuda_kv_cache {
  mi_cuda_model* model = nullptr;
  int32_t n_ctx = 0;
  cudaStream_t stream = nullptr;
  uint8_t* buf = nullptr;
  float* cache = nullptr;  // [layer][k|v][n_ctx][HKV][D]
  float2* rope = nullptr;
  float *x = nullptr, *x2 = nullptr, *qkv = nullptr, *attn = nullptr, *act = nullptr;
  // Q8_0_ACT inputs of the O and down GEMVs, quantized by their producers
  uint8_t *attn_q = nullptr, *act_q = nullptr;
  bool quant_attn = false;  // head_dim % 32 == 0: attention emits whole blocks
  float* logits = nullptr;
  float* scores = nullptr;
  float* part_val = nullptr;
  int32_t* part_idx = nullptr;
  int32_t* tokens = nullptr;
  StepState* state = nullptr;
  StepState* h_state = nullptr;  // pinned
  // pinned: the device state as read back by the last check_state_error; valid
  // (seen_valid) until the next call that enqueues work on the stream
  StepState* h_seen = nullptr;
  bool seen_valid = false;
  int32_t* h_tokens = nullptr;   // pinned staging, n_ctx + 1
  cudaGraphExec_t g_head = nullptr, g_nohead = nullptr;
  // the labelled fast mode's step graphs (persistent step only), captured by
  // the first mi_cuda_qwen2_set_fast_mode(kv, 1); `fast` selects them
  cudaGraphExec_t g_fast_head = nullptr, g_fast_nohead = nullptr;
  bool fast = false;
  int32_t kernels_per_step = 0;
  uint64_t* trace = nullptr;  // [slot][4] globaltimer stamps of the last step
  int32_t trace_slots = 0;
  bool pdl = true;
  // Tensor parallelism: exchange words (see mi_internal.h) in one allocation
  // that every peer maps; offsets in words. epoch = the current step's tag.
  uint64_t* xbuf = nullptr;
  size_t xwords = 0;
  size_t x_qkv = 0, x_h1 = 0, x_act = 0, x_h2 = 0, x_cand = 0;
  uint64_t* peer[kMaxRanks] = {};
  bool connected = false;
  uint32_t* epoch = nullptr;
  GemvPlan plan_qkv{}, plan_o{}, plan_gu{}, plan_down{}, plan_head{};
  // One GPU, shapes that fit: the QKV GEMV and the attention run as one
  // cluster kernel per layer (qkv_attn.cu).
  QkvAttnPlan plan_fused{};
  bool fused = false;
  // One GPU, shapes that fit: the whole step as one persistent kernel
  // (decode_persist.cu); its hand-over counters (never reset between steps:
  // targets grow with the step epoch), the epoch, the closing ticket, and the
  // layers' weight pointers.
  PersistPlan plan_persist{};
  bool persist = false;
  unsigned long long* pctr = nullptr;  // [n_layer][4] | epoch | ticket
  PersistLayer* d_layers = nullptr;
  cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};
  // Batched-prefill workspace, allocated on first use and grown to the largest
  // batch: residual streams X / X2 [T][E], q|k|v [T][E + 2kvd], rotated q
  // [T][E], the split Q8_0_ACT inputs of the E-wide and FF-wide GEMMs, and
  // (only when every row's logits are requested) logits [T][n_vocab].
  uint8_t* pbuf = nullptr;
  int64_t pcap = 0, plog_cap = 0;
  float *pX = nullptr, *pX2 = nullptr, *pQKV = nullptr, *pQR = nullptr, *pLogits = nullptr;
  int8_t *pAqE = nullptr, *pAqF = nullptr;
  float *pAdE = nullptr, *pAdF = nullptr;
};

namespace {

// Uploads GGUF Q8_0 rows [s0, s1) of `t` into packed matrix `dst` through
// pinned staging; source row i lands on packed row (i/4)*gstride + row_offset
// + i%4 (see launch_pack_q8_0), which the caller keeps inside dst.
int upload_q8_rows(const GgufTensor* t, int64_t s0, int64_t s1, const Mat& dst, int64_t row_offset,
                   int64_t gstride, uint8_t* d_stage, uint8_t* h_stage, size_t stage_bytes,
                   cudaStream_t s) {
  const int64_t K = t->ne[0];
  if (s1 <= s0) return MI_CUDA_OK;
  const int64_t lo = (s0 >> 2) * gstride + row_offset + (s0 & 3);
  const int64_t hi = ((s1 - 1) >> 2) * gstride + row_offset + ((s1 - 1) & 3);
  if (s0 < 0 || s1 > t->ne[1] || lo < 0 || hi >= dst.npad || row_offset % 4 != 0)
    return fail(MI_CUDA_ERR_ARG, "internal: packed row range outside its matrix");
  const size_t row = (size_t)(K / 32 * 34);
  const int64_t rows_per = std::max<int64_t>(4, (int64_t)(stage_bytes / row) / 4 * 4);
  for (int64_t r0 = s0; r0 < s1; r0 += rows_per) {
    const int64_t rn = std::min(rows_per, s1 - r0);
    CK(cudaStreamSynchronize(s));
    std::memcpy(h_stage, t->data + (size_t)r0 * row, (size_t)rn * row);
    CK(cudaMemcpyAsync(d_stage, h_stage, (size_t)rn * row, cudaMemcpyHostToDevice, s));
    CK(launch_pack_q8_0(d_stage, K, rn, r0, dst.w, dst.npad, row_offset, gstride, s));
  }
  return MI_CUDA_OK;
}

int upload_q8(const GgufTensor* t, const Mat& dst, int64_t row_offset, int64_t gstride,
              uint8_t* d_stage, uint8_t* h_stage, size_t stage_bytes, cudaStream_t s) {
  return upload_q8_rows(t, 0, t->ne[1], dst, row_offset, gstride, d_stage, h_stage, stage_bytes, s);
}

int upload_f32(const GgufTensor* t, float* dst, cudaStream_t s) {
  CK(cudaMemcpyAsync(dst, t->data, t->nbytes, cudaMemcpyHostToDevice, s));
  CK(cudaStreamSynchronize(s));
  return MI_CUDA_OK;
}

// Elements [e0, e1) of an F32 tensor to dst.
int upload_f32_range(const GgufTensor* t, int64_t e0, int64_t e1, float* dst, cudaStream_t s) {
  if (e1 <= e0) return MI_CUDA_OK;
  CK(cudaMemcpyAsync(dst, t->data + e0 * 4, (size_t)(e1 - e0) * 4, cudaMemcpyHostToDevice, s));
  CK(cudaStreamSynchronize(s));
  return MI_CUDA_OK;
}

void shard_range(int64_t units, int rank, int world, int64_t* first, int64_t* count) {
  *first = units * rank / world;
  *count = units * (rank + 1) / world - *first;
}

}  // namespace

namespace {

// The batched prefill's GEMMs run on the tensor cores from a second copy of
// each weight matrix in their tile layout (fp16 quants and float scales,
// about 2.13 bytes per weight), made on the first batched prefill of the
// model (a decode-only user never pays for it). MI_CUDA_TC_GEMM=0 skips it,
// as does a failed allocation, and the prefill then uses the CUDA-core GEMM.
int pack_prefill_copies(mi_cuda_model* m, cudaStream_t s) {
  if (m->tc_tried) return MI_CUDA_OK;
  m->tc_tried = true;
  const char* env = std::getenv("MI_CUDA_TC_GEMM");
  if (env && std::strcmp(env, "0") == 0) return MI_CUDA_OK;
  std::vector<Mat*> mats;
  for (auto& L : m->layers) {
    mats.push_back(&L.qkv);
    mats.push_back(&L.o);
    mats.push_back(&L.gateup);
    mats.push_back(&L.down);
  }
  mats.push_back(&m->lm_head);
  auto bytes_of = [](const Mat& x) {
    const size_t n = (size_t)tc_rows(x.npad);
    return a256(tc_weight_bytes((int64_t)n, x.K)) + a256(n * (size_t)(x.K / 32) * 4);
  };
  size_t total = 0;
  for (const Mat* x : mats) total += bytes_of(*x);
  if (cudaMalloc(&m->tc_buf, total) != cudaSuccess) {
    cudaGetLastError();  // (clears the allocation error; the CUDA-core GEMM serves)
    m->tc_buf = nullptr;
    return MI_CUDA_OK;
  }
  m->tc_bytes = total;
  size_t off = 0;
  for (Mat* x : mats) {
    const int64_t n = tc_rows(x->npad);
    x->wt = m->tc_buf + off;
    x->st = (float*)(m->tc_buf + off + a256(tc_weight_bytes(n, x->K)));
    off += bytes_of(*x);
    CK(launch_pack_tc(x->w, x->K, x->npad, n, x->wt, x->st, s));
  }
  CK(cudaStreamSynchronize(s));
  return MI_CUDA_OK;
}

struct ModelDeleter {
  void operator()(mi_cuda_model* m) const { mi_cuda_qwen2_model_free(m); }
};
struct KvCacheDeleter {
  void operator()(mi_cuda_kv_cache* kv) const { mi_cuda_kv_cache_free(kv); }
};

int load_model(const char* gguf_path, int device, int rank, int world, mi_cuda_model** out) {
  if (!gguf_path || !out) return fail(MI_CUDA_ERR_ARG, "mi_cuda_qwen2_model_load: null argument");
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
    return fail(MI_CUDA_ERR_ARG, "mi_cuda_qwen2_model_load_shard: rank / world out of range (world <= 8)");
  *out = nullptr;
  std::string err;
  DeviceCtx* ctx = device_ctx(device, &err);
  if (!ctx) return fail(MI_CUDA_ERR_CUDA, err);
  CK(cudaSetDevice(device));
  GgufFile g;
  if (!g.open(gguf_path, &err)) return fail(MI_CUDA_ERR_IO, err);

  // Hyperparameters: the same keys as mi_qwen2_hparams_load (ref src/model_qwen2.cpp:426-464).
  mi_cuda_qwen2_hparams hp{};
  uint32_t u[6];
  const char* keys[6] = {"qwen2.embedding_length", "qwen2.block_count",
                         "qwen2.attention.head_count", "qwen2.attention.head_count_kv",
                         "qwen2.feed_forward_length", "qwen2.context_length"};
  for (int i = 0; i < 6; i++)
    if (!g.get_u32(keys[i], &u[i]))
      return fail(MI_CUDA_ERR_FORMAT, std::string("qwen2 hparams: missing or wrong-typed key '") + keys[i] + "'");
  if (!g.get_f32("qwen2.rope.freq_base", &hp.rope_freq_base) ||
      !g.get_f32("qwen2.attention.layer_norm_rms_epsilon", &hp.rms_eps))
    return fail(MI_CUDA_ERR_FORMAT, "qwen2 hparams: missing rope.freq_base or layer_norm_rms_epsilon");
  hp.n_embd = (int32_t)u[0];
  hp.n_layer = (int32_t)u[1];
  hp.n_head = (int32_t)u[2];
  hp.n_head_kv = (int32_t)u[3];
  hp.n_ff = (int32_t)u[4];
  hp.n_ctx_train = (int32_t)u[5];
  if (hp.n_head == 0 || hp.n_embd % hp.n_head != 0)
    return fail(MI_CUDA_ERR_FORMAT, "qwen2 hparams: embedding_length is not divisible by head_count");
  if (hp.n_head_kv == 0 || hp.n_head % hp.n_head_kv != 0)
    return fail(MI_CUDA_ERR_FORMAT, "qwen2 hparams: head_count is not a multiple of head_count_kv");
  hp.head_dim = hp.n_embd / hp.n_head;
  const GgufTensor* te = g.find("token_embd.weight");
  if (!te) return fail(MI_CUDA_ERR_FORMAT, "missing tensor token_embd.weight");
  hp.n_vocab = (int32_t)te->ne[1];
  const int64_t E = hp.n_embd, D = hp.head_dim, kvd = (int64_t)hp.n_head_kv * D, FF = hp.n_ff;
  if (E % 64 != 0 || FF % 64 != 0 || D % 4 != 0 || D > 256)
    return fail(MI_CUDA_ERR_FORMAT,
                "unsupported shape (n_embd and n_ff multiples of 64, head_dim a multiple of 4 up to 256)");

  auto need = [&](const std::string& name, uint32_t type, int64_t ne0, int64_t ne1,
                  const GgufTensor** t) -> int {
    *t = g.find(name);
    if (!*t) return fail(MI_CUDA_ERR_FORMAT, "missing weight tensor: " + name);
    if ((*t)->type != type)
      return fail(MI_CUDA_ERR_FORMAT, "weight " + name + (type == kGgmlQ8_0 ? " must be Q8_0" : " must be F32"));
    if ((*t)->ne[0] != ne0 || (*t)->ne[1] != ne1)
      return fail(MI_CUDA_ERR_FORMAT, "weight " + name + " has an unexpected shape");
    return MI_CUDA_OK;
  };

  // Any early return releases the partly loaded model with its device memory.
  std::unique_ptr<mi_cuda_model, ModelDeleter> m(new mi_cuda_model());
  m->device = device;
  m->ctx = ctx;
  m->hp = hp;
  const GgufTensor* tout = g.find("output.weight");
  m->tied = tout == nullptr;
  int rc;
  rc = need("token_embd.weight", kGgmlQ8_0, E, hp.n_vocab, &te);
    if (rc) return rc;
  if (!m->tied && (rc = need("output.weight", kGgmlQ8_0, E, hp.n_vocab, &tout))) return rc;
  const GgufTensor* tnorm;
  rc = need("output_norm.weight", kGgmlF32, E, 1, &tnorm);
    if (rc) return rc;

  // This rank's rows of every GEMV (all rows when world == 1).
  m->rank = rank;
  m->world = world;
  Shard& sh = m->sh;
  shard_range((E + 2 * kvd) / 8, rank, world, &sh.qkv0, &sh.nqkv);
  shard_range(E / 8, rank, world, &sh.o0, &sh.no);
  shard_range(FF / 32, rank, world, &sh.ff0, &sh.nff);
  shard_range((hp.n_vocab + 7) / 8, rank, world, &sh.v0, &sh.nv);
  sh.qkv0 *= 8;
  sh.nqkv *= 8;
  sh.o0 *= 8;
  sh.no *= 8;
  sh.v0 *= 8;
  sh.nv = std::min<int64_t>(sh.nv * 8, hp.n_vocab - sh.v0);
  if (world > 1 && (sh.nqkv == 0 || sh.no == 0 || sh.nff == 0 || sh.nv <= 0))
    return fail(MI_CUDA_ERR_ARG, "model too small for this many ranks");
  // A sharded model keeps its own rows of the LM head (tied or not).
  const bool own_head = !m->tied || world > 1;

  // One device allocation for every weight (256-byte aligned sub-buffers).
  size_t total = a256(packed_bytes(E, hp.n_vocab)) + a256(E * 4);
  if (own_head) total += a256(packed_bytes(E, sh.nv));
  const size_t per_layer = a256(packed_bytes(E, sh.nqkv)) + a256(sh.nqkv * 4) +
                           a256(packed_bytes(E, sh.no)) + a256(packed_bytes(E, 64 * sh.nff)) +
                           a256(packed_bytes(FF, sh.no)) + 2 * a256(E * 4);
  total += per_layer * (size_t)hp.n_layer;
  CK(cudaMalloc(&m->buf, total));
  m->bytes = total;
  size_t off = 0;
  auto take = [&](size_t b) {
    uint8_t* p = m->buf + off;
    off += a256(b);
    return p;
  };
  auto mat = [&](int64_t K, int64_t N) {
    Mat x;
    x.K = K;
    x.N = N;
    x.npad = npad8(N);
    x.w = take(packed_bytes(K, N));
    return x;
  };
  m->embed = mat(E, hp.n_vocab);
  m->lm_head = own_head ? mat(E, sh.nv) : m->embed;
  m->output_norm = (float*)take(E * 4);
  m->layers.resize((size_t)hp.n_layer);
  for (auto& L : m->layers) {
    L.qkv = mat(E, sh.nqkv);
    L.bqkv = (float*)take(sh.nqkv * 4);
    L.o = mat(E, sh.no);
    L.gateup = mat(E, 64 * sh.nff);
    L.down = mat(FF, sh.no);
    L.attn_norm = (float*)take(E * 4);
    L.ffn_norm = (float*)take(E * 4);
  }
  CK(cudaMemset(m->buf, 0, total));

  cudaStream_t s;
  CK(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  const size_t stage = 64u << 20;
  uint8_t *d_stage = nullptr, *h_stage = nullptr;
  cudaError_t e = cudaMalloc(&d_stage, stage);
  if (e == cudaSuccess) e = cudaMallocHost(&h_stage, stage);
  auto cleanup = [&]() {
    cudaStreamSynchronize(s);
    if (d_stage) cudaFree(d_stage);
    if (h_stage) cudaFreeHost(h_stage);
    cudaStreamDestroy(s);
  };
  if (e != cudaSuccess) {
    cleanup();
    return fail(MI_CUDA_ERR_CUDA, "staging allocation failed");
  }
  rc = upload_q8(te, m->embed, 0, 4, d_stage, h_stage, stage, s);
  if (!rc && own_head)
    rc = upload_q8_rows(m->tied ? te : tout, sh.v0, sh.v0 + sh.nv, m->lm_head, -sh.v0, 4, d_stage,
                        h_stage, stage, s);
  if (!rc) rc = upload_f32(tnorm, m->output_norm, s);
  const int64_t q0 = sh.qkv0, q1 = sh.qkv0 + sh.nqkv, r0 = sh.o0, r1 = sh.o0 + sh.no;
  const int64_t a0 = 32 * sh.ff0, a1 = 32 * (sh.ff0 + sh.nff);
  for (int l = 0; !rc && l < hp.n_layer; l++) {
    Layer& L = m->layers[(size_t)l];
    const std::string b = "blk." + std::to_string(l) + ".";
    const GgufTensor *an, *wq, *bq, *wk, *bk, *wv, *bv, *wo, *fn, *wg, *wu, *wd;
    rc = need(b + "attn_norm.weight", kGgmlF32, E, 1, &an);
    if (rc) break;
    rc = need(b + "attn_q.weight", kGgmlQ8_0, E, E, &wq);
    if (rc) break;
    rc = need(b + "attn_q.bias", kGgmlF32, E, 1, &bq);
    if (rc) break;
    rc = need(b + "attn_k.weight", kGgmlQ8_0, E, kvd, &wk);
    if (rc) break;
    rc = need(b + "attn_k.bias", kGgmlF32, kvd, 1, &bk);
    if (rc) break;
    rc = need(b + "attn_v.weight", kGgmlQ8_0, E, kvd, &wv);
    if (rc) break;
    rc = need(b + "attn_v.bias", kGgmlF32, kvd, 1, &bv);
    if (rc) break;
    rc = need(b + "attn_output.weight", kGgmlQ8_0, E, E, &wo);
    if (rc) break;
    rc = need(b + "ffn_norm.weight", kGgmlF32, E, 1, &fn);
    if (rc) break;
    rc = need(b + "ffn_gate.weight", kGgmlQ8_0, E, FF, &wg);
    if (rc) break;
    rc = need(b + "ffn_up.weight", kGgmlQ8_0, E, FF, &wu);
    if (rc) break;
    rc = need(b + "ffn_down.weight", kGgmlQ8_0, FF, E, &wd);
    if (rc) break;
    // Q | K | V stacked in one matrix (this rank's rows [q0, q1) of it);
    // gate/up interleaved by groups of 4 rows.
    const int64_t qa = std::max<int64_t>(0, q0), qb = std::min<int64_t>(E, q1);
    const int64_t ka = std::max<int64_t>(0, q0 - E), kb = std::min<int64_t>(kvd, q1 - E);
    const int64_t va = std::max<int64_t>(0, q0 - E - kvd), vb = std::min<int64_t>(kvd, q1 - E - kvd);
    rc = upload_q8_rows(wq, qa, qb, L.qkv, -q0, 4, d_stage, h_stage, stage, s);
    if (rc) break;
    rc = upload_q8_rows(wk, ka, kb, L.qkv, E - q0, 4, d_stage, h_stage, stage, s);
    if (rc) break;
    rc = upload_q8_rows(wv, va, vb, L.qkv, E + kvd - q0, 4, d_stage, h_stage, stage, s);
    if (rc) break;
    rc = upload_q8_rows(wo, r0, r1, L.o, -r0, 4, d_stage, h_stage, stage, s);
    if (rc) break;
    rc = upload_q8_rows(wg, a0, a1, L.gateup, -2 * a0, 8, d_stage, h_stage, stage, s);
    if (rc) break;
    rc = upload_q8_rows(wu, a0, a1, L.gateup, 4 - 2 * a0, 8, d_stage, h_stage, stage, s);
    if (rc) break;
    rc = upload_q8_rows(wd, r0, r1, L.down, -r0, 4, d_stage, h_stage, stage, s);
    if (rc) break;
    rc = upload_f32(an, L.attn_norm, s);
    if (rc) break;
    rc = upload_f32(fn, L.ffn_norm, s);
    if (rc) break;
    rc = upload_f32_range(bq, qa, qb, L.bqkv + (qa - q0), s);
    if (rc) break;
    rc = upload_f32_range(bk, ka, kb, L.bqkv + (E + ka - q0), s);
    if (rc) break;
    rc = upload_f32_range(bv, va, vb, L.bqkv + (E + kvd + va - q0), s);
    if (rc) break;
  }
  cleanup();
  if (!rc && cudaGetLastError() != cudaSuccess) rc = fail(MI_CUDA_ERR_CUDA, "weight upload failed");
  if (rc) return rc;
  *out = m.release();
  return MI_CUDA_OK;
}

}  // namespace

extern "C" {

int mi_cuda_qwen2_model_load(const char* gguf_path, int device, mi_cuda_model** out) {
  return load_model(gguf_path, device, 0, 1, out);
}

int mi_cuda_qwen2_model_load_shard(const char* gguf_path, int device, int rank, int world,
                                   mi_cuda_model** out) {
  return load_model(gguf_path, device, rank, world, out);
}

int mi_cuda_tp_shard_range(int64_t n_units, int rank, int world, int64_t* first, int64_t* count) {
  if (n_units < 0 || world < 1 || rank < 0 || rank >= world || !first || !count)
    return fail(MI_CUDA_ERR_ARG, "mi_cuda_tp_shard_range: bad arguments");
  shard_range(n_units, rank, world, first, count);
  return MI_CUDA_OK;
}

void mi_cuda_qwen2_model_free(mi_cuda_model* model) {
  if (!model) return;
  cudaSetDevice(model->device);
  cudaFree(model->buf);
  if (model->tc_buf) cudaFree(model->tc_buf);
  delete model;
}

int mi_cuda_qwen2_get_hparams(const mi_cuda_model* model, mi_cuda_qwen2_hparams* out) {
  if (!model || !out) return fail(MI_CUDA_ERR_ARG, "null argument");
  *out = model->hp;
  return MI_CUDA_OK;
}

size_t mi_cuda_qwen2_weight_bytes(const mi_cuda_model* model) { return model ? model->bytes : 0; }

}  // extern "C"

namespace {

// Enqueues one decode step (n_tokens = 1) on kv->stream; with_head adds the
// LM head + greedy argmax, otherwise the step only advances the position.
// With a sharded model (world > 1) every GEMV computes this rank's rows and
// stores them into every rank's exchange words; the consumers read those.
int enqueue_step(mi_cuda_kv_cache* kv, bool with_head, int32_t* n_kernels) {
  mi_cuda_model* m = kv->model;
  const mi_cuda_qwen2_hparams& hp = m->hp;
  const Shard& sh = m->sh;
  const int64_t E = hp.n_embd, D = hp.head_dim, kvd = (int64_t)hp.n_head_kv * D, FF = hp.n_ff;
  const int64_t nqkv_full = E + 2 * kvd, act_words = FF / 32 * 9;
  const bool tp = m->world > 1;
  const ExpTab et = m->ctx->et;
  int32_t* err = &kv->state->err;
  const size_t layer_floats = (size_t)2 * kv->n_ctx * kvd;
  // exchange words of output `off` (+ layer offset) on every rank
  auto outs = [&](GemvParams& g, size_t off) {
    g.n_ranks = m->world;
    g.rank = m->rank;
    g.epoch = kv->epoch;
    for (int r = 0; r < m->world; r++) g.out_ll[r] = kv->peer[r] + off;
  };
  auto local = [&](size_t off) -> const uint64_t* { return kv->xbuf + off; };
  if (kv->persist) {
    PersistParams q{};
    q.n_layer = hp.n_layer;
    q.E = (int32_t)E;
    q.H = hp.n_head;
    q.HKV = hp.n_head_kv;
    q.D = (int32_t)D;
    q.FF = (int32_t)FF;
    q.V = hp.n_vocab;
    q.n_ctx = kv->n_ctx;
    q.qkv_npad = m->layers[0].qkv.npad;
    q.gu_npad = m->layers[0].gateup.npad;
    q.head_npad = m->lm_head.npad;
    q.eps = hp.rms_eps;
    q.scale = 1.0f / std::sqrt((float)hp.head_dim);
    q.layers = kv->d_layers;
    q.embed = m->embed.w;
    q.embed_npad = m->embed.npad;
    q.head = m->lm_head.w;
    q.out_norm = m->output_norm;
    q.cache = kv->cache;
    q.rope = kv->rope;
    q.x = kv->x;
    q.x2 = kv->x2;
    q.act_q = kv->act_q;
    q.logits = kv->logits;
    q.scores = kv->scores;
    q.part_val = kv->part_val;
    q.part_idx = kv->part_idx;
    q.tokens = kv->tokens;
    q.tokens_len = kv->n_ctx + 1;
    q.with_head = with_head ? 1 : 0;
    q.pos = &kv->state->pos;
    q.next_token = &kv->state->next_token;
    q.feedback = &kv->state->feedback;
    q.err = err;
    q.ctr = kv->pctr;
    q.epoch = kv->pctr + (size_t)hp.n_layer * 4;
    q.ticket = (uint32_t*)(kv->pctr + (size_t)hp.n_layer * 4 + 1);
    q.et = et;
    q.trace = kv->trace;
    q.fast = kv->fast ? 1 : 0;
    CK(launch_persist(q, kv->plan_persist, kv->stream));
    if (n_kernels) *n_kernels = 1;
    return MI_CUDA_OK;
  }
  int count = 0;
  bool pdl = false;  // the first kernel of a step has no in-graph predecessor
  for (int l = 0; l < hp.n_layer; l++) {
    const Layer& L = m->layers[(size_t)l];
    const size_t o_qkv = kv->x_qkv + (size_t)l * nqkv_full, o_h1 = kv->x_h1 + (size_t)l * E,
                 o_act = kv->x_act + (size_t)l * act_words, o_h2 = kv->x_h2 + (size_t)l * E,
                 o_prev = l > 0 ? kv->x_h2 + (size_t)(l - 1) * E : 0;
    float* const cache_k = kv->cache + (size_t)l * layer_floats;
    float* const cache_v = cache_k + (size_t)kv->n_ctx * kvd;
    if (kv->fused) {
      QkvAttnParams f{};
      f.w = L.qkv.w;
      f.K = E;
      f.n_pad = L.qkv.npad;
      f.bias = L.bqkv;
      f.pro = l == 0 ? PRO_EMBED_NORM : PRO_NORM_QUANT;
      f.tokens_len = kv->n_ctx + 1;
      f.x = kv->x;
      f.norm_w = L.attn_norm;
      f.eps = hp.rms_eps;
      f.embed = m->embed.w;
      f.embed_npad = m->embed.npad;
      f.embed_rows = hp.n_vocab;
      f.tokens = kv->tokens;
      f.x_out = kv->x;
      f.cache_k = cache_k;
      f.cache_v = cache_v;
      f.head_dim = (int32_t)D;
      f.n_head = hp.n_head;
      f.n_head_kv = hp.n_head_kv;
      f.n_ctx = kv->n_ctx;
      f.pos = &kv->state->pos;
      f.rope_cs = kv->rope;
      f.scale = 1.0f / std::sqrt((float)hp.head_dim);
      f.scores = kv->scores;
      f.scores_stride = kv->n_ctx;
      f.out = kv->quant_attn ? nullptr : kv->attn;
      f.act_out = kv->quant_attn ? kv->attn_q : nullptr;
      f.et = et;
      f.err = err;
      f.trace = kv->trace;
      f.trace_slot = count;
      f.trace_slot_q = 4 * hp.n_layer + 1 + 2 * l;
      f.trace_slot_kv = f.trace_slot_q + 1;
      CK(launch_qkv_attn(f, kv->plan_fused, kv->stream, pdl));
      pdl = kv->pdl;
      count++;
    } else {
      GemvParams p{};
      p.w = L.qkv.w;
      p.K = E;
      p.N = L.qkv.N;
      p.n_pad = L.qkv.npad;
      p.pro = l == 0 ? PRO_EMBED_NORM : PRO_NORM_QUANT;
      p.x = kv->x;
      p.norm_w = L.attn_norm;
      p.eps = hp.rms_eps;
      p.embed = m->embed.w;
      p.embed_npad = m->embed.npad;
      p.embed_rows = hp.n_vocab;
      p.tokens = kv->tokens;
      p.tokens_len = kv->n_ctx + 1;
      p.pos = &kv->state->pos;
      p.x_out = kv->x;
      p.epi = EPI_BIAS;
      p.bias = L.bqkv;
      p.out = kv->qkv;
      p.et = et;
      p.err = err;
      p.trace = kv->trace;
      p.trace_slot = count;
      if (tp) {
        p.row0 = sh.qkv0;
        if (l > 0) p.x_ll = local(o_prev);
        outs(p, o_qkv);
      }
      CK(launch_gemv(p, kv->plan_qkv, kv->stream, pdl, tp));
      pdl = kv->pdl;
      count++;

      AttnParams a{};
      a.qkv = kv->qkv;
      a.cache_k = cache_k;
      a.cache_v = cache_v;
      a.head_dim = (int32_t)D;
      a.n_head = hp.n_head;
      a.n_head_kv = hp.n_head_kv;
      a.pos = &kv->state->pos;
      a.rope_cs = kv->rope;
      a.scale = 1.0f / std::sqrt((float)hp.head_dim);
      a.n_ctx = kv->n_ctx;
      a.scores = kv->scores;
      a.scores_stride = kv->n_ctx;
      a.out = kv->quant_attn ? nullptr : kv->attn;
      a.act_out = kv->quant_attn ? kv->attn_q : nullptr;
      a.et = et;
      a.err = err;
      a.trace = kv->trace;
      a.trace_slot = count;
      if (tp) {
        a.qkv_ll = local(o_qkv);
        a.epoch = kv->epoch;
      }
      CK(launch_attn_decode(a, true, kv->stream, pdl, tp));
      count++;
    }

    GemvParams o{};
    o.w = L.o.w;
    o.K = E;
    o.N = L.o.N;
    o.n_pad = L.o.npad;
    o.pro = kv->quant_attn ? PRO_ACT : PRO_QUANT;
    o.act = kv->attn_q;
    o.x = kv->attn;
    o.epi = EPI_RESID;
    o.resid = kv->x;
    o.out = kv->x2;
    o.et = et;
    o.err = err;
    o.trace = kv->trace;
    o.trace_slot = count;
    if (tp) {
      o.row0 = sh.o0;
      if (l > 0) o.resid_ll = local(o_prev);
      outs(o, o_h1);
    }
    CK(launch_gemv(o, kv->plan_o, kv->stream, pdl, tp));
    count++;

    GemvParams gu{};
    gu.w = L.gateup.w;
    gu.K = E;
    gu.N = L.gateup.N;
    gu.n_pad = L.gateup.npad;
    gu.pro = PRO_NORM_QUANT;
    gu.x = kv->x2;
    gu.norm_w = L.ffn_norm;
    gu.eps = hp.rms_eps;
    gu.epi = EPI_SILU_GATEUP_Q;
    gu.act_out = kv->act_q;
    gu.et = et;
    gu.err = err;
    gu.trace = kv->trace;
    gu.trace_slot = count;
    if (tp) {
      gu.row0 = 64 * sh.ff0;
      gu.x_ll = local(o_h1);
      outs(gu, o_act);
    }
    CK(launch_gemv(gu, kv->plan_gu, kv->stream, pdl, tp));
    count++;

    GemvParams dn{};
    dn.w = L.down.w;
    dn.K = FF;
    dn.N = L.down.N;
    dn.n_pad = L.down.npad;
    dn.pro = PRO_ACT;
    dn.act = kv->act_q;
    dn.epi = EPI_RESID;
    dn.resid = kv->x2;
    dn.out = kv->x;
    dn.et = et;
    dn.err = err;
    dn.trace = kv->trace;
    dn.trace_slot = count;
    if (tp) {
      dn.row0 = sh.o0;
      dn.act_ll = local(o_act);
      dn.resid_ll = local(o_h1);
      outs(dn, o_h2);
    }
    CK(launch_gemv(dn, kv->plan_down, kv->stream, pdl, tp));
    count++;
  }
  if (with_head) {
    GemvParams h{};
    h.w = m->lm_head.w;
    h.K = E;
    h.N = m->lm_head.N;
    h.n_pad = m->lm_head.npad;
    h.pro = PRO_NORM_QUANT;
    h.x = kv->x;
    h.norm_w = m->output_norm;
    h.eps = hp.rms_eps;
    h.epi = EPI_ARGMAX;
    h.out = kv->logits;
    h.part_val = kv->part_val;
    h.part_idx = kv->part_idx;
    h.counter = &kv->state->counter;
    h.next_token = &kv->state->next_token;
    h.tokens_rw = kv->tokens;
    h.tokens_len = kv->n_ctx + 1;
    h.pos_rw = &kv->state->pos;
    h.feedback = &kv->state->feedback;
    h.et = et;
    h.err = err;
    h.trace = kv->trace;
    h.trace_slot = count;
    if (tp) {
      h.row0 = sh.v0;
      h.x_ll = local(kv->x_h2 + (size_t)(hp.n_layer - 1) * E);
      outs(h, kv->x_cand);
      h.epoch_rw = kv->epoch;
    }
    CK(launch_gemv(h, kv->plan_head, kv->stream, pdl, tp));
  } else {
    CK(launch_advance(&kv->state->pos, kv->stream, pdl, tp ? kv->epoch : nullptr));
  }
  count++;
  if (n_kernels) *n_kernels = count;
  return MI_CUDA_OK;
}

int capture(mi_cuda_kv_cache* kv, bool with_head, cudaGraphExec_t* out, int32_t* n_kernels) {
  CK(cudaStreamBeginCapture(kv->stream, cudaStreamCaptureModeThreadLocal));
  int rc = enqueue_step(kv, with_head, n_kernels);
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamEndCapture(kv->stream, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (e != cudaSuccess) return fail(MI_CUDA_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(e));
  e = cudaGraphInstantiate(out, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return fail(MI_CUDA_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
  return MI_CUDA_OK;
}

// Workspace for a batch of n tokens (every row's logits when all_logits).
int ensure_prefill_ws(mi_cuda_kv_cache* kv, int64_t n, bool all_logits) {
  const mi_cuda_qwen2_hparams& hp = kv->model->hp;
  const int64_t E = hp.n_embd, FF = hp.n_ff, kvd = (int64_t)hp.n_head_kv * hp.head_dim;
  if (n > kv->pcap) {
    CK(cudaStreamSynchronize(kv->stream));
    if (kv->pbuf) CK(cudaFree(kv->pbuf));
    kv->pbuf = nullptr;
    kv->pcap = 0;
    size_t off = 0;
    auto slot = [&](size_t b) {
      const size_t o = off;
      off += a256(b);
      return o;
    };
    const size_t oX = slot(n * E * 4), oX2 = slot(n * E * 4), oQKV = slot(n * (E + 2 * kvd) * 4),
                 oQR = slot(n * E * 4), oAqE = slot(n * E), oAdE = slot(n * (E / 32) * 4), oAqF = slot(n * FF),
                 oAdF = slot(n * (FF / 32) * 4);
    CK(cudaMalloc(&kv->pbuf, off));
    kv->pX = (float*)(kv->pbuf + oX);
    kv->pX2 = (float*)(kv->pbuf + oX2);
    kv->pQKV = (float*)(kv->pbuf + oQKV);
    kv->pQR = (float*)(kv->pbuf + oQR);
    kv->pAqE = (int8_t*)(kv->pbuf + oAqE);
    kv->pAdE = (float*)(kv->pbuf + oAdE);
    kv->pAqF = (int8_t*)(kv->pbuf + oAqF);
    kv->pAdF = (float*)(kv->pbuf + oAdF);
    kv->pcap = n;
  }
  if (all_logits && n > kv->plog_cap) {
    CK(cudaStreamSynchronize(kv->stream));
    if (kv->pLogits) CK(cudaFree(kv->pLogits));
    kv->pLogits = nullptr;
    kv->plog_cap = 0;
    CK(cudaMalloc(&kv->pLogits, (size_t)n * hp.n_vocab * 4));
    kv->plog_cap = n;
  }
  return MI_CUDA_OK;
}

// Enqueues a batched prefill of tokens[n_past .. n_past + n) (already in the
// device token buffer): every layer for all n tokens at once, then the LM head
// and greedy argmax for the last token (the StepState must hold pos =
// n_past + n - 1; the head advances it). With all_logits the logits of every
// row land in kv->pLogits (rows 0 .. n-2; the last row is kv->logits).
int enqueue_prefill(mi_cuda_kv_cache* kv, int32_t n, int32_t n_past, bool all_logits) {
  mi_cuda_model* m = kv->model;
  const mi_cuda_qwen2_hparams& hp = m->hp;
  const int64_t E = hp.n_embd, D = hp.head_dim, kvd = (int64_t)hp.n_head_kv * D, FF = hp.n_ff;
  const int64_t row_qkv = E + 2 * kvd;
  const ExpTab et = m->ctx->et;
  int32_t* err = &kv->state->err;
  const size_t layer_floats = (size_t)2 * kv->n_ctx * kvd;
  cudaStream_t s = kv->stream;
  if (int rc = ensure_prefill_ws(kv, n, all_logits)) return rc;
  for (int l = 0; l < hp.n_layer; l++) {
    const Layer& L = m->layers[(size_t)l];
    NormQuantParams nq{};
    nq.K = E;
    nq.x = kv->pX;
    if (l == 0) {
      nq.embed = m->embed.w;
      nq.embed_npad = m->embed.npad;
      nq.embed_rows = hp.n_vocab;
      nq.tokens = kv->tokens + n_past;
      nq.x_out = kv->pX;
    }
    nq.norm_w = L.attn_norm;
    nq.eps = hp.rms_eps;
    nq.q_out = kv->pAqE;
    nq.d_out = kv->pAdE;
    nq.err = err;
    CK(launch_norm_quant(nq, n, s));

    GemmParams g{};
    g.w = L.qkv.w;
    g.K = E;
    g.N = L.qkv.N;
    g.n_pad = L.qkv.npad;
    g.act_qs = kv->pAqE;
    g.act_d = kv->pAdE;
    g.act_stride = E;
    g.M = n;
    g.epi = EPI_BIAS;
    g.bias = L.bqkv;
    g.out = kv->pQKV;
    g.out_stride = row_qkv;
    g.et = et;
    g.wt = L.qkv.wt;
    g.st = L.qkv.st;
    g.err = err;
    CK(launch_gemm(g, s));

    float* ck = kv->cache + (size_t)l * layer_floats;
    float* cv = ck + (size_t)kv->n_ctx * kvd;
    CK(launch_rope_kv(kv->pQKV, row_qkv, (int32_t)D, hp.n_head, hp.n_head_kv, n_past, n, kv->rope, kv->pQR,
                      ck, cv, s));

    const int32_t n_rep = hp.n_head / hp.n_head_kv;
    const bool quant_in_attn = (n_rep * D) % 32 == 0;
    if (prefill_attn_fits((int32_t)D, n_rep, (int64_t)n_past + n)) {
      PrefillAttnParams pa{};
      pa.q_rot = kv->pQR;
      pa.cache_k = ck;
      pa.cache_v = cv;
      pa.head_dim = (int32_t)D;
      pa.n_head = hp.n_head;
      pa.n_head_kv = hp.n_head_kv;
      pa.n_rep = n_rep;
      pa.n_past = n_past;
      pa.scale = 1.0f / std::sqrt((float)hp.head_dim);
      pa.row = E;
      if (quant_in_attn) {
        pa.act_qs = kv->pAqE;
        pa.act_d = kv->pAdE;
      } else {
        pa.out = kv->pX2;
      }
      pa.et = et;
      CK(launch_attn_prefill(pa, n, s));
    } else {
      AttnParams a{};
      a.q_rot = kv->pQR;
      a.cache_k = ck;
      a.cache_v = cv;
      a.head_dim = (int32_t)D;
      a.n_head = hp.n_head;
      a.n_head_kv = hp.n_head_kv;
      a.n_kv_fixed = n_past + 1;
      a.scale = 1.0f / std::sqrt((float)hp.head_dim);
      a.n_ctx = kv->n_ctx;
      a.scores = kv->scores;
      a.scores_stride = kv->n_ctx;
      if (kv->quant_attn) {
        a.act_qs = kv->pAqE;  // whole 32-element blocks per head: quantized in the epilogue
        a.act_d = kv->pAdE;
      } else {
        a.out = kv->pX2;  // F32 rows, quantized below (X2 is free until the O projection)
      }
      a.et = et;
      a.err = err;
      CK(launch_attn_decode(a, false, s, false, false, n));
    }
    const bool f32_attn = prefill_attn_fits((int32_t)D, n_rep, (int64_t)n_past + n) ? !quant_in_attn
                                                                                     : !kv->quant_attn;
    if (f32_attn) {
      NormQuantParams aq{};
      aq.K = E;
      aq.x = kv->pX2;
      aq.q_out = kv->pAqE;
      aq.d_out = kv->pAdE;
      aq.err = err;
      CK(launch_norm_quant(aq, n, s));
    }

    GemmParams o = g;
    o.w = L.o.w;
    o.N = L.o.N;
    o.n_pad = L.o.npad;
    o.epi = EPI_RESID;
    o.bias = nullptr;
    o.resid = kv->pX;
    o.out = kv->pX2;
    o.out_stride = E;
    o.wt = L.o.wt;
    o.st = L.o.st;
    CK(launch_gemm(o, s));

    nq = NormQuantParams{};
    nq.K = E;
    nq.x = kv->pX2;
    nq.norm_w = L.ffn_norm;
    nq.eps = hp.rms_eps;
    nq.q_out = kv->pAqE;
    nq.d_out = kv->pAdE;
    nq.err = err;
    CK(launch_norm_quant(nq, n, s));

    GemmParams gu = g;
    gu.w = L.gateup.w;
    gu.N = L.gateup.N;
    gu.n_pad = L.gateup.npad;
    gu.epi = EPI_SILU_GATEUP_Q;
    gu.bias = nullptr;
    gu.out = nullptr;
    gu.q_out = kv->pAqF;
    gu.d_out = kv->pAdF;
    gu.q_stride = FF;
    gu.wt = L.gateup.wt;
    gu.st = L.gateup.st;
    CK(launch_gemm(gu, s));

    GemmParams dn{};
    dn.w = L.down.w;
    dn.K = FF;
    dn.N = L.down.N;
    dn.n_pad = L.down.npad;
    dn.act_qs = kv->pAqF;
    dn.act_d = kv->pAdF;
    dn.act_stride = FF;
    dn.M = n;
    dn.epi = EPI_RESID;
    dn.resid = kv->pX2;
    dn.out = kv->pX;
    dn.out_stride = E;
    dn.et = et;
    dn.wt = L.down.wt;
    dn.st = L.down.st;
    dn.err = err;
    CK(launch_gemm(dn, s));
  }
  if (all_logits && n > 1) {
    NormQuantParams nq{};
    nq.K = E;
    nq.x = kv->pX;
    nq.norm_w = m->output_norm;
    nq.eps = hp.rms_eps;
    nq.q_out = kv->pAqE;
    nq.d_out = kv->pAdE;
    nq.err = err;
    CK(launch_norm_quant(nq, n - 1, s));
    GemmParams h{};
    h.w = m->lm_head.w;
    h.K = E;
    h.N = m->lm_head.N;
    h.n_pad = m->lm_head.npad;
    h.act_qs = kv->pAqE;
    h.act_d = kv->pAdE;
    h.act_stride = E;
    h.M = n - 1;
    h.epi = EPI_STORE;
    h.out = kv->pLogits;
    h.out_stride = hp.n_vocab;
    h.et = et;
    h.wt = m->lm_head.wt;
    h.st = m->lm_head.st;
    h.err = err;
    CK(launch_gemm(h, s));
  }
  // LM head + greedy argmax of the last token (the decode kernel, on row n-1).
  GemvParams h{};
  h.w = m->lm_head.w;
  h.K = E;
  h.N = m->lm_head.N;
  h.n_pad = m->lm_head.npad;
  h.pro = PRO_NORM_QUANT;
  h.x = kv->pX + (size_t)(n - 1) * E;
  h.norm_w = m->output_norm;
  h.eps = hp.rms_eps;
  h.epi = EPI_ARGMAX;
  h.out = kv->logits;
  h.part_val = kv->part_val;
  h.part_idx = kv->part_idx;
  h.counter = &kv->state->counter;
  h.next_token = &kv->state->next_token;
  h.tokens_rw = kv->tokens;
  h.tokens_len = kv->n_ctx + 1;
  h.pos_rw = &kv->state->pos;
  h.feedback = &kv->state->feedback;
  h.et = et;
  h.err = err;
  CK(launch_gemv(h, kv->plan_head, s, false));
  return MI_CUDA_OK;
}

// Batched prefill applies to unsharded models; MI_CUDA_PREFILL=stepwise keeps
// prompts on the per-position decode graph (for A/B comparisons).
bool use_batched_prefill(mi_cuda_kv_cache* kv, int32_t n) {
  if (n < 2 || kv->model->world > 1) return false;
  const char* e = std::getenv("MI_CUDA_PREFILL");
  return !(e && std::strcmp(e, "stepwise") == 0);
}

// The step graphs exist (a sharded model's KV cache gets them at connect).
int graphs_ready(mi_cuda_kv_cache* kv) {
  if (!kv->g_head || !kv->g_nohead)
    return fail(MI_CUDA_ERR_STATE, "sharded model: call mi_cuda_tp_connect before running steps");
  return MI_CUDA_OK;
}

// The step graphs of the current mode (exact, or the labelled fast mode).
cudaGraphExec_t head_graph(const mi_cuda_kv_cache* kv) { return kv->fast ? kv->g_fast_head : kv->g_head; }
cudaGraphExec_t nohead_graph(const mi_cuda_kv_cache* kv) { return kv->fast ? kv->g_fast_nohead : kv->g_nohead; }

int check_state_error(mi_cuda_kv_cache* kv) {
  // The step state (error word, next token) into pinned memory behind the
  // stream's work: one host round trip per call, and mi_cuda_qwen2_last_token
  // right after needs none.
  kv->seen_valid = false;
  CK(cudaMemcpyAsync(kv->h_seen, kv->state, sizeof(StepState), cudaMemcpyDeviceToHost, kv->stream));
  CK(cudaStreamSynchronize(kv->stream));
  const int32_t err = kv->h_seen->err;
  if (!err) kv->seen_valid = true;
  if (err) {
    CK(cudaMemset(&kv->state->err, 0, 4));
    if (err == MI_CUDA_ERR_TIMEOUT) return fail(MI_CUDA_ERR_TIMEOUT, "a device-side wait timed out");
    if (err == MI_CUDA_ERR_STATE) return fail(MI_CUDA_ERR_STATE, "decode position outside the KV cache");
    return fail(err, "a kernel reported an invalid token id or position");
  }
  return MI_CUDA_OK;
}

}  // namespace

extern "C" {

int mi_cuda_kv_cache_init(mi_cuda_model* m, int32_t n_ctx, mi_cuda_kv_cache** out) {
  if (!m || !out || n_ctx <= 0) return fail(MI_CUDA_ERR_ARG, "mi_cuda_kv_cache_init: bad arguments");
  *out = nullptr;
  CK(cudaSetDevice(m->device));
  const mi_cuda_qwen2_hparams& hp = m->hp;
  const int64_t E = hp.n_embd, D = hp.head_dim, kvd = (int64_t)hp.n_head_kv * D, FF = hp.n_ff;
  // Any early return releases the partly built cache with everything it holds.
  std::unique_ptr<mi_cuda_kv_cache, KvCacheDeleter> kv(new mi_cuda_kv_cache());
  kv->model = m;
  kv->n_ctx = n_ctx;
  // MI_CUDA_NO_PDL=1 captures the step without programmatic dependent launch
  // (plain stream order), for comparing the two schedules.
  if (const char* e = std::getenv("MI_CUDA_NO_PDL")) kv->pdl = std::atoi(e) == 0;
  const int sms = m->ctx->num_sms;
  kv->quant_attn = D % 32 == 0;
  const Shard& sh = m->sh;
  kv->plan_qkv = plan_gemv(E, sh.nqkv, sms, PRO_EMBED_NORM);
  kv->plan_o = plan_gemv(E, sh.no, sms, kv->quant_attn ? PRO_ACT : PRO_QUANT);
  // whole 32-element blocks of the FFN activation (64 packed gate/up rows
  // each) per CTA: one block at narrow K; at wide K (one CTA per SM) enough
  // blocks that every SM has a CTA in a single wave
  const int64_t bpc = E / 32 >= 64 ? std::min<int64_t>(8, (sh.nff + sms - 1) / sms) : 1;
  kv->plan_gu = plan_gemv(E, 64 * sh.nff, sms, PRO_NORM_QUANT, (int32_t)(64 * bpc));
  kv->plan_down = plan_gemv(FF, sh.no, sms, PRO_ACT);
  kv->plan_head = plan_gemv(E, sh.nv, sms, PRO_NORM_QUANT);
  // The fused QKV + attention kernel where the shape fits it (one GPU);
  // MI_CUDA_FUSED_ATTN=0 keeps the GEMV + attention kernel pair, and
  // MI_CUDA_FUSED_SMEM_KB sets its shared-memory budget (for comparisons).
  if (m->world == 1) {
    const char* fe = std::getenv("MI_CUDA_FUSED_ATTN");
    size_t budget = kFusedSmemBudget;
    if (const char* b = std::getenv("MI_CUDA_FUSED_SMEM_KB"))
      if (std::atoi(b) > 0) budget = (size_t)std::atoi(b) * 1024;
    if (!(fe && std::atoi(fe) == 0)) {
      kv->plan_fused = plan_qkv_attn(E, (int32_t)D, hp.n_head, hp.n_head_kv, n_ctx, budget);
      kv->fused = kv->plan_fused.ok;
    }
  }

  // The persistent one-kernel step where the shape fits it (one GPU);
  // MI_CUDA_PERSIST=0 keeps the kernel-per-phase graph (for comparisons).
  if (m->world == 1) {
    const char* pe = std::getenv("MI_CUDA_PERSIST");
    if (!(pe && std::atoi(pe) == 0)) {
      kv->plan_persist = plan_persist(E, (int32_t)D, hp.n_head, hp.n_head_kv, FF, hp.n_vocab, hp.n_layer, n_ctx,
                                      sms);
      kv->persist = kv->plan_persist.ok;
    }
  }

  const size_t cache_bytes = (size_t)hp.n_layer * 2 * n_ctx * kvd * 4;
  const size_t rope_bytes = (size_t)n_ctx * (D / 2) * 8;
  size_t off = 0;
  auto slot = [&](size_t b) {
    size_t o = off;
    off += a256(b);
    return o;
  };
  const size_t o_cache = slot(cache_bytes), o_rope = slot(rope_bytes), o_x = slot(E * 4),
               o_x2 = slot(E * 4), o_qkv = slot((E + 2 * kvd) * 4), o_attn = slot(E * 4),
               o_act = slot(FF * 4), o_logits = slot((size_t)hp.n_vocab * 4),
               o_scores = slot((size_t)hp.n_head * n_ctx * 4), o_pv = slot(1024 * 4),
               o_pi = slot(1024 * 4), o_tok = slot((size_t)(n_ctx + 1) * 4),
               o_state = slot(sizeof(StepState)), o_attnq = slot(E / 32 * 36),
               o_actq = slot(FF / 32 * 36),
               o_trace = slot((size_t)(6 * hp.n_layer + 1) * kTraceStamps * 8), o_epoch = slot(4),
               o_pctr = slot(((size_t)hp.n_layer * 4 + 2) * 8),
               o_play = slot((size_t)hp.n_layer * sizeof(PersistLayer));
  CK(cudaMalloc(&kv->buf, off));
  CK(cudaMemset(kv->buf, 0, off));
  kv->cache = (float*)(kv->buf + o_cache);
  kv->rope = (float2*)(kv->buf + o_rope);
  kv->x = (float*)(kv->buf + o_x);
  kv->x2 = (float*)(kv->buf + o_x2);
  kv->qkv = (float*)(kv->buf + o_qkv);
  kv->attn = (float*)(kv->buf + o_attn);
  kv->act = (float*)(kv->buf + o_act);
  kv->logits = (float*)(kv->buf + o_logits);
  kv->scores = (float*)(kv->buf + o_scores);
  kv->part_val = (float*)(kv->buf + o_pv);
  kv->part_idx = (int32_t*)(kv->buf + o_pi);
  kv->tokens = (int32_t*)(kv->buf + o_tok);
  kv->state = (StepState*)(kv->buf + o_state);
  kv->attn_q = kv->buf + o_attnq;
  kv->act_q = kv->buf + o_actq;
  kv->trace = (uint64_t*)(kv->buf + o_trace);
  // one slot per kernel of a step; the fused QKV + attention kernel adds two
  // detail slots per layer after the step's slots
  kv->trace_slots = kv->persist ? 2 * hp.n_layer + 1 : 6 * hp.n_layer + 1;
  kv->epoch = (uint32_t*)(kv->buf + o_epoch);
  kv->pctr = (unsigned long long*)(kv->buf + o_pctr);
  kv->d_layers = (PersistLayer*)(kv->buf + o_play);
  {
    std::vector<PersistLayer> pl((size_t)hp.n_layer);
    for (int l = 0; l < hp.n_layer; l++) {
      const Layer& L = m->layers[(size_t)l];
      pl[(size_t)l] = PersistLayer{L.qkv.w, L.bqkv, L.attn_norm, L.o.w, L.gateup.w, L.ffn_norm, L.down.w};
    }
    CK(cudaMemcpy(kv->d_layers, pl.data(), pl.size() * sizeof(PersistLayer), cudaMemcpyHostToDevice));
  }
  const uint32_t one = 1u;  // exchange words start zeroed: tag 0 is never current
  CK(cudaMemcpy(kv->epoch, &one, 4, cudaMemcpyHostToDevice));
  if (kv->plan_head.grid > 1024) return fail(MI_CUDA_ERR_ARG, "LM head grid too large");

  std::vector<float> cs((size_t)n_ctx * (D / 2) * 2);
  build_rope_table(0, n_ctx, (int32_t)D, hp.rope_freq_base, cs.data());
  CK(cudaMemcpy(kv->rope, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
  CK(cudaMallocHost(&kv->h_state, sizeof(StepState)));
  CK(cudaMallocHost(&kv->h_seen, sizeof(StepState)));
  CK(cudaMallocHost(&kv->h_tokens, (size_t)(n_ctx + 1) * 4));
  CK(cudaStreamCreateWithFlags(&kv->stream, cudaStreamNonBlocking));
  for (auto& e : kv->ev) CK(cudaEventCreate(&e));

  if (m->world > 1) {
    // Exchange words; the step graphs are captured by mi_cuda_tp_connect once
    // every rank's buffer is mapped.
    kv->x_qkv = 0;
    kv->x_h1 = kv->x_qkv + (size_t)hp.n_layer * (E + 2 * kvd);
    kv->x_act = kv->x_h1 + (size_t)hp.n_layer * E;
    kv->x_h2 = kv->x_act + (size_t)hp.n_layer * (FF / 32 * 9);
    kv->x_cand = kv->x_h2 + (size_t)hp.n_layer * E;
    kv->xwords = kv->x_cand + 2 * kMaxRanks;
    CK(cudaMalloc(&kv->xbuf, kv->xwords * 8));
    CK(cudaMemset(kv->xbuf, 0, kv->xwords * 8));
    CK(cudaDeviceSynchronize());
    *out = kv.release();
    return MI_CUDA_OK;
  }
  int rc = capture(kv.get(), true, &kv->g_head, &kv->kernels_per_step);
  if (!rc) rc = capture(kv.get(), false, &kv->g_nohead, nullptr);
  if (rc && kv->persist) {
    // Retry with the kernel-per-phase step if the persistent launch was refused.
    kv->persist = false;
    if (kv->g_head) cudaGraphExecDestroy(kv->g_head);
    kv->g_head = nullptr;
    cudaGetLastError();
    rc = capture(kv.get(), true, &kv->g_head, &kv->kernels_per_step);
    if (!rc) rc = capture(kv.get(), false, &kv->g_nohead, nullptr);
  }
  if (rc && kv->fused) {
    // Retry with the two-kernel QKV + attention path if the cluster launch was refused.
    kv->fused = false;
    if (kv->g_head) cudaGraphExecDestroy(kv->g_head);
    kv->g_head = nullptr;
    cudaGetLastError();
    rc = capture(kv.get(), true, &kv->g_head, &kv->kernels_per_step);
    if (!rc) rc = capture(kv.get(), false, &kv->g_nohead, nullptr);
  }
  if (rc) {
    // Retry without programmatic dependent launch if the graph refused it.
    kv->pdl = false;
    if (kv->g_head) cudaGraphExecDestroy(kv->g_head);
    kv->g_head = nullptr;
    cudaGetLastError();
    rc = capture(kv.get(), true, &kv->g_head, &kv->kernels_per_step);
    if (!rc) rc = capture(kv.get(), false, &kv->g_nohead, nullptr);
    if (rc) return rc;
  }
  *out = kv.release();
  return MI_CUDA_OK;
}

int mi_cuda_tp_exchange_handle(mi_cuda_kv_cache* kv, void* handle_out) {
  if (!kv || !handle_out || !kv->xbuf)
    return fail(MI_CUDA_ERR_ARG, "mi_cuda_tp_exchange_handle: not a sharded model's KV cache");
  CK(cudaSetDevice(kv->model->device));
  cudaIpcMemHandle_t h;
  CK(cudaIpcGetMemHandle(&h, kv->xbuf));
  std::memcpy(handle_out, &h, sizeof(h));
  return MI_CUDA_OK;
}

int mi_cuda_tp_connect(mi_cuda_kv_cache* kv, const void* handles) {
  if (!kv || !handles || !kv->xbuf || kv->connected)
    return fail(MI_CUDA_ERR_ARG, "mi_cuda_tp_connect: bad arguments or already connected");
  mi_cuda_model* m = kv->model;
  CK(cudaSetDevice(m->device));
  for (int r = 0; r < m->world; r++) {
    if (r == m->rank) {
      kv->peer[r] = kv->xbuf;
      continue;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, (const uint8_t*)handles + (size_t)r * sizeof(h), sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess)
      return fail(MI_CUDA_ERR_CUDA, std::string("cudaIpcOpenMemHandle (rank ") + std::to_string(r) +
                                        "): " + cudaGetErrorString(e));
    kv->peer[r] = (uint64_t*)p;
  }
  int rc = capture(kv, true, &kv->g_head, &kv->kernels_per_step);
  if (!rc) rc = capture(kv, false, &kv->g_nohead, nullptr);
  if (rc) return rc;
  kv->connected = true;
  return MI_CUDA_OK;
}

int32_t mi_cuda_ipc_handle_bytes(void) { return (int32_t)sizeof(cudaIpcMemHandle_t); }

void mi_cuda_kv_cache_free(mi_cuda_kv_cache* kv) {
  if (!kv) return;
  cudaSetDevice(kv->model->device);
  if (kv->stream) cudaStreamSynchronize(kv->stream);
  for (int r = 0; r < kMaxRanks; r++)
    if (kv->peer[r] && kv->peer[r] != kv->xbuf) cudaIpcCloseMemHandle(kv->peer[r]);
  if (kv->xbuf) cudaFree(kv->xbuf);
  if (kv->pbuf) cudaFree(kv->pbuf);
  if (kv->pLogits) cudaFree(kv->pLogits);
  if (kv->g_head) cudaGraphExecDestroy(kv->g_head);
  if (kv->g_nohead) cudaGraphExecDestroy(kv->g_nohead);
  if (kv->g_fast_head) cudaGraphExecDestroy(kv->g_fast_head);
  if (kv->g_fast_nohead) cudaGraphExecDestroy(kv->g_fast_nohead);
  for (auto& e : kv->ev)
    if (e) cudaEventDestroy(e);
  if (kv->stream) cudaStreamDestroy(kv->stream);
  if (kv->h_state) cudaFreeHost(kv->h_state);
  if (kv->h_seen) cudaFreeHost(kv->h_seen);
  if (kv->h_tokens) cudaFreeHost(kv->h_tokens);
  cudaFree(kv->buf);
  delete kv;
}

int mi_cuda_qwen2_set_position(mi_cuda_kv_cache* kv, const int32_t* h_tokens, int32_t n,
                               int32_t pos) {
  if (!kv || n < 0 || n > kv->n_ctx + 1 || pos < 0 || pos > kv->n_ctx || (n > 0 && !h_tokens))
    return fail(MI_CUDA_ERR_ARG, "mi_cuda_qwen2_set_position: bad arguments");
  kv->seen_valid = false;
  CK(cudaSetDevice(kv->model->device));
  CK(cudaStreamSynchronize(kv->stream));
  if (n > 0) {
    std::memcpy(kv->h_tokens, h_tokens, (size_t)n * 4);
    CK(cudaMemcpyAsync(kv->tokens, kv->h_tokens, (size_t)n * 4, cudaMemcpyHostToDevice, kv->stream));
  }
  *kv->h_state = StepState{};
  kv->h_state->pos = pos;
  kv->h_state->feedback = 1;
  CK(cudaMemcpyAsync(kv->state, kv->h_state, sizeof(StepState), cudaMemcpyHostToDevice, kv->stream));
  // a fresh start for the persistent step's hand-over counters (a step that
  // gave up part-way leaves them behind their targets)
  CK(cudaMemsetAsync(kv->pctr, 0, ((size_t)kv->model->hp.n_layer * 4 + 2) * 8, kv->stream));
  return MI_CUDA_OK;
}

int mi_cuda_qwen2_decode_steps(mi_cuda_kv_cache* kv, int32_t n_steps, int32_t pos0,
                               int32_t period) {
  if (!kv || n_steps < 0 || period < 0 || pos0 < 0 || pos0 >= kv->n_ctx)
    return fail(MI_CUDA_ERR_ARG, "mi_cuda_qwen2_decode_steps: bad arguments");
  if (int rc = graphs_ready(kv)) return rc;
  kv->seen_valid = false;
  CK(cudaSetDevice(kv->model->device));
  for (int32_t i = 0; i < n_steps; i++) {
    if (period > 0 && i > 0 && i % period == 0) CK(launch_set_pos(&kv->state->pos, pos0, kv->stream));
    CK(cudaGraphLaunch(head_graph(kv), kv->stream));
  }
  return MI_CUDA_OK;
}

int mi_cuda_qwen2_read_tokens(mi_cuda_kv_cache* kv, int32_t first, int32_t n, int32_t* h_out) {
  if (!kv || !h_out || first < 0 || n < 0 || first + n > kv->n_ctx + 1)
    return fail(MI_CUDA_ERR_ARG, "mi_cuda_qwen2_read_tokens: bad arguments");
  CK(cudaSetDevice(kv->model->device));
  CK(cudaMemcpyAsync(kv->h_tokens + first, kv->tokens + first, (size_t)n * 4, cudaMemcpyDeviceToHost,
                     kv->stream));
  int rc = check_state_error(kv);
  if (rc) return rc;
  std::memcpy(h_out, kv->h_tokens + first, (size_t)n * 4);
  return MI_CUDA_OK;
}

mi_cuda_stream mi_cuda_qwen2_stream(mi_cuda_kv_cache* kv) { return kv ? (mi_cuda_stream)kv->stream : nullptr; }

int32_t mi_cuda_qwen2_kernels_per_step(mi_cuda_kv_cache* kv) { return kv ? kv->kernels_per_step : 0; }

int mi_cuda_qwen2_set_fast_mode(mi_cuda_kv_cache* kv, int32_t on) {
  if (!kv || (on != 0 && on != 1)) return fail(MI_CUDA_ERR_ARG, "mi_cuda_qwen2_set_fast_mode: bad arguments");
  if (on && !kv->persist)
    return fail(MI_CUDA_ERR_STATE, "fast mode needs the persistent one-kernel step (one GPU, a supported shape)");
  if ((on != 0) == kv->fast) return MI_CUDA_OK;
  kv->seen_valid = false;
  CK(cudaSetDevice(kv->model->device));
  CK(cudaStreamSynchronize(kv->stream));
  if (on && !kv->g_fast_head) {
    kv->fast = true;
    int rc = capture(kv, true, &kv->g_fast_head, nullptr);
    if (!rc) rc = capture(kv, false, &kv->g_fast_nohead, nullptr);
    kv->fast = false;
    if (rc) {
      if (kv->g_fast_head) cudaGraphExecDestroy(kv->g_fast_head);
      kv->g_fast_head = nullptr;
      cudaGetLastError();
      return rc;
    }
  }
  kv->fast = on != 0;
  return MI_CUDA_OK;
}

int32_t mi_cuda_qwen2_fast_mode(mi_cuda_kv_cache* kv) { return kv && kv->fast ? 1 : 0; }

int mi_cuda_qwen2_step_trace(mi_cuda_kv_cache* kv, uint64_t* h_out, int32_t max_slots,
                             int32_t* n_slots) {
  if (!kv || !h_out || max_slots < 0 || !n_slots)
    return fail(MI_CUDA_ERR_ARG, "mi_cuda_qwen2_step_trace: bad arguments");
  CK(cudaSetDevice(kv->model->device));
  CK(cudaStreamSynchronize(kv->stream));
  const int32_t n = std::min(max_slots, kv->trace_slots);
  CK(cudaMemcpy(h_out, kv->trace, (size_t)n * kTraceStamps * 8, cudaMemcpyDeviceToHost));
  *n_slots = n;
  return MI_CUDA_OK;
}

int mi_cuda_qwen2_forward(mi_cuda_model* m, mi_cuda_kv_cache* kv, const int32_t* h_tokens,
                          int32_t n_tokens, int32_t n_past, int32_t last_logits_only,
                          float* h_logits_out) {
  if (!m || !kv || kv->model != m || !h_tokens || n_tokens <= 0 || n_past < 0)
    return fail(MI_CUDA_ERR_ARG, "mi_cuda_qwen2_forward: bad arguments");
  if (n_past + n_tokens > kv->n_ctx)
    return fail(MI_CUDA_ERR_STATE, "mi_cuda_qwen2_forward: n_past + n_tokens exceeds n_ctx");
  if (int rc = graphs_ready(kv)) return rc;
  for (int32_t i = 0; i < n_tokens; i++)
    if (h_tokens[i] < 0 || h_tokens[i] >= m->hp.n_vocab)
      return fail(MI_CUDA_ERR_ARG, "mi_cuda_qwen2_forward: token id out of range");
  kv->seen_valid = false;
  CK(cudaSetDevice(m->device));
  CK(cudaStreamSynchronize(kv->stream));
  std::memcpy(kv->h_tokens + n_past, h_tokens, (size_t)n_tokens * 4);
  CK(cudaMemcpyAsync(kv->tokens + n_past, kv->h_tokens + n_past, (size_t)n_tokens * 4,
                     cudaMemcpyHostToDevice, kv->stream));
  *kv->h_state = StepState{};
  kv->h_state->pos = n_past;
  kv->h_state->feedback = 0;
  const size_t V = (size_t)m->hp.n_vocab;
  if (use_batched_prefill(kv, n_tokens)) {
    if (int rc = pack_prefill_copies(m, kv->stream)) return rc;
    kv->h_state->pos = n_past + n_tokens - 1;
    CK(cudaMemcpyAsync(kv->state, kv->h_state, sizeof(StepState), cudaMemcpyHostToDevice, kv->stream));
    const bool all = !last_logits_only && h_logits_out;
    if (int rc = enqueue_prefill(kv, n_tokens, n_past, all)) return rc;
    if (h_logits_out) {
      if (all)
        CK(cudaMemcpyAsync(h_logits_out, kv->pLogits, (size_t)(n_tokens - 1) * V * 4, cudaMemcpyDeviceToHost,
                           kv->stream));
      float* last = h_logits_out + (last_logits_only ? 0 : (size_t)(n_tokens - 1) * V);
      CK(cudaMemcpyAsync(last, kv->logits, V * 4, cudaMemcpyDeviceToHost, kv->stream));
    }
    return check_state_error(kv);
  }
  CK(cudaMemcpyAsync(kv->state, kv->h_state, sizeof(StepState), cudaMemcpyHostToDevice, kv->stream));
  for (int32_t t = 0; t < n_tokens; t++) {
    const bool head = !last_logits_only || t == n_tokens - 1;
    CK(cudaGraphLaunch(head ? head_graph(kv) : nohead_graph(kv), kv->stream));
    if (head && h_logits_out) {
      // a sharded model fills its rows [v0, v0 + nv) of each logits row
      float* dst = h_logits_out + (last_logits_only ? 0 : (size_t)t * V) + m->sh.v0;
      CK(cudaMemcpyAsync(dst, kv->logits, (size_t)m->sh.nv * 4, cudaMemcpyDeviceToHost, kv->stream));
    }
  }
  return check_state_error(kv);
}

int mi_cuda_qwen2_last_token(mi_cuda_kv_cache* kv, int32_t* h_token_out) {
  if (!kv || !h_token_out) return fail(MI_CUDA_ERR_ARG, "null argument");
  if (kv->seen_valid) {  // nothing enqueued since the state was read back
    *h_token_out = kv->h_seen->next_token;
    return MI_CUDA_OK;
  }
  CK(cudaSetDevice(kv->model->device));
  CK(cudaMemcpyAsync(&kv->h_state->next_token, &kv->state->next_token, 4, cudaMemcpyDeviceToHost,
                     kv->stream));
  CK(cudaStreamSynchronize(kv->stream));
  *h_token_out = kv->h_state->next_token;
  return MI_CUDA_OK;
}

int32_t mi_cuda_qwen2_sample_greedy(const float* h_logits, int32_t n_vocab) {
  int32_t best = 0;
  float bv = h_logits[0];
  for (int32_t i = 1; i < n_vocab; i++)
    if (h_logits[i] > bv) {
      bv = h_logits[i];
      best = i;
    }
  return best;
}

int mi_cuda_qwen2_generate(mi_cuda_model* m, mi_cuda_kv_cache* kv, const int32_t* h_prompt,
                           int32_t n_prompt, int32_t n_predict, int32_t* h_tokens_out,
                           double* prefill_ms, double* decode_ms) {
  if (!m || !kv || kv->model != m || !h_prompt || n_prompt <= 0 || n_predict <= 0 || !h_tokens_out)
    return fail(MI_CUDA_ERR_ARG, "mi_cuda_qwen2_generate: bad arguments");
  if (n_prompt > kv->n_ctx) return fail(MI_CUDA_ERR_STATE, "prompt longer than n_ctx");
  if (int rc = graphs_ready(kv)) return rc;
  for (int32_t i = 0; i < n_prompt; i++)
    if (h_prompt[i] < 0 || h_prompt[i] >= m->hp.n_vocab)
      return fail(MI_CUDA_ERR_ARG, "mi_cuda_qwen2_generate: token id out of range");
  int rc = mi_cuda_qwen2_set_position(kv, h_prompt, n_prompt, 0);
  if (rc) return rc;
  // The reference loop stops once n_past reaches n_ctx (src/main.cpp:409-423).
  const int32_t n_decode = std::min<int32_t>(n_predict - 1, kv->n_ctx - n_prompt);
  if (use_batched_prefill(kv, n_prompt))
    if (int rc2 = pack_prefill_copies(kv->model, kv->stream)) return rc2;
  CK(cudaEventRecord(kv->ev[0], kv->stream));
  if (use_batched_prefill(kv, n_prompt)) {
    // the prompt in one batch; its LM head feeds the first token back
    kv->h_state->pos = n_prompt - 1;
    CK(cudaMemcpyAsync(kv->state, kv->h_state, sizeof(StepState), cudaMemcpyHostToDevice, kv->stream));
    if (int rc2 = enqueue_prefill(kv, n_prompt, 0, false)) return rc2;
  } else {
    for (int32_t t = 0; t + 1 < n_prompt; t++) CK(cudaGraphLaunch(nohead_graph(kv), kv->stream));
    CK(cudaGraphLaunch(head_graph(kv), kv->stream));
  }
  CK(cudaEventRecord(kv->ev[1], kv->stream));
  for (int32_t i = 0; i < n_decode; i++) CK(cudaGraphLaunch(head_graph(kv), kv->stream));
  CK(cudaEventRecord(kv->ev[2], kv->stream));
  const int32_t produced = 1 + n_decode;
  CK(cudaMemcpyAsync(kv->h_tokens, kv->tokens + n_prompt, (size_t)produced * 4,
                     cudaMemcpyDeviceToHost, kv->stream));
  rc = check_state_error(kv);
  if (rc) return rc;
  std::memcpy(h_tokens_out, kv->h_tokens, (size_t)produced * 4);
  for (int32_t i = produced; i < n_predict; i++) h_tokens_out[i] = -1;
  float a = 0, b = 0;
  CK(cudaEventElapsedTime(&a, kv->ev[0], kv->ev[1]));
  CK(cudaEventElapsedTime(&b, kv->ev[1], kv->ev[2]));
  if (prefill_ms) *prefill_ms = a;
  if (decode_ms) *decode_ms = b;
  return MI_CUDA_OK;
}

}  // extern "C"
