// Per-op C-ABI entry points (include/mi_cuda.h) and the library's per-device
// state: the expf exception table on the device, the device error word, and
// the small scratch buffers the op entry points use.
#include <dlfcn.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "mi_cuda.h"
#include "mi_expf_core.h"
#include "mi_internal.h"

namespace mi {

namespace {

thread_local std::string g_error;
std::mutex g_mu;
std::vector<DeviceCtx*> g_ctx;

std::string lib_dir() {
  Dl_info info{};
  if (dladdr((void*)&lib_dir, &info) && info.dli_fname) {
    std::string p = info.dli_fname;
    size_t k = p.rfind('/');
    if (k != std::string::npos) return p.substr(0, k);
  }
  return ".";
}

bool load_expf_table(DeviceCtx* c, std::string* err) {
  const char* env = std::getenv("MI_CUDA_EXPF_TABLE");
  const std::string path = env ? env : lib_dir() + "/expf_exceptions.bin";
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) {
    *err = "expf exception table not found at " + path + " (build the library first)";
    return false;
  }
  mi_expf_table_header h{};
  bool ok = std::fread(&h, sizeof(h), 1, f) == 1 && h.magic == MI_EXPF_MAGIC &&
            h.log2_buckets >= 1 && h.log2_buckets <= 28;
  std::vector<uint32_t> slots;
  if (ok) {
    slots.resize(((size_t)1 << h.log2_buckets) * MI_EXPF_SLOTS * 2);
    ok = std::fread(slots.data(), 4, slots.size(), f) == slots.size();
  }
  std::fclose(f);
  if (!ok) {
    *err = "expf exception table " + path + " is corrupt";
    return false;
  }
  uint32_t core = 0, libm = 0;
  expf_fingerprints(&core, &libm);
  if (core != h.core_checksum || libm != h.libm_checksum) {
    *err = "expf exception table " + path +
           " was built for a different libm or build of the exp core; rebuild it on this host";
    return false;
  }
  if (cudaMalloc(&c->et_buf, slots.size() * 4) != cudaSuccess ||
      cudaMemcpy(c->et_buf, slots.data(), slots.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
    *err = "failed to upload the expf table";
    return false;
  }
  c->et.buckets = (const uint4*)c->et_buf;
  c->et.log2b = h.log2_buckets;
  c->et.mul1 = h.mul1;
  c->et.mul2 = h.mul2;
  c->et.filter = (h.flags & MI_EXPF_FLAG_TIE_FILTER) ? 1u : 0u;
  return true;
}

}  // namespace

void set_error(const std::string& msg) { g_error = msg; }

DeviceCtx* device_ctx(int device, std::string* err) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (device < 0) {
    *err = "invalid device";
    return nullptr;
  }
  if ((size_t)device < g_ctx.size() && g_ctx[(size_t)device]) return g_ctx[(size_t)device];
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device >= n) {
    *err = "CUDA device " + std::to_string(device) + " is not available";
    return nullptr;
  }
  if (cudaSetDevice(device) != cudaSuccess) {
    *err = "cudaSetDevice failed";
    return nullptr;
  }
  auto* c = new DeviceCtx();
  c->device = device;
  cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device);
  if (!load_expf_table(c, err)) {
    delete c;
    return nullptr;
  }
  if (prepare_kernels() != cudaSuccess) {
    *err = "cudaFuncSetAttribute failed";
    delete c;
    return nullptr;
  }
  if (cudaMalloc(&c->err, 4) != cudaSuccess || cudaMemset(c->err, 0, 4) != cudaSuccess ||
      cudaMalloc(&c->am_val, 1024 * 4) != cudaSuccess ||
      cudaMalloc(&c->am_idx, 1024 * 4) != cudaSuccess ||
      cudaMalloc(&c->am_counter, 4) != cudaSuccess ||
      cudaMemset(c->am_counter, 0, 4) != cudaSuccess) {
    *err = "device allocation failed during init";
    delete c;
    return nullptr;
  }
  if (g_ctx.size() <= (size_t)device) g_ctx.resize((size_t)device + 1, nullptr);
  g_ctx[(size_t)device] = c;
  return c;
}

const DeviceCtx* existing_device_ctx(int device) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (device < 0 || (size_t)device >= g_ctx.size()) return nullptr;
  return g_ctx[(size_t)device];
}

DeviceCtx* current_ctx(std::string* err) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    *err = "no CUDA device";
    return nullptr;
  }
  return device_ctx(dev, err);
}

}  // namespace mi

using namespace mi;

namespace {

int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return MI_CUDA_OK;
  return fail(MI_CUDA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

#define MI_CTX(c)                                          \
  std::string _err;                                        \
  DeviceCtx* c = current_ctx(&_err);                       \
  if (!c) return fail(MI_CUDA_ERR_CUDA, _err)

#define MI_REQUIRE(cond, msg) \
  if (!(cond)) return fail(MI_CUDA_ERR_ARG, msg)

cudaStream_t S(mi_cuda_stream s) { return (cudaStream_t)s; }

int64_t npad8(int64_t n) { return (n + 7) / 8 * 8; }

}  // namespace

extern "C" {

const char* mi_cuda_last_error(void) { return g_error.c_str(); }

int mi_cuda_init(int device) {
  std::string err;
  if (!device_ctx(device, &err)) return fail(MI_CUDA_ERR_CUDA, err);
  if (cudaSetDevice(device) != cudaSuccess) return fail(MI_CUDA_ERR_CUDA, "cudaSetDevice failed");
  return MI_CUDA_OK;
}

int mi_cuda_device_error(int device, int32_t* code_out) {
  std::string err;
  DeviceCtx* c = device_ctx(device, &err);
  if (!c) return fail(MI_CUDA_ERR_CUDA, err);
  cudaSetDevice(device);
  int32_t v = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(&v, c->err, 4, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemset(c->err, 0, 4);
  if (code_out) *code_out = v;
  return cuda_status(e, "mi_cuda_device_error");
}

size_t mi_cuda_q8_0_packed_bytes(int64_t k, int64_t n) {
  if (k <= 0 || n <= 0 || k % 32 != 0) return 0;
  const int64_t np = npad8(n);
  return (size_t)(np * k + np * (k / 32) * 2);
}

int mi_cuda_q8_0_pack(const void* d_raw, int64_t k, int64_t n, void* d_packed, mi_cuda_stream s) {
  MI_CTX(c);
  MI_REQUIRE(d_raw && d_packed && k > 0 && n > 0 && k % 32 == 0, "mi_cuda_q8_0_pack: bad arguments");
  const int64_t np = npad8(n);
  cudaError_t e = launch_zero_pad_rows((uint8_t*)d_packed, k, np, S(s));
  if (e == cudaSuccess)
    e = launch_pack_q8_0((const uint8_t*)d_raw, k, n, 0, (uint8_t*)d_packed, np, 0, 4, S(s));
  return cuda_status(e, "mi_cuda_q8_0_pack");
}

int mi_cuda_quantize_q8_0_act(const float* d_x, int64_t k, int64_t m, void* d_act,
                              mi_cuda_stream s) {
  MI_CTX(c);
  MI_REQUIRE(d_x && d_act && k > 0 && m >= 0 && k % 32 == 0, "mi_cuda_quantize_q8_0_act: bad arguments");
  return cuda_status(launch_quantize_act(d_x, k, m, (uint8_t*)d_act, S(s)), "quantize_q8_0_act");
}

static int mul_mat_common(const void* d_w, int64_t k, int64_t n, const void* d_in, int64_t m,
                          float* d_dst, mi_cuda_stream s, int pro) {
  MI_CTX(c);
  MI_REQUIRE(d_w && d_in && d_dst && k > 0 && n > 0 && m >= 0 && k % 32 == 0,
             "mi_cuda_mul_mat_q8_0: bad arguments");
  const GemvPlan plan = plan_gemv(k, n, c->num_sms, pro);
  for (int64_t j = 0; j < m; j++) {
    GemvParams p{};
    p.w = (const uint8_t*)d_w;
    p.K = k;
    p.N = n;
    p.n_pad = npad8(n);
    p.pro = pro;
    p.epi = EPI_STORE;
    if (pro == PRO_ACT) p.act = (const uint8_t*)d_in + j * (k / 32) * 36;
    else p.x = (const float*)d_in + j * k;
    p.out = d_dst + j * n;
    p.et = c->et;
    p.err = c->err;
    cudaError_t e = launch_gemv(p, plan, S(s), false);
    if (e != cudaSuccess) return cuda_status(e, "mul_mat_q8_0");
  }
  return MI_CUDA_OK;
}

int mi_cuda_mul_mat_q8_0(const void* d_w_packed, int64_t k, int64_t n, const void* d_act,
                         int64_t m, float* d_dst, mi_cuda_stream s) {
  return mul_mat_common(d_w_packed, k, n, d_act, m, d_dst, s, PRO_ACT);
}

int mi_cuda_mul_mat_q8_0_f32(const void* d_w_packed, int64_t k, int64_t n, const float* d_x,
                             int64_t m, float* d_dst, mi_cuda_stream s) {
  return mul_mat_common(d_w_packed, k, n, d_x, m, d_dst, s, PRO_QUANT);
}

int mi_cuda_mul_mat_q8_0_scalar(const void* d_w_packed, int64_t k, int64_t n, const void* d_act,
                                int64_t m, float* d_dst, mi_cuda_stream s) {
  MI_CTX(c);
  MI_REQUIRE(d_w_packed && d_act && d_dst && k > 0 && n > 0 && m >= 0 && m <= 65535 && k % 32 == 0,
             "mi_cuda_mul_mat_q8_0_scalar: bad arguments");
  return cuda_status(launch_gemv_scalar_order((const uint8_t*)d_w_packed, k, n, npad8(n),
                                              (const uint8_t*)d_act, m, d_dst, S(s)),
                     "mul_mat_q8_0_scalar");
}

int mi_cuda_q8_0_block_isums(const void* d_w_packed, int64_t k, int64_t n, const void* d_act,
                             int32_t* d_isums, mi_cuda_stream s) {
  MI_CTX(c);
  MI_REQUIRE(d_w_packed && d_act && d_isums && k > 0 && n > 0 && k % 32 == 0,
             "mi_cuda_q8_0_block_isums: bad arguments");
  return cuda_status(launch_block_isums((const uint8_t*)d_w_packed, k, n, npad8(n),
                                        (const uint8_t*)d_act, d_isums, S(s)),
                     "q8_0_block_isums");
}

int mi_cuda_get_rows_q8_0(const void* d_table_packed, int64_t ne0, int64_t n_rows,
                          const int32_t* d_ids, int64_t n_ids, float* d_dst, mi_cuda_stream s) {
  MI_CTX(c);
  MI_REQUIRE(d_table_packed && d_ids && d_dst && ne0 > 0 && ne0 % 32 == 0 && n_rows > 0,
             "mi_cuda_get_rows_q8_0: bad arguments");
  return cuda_status(launch_get_rows((const uint8_t*)d_table_packed, ne0, npad8(n_rows), d_ids,
                                     n_ids, d_dst, S(s)),
                     "get_rows_q8_0");
}

int mi_cuda_rms_norm(const float* d_x, int64_t ne0, int64_t n_rows, float eps, float* d_dst,
                     mi_cuda_stream s) {
  MI_CTX(c);
  MI_REQUIRE(d_x && d_dst && ne0 > 0 && n_rows >= 0, "mi_cuda_rms_norm: bad arguments");
  return cuda_status(launch_rms_norm(d_x, ne0, n_rows, eps, d_dst, S(s)), "rms_norm");
}

int mi_cuda_mul(const float* d_a, const float* d_b, int64_t ne0, int64_t n_rows, int64_t b_rows,
                float* d_dst, mi_cuda_stream s) {
  MI_CTX(c);
  MI_REQUIRE(d_a && d_b && d_dst && (b_rows == 1 || b_rows == n_rows), "mi_cuda_mul: bad arguments");
  return cuda_status(launch_binop(0, d_a, d_b, ne0, n_rows, b_rows, 0.0f, d_dst, S(s)), "mul");
}

int mi_cuda_add(const float* d_a, const float* d_b, int64_t ne0, int64_t n_rows, int64_t b_rows,
                float* d_dst, mi_cuda_stream s) {
  MI_CTX(c);
  MI_REQUIRE(d_a && d_b && d_dst && (b_rows == 1 || b_rows == n_rows), "mi_cuda_add: bad arguments");
  return cuda_status(launch_binop(1, d_a, d_b, ne0, n_rows, b_rows, 0.0f, d_dst, S(s)), "add");
}

int mi_cuda_scale(const float* d_x, int64_t n, float v, float* d_dst, mi_cuda_stream s) {
  MI_CTX(c);
  MI_REQUIRE(d_x && d_dst && n >= 0, "mi_cuda_scale: bad arguments");
  return cuda_status(launch_binop(2, d_x, nullptr, n, 1, 1, v, d_dst, S(s)), "scale");
}

int mi_cuda_silu(const float* d_x, int64_t n, float* d_dst, mi_cuda_stream s) {
  MI_CTX(c);
  MI_REQUIRE(d_x && d_dst && n >= 0, "mi_cuda_silu: bad arguments");
  return cuda_status(launch_silu(d_x, n, d_dst, c->et, S(s)), "silu");
}

int mi_cuda_expf(const float* d_x, int64_t n, float* d_y, mi_cuda_stream s) {
  MI_CTX(c);
  MI_REQUIRE(d_x && d_y && n >= 0, "mi_cuda_expf: bad arguments");
  return cuda_status(launch_expf(d_x, n, d_y, c->et, S(s)), "expf");
}

int mi_cuda_expf_verify(uint64_t first, uint64_t count, uint64_t* n_mismatch) {
  MI_CTX(c);
  MI_REQUIRE(n_mismatch && first + count <= (1ull << 32), "mi_cuda_expf_verify: bad arguments");
  const int64_t chunk = 1 << 26;
  float* d = nullptr;
  float* h = nullptr;
  cudaError_t e = cudaMalloc(&d, (size_t)chunk * 4);
  if (e == cudaSuccess) e = cudaMallocHost(&h, (size_t)chunk * 4);
  uint64_t total = 0;
  for (uint64_t off = 0; off < count && e == cudaSuccess; off += (uint64_t)chunk) {
    const int64_t nn = (int64_t)std::min<uint64_t>((uint64_t)chunk, count - off);
    e = launch_expf_range(first + off, nn, d, c->et, 0);
    if (e == cudaSuccess) e = cudaMemcpy(h, d, (size_t)nn * 4, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) total += expf_count_mismatch(first + off, nn, h);
  }
  if (d) cudaFree(d);
  if (h) cudaFreeHost(h);
  *n_mismatch = total;
  return cuda_status(e, "expf_verify");
}

int mi_cuda_rope_neox(const float* d_x, int64_t head_dim, int64_t n_head, int64_t n_tokens,
                      int32_t n_past, int32_t n_dims, float freq_base, float* d_dst,
                      mi_cuda_stream s) {
  MI_CTX(c);
  MI_REQUIRE(d_x && d_dst && head_dim > 0 && n_dims > 0 && n_dims <= head_dim && n_dims % 2 == 0 &&
                 n_past >= 0 && n_tokens >= 0,
             "mi_cuda_rope_neox: bad arguments");
  const int32_t need = n_past + (int32_t)n_tokens;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!c->rope || c->rope_n_pos < need || c->rope_n_dims != n_dims || c->rope_base != freq_base) {
    int32_t n_pos = std::max<int32_t>(need, std::max<int32_t>(4096, c->rope_n_pos));
    std::vector<float> cs((size_t)n_pos * (n_dims / 2) * 2);
    build_rope_table(0, n_pos, n_dims, freq_base, cs.data());
    cudaDeviceSynchronize();  // no kernel may still read the old table
    if (c->rope) cudaFree(c->rope);
    c->rope = nullptr;
    cudaError_t e = cudaMalloc(&c->rope, cs.size() * 4);
    if (e == cudaSuccess) e = cudaMemcpy(c->rope, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_status(e, "rope table");
    c->rope_n_pos = n_pos;
    c->rope_n_dims = n_dims;
    c->rope_base = freq_base;
  }
  return cuda_status(launch_rope(d_x, head_dim, n_head, n_tokens, n_dims,
                                 c->rope + (size_t)n_past * (n_dims / 2), d_dst, S(s)),
                     "rope");
}

int mi_cuda_attn_qk(const float* d_q, const float* d_cache_k, int64_t head_dim, int64_t n_head,
                    int64_t n_head_kv, int64_t n_kv, int64_t n_tokens, float* d_scores,
                    mi_cuda_stream s) {
  MI_CTX(c);
  MI_REQUIRE(d_q && d_cache_k && d_scores && head_dim > 0 && n_head_kv > 0 &&
                 n_head % n_head_kv == 0 && n_kv >= n_tokens,
             "mi_cuda_attn_qk: bad arguments");
  return cuda_status(launch_attn_qk(d_q, d_cache_k, head_dim, n_head, n_head_kv, n_kv, n_tokens,
                                    d_scores, S(s)),
                     "attn_qk");
}

int mi_cuda_softmax(const float* d_x, int64_t n_kv, int64_t n_tokens, int64_t n_head,
                    int32_t n_past, float scale, float* d_dst, mi_cuda_stream s) {
  MI_CTX(c);
  MI_REQUIRE(d_x && d_dst && n_kv > 0 && n_past >= 0, "mi_cuda_softmax: bad arguments");
  return cuda_status(launch_softmax(d_x, n_kv, n_tokens, n_head, n_past, scale, d_dst, c->et, S(s)),
                     "softmax");
}

int mi_cuda_attn_kqv(const float* d_probs, const float* d_cache_v, int64_t head_dim,
                     int64_t n_head, int64_t n_head_kv, int64_t n_kv, int64_t n_tokens,
                     float* d_dst, mi_cuda_stream s) {
  MI_CTX(c);
  MI_REQUIRE(d_probs && d_cache_v && d_dst && head_dim > 0 && n_head_kv > 0 &&
                 n_head % n_head_kv == 0,
             "mi_cuda_attn_kqv: bad arguments");
  return cuda_status(launch_attn_kqv(d_probs, d_cache_v, head_dim, n_head, n_head_kv, n_kv,
                                     n_tokens, d_dst, S(s)),
                     "attn_kqv");
}

size_t mi_cuda_attention_decode_scratch_bytes(int64_t n_head, int64_t n_kv) {
  return (size_t)(n_head * n_kv * 4);
}

int mi_cuda_attention_decode(const float* d_q, const float* d_cache_k, const float* d_cache_v,
                             int64_t head_dim, int64_t n_head, int64_t n_head_kv, int64_t n_kv,
                             float scale, void* d_scratch, float* d_dst, mi_cuda_stream s) {
  MI_CTX(c);
  MI_REQUIRE(d_q && d_cache_k && d_cache_v && d_scratch && d_dst && head_dim > 0 &&
                 head_dim <= 256 && head_dim % 4 == 0 && n_head > 0 && n_head < (1ll << 31) &&
                 n_head_kv > 0 && n_head % n_head_kv == 0 && n_kv > 0 && n_kv < (1ll << 31),
             "mi_cuda_attention_decode: bad arguments");
  AttnParams p{};
  p.q_rot = d_q;
  p.cache_k = (float*)d_cache_k;
  p.cache_v = (float*)d_cache_v;
  p.head_dim = (int32_t)head_dim;
  p.n_head = (int32_t)n_head;
  p.n_head_kv = (int32_t)n_head_kv;
  p.n_kv_fixed = (int32_t)n_kv;
  p.scale = scale;
  p.scores = (float*)d_scratch;
  p.scores_stride = n_kv;
  p.out = d_dst;
  p.et = c->et;
  p.err = c->err;
  return cuda_status(launch_attn_decode(p, false, S(s), false), "attention_decode");
}

size_t mi_cuda_attention_decode_split_scratch_bytes(int64_t n_head, int64_t n_head_kv, int64_t n_kv,
                                                    int64_t head_dim) {
  if (n_head <= 0 || n_head_kv <= 0 || n_kv <= 0 || head_dim <= 0) return 0;
  return attn_split_scratch_bytes(n_head, n_kv, n_head_kv, head_dim);
}

int mi_cuda_attention_decode_split(const float* d_q, const float* d_cache_k, const float* d_cache_v,
                                   int64_t head_dim, int64_t n_head, int64_t n_head_kv, int64_t n_kv,
                                   float scale, void* d_scratch, float* d_dst, mi_cuda_stream s) {
  MI_CTX(c);
  MI_REQUIRE(d_q && d_cache_k && d_cache_v && d_scratch && d_dst && n_kv > 0 && n_kv < (1ll << 31) &&
                 attn_split_fits(head_dim, n_head, n_head_kv) && (uintptr_t)d_cache_k % 16 == 0 &&
                 (uintptr_t)d_cache_v % 16 == 0 && (uintptr_t)d_scratch % 16 == 0,
             "mi_cuda_attention_decode_split: bad arguments (16-byte aligned caches and scratch)");
  return cuda_status(launch_attn_split(d_q, d_cache_k, d_cache_v, head_dim, n_head, n_head_kv, n_kv, scale,
                                       c->et, c->err, (float*)d_scratch, d_dst, S(s)),
                     "attention_decode_split");
}

int mi_cuda_argmax(const float* d_x, int64_t n, int32_t* d_out, mi_cuda_stream s) {
  MI_CTX(c);
  MI_REQUIRE(d_x && d_out && n > 0 && n < (1ll << 31), "mi_cuda_argmax: bad arguments");
  return cuda_status(launch_argmax(d_x, n, c->am_val, c->am_idx, c->am_counter, d_out, S(s)),
                     "argmax");
}

}  // extern "C"
