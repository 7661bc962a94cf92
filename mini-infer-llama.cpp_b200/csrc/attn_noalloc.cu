// mi_cuda_attention_decode_noalloc: the fused decode-attention op without a
// caller-provided scratch buffer and without any device allocation.
//
// Who needs it: callers that hold only their input and output buffers and may
// not allocate device memory on the call path -- a host whose runtime contract is
// "no allocation after start-up" (mini-infer's own decode step makes zero heap
// allocations, reference tests/test_zero_alloc.cpp), code running while the
// caller records its own CUDA graph (cudaMalloc is not a capturable operation),
// or a plugin host that owns all device memory through its own pool.
//
// The per-head score scratch lives in g_attn_scratch, a file-scope __device__
// array of kMaxScratchFloats floats (4 MiB): every GPU that loads the library
// holds it until the process exits. Host code cannot use the array's name as a
// device address (in host code it names a host-side shadow), so the first call
// on each device looks the device address up with cudaGetSymbolAddress, with
// that device current, and caches it; that first call may load the module and
// should therefore come before any stream capture. Later calls only launch.
//
// All calls on a device share the one array, which keeps the last call's
// contents; the kernel writes every score before reading it, so nothing needs
// clearing. Calls whose kernels can overlap on the GPU (different streams with
// no ordering between them) race on the array and must be serialized by the
// caller.
#include <mutex>
#include <string>

#include "mi_cuda.h"
#include "mi_internal.h"

namespace {

constexpr int64_t kMaxScratchFloats = 1 << 20;  // n_head * n_kv <= 1,048,576
constexpr int kMaxDevices = 64;

__device__ __align__(256) float g_attn_scratch[kMaxScratchFloats];

float* g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mu;

int fail(int code, const char* msg) {
  mi::set_error(msg);
  return code;
}

}  // namespace

extern "C" int mi_cuda_attention_decode_noalloc(const float* d_q, const float* d_cache_k,
                                                const float* d_cache_v, int64_t head_dim,
                                                int64_t n_head, int64_t n_head_kv, int64_t n_kv,
                                                float scale, float* d_dst, mi_cuda_stream s) {
  if (!d_q || !d_cache_k || !d_cache_v || !d_dst || head_dim <= 0 || head_dim > 256 ||
      head_dim % 4 != 0 || n_head <= 0 || n_head >= (1ll << 31) || n_head_kv <= 0 ||
      n_head % n_head_kv != 0 || n_kv <= 0 || n_kv >= (1ll << 31))
    return fail(MI_CUDA_ERR_ARG, "mi_cuda_attention_decode_noalloc: bad arguments");
  if (n_head * n_kv > kMaxScratchFloats)
    return fail(MI_CUDA_ERR_ARG,
                "mi_cuda_attention_decode_noalloc: n_head * n_kv exceeds the static scratch "
                "capacity of 1048576 scores; use mi_cuda_attention_decode with a caller buffer");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(MI_CUDA_ERR_CUDA, "mi_cuda_attention_decode_noalloc: no usable current device");
  // The expf table comes from mi_cuda_init, which is where the library makes its
  // one-time allocations; this entry point never creates that context itself.
  const mi::DeviceCtx* ctx = mi::existing_device_ctx(dev);
  if (!ctx)
    return fail(MI_CUDA_ERR_STATE,
                "mi_cuda_attention_decode_noalloc: call mi_cuda_init(device) once at start-up first");
  float* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[dev]) {
      void* p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
      if (e != cudaSuccess || !p)
        return fail(MI_CUDA_ERR_CUDA, "mi_cuda_attention_decode_noalloc: cudaGetSymbolAddress failed");
      g_scratch_addr[dev] = (float*)p;
    }
    scratch = g_scratch_addr[dev];
  }
  mi::AttnParams p{};
  p.q_rot = d_q;
  p.cache_k = (float*)d_cache_k;
  p.cache_v = (float*)d_cache_v;
  p.head_dim = (int32_t)head_dim;
  p.n_head = (int32_t)n_head;
  p.n_head_kv = (int32_t)n_head_kv;
  p.n_kv_fixed = (int32_t)n_kv;
  p.scale = scale;
  p.scores = scratch;
  p.scores_stride = n_kv;
  p.out = d_dst;
  p.et = ctx->et;
  p.err = ctx->err;
  cudaError_t e = mi::launch_attn_decode(p, false, (cudaStream_t)s, false);
  if (e != cudaSuccess) return fail(MI_CUDA_ERR_CUDA, cudaGetErrorString(e));
  return MI_CUDA_OK;
}
