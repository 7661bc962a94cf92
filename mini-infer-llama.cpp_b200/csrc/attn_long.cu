// Exact decode attention of one query at long context (op mode, from 512
// positions): the reference's ATTN_QK / SOFTMAX / ATTN_KQV
// (src/ops_cpu.cpp:304-410) with every sum in the reference's order, spread
// over the GPU instead of one CTA per head.
//
// Only two of the reference's sums are chains: the softmax denominator and
// every output's value sum run over all n_kv positions in order. The rest is
// independent per position, so:
//   1. scores: CTAs of (128 positions, KV head) compute s[h][t] = (the d-
//      ascending dot of K row t and q_h, each product and sum rounded) *
//      scale for the KV head's n_rep query heads;
//   2. softmax: a CTA per head reads its scores into shared memory, takes
//      the maximum (order-free), e[t] = expf(s - max) (libm-exact), sums e in
//      order with spec_ordered_sum (bit-identical to the serial chain), and
//      writes p[t] = e[t] * (1 / sum) over the scores;
//   3. values: a CTA per (head, 8 outputs) streams p and its 8 V columns
//      through shared memory (double-buffered asynchronous copies: 16 bytes
//      of V, 4 bytes of p each) while 8 threads run the 8 ordered chains
//      out[o] += V[t][o] * p[t].
// K and V must be 16-byte aligned (the router checks).
// The chains of step 3 (n_kv dependent adds each) set the floor: ~4-5 cycles
// per position.
#include "mi_device.cuh"

namespace mi {

namespace {

constexpr int kLongNT = 256;
constexpr int kSoftNT = 1024;   // softmax CTA: the exponentials and 32 speculative segments
constexpr int kScoreTile = 128;   // positions per score CTA
constexpr int kValChunk = 2048;   // positions per value chunk (double-buffered; a multiple of 32)
constexpr int kValOut = 8;        // output chains per value CTA

// ---- 1. scores ----
__global__ void __launch_bounds__(kLongNT) attn_long_scores_kernel(const float* q, const float* ck, int D, int H,
                                                                  int HKV, int n_kv, float scale, float* sc,
                                                                  int64_t stride) {
  extern __shared__ __align__(16) float sm[];
  const int tid = threadIdx.x;
  const int kvh = blockIdx.y, t0 = blockIdx.x * kScoreTile;
  const int n_rep = H / HKV, h0 = kvh * n_rep, KP = D + 1, rows = min(kScoreTile, n_kv - t0);
  float* qs = sm;                // [R][D]
  float* Ks = qs + n_rep * D;    // [kScoreTile][D + 1] (odd stride: a warp reads 32 rows at one d)
  for (int e = tid; e < n_rep * D; e += kLongNT) qs[e] = q[(size_t)h0 * D + e];
  const size_t rs = (size_t)HKV * D;
  const int D4 = D >> 2;
  // the tile's K rows, eight 16-byte loads per thread in flight at a time
  for (int base = 0; base < rows * D4; base += 8 * kLongNT) {
    float4 v[8];
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int e = base + u * kLongNT + tid;
      if (e < rows * D4) {
        const int t = e / D4, c = e - t * D4;
        v[u] = __ldg((const float4*)(ck + (size_t)(t0 + t) * rs + (size_t)kvh * D) + c);
      }
    }
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int e = base + u * kLongNT + tid;
      if (e < rows * D4) {
        const int t = e / D4, c = e - t * D4;
        float* d = Ks + t * KP + 4 * c;
        d[0] = v[u].x;
        d[1] = v[u].y;
        d[2] = v[u].z;
        d[3] = v[u].w;
      }
    }
  }
  __syncthreads();
  for (int it = tid; it < rows * n_rep; it += kLongNT) {
    const int r = it / rows, t = it - r * rows;
    const float acc = ordered_dot(0.0f, Ks + t * KP, 1, qs + r * D, D);
    sc[(size_t)(h0 + r) * stride + t0 + t] = __fmul_rn(acc, scale);
  }
}

// ---- 2. softmax ----
__global__ void __launch_bounds__(kSoftNT) attn_long_softmax_kernel(float* sc, int64_t stride, int n_kv, ExpTab et) {
  extern __shared__ __align__(16) float es[];  // [n_kv (+ slack)], then the spec-sum scratch
  __shared__ float red[kSoftNT / 32];
  __shared__ float inv_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* row = sc + (size_t)blockIdx.x * stride;
  uint8_t* scratch = (uint8_t*)(es + ((n_kv + 3) / 4 * 4) + kChainSlackBytes / 4);
  // the row into shared memory, eight loads per thread in flight at a time
  float m = -INFINITY;
  for (int base = 0; base < n_kv; base += 8 * kSoftNT) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int i = base + u * kSoftNT + tid;
      v[u] = i < n_kv ? __ldcg(row + i) : -INFINITY;
    }
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int i = base + u * kSoftNT + tid;
      if (i < n_kv) es[i] = v[u];
      m = fmaxf(m, v[u]);
    }
  }
  m = warp_max(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  float mx = red[0];
  for (int w = 1; w < kSoftNT / 32; w++) mx = fmaxf(mx, red[w]);
  for (int i = tid; i < n_kv; i += kSoftNT) es[i] = expf_exact(__fsub_rn(es[i], mx), et);
  __syncthreads();
  // the denominator: one ordered chain (src/ops_cpu.cpp:331-336)
  const float sum = spec_ordered_sum<kSoftNT, 4>(es, n_kv, scratch);
  if (tid == 0) inv_s = __fdiv_rn(1.0f, sum);
  __syncthreads();
  const float inv = inv_s;
  // p = e * (1 / sum) (src/ops_cpu.cpp:338-341), over the scores
  for (int i = tid; i < n_kv; i += kSoftNT) row[i] = __fmul_rn(es[i], inv);
}

// ---- 3. values ----
__global__ void __launch_bounds__(kLongNT) attn_long_values_kernel(const float* p, int64_t stride, const float* cv,
                                                                  int D, int H, int HKV, int n_kv, float* out) {
  extern __shared__ __align__(16) float vsm[];  // V [2][kValChunk][8], then p [2][kValChunk]
  auto vbuf = [&](int b) { return vsm + b * (kValChunk * kValOut); };
  auto pbuf = [&](int b) { return vsm + 2 * kValChunk * kValOut + b * kValChunk; };
  const int tid = threadIdx.x;
  const int h = blockIdx.x, o0 = blockIdx.y * kValOut;
  const int kvh = h / (H / HKV);
  const float* prow = p + (size_t)h * stride;
  const float* vb = cv + (size_t)kvh * D + o0;
  const size_t rs = (size_t)HKV * D;
  const int n_chunks = (n_kv + kValChunk - 1) / kValChunk;
  // chunk c into buffer c & 1: per position 8 V floats (two 16-byte copies)
  // and its probability (a 4-byte copy: a head's row need not be 16-byte
  // aligned)
  auto issue = [&](int c) {
    if (c < n_chunks) {
      const int b = c & 1, t0 = c * kValChunk, rows = min(kValChunk, n_kv - t0);
      for (int e = tid; e < rows * 2; e += kLongNT) {
        const int t = e >> 1, hf = e & 1;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(vbuf(b) + t * kValOut + 4 * hf)),
                     "l"(vb + (size_t)(t0 + t) * rs + 4 * hf)
                     : "memory");
      }
      for (int t = tid; t < rows; t += kLongNT)
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(pbuf(b) + t)), "l"(prow + t0 + t)
                     : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  issue(0);
  float acc = 0.0f;
  for (int c = 0; c < n_chunks; c++) {
    issue(c + 1);
    asm volatile("cp.async.wait_group 1;" ::: "memory");  // chunk c landed
    __syncthreads();
    const int b = c & 1, rows = min(kValChunk, n_kv - c * kValChunk);
    if (tid < kValOut) {
      // out[o] = sum_t V[t][o] * p[t], t ascending (src/ops_cpu.cpp:402-406)
      const float* v = vbuf(b) + tid;
      const float* pp = pbuf(b);
      if (rows == kValChunk) {
        // two register batches of 16 positions, ping-pong: the loads of the
        // next batch are in flight while the current batch's adds run
        float a0[16], w0[16], a1[16], w1[16];
#pragma unroll
        for (int u = 0; u < 16; u++) {
          a0[u] = v[u * kValOut];
          w0[u] = pp[u];
        }
        for (int t = 0; t < kValChunk; t += 32) {
#pragma unroll
          for (int u = 0; u < 16; u++) {
            a1[u] = v[(t + 16 + u) * kValOut];
            w1[u] = pp[t + 16 + u];
          }
#pragma unroll
          for (int u = 0; u < 16; u++) acc = __fadd_rn(acc, __fmul_rn(a0[u], w0[u]));
          if (t + 32 < kValChunk) {
#pragma unroll
            for (int u = 0; u < 16; u++) {
              a0[u] = v[(t + 32 + u) * kValOut];
              w0[u] = pp[t + 32 + u];
            }
          }
#pragma unroll
          for (int u = 0; u < 16; u++) acc = __fadd_rn(acc, __fmul_rn(a1[u], w1[u]));
        }
      } else {
        int t = 0;
        for (; t + 16 <= rows; t += 16) {
          float a[16], w[16];
#pragma unroll
          for (int u = 0; u < 16; u++) {
            a[u] = v[(t + u) * kValOut];
            w[u] = pp[t + u];
          }
#pragma unroll
          for (int u = 0; u < 16; u++) acc = __fadd_rn(acc, __fmul_rn(a[u], w[u]));
        }
        for (; t < rows; t++) acc = __fadd_rn(acc, __fmul_rn(v[t * kValOut], pp[t]));
      }
    }
    __syncthreads();  // buffer b is refilled by the next iteration's issue
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  if (tid < kValOut && o0 + tid < D) out[(size_t)h * D + o0 + tid] = acc;
}

constexpr size_t kValSmem = (size_t)2 * kValChunk * (kValOut + 1) * 4;

size_t softmax_smem(int n_kv) {
  return ((size_t)(n_kv + 3) / 4 * 4) * 4 + kChainSlackBytes + (size_t)spec_sum_scratch_bytes(kSoftNT / 32, 4) + 16;
}

}  // namespace

// The kernels' shared-memory attributes, once per device (at its init): the
// largest sizes attn_long_fits admits.
cudaError_t prepare_attn_long_kernels(int optin) {
  cudaError_t e = cudaFuncSetAttribute(attn_long_values_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kValSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attn_long_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(((size_t)16 * 256 + (size_t)kScoreTile * 257) * 4));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attn_long_softmax_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - 1024);
  return e;
}

bool attn_long_fits(int64_t head_dim, int64_t n_head, int64_t n_head_kv, int64_t n_kv, int optin) {
  return head_dim % kValOut == 0 && head_dim <= 256 && n_head_kv > 0 && n_head % n_head_kv == 0 &&
         n_head / n_head_kv <= 16 && n_kv > 0 && (int64_t)softmax_smem((int)n_kv) <= (int64_t)optin - 1024;
}

cudaError_t launch_attn_decode_long(const AttnParams& p, cudaStream_t s) {
  const int D = p.head_dim, H = p.n_head, HKV = p.n_head_kv, n_kv = p.n_kv_fixed;
  const int n_rep = H / HKV;
  const size_t sc_smem = ((size_t)n_rep * D + (size_t)kScoreTile * (D + 1)) * 4;
  const size_t sm_smem = softmax_smem(n_kv);
  cudaError_t e = cudaSuccess;
  attn_long_scores_kernel<<<dim3((unsigned)((n_kv + kScoreTile - 1) / kScoreTile), (unsigned)HKV), kLongNT, sc_smem,
                            s>>>(p.q_rot, p.cache_k, D, H, HKV, n_kv, p.scale, p.scores, p.scores_stride);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  attn_long_softmax_kernel<<<(unsigned)H, kSoftNT, sm_smem, s>>>(p.scores, p.scores_stride, n_kv, p.et);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  attn_long_values_kernel<<<dim3((unsigned)H, (unsigned)(D / kValOut)), kLongNT, kValSmem, s>>>(
      p.scores, p.scores_stride, p.cache_v, D, H, HKV, n_kv, p.out);
  return cudaGetLastError();
}

}  // namespace mi
