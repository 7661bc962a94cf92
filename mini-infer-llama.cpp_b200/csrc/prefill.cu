// Batched prefill: a whole prompt (T tokens) through a layer at once, with the
// reference's arithmetic per (row, token) unchanged.
//
// The reference's batched forward computes every mul_mat element with the same
// vec_dot as decode (ref src/ops_cpu.cpp:177-268: rows split over threads, the
// per-row dot per column), its rms_norm / quantize per token row, and causal
// attention whose masked terms are exact zeros (src/ops_cpu.cpp:304-410); its
// own test asserts that batched and token-by-token forwards agree bit for bit
// (tests/test_model_qwen2.cpp:186-288). So the prefill kernels compute, for each
// token, exactly what the decode kernels compute -- only many tokens per launch:
//   * gemm_q8_kernel: a 64-row x 32-token tile per CTA; each thread owns 2 rows
//     x 4 tokens x the 8 AVX2 lane accumulators, blocks in order, so each
//     (row, token) keeps the decode GEMV's lane chains and hsum order;
//   * prefill_norm_quant_kernel: per token, [embedding lookup,] rms_norm * w and
//     the Q8_0_ACT quantizer, written in a split layout (quants, then scales);
//   * prefill_rope_kv_kernel: per token, RoPE of q and k and the KV-cache rows;
//   * attention: the decode attention kernel, one CTA per (head, query), with
//     n_kv = n_past + t + 1 for query t.
#include <algorithm>

#include "mi_device.cuh"

namespace mi {

namespace {

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

}  // namespace

// ---------------------------------------------------------------------------
// Exact Q8_0 GEMM: out[t][r] = dot(W row r, act row t) for a 64 x 32 tile.
// ---------------------------------------------------------------------------
constexpr int kGemmBN = 64;  // weight rows per CTA (16 groups of 4)
constexpr int kGemmBM = 32;  // tokens per CTA
constexpr int kGemmKB = 12;  // 32-element blocks per stage
constexpr int kGemmStages = 2;  // ~88 KB of shared memory: two CTAs per SM
constexpr int kGemmWStride = kGemmKB * 128 + 16;  // bytes per group in a stage (padded)
// A lane partial p = dp4a(w, a) satisfies |p| <= 4 * 127 * 127 < 2^22. With
// the accumulator input bits(1.5 * 2^23) the dp4a result is the bit pattern of
// the float 1.5 * 2^23 + p (exactly: the sum stays in [2^23, 2^24), where
// floats are the integers), and subtracting 1.5 * 2^23 gives (float)p exactly.
// This keeps the conversion off the int-to-float unit, whose rate (a quarter
// of the FMA rate) bounds the GEMM otherwise.
constexpr int kBiasI = 0x4B400000;
constexpr float kBiasF = 12582912.0f;

struct GemmSmem {
  static constexpr int wq = 0;
  static constexpr int wd = wq + 16 * kGemmWStride;
  static constexpr int aq = wd + 16 * kGemmKB * 8;
  static constexpr int ad = aq + kGemmBM * kGemmKB * 32;
  static constexpr int stage = ad + kGemmBM * kGemmKB * 4;
  static constexpr int res = kGemmStages * stage;  // [64 rows][32 tokens] floats (gate/up epilogue)
  static constexpr int total = res + kGemmBN * kGemmBM * 4;
};

__global__ void __launch_bounds__(256, 2) gemm_q8_kernel(const GemmParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t K = p.K;
  const int nb = (int)(K >> 5);
  const int64_t R0 = (int64_t)blockIdx.x * kGemmBN, T0 = (int64_t)blockIdx.y * kGemmBM;
  const int64_t G0 = R0 >> 2;
  const int64_t n_groups = p.n_pad >> 2;
  const uint8_t* wq = p.w;
  const uint8_t* wd = p.w + p.n_pad * K;
  const int n_k = (nb + kGemmKB - 1) / kGemmKB;

  auto load_stage = [&](int kt) {
    uint8_t* st = smem + (kt % kGemmStages) * GemmSmem::stage;
    const int c0 = kt * kGemmKB, kbb = min(kGemmKB, nb - c0);
    // weight quants: 16 groups x kbb blocks x 128 B, 16-byte pieces
    for (int c = tid; c < 16 * kbb * 8; c += 256) {
      const int g = c / (kbb * 8), off = c - g * (kbb * 8);
      if (G0 + g < n_groups)
        cp_async16(st + GemmSmem::wq + g * kGemmWStride + off * 16,
                   wq + (G0 + g) * 4 * K + (int64_t)c0 * 128 + off * 16);
    }
    // weight scales: 4 fp16 per group and block (8 B)
    for (int c = tid; c < 16 * kbb; c += 256) {
      const int g = c / kbb, i = c - g * kbb;
      if (G0 + g < n_groups)
        cp_async8(st + GemmSmem::wd + (g * kGemmKB + i) * 8, wd + ((G0 + g) * nb + c0 + i) * 8);
    }
    // activation quants: 32 tokens x kbb x 32 B
    for (int c = tid; c < kGemmBM * kbb * 2; c += 256) {
      const int t = c / (kbb * 2), off = c - t * (kbb * 2);
      if (T0 + t < p.M)
        cp_async16(st + GemmSmem::aq + t * kGemmKB * 32 + off * 16,
                   p.act_qs + (T0 + t) * p.act_stride + (int64_t)c0 * 32 + off * 16);
    }
    // activation scales
    for (int c = tid; c < kGemmBM * kbb; c += 256) {
      const int t = c / kbb, i = c - t * kbb;
      if (T0 + t < p.M)
        cp_async4(st + GemmSmem::ad + (t * kGemmKB + i) * 4, p.act_d + (T0 + t) * (p.act_stride >> 5) + c0 + i);
    }
  };

  // thread tile: rows 2l, 2l+1 (group l/2, rows 2(l&1), 2(l&1)+1 of it) x
  // tokens 4w..4w+3, 8 lane accumulators each
  float acc[2][4][8];
#pragma unroll
  for (int r = 0; r < 2; r++)
#pragma unroll
    for (int t = 0; t < 4; t++)
#pragma unroll
      for (int j = 0; j < 8; j++) acc[r][t][j] = 0.0f;
  const int g = lane >> 1, pr = (lane & 1) * 2;

#pragma unroll
  for (int s = 0; s < kGemmStages - 1; s++) {
    if (s < n_k) load_stage(s);
    cp_async_commit();
  }
  for (int kt = 0; kt < n_k; kt++) {
    cp_async_wait<kGemmStages - 2>();
    __syncthreads();
    if (kt + kGemmStages - 1 < n_k) load_stage(kt + kGemmStages - 1);
    cp_async_commit();
    const uint8_t* st = smem + (kt % kGemmStages) * GemmSmem::stage;
    const int kbb = min(kGemmKB, nb - kt * kGemmKB);
    const uint8_t* wrow = st + GemmSmem::wq + g * kGemmWStride + pr * 32;
    const __half* wsc = (const __half*)(st + GemmSmem::wd) + g * kGemmKB * 4 + pr;
    const uint8_t* abase = st + GemmSmem::aq + (warp * 4) * kGemmKB * 32;
    const float* adb = (const float*)(st + GemmSmem::ad) + (warp * 4) * kGemmKB;
    for (int i = 0; i < kbb; i++) {
      int w[2][8];
      {
        const uint4 a0 = *(const uint4*)(wrow + i * 128);
        const uint4 a1 = *(const uint4*)(wrow + i * 128 + 16);
        const uint4 b0 = *(const uint4*)(wrow + i * 128 + 32);
        const uint4 b1 = *(const uint4*)(wrow + i * 128 + 48);
        w[0][0] = (int)a0.x; w[0][1] = (int)a0.y; w[0][2] = (int)a0.z; w[0][3] = (int)a0.w;
        w[0][4] = (int)a1.x; w[0][5] = (int)a1.y; w[0][6] = (int)a1.z; w[0][7] = (int)a1.w;
        w[1][0] = (int)b0.x; w[1][1] = (int)b0.y; w[1][2] = (int)b0.z; w[1][3] = (int)b0.w;
        w[1][4] = (int)b1.x; w[1][5] = (int)b1.y; w[1][6] = (int)b1.z; w[1][7] = (int)b1.w;
      }
      const float sw0 = __half2float(wsc[i * 4]), sw1 = __half2float(wsc[i * 4 + 1]);
#pragma unroll
      for (int t = 0; t < 4; t++) {
        const uint4 q0 = *(const uint4*)(abase + t * kGemmKB * 32 + i * 32);
        const uint4 q1 = *(const uint4*)(abase + t * kGemmKB * 32 + i * 32 + 16);
        const int a[8] = {(int)q0.x, (int)q0.y, (int)q0.z, (int)q0.w,
                          (int)q1.x, (int)q1.y, (int)q1.z, (int)q1.w};
        const float da = adb[t * kGemmKB + i];
        const float d0 = __fmul_rn(sw0, da), d1 = __fmul_rn(sw1, da);
#pragma unroll
        for (int j = 0; j < 8; j++) {
          acc[0][t][j] = __fmaf_rn(__fsub_rn(__int_as_float(__dp4a(w[0][j], a[j], kBiasI)), kBiasF), d0,
                                   acc[0][t][j]);
          acc[1][t][j] = __fmaf_rn(__fsub_rn(__int_as_float(__dp4a(w[1][j], a[j], kBiasI)), kBiasF), d1,
                                   acc[1][t][j]);
        }
      }
    }
  }
  cp_async_wait<0>();

  // hsum_ps order per (row, token): ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7))
  float dot[2][4];
#pragma unroll
  for (int r = 0; r < 2; r++)
#pragma unroll
    for (int t = 0; t < 4; t++) {
      const float* a = acc[r][t];
      dot[r][t] = __fadd_rn(__fadd_rn(__fadd_rn(a[0], a[4]), __fadd_rn(a[1], a[5])),
                            __fadd_rn(__fadd_rn(a[2], a[6]), __fadd_rn(a[3], a[7])));
    }

  if (p.epi == EPI_SILU_GATEUP_Q) {
    // The tile's 64 packed rows are the gate/up rows of one 32-element block
    // of the FFN activation: silu(gate) * up per element, then the down
    // projection's quantize node, per token.
    float* res = (float*)(smem + GemmSmem::res);
    __syncthreads();
#pragma unroll
    for (int r = 0; r < 2; r++)
#pragma unroll
      for (int t = 0; t < 4; t++) res[(2 * lane + r) * kGemmBM + warp * 4 + t] = dot[r][t];
    __syncthreads();
    const int64_t blk = R0 >> 6;
    const int e = lane;  // activation element within the block
    const int lr = (e >> 2) * 8 + (e & 3);
    for (int t = warp; t < kGemmBM; t += 8) {
      const int64_t tok = T0 + t;
      if (tok >= p.M) break;
      const float v = __fmul_rn(silu_exact(res[lr * kGemmBM + t], p.et), res[(lr + 4) * kGemmBM + t]);
      float d;
      const int8_t q = quantize_lane(v, &d);
      p.q_out[tok * p.q_stride + blk * 32 + e] = q;
      if (e == 0) p.d_out[tok * (p.q_stride >> 5) + blk] = d;
    }
    return;
  }
#pragma unroll
  for (int t = 0; t < 4; t++) {
    const int64_t tok = T0 + warp * 4 + t;
    if (tok >= p.M) continue;
#pragma unroll
    for (int r = 0; r < 2; r++) {
      const int64_t row = R0 + 2 * lane + r;
      if (row >= p.N) continue;
      float v = dot[r][t];
      if (p.epi == EPI_BIAS) v = __fadd_rn(v, p.bias[row]);
      else if (p.epi == EPI_RESID) v = __fadd_rn(p.resid[tok * p.out_stride + row], v);
      p.out[tok * p.out_stride + row] = v;
    }
  }
}

cudaError_t prepare_gemm_kernel() {
  return cudaFuncSetAttribute(gemm_q8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              GemmSmem::total);
}

cudaError_t launch_gemm(const GemmParams& p, cudaStream_t s) {
  if (p.M <= 0) return cudaSuccess;
  if (p.wt) return launch_gemm_tc(p, s);
  if (p.K % 32 != 0 || (p.epi == EPI_SILU_GATEUP_Q && p.n_pad % kGemmBN != 0)) return cudaErrorInvalidValue;
  dim3 grid((unsigned)((p.n_pad + kGemmBN - 1) / kGemmBN), (unsigned)((p.M + kGemmBM - 1) / kGemmBM));
  gemm_q8_kernel<<<grid, 256, GemmSmem::total, s>>>(p);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Per-token [embedding,] rms_norm * w and Q8_0_ACT quantize (split layout).
// One CTA per token: the same steps as the GEMV prologue of the decode path.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) prefill_norm_quant_kernel(const NormQuantParams p) {
  extern __shared__ __align__(16) float xs[];  // [K] values, then [K + slack] squares
  __shared__ __align__(16) uint8_t spec[spec_sum_scratch_bytes(8, 4)];
  __shared__ float scale_sh;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t t = blockIdx.x, K = p.K;
  const int nb = (int)(K >> 5);
  float* sq = xs + K;
  if (p.embed) {
    int tok = p.tokens[t];
    if (tok < 0 || tok >= p.embed_rows) {
      if (tid == 0) atomicExch(p.err, 1 /* MI_CUDA_ERR_ARG */);
      tok = 0;
    }
    for (int64_t k = tid; k < K; k += 256) {
      const int64_t b = k >> 5;
      const float v = __fmul_rn((float)packed_qs(p.embed, K, tok, b)[k & 31],
                                packed_scale(p.embed, K, p.embed_npad, tok, b));
      xs[k] = v;
      p.x_out[t * K + k] = v;
    }
  } else {
    for (int64_t k = tid; k < K; k += 256) xs[k] = p.x[t * K + k];
  }
  __syncthreads();
  float scale = 1.0f;
  if (p.norm_w) {
    for (int64_t k = tid; k < K; k += 256) sq[k] = __fmul_rn(xs[k], xs[k]);
    __syncthreads();
    const float ss = K <= 1024 ? spec_ordered_sum<256, 2>(sq, (int)K, spec)
                               : spec_ordered_sum<256, 4>(sq, (int)K, spec);
    if (tid == 0) scale_sh = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), p.eps)));
    __syncthreads();
    scale = scale_sh;
  }
  for (int b = warp; b < nb; b += 8) {
    const int64_t k = (int64_t)b * 32 + lane;
    const float v = p.norm_w ? __fmul_rn(__fmul_rn(xs[k], scale), p.norm_w[k]) : xs[k];
    float d;
    p.q_out[t * K + k] = quantize_lane(v, &d);
    if (lane == 0) p.d_out[t * nb + b] = d;
  }
}

cudaError_t launch_norm_quant(const NormQuantParams& p, int64_t n_tokens, cudaStream_t s) {
  if (n_tokens <= 0) return cudaSuccess;
  const size_t smem = (size_t)(2 * p.K) * 4 + kChainSlackBytes;
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(prefill_norm_quant_kernel,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  prefill_norm_quant_kernel<<<(unsigned)n_tokens, 256, smem, s>>>(p);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Per-token NEOX RoPE of q and k (src/ops_cpu.cpp:270-302) and the KV-cache
// append (MI_OP_CPY, src/ops_cpu.cpp:446-460) at positions n_past + t.
// qkv rows are [q (n_head*hd) | k (n_head_kv*hd) | v (n_head_kv*hd)].
// ---------------------------------------------------------------------------
__global__ void prefill_rope_kv_kernel(const float* qkv, int64_t row, int32_t head_dim, int32_t n_head,
                                       int32_t n_head_kv, int32_t n_past, const float2* rope_cs,
                                       float* q_rot, float* cache_k, float* cache_v) {
  const int64_t t = blockIdx.x;
  const int half = head_dim >> 1;
  const float* src = qkv + t * row;
  const float2* cs = rope_cs + (int64_t)(n_past + t) * half;
  const int nq = n_head * half, nk = n_head_kv * half;
  for (int e = threadIdx.x; e < nq + nk; e += blockDim.x) {
    const bool isq = e < nq;
    const int ee = isq ? e : e - nq;
    const int h = ee / half, i = ee - h * half;
    const float* x = src + (isq ? 0 : (int64_t)n_head * head_dim) + (int64_t)h * head_dim;
    const float2 c = cs[i];
    const float x0 = x[i], x1 = x[i + half];
    const float y0 = __fsub_rn(__fmul_rn(x0, c.x), __fmul_rn(x1, c.y));
    const float y1 = __fadd_rn(__fmul_rn(x0, c.y), __fmul_rn(x1, c.x));
    float* d = isq ? q_rot + (t * n_head + h) * head_dim
                   : cache_k + ((int64_t)(n_past + t) * n_head_kv + h) * head_dim;
    d[i] = y0;
    d[i + half] = y1;
  }
  const int kvd = n_head_kv * head_dim;
  const float* v = src + (int64_t)(n_head + n_head_kv) * head_dim;
  for (int e = threadIdx.x; e < kvd; e += blockDim.x) cache_v[(int64_t)(n_past + t) * kvd + e] = v[e];
}

cudaError_t launch_rope_kv(const float* qkv, int64_t row, int32_t head_dim, int32_t n_head,
                           int32_t n_head_kv, int32_t n_past, int64_t n_tokens, const float2* rope_cs,
                           float* q_rot, float* cache_k, float* cache_v, cudaStream_t s) {
  if (n_tokens <= 0) return cudaSuccess;
  prefill_rope_kv_kernel<<<(unsigned)n_tokens, 256, 0, s>>>(qkv, row, head_dim, n_head, n_head_kv, n_past,
                                                            rope_cs, q_rot, cache_k, cache_v);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Prefill attention: one CTA per (KV head, query t) runs the reference's
// attention for the n_rep query heads that share the KV head (GQA mapping
// h = kvh * n_rep + r, src/ops_cpu.cpp:356-410), at n_kv = n_past + t + 1:
//   scores  s[r][k] = (sum over d, in order, of K[k][d] * q[r][d]) * scale,
//   softmax max, e = expf(s - max), the denominator as one ordered chain,
//           p = e * (1 / sum),
//   out[r][o] = sum over k, in order, of V[k][o] * p[r][k].
// Register-blocked: in the score phase a thread owns one key of the tile and
// the chains of up to 8 heads (q in shared memory as [d][8], read as two
// broadcast float4 per d; the K row as float4); in the value phase a thread
// owns 2 outputs of one head, reading four probabilities as a float4 and the
// four V row pieces as float2 per step. Every chain keeps the reference's order (multiply, then
// add, each rounded).
// ---------------------------------------------------------------------------
struct PfAttnShape {
  int kt, rg;  // keys per tile, threads per key (each owning 8 / rg heads)
  size_t smem(int D, int R, int64_t cap) const {
    return ((size_t)8 * D + (size_t)kt * (D + 4) + (size_t)R * cap) * 4 + kChainSlackBytes;
  }
};
// 128-key tiles (two threads per key up to head_dim 128) keep the shared
// memory of a CTA near 66 KB at 1024 positions (0.5B shape), so three CTAs
// share an SM; 256-key tiles (two CTAs per SM) measured 10% slower for the
// whole prefill, 64-key tiles 5% slower.
__host__ __device__ inline PfAttnShape pf_attn_shape(int D) {
  return D <= 128 ? PfAttnShape{128, 2} : PfAttnShape{64, 4};
}

// A product then a sum, two lanes at a time, each rounded on its own. (Two
// scalar operations per lane: ptxas may fuse an f32x2 multiply and the f32x2
// add that consumes it into one FMA, which rounds once.)
__device__ __forceinline__ float2 mul2s(float2 a, float2 b) {
  return make_float2(__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y));
}
__device__ __forceinline__ float2 add2s(float2 a, float2 b) {
  return make_float2(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y));
}

// RG threads per key in the score phase (each owning 8 / RG heads), a
// compile-time constant so the head-pair loops carry no predicated-off work.
template <int RG>
__global__ void __launch_bounds__(256) attn_prefill_kernel(const PrefillAttnParams p) {
  extern __shared__ __align__(16) float sm[];
  __shared__ float mx[8], inv[8];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kvh = blockIdx.x, t = blockIdx.y;
  const int D = p.head_dim, R = p.n_rep, HKV = p.n_head_kv, KP = D + 4;
  constexpr int KT = 256 / RG;
  const int n_kv = p.n_past + t + 1;
  const int cap = p.sc_stride;  // score row stride (>= n_kv, a multiple of 4)
  float* qs = sm;            // [D][8]: q[r][d] at d*8 + r (r >= R: zero)
  float* Ts = qs + 8 * D;    // K tile [KT][D + 4], then V tile [KT][D], then the outputs [R][D]
  float* sc = Ts + KT * KP;  // [R][cap]
  const size_t rs = (size_t)HKV * D;
  const float* kb = p.cache_k + (size_t)kvh * D;
  const float* vb = p.cache_v + (size_t)kvh * D;
  const int h0 = kvh * R;
  for (int e = tid; e < 8 * D; e += 256) {
    const int d = e >> 3, r = e & 7;
    qs[e] = r < R ? p.q_rot[((size_t)t * p.n_head + h0 + r) * D + d] : 0.0f;
  }
  const int n_chunks = (n_kv + KT - 1) / KT;
  const int sh4 = __ffs(D >> 2) - 1;  // log2(D / 4): head_dim is a power of two here
  // ---- scores ----
  constexpr int npair = 4 / RG;
  const int kk = tid % KT, rgi = tid / KT;  // head pairs rgi*npair ..
  for (int c = 0; c < n_chunks; c++) {
    const int c0 = c * KT, rows = min(KT, n_kv - c0);
    __syncthreads();
    for (int e = tid; e < rows * (D >> 2); e += 256) {
      const int r = e >> sh4, q4 = e & ((D >> 2) - 1);
      *(float4*)(Ts + r * KP + q4 * 4) = *(const float4*)(kb + (size_t)(c0 + r) * rs + q4 * 4);
    }
    __syncthreads();
    if (kk < rows) {
      const float* kr = Ts + kk * KP;
      float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      for (int d4 = 0; d4 < (D >> 2); d4++) {
        const float4 kv = *(const float4*)(kr + 4 * d4);
        const float kd[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const float2 k2 = make_float2(kd[i], kd[i]);
          const float2* q2 = (const float2*)(qs + (4 * d4 + i) * 8) + rgi * npair;
#pragma unroll
          for (int j = 0; j < 4; j++)
            if (j < npair) acc[j] = add2s(acc[j], mul2s(k2, q2[j]));
        }
      }
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int r = 2 * (rgi * npair + j);
        if (j < npair && r < R) sc[r * cap + c0 + kk] = __fmul_rn(acc[j].x, p.scale);
        if (j < npair && r + 1 < R) sc[(r + 1) * cap + c0 + kk] = __fmul_rn(acc[j].y, p.scale);
      }
    }
  }
  __syncthreads();
  // ---- softmax: the maximum per head (order-free), expf, the ordered denominator ----
  if (warp < R) {
    float m = -INFINITY;
    for (int k = lane; k < n_kv; k += 32) m = fmaxf(m, sc[warp * cap + k]);
    m = warp_max(m);
    if (lane == 0) mx[warp] = m;
  }
  __syncthreads();
  {
    // element e = r * n_kv + k, stepping by the CTA size without a division
    int r = tid / n_kv, k = tid - r * n_kv;
    for (; r < R;) {
      float* a = sc + r * cap + k;
      *a = expf_exact(__fsub_rn(*a, mx[r]), p.et);
      k += 256;
      while (k >= n_kv) {
        k -= n_kv;
        r++;
      }
    }
  }
  __syncthreads();
  if (warp < R && lane == 0) inv[warp] = __fdiv_rn(1.0f, ordered_sum_smem(sc + warp * cap, n_kv));
  __syncthreads();
  // p = e * (1 / sum), four at a time (entries past n_kv are never read)
  for (int r = 0; r < R; r++)
    for (int k4 = tid; 4 * k4 < n_kv; k4 += 256) {
      float4* a = (float4*)(sc + r * cap) + k4;
      const float iv = inv[r];
      float4 v = *a;
      v.x = __fmul_rn(v.x, iv);
      v.y = __fmul_rn(v.y, iv);
      v.z = __fmul_rn(v.z, iv);
      v.w = __fmul_rn(v.w, iv);
      *a = v;
    }
  // ---- values: unit u = (head r, outputs 2*o2, 2*o2 + 1) ----
  const int D2 = D >> 1, n_units = R * D2;
  constexpr int kMaxUnits = 4;  // R * D / 2 <= 1024
  float2 acc[kMaxUnits];
#pragma unroll
  for (int j = 0; j < kMaxUnits; j++) acc[j] = make_float2(0.f, 0.f);
  for (int c = 0; c < n_chunks; c++) {
    const int c0 = c * KT, rows = min(KT, n_kv - c0);
    __syncthreads();
    for (int e = tid; e < rows * (D >> 2); e += 256) {
      const int r = e >> sh4, q4 = e & ((D >> 2) - 1);
      *(float4*)(Ts + r * D + q4 * 4) = *(const float4*)(vb + (size_t)(c0 + r) * rs + q4 * 4);
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kMaxUnits; j++) {
      const int u = tid + 256 * j;
      if (u >= n_units) break;
      const int r = u / D2, o2 = u - r * D2;
      const float* pr = sc + r * cap + c0;
      const float* vr = Ts + 2 * o2;
      float2 a = acc[j];
      int k = 0;
      for (; k + 4 <= rows; k += 4) {
        const float4 p4 = *(const float4*)(pr + k);
        const float pk[4] = {p4.x, p4.y, p4.z, p4.w};
        float2 v[4];
#pragma unroll
        for (int i = 0; i < 4; i++) v[i] = *(const float2*)(vr + (k + i) * D);
#pragma unroll
        for (int i = 0; i < 4; i++) a = add2s(a, mul2s(v[i], make_float2(pk[i], pk[i])));
      }
      for (; k < rows; k++) a = add2s(a, mul2s(*(const float2*)(vr + k * D), make_float2(pr[k], pr[k])));
      acc[j] = a;
    }
  }
  __syncthreads();
  float* outs = Ts;  // [R][D], the concatenated heads' outputs
#pragma unroll
  for (int j = 0; j < kMaxUnits; j++) {
    const int u = tid + 256 * j;
    if (u >= n_units) break;
    *(float2*)(outs + 2 * u) = acc[j];
  }
  __syncthreads();
  for (int e = tid; e < R * D; e += 256) {
    const size_t col = (size_t)h0 * D + e;  // element of the concatenated heads
    if (p.act_qs) {
      // the O projection's quantize node, one 32-element block per warp
      // (R * D is a multiple of 32, so the loop bound is warp-uniform)
      float d;
      const int8_t q = quantize_lane(outs[e], &d);
      p.act_qs[(size_t)t * p.row + col] = q;
      if (lane == 0) p.act_d[((size_t)t * p.row + col) >> 5] = d;
    } else {
      p.out[(size_t)t * p.row + col] = outs[e];
    }
  }
}

bool prefill_attn_fits(int32_t head_dim, int32_t n_rep, int64_t max_kv) {
  const int64_t cap = (max_kv + 3) / 4 * 4;
  return n_rep <= 8 && head_dim >= 4 && head_dim <= 256 && (head_dim & (head_dim - 1)) == 0 &&
         n_rep * head_dim <= 2048 &&
         pf_attn_shape(head_dim).smem(head_dim, n_rep, cap) <= 200 * 1024;
}

cudaError_t launch_attn_prefill(const PrefillAttnParams& p, int64_t n_tokens, cudaStream_t s) {
  if (n_tokens <= 0) return cudaSuccess;
  PrefillAttnParams q = p;
  const int64_t max_kv = p.n_past + n_tokens;
  if (!prefill_attn_fits(p.head_dim, p.n_rep, max_kv)) return cudaErrorInvalidValue;
  if (p.act_qs && (p.n_rep * p.head_dim) % 32 != 0) return cudaErrorInvalidValue;
  q.sc_stride = (int32_t)((max_kv + 3) / 4 * 4);
  const size_t smem = pf_attn_shape(p.head_dim).smem(p.head_dim, p.n_rep, q.sc_stride);
  const int rg = pf_attn_shape(p.head_dim).rg;
  auto kern = rg == 2 ? attn_prefill_kernel<2> : (rg == 4 ? attn_prefill_kernel<4> : attn_prefill_kernel<1>);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<dim3((unsigned)p.n_head_kv, (unsigned)n_tokens), 256, smem, s>>>(q);
  return cudaGetLastError();
}

}  // namespace mi
