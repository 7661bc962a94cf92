// Decode attention, split over positions (a labelled fast mode, not
// bit-exact). No counterpart in the reference.
//
// The reference's ATTN_QK / SOFTMAX / ATTN_KQV (ref src/ops_cpu.cpp:304-410)
// sum the softmax denominator and every output's value sum as one chain over
// all n_kv positions; the exact kernel keeps those chains, which makes long
// contexts latency-bound (a 32768-long dependent chain per output). This mode
// splits the positions over many CTAs and combines their partial results
// (per-split maximum, denominator and unnormalized value sums, rescaled to the
// global maximum), the way split-K decode attention kernels do. Each term is
// the same (libm-exact expf of the same scores), but the sums are regrouped
// and the products fused,
// so results differ from the reference's in the last bits. The exact kernel
// stays the one the decode path uses.
//
// Grid (splits, n_head_kv): a CTA takes the n_rep query heads of one KV head
// over one range of up to 128 positions, requests all of its K / V rows at
// once, and writes (maximum, denominator, unnormalized value sums) per head;
// a second kernel combines the splits.
#include <algorithm>

#include "mi_device.cuh"

namespace mi {

namespace {

constexpr int kSplitNT = 256;
constexpr int kSplitMaxPos = 128;  // positions per CTA
constexpr int kSplitMaxRep = 16;   // query heads per KV head
constexpr int kSplitMaxD = 128;
constexpr int kMaxSplits = 1024;

// Shared memory of one CTA for head_dim D: q [D][16], K rows [P][D + 4]
// (padded: a warp's lanes read 32 different rows at the same d), V rows
// [P][D], probabilities [16][P].
__host__ __device__ inline size_t split_smem_bytes(int D) {
  return ((size_t)D * 16 + (size_t)kSplitMaxPos * (D + 4) + (size_t)kSplitMaxPos * D + 16 * kSplitMaxPos) * 4;
}

// One CTA: the n_rep query heads of KV head blockIdx.y over positions
// [s * per_split, +per_split), all of its K and V rows requested at once
// (16-byte asynchronous copies), so every CTA's loads are in flight
// together; then the scores (a thread per (position, group of 4 heads)), the
// softmax of this range (a warp per head), and the value sums (a thread per
// (head, 4 outputs)).
__global__ void __launch_bounds__(kSplitNT) attn_split_kernel(const float* q, const float* ck, const float* cv,
                                                              int D, int H, int HKV, int n_kv, float scale,
                                                              int per_split, ExpTab et, float* part) {
  extern __shared__ __align__(16) float sm[];
  __shared__ float m_s[kSplitMaxRep], l_s[kSplitMaxRep];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kvh = blockIdx.y, s = blockIdx.x, S = gridDim.x;
  const int n_rep = H / HKV, h0 = kvh * n_rep, KP = D + 4, D4 = D >> 2;
  const int t0 = s * per_split, cnt = min(n_kv, t0 + per_split) - t0;
  float* q_s = sm;                                   // [D][16]
  float* K_s = q_s + D * 16;                         // [P][D + 4]
  float* V_s = K_s + kSplitMaxPos * KP;              // [P][D]
  float* p_s = V_s + kSplitMaxPos * D;               // [16][P]
  const size_t rs = (size_t)HKV * D;
  // every K / V row piece of the range as one 16-byte asynchronous copy, all
  // in flight at once (K into padded rows)
  const int sh4 = __ffs(D4) - 1;  // log2(D / 4): head_dim is a power of two here
  for (int e = tid; e < cnt * D4; e += kSplitNT) {
    const int t = e >> sh4, c = e & (D4 - 1);
    const size_t off = (size_t)(t0 + t) * rs + (size_t)kvh * D + (size_t)c * 4;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(K_s + t * KP + 4 * c)), "l"(ck + off)
                 : "memory");
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(V_s + t * D + 4 * c)), "l"(cv + off)
                 : "memory");
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  for (int e = tid; e < D * 16; e += kSplitNT) {
    const int d = e >> 4, r = e & 15;
    q_s[e] = r < n_rep ? q[(size_t)(h0 + r) * D + d] : 0.0f;
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();  // (the rows and q_s)
  {
    // scores: item = (position t, heads 4g..4g+3)
    const int G = (n_rep + 3) >> 2;
    for (int it = tid; it < cnt * G; it += kSplitNT) {
      const int t = it % cnt, g = it / cnt;
      const float* kr = K_s + t * KP;
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      for (int d4 = 0; d4 < D4; d4++) {
        const float4 kv = *(const float4*)(kr + 4 * d4);
        const float kd[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const float4 qq = *(const float4*)(q_s + (4 * d4 + i) * 16 + 4 * g);
          a0 = __fmaf_rn(kd[i], qq.x, a0);
          a1 = __fmaf_rn(kd[i], qq.y, a1);
          a2 = __fmaf_rn(kd[i], qq.z, a2);
          a3 = __fmaf_rn(kd[i], qq.w, a3);
        }
      }
      const float av[4] = {a0, a1, a2, a3};
#pragma unroll
      for (int i = 0; i < 4; i++)
        if (4 * g + i < n_rep) p_s[(4 * g + i) * kSplitMaxPos + t] = __fmul_rn(av[i], scale);
    }
  }
  __syncthreads();
  {
    // softmax of this range, a warp per head (order-free sums: fast mode)
    for (int r = warp; r < n_rep; r += kSplitNT / 32) {
      float* pr = p_s + r * kSplitMaxPos;
      float m = -INFINITY;
      for (int t = lane; t < cnt; t += 32) m = fmaxf(m, pr[t]);
      m = warp_max(m);
      float l = 0.0f;
      for (int t = lane; t < cnt; t += 32) {
        const float e = expf_exact(__fsub_rn(pr[t], m), et);
        pr[t] = e;
        l = __fadd_rn(l, e);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) l = __fadd_rn(l, __shfl_xor_sync(0xffffffffu, l, o));
      if (lane == 0) {
        m_s[r] = m;
        l_s[r] = l;
      }
    }
  }
  __syncthreads();
  {
    // values: unit = (head r, outputs 4*o4 .. 4*o4 + 3, half of the positions);
    // both halves' sums go to shared memory and meet there (fast mode:
    // regrouped sums)
    float* half_s = K_s;  // [2][n_rep * D] (the K rows are no longer needed)
    const int n_units = n_rep * D4, hcut = (cnt + 1) >> 1;
    for (int u = tid; u < 2 * n_units; u += kSplitNT) {
      const int hf = u >= n_units, uu = u - hf * n_units;
      const int r = uu / D4, o4 = uu - r * D4;
      const float* pr = p_s + r * kSplitMaxPos;
      const float* vr = V_s + 4 * o4;
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int t = hf ? hcut : 0, te = hf ? cnt : hcut; t < te; t++) {
        const float pt = pr[t];
        const float4 v = *(const float4*)(vr + t * D);
        a.x = __fmaf_rn(pt, v.x, a.x);
        a.y = __fmaf_rn(pt, v.y, a.y);
        a.z = __fmaf_rn(pt, v.z, a.z);
        a.w = __fmaf_rn(pt, v.w, a.w);
      }
      *(float4*)(half_s + hf * n_units * 4 + 4 * uu) = a;
    }
    __syncthreads();
    for (int e = tid; e < n_rep * D; e += kSplitNT) {
      const int r = e / D, o = e - r * D;
      part[((size_t)(h0 + r) * S + s) * (D + 2) + 2 + o] = __fadd_rn(half_s[e], half_s[n_units * 4 + e]);
    }
    if (tid < n_rep) {
      float* ph = part + ((size_t)(h0 + tid) * S + s) * (D + 2);
      ph[0] = m_s[tid];
      ph[1] = l_s[tid];
    }
  }
}

// out[h][o] = sum_s acc_s[o] * e^(m_s - M) / sum_s l_s * e^(m_s - M), M the
// largest split maximum. Grid (heads, ceil(D / 32)): each CTA forms the split
// weights (one exponential per split, in parallel), then its 8 warps sum
// interleaved eighths of the splits for 32 outputs, combined in shared memory.
constexpr int kCombineNT = 256;
__global__ void __launch_bounds__(kCombineNT) attn_split_combine_kernel(const float* part, int D, int S, ExpTab et,
                                                                       float* out) {
  __shared__ float w_s[kMaxSplits];
  __shared__ float red[kCombineNT / 32];
  __shared__ float sums[kCombineNT / 32][32];
  const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const size_t st = (size_t)D + 2;
  const float* ph = part + (size_t)h * S * st;
  float m = -INFINITY;
  for (int s = tid; s < S; s += kCombineNT) m = fmaxf(m, ph[s * st]);
  m = warp_max(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  float M = red[0];
  for (int w = 1; w < kCombineNT / 32; w++) M = fmaxf(M, red[w]);
  __syncthreads();
  float l = 0.0f;
  for (int s = tid; s < S; s += kCombineNT) {
    const float w = expf_exact(__fsub_rn(ph[s * st], M), et);
    w_s[s] = w;
    l = __fmaf_rn(ph[s * st + 1], w, l);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) l = __fadd_rn(l, __shfl_xor_sync(0xffffffffu, l, o));
  if (lane == 0) red[warp] = l;
  __syncthreads();
  float L = red[0];
  for (int w = 1; w < kCombineNT / 32; w++) L = __fadd_rn(L, red[w]);
  const int o = blockIdx.y * 32 + lane;
  float a = 0.0f;
  if (o < D) {
#pragma unroll 4
    for (int s = warp; s < S; s += kCombineNT / 32) a = __fmaf_rn(ph[s * st + 2 + o], w_s[s], a);
  }
  sums[warp][lane] = a;
  __syncthreads();
  if (warp == 0 && o < D) {
    float t = sums[0][lane];
    for (int w = 1; w < kCombineNT / 32; w++) t = __fadd_rn(t, sums[w][lane]);
    out[(size_t)h * D + o] = __fdiv_rn(t, L);
  }
}

}  // namespace

bool attn_split_fits(int64_t head_dim, int64_t n_head, int64_t n_head_kv) {
  return head_dim >= 4 && head_dim <= kSplitMaxD && (head_dim & (head_dim - 1)) == 0 && n_head > 0 &&
         n_head < (1ll << 31) && n_head_kv > 0 && n_head % n_head_kv == 0 &&
         n_head / n_head_kv <= kSplitMaxRep;
}

// Splits of up to 128 positions (a multiple of 32), about two CTAs per SM of a
// 148-SM B200 when the context allows (at most kMaxSplits per head).
void attn_split_shape(int64_t n_kv, int64_t n_head_kv, int32_t* n_splits, int32_t* per_split) {
  const int64_t want = (std::max<int64_t>(1, n_kv) * std::max<int64_t>(1, n_head_kv) + 295) / 296;
  int64_t per = std::min<int64_t>(kSplitMaxPos, std::max<int64_t>(32, (want + 31) / 32 * 32));
  while ((n_kv + per - 1) / per > kMaxSplits && per < kSplitMaxPos) per += 32;
  *per_split = (int32_t)per;
  *n_splits = (int32_t)std::max<int64_t>(1, (n_kv + per - 1) / per);
}

size_t attn_split_scratch_bytes(int64_t n_head, int64_t n_kv, int64_t n_head_kv, int64_t head_dim) {
  int32_t S = 0, per = 0;
  attn_split_shape(n_kv, n_head_kv, &S, &per);
  return (size_t)n_head * S * (head_dim + 2) * 4;
}

cudaError_t launch_attn_split(const float* q, const float* ck, const float* cv, int64_t D, int64_t H, int64_t HKV,
                              int64_t n_kv, float scale, const ExpTab& et, int32_t* err, float* part, float* out,
                              cudaStream_t s) {
  int32_t S = 0, per = 0;
  attn_split_shape(n_kv, HKV, &S, &per);
  (void)err;  // (no bounded waits in this mode's kernels)
  if (S > kMaxSplits) return cudaErrorInvalidValue;
  const size_t smem = split_smem_bytes((int)D);
  static size_t smem_set = 0;  // (the attribute once per largest size; a host call per launch costs microseconds)
  cudaError_t e = cudaSuccess;
  if (smem > smem_set) {
    e = cudaFuncSetAttribute(attn_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)split_smem_bytes(kSplitMaxD));
    if (e != cudaSuccess) return e;
    smem_set = split_smem_bytes(kSplitMaxD);
  }
  attn_split_kernel<<<dim3((unsigned)S, (unsigned)HKV), kSplitNT, smem, s>>>(q, ck, cv, (int)D, (int)H, (int)HKV,
                                                                             (int)n_kv, scale, per, et, part);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  attn_split_combine_kernel<<<dim3((unsigned)H, (unsigned)((D + 31) / 32)), kCombineNT, 0, s>>>(part, (int)D, S, et,
                                                                                                out);
  return cudaGetLastError();
}

}  // namespace mi
