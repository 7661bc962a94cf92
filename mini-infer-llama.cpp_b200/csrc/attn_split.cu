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
// the same (scores d ascending, libm-exact expf), but the sums are regrouped,
// so results differ from the reference's in the last bits. The exact kernel
// stays the one the decode path uses.
//
// Grid (splits, n_head_kv): a CTA takes the n_rep query heads of one KV head
// over one range of positions, streaming K / V tiles of 32 positions through
// shared memory once for all n_rep heads, with an online softmax per head.
#include <algorithm>

#include "mi_device.cuh"

namespace mi {

namespace {

constexpr int kSplitNT = 256;
constexpr int kSplitTile = 32;     // positions per shared-memory tile (one per lane)
constexpr int kSplitMaxRep = 16;   // query heads per KV head
constexpr int kSplitMaxD = 128;
constexpr int kSplitAcc = kSplitMaxRep * kSplitMaxD / kSplitNT;  // (head, output) pairs per thread

__global__ void __launch_bounds__(kSplitNT) attn_split_kernel(const float* q, const float* ck, const float* cv,
                                                              int D, int H, int HKV, int n_kv, float scale,
                                                              int per_split, ExpTab et, float* part) {
  __shared__ float q_s[kSplitMaxRep * kSplitMaxD];
  __shared__ float Kt[kSplitTile * (kSplitMaxD + 1)];
  __shared__ __align__(16) float Vt[kSplitTile * kSplitMaxD];
  __shared__ float p_s[kSplitMaxRep * kSplitTile];
  __shared__ float m_s[kSplitMaxRep], l_s[kSplitMaxRep], c_s[kSplitMaxRep];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kvh = blockIdx.y, s = blockIdx.x, S = gridDim.x;
  const int n_rep = H / HKV, h0 = kvh * n_rep, KP = D + 1, D4 = D >> 2;
  const int t0 = s * per_split, t1 = min(n_kv, t0 + per_split);
  const size_t rs = (size_t)HKV * D;
  const int n_pairs = n_rep * D;
  for (int e = tid; e < n_pairs; e += kSplitNT) q_s[e] = q[(size_t)h0 * D + e];
  if (tid < n_rep) {
    m_s[tid] = -INFINITY;
    l_s[tid] = 0.0f;
  }
  float acc[kSplitAcc];
#pragma unroll
  for (int u = 0; u < kSplitAcc; u++) acc[u] = 0.0f;
  __syncthreads();
  for (int c0 = t0; c0 < t1; c0 += kSplitTile) {
    const int cnt = min(kSplitTile, t1 - c0);
    for (int e = tid; e < cnt * D4; e += kSplitNT) {
      const int r = e / D4, c = e - r * D4;
      const size_t off = (size_t)(c0 + r) * rs + (size_t)kvh * D + (size_t)c * 4;
      const float4 kv = *(const float4*)(ck + off);
      const float4 vv = *(const float4*)(cv + off);
      float* kd = Kt + r * KP + c * 4;
      kd[0] = kv.x;
      kd[1] = kv.y;
      kd[2] = kv.z;
      kd[3] = kv.w;
      *(float4*)(Vt + r * D + c * 4) = vv;
    }
    __syncthreads();
    for (int e = tid; e < n_rep * kSplitTile; e += kSplitNT) {
      const int r = e / kSplitTile, t = e - r * kSplitTile;
      p_s[e] = t < cnt ? __fmul_rn(ordered_dot(0.0f, Kt + t * KP, 1, q_s + r * D, D), scale) : -INFINITY;
    }
    __syncthreads();
    // Online softmax, one warp per head: new maximum, this tile's terms, the
    // factor that rescales what was accumulated under the old maximum.
    for (int r = warp; r < n_rep; r += kSplitNT / 32) {
      const float sc = p_s[r * kSplitTile + lane];
      const float m_old = m_s[r];
      const float m_new = fmaxf(m_old, warp_max(sc));
      const float p = expf_exact(__fsub_rn(sc, m_new), et);
      float sum = p;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
      p_s[r * kSplitTile + lane] = p;
      if (lane == 0) {
        const float corr = expf_exact(__fsub_rn(m_old, m_new), et);
        c_s[r] = corr;
        l_s[r] = __fmaf_rn(l_s[r], corr, sum);
        m_s[r] = m_new;
      }
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < kSplitAcc; u++) {
      const int e = tid + u * kSplitNT;
      if (e < n_pairs) {
        const int r = e / D, o = e - r * D;
        float a = __fmul_rn(acc[u], c_s[r]);
        for (int t = 0; t < cnt; t++) a = __fmaf_rn(p_s[r * kSplitTile + t], Vt[t * D + o], a);
        acc[u] = a;
      }
    }
    __syncthreads();
  }
  // partial of (head h0 + r, split s): maximum, denominator, unnormalized sums
#pragma unroll
  for (int u = 0; u < kSplitAcc; u++) {
    const int e = tid + u * kSplitNT;
    if (e < n_pairs) {
      const int r = e / D, o = e - r * D;
      part[((size_t)(h0 + r) * S + s) * (D + 2) + 2 + o] = acc[u];
    }
  }
  if (tid < n_rep) {
    float* ph = part + ((size_t)(h0 + tid) * S + s) * (D + 2);
    ph[0] = m_s[tid];
    ph[1] = l_s[tid];
  }
}

// out[h][o] = sum_s acc_s[o] * e^(m_s - M) / sum_s l_s * e^(m_s - M), M the
// largest split maximum. The split weights are formed in parallel (one
// exponential per split), then each output thread runs over the splits.
constexpr int kCombineNT = 128;
constexpr int kMaxSplits = 1024;
__global__ void __launch_bounds__(kCombineNT) attn_split_combine_kernel(const float* part, int D, int S, ExpTab et,
                                                                       float* out) {
  __shared__ float w_s[kMaxSplits];
  __shared__ float red[kCombineNT / 32];
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
  if (tid < D) {
    float a = 0.0f;
#pragma unroll 8
    for (int s = 0; s < S; s++) a = __fmaf_rn(ph[s * st + 2 + tid], w_s[s], a);
    out[(size_t)h * D + tid] = __fdiv_rn(a, L);
  }
}

}  // namespace

bool attn_split_fits(int64_t head_dim, int64_t n_head, int64_t n_head_kv) {
  return head_dim >= 4 && head_dim <= kSplitMaxD && head_dim % 4 == 0 && n_head > 0 &&
         n_head < (1ll << 31) && n_head_kv > 0 && n_head % n_head_kv == 0 &&
         n_head / n_head_kv <= kSplitMaxRep;
}

// Splits of whole tiles, about four CTAs per SM of a 148-SM B200 in total
// (at most kMaxSplits per head).
void attn_split_shape(int64_t n_kv, int64_t n_head_kv, int32_t* n_splits, int32_t* per_split) {
  const int64_t tiles = std::max<int64_t>(1, (n_kv + kSplitTile - 1) / kSplitTile);
  const int64_t target = std::max<int64_t>(1, 592 / std::max<int64_t>(1, n_head_kv));
  const int64_t tiles_per = (tiles + target - 1) / target;
  const int64_t per = tiles_per * kSplitTile;
  *per_split = (int32_t)per;
  *n_splits = (int32_t)std::max<int64_t>(1, (n_kv + per - 1) / per);
}

size_t attn_split_scratch_bytes(int64_t n_head, int64_t n_kv, int64_t n_head_kv, int64_t head_dim) {
  int32_t S = 0, per = 0;
  attn_split_shape(n_kv, n_head_kv, &S, &per);
  return (size_t)n_head * S * (head_dim + 2) * 4;
}

cudaError_t launch_attn_split(const float* q, const float* ck, const float* cv, int64_t D, int64_t H, int64_t HKV,
                              int64_t n_kv, float scale, const ExpTab& et, float* part, float* out,
                              cudaStream_t s) {
  int32_t S = 0, per = 0;
  attn_split_shape(n_kv, HKV, &S, &per);
  attn_split_kernel<<<dim3((unsigned)S, (unsigned)HKV), kSplitNT, 0, s>>>(q, ck, cv, (int)D, (int)H, (int)HKV,
                                                                          (int)n_kv, scale, per, et, part);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  attn_split_combine_kernel<<<(unsigned)H, kCombineNT, 0, s>>>(part, (int)D, S, et, out);
  return cudaGetLastError();
}

}  // namespace mi
