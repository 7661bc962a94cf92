// Decode attention, split over positions (a labelled fast mode, not
// bit-exact). No counterpart in the reference.
//
// The reference's ATTN_QK / SOFTMAX / ATTN_KQV (ref src/ops_cpu.cpp:304-410)
// sum the softmax denominator and every output's value sum as one chain over
// all n_kv positions; the exact kernel keeps those chains, which makes long
// contexts latency-bound (a 32768-long dependent chain per output). This mode
// splits the positions over many CTAs and combines their partial results
// (per-split maximum, denominator and unnormalized value sums, rescaled to the
// global maximum), the way split-K decode attention kernels do. The sums are
// regrouped, the products fused and the exponentials CUDA's expf, so results
// differ from the reference's in the last bits (tested within max-abs 1e-5).
// The exact kernel stays the one the decode path uses.
//
// Grid (splits, n_head_kv): a CTA takes the n_rep query heads of one KV head
// over one range of positions and streams it through shared memory in
// sub-chunks of 32 positions (a ring of three buffers of 16-byte
// asynchronous copies: two sub-chunks in flight while one is computed), with
// an online softmax across the sub-chunks; it writes (maximum, denominator,
// unnormalized value sums) per head. A second kernel, chained by
// programmatic dependent launch, combines the splits.
#include <algorithm>

#include "mi_device.cuh"

namespace mi {

namespace {

constexpr int kSplitNT = 256;
constexpr int kSub = 32;           // positions per sub-chunk
constexpr int kBuf = 3;            // sub-chunk buffers (two in flight)
constexpr int kSplitMaxRep = 16;   // query heads per KV head
constexpr int kSplitMaxD = 128;
constexpr int kMaxSplits = 4096;
constexpr int kMaxPerSplit = 2048;  // positions per CTA

// Shared memory of one CTA for head_dim D and n_rep query heads: q [R][D],
// K sub-chunks [kBuf][32][D + 4] (rows padded: a warp's lanes read 32
// different rows at one d), V sub-chunks [kBuf][32][D], probabilities
// [R][32], per-head rescale factors and running state [3][R].
__host__ __device__ inline size_t split_smem_bytes(int D, int R) {
  return ((size_t)R * D + (size_t)kBuf * kSub * (D + 4) + (size_t)kBuf * kSub * D + (size_t)R * kSub + 3 * R) * 4;
}

// Value units of a CTA: (head r, outputs 4*o4 .. 4*o4 + 3, part of the
// sub-chunk's positions); NP parts so that the units fill the threads.
__host__ __device__ inline int split_parts(int n_rep, int D) {
  const int base = n_rep * (D / 4);
  int np = 1;
  while (np < 4 && base * np * 2 <= kSplitNT) np *= 2;
  return np;
}

// D (head_dim) is a compile-time constant so the dot and value loops unroll.
template <int D>
__global__ void __launch_bounds__(kSplitNT) attn_split_kernel(const float* q, const float* ck, const float* cv,
                                                              int H, int HKV, int n_kv, float scale, int per_split,
                                                              float* part) {
  extern __shared__ __align__(16) float sm[];
  constexpr int KP = D + 4, D4 = D >> 2;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kvh = blockIdx.y, s = blockIdx.x, S = gridDim.x;
  const int n_rep = H / HKV, h0 = kvh * n_rep;
  const int t0 = s * per_split, cnt = min(n_kv, t0 + per_split) - t0;
  const int nsub = (cnt + kSub - 1) / kSub;
  float* q_s = sm;                            // [R][D]
  float* K_b = q_s + n_rep * D;               // [kBuf][32][D + 4]
  float* V_b = K_b + kBuf * kSub * KP;        // [kBuf][32][D]
  float* p_s = V_b + kBuf * kSub * D;         // [R][32]
  float* sc_s = p_s + n_rep * kSub;           // [R] rescale of this sub-chunk
  float* m_s = sc_s + n_rep;                  // [R] running maximum
  float* l_s = m_s + n_rep;                   // [R] running denominator
  const size_t rs = (size_t)HKV * D;
  constexpr int sh4 = D4 == 1 ? 0 : D4 == 2 ? 1 : D4 == 4 ? 2 : D4 == 8 ? 3 : D4 == 16 ? 4 : 5;  // log2(D / 4)
  // sub-chunk c of the range into buffer c % kBuf (one commit group per call,
  // empty past the range)
  auto issue = [&](int c) {
    if (c < nsub) {
      const int b = c % kBuf, tb = c * kSub, rows = min(kSub, cnt - tb);
      float* Kd = K_b + b * kSub * KP;
      float* Vd = V_b + b * kSub * D;
      for (int e = tid; e < rows * D4; e += kSplitNT) {
        const int t = e >> sh4, cc = e & (D4 - 1);
        const size_t off = (size_t)(t0 + tb + t) * rs + (size_t)kvh * D + (size_t)cc * 4;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(Kd + t * KP + 4 * cc)),
                     "l"(ck + off)
                     : "memory");
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(Vd + t * D + 4 * cc)),
                     "l"(cv + off)
                     : "memory");
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  issue(0);
  issue(1);
  for (int e = tid; e < n_rep * D; e += kSplitNT) q_s[e] = q[(size_t)h0 * D + e];
  if (tid < n_rep) {
    m_s[tid] = -INFINITY;
    l_s[tid] = 0.0f;
  }
  // value units: thread tid owns units tid and tid + kSplitNT (float4 sums
  // carried over the sub-chunks, rescaled as the running maximum grows)
  const int NP = split_parts(n_rep, D), n_units = n_rep * D4 * NP, plen = kSub / NP;
  float4 acc[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
  for (int c = 0; c < nsub; c++) {
    const int b = c % kBuf, rows = min(kSub, cnt - c * kSub);
    asm volatile("cp.async.wait_group 1;" ::: "memory");  // sub-chunk c (groups complete in order)
    __syncthreads();  // every thread's copies of c; buffer (c + 2) % kBuf no longer read
    issue(c + 2);
    const float* Kc = K_b + b * kSub * KP;
    const float* Vc = V_b + b * kSub * D;
    // scores: item (position t, head r), fused dot products
    for (int it = tid; it < kSub * n_rep; it += kSplitNT) {
      const int t = it & (kSub - 1), r = it >> 5;
      float v = -INFINITY;
      if (t < rows) {
        const float* kr = Kc + t * KP;
        const float* qr = q_s + r * D;
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
        for (int d4 = 0; d4 < D4; d4++) {
          const float4 kv = *(const float4*)(kr + 4 * d4);
          const float4 qv = *(const float4*)(qr + 4 * d4);
          a0 = __fmaf_rn(kv.x, qv.x, a0);
          a1 = __fmaf_rn(kv.y, qv.y, a1);
          a2 = __fmaf_rn(kv.z, qv.z, a2);
          a3 = __fmaf_rn(kv.w, qv.w, a3);
        }
        v = __fmul_rn(__fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3)), scale);
      }
      p_s[r * kSub + t] = v;
    }
    __syncthreads();
    // online softmax: a warp per head (lane = position of the sub-chunk)
    for (int r = warp; r < n_rep; r += kSplitNT / 32) {
      const float x = p_s[r * kSub + lane];
      const float mo = m_s[r];
      const float mn = fmaxf(mo, warp_max(x));
      const float e = lane < rows ? expf(x - mn) : 0.0f;
      float l = e;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) l = __fadd_rn(l, __shfl_xor_sync(0xffffffffu, l, o));
      p_s[r * kSub + lane] = e;
      if (lane == 0) {
        const float scl = mo == -INFINITY ? 0.0f : expf(mo - mn);
        sc_s[r] = scl;
        l_s[r] = __fmaf_rn(l_s[r], scl, l);
        m_s[r] = mn;
      }
    }
    __syncthreads();
    // value sums of this sub-chunk into the carried units
#pragma unroll
    for (int k = 0; k < 2; k++) {
      const int u = tid + k * kSplitNT;
      if (u < n_units) {
        const int pt = u / (n_rep * D4), ru = u - pt * (n_rep * D4);
        const int r = ru / D4, o4 = ru - r * D4;
        const float scl = sc_s[r];
        float4 a = acc[k];
        a.x = __fmul_rn(a.x, scl);
        a.y = __fmul_rn(a.y, scl);
        a.z = __fmul_rn(a.z, scl);
        a.w = __fmul_rn(a.w, scl);
        const float* pr = p_s + r * kSub;
        const int tb = pt * plen, te = min(rows, tb + plen);
#pragma unroll 4
        for (int t = tb; t < te; t++) {
          const float pv = pr[t];
          const float4 v = *(const float4*)(Vc + t * D + 4 * o4);
          a.x = __fmaf_rn(pv, v.x, a.x);
          a.y = __fmaf_rn(pv, v.y, a.y);
          a.z = __fmaf_rn(pv, v.z, a.z);
          a.w = __fmaf_rn(pv, v.w, a.w);
        }
        acc[k] = a;
      }
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  // the parts of every unit meet in shared memory (the K buffers are free)
  float* red = K_b;  // [NP][n_rep * D]
#pragma unroll
  for (int k = 0; k < 2; k++) {
    const int u = tid + k * kSplitNT;
    if (u < n_units) *(float4*)(red + 4 * u) = acc[k];
  }
  __syncthreads();
  for (int e = tid; e < n_rep * D; e += kSplitNT) {
    float v = red[e];
    for (int pt = 1; pt < NP; pt++) v = __fadd_rn(v, red[pt * n_rep * D + e]);
    const int r = e / D, o = e - r * D;
    part[((size_t)(h0 + r) * S + s) * (D + 2) + 2 + o] = v;
  }
  if (tid < n_rep) {
    float* ph = part + ((size_t)(h0 + tid) * S + s) * (D + 2);
    ph[0] = m_s[tid];
    ph[1] = l_s[tid];
  }
  __syncthreads();
  pdl_trigger();  // the combine kernel may launch; it waits for this grid's stores
}

// out[h][o] = sum_s acc_s[o] * e^(m_s - M) / sum_s l_s * e^(m_s - M), M the
// largest split maximum. Grid (heads, ceil(D / 8)): a thread per split (in
// strides), the eight outputs' sums and the denominator reduced over the CTA.
constexpr int kCombineNT = 256;
constexpr int kCombineOut = 8;
__global__ void __launch_bounds__(kCombineNT) attn_split_combine_kernel(const float* part, int D, int S, float* out) {
  __shared__ float red[kCombineNT / 32][kCombineOut + 1];
  pdl_wait();  // the split kernel's partial records are complete and visible
  const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int o0 = blockIdx.y * kCombineOut, no = min(kCombineOut, D - o0);
  const size_t st = (size_t)D + 2;
  const float* ph = part + (size_t)h * S * st;
  float m = -INFINITY;
  for (int s = tid; s < S; s += kCombineNT) m = fmaxf(m, ph[s * st]);
  m = warp_max(m);
  if (lane == 0) red[warp][0] = m;
  __syncthreads();
  float M = red[0][0];
  for (int w = 1; w < kCombineNT / 32; w++) M = fmaxf(M, red[w][0]);
  __syncthreads();
  float l = 0.0f, a[kCombineOut];
#pragma unroll
  for (int i = 0; i < kCombineOut; i++) a[i] = 0.0f;
  for (int s = tid; s < S; s += kCombineNT) {
    const float* rec = ph + s * st;
    const float w = expf(rec[0] - M);
    l = __fmaf_rn(rec[1], w, l);
#pragma unroll
    for (int i = 0; i < kCombineOut; i++)
      if (i < no) a[i] = __fmaf_rn(rec[2 + o0 + i], w, a[i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    l = __fadd_rn(l, __shfl_xor_sync(0xffffffffu, l, o));
#pragma unroll
    for (int i = 0; i < kCombineOut; i++) a[i] = __fadd_rn(a[i], __shfl_xor_sync(0xffffffffu, a[i], o));
  }
  if (lane == 0) {
    red[warp][0] = l;
#pragma unroll
    for (int i = 0; i < kCombineOut; i++) red[warp][1 + i] = a[i];
  }
  __syncthreads();
  if (tid < no) {
    float L = red[0][0], A = red[0][1 + tid];
    for (int w = 1; w < kCombineNT / 32; w++) {
      L = __fadd_rn(L, red[w][0]);
      A = __fadd_rn(A, red[w][1 + tid]);
    }
    out[(size_t)h * D + o0 + tid] = __fdiv_rn(A, L);
  }
}

}  // namespace

// The split kernels' shared-memory attribute, once per device (at its init).
cudaError_t prepare_attn_split_kernels() {
  const int most = (int)split_smem_bytes(kSplitMaxD, kSplitMaxRep);
  const void* fns[] = {(const void*)attn_split_kernel<4>,  (const void*)attn_split_kernel<8>,
                       (const void*)attn_split_kernel<16>, (const void*)attn_split_kernel<32>,
                       (const void*)attn_split_kernel<64>, (const void*)attn_split_kernel<128>};
  for (const void* f : fns) {
    const cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, most);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

bool attn_split_fits(int64_t head_dim, int64_t n_head, int64_t n_head_kv) {
  return head_dim >= 4 && head_dim <= kSplitMaxD && (head_dim & (head_dim - 1)) == 0 && n_head > 0 &&
         n_head < (1ll << 31) && n_head_kv > 0 && n_head % n_head_kv == 0 &&
         n_head / n_head_kv <= kSplitMaxRep;
}

// Positions per CTA: a multiple of 32, chosen so that the CTAs of all KV
// heads are about 4 per SM of a 148-SM B200 (one wave, every CTA streaming).
void attn_split_shape(int64_t n_kv, int64_t n_head_kv, int32_t* n_splits, int32_t* per_split) {
  const int64_t want = (std::max<int64_t>(1, n_kv) * std::max<int64_t>(1, n_head_kv) + 591) / 592;
  int64_t per = std::min<int64_t>(kMaxPerSplit, std::max<int64_t>(kSub, (want + kSub - 1) / kSub * kSub));
  while ((n_kv + per - 1) / per > kMaxSplits && per < kMaxPerSplit) per += kSub;
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
  (void)et;   // (this mode uses CUDA's expf: its sums are regrouped anyway)
  if (S > kMaxSplits) return cudaErrorInvalidValue;
  const size_t smem = split_smem_bytes((int)D, (int)(H / HKV));
  cudaError_t e = cudaSuccess;
  const dim3 grid((unsigned)S, (unsigned)HKV);
  switch (D) {
#define MI_SPLIT_CASE(DD)                                                                                     \
  case DD:                                                                                                   \
    attn_split_kernel<DD><<<grid, kSplitNT, smem, s>>>(q, ck, cv, (int)H, (int)HKV, (int)n_kv, scale, per, part); \
    break;
    MI_SPLIT_CASE(4)
    MI_SPLIT_CASE(8)
    MI_SPLIT_CASE(16)
    MI_SPLIT_CASE(32)
    MI_SPLIT_CASE(64)
    MI_SPLIT_CASE(128)
#undef MI_SPLIT_CASE
    default:
      return cudaErrorInvalidValue;
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  // the combine, launched as the split kernel's programmatic dependent: its
  // CTAs start as the split CTAs finish and wait (griddepcontrol.wait) for
  // the whole grid's stores
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)H, (unsigned)((D + kCombineOut - 1) / kCombineOut));
  cfg.blockDim = dim3(kCombineNT);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, attn_split_combine_kernel, (const float*)part, (int)D, (int)S, out);
}

}  // namespace mi
