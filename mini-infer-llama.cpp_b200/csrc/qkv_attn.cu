// Fused QKV projection + decode attention for the decode executor on one GPU
// (sm_100a): one thread-block cluster per KV head.
//
// It performs, for one layer of one decode step, what the QKV GEMV kernel and
// the executor-mode attention kernel do back to back -- the attention rms_norm
// + MUL weight (ref src/ops_cpu.cpp:154-160), the quantize node
// (src/ops_cpu.cpp:462-479), the Q8_0 MUL_MAT of the stacked Q|K|V weights
// with the AVX2 lane order (src/ops_cpu.cpp:226-237, src/quant_avx2.cpp:170-181)
// plus bias, RoPE (src/ops_cpu.cpp:270-302), the KV-cache append
// (src/ops_cpu.cpp:446-460) and ATTN_QK / SOFTMAX / ATTN_KQV
// (src/ops_cpu.cpp:304-410) -- with the same operations in the same order, so
// its outputs are bit-identical to the two-kernel path. What it removes is the
// kernel boundary between the projection and the attention: the attention of
// a query head needs only its own 64..256 q rows and its KV head's k and v
// rows, so those are computed inside the head's cluster and handed over
// through distributed shared memory behind one cluster barrier.
//
// Cluster of n_rep + 1 CTAs for KV head kvh:
//   CTA c < n_rep  (query CTA of head h = kvh * n_rep + c): streams its q rows'
//                  weights and the cached K / V positions into shared memory
//                  before the dependency wait; prologue; q rows; bias; RoPE;
//                  waits for k / v; attention; the O projection's quantize.
//   CTA n_rep      (k/v CTA): streams the k and v rows' weights; prologue; k
//                  and v rows; bias; RoPE on k; appends k, v to the cache and
//                  stores them into every query CTA's kr / vr; arrives.
#include <algorithm>

#include "mi_device.cuh"

namespace mi {

namespace {

constexpr unsigned FULL = 0xffffffffu;
constexpr int kNT = 256, kNW = kNT / 32;
constexpr int kScoresOnChipMax = 8192;  // scores kept in shared memory up to this many positions

__host__ __device__ inline size_t up16(size_t v) { return (v + 15) / 16 * 16; }
__host__ __device__ inline size_t up128(size_t v) { return (v + 127) / 128 * 128; }

// Dynamic shared memory of the fused kernel, computed identically on host and
// device: [0, 8) the weights' mbarrier, [16, 64) broadcast scalars, the
// quantized activation, the F32 input, the rms_norm squares (+ chain slack),
// the ordered-sum scratch, the CTA's row results; then region A (the q rows'
// or the k rows' weights) and region B (the v rows' weights in the k/v CTA;
// K tile, V tile and scores in a query CTA).
struct FusedSmem {
  size_t aq, ad, xs, sq, spec, res, wa, wb, ks, vs, sc, total;
};

__host__ __device__ inline size_t fused_weight_bytes(int64_t K, int32_t D) {
  return up128((size_t)D * (size_t)K + (size_t)D * (size_t)(K / 32) * 2);
}

__host__ __device__ inline FusedSmem fused_smem(int64_t K, int32_t D, int32_t kt, size_t sc_bytes) {
  FusedSmem L;
  size_t off = 64;
  L.aq = off;
  off += up16((size_t)K);
  L.ad = off;
  off += up16((size_t)(K / 32) * 4);
  L.xs = off;
  off += (size_t)K * 4;
  L.sq = off;
  off += (size_t)K * 4 + kChainSlackBytes;
  L.spec = off;
  off += up16((size_t)spec_sum_scratch_bytes(8, 4));
  L.res = off;
  off += up16((size_t)2 * D * 4);
  off = up128(off);
  const size_t wbytes = fused_weight_bytes(K, D);
  L.wa = off;
  off += wbytes;
  L.wb = off;
  L.ks = off;
  L.vs = L.ks + (size_t)kt * (D + 1) * 4;
  L.sc = L.vs + (size_t)kt * D * 4;
  const size_t tile_end = L.sc + sc_bytes;
  L.total = off + wbytes > tile_end ? off + wbytes : tile_end;
  return L;
}

__global__ void __launch_bounds__(kNT, 1) qkv_attn_kernel(const QkvAttnParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(16) float qr[256], kr[256], vr[256];
  __shared__ float red[kNW];
  __shared__ float sh[2];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t K = p.K;
  const int nb = (int)(K >> 5);
  const int D = p.head_dim, half = D >> 1, D4 = D >> 2, HKV = p.n_head_kv;
  const int n_rep = p.n_head / HKV;
  const int crank = (int)cluster_ctarank();
  const int kvh = (int)blockIdx.x / (n_rep + 1);
  const bool kv_cta = crank == n_rep;
  const int h = kvh * n_rep + crank;  // query head (query CTAs)
  const int KT = p.kv_tile, KP = D + 1;
  const FusedSmem L = fused_smem(K, D, KT, 0);
  uint64_t* bar = (uint64_t*)smem;         // the CTA's weight copies
  uint64_t* bar_kv = (uint64_t*)(smem + 8);  // query CTAs: k and v from the k/v CTA
  float* misc = (float*)(smem + 16);
  int8_t* aq = (int8_t*)(smem + L.aq);
  float* ad = (float*)(smem + L.ad);
  float* xs = (float*)(smem + L.xs);
  float* res = (float*)(smem + L.res);
  float* Ks = (float*)(smem + L.ks);
  float* Vs = (float*)(smem + L.vs);
  const size_t rs = (size_t)HKV * D;
  const float* kbase = p.cache_k + (size_t)kvh * D;
  const float* vbase = p.cache_v + (size_t)kvh * D;
  const int64_t E = (int64_t)p.n_head * D;

  auto mark = [&](int point) {
    if (p.trace && tid == 0 && (blockIdx.x == 0 || (int)blockIdx.x == n_rep))
      p.trace[(size_t)(blockIdx.x == 0 ? p.trace_slot_q : p.trace_slot_kv) * kTracePoints + point] =
          globaltimer_ns();
  };
  trace_mark(p.trace, p.trace_slot, 0);
  mark(0);

  // pos was set before this step's graph started and changes only at its end,
  // so every CTA of the grid takes the same branch here.
  const int n_past = *p.pos;
  if (n_past < 0 || n_past >= p.n_ctx) {  // no cache row / RoPE entry for this position
    pdl_trigger();
    if (tid == 0 && blockIdx.x == 0) atomicExch(p.err, 6 /* MI_CUDA_ERR_STATE */);
    return;
  }
  const int n_kv = n_past + 1;

  // ---- before the dependency wait: weights and cached K / V into shared memory ----
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_init(bar_kv, 1);
    fence_mbar_init();
  }
  __syncthreads();
  // Cluster phase 0: every CTA's barriers are initialized (the k/v CTA stores
  // into the query CTAs' shared memory only after it).
  cluster_arrive_relaxed();
  if (tid == 0) {
    if (!kv_cta) mbar_arrive_expect_tx(bar_kv, (uint32_t)(2 * D * 4));
    // D rows from packed row r (a multiple of 8): quants at r * K, scales at
    // r * nb * 2 bytes into the scale plane
    const uint32_t qb = (uint32_t)((int64_t)D * K), db = (uint32_t)(D * nb * 2);
    const uint8_t* wd = p.w + p.n_pad * K;
    const uint64_t wpol = l2_evict_first_policy();  // weights are read once per step
    mbar_arrive_expect_tx(bar, (kv_cta ? 2u : 1u) * (qb + db));
    const int64_t ra = kv_cta ? E + (int64_t)kvh * D : (int64_t)h * D;
    bulk_load_hint(smem + L.wa, p.w + ra * K, qb, bar, wpol);
    bulk_load_hint(smem + L.wa + (size_t)D * K, wd + ra * nb * 2, db, bar, wpol);
    if (kv_cta) {
      const int64_t rb = E + (int64_t)HKV * D + (int64_t)kvh * D;
      bulk_load_hint(smem + L.wb, p.w + rb * K, qb, bar, wpol);
      bulk_load_hint(smem + L.wb + (size_t)D * K, wd + rb * nb * 2, db, bar, wpol);
    }
  }
  // The weights' other operands, into registers: rms_norm weights of this
  // lane's first four blocks; the RoPE pair and bias of element tid (q rows,
  // or k rows) and of v element tid.
  float nw[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int u = 0; u < 4; u++)
    if (warp + u * kNW < nb) nw[u] = p.norm_w[(int64_t)(warp + u * kNW) * 32 + lane];
  float2 rc = make_float2(0.0f, 0.0f);
  float b_lo = 0.0f, b_hi = 0.0f, b_v = 0.0f;
  {
    const float* b0 = p.bias + (kv_cta ? E + (int64_t)kvh * D : (int64_t)h * D);
    if (tid < half) {
      rc = p.rope_cs[(size_t)n_past * half + tid];
      b_lo = b0[tid];
      b_hi = b0[tid + half];
    }
    if (kv_cta && tid < D) b_v = p.bias[E + (int64_t)HKV * D + (int64_t)kvh * D + tid];
  }
  // Rows [c0, c0 + rows) of the cache into the K / V tiles (row n_past, this
  // step's, comes from kr / vr); four 16-byte loads in flight per thread.
  auto load_k = [&](int c0, int rows) {
    const int total = rows * D4;
    for (int e0 = tid; e0 < total; e0 += 4 * kNT) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int e = e0 + u * kNT, r = e / D4, c = e - r * D4;
        if (e < total && c0 + r != n_past) v[u] = *(const float4*)(kbase + (size_t)(c0 + r) * rs + c * 4);
      }
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int e = e0 + u * kNT, r = e / D4, c = e - r * D4;
        if (e < total && c0 + r != n_past) {
          float* d = Ks + (size_t)r * KP + c * 4;
          d[0] = v[u].x;
          d[1] = v[u].y;
          d[2] = v[u].z;
          d[3] = v[u].w;
        }
      }
    }
  };
  auto load_v = [&](int c0, int rows) {
    const int total = rows * D4;
    for (int e0 = tid; e0 < total; e0 += 4 * kNT) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int e = e0 + u * kNT, r = e / D4, c = e - r * D4;
        if (e < total && c0 + r != n_past) v[u] = *(const float4*)(vbase + (size_t)(c0 + r) * rs + c * 4);
      }
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int e = e0 + u * kNT, r = e / D4, c = e - r * D4;
        if (e < total && c0 + r != n_past) *(float4*)(Vs + (size_t)r * D + c * 4) = v[u];
      }
    }
  };
  const int rows0 = min(KT, n_kv);
  if (!kv_cta) {
    load_k(0, rows0);
    load_v(0, rows0);
  }
  pdl_trigger();
  pdl_wait_cta();
  trace_mark(p.trace, p.trace_slot, 1);
  mark(1);

  // ---- prologue: x (or the embedding row), rms_norm, quantize ----
  if (p.pro == PRO_EMBED_NORM) {
    // mi_compute_get_rows on the Q8_0 embedding (ref src/ops_cpu.cpp:128-139).
    int tok = n_past < p.tokens_len ? p.tokens[n_past] : -1;
    if (tok < 0 || tok >= p.embed_rows) {
      if (tid == 0) atomicExch(p.err, 1 /* MI_CUDA_ERR_ARG */);
      tok = 0;
    }
    for (int64_t k = tid; k < K; k += kNT) {
      const int64_t b = k >> 5;
      const float d = packed_scale(p.embed, K, p.embed_npad, tok, b);
      const float v = __fmul_rn((float)packed_qs(p.embed, K, tok, b)[k & 31], d);
      xs[k] = v;
      if (blockIdx.x == 0) p.x_out[k] = v;
    }
  } else {
    const float4* x4 = (const float4*)p.x;
    float4* xs4 = (float4*)xs;
    for (int64_t k = tid; k < K / 4; k += kNT) xs4[k] = x4[k];
  }
  __syncthreads();
  mark(2);
  {
    float* sq = (float*)(smem + L.sq);
    for (int64_t k = tid; k < K; k += kNT) sq[k] = __fmul_rn(xs[k], xs[k]);
    __syncthreads();
    const float ss = K <= 1024 ? spec_ordered_sum<kNT, 2>(sq, (int)K, smem + L.spec)
                               : spec_ordered_sum<kNT, 4>(sq, (int)K, smem + L.spec);
    if (tid == 0) {
      const float mean = __fdiv_rn(ss, (float)K);
      misc[0] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
    }
    __syncthreads();
    mark(3);
  }
  {
    // rms_norm then MUL weight, quantized; four blocks per iteration overlap
    // the quantizer's divisions. The warp's blocks are warp + u*kNW.
    const float scale = misc[0];
    auto value = [&](int64_t k, float nwk) { return __fmul_rn(__fmul_rn(xs[k], scale), nwk); };
    int b = warp;
    for (; b + 3 * kNW < nb; b += 4 * kNW) {
      float v[4], d[4];
      int8_t q[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int64_t k = (int64_t)(b + u * kNW) * 32 + lane;
        v[u] = value(k, b == warp ? nw[u] : p.norm_w[k]);
      }
#pragma unroll
      for (int u = 0; u < 4; u++) q[u] = quantize_lane(v[u], &d[u]);
#pragma unroll
      for (int u = 0; u < 4; u++) {
        aq[(int64_t)(b + u * kNW) * 32 + lane] = q[u];
        if (lane == 0) ad[b + u * kNW] = d[u];
      }
    }
    if (b == warp) {  // fewer than four blocks for this warp: all preloaded
#pragma unroll
      for (int u = 0; u < 3; u++) {
        if (b + u * kNW >= nb) break;
        const int64_t k = (int64_t)(b + u * kNW) * 32 + lane;
        float d;
        aq[k] = quantize_lane(value(k, nw[u]), &d);
        if (lane == 0) ad[b + u * kNW] = d;
      }
    } else {
      for (; b < nb; b += kNW) {
        const int64_t k = (int64_t)b * 32 + lane;
        float d;
        aq[k] = quantize_lane(value(k, p.norm_w[k]), &d);
        if (lane == 0) ad[b] = d;
      }
    }
  }
  __syncthreads();
  trace_mark(p.trace, p.trace_slot, 2);
  mark(4);

  // ---- the CTA's rows: 2 threads per row, four lane chains each ----
  // Lanes 8w'..8w'+7 of a warp take group 4*warp + w' (rows r4 = 0..3, halves
  // h = 0/1); thread h keeps the chains of lanes 4h..4h+3 from one 16-byte
  // load of the block's quants and of the activation.
  const bool ok = __syncthreads_and(mbar_wait_bounded(bar, 0u, p.err));
  if (ok) {
    const int gw = lane >> 3, r4 = (lane >> 1) & 3, hh = lane & 1;
    const uint4* aq16 = (const uint4*)aq;
    const int n_groups = (kv_cta ? 2 : 1) * D4;  // row groups of 4
    for (int g0 = warp * 4; g0 < n_groups; g0 += kNW * 4) {
      const int g = g0 + gw;
      const bool valid = g < n_groups;
      const int gc = valid ? g : g0;  // out-of-range groups recompute g0, never store
      const int blk = gc / D4, gg = gc - blk * D4;
      const uint8_t* base = smem + (blk ? L.wb : L.wa);
      const uint4* gq = (const uint4*)(base + (size_t)gg * 4 * K);
      const __half* gd = (const __half*)(base + (size_t)D * K) + (size_t)gg * nb * 4;
      float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
#pragma unroll 2
      for (int i = 0; i < nb; i++) {
        const uint4 w = gq[i * 8 + (lane & 7)];
        const uint4 a = aq16[i * 2 + hh];
        const float dxdy = __fmul_rn(__half2float(gd[i * 4 + r4]), ad[i]);
        a0 = __fmaf_rn(__int2float_rn(__dp4a((int)w.x, (int)a.x, 0)), dxdy, a0);
        a1 = __fmaf_rn(__int2float_rn(__dp4a((int)w.y, (int)a.y, 0)), dxdy, a1);
        a2 = __fmaf_rn(__int2float_rn(__dp4a((int)w.z, (int)a.z, 0)), dxdy, a2);
        a3 = __fmaf_rn(__int2float_rn(__dp4a((int)w.w, (int)a.w, 0)), dxdy, a3);
      }
      // hsum ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7))
      const float s0 = __fadd_rn(a0, __shfl_xor_sync(FULL, a0, 1));
      const float s1 = __fadd_rn(a1, __shfl_xor_sync(FULL, a1, 1));
      const float s2 = __fadd_rn(a2, __shfl_xor_sync(FULL, a2, 1));
      const float s3 = __fadd_rn(a3, __shfl_xor_sync(FULL, a3, 1));
      if (valid && hh == 0) res[g * 4 + r4] = __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
    }
  }
  __syncthreads();
  mark(5);

  // ---- bias, RoPE ----
  if (tid < half) {
    const float a0 = __fadd_rn(res[tid], b_lo), a1 = __fadd_rn(res[tid + half], b_hi);
    float* dst = kv_cta ? kr : qr;
    dst[tid] = __fsub_rn(__fmul_rn(a0, rc.x), __fmul_rn(a1, rc.y));
    dst[tid + half] = __fadd_rn(__fmul_rn(a0, rc.y), __fmul_rn(a1, rc.x));
  }
  if (kv_cta && tid < D) vr[tid] = __fadd_rn(res[D + tid], b_v);
  __syncthreads();
  mark(6);

  // ---- k / v hand-over ----
  // The k/v CTA stores k and v into every query CTA's kr / vr with st.async,
  // counted on that CTA's bar_kv; a query CTA waits on its own barrier.
  // Cluster phase 1: every query CTA has received them (the k/v CTA exits
  // only then).
  if (kv_cta) {
    cluster_wait_acquire();  // phase 0
    const int per = D >> 1;  // float4s per query CTA: k then v
    for (int e = tid; e < n_rep * per; e += kNT) {
      const int c = e / per, i4 = e - c * per;
      const float* src = i4 < D4 ? kr + 4 * i4 : vr + 4 * (i4 - D4);
      dsmem_store_async(dsmem_addr(src, (uint32_t)c), *(const float4*)src, dsmem_addr(bar_kv, (uint32_t)c));
    }
    if (ok && tid < D) {  // the KV-cache append
      p.cache_k[((size_t)n_past * HKV + kvh) * D + tid] = kr[tid];
      p.cache_v[((size_t)n_past * HKV + kvh) * D + tid] = vr[tid];
    }
    mark(7);
    cluster_arrive_relaxed();
    cluster_wait_acquire();  // phase 1
    if (!ok && tid == 0) (void)mbar_wait_bounded(bar, 0u, nullptr);
    return;
  }
  (void)mbar_wait_bounded(bar_kv, 0u, p.err);
  if (n_past < KT && tid < D) {
    Ks[(size_t)n_past * KP + tid] = kr[tid];
    Vs[(size_t)n_past * D + tid] = vr[tid];
  }
  cluster_wait_acquire();  // phase 0
  cluster_arrive_relaxed();
  __syncthreads();
  trace_mark(p.trace, p.trace_slot, 4);
  mark(7);
  if (!ok) {
    // Copies that did not land get a bounded chance before the shared memory
    // is released.
    if (tid == 0) (void)mbar_wait_bounded(bar, 0u, nullptr);
    cluster_wait_acquire();
    return;
  }

  // ---- attention of head h ----
  float* sc = p.scores_in_smem ? (float*)(smem + L.sc) : p.scores + (size_t)h * p.scores_stride;
  const int n_chunks = (n_kv + KT - 1) / KT;
  // scores[i] * scale, d ascending with separate roundings (src/ops_cpu.cpp:373-376).
  float lmax = -INFINITY;
  for (int c = 0; c < n_chunks; c++) {
    const int c0 = c * KT, rows = min(KT, n_kv - c0);
    if (c > 0) {
      __syncthreads();
      load_k(c0, rows);
      if (n_past >= c0 && n_past < c0 + rows)
        for (int i = tid; i < D; i += kNT) Ks[(size_t)(n_past - c0) * KP + i] = kr[i];
      __syncthreads();
    }
    for (int i = tid; i < rows; i += kNT) {
      const float acc = ordered_dot(0.0f, Ks + (size_t)i * KP, 1, qr, D);
      const float v = __fmul_rn(acc, p.scale);
      sc[c0 + i] = v;
      lmax = fmaxf(lmax, v);
    }
  }
  trace_mark(p.trace, p.trace_slot, 5);
  lmax = warp_max(lmax);
  if (lane == 0) red[warp] = lmax;
  __syncthreads();
  float mx = red[0];  // every thread reduces the warps' maxima (order-free)
  for (int w = 1; w < kNW; w++) mx = fmaxf(mx, red[w]);
  for (int i = tid; i < n_kv; i += kNT) sc[i] = expf_exact(__fsub_rn(sc[i], mx), p.et);
  __syncthreads();
  trace_mark(p.trace, p.trace_slot, 6);
  // The softmax denominator: one ordered chain (src/ops_cpu.cpp:331-336).
  if (tid == 0) {
    float sum = 0.0f;
    if (p.scores_in_smem) {
      sum = ordered_sum_smem(sc, n_kv);
    } else {
#pragma unroll 8
      for (int i = 0; i < n_kv; i++) sum = __fadd_rn(sum, sc[i]);
    }
    sh[1] = __fdiv_rn(1.0f, sum);
  }
  __syncthreads();
  const float inv = sh[1];
  trace_mark(p.trace, p.trace_slot, 7);

  // out[o] = sum_t V[o, kvh, t] * P[t], t ascending (src/ops_cpu.cpp:402-406).
  float acc = 0.0f;
  for (int c = 0; c < n_chunks; c++) {
    const int c0 = c * KT, rows = min(KT, n_kv - c0);
    if (c > 0) {
      __syncthreads();
      load_v(c0, rows);
      if (n_past >= c0 && n_past < c0 + rows)
        for (int i = tid; i < D; i += kNT) Vs[(size_t)(n_past - c0) * D + i] = vr[i];
      __syncthreads();
    }
    if (tid < D) acc = ordered_dot_scaled(acc, Vs + tid, D, sc + c0, inv, rows);
  }
  trace_mark(p.trace, p.trace_slot, 3);
  if (p.act_out) {
    // The O projection's quantize node (src/ops_cpu.cpp:462-479) for this head's
    // outputs: warp w holds block h*D/32 + w of the concatenated heads.
    if (tid < D) {
      float d;
      const int8_t q = quantize_lane(acc, &d);
      uint8_t* blk = p.act_out + ((size_t)h * (D >> 5) + (tid >> 5)) * 36;
      ((int8_t*)blk)[4 + lane] = q;
      if (lane == 0) *(float*)blk = d;
    }
  } else if (tid < D) {
    p.out[(size_t)h * D + tid] = acc;
  }
  cluster_wait_acquire();  // phase 1
}

int g_optin = 0;  // the device's opt-in shared memory per block (prepare_qkv_attn_kernel)

}  // namespace

cudaError_t prepare_qkv_attn_kernel(int optin) {
  cudaFuncAttributes f{};
  cudaError_t e = cudaFuncGetAttributes(&f, qkv_attn_kernel);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(qkv_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             optin - (int)f.sharedSizeBytes);
  if (e == cudaSuccess) e = set_carveout(qkv_attn_kernel);
  if (e == cudaSuccess) g_optin = optin - (int)f.sharedSizeBytes;
  return e;
}

QkvAttnPlan plan_qkv_attn(int64_t K, int32_t D, int32_t n_head, int32_t n_head_kv, int32_t n_ctx,
                          size_t smem_budget) {
  QkvAttnPlan pl{};
  if (D < 8 || D > 256 || D % 8 != 0 || n_head_kv <= 0 || n_head % n_head_kv != 0 || K % 32 != 0 ||
      K < 32 || n_ctx <= 0)
    return pl;
  const int32_t n_rep = n_head / n_head_kv;
  if (n_rep + 1 > 8) return pl;  // portable cluster size
  const size_t sc = n_ctx <= kScoresOnChipMax ? up16((size_t)n_ctx * 4) + kChainSlackBytes : 0;
  const size_t fixed = fused_smem(K, D, 0, 0).wb;  // everything before region B
  const size_t row = (size_t)(2 * D + 1) * 4;      // one K and one V position
  if (smem_budget < fixed + sc + 32 * row) return pl;
  int64_t kt = (int64_t)((smem_budget - fixed - sc) / row);
  kt = std::min<int64_t>(256, kt) / 32 * 32;
  const FusedSmem L = fused_smem(K, D, (int32_t)kt, sc);
  if (L.total > smem_budget || (g_optin > 0 && L.total > (size_t)g_optin)) return pl;
  // Weight copies: one mbarrier phase counts at most 2^20 - 1 bytes.
  if (2 * fused_weight_bytes(K, D) >= (1u << 20)) return pl;
  pl.ok = true;
  pl.cluster = n_rep + 1;
  pl.kv_tile = (int32_t)kt;
  pl.scores_in_smem = sc > 0 ? 1 : 0;
  pl.smem = L.total;
  // The device must be able to hold one cluster.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(n_head_kv * pl.cluster));
  cfg.blockDim = dim3(kNT);
  cfg.dynamicSmemBytes = pl.smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)pl.cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, qkv_attn_kernel, &cfg) != cudaSuccess || n < 1) {
    cudaGetLastError();
    pl.ok = false;
  }
  return pl;
}

cudaError_t launch_qkv_attn(const QkvAttnParams& p, const QkvAttnPlan& plan, cudaStream_t s, bool pdl) {
  if (!plan.ok) return cudaErrorInvalidValue;
  QkvAttnParams q = p;
  q.kv_tile = plan.kv_tile;
  q.scores_in_smem = plan.scores_in_smem;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(p.n_head_kv * plan.cluster));
  cfg.blockDim = dim3(kNT);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)plan.cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, qkv_attn_kernel, q);
}

}  // namespace mi
