// CUDA kernels of the decode path (sm_100a) and their launchers.
//
// Every kernel reproduces the reference's IEEE operation order (see
// mi_device.cuh); the comment above each names the reference code it
// replaces.
#include <algorithm>
#include <cstdio>
#include <cstdlib>

#include "mi_device.cuh"

namespace mi {

namespace {

constexpr unsigned FULL = 0xffffffffu;
// Shortest chain evaluated with spec_ordered_sum; below it one thread's serial
// chain is faster than the CTA-wide speculation's fixed cost.
constexpr int kSpecSumMin = 256;

// Shared-memory map of the GEMV kernel, computed identically on host and
// device: [0,256) mbarriers, [256,320) broadcast scalars, activation quants,
// activation scales, per-row results, F32 input staging (norm prologues),
// then n_stages weight stages, each stage_rows rows by kc blocks of K (the
// groups' quants, then their scales).
struct GemvSmem {
  size_t act_qs, act_d, res, xs, sq, spec, stages, stage_bytes, total;
};

__host__ __device__ inline GemvSmem gemv_smem(int64_t K, int32_t rows_per_cta, int32_t stage_rows,
                                              int32_t n_stages, int32_t pro, int32_t stage_x,
                                              int32_t kc) {
  GemvSmem L;
  size_t off = 320;
  L.act_qs = off;
  off += (size_t)((K + 15) / 16 * 16);
  L.act_d = off;
  off += (size_t)((K / 32 * 4 + 15) / 16 * 16);
  L.res = off;
  off += (size_t)(((int64_t)rows_per_cta * 4 + 15) / 16 * 16);
  L.xs = off;
  if (pro >= PRO_NORM_QUANT || (pro == PRO_QUANT && stage_x)) off += (size_t)(K * 4);
  L.sq = off;  // squares for the rms_norm chain, plus the chain loads' slack
  if (pro >= PRO_NORM_QUANT) off += (size_t)(K * 4 + kChainSlackBytes);
  L.spec = off;  // spec_ordered_sum scratch for that chain (8 warps, up to 4 chains a lane)
  if (pro >= PRO_NORM_QUANT) off += (size_t)((spec_sum_scratch_bytes(8, 4) + 15) / 16 * 16);
  off = (off + 127) / 128 * 128;
  L.stages = off;
  L.stage_bytes = (size_t)(((int64_t)stage_rows * kc * 34 + 127) / 128 * 128);
  off += (size_t)n_stages * L.stage_bytes;
  L.total = off;
  return L;
}

}  // namespace

// ---------------------------------------------------------------------------
// Q8_0 GEMV: out[r] = dot(W row r, act) for the CTA's contiguous rows.
//
// Replaces mi_compute_mul_mat's Q8_0 branch (ref src/ops_cpu.cpp:226-237) and
// the quantize node in front of it (src/ops_cpu.cpp:462-479). Per row, eight
// lanes each keep the AVX2 kernel's accumulator chain (ref
// src/quant_avx2.cpp:170-181): lane j of block i adds the int32 dot of bytes
// 4j..4j+3 (one dp4a, exactly the maddubs+madd lane partial) times
// fp16(w.d)*a.d with one FMA, blocks in order; the row result is the hsum_ps
// order ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7)) (src/quant_avx2.cpp:74-83).
//
// Data flow: thread 0 issues bulk async copies of the CTA's weight rows into
// shared-memory stages before waiting on the previous kernel (programmatic
// dependent launch), so weight streaming overlaps the predecessor; then the
// prologue builds the quantized activation in shared memory (optionally after
// the embedding lookup and rms_norm), the warps consume the stages, and the
// epilogue applies bias / residual / SiLU*up / argmax.
//
// Wide rows (n_chunks > 1): a stage holds a K-chunk of up to 8 row groups;
// the tiles run chunk by chunk through one pass of rows, and each warp keeps
// its group's lane accumulators across the chunks, so the per-lane block
// order is unchanged.
// ---------------------------------------------------------------------------
template <int NT, int TPR, bool TP>
__global__ void __launch_bounds__(NT, 2) gemv_q8_kernel(const GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int NW = NT / 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t K = p.K;
  const int nb = (int)(K >> 5);
  const int kc = p.kc, n_chunks = p.n_chunks;
  const GemvSmem L = gemv_smem(K, p.rows_per_cta, p.stage_rows, p.n_stages, p.pro, p.stage_x, kc);
  uint64_t* bars = (uint64_t*)smem;
  float* misc = (float*)(smem + 256);
  int8_t* aq = (int8_t*)(smem + L.act_qs);
  float* ad = (float*)(smem + L.act_d);
  float* res = (float*)(smem + L.res);
  float* xs = (float*)(smem + L.xs);
  uint8_t* stages = smem + L.stages;

  const int64_t r0 = (int64_t)blockIdx.x * p.rows_per_cta;
  const int64_t r1 = min(r0 + (int64_t)p.rows_per_cta, p.n_pad);
  const int nrows = (int)(r1 - r0);
  const int n_tiles = (nrows + p.stage_rows - 1) / p.stage_rows * n_chunks;
  const uint8_t* wq = p.w;
  const uint8_t* wd = p.w + p.n_pad * K;

  const uint64_t wpol = l2_evict_first_policy();  // weights are read once per step
  auto issue = [&](int t) {
    const int s = t % p.n_stages;
    const int pass = n_chunks == 1 ? t : t / n_chunks, ch = t - pass * n_chunks;
    const int64_t tr0 = r0 + (int64_t)pass * p.stage_rows;
    const int rows = (int)min((int64_t)p.stage_rows, r1 - tr0);
    uint8_t* st = stages + (size_t)s * L.stage_bytes;
    if (n_chunks == 1) {
      const uint32_t qb = (uint32_t)(rows * K), db = (uint32_t)(rows * nb * 2);
      mbar_arrive_expect_tx(&bars[s], qb + db);
      bulk_load_hint(st, wq + tr0 * K, qb, &bars[s], wpol);
      bulk_load_hint(st + (size_t)p.stage_rows * K, wd + tr0 * nb * 2, db, &bars[s], wpol);
    } else {
      // blocks [c0, c0 + kcb) of each 4-row group: 128 B of quants and 8 B of
      // scales per block, contiguous in the packed layout (nb and kc even keep
      // every copy 16-byte aligned)
      const int c0 = ch * kc, kcb = min(kc, nb - c0), ng = rows >> 2;
      const uint32_t qb = 128u * (uint32_t)kcb, db = 8u * (uint32_t)kcb;
      mbar_arrive_expect_tx(&bars[s], (uint32_t)ng * (qb + db));
      const int64_t g0 = tr0 >> 2;
      uint8_t* sdst = st + (size_t)p.stage_rows * 32 * kc;
      for (int g = 0; g < ng; g++) {
        bulk_load_hint(st + (size_t)g * 128 * kc, wq + (g0 + g) * 4 * K + (int64_t)c0 * 128, qb, &bars[s], wpol);
        bulk_load_hint(sdst + (size_t)g * 8 * kc, wd + ((g0 + g) * nb + c0) * 8, db, &bars[s], wpol);
      }
    }
  };

  // Warp-stream mode (TPR == 0, wide rows): warp w streams the CTA's groups
  // w, w + NW, ... K-chunk by K-chunk through its own ring of S stages (its
  // lane 0 issues the copies), with 8 threads per row; no CTA-wide barrier
  // until the epilogue.
  const int ngroups_cta = nrows >> 2;
  const int active_warps = TPR == 0 ? (int)min((int64_t)NW, ((int64_t)p.rows_per_cta + 3) >> 2) : 1;
  const int S = TPR == 0 ? p.n_stages / active_warps : p.n_stages;
  const int my_tiles = TPR == 0 && ngroups_cta > warp ? (ngroups_cta - warp + NW - 1) / NW * n_chunks : 0;
  uint64_t* wbars = bars + (TPR == 0 ? warp * S : 0);
  uint8_t* wring = stages + (TPR == 0 ? (size_t)warp * S * L.stage_bytes : 0);
  auto wissue = [&](int tau) {
    const int s = tau % S;
    const int gk = n_chunks == 1 ? tau : tau / n_chunks, ch = tau - gk * n_chunks;
    const int64_t G = (r0 >> 2) + warp + (int64_t)gk * NW;
    const int c0 = ch * kc, kcb = min(kc, nb - c0);
    uint8_t* st = wring + (size_t)s * L.stage_bytes;
    mbar_arrive_expect_tx(&wbars[s], 136u * (uint32_t)kcb);
    bulk_load_hint(st, wq + G * 4 * K + (int64_t)c0 * 128, 128u * (uint32_t)kcb, &wbars[s], wpol);
    bulk_load_hint(st + (size_t)128 * kc, wd + (G * nb + c0) * 8, 8u * (uint32_t)kcb, &wbars[s], wpol);
  };

  trace_mark(p.trace, p.trace_slot, 0);
  if (tid == 0) {
    for (int s = 0; s < p.n_stages; s++) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (TPR == 0) {
    if (lane == 0)
      for (int t = 0; t < min(my_tiles, S); t++) wissue(t);
  } else if (tid == 0) {
    for (int t = 0; t < min(n_tiles, p.n_stages); t++) issue(t);
  }
  // Operands that do not depend on the predecessor -- the bias of the CTA's
  // first NT rows, the rms_norm weights of this lane's first four blocks --
  // are loaded before the dependency wait, the residual right after it, so
  // their latency overlaps the wait, the prologue and the chains.
  float pre = 0.0f;
  if (!TP && p.epi == EPI_BIAS && tid < nrows && r0 + tid < p.N) pre = p.bias[r0 + tid];
  float nw[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  if (p.pro >= PRO_NORM_QUANT)
#pragma unroll
    for (int u = 0; u < 4; u++)
      if (warp + u * NW < nb) nw[u] = p.norm_w[(int64_t)(warp + u * NW) * 32 + lane];
  pdl_trigger();
  pdl_wait_cta();
  trace_mark(p.trace, p.trace_slot, 1);
  if (!TP && p.epi == EPI_RESID && tid < nrows && r0 + tid < p.N) pre = p.resid[r0 + tid];

  // ---- prologue: the quantized activation in shared memory ----
  if (TP && p.pro == PRO_ACT && p.act_ll) {
    // Q8_0_ACT blocks as exchange words: word 0 the scale, 1..8 the quants.
    const uint32_t tag = *p.epoch;
    bool dead = false;
    for (int e = tid; e < nb * 9; e += NT) {
      const int b = e / 9, w = e - b * 9;
      const uint32_t v = ll_wait(p.act_ll + e, tag, p.err, dead);
      if (w == 0) ad[b] = __uint_as_float(v);
      else ((uint32_t*)(aq + 32 * b))[w - 1] = v;
    }
  } else if (p.pro == PRO_ACT) {
    for (int b = tid; b < nb; b += NT) {
      const uint8_t* src = p.act + (size_t)b * 36;
      ad[b] = *(const float*)src;
      const uint32_t* sq = (const uint32_t*)(src + 4);
      uint32_t* dq = (uint32_t*)(aq + 32 * b);
#pragma unroll
      for (int k = 0; k < 8; k++) dq[k] = sq[k];
    }
  } else {
    float scale = 1.0f;
    if (p.pro == PRO_EMBED_NORM) {
      // mi_compute_get_rows on the Q8_0 embedding (ref src/ops_cpu.cpp:128-139).
      const int32_t pos = *p.pos;
      int tok = (pos >= 0 && pos < p.tokens_len) ? p.tokens[pos] : -1;
      if (tok < 0 || tok >= p.embed_rows) {
        if (tid == 0) atomicExch(p.err, 1 /* MI_CUDA_ERR_ARG */);
        tok = 0;
      }
      for (int64_t k = tid; k < K; k += NT) {
        const int64_t b = k >> 5;
        const float d = packed_scale(p.embed, K, p.embed_npad, tok, b);
        const float v = __fmul_rn((float)packed_qs(p.embed, K, tok, b)[k & 31], d);
        xs[k] = v;
        if (blockIdx.x == 0) p.x_out[k] = v;
      }
    } else if (TP && p.x_ll) {
      const uint32_t tag = *p.epoch;
      bool dead = false;
      for (int64_t k = tid; k < K; k += NT) xs[k] = __uint_as_float(ll_wait(p.x_ll + k, tag, p.err, dead));
    } else if (p.pro >= PRO_NORM_QUANT || p.stage_x) {
      // All loads of x in flight at once (K is a multiple of 32).
      const float4* x4 = (const float4*)p.x;
      float4* xs4 = (float4*)xs;
      for (int64_t k = tid; k < K / 4; k += NT) xs4[k] = x4[k];
    }
    __syncthreads();
    if (p.pro >= PRO_NORM_QUANT) {
      // mi_compute_rms_norm (ref src/ops_cpu.cpp:154-160): the squares in
      // parallel, then their sum as one ordered chain.
      float* sq = (float*)(smem + L.sq);
      for (int64_t k = tid; k < K; k += NT) sq[k] = __fmul_rn(xs[k], xs[k]);
      __syncthreads();
      const float ss = K <= 1024 ? spec_ordered_sum<NT, 2>(sq, (int)K, smem + L.spec)
                                 : spec_ordered_sum<NT, 4>(sq, (int)K, smem + L.spec);
      if (tid == 0) {
        const float mean = __fdiv_rn(ss, (float)K);
        misc[0] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
      }
      __syncthreads();
      scale = misc[0];
    }
    // One block per warp at a time would serialize the quantizer's two
    // divisions; four independent blocks per iteration overlap them. The
    // warp's blocks are warp + u*NW; the first four use the preloaded norm
    // weights nw[u].
    auto value = [&](int64_t k, float nwk) {
      if (p.pro >= PRO_NORM_QUANT) return __fmul_rn(__fmul_rn(xs[k], scale), nwk);  // rms_norm, then MUL weight
      return p.stage_x ? xs[k] : p.x[k];
    };
    auto nw_at = [&](int64_t k) { return p.pro >= PRO_NORM_QUANT ? p.norm_w[k] : 0.0f; };
    int b = warp;
    for (; b + 3 * NW < nb; b += 4 * NW) {
      float v[4], d[4];
      int8_t q[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int64_t k = (int64_t)(b + u * NW) * 32 + lane;
        v[u] = value(k, b == warp ? nw[u] : nw_at(k));
      }
#pragma unroll
      for (int u = 0; u < 4; u++) q[u] = quantize_lane(v[u], &d[u]);
#pragma unroll
      for (int u = 0; u < 4; u++) {
        aq[(int64_t)(b + u * NW) * 32 + lane] = q[u];
        if (lane == 0) ad[b + u * NW] = d[u];
      }
    }
    if (b == warp) {  // fewer than four blocks for this warp: all preloaded
#pragma unroll
      for (int u = 0; u < 3; u++) {
        if (b + u * NW >= nb) break;
        const int64_t k = (int64_t)(b + u * NW) * 32 + lane;
        float d;
        aq[k] = quantize_lane(value(k, nw[u]), &d);
        if (lane == 0) ad[b + u * NW] = d;
      }
    } else {
      for (; b < nb; b += NW) {
        const int64_t k = (int64_t)b * 32 + lane;
        float d;
        aq[k] = quantize_lane(value(k, nw_at(k)), &d);
        if (lane == 0) ad[b] = d;
      }
    }
  }
  __syncthreads();
  trace_mark(p.trace, p.trace_slot, 2);

  // ---- weight tiles ----
  const int rr = lane >> 3, j = lane & 7;
  const int* aq4 = (const int*)aq;
  bool ok = true;
  float acc_run = 0.0f;  // wide rows: the warp's lane accumulator between K-chunks
  if (TPR == 0) {
    int tau = 0;
    float acc = 0.0f;
    for (; tau < my_tiles; tau++) {
      const int s = tau % S;
      ok = mbar_wait_bounded(&wbars[s], (uint32_t)((tau / S) & 1), p.err);
      if (!__all_sync(FULL, ok)) {
        ok = false;
        break;
      }
      const int gk = n_chunks == 1 ? tau : tau / n_chunks, ch = tau - gk * n_chunks;
      const int c0 = ch * kc, kcb = min(kc, nb - c0);
      const uint8_t* st = wring + (size_t)s * L.stage_bytes;
      const uint32_t* gq = (const uint32_t*)st;
      const __half* gd = (const __half*)(st + (size_t)128 * kc);
      if (ch == 0) acc = 0.0f;
#pragma unroll 4
      for (int i = 0; i < kcb; i++) {
        const int pi = __dp4a((int)gq[i * 32 + lane], aq4[(c0 + i) * 8 + j], 0);
        const float dxdy = __fmul_rn(__half2float(gd[i * 4 + rr]), ad[c0 + i]);
        acc = __fmaf_rn(__int2float_rn(pi), dxdy, acc);
      }
      __syncwarp();
      if (lane == 0 && tau + S < my_tiles) wissue(tau + S);
      if (ch + 1 == n_chunks) {
        const float s4 = __fadd_rn(acc, __shfl_xor_sync(FULL, acc, 4));
        const float s1 = __fadd_rn(s4, __shfl_xor_sync(FULL, s4, 1));
        const float s2 = __fadd_rn(s1, __shfl_xor_sync(FULL, s1, 2));
        if (j == 0) res[(warp + gk * NW) * 4 + rr] = s2;
      }
    }
    if (__syncthreads_or(!ok)) {
      // Copies this warp issued and did not consume get a bounded chance to
      // land before the CTA's shared memory is released.
      if (lane == 0)
        for (int t = tau; t < min(my_tiles, tau + S); t++)
          (void)mbar_wait_bounded(&wbars[t % S], (uint32_t)((t / S) & 1), nullptr);
      return;
    }
  }
  for (int t = 0; TPR != 0 && t < n_tiles; t++) {
    const int s = t % p.n_stages;
    ok = mbar_wait_bounded(&bars[s], (uint32_t)((t / p.n_stages) & 1), p.err);
    if (!__syncthreads_and(ok)) {
      ok = false;
      break;
    }
    const uint8_t* st = stages + (size_t)s * L.stage_bytes;
    const uint32_t* sq = (const uint32_t*)st;
    if (TPR == 8) {
      const int pass = n_chunks == 1 ? t : t / n_chunks, ch = t - pass * n_chunks;
      const int64_t tr0 = r0 + (int64_t)pass * p.stage_rows;
      const int ngroups = (int)(min((int64_t)p.stage_rows, r1 - tr0) >> 2);
      const int c0 = ch * kc, kcb = min(kc, nb - c0);
      const __half* sd = (const __half*)(st + (size_t)p.stage_rows * 32 * kc);
      // 8 threads per row, one lane each; a warp covers one group of 4 rows
      // (with K-chunks at most one, whose accumulator carries to the next chunk).
      for (int g = warp; g < ngroups; g += NW) {
        const uint32_t* gq = sq + (size_t)g * 32 * kc;
        const __half* gd = sd + (size_t)g * 4 * kc;
        const float acc = lane_chain(ch == 0 ? 0.0f : acc_run, gq, gd, aq4 + c0 * 8, ad + c0, kcb, lane, j, rr);
        if (ch + 1 < n_chunks) {
          acc_run = acc;
          continue;
        }
        const float s4 = __fadd_rn(acc, __shfl_xor_sync(FULL, acc, 4));
        const float s1 = __fadd_rn(s4, __shfl_xor_sync(FULL, s4, 1));
        const float s2 = __fadd_rn(s1, __shfl_xor_sync(FULL, s1, 2));
        if (j == 0) res[pass * p.stage_rows + g * 4 + rr] = s2;
      }
    } else {
      // 2 threads per row, lanes 4h..4h+3 each from one 16-byte load; a warp
      // covers 4 groups (16 rows). Thread h=0 ends with l0..l3, its partner
      // (lane ^ 1) with l4..l7. (Whole rows per stage: n_chunks == 1.)
      const int64_t tr0 = r0 + (int64_t)t * p.stage_rows;
      const int ngroups = (int)(min((int64_t)p.stage_rows, r1 - tr0) >> 2);
      const __half* sd = (const __half*)(st + (size_t)p.stage_rows * K);
      const int gw = lane >> 3, r4 = (lane >> 1) & 3, h = lane & 1;
      const uint4* aq16 = (const uint4*)aq;
      for (int g0 = warp * 4; g0 < ngroups; g0 += NW * 4) {
        const int g = g0 + gw;
        const bool valid = g < ngroups;
        const int gc = valid ? g : g0;  // out-of-range groups recompute g0, never store
        const uint4* gq = (const uint4*)(sq + (size_t)gc * K);
        const __half* gd = sd + (size_t)gc * nb * 4;
        float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
#pragma unroll 2
        for (int i = 0; i < nb; i++) {
          const uint4 w = gq[i * 8 + (lane & 7)];
          const uint4 a = aq16[i * 2 + h];
          const float dxdy = __fmul_rn(__half2float(gd[i * 4 + r4]), ad[i]);
          a0 = __fmaf_rn(__int2float_rn(__dp4a((int)w.x, (int)a.x, 0)), dxdy, a0);
          a1 = __fmaf_rn(__int2float_rn(__dp4a((int)w.y, (int)a.y, 0)), dxdy, a1);
          a2 = __fmaf_rn(__int2float_rn(__dp4a((int)w.z, (int)a.z, 0)), dxdy, a2);
          a3 = __fmaf_rn(__int2float_rn(__dp4a((int)w.w, (int)a.w, 0)), dxdy, a3);
        }
        const float s0 = __fadd_rn(a0, __shfl_xor_sync(FULL, a0, 1));
        const float s1 = __fadd_rn(a1, __shfl_xor_sync(FULL, a1, 1));
        const float s2 = __fadd_rn(a2, __shfl_xor_sync(FULL, a2, 1));
        const float s3 = __fadd_rn(a3, __shfl_xor_sync(FULL, a3, 1));
        if (valid && h == 0)
          res[t * p.stage_rows + g * 4 + r4] = __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
      }
    }
    __syncthreads();
    if (tid == 0 && t + p.n_stages < n_tiles) {
      fence_proxy_async_smem();
      issue(t + p.n_stages);
    }
  }
  if (!ok) {
    // Give copies still in flight a bounded chance to land before the CTA's
    // shared memory is released.
    if (tid == 0)
      for (int t = 0; t < min(n_tiles, p.n_stages); t++)
        (void)mbar_wait_bounded(&bars[t], 0u, nullptr);
    return;
  }

  // ---- epilogue ----
  trace_mark(p.trace, p.trace_slot, 3);
  if (p.epi == EPI_SILU_GATEUP_Q) {
    // Each 64 packed rows of the CTA are the gate/up rows of one 32-element
    // block of act: act[a] = silu(gate) * up, then the down projection's
    // quantize node. Warp w handles the CTA's block w.
    if (warp < (nrows >> 6)) {
      const int64_t rb = r0 + 64 * warp;               // the block's first packed row
      const int64_t a = (rb >> 3) * 4 + lane;           // act element of this lane
      const int lr = (int)((a >> 2) * 8 + (a & 3) - r0);  // its gate row, local
      const float v = __fmul_rn(silu_exact(res[lr], p.et), res[lr + 4]);
      float d;
      const int8_t q = quantize_lane(v, &d);
      if (TP && p.out_ll[0]) {
        // the block as 9 exchange words, into every rank's copy
        const uint32_t b0 = (uint8_t)q;
        const uint32_t b1 = __shfl_down_sync(FULL, b0, 1), b2 = __shfl_down_sync(FULL, b0, 2),
                       b3 = __shfl_down_sync(FULL, b0, 3);
        const uint32_t word = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
        const int64_t blk = (p.row0 + rb) >> 6;
        const uint32_t tag = *p.epoch;
        for (int rk = 0; rk < p.n_ranks; rk++) {
          uint64_t* dst = p.out_ll[rk] + blk * 9;
          if (lane == 0) ll_store(dst, __float_as_uint(d), tag);
          if ((lane & 3) == 0) ll_store(dst + 1 + (lane >> 2), word, tag);
        }
      } else {
        uint8_t* blk = p.act_out + (size_t)(rb >> 6) * 36;
        ((int8_t*)blk)[4 + lane] = q;
        if (lane == 0) *(float*)blk = d;
      }
    }
    return;
  }
  if (p.epi == EPI_SILU_GATEUP) {
    for (int lr = tid; lr < nrows; lr += NT) {
      const int64_t r = r0 + lr;
      if ((r & 7) >= 4 || r >= p.N) continue;
      const float g = res[lr], u = res[lr + 4];
      p.out[(r >> 3) * 4 + (r & 7)] = __fmul_rn(silu_exact(g, p.et), u);  // mul(silu(gate), up)
    }
    return;
  }
  if (TP && p.epi != EPI_ARGMAX && p.out_ll[0]) {
    // rows [row0 + r0, ...) of the full vector, into every rank's copy
    const uint32_t tag = *p.epoch;
    bool dead = false;
    for (int lr = tid; lr < nrows; lr += NT) {
      const int64_t r = r0 + lr;
      if (r >= p.N) continue;
      const int64_t g = p.row0 + r;
      float v = res[lr];
      if (p.epi == EPI_BIAS) {
        v = __fadd_rn(v, p.bias[r]);
      } else if (p.epi == EPI_RESID) {
        const float rv = p.resid_ll ? __uint_as_float(ll_wait(p.resid_ll + g, tag, p.err, dead)) : p.resid[g];
        v = __fadd_rn(rv, v);
      }
      for (int rk = 0; rk < p.n_ranks; rk++) ll_store(p.out_ll[rk] + g, __float_as_uint(v), tag);
    }
    return;
  }
  if (p.epi != EPI_ARGMAX) {
    for (int lr = tid; lr < nrows; lr += NT) {
      const int64_t r = r0 + lr;
      if (r >= p.N) continue;
      float v = res[lr];
      if (p.epi == EPI_BIAS) v = __fadd_rn(v, lr == tid ? pre : p.bias[r]);
      else if (p.epi == EPI_RESID) v = __fadd_rn(lr == tid ? pre : p.resid[r], v);
      p.out[r] = v;
    }
    return;
  }

  // EPI_ARGMAX: logits plus mi_qwen2_sample_greedy (ref src/model_qwen2.cpp:690-700):
  // the first index of the maximum.
  float bv = -INFINITY;
  int32_t bi = 0x7fffffff;
  for (int lr = tid; lr < nrows; lr += NT) {
    const int64_t r = r0 + lr;
    if (r >= p.N) continue;
    const float v = res[lr];
    p.out[r] = v;
    if (v > bv || bi == 0x7fffffff) {
      bv = v;
      bi = (int32_t)(TP ? p.row0 + r : r);
    }
  }
  __shared__ float red_v[NW];
  __shared__ int32_t red_i[NW];
  __shared__ uint32_t ticket;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(FULL, bv, o);
    const int32_t oi = __shfl_xor_sync(FULL, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if (lane == 0) {
    red_v[warp] = bv;
    red_i[warp] = bi;
  }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < NW; w++)
      if (red_v[w] > bv || (red_v[w] == bv && red_i[w] < bi)) {
        bv = red_v[w];
        bi = red_i[w];
      }
    p.part_val[blockIdx.x] = bv;
    p.part_idx[blockIdx.x] = bi;
    __threadfence();
    ticket = atomicAdd(p.counter, 1u);
  }
  __syncthreads();
  if (ticket != gridDim.x - 1) return;
  // Last CTA: reduce the per-CTA winners in CTA order.
  if (tid == 0) {
    __threadfence();
    float best = __ldcg(&p.part_val[0]);
    int32_t besti = __ldcg(&p.part_idx[0]);
    for (unsigned c = 1; c < gridDim.x; c++) {
      const float v = __ldcg(&p.part_val[c]);
      const int32_t i = __ldcg(&p.part_idx[c]);
      if (v > best || (v == best && i < besti)) {
        best = v;
        besti = i;
      }
    }
    if (TP && p.out_ll[0]) {
      // This rank's winner to every rank; then the first maximum over the
      // ranks, whose row ranges are in rank order.
      const uint32_t tag = *p.epoch;
      for (int rk = 0; rk < p.n_ranks; rk++) {
        ll_store(p.out_ll[rk] + 2 * p.rank, __float_as_uint(best), tag);
        ll_store(p.out_ll[rk] + 2 * p.rank + 1, (uint32_t)besti, tag);
      }
      const uint64_t* own = p.out_ll[p.rank];
      bool dead = false;
      for (int rk = 0; rk < p.n_ranks; rk++) {
        const float v = __uint_as_float(ll_wait(own + 2 * rk, tag, p.err, dead));
        const int32_t i = (int32_t)ll_wait(own + 2 * rk + 1, tag, p.err, dead);
        if (rk == 0 || v > best || (v == best && i < besti)) {
          best = v;
          besti = i;
        }
      }
      *p.epoch_rw = tag + 1u;
    }
    *p.next_token = besti;
    const int32_t pos = *p.pos_rw;
    if (*p.feedback && pos >= 0 && pos + 1 < p.tokens_len) p.tokens_rw[pos + 1] = besti;
    *p.pos_rw = pos + 1;
    *p.counter = 0u;
  }
}

cudaError_t prepare_attn_kernels(int optin);

GemvPlan plan_gemv(int64_t k, int64_t n, int num_sms, int pro, int32_t rows_per_cta) {
  GemvPlan pl{};
  const int64_t n_pad = (n + 7) / 8 * 8;
  const int64_t nb = k / 32;
  const size_t limit = 220 * 1024;
  pl.threads = 256;
  pl.kc = (int32_t)nb;
  pl.n_chunks = 1;
  if (nb >= 64 && nb % 2 == 0) {
    // Wide rows (K >= 2048). Rows per CTA are a multiple of 4 (one CTA per SM
    // or the caller's count). Default: warp-stream mode (tpr 0), each active
    // warp owning a ring of S stages of one group's K-chunk, S = 3, the chunk
    // as large as shared memory allows. MI_CUDA_GEMV_WIDE="0,S,stage_kb",
    // "8,rows,stage_kb" or "2,rows,stage_kb" picks the mode and shape (tuning
    // sweeps; clamped; mode 2 needs whole rows per stage, else it runs as 8).
    const int64_t groups = n_pad / 4;
    const int64_t target = std::max<int64_t>(1, std::min<int64_t>(num_sms, groups));
    pl.rows_per_cta = rows_per_cta > 0 ? rows_per_cta : (int32_t)((groups + target - 1) / target * 4);
    pl.grid = (int)((n_pad + pl.rows_per_cta - 1) / pl.rows_per_cta);
    int mode = 0, ov_a = 0, ov_kb = 0;
    if (const char* e = std::getenv("MI_CUDA_GEMV_WIDE")) {
      int m = 0, x = 0, kb = 0;
      if (std::sscanf(e, "%d,%d,%d", &m, &x, &kb) == 3 && (m == 0 || m == 8 || m == 2) && x > 0 && kb >= 0) {
        mode = m;
        ov_a = x;
        ov_kb = kb;
      }
    }
    pl.stage_x = 1;
    // Narrow CTAs of moderately wide rows (the 0.5B FFN down projection) keep
    // the shared-stage kernel.
    if (!std::getenv("MI_CUDA_GEMV_WIDE") && pl.rows_per_cta < 16 && nb < 256) mode = 8;
    if (mode == 0) {
      pl.tpr = 0;
      pl.stage_rows = 4;
      const int64_t active = std::min<int64_t>(8, (pl.rows_per_cta + 3) / 4);
      const int64_t S = ov_a > 0 ? std::min(ov_a, 4) : 3;
      for (;;) {
        const int64_t fixed = (int64_t)gemv_smem(k, pl.rows_per_cta, 4, 0, pro, pl.stage_x, 2).total;
        const int64_t per_warp = ((int64_t)limit - fixed) / active;
        int64_t kc = (per_warp / (S * 136) - 1) & ~1;  // 136 B per block, 128-byte stage rounding
        if (ov_kb > 0) kc = std::min<int64_t>(kc, ((int64_t)ov_kb * 1024 / 136) & ~1);
        kc = std::max<int64_t>(2, std::min<int64_t>(nb, kc));
        pl.kc = (int32_t)kc;
        pl.n_chunks = (int32_t)((nb + kc - 1) / kc);
        pl.n_stages = (int32_t)(active * S);
        pl.smem = gemv_smem(k, pl.rows_per_cta, 4, pl.n_stages, pro, pl.stage_x, pl.kc).total;
        if (pl.smem <= limit || !(pl.stage_x && pro == PRO_QUANT)) break;
        pl.stage_x = 0;  // very wide K: quantize from global
      }
      return pl;
    }
    pl.tpr = 8;
    pl.stage_rows = std::min<int32_t>(pl.rows_per_cta, std::max(4, std::min(32, (ov_a > 0 ? ov_a : 32) / 4 * 4)));
    const int64_t stage_bytes = (ov_kb > 0 ? ov_kb : 64) * 1024;
    int64_t kc = std::min<int64_t>(nb, (stage_bytes / (pl.stage_rows * 34)) & ~1);
    if (kc < 2) kc = 2;
    for (;;) {
      pl.kc = (int32_t)kc;
      pl.n_chunks = (int32_t)((nb + kc - 1) / kc);
      const int64_t tiles = (int64_t)(pl.rows_per_cta + pl.stage_rows - 1) / pl.stage_rows * pl.n_chunks;
      pl.n_stages = (int32_t)std::min<int64_t>(tiles, 4);
      for (;;) {
        pl.smem = gemv_smem(k, pl.rows_per_cta, pl.stage_rows, pl.n_stages, pro, pl.stage_x, pl.kc).total;
        if (pl.smem <= limit || pl.n_stages <= 2) break;
        pl.n_stages--;
      }
      if (pl.smem <= limit) break;
      if (pl.stage_x && pro == PRO_QUANT) {
        pl.stage_x = 0;  // very wide K: quantize from global
      } else if (kc > 2) {
        kc = std::max<int64_t>(2, (kc / 2) & ~1);
      } else {
        break;
      }
    }
    if (mode == 2 && pl.n_chunks == 1) pl.tpr = 2;
    return pl;
  }
  const int64_t groups8 = n_pad / 8;
  const int64_t target = std::max<int64_t>(1, std::min<int64_t>(num_sms, groups8));
  pl.rows_per_cta = rows_per_cta > 0 ? rows_per_cta
                                     : (int32_t)(((n_pad + target - 1) / target + 7) / 8 * 8);
  pl.grid = (int)((n_pad + pl.rows_per_cta - 1) / pl.rows_per_cta);
  const int64_t row_bytes = k + k / 32 * 2;
  const int64_t big = 72 * 1024, stream_stage = 62 * 1024;
  int64_t sr = std::max<int64_t>(8, (big / row_bytes) / 8 * 8);
  sr = std::min<int64_t>(sr, pl.rows_per_cta);
  int64_t tiles = (pl.rows_per_cta + sr - 1) / sr;
  if (tiles > 4) {  // streaming (LM head): a ring of stages
    sr = std::max<int64_t>(8, (stream_stage / row_bytes) / 8 * 8);
    tiles = (pl.rows_per_cta + sr - 1) / sr;
  }
  pl.stage_rows = (int32_t)sr;
  // 2 threads per row with 16-byte loads: a quarter of the shared-memory loads
  // of 8 threads per row, and the same code as the other narrow GEMVs of the
  // step (measured faster on B200 even for 8-row CTAs, where only 16 threads
  // of the CTA compute).
  pl.tpr = 2;
  if (const char* e = std::getenv("MI_CUDA_GEMV_TPR")) {
    const int v = std::atoi(e);
    if (v == 2 || v == 8) pl.tpr = v;
  }
  pl.n_stages = (int32_t)std::min<int64_t>(tiles, 4);
  pl.stage_x = 1;
  for (;;) {
    pl.smem = gemv_smem(k, pl.rows_per_cta, pl.stage_rows, pl.n_stages, pro, pl.stage_x, pl.kc).total;
    if (pl.smem <= limit) break;
    if (pl.n_stages > 1) pl.n_stages--;
    else if (pl.stage_x && pro == PRO_QUANT) pl.stage_x = 0;  // very wide K: quantize from global
    else break;
  }
  return pl;
}

namespace {
template <int TPR, bool TP>
cudaError_t set_gemv_smem(int optin) {
  cudaFuncAttributes f{};
  cudaError_t e = cudaFuncGetAttributes(&f, gemv_q8_kernel<256, TPR, TP>);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemv_q8_kernel<256, TPR, TP>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             optin - (int)f.sharedSizeBytes);
  if (e == cudaSuccess) e = set_carveout(gemv_q8_kernel<256, TPR, TP>);
  return e;
}
}  // namespace

cudaError_t prepare_kernels() {
  int dev = 0, optin = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e == cudaSuccess) e = set_gemv_smem<8, false>(optin);
  if (e == cudaSuccess) e = set_gemv_smem<2, false>(optin);
  if (e == cudaSuccess) e = set_gemv_smem<0, false>(optin);
  if (e == cudaSuccess) e = set_gemv_smem<8, true>(optin);
  if (e == cudaSuccess) e = set_gemv_smem<2, true>(optin);
  if (e == cudaSuccess) e = set_gemv_smem<0, true>(optin);
  if (e == cudaSuccess) e = prepare_attn_kernels(optin);
  if (e == cudaSuccess) e = prepare_gemm_kernel();
  if (e == cudaSuccess) e = prepare_gemm_tc_kernel();
  if (e == cudaSuccess) e = prepare_qkv_attn_kernel(optin);
  if (e == cudaSuccess) e = prepare_persist_kernel(optin);
  if (e == cudaSuccess) e = prepare_attn_split_kernels();
  if (e == cudaSuccess) e = prepare_attn_long_kernels(optin);
  return e;
}

// One kernel function serves every prologue/epilogue combination of a thread
// mapping: consecutive GEMVs of a step then run the same code, which is still
// in the SMs' instruction caches (measured: per-variant instantiations made
// the decode step about 2.5% slower).
cudaError_t launch_gemv(const GemvParams& p, const GemvPlan& plan, cudaStream_t s, bool pdl,
                        bool tp) {
  GemvParams q = p;
  q.rows_per_cta = plan.rows_per_cta;
  q.stage_rows = plan.stage_rows;
  q.n_stages = plan.n_stages;
  q.stage_x = plan.stage_x;
  q.kc = plan.kc;
  q.n_chunks = plan.n_chunks;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)plan.grid);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (tp) {
    if (plan.tpr == 0) return cudaLaunchKernelEx(&cfg, gemv_q8_kernel<256, 0, true>, q);
    return plan.tpr == 2 ? cudaLaunchKernelEx(&cfg, gemv_q8_kernel<256, 2, true>, q)
                         : cudaLaunchKernelEx(&cfg, gemv_q8_kernel<256, 8, true>, q);
  }
  if (plan.tpr == 0) return cudaLaunchKernelEx(&cfg, gemv_q8_kernel<256, 0, false>, q);
  if (plan.tpr == 2) return cudaLaunchKernelEx(&cfg, gemv_q8_kernel<256, 2, false>, q);
  return cudaLaunchKernelEx(&cfg, gemv_q8_kernel<256, 8, false>, q);
}

// ---------------------------------------------------------------------------
// Decode attention: MI_OP_ATTN_QK + MI_OP_SOFTMAX + MI_OP_ATTN_KQV for one
// query token (ref src/ops_cpu.cpp:304-410), one CTA per query head, the GQA
// mapping kvh = h / n_rep applied by index (no K/V copy). In executor mode it
// also performs the step's RoPE on q and k (src/ops_cpu.cpp:270-302) and the
// KV-cache append (MI_OP_CPY, src/ops_cpu.cpp:446-460).
//
// K and V are staged through shared memory in chunks of kv_tile positions (K
// rows padded to head_dim + 1 floats so the per-position dot products read
// conflict-free columns). In executor mode the first chunk -- every cached
// position before this step's -- is loaded before the dependency wait, so the
// loads overlap the QKV GEMV. Scores stay in shared memory when they fit.
// Every chain keeps the reference's order: d ascending in QK, the softmax
// denominator over positions in order, t ascending in KV.
// ---------------------------------------------------------------------------
template <bool EXEC, bool SPEC, bool TP>
__global__ void __launch_bounds__(256) attn_decode_kernel(const AttnParams p) {
  extern __shared__ __align__(16) float sm[];
  __shared__ float qr[256], kr[256], vr[256];
  __shared__ float red[8];
  __shared__ float sh[2];
  __shared__ __align__(16) uint8_t spec[SPEC ? spec_sum_scratch_bytes(8, 4) : 16];
  const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int NT = blockDim.x;
  const int D = p.head_dim, half = D >> 1, HKV = p.n_head_kv, D4 = D >> 2;
  const int kvh = h / (p.n_head / HKV);
  const int KT = p.kv_tile, KP = D + 1;
  float* Ks = sm;
  float* Vs = Ks + (size_t)KT * KP;
  float* scs = Vs + (size_t)KT * D;
  const size_t rs = (size_t)HKV * D;
  const float* kbase = p.cache_k + (size_t)kvh * D;
  const float* vbase = p.cache_v + (size_t)kvh * D;

  int n_past, n_kv;
  if (EXEC) {
    // pos was set before this step's graph started and changes only at its end.
    n_past = *p.pos;
    if (n_past < 0 || n_past >= p.n_ctx) {  // no cache row / RoPE entry for this position
      pdl_trigger();
      if (tid == 0) atomicExch(p.err, 6 /* MI_CUDA_ERR_STATE */);
      return;
    }
    n_kv = n_past + 1;
  } else {
    n_kv = p.n_kv_fixed + (int)blockIdx.y;  // batched queries: query t sees n_kv_fixed + t keys
    n_past = n_kv - 1;
  }
  // Rows [c0, c0 + rows) of the cache into the K / V chunk buffers; in executor
  // mode row n_past is this step's and comes from kr / vr instead.
  // Four 16-byte loads in flight per thread before their shared-memory stores.
  auto load_k = [&](int c0, int rows) {
    const int total = rows * D4;
    for (int e0 = tid; e0 < total; e0 += 4 * NT) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int e = e0 + u * NT, r = e / D4, c = e - r * D4;
        if (e < total && !(EXEC && c0 + r == n_past))
          v[u] = *(const float4*)(kbase + (size_t)(c0 + r) * rs + c * 4);
      }
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int e = e0 + u * NT, r = e / D4, c = e - r * D4;
        if (e < total && !(EXEC && c0 + r == n_past)) {
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
    for (int e0 = tid; e0 < total; e0 += 4 * NT) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int e = e0 + u * NT, r = e / D4, c = e - r * D4;
        if (e < total && !(EXEC && c0 + r == n_past))
          v[u] = *(const float4*)(vbase + (size_t)(c0 + r) * rs + c * 4);
      }
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int e = e0 + u * NT, r = e / D4, c = e - r * D4;
        if (e < total && !(EXEC && c0 + r == n_past)) *(float4*)(Vs + (size_t)r * D + c * 4) = v[u];
      }
    }
  };
  const int rows0 = min(KT, n_kv);
  trace_mark(p.trace, p.trace_slot, 0);
  if (EXEC) {
    load_k(0, rows0);
    load_v(0, rows0);
  }
  pdl_trigger();
  pdl_wait_cta();
  trace_mark(p.trace, p.trace_slot, 1);
  if (EXEC) {
    const float2* cs = p.rope_cs + (size_t)n_past * half;
    const size_t qo = (size_t)h * D, ko = (size_t)p.n_head * D + (size_t)kvh * D,
                 vo = (size_t)(p.n_head + HKV) * D + (size_t)kvh * D;
    const float* q = p.qkv + qo;
    const float* k = p.qkv + ko;
    const float* v = p.qkv + vo;
    uint32_t tag = 0u;
    bool dead = false;
    if (TP) tag = *p.epoch;
    for (int i = tid; i < half; i += NT) {
      const float2 c = cs[i];
      float q0, q1, k0, k1;
      if (TP) {
        q0 = __uint_as_float(ll_wait(p.qkv_ll + qo + i, tag, p.err, dead));
        q1 = __uint_as_float(ll_wait(p.qkv_ll + qo + i + half, tag, p.err, dead));
        k0 = __uint_as_float(ll_wait(p.qkv_ll + ko + i, tag, p.err, dead));
        k1 = __uint_as_float(ll_wait(p.qkv_ll + ko + i + half, tag, p.err, dead));
      } else {
        q0 = q[i];
        q1 = q[i + half];
        k0 = k[i];
        k1 = k[i + half];
      }
      qr[i] = __fsub_rn(__fmul_rn(q0, c.x), __fmul_rn(q1, c.y));
      qr[i + half] = __fadd_rn(__fmul_rn(q0, c.y), __fmul_rn(q1, c.x));
      kr[i] = __fsub_rn(__fmul_rn(k0, c.x), __fmul_rn(k1, c.y));
      kr[i + half] = __fadd_rn(__fmul_rn(k0, c.y), __fmul_rn(k1, c.x));
    }
    for (int i = tid; i < D; i += NT)
      vr[i] = TP ? __uint_as_float(ll_wait(p.qkv_ll + vo + i, tag, p.err, dead)) : v[i];
    __syncthreads();
    if (h % (p.n_head / HKV) == 0) {
      float* kd = p.cache_k + ((size_t)n_past * HKV + kvh) * D;
      float* vd = p.cache_v + ((size_t)n_past * HKV + kvh) * D;
      for (int i = tid; i < D; i += NT) {
        kd[i] = kr[i];
        vd[i] = vr[i];
      }
    }
    if (n_past < KT)
      for (int i = tid; i < D; i += NT) {
        Ks[(size_t)n_past * KP + i] = kr[i];
        Vs[(size_t)n_past * D + i] = vr[i];
      }
  } else {
    for (int i = tid; i < D; i += NT) qr[i] = p.q_rot[((size_t)blockIdx.y * p.n_head + h) * D + i];
    load_k(0, rows0);
    load_v(0, rows0);
  }
  __syncthreads();
  trace_mark(p.trace, p.trace_slot, 2);
  float* sc = p.scores_in_smem ? scs : p.scores + (size_t)h * p.scores_stride;
  const int n_chunks = (n_kv + KT - 1) / KT;

  // scores[i] * scale, d ascending with separate roundings (src/ops_cpu.cpp:373-376).
  float lmax = -INFINITY;
  for (int c = 0; c < n_chunks; c++) {
    const int c0 = c * KT, rows = min(KT, n_kv - c0);
    if (c > 0) {
      __syncthreads();
      load_k(c0, rows);
      if (EXEC && n_past >= c0 && n_past < c0 + rows)
        for (int i = tid; i < D; i += NT) Ks[(size_t)(n_past - c0) * KP + i] = kr[i];
      __syncthreads();
    }
    for (int i = tid; i < rows; i += NT) {
      const float acc = ordered_dot(0.0f, Ks + (size_t)i * KP, 1, qr, D);
      const float v = __fmul_rn(acc, p.scale);
      sc[c0 + i] = v;
      lmax = fmaxf(lmax, v);
    }
  }
  trace_mark(p.trace, p.trace_slot, 4);
  lmax = warp_max(lmax);
  if (lane == 0) red[warp] = lmax;
  __syncthreads();
  float mx = red[0];  // every thread reduces the warps' maxima (order-free)
  for (int w = 1; w < (NT >> 5); w++) mx = fmaxf(mx, red[w]);
  for (int i = tid; i < n_kv; i += NT) sc[i] = expf_exact(__fsub_rn(sc[i], mx), p.et);
  __syncthreads();
  trace_mark(p.trace, p.trace_slot, 5);
  // The softmax denominator: one ordered chain (src/ops_cpu.cpp:331-336),
  // evaluated by the whole CTA with spec_ordered_sum when it is long (the SPEC
  // instantiation; the code costs the short-context kernel registers and
  // time even when not taken, so that one leaves it out).
  if (SPEC && p.scores_in_smem && n_kv >= kSpecSumMin) {
    const float sum = n_kv <= 1024 ? spec_ordered_sum<256, 2>(sc, n_kv, spec)
                                   : spec_ordered_sum<256, 4>(sc, n_kv, spec);
    if (tid == 0) sh[1] = __fdiv_rn(1.0f, sum);
  } else if (tid == 0) {
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
  trace_mark(p.trace, p.trace_slot, 6);

  // out[o] = sum_t V[o, kvh, t] * P[t], t ascending (src/ops_cpu.cpp:402-406).
  float acc = 0.0f;
  for (int c = 0; c < n_chunks; c++) {
    const int c0 = c * KT, rows = min(KT, n_kv - c0);
    if (c > 0) {
      __syncthreads();
      load_v(c0, rows);
      if (EXEC && n_past >= c0 && n_past < c0 + rows)
        for (int i = tid; i < D; i += NT) Vs[(size_t)(n_past - c0) * D + i] = vr[i];
      __syncthreads();
    }
    if (tid < D) acc = ordered_dot_scaled(acc, Vs + tid, D, sc + c0, inv, rows);
  }
  trace_mark(p.trace, p.trace_slot, 7);
  trace_mark(p.trace, p.trace_slot, 3);
  if (tid < D && p.out) p.out[((size_t)blockIdx.y * p.n_head + h) * D + tid] = acc;
  if (p.act_qs && tid < D) {
    // Batched queries: this head's outputs quantized into row blockIdx.y of
    // the split Q8_0_ACT layout (the O projection's input).
    float d;
    const int8_t q = quantize_lane(acc, &d);
    const size_t row = (size_t)blockIdx.y * p.n_head * D;
    p.act_qs[row + (size_t)h * D + tid] = q;
    if (lane == 0) p.act_d[(row + (size_t)h * D + tid) >> 5] = d;
  } else if (p.act_out && tid < D) {
    // The O projection's quantize node (src/ops_cpu.cpp:462-479) for this head's
    // outputs: warp w holds block h*D/32 + w of the concatenated heads.
    float d;
    const int8_t q = quantize_lane(acc, &d);
    uint8_t* blk = p.act_out + ((size_t)h * (D >> 5) + (tid >> 5)) * 36;
    ((int8_t*)blk)[4 + lane] = q;
    if (lane == 0) *(float*)blk = d;
  }
}

namespace {
constexpr int kAttnSmemBudget = 140 * 1024;  // dynamic shared memory per CTA (op mode)
// Executor mode: one CTA per head (14 or 28 CTAs), so a larger K/V tile costs
// no concurrency and keeps every position of a decode step in the tile that is
// loaded before the dependency wait (192 positions at head_dim 128).
constexpr int kExecAttnSmemBudget = 210 * 1024;
constexpr int kScoresSmemMax = 8192;         // scores kept on chip up to this many positions
constexpr int kLongMin = 512;                // op mode, one query: attn_long.cu from this many positions
}  // namespace

namespace {
template <bool EXEC, bool SPEC, bool TP>
cudaError_t set_attn_smem(int optin) {
  cudaFuncAttributes f{};
  cudaError_t e = cudaFuncGetAttributes(&f, attn_decode_kernel<EXEC, SPEC, TP>);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attn_decode_kernel<EXEC, SPEC, TP>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             optin - (int)f.sharedSizeBytes);
  if (e == cudaSuccess) e = set_carveout(attn_decode_kernel<EXEC, SPEC, TP>);
  return e;
}
}  // namespace

int g_attn_optin = 0;  // the device's opt-in shared memory per block (set once)

cudaError_t prepare_attn_kernels(int optin) {
  g_attn_optin = optin;
  cudaError_t e = set_attn_smem<true, false, false>(optin);
  if (e == cudaSuccess) e = set_attn_smem<true, false, true>(optin);
  if (e == cudaSuccess) e = set_attn_smem<false, false, false>(optin);
  if (e == cudaSuccess) e = set_attn_smem<false, true, false>(optin);
  return e;
}

cudaError_t launch_attn_decode(const AttnParams& p, bool exec_mode, cudaStream_t s, bool pdl,
                               bool tp, int32_t n_queries) {
  AttnParams q = p;
  // Positions the scores may need: n_ctx in executor mode, n_kv otherwise
  // (of the last query when several are batched).
  const int64_t max_kv = exec_mode ? p.n_ctx : p.n_kv_fixed + std::max(1, n_queries) - 1;
  q.scores_in_smem = max_kv <= kScoresSmemMax ? 1 : 0;
  if (n_queries > 1 && (exec_mode || !q.scores_in_smem)) return cudaErrorInvalidValue;
  const int64_t sc_bytes = q.scores_in_smem ? ((max_kv * 4 + 15) / 16 * 16 + kChainSlackBytes) : 0;
  const int64_t row_bytes = (int64_t)(2 * p.head_dim + 1) * 4;
  // Batched queries launch thousands of CTAs: small K/V tiles keep several
  // of them resident per SM.
  const int64_t budget = n_queries > 1 ? 40 * 1024 + sc_bytes : exec_mode ? kExecAttnSmemBudget : kAttnSmemBudget;
  int64_t kt = (budget - sc_bytes) / row_bytes;
  kt = std::min<int64_t>(256, kt) / 32 * 32;
  if (kt < 32) kt = 32;
  if (n_queries > 1) kt = std::min<int64_t>(kt, 64);
  q.kv_tile = (int32_t)kt;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.n_head, (unsigned)std::max(1, n_queries));
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = (size_t)(kt * row_bytes + sc_bytes);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (exec_mode && tp) return cudaLaunchKernelEx(&cfg, attn_decode_kernel<true, false, true>, q);
  if (exec_mode) return cudaLaunchKernelEx(&cfg, attn_decode_kernel<true, false, false>, q);
  // one query of at least kLongMin positions: the kernels that spread the
  // independent parts over the GPU (attn_long.cu), same order of every sum
  // (one CTA per head walks every position itself: 55 us at 1024 positions,
  // 3 ms at 32768)
  if (n_queries <= 1 && p.n_kv_fixed >= kLongMin && p.out && !p.act_out && !p.act_qs &&
      ((uintptr_t)p.cache_k % 16 == 0) && ((uintptr_t)p.cache_v % 16 == 0) &&
      attn_long_fits(p.head_dim, p.n_head, p.n_head_kv, p.n_kv_fixed, g_attn_optin))
    return launch_attn_decode_long(q, s);
  if (q.scores_in_smem && max_kv >= kSpecSumMin)
    return cudaLaunchKernelEx(&cfg, attn_decode_kernel<false, true, false>, q);
  return cudaLaunchKernelEx(&cfg, attn_decode_kernel<false, false, false>, q);
}

// ---------------------------------------------------------------------------
// Small ops
// ---------------------------------------------------------------------------

// GGUF Q8_0 rows -> packed layout. Source row i goes to packed row
// (i/4)*group_stride + row_offset + i%4 (row_offset a multiple of 4), which
// lets one packed matrix hold Q|K|V stacked or gate/up interleaved by groups.
__global__ void pack_q8_0_kernel(const uint8_t* raw, int64_t K, int64_t n, int64_t src_row0,
                                 uint8_t* dst, int64_t npad, int64_t row_offset, int64_t gstride) {
  const int64_t nb = K / 32;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * nb) return;
  const int64_t i = src_row0 + idx / nb, b = idx % nb;
  const int64_t r = (i >> 2) * gstride + row_offset + (i & 3);
  const uint16_t* src = (const uint16_t*)(raw + idx * 34);
  uint32_t* q = (uint32_t*)(dst + (r >> 2) * 4 * K + b * 128 + (r & 3) * 32);
#pragma unroll
  for (int w = 0; w < 8; w++) q[w] = (uint32_t)src[1 + 2 * w] | ((uint32_t)src[2 + 2 * w] << 16);
  uint16_t* d = (uint16_t*)(dst + npad * K);
  d[((r >> 2) * nb + b) * 4 + (r & 3)] = src[0];
}

cudaError_t launch_pack_q8_0(const uint8_t* raw, int64_t k, int64_t n, int64_t src_row0,
                             uint8_t* dst, int64_t dst_npad, int64_t row_offset,
                             int64_t group_stride, cudaStream_t s) {
  const int64_t total = n * (k / 32);
  if (total == 0) return cudaSuccess;
  pack_q8_0_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(
      raw, k, n, src_row0, dst, dst_npad, row_offset, group_stride);
  return cudaGetLastError();
}

cudaError_t launch_zero_pad_rows(uint8_t* dst, int64_t k, int64_t n_pad, cudaStream_t s) {
  return cudaMemsetAsync(dst, 0, (size_t)(n_pad * k + n_pad * (k / 32) * 2), s);
}

// mi_compute_quantize_q8_0 (src/ops_cpu.cpp:462-479): one warp per block.
__global__ void quantize_act_kernel(const float* x, int64_t K, int64_t m, uint8_t* act) {
  const int64_t nb = K / 32;
  const int64_t blk = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (blk >= m * nb) return;
  const int64_t row = blk / nb, b = blk % nb;
  float d;
  const int8_t q = quantize_lane(x[row * K + b * 32 + lane], &d);
  uint8_t* out = act + (row * nb + b) * 36;
  ((int8_t*)out)[4 + lane] = q;
  if (lane == 0) *(float*)out = d;
}

cudaError_t launch_quantize_act(const float* x, int64_t k, int64_t m, uint8_t* act,
                                cudaStream_t s) {
  const int64_t warps = m * (k / 32);
  if (warps == 0) return cudaSuccess;
  quantize_act_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, s>>>(x, k, m, act);
  return cudaGetLastError();
}

// Per-block int32 sums through the GEMV's lane partials.
__global__ void block_isums_kernel(const uint8_t* w, int64_t K, int64_t n, int64_t npad,
                                   const uint8_t* act, int32_t* isums) {
  const int64_t nb = K / 32;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * nb) return;
  const int64_t r = idx / nb, b = idx % nb;
  const int* wq = (const int*)packed_qs(w, K, r, b);
  const int* aq = (const int*)(act + b * 36 + 4);
  int s = 0;
#pragma unroll
  for (int j = 0; j < 8; j++) s += __dp4a(wq[j], aq[j], 0);
  isums[idx] = s;
}

cudaError_t launch_block_isums(const uint8_t* w, int64_t k, int64_t n, int64_t n_pad,
                               const uint8_t* act, int32_t* isums, cudaStream_t s) {
  const int64_t total = n * (k / 32);
  if (total == 0) return cudaSuccess;
  block_isums_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(w, k, n, n_pad, act, isums);
  return cudaGetLastError();
}

// The reference's scalar dispatch of the Q8_0 x Q8_0_ACT dot, selected there
// by MI_QUANT_FORCE_SCALAR (ref src/quant.cpp:221-230, 232-239): one
// accumulator per row, acc = fma((float)isum_i, fp16(w.d_i) * a.d_i, acc) over
// blocks i in order, isum_i the block's exact int32 sum. One warp per (row,
// column): the lanes form 32 blocks' sums and scale products at a time, then
// every lane runs the chain over them in block order (shuffled from lane t).
__global__ void gemv_q8_scalar_order_kernel(const uint8_t* w, int64_t K, int64_t n, int64_t npad,
                                            const uint8_t* act, float* dst) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t j = blockIdx.y;
  if (r >= n) return;  // whole warps
  const int64_t nb = K / 32;
  const uint8_t* a = act + j * nb * 36;
  float acc = 0.0f;
  for (int64_t b0 = 0; b0 < nb; b0 += 32) {
    int isum = 0;
    float dxdy = 0.0f;
    const int64_t b = b0 + lane;
    if (b < nb) {
      const int* wq = (const int*)packed_qs(w, K, r, b);
      const int* aq = (const int*)(a + b * 36 + 4);
#pragma unroll
      for (int k = 0; k < 8; k++) isum = __dp4a(wq[k], aq[k], isum);
      dxdy = __fmul_rn(packed_scale(w, K, npad, r, b), *(const float*)(a + b * 36));
    }
    const int cnt = (int)min((int64_t)32, nb - b0);
    for (int t = 0; t < cnt; t++) {
      const int is = __shfl_sync(FULL, isum, t);
      const float dx = __shfl_sync(FULL, dxdy, t);
      acc = __fmaf_rn(__int2float_rn(is), dx, acc);
    }
  }
  if (lane == 0) dst[j * n + r] = acc;
}

cudaError_t launch_gemv_scalar_order(const uint8_t* w, int64_t k, int64_t n, int64_t n_pad,
                                     const uint8_t* act, int64_t m, float* dst, cudaStream_t s) {
  if (n == 0 || m == 0) return cudaSuccess;
  const dim3 grid((unsigned)((n + 7) / 8), (unsigned)m);
  gemv_q8_scalar_order_kernel<<<grid, 256, 0, s>>>(w, k, n, n_pad, act, dst);
  return cudaGetLastError();
}

// mi_compute_get_rows on a Q8_0 table (src/ops_cpu.cpp:128-139).
__global__ void get_rows_kernel(const uint8_t* table, int64_t ne0, int64_t npad,
                                const int32_t* ids, int64_t n_ids, float* dst) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n_ids * ne0) return;
  const int64_t j = idx / ne0, k = idx % ne0;
  const int64_t tok = ids[j];
  const float d = packed_scale(table, ne0, npad, tok, k >> 5);
  dst[idx] = __fmul_rn((float)packed_qs(table, ne0, tok, k >> 5)[k & 31], d);
}

cudaError_t launch_get_rows(const uint8_t* table, int64_t ne0, int64_t n_pad,
                            const int32_t* ids, int64_t n_ids, float* dst, cudaStream_t s) {
  const int64_t total = n_ids * ne0;
  if (total == 0) return cudaSuccess;
  get_rows_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(table, ne0, n_pad, ids, n_ids,
                                                                   dst);
  return cudaGetLastError();
}

// mi_compute_rms_norm (src/ops_cpu.cpp:143-165): one CTA per row. Rows that
// fit in shared memory sum their squares with spec_ordered_sum; longer rows
// keep one thread's serial chain.
namespace {
constexpr int64_t kRmsStagedMax = 10240;  // 40 KB of squares + static scratch stay under 48 KB
}

__global__ void __launch_bounds__(256) rms_norm_kernel(const float* x, int64_t ne0, float eps,
                                                       float* dst, int staged) {
  extern __shared__ __align__(16) float sqs[];
  __shared__ __align__(16) uint8_t spec[spec_sum_scratch_bytes(8, 4)];
  __shared__ float scale;
  const float* xr = x + (int64_t)blockIdx.x * ne0;
  if (staged) {
    for (int64_t i = threadIdx.x; i < ne0; i += 256) sqs[i] = __fmul_rn(xr[i], xr[i]);
    __syncthreads();
    const float ss = ne0 <= 1024 ? spec_ordered_sum<256, 2>(sqs, (int)ne0, spec)
                                 : spec_ordered_sum<256, 4>(sqs, (int)ne0, spec);
    if (threadIdx.x == 0) {
      const float mean = __fdiv_rn(ss, (float)ne0);
      scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    }
  } else if (threadIdx.x == 0) {
    float ss = 0.0f;
    for (int64_t i = 0; i < ne0; i++) ss = __fadd_rn(ss, __fmul_rn(xr[i], xr[i]));
    const float mean = __fdiv_rn(ss, (float)ne0);
    scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
  }
  __syncthreads();
  for (int64_t i = threadIdx.x; i < ne0; i += blockDim.x)
    dst[(int64_t)blockIdx.x * ne0 + i] = __fmul_rn(xr[i], scale);
}

cudaError_t launch_rms_norm(const float* x, int64_t ne0, int64_t n_rows, float eps, float* dst,
                            cudaStream_t s) {
  if (n_rows == 0) return cudaSuccess;
  const int staged = ne0 <= kRmsStagedMax ? 1 : 0;
  const size_t smem = staged ? (size_t)ne0 * 4 + kChainSlackBytes : 0;
  rms_norm_kernel<<<(unsigned)n_rows, 256, smem, s>>>(x, ne0, eps, dst, staged);
  return cudaGetLastError();
}

// ew_binop (src/ops_cpu.cpp:56-80): op 0 = mul, 1 = add, 2 = scale by v.
__global__ void binop_kernel(int op, const float* a, const float* b, int64_t ne0, int64_t n_rows,
                             int64_t b_rows, float v, float* dst) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= ne0 * n_rows) return;
  const int64_t r = idx / ne0, i = idx % ne0;
  const float x = a[idx];
  float y;
  if (op == 2) {
    y = __fmul_rn(x, v);
  } else {
    const float bb = b[(b_rows > 1 ? r : 0) * ne0 + i];
    y = op == 0 ? __fmul_rn(x, bb) : __fadd_rn(x, bb);
  }
  dst[idx] = y;
}

cudaError_t launch_binop(int op, const float* a, const float* b, int64_t ne0, int64_t n_rows,
                         int64_t b_rows, float v, float* dst, cudaStream_t s) {
  const int64_t total = ne0 * n_rows;
  if (total == 0) return cudaSuccess;
  binop_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(op, a, b, ne0, n_rows, b_rows, v,
                                                                dst);
  return cudaGetLastError();
}

__global__ void silu_kernel(const float* x, int64_t n, float* dst, const ExpTab et) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = silu_exact(x[i], et);
}

cudaError_t launch_silu(const float* x, int64_t n, float* dst, const ExpTab& et, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  silu_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(x, n, dst, et);
  return cudaGetLastError();
}

__global__ void expf_range_kernel(uint64_t first, int64_t n, float* dst, const ExpTab et) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = expf_exact(__uint_as_float((uint32_t)(first + (uint64_t)i)), et);
}

cudaError_t launch_expf_range(uint64_t first, int64_t count, float* dst, const ExpTab& et,
                              cudaStream_t s) {
  if (count == 0) return cudaSuccess;
  expf_range_kernel<<<(unsigned)((count + 255) / 256), 256, 0, s>>>(first, count, dst, et);
  return cudaGetLastError();
}

__global__ void expf_kernel(const float* x, int64_t n, float* dst, const ExpTab et) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = expf_exact(x[i], et);
}

cudaError_t launch_expf(const float* x, int64_t n, float* dst, const ExpTab& et, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  expf_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(x, n, dst, et);
  return cudaGetLastError();
}

// mi_compute_rope NEOX (src/ops_cpu.cpp:270-302); cs[t][p] holds the (cos, sin)
// of position n_past + t.
__global__ void rope_kernel(const float* x, int64_t hd, int64_t nh, int64_t nt, int32_t n_dims,
                            const float2* cs, float* dst) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= nt * nh * hd) return;
  const int64_t i = idx % hd, row = idx / hd, t = row / nh;
  const int64_t half = n_dims / 2;
  const float* xr = x + row * hd;
  float y;
  if (i >= n_dims) {
    y = xr[i];
  } else {
    const int64_t pp = i < half ? i : i - half;
    const float2 c = cs[t * half + pp];
    const float x0 = xr[pp], x1 = xr[pp + half];
    y = i < half ? __fsub_rn(__fmul_rn(x0, c.x), __fmul_rn(x1, c.y))
                 : __fadd_rn(__fmul_rn(x0, c.y), __fmul_rn(x1, c.x));
  }
  dst[idx] = y;
}

cudaError_t launch_rope(const float* x, int64_t head_dim, int64_t n_head, int64_t n_tokens,
                        int32_t n_dims, const float2* cs, float* dst, cudaStream_t s) {
  const int64_t total = n_tokens * n_head * head_dim;
  if (total == 0) return cudaSuccess;
  rope_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(x, head_dim, n_head, n_tokens,
                                                               n_dims, cs, dst);
  return cudaGetLastError();
}

// mi_compute_attn_qk (src/ops_cpu.cpp:356-380), one thread per (h, j, i).
__global__ void attn_qk_kernel(const float* q, const float* k, int64_t hd, int64_t nh,
                               int64_t nhkv, int64_t n_kv, int64_t nt, float* scores) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= nh * nt * n_kv) return;
  const int64_t i = idx % n_kv, hj = idx / n_kv, j = hj % nt, h = hj / nt;
  const int64_t kvh = h / (nh / nhkv);
  const float* kr = k + (i * nhkv + kvh) * hd;
  const float* qr = q + (j * nh + h) * hd;
  float acc = 0.0f;
  for (int64_t d = 0; d < hd; d++) acc = __fadd_rn(acc, __fmul_rn(kr[d], qr[d]));
  scores[idx] = acc;
}

cudaError_t launch_attn_qk(const float* q, const float* k, int64_t hd, int64_t nh, int64_t nhkv,
                           int64_t n_kv, int64_t nt, float* scores, cudaStream_t s) {
  const int64_t total = nh * nt * n_kv;
  if (total == 0) return cudaSuccess;
  attn_qk_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(q, k, hd, nh, nhkv, n_kv, nt,
                                                                  scores);
  return cudaGetLastError();
}

// mi_compute_softmax (src/ops_cpu.cpp:304-346): one CTA per (h, j) row.
__global__ void softmax_kernel(const float* x, int64_t n_kv, int64_t nt, int32_t n_past,
                               float scale, float* dst, const ExpTab et) {
  __shared__ float red[8];
  __shared__ float sh[2];
  const int64_t row = blockIdx.x, j = row % nt;
  const float* xr = x + row * n_kv;
  float* yr = dst + row * n_kv;
  int64_t allowed = n_past + j + 1;
  if (allowed > n_kv) allowed = n_kv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float m = -INFINITY;
  for (int64_t i = tid; i < allowed; i += blockDim.x) m = fmaxf(m, __fmul_rn(xr[i], scale));
  m = warp_max(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (tid == 0) {
    float mm = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); w++) mm = fmaxf(mm, red[w]);
    sh[0] = mm;
  }
  __syncthreads();
  const float mx = sh[0];
  for (int64_t i = tid; i < allowed; i += blockDim.x)
    yr[i] = expf_exact(__fsub_rn(__fmul_rn(xr[i], scale), mx), et);
  __syncthreads();
  if (tid == 0) {
    float sum = 0.0f;
    for (int64_t i = 0; i < allowed; i++) sum = __fadd_rn(sum, yr[i]);
    sh[1] = __fdiv_rn(1.0f, sum);
  }
  __syncthreads();
  const float inv = sh[1];
  for (int64_t i = tid; i < n_kv; i += blockDim.x) yr[i] = i < allowed ? __fmul_rn(yr[i], inv) : 0.0f;
}

cudaError_t launch_softmax(const float* x, int64_t n_kv, int64_t nt, int64_t nh, int32_t n_past,
                           float scale, float* dst, const ExpTab& et, cudaStream_t s) {
  if (nt * nh == 0) return cudaSuccess;
  softmax_kernel<<<(unsigned)(nt * nh), 256, 0, s>>>(x, n_kv, nt, n_past, scale, dst, et);
  return cudaGetLastError();
}

// mi_compute_attn_kqv (src/ops_cpu.cpp:386-410), one thread per (h, o, j).
__global__ void attn_kqv_kernel(const float* pr, const float* v, int64_t hd, int64_t nh,
                                int64_t nhkv, int64_t n_kv, int64_t nt, float* dst) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= nh * hd * nt) return;
  const int64_t o = idx % hd, hj = idx / hd, h = hj % nh, j = hj / nh;
  const int64_t kvh = h / (nh / nhkv);
  const float* p = pr + (h * nt + j) * n_kv;
  float acc = 0.0f;
  for (int64_t t = 0; t < n_kv; t++) acc = __fadd_rn(acc, __fmul_rn(v[(t * nhkv + kvh) * hd + o], p[t]));
  dst[idx] = acc;
}

cudaError_t launch_attn_kqv(const float* p, const float* v, int64_t hd, int64_t nh, int64_t nhkv,
                            int64_t n_kv, int64_t nt, float* dst, cudaStream_t s) {
  const int64_t total = nh * hd * nt;
  if (total == 0) return cudaSuccess;
  attn_kqv_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(p, v, hd, nh, nhkv, n_kv, nt,
                                                                   dst);
  return cudaGetLastError();
}

// First index of the maximum: per-CTA winners, the last CTA reduces them.
__global__ void argmax_kernel(const float* x, int64_t n, float* part_val, int32_t* part_idx,
                              uint32_t* counter, int32_t* out) {
  __shared__ float rv[8];
  __shared__ int32_t ri[8];
  __shared__ uint32_t ticket;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float bv = -INFINITY;
  int32_t bi = 0x7fffffff;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + tid; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    if (v > bv || bi == 0x7fffffff) {
      bv = v;
      bi = (int32_t)i;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(FULL, bv, o);
    const int32_t oi = __shfl_xor_sync(FULL, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if (lane == 0) {
    rv[warp] = bv;
    ri[warp] = bi;
  }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); w++)
      if (rv[w] > bv || (rv[w] == bv && ri[w] < bi)) {
        bv = rv[w];
        bi = ri[w];
      }
    part_val[blockIdx.x] = bv;
    part_idx[blockIdx.x] = bi;
    __threadfence();
    ticket = atomicAdd(counter, 1u);
  }
  __syncthreads();
  if (ticket != gridDim.x - 1 || tid != 0) return;
  __threadfence();
  float best = __ldcg(&part_val[0]);
  int32_t besti = __ldcg(&part_idx[0]);
  for (unsigned c = 1; c < gridDim.x; c++) {
    const float v = __ldcg(&part_val[c]);
    const int32_t i = __ldcg(&part_idx[c]);
    if (v > best || (v == best && i < besti)) {
      best = v;
      besti = i;
    }
  }
  *out = besti;
  *counter = 0u;
}

cudaError_t launch_argmax(const float* x, int64_t n, float* part_val, int32_t* part_idx,
                          uint32_t* counter, int32_t* out, cudaStream_t s) {
  if (n <= 0) return cudaErrorInvalidValue;
  const int64_t g = std::min<int64_t>(148, (n + 255) / 256);
  argmax_kernel<<<(unsigned)g, 256, 0, s>>>(x, n, part_val, part_idx, counter, out);
  return cudaGetLastError();
}

__global__ void advance_kernel(int32_t* pos, uint32_t* epoch) {
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x == 0) {
    *pos += 1;
    if (epoch) *epoch += 1u;
  }
}

cudaError_t launch_advance(int32_t* pos, cudaStream_t s, bool pdl, uint32_t* epoch) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(32);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, advance_kernel, pos, epoch);
}

__global__ void set_pos_kernel(int32_t* pos, int32_t value) {
  if (threadIdx.x == 0) *pos = value;
}

cudaError_t launch_set_pos(int32_t* pos, int32_t value, cudaStream_t s) {
  set_pos_kernel<<<1, 32, 0, s>>>(pos, value);
  return cudaGetLastError();
}

}  // namespace mi
