// Persistent decode step (sm_100a, one GPU): the whole decode step -- every
// layer and the LM head -- as ONE kernel launch whose CTAs stay resident.
//
// Same operations in the same order as the kernel-per-phase step graph
// (qwen2_exec.cu, with qkv_attn.cu and gemv_q8_kernel), so the logits are
// bit-identical to it and to the reference's AVX2 path: rms_norm as one
// ordered chain (src/ops_cpu.cpp:154-160), the Q8_0_ACT quantizer
// (src/quant.cpp:199-218), the Q8_0 dot with the AVX2 lane order
// (src/quant_avx2.cpp:170-181), RoPE, KV append, attention
// (src/ops_cpu.cpp:270-410), SiLU * up, greedy argmax
// (src/model_qwen2.cpp:690-700).
//
// What changes is the schedule. A step of the 0.5B shape is ~100 dependent
// phases of a few microseconds each; as separate kernels every phase pays a
// launch hand-off, and code that runs once per launch is fetched cold. Here:
//  * CTAs [0, n_attn) are the attention CTAs, ONE thread-block cluster of
//    n_kv_head * (n_rep + 1) CTAs (per KV head n_rep query CTAs + one k/v CTA;
//    16 for the 0.5B shape, a non-portable cluster size): per layer rms_norm
//    + quantize, their Q|K|V rows, RoPE, the k/v hand-over through
//    distributed shared memory, the KV append, the decode attention of one
//    head and its quantize (the O projection's input node). Each head's
//    Q8_0_ACT blocks go into every cluster CTA's shared memory (st.async,
//    counted on an mbarrier), so the whole cluster then runs the O
//    projection (+ residual) on its own, each CTA its rows, with no grid-wide
//    hand-over between attention and O.
//  * the other n_gemv CTAs run, per layer, the FFN gate/up (rms_norm +
//    quantize prologue, SiLU * up + quantize epilogue) and the down
//    projection (+ residual), each CTA its own rows; then the LM head and its
//    argmax.
//  * phases hand over through monotonic device counters (one per layer and
//    phase): a producer CTA's threads store their outputs, the CTA
//    synchronizes, one thread increments with release semantics; a consumer's thread 0
//    polls with acquire loads until the count of this step is reached. Every
//    poll is bounded (kSpinLimit) and records MI_CUDA_ERR_TIMEOUT on expiry.
//  * every CTA streams the weights of its coming work items, in order, into
//    a ring in shared memory with bulk async copies (one mbarrier per item),
//    so weights arrive ahead of the phases that need them.
//
// FAST = true is a labelled fast mode (not bit-identical to the reference,
// never reported as parity): the same schedule and hand-overs, but the sums
// the reference computes as sequential chains are regrouped -- rms_norm's sum
// of squares and the softmax denominator as block trees, the attention value
// sums split over thread groups, the QK dots as four interleaved chains, the
// down projection's 152-block lane chains split over the CTA's warps -- and
// the softmax uses CUDA's expf.
#include <algorithm>
#include <cstdlib>

#include "mi_device.cuh"

namespace mi {

namespace {

constexpr unsigned FULL = 0xffffffffu;
constexpr int kNT = 256, kNW = kNT / 32;
constexpr int kQ = 16;               // ring items in flight per CTA (one mbarrier each)
constexpr int kHeadChunkGroups = 16;  // LM-head rows per ring item: 16 groups of 4
constexpr int kMaxRes = 256;          // rows of one work item
constexpr int kScoresOnChipMax = 8192;
// The thread that owns the weight ring (issues its bulk copies). Issuing a
// bulk copy holds the thread while the SM's copy engine is busy with earlier
// copies (~0.5 us per 64 KB item in the LM head); moving the issue to a thread
// of another warp only moved that time into the ring waits and slowed the
// layers by ~2 us each on B200, so thread 0 issues, after the CTA's signal.
constexpr int kIssuer = 0;


__host__ __device__ inline size_t up16(size_t v) { return (v + 15) / 16 * 16; }
__host__ __device__ inline size_t up128(size_t v) { return (v + 127) / 128 * 128; }

// Bytes of G row groups (4 rows each) of a packed matrix with K columns in the
// ring: the groups' quants, then their fp16 scales.
__host__ __device__ inline size_t groups_bytes(int G, int64_t K) {
  return up128((size_t)G * 4 * (size_t)K + (size_t)G * (size_t)(K / 32) * 8);
}

// Dynamic shared memory, identical on host and device: [0,256) mbarriers,
// [256,512) ring bookkeeping, then the activation region, then the weight
// ring; query CTAs add the K / V tiles and the scores after their ring.
struct PSmem {
  size_t lay, aq, ad, xs, sq, spec, res, oq, od, ring, total;
};
constexpr int kMaxLayers = 128;
__host__ __device__ inline PSmem persist_smem(int64_t E, int64_t FF, int n_layer) {
  PSmem L;
  size_t off = 512;
  L.lay = off;  // the layers' weight pointers (read by the ring's issue logic)
  off += up16((size_t)n_layer * sizeof(PersistLayer));
  const int64_t KM = E > FF ? E : FF;
  L.aq = off;
  off += up16((size_t)KM);
  L.ad = off;
  off += up16((size_t)(KM / 32) * 4);
  L.xs = off;
  off += (size_t)E * 4;
  L.sq = off;
  off += (size_t)E * 4 + kChainSlackBytes;
  L.spec = off;
  off += up16((size_t)spec_sum_scratch_bytes(kNW, 2));
  L.res = off;
  off += (size_t)kMaxRes * 4;
  L.oq = off;  // attention CTAs: the O projection's Q8_0_ACT input, from every head
  off += up16((size_t)E);
  L.od = off;
  off += up16((size_t)(E / 32) * 4);
  L.ring = up128(off);
  L.total = L.ring;
  return L;
}

struct Role {
  bool attn, kv;
  int h, kvh;
  int o_g0, o_g1;    // O rows (attention CTAs) or down rows (projection CTAs), in groups of 4
  int gu_b0, gu_b1;  // FFN activation blocks (64 packed gate/up rows each)
  int hd_g0, hd_g1;  // LM-head row groups
  int n_main;        // items before the LM head
  int n_items;
};

struct ItemDesc {
  const uint8_t* w;  // packed matrix
  int64_t K, npad;
  int g0[2], G[2];   // up to two group ranges
  int n;
};

__device__ inline ItemDesc item_desc(const PersistParams& p, const PersistLayer* lay, const Role& r, int it) {
  ItemDesc d{};
  d.n = 1;
  if (it < r.n_main) {
    const int l = it >> 1, kind = it & 1;  // two items a layer
    const PersistLayer& L = lay[l];
    if (r.attn && kind == 1) {
      d.w = L.o;
      d.K = p.E;
      d.npad = p.E;
      d.g0[0] = r.o_g0;
      d.G[0] = r.o_g1 - r.o_g0;
    } else if (r.attn) {
      d.w = L.qkv;
      d.K = p.E;
      d.npad = p.qkv_npad;
      const int gd = p.D / 4;
      if (r.kv) {
        d.n = 2;
        d.g0[0] = (p.E + r.kvh * p.D) / 4;
        d.G[0] = gd;
        d.g0[1] = (p.E + p.HKV * p.D + r.kvh * p.D) / 4;
        d.G[1] = gd;
      } else {
        d.g0[0] = r.h * gd;
        d.G[0] = gd;
      }
    } else {
      if (kind == 0) {
        d.w = L.gateup;
        d.K = p.E;
        d.npad = p.gu_npad;
        d.g0[0] = 16 * r.gu_b0;
        d.G[0] = 16 * (r.gu_b1 - r.gu_b0);
      } else {
        d.w = L.down;
        d.K = p.FF;
        d.npad = p.E;
        d.g0[0] = r.o_g0;
        d.G[0] = r.o_g1 - r.o_g0;
      }
    }
  } else {
    const int c = it - r.n_main;
    d.w = p.head;
    d.K = p.E;
    d.npad = p.head_npad;
    d.g0[0] = r.hd_g0 + c * kHeadChunkGroups;
    d.G[0] = max(0, min(kHeadChunkGroups, r.hd_g1 - d.g0[0]));
  }
  return d;
}

__device__ inline uint32_t item_bytes(const ItemDesc& d) {
  uint32_t b = 0;
  for (int i = 0; i < d.n; i++) b += (uint32_t)groups_bytes(d.G[i], d.K);
  return b;
}

// Ring bookkeeping in shared memory (kIssuer writes, every thread reads the
// offsets after the item's mbarrier completes).
struct RingState {
  uint32_t head, tail;  // monotonic byte positions (issued / freed)
  int32_t next, freed;  // next item to issue, items freed
  uint32_t off[kQ], end[kQ];
};

__device__ inline unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ inline void pstamp(const PersistParams& p, int slot, int point) {
  if (p.trace) p.trace[(size_t)slot * kTracePoints + point] = globaltimer_ns();
}

template <bool FAST>
__global__ void __launch_bounds__(kNT, 1) persist_step_kernel(const PersistParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(16) float qr[128], kr[128], vr[128];
  __shared__ float red_f[kNW], red_s[kNW];
  __shared__ int32_t red_i[kNW];
  __shared__ float misc[4];
  __shared__ int s_dead;
  __shared__ uint32_t s_ticket;
  __shared__ __align__(16) int8_t ostage_q[128];  // a query CTA's head output, quantized
  __shared__ float ostage_d[4];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cta = (int)blockIdx.x, G = (int)gridDim.x;
  const int E = p.E, D = p.D, HKV = p.HKV, FF = p.FF;
  const int n_rep = p.H / HKV, CK = n_rep + 1;  // CTAs per KV head
  const int nbE = E / 32, nbF = FF / 32;
  const PSmem L = persist_smem(E, FF, p.n_layer);
  uint64_t* bars = (uint64_t*)smem;      // kQ ring barriers
  uint64_t* bar_kv = bars + kQ;          // query CTAs: k / v from the k/v CTA
  uint64_t* bar_o = bars + kQ + 1;       // attention CTAs: every head's output (the O input)
  RingState* rs = (RingState*)(smem + 256);
  int8_t* aq = (int8_t*)(smem + L.aq);
  float* ad = (float*)(smem + L.ad);
  float* xs = (float*)(smem + L.xs);
  float* sq = (float*)(smem + L.sq);
  float* res = (float*)(smem + L.res);
  int8_t* oq = (int8_t*)(smem + L.oq);
  float* od = (float*)(smem + L.od);
  uint8_t* ring = smem + L.ring;
  PersistLayer* lay = (PersistLayer*)(smem + L.lay);
  for (int i = tid; i < p.n_layer * (int)(sizeof(PersistLayer) / 8); i += kNT)
    ((uint64_t*)lay)[i] = ((const uint64_t*)p.layers)[i];

  // ---- role and work ranges ----
  Role r{};
  r.attn = cta < p.n_attn;
  const int W = p.n_gemv;
  if (r.attn) {
    r.kvh = cta / CK;
    const int c = cta - r.kvh * CK;
    r.kv = c == n_rep;
    r.h = r.kvh * n_rep + c;
    const int GO = E / 4;
    r.o_g0 = (int)((int64_t)cta * GO / p.n_attn);
    r.o_g1 = (int)((int64_t)(cta + 1) * GO / p.n_attn);
    r.n_main = 2 * p.n_layer;
    r.n_items = r.n_main;
  } else {
    const int wi = cta - p.n_attn;
    const int GO = E / 4, GV = (int)(p.head_npad / 4);
    r.o_g0 = (int)((int64_t)wi * GO / W);
    r.o_g1 = (int)((int64_t)(wi + 1) * GO / W);
    r.gu_b0 = (int)((int64_t)wi * nbF / W);
    r.gu_b1 = (int)((int64_t)(wi + 1) * nbF / W);
    r.hd_g0 = (int)((int64_t)wi * GV / W);
    r.hd_g1 = (int)((int64_t)(wi + 1) * GV / W);
    r.n_main = 2 * p.n_layer;
    r.n_items = r.n_main + (p.with_head ? (r.hd_g1 - r.hd_g0 + kHeadChunkGroups - 1) / kHeadChunkGroups : 0);
  }
  const bool query = r.attn && !r.kv;
  // ring bytes: the whole space after the activation region, except in query
  // CTAs, whose K / V tiles and scores follow a ring of ring_attn bytes
  const uint32_t R = query ? (uint32_t)p.ring_attn : (uint32_t)p.ring_gemv;
  const int KT = p.kv_tile, KP = D + 1;
  float* Ks = (float*)(ring + p.ring_attn);
  float* Vs = Ks + (size_t)KT * KP;
  float* scs = Vs + (size_t)KT * D;

  const int n_past = *p.pos;
  if (n_past < 0 || n_past >= p.n_ctx) {  // every CTA reads the same pos
    if (tid == 0 && cta == 0) atomicExch(p.err, 6 /* MI_CUDA_ERR_STATE */);
    return;
  }
  const int n_kv = n_past + 1;
  const unsigned long long epoch = *p.epoch;
  const int tr_attn = cta == 0 && tid == 0, tr_gemv = cta == p.n_attn && tid == 0;

  if (tid == 0) {
    for (int i = 0; i <= kQ + 1; i++) mbar_init(&bars[i], 1);
    fence_mbar_init();
    rs->head = rs->tail = 0u;
    rs->next = rs->freed = 0;
    s_dead = 0;
  }
  __syncthreads();
  // cluster phase: every CTA's barriers are initialized before any k/v CTA
  // stores into a peer's shared memory
  cluster_arrive_relaxed();
  cluster_wait_acquire();

  // ---- weight ring (thread 0) ----
  const uint64_t wpol = l2_evict_first_policy();  // weights are read once per step
  auto issue_more = [&]() {
    fence_proxy_async_smem();
    while (rs->next < r.n_items && rs->next - rs->freed < kQ) {
      const ItemDesc d = item_desc(p, lay, r, rs->next);
      const uint32_t bytes = item_bytes(d);
      const uint32_t off0 = rs->head % R;
      const uint32_t pad = off0 + bytes > R ? R - off0 : 0u;
      if (rs->head + pad + bytes - rs->tail > R) break;
      rs->head += pad;
      const uint32_t off = rs->head % R;
      const int slot = rs->next % kQ;
      rs->off[slot] = off;
      rs->end[slot] = rs->head + bytes;
      uint32_t tx = 0;
      for (int i = 0; i < d.n; i++)
        tx += (uint32_t)(d.G[i] * 4 * d.K + d.G[i] * (d.K / 32) * 8);
      mbar_arrive_expect_tx(&bars[slot], tx);
      uint32_t o = off;
      for (int i = 0; i < d.n; i++) {
        if (d.G[i] > 0) {
          const uint32_t qb = (uint32_t)(d.G[i] * 4 * d.K), db = (uint32_t)(d.G[i] * (d.K / 32) * 8);
          bulk_load_hint(ring + o, d.w + (int64_t)d.g0[i] * 4 * d.K, qb, &bars[slot], wpol);
          bulk_load_hint(ring + o + qb, d.w + d.npad * d.K + (int64_t)d.g0[i] * (d.K / 32) * 8, db, &bars[slot],
                         wpol);
        }
        o += (uint32_t)groups_bytes(d.G[i], d.K);
      }
      rs->head += bytes;
      rs->next++;
    }
  };
  // Waits for item `it` (every thread); returns its ring address.
  auto wait_item = [&](int it) -> const uint8_t* {
    const int slot = it % kQ;
    if (!s_dead && !mbar_wait_bounded(&bars[slot], (uint32_t)((it / kQ) & 1), p.err)) s_dead = 1;
    return ring + rs->off[slot];
  };
  // After every thread is done with item `it` (the caller has synchronized
  // the CTA since its last read of it): frees it and issues more.
  // After a time-out the CTA stops issuing and keeps the item unfreed, so the
  // drain at the end of the kernel still waits (bounded) for its copies and
  // no mbarrier is re-armed while a copy counted on it may be in flight.
  auto free_item = [&](int it) {
    if (tid == kIssuer && !s_dead) {
      rs->tail = rs->end[it % kQ];
      rs->freed = it + 1;
      issue_more();
    }
  };
  if (tid == kIssuer) issue_more();

  // ---- hand-over counters ----
  auto wait_ctr = [&](const unsigned long long* c, unsigned long long target) {
    if (tid == 0 && !s_dead) {
      uint32_t it = 0;
      while (ld_acquire_u64(c) < target) {
        if (++it >= kSpinLimit || ((it & 1023u) == 0 && *(volatile int32_t*)p.err != 0)) {
          atomicExch(p.err, 5 /* MI_CUDA_ERR_TIMEOUT */);
          s_dead = 1;
          break;
        }
      }
    }
    __syncthreads();
  };
  // After the CTA barrier, one release add publishes every thread's stores
  // made before it (the barrier orders them before thread 0's release).
  auto signal_ctr = [&](unsigned long long* c) {
    __syncthreads();
    if (tid == 0) {
      asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(c), "l"(1ull) : "memory");
    }
  };

  // ---- building blocks ----
  // x (coherent loads from L2; or the embedding row) -> xs; rms_norm with
  // norm_w; quantized into aq / ad (src/ops_cpu.cpp:154-160, 462-479).
  // nw: this lane's norm weights of blocks warp + u * kNW (load_nw), loaded
  // before the caller's wait so their latency overlaps it.
  auto load_nw = [&](const float* norm_w, float (&nw)[4]) {
#pragma unroll
    for (int u = 0; u < 4; u++) nw[u] = warp + u * kNW < nbE ? norm_w[(warp + u * kNW) * 32 + lane] : 0.0f;
  };
  auto norm_quant = [&](const float* x, bool embed, const float (&nw)[4]) {
    if (embed) {
      // mi_compute_get_rows on the Q8_0 embedding (ref src/ops_cpu.cpp:128-139)
      int tok = n_past < p.tokens_len ? p.tokens[n_past] : -1;
      if (tok < 0 || tok >= p.V) {
        if (tid == 0) atomicExch(p.err, 1 /* MI_CUDA_ERR_ARG */);
        tok = 0;
      }
      for (int k = tid; k < E; k += kNT) {
        const float v = __fmul_rn((float)packed_qs(p.embed, E, tok, k >> 5)[k & 31],
                                  packed_scale(p.embed, E, p.embed_npad, tok, k >> 5));
        xs[k] = v;
        if (!FAST) sq[k] = __fmul_rn(v, v);
      }
    } else {
      // x, and (exact mode) its squares for the ordered sum, from the same registers
      for (int k = tid; k < E / 4; k += kNT) {
        const float4 v = __ldcg((const float4*)x + k);
        ((float4*)xs)[k] = v;
        if (!FAST)
          ((float4*)sq)[k] = make_float4(__fmul_rn(v.x, v.x), __fmul_rn(v.y, v.y), __fmul_rn(v.z, v.z),
                                         __fmul_rn(v.w, v.w));
      }
    }
    __syncthreads();
    float scale;
    if constexpr (FAST) {
      // fast mode: the sum of squares as a block tree
      float part = 0.0f;
      for (int k = tid; k < E; k += kNT) part = fmaf(xs[k], xs[k], part);
      part = warp_sum_tree(part);
      if (lane == 0) red_s[warp] = part;
      __syncthreads();
      float ss = 0.0f;
#pragma unroll
      for (int w = 0; w < kNW; w++) ss += red_s[w];
      scale = rsqrtf(ss / (float)E + p.eps);
    } else {
      const float ss = spec_ordered_sum<kNT, 2>(sq, E, smem + L.spec);
      if (tid == 0) misc[0] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)E), p.eps)));
      __syncthreads();
      scale = misc[0];
    }
    // four blocks per warp at once overlap the quantizer's divisions
    float v[4], d[4];
    int8_t q[4];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int b = warp + u * kNW;
      v[u] = b < nbE ? __fmul_rn(__fmul_rn(xs[b * 32 + lane], scale), nw[u]) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < 4; u++) q[u] = quantize_lane(v[u], &d[u]);
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int b = warp + u * kNW;
      if (b < nbE) {
        aq[b * 32 + lane] = q[u];
        if (lane == 0) ad[b] = d[u];
      }
    }
    __syncthreads();
  };
  // Fast mode: the down projection's rows with each row's blocks split over
  // the CTA's warps (warp w takes blocks [w nb / kNW, (w+1) nb / kNW) of every
  // group; lanes as rows_8t), partials summed through shared memory (sq).
  // Needs Gt * 4 * kNW <= E floats of scratch: rows_8t otherwise.
  auto rows_8t_split = [&](const uint8_t* base, const ItemDesc& d) {
    const int K = (int)d.K, nb = K / 32, Gt = d.G[0];
    const int rr = lane >> 3, j = lane & 7;
    const int b0 = warp * nb / kNW, b1 = (warp + 1) * nb / kNW;
    for (int g = 0; g < Gt; g++) {
      const uint32_t* gq = (const uint32_t*)(base + (size_t)g * 4 * K) + (size_t)b0 * 32;
      const __half* gd = (const __half*)(base + (size_t)Gt * 4 * K) + (size_t)g * nb * 4 + (size_t)b0 * 4;
      float acc = lane_chain(0.0f, gq, gd, (const int*)aq + b0 * 8, ad + b0, b1 - b0, lane, j, rr);
      acc += __shfl_xor_sync(FULL, acc, 4);
      acc += __shfl_xor_sync(FULL, acc, 1);
      acc += __shfl_xor_sync(FULL, acc, 2);
      if (j == 0) sq[warp * Gt * 4 + g * 4 + rr] = acc;
    }
    __syncthreads();
    for (int i = tid; i < Gt * 4; i += kNT) {
      float s = 0.0f;
#pragma unroll
      for (int w = 0; w < kNW; w++) s += sq[w * Gt * 4 + i];
      res[i] = s;
    }
    __syncthreads();
  };
  // Q8_0_ACT blocks from global memory (coherent loads) into aq / ad: eight
  // loads per thread in flight before any is stored (one L2 round trip for
  // the down projection's 1368 words, where a load-store loop measured
  // ~0.6 us slower).
  auto load_act = [&](const uint8_t* g, int nb) {
    const uint32_t* w = (const uint32_t*)g;
    const int n = nb * 9;
    for (int base = 0; base < n; base += 8 * kNT) {
      uint32_t v[8];
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const int e = base + u * kNT + tid;
        v[u] = e < n ? __ldcg(w + e) : 0u;
      }
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const int e = base + u * kNT + tid;
        if (e < n) {
          const int b = e / 9, k = e - b * 9;
          if (k == 0) ad[b] = __uint_as_float(v[u]);
          else ((uint32_t*)(aq + 32 * b))[k - 1] = v[u];
        }
      }
    }
    __syncthreads();
  };
  // Rows of an item, 2 threads per row, against the Q8_0_ACT vector a_q / a_d
  // (K elements): res[4g + r] = dot(row, act), the AVX2 lane order.
  auto rows_2t = [&](const uint8_t* base, const ItemDesc& d, const int8_t* a_q, const float* a_d) {
    const int K = (int)d.K, nb = K / 32, Gt = d.G[0] + (d.n > 1 ? d.G[1] : 0);
    const int gw = lane >> 3, r4 = (lane >> 1) & 3, hh = lane & 1;
    const uint4* aq16 = (const uint4*)a_q;
    for (int g0 = warp * 4; g0 < Gt; g0 += kNW * 4) {
      const int g = g0 + gw;
      const bool valid = g < Gt;
      int gc = valid ? g : g0;
      const uint8_t* rb = base;
      int Gr = d.G[0];
      if (gc >= d.G[0]) {
        rb = base + groups_bytes(d.G[0], d.K);
        gc -= d.G[0];
        Gr = d.G[1];
      }
      const uint4* gq = (const uint4*)(rb + (size_t)gc * 4 * K);
      const __half* gd = (const __half*)(rb + (size_t)Gr * 4 * K) + (size_t)gc * nb * 4;
      float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
#pragma unroll 4
      for (int i = 0; i < nb; i++) {
        const uint4 w = gq[i * 8 + (lane & 7)];
        const uint4 a = aq16[i * 2 + hh];
        const float dxdy = __fmul_rn(__half2float(gd[i * 4 + r4]), a_d[i]);
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
    __syncthreads();
  };
  // Rows of an item with long rows, 8 threads per row (one AVX2 lane each; a
  // warp per group of 4 rows).
  auto rows_8t = [&](const uint8_t* base, const ItemDesc& d) {
    const int K = (int)d.K, nb = K / 32, Gt = d.G[0];
    const int rr = lane >> 3, j = lane & 7;
    for (int g = warp; g < Gt; g += kNW) {
      const uint32_t* gq = (const uint32_t*)(base + (size_t)g * 4 * K);
      const __half* gd = (const __half*)(base + (size_t)Gt * 4 * K) + (size_t)g * nb * 4;
      const float acc = lane_chain(0.0f, gq, gd, (const int*)aq, ad, nb, lane, j, rr);
      const float s4 = __fadd_rn(acc, __shfl_xor_sync(FULL, acc, 4));
      const float s1 = __fadd_rn(s4, __shfl_xor_sync(FULL, s4, 1));
      const float s2 = __fadd_rn(s1, __shfl_xor_sync(FULL, s1, 2));
      if (j == 0) res[g * 4 + rr] = s2;
    }
    __syncthreads();
  };

  unsigned long long* const ctr = p.ctr;
  const unsigned long long tA = (epoch + 1ull) * (unsigned long long)p.n_attn;
  const unsigned long long tW = (epoch + 1ull) * (unsigned long long)W;

  if (r.attn) {
    // ===================== attention CTAs =====================
    const float* bias_base = nullptr;
    for (int l = 0; l < p.n_layer; l++) {
      const PersistLayer& Ly = lay[l];
      float* cache_k = p.cache + (size_t)l * 2 * p.n_ctx * HKV * D;
      float* cache_v = cache_k + (size_t)p.n_ctx * HKV * D;
      const float* kbase = cache_k + (size_t)r.kvh * D;
      const float* vbase = cache_v + (size_t)r.kvh * D;
      const size_t rsd = (size_t)HKV * D;
      if (tr_attn) pstamp(p, 2 * l, 0);
      // operands that do not depend on this step's previous phases
      bias_base = Ly.bqkv + (r.kv ? E + r.kvh * D : r.h * D);
      const int half = D / 2;
      float2 rc = make_float2(0.0f, 0.0f);
      float b_lo = 0.0f, b_hi = 0.0f, b_v = 0.0f;
      if (tid < half) {
        rc = p.rope[(size_t)n_past * half + tid];
        b_lo = bias_base[tid];
        b_hi = bias_base[tid + half];
      }
      if (r.kv && tid < D) b_v = Ly.bqkv[E + HKV * D + r.kvh * D + tid];
      // cached K / V rows [c0, c0 + rows) into the tiles (position n_past,
      // this step's, comes from kr / vr)
      // (with_k / with_v: which of the two tiles to fill)
      auto load_kv = [&](int c0, int rows, bool with_k, bool with_v) {
        const int D4 = D / 4, total = rows * D4;
        for (int e0 = tid; e0 < total; e0 += 4 * kNT) {
          float4 vk[4], vv[4];
#pragma unroll
          for (int u = 0; u < 4; u++) {
            const int e = e0 + u * kNT, rw = e / D4, c = e - rw * D4;
            if (e < total && c0 + rw != n_past) {
              if (with_k) vk[u] = __ldcg((const float4*)(kbase + (size_t)(c0 + rw) * rsd) + c);
              if (with_v) vv[u] = __ldcg((const float4*)(vbase + (size_t)(c0 + rw) * rsd) + c);
            }
          }
#pragma unroll
          for (int u = 0; u < 4; u++) {
            const int e = e0 + u * kNT, rw = e / D4, c = e - rw * D4;
            if (e < total && c0 + rw != n_past) {
              if (with_k) {
                float* dk = Ks + (size_t)rw * KP + c * 4;
                dk[0] = vk[u].x;
                dk[1] = vk[u].y;
                dk[2] = vk[u].z;
                dk[3] = vk[u].w;
              }
              if (with_v) *(float4*)(Vs + (size_t)rw * D + c * 4) = vv[u];
            }
          }
        }
      };
      // every head's output of this layer, into oq / od (phase l of bar_o;
      // the previous phase completed before this CTA's O rows of layer l-1,
      // and no head of layer l can finish before every attention CTA has
      // stored its x2 rows of layer l-1)
      if (tid == 0) mbar_arrive_expect_tx(bar_o, (uint32_t)(p.H * (D + 4 * (D / 32))));
      if (query) {
        if (tid == 0) mbar_arrive_expect_tx(bar_kv, (uint32_t)(2 * D * 4));
        load_kv(0, min(KT, n_kv), true, true);
      }
      float nw[4];
      load_nw(Ly.attn_norm, nw);
      // ---- x of this layer: the embedding (layer 0) or the down output ----
      if (l > 0) wait_ctr(&ctr[(size_t)(l - 1) * 4 + 3], tW);
      if (tr_attn) pstamp(p, 2 * l, 1);
      norm_quant(p.x, l == 0, nw);  // xs keeps x: the O rows' residual
      if (tr_attn) pstamp(p, 2 * l, 2);
      // ---- the CTA's q rows, or k and v rows ----
      const ItemDesc d = item_desc(p, lay, r, 2 * l);
      const uint8_t* wbase = wait_item(2 * l);
      rows_2t(wbase, d, aq, ad);  // ends with a CTA barrier: the item may be reused
      if (tr_attn) pstamp(p, 2 * l, 3);
      // ---- bias, RoPE (ref src/ops_cpu.cpp:286-297), v ----
      if (tid < half) {
        const float a0 = __fadd_rn(res[tid], b_lo), a1 = __fadd_rn(res[tid + half], b_hi);
        float* dst = r.kv ? kr : qr;
        dst[tid] = __fsub_rn(__fmul_rn(a0, rc.x), __fmul_rn(a1, rc.y));
        dst[tid + half] = __fadd_rn(__fmul_rn(a0, rc.y), __fmul_rn(a1, rc.x));
      }
      if (r.kv && tid < D) vr[tid] = __fadd_rn(res[D + tid], b_v);
      __syncthreads();
      if (r.kv) {
        // k / v into the query CTAs of this KV head (cluster ranks
        // kvh * (n_rep + 1) + c; st.async, counted on the receiver's bar_kv),
        // then the KV-cache append
        if (!s_dead) {
          const int per = D >> 1;
          for (int e = tid; e < n_rep * per; e += kNT) {
            const int c = e / per, i4 = e - c * per;
            const uint32_t rk = (uint32_t)(r.kvh * CK + c);
            const float* src = i4 < D / 4 ? kr + 4 * i4 : vr + 4 * (i4 - D / 4);
            dsmem_store_async(dsmem_addr(src, rk), *(const float4*)src, dsmem_addr(bar_kv, rk));
          }
        }
        if (tid < D) {
          cache_k[((size_t)n_past * HKV + r.kvh) * D + tid] = kr[tid];
          cache_v[((size_t)n_past * HKV + r.kvh) * D + tid] = vr[tid];
        }
        __syncthreads();
      } else {
      // ---- query CTA: the decode attention of head h ----
      if (!s_dead && !mbar_wait_bounded(bar_kv, (uint32_t)(l & 1), p.err)) s_dead = 1;
      if (n_past < KT && tid < D) {
        Ks[(size_t)n_past * KP + tid] = kr[tid];
        Vs[(size_t)n_past * D + tid] = vr[tid];
      }
      __syncthreads();
      if (tr_attn) pstamp(p, 2 * l, 4);
      float* sc = p.scores_in_smem ? scs : p.scores + (size_t)r.h * p.n_ctx;
      const int n_chunks = (n_kv + KT - 1) / KT;
      float lmax = -INFINITY;
      for (int c = 0; c < n_chunks; c++) {
        const int c0 = c * KT, rows = min(KT, n_kv - c0);
        if (c > 0) {
          __syncthreads();
          load_kv(c0, rows, true, false);  // the V tile keeps chunk 0 for the value sums
          if (n_past >= c0 && n_past < c0 + rows)
            for (int i = tid; i < D; i += kNT) Ks[(size_t)(n_past - c0) * KP + i] = kr[i];
          __syncthreads();
        }
        // scores[i] * scale, d ascending with separate roundings (src/ops_cpu.cpp:373-376)
        for (int i = tid; i < rows; i += kNT) {
          float dot;
          if constexpr (FAST) {
            // fast mode: four interleaved chains
            const float* kr_ = Ks + (size_t)i * KP;
            float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
            for (int e = 0; e < D; e += 4) {
              s0 = fmaf(kr_[e], qr[e], s0);
              s1 = fmaf(kr_[e + 1], qr[e + 1], s1);
              s2 = fmaf(kr_[e + 2], qr[e + 2], s2);
              s3 = fmaf(kr_[e + 3], qr[e + 3], s3);
            }
            dot = (s0 + s1) + (s2 + s3);
          } else {
            dot = ordered_dot(0.0f, Ks + (size_t)i * KP, 1, qr, D);
          }
          const float v = __fmul_rn(dot, p.scale);
          sc[c0 + i] = v;
          lmax = fmaxf(lmax, v);
        }
      }
      lmax = warp_max(lmax);
      if (lane == 0) red_f[warp] = lmax;
      __syncthreads();
      float mx = red_f[0];
      for (int w = 1; w < kNW; w++) mx = fmaxf(mx, red_f[w]);
      float inv;
      if constexpr (FAST) {
        // fast mode: exp and the denominator's block tree in one pass
        float ls = 0.0f;
        for (int i = tid; i < n_kv; i += kNT) {
          const float e = expf(sc[i] - mx);
          sc[i] = e;
          ls += e;
        }
        ls = warp_sum_tree(ls);
        if (lane == 0) red_s[warp] = ls;
        __syncthreads();
        if (tr_attn) pstamp(p, 2 * l, 5);
        float sum = 0.0f;
#pragma unroll
        for (int w = 0; w < kNW; w++) sum += red_s[w];
        inv = 1.0f / sum;
      } else {
        for (int i = tid; i < n_kv; i += kNT) sc[i] = expf_exact(__fsub_rn(sc[i], mx), p.et);
        __syncthreads();
        if (tr_attn) pstamp(p, 2 * l, 5);
        // the softmax denominator: one ordered chain (src/ops_cpu.cpp:331-336)
        if (tid == 0) {
          float sum = 0.0f;
          if (p.scores_in_smem) {
            sum = ordered_sum_smem(sc, n_kv);
          } else {
#pragma unroll 8
            for (int i = 0; i < n_kv; i++) sum = __fadd_rn(sum, sc[i]);
          }
          misc[1] = __fdiv_rn(1.0f, sum);
        }
        __syncthreads();
        inv = misc[1];
      }
      if (tr_attn) pstamp(p, 2 * l, 6);
      // out[o] = sum_t V[o, kvh, t] * P[t], t ascending (src/ops_cpu.cpp:402-406);
      // the K / V tiles of the next layer replace these only after this loop.
      // Fast mode: NG = kNT / D thread groups each take every NG-th position,
      // their partials meet in shared memory (res), normalized at the end.
      const int NG = FAST ? kNT / D : 1, grp = tid / D, o_el = tid - grp * D;
      float acc = 0.0f;
      for (int c = 0; c < n_chunks; c++) {
        const int c0 = c * KT, rows = min(KT, n_kv - c0);
        if (c > 0) {
          __syncthreads();
          load_kv(c0, rows, false, true);
          if (n_past >= c0 && n_past < c0 + rows)
            for (int i = tid; i < D; i += kNT) Vs[(size_t)(n_past - c0) * D + i] = vr[i];
          __syncthreads();
        }
        if constexpr (FAST) {
          if (grp < NG)
            for (int i = grp; i < rows; i += NG) acc = fmaf(Vs[(size_t)i * D + o_el], sc[c0 + i], acc);
        } else {
          if (tid < D) acc = ordered_dot_scaled_pp(acc, Vs + tid, D, sc + c0, inv, rows);
        }
      }
      if constexpr (FAST) {
        if (grp < NG) res[tid] = acc;
        __syncthreads();
        if (tid < D) {
          float s = 0.0f;
          for (int g2 = 0; g2 < NG; g2++) s += res[g2 * D + tid];
          acc = s * inv;
        }
      }
      // the O projection's quantize node (src/ops_cpu.cpp:462-479) for this
      // head's outputs (warp w holds block h*D/32 + w), then the blocks into
      // every attention CTA's oq / od: D/4 words of quants and D/32 scales
      // per receiver, counted on its bar_o
      if (tid < D) {
        float dq;
        ostage_q[tid] = quantize_lane(acc, &dq);
        if (lane == 0) ostage_d[tid >> 5] = dq;
      }
      __syncthreads();
      if (!s_dead) {
        const int nw = D / 4 + D / 32;
        for (int e = tid; e < p.n_attn * nw; e += kNT) {
          const int rk = e / nw, w = e - rk * nw;
          const bool quant = w < D / 4;
          const uint32_t v = quant ? ((const uint32_t*)ostage_q)[w] : __float_as_uint(ostage_d[w - D / 4]);
          const void* dst = quant ? (const void*)(oq + r.h * D + 4 * w) : (const void*)(od + r.h * (D / 32) + (w - D / 4));
          dsmem_store_async_u32(dsmem_addr(dst, (uint32_t)rk), v, dsmem_addr(bar_o, (uint32_t)rk));
        }
      }
      }  // query CTA
      // ---- O projection + residual on the cluster: x2 = x + W_o . attn ----
      {
        const ItemDesc dO = item_desc(p, lay, r, 2 * l + 1);
        const int rows = 4 * dO.G[0], r0 = 4 * dO.g0[0];
        if (!s_dead && !mbar_wait_bounded(bar_o, (uint32_t)(l & 1), p.err)) s_dead = 1;
        const uint8_t* wb = wait_item(2 * l + 1);
        if (rows > 0) rows_2t(wb, dO, oq, od);
        for (int i = tid; i < rows; i += kNT) p.x2[r0 + i] = __fadd_rn(xs[r0 + i], res[i]);
        signal_ctr(&ctr[(size_t)l * 4 + 1]);
        // the layer's two ring items are freed only after its last signal:
        // issuing a copy holds thread 0 for up to ~0.5 us, which on the
        // slowest CTA would delay every consumer of its signal
        free_item(2 * l);
        free_item(2 * l + 1);
        if (tr_attn) pstamp(p, 2 * l, 7);
      }
    }
  } else {
    // ===================== projection CTAs =====================
    for (int l = 0; l < p.n_layer; l++) {
      const PersistLayer& Ly = lay[l];
      // ---- gate/up: rms_norm(x2) * ffn_norm, quantize; silu(gate) * up, quantize ----
      {
        const ItemDesc d = item_desc(p, lay, r, 2 * l);
        if (tr_gemv) pstamp(p, 2 * l + 1, 0);
        float nw[4];
        load_nw(Ly.ffn_norm, nw);
        if (tr_gemv) pstamp(p, 2 * l + 1, 1);
        wait_ctr(&ctr[(size_t)l * 4 + 1], tA);
        if (tr_gemv) pstamp(p, 2 * l + 1, 2);
        norm_quant(p.x2, false, nw);  // xs keeps x2: the down rows' residual
        if (tr_gemv) pstamp(p, 2 * l + 1, 3);
        const uint8_t* wb = wait_item(2 * l);
        if (d.G[0] > 0) rows_2t(wb, d, aq, ad);
        // each 64 packed rows are the gate / up rows of one 32-element block:
        // act[a] = silu(gate) * up, then the down projection's quantize node
        for (int j = warp; j < r.gu_b1 - r.gu_b0; j += kNW) {
          const int a = 32 * j + lane;                  // element of the CTA's blocks
          const int lr = (a >> 2) * 8 + (a & 3);        // its gate row, local
          const float v = __fmul_rn(silu_exact(res[lr], p.et), res[lr + 4]);
          float dq;
          const int8_t q = quantize_lane(v, &dq);
          uint8_t* blk = p.act_q + (size_t)(r.gu_b0 + j) * 36;
          ((int8_t*)blk)[4 + lane] = q;
          if (lane == 0) *(float*)blk = dq;
        }
        signal_ctr(&ctr[(size_t)l * 4 + 2]);
        if (tr_gemv) pstamp(p, 2 * l + 1, 4);
      }
      // ---- down projection + residual: x = x2 + W_down . act ----
      {
        const ItemDesc d = item_desc(p, lay, r, 2 * l + 1);
        const int rows = 4 * d.G[0], r0 = 4 * d.g0[0];
        wait_ctr(&ctr[(size_t)l * 4 + 2], tW);
        if (tr_gemv) pstamp(p, 2 * l + 1, 5);
        load_act(p.act_q, nbF);
        const uint8_t* wb = wait_item(2 * l + 1);
        if (rows > 0) {
          if (FAST && rows * kNW <= E) rows_8t_split(wb, d);
          else rows_8t(wb, d);
        }
        for (int i = tid; i < rows; i += kNT) p.x[r0 + i] = __fadd_rn(xs[r0 + i], res[i]);
        signal_ctr(&ctr[(size_t)l * 4 + 3]);
        free_item(2 * l);  // (after the layer's last signal, as above)
        free_item(2 * l + 1);
        if (tr_gemv) pstamp(p, 2 * l + 1, 6);
      }
    }
    // ---- LM head: rms_norm(x) * output_norm, quantize; logits; argmax ----
    if (p.with_head) {
      float nw[4];
      load_nw(p.out_norm, nw);
      wait_ctr(&ctr[(size_t)(p.n_layer - 1) * 4 + 3], tW);
      if (tr_gemv) pstamp(p, 2 * p.n_layer, 0);
      norm_quant(p.x, false, nw);
      if (tr_gemv) pstamp(p, 2 * p.n_layer, 1);
      float bv = -INFINITY;
      int32_t bi = 0x7fffffff;
      // trace: thread 0's time waiting for LM-head ring items, and the rest
      uint64_t t_wait = 0, t_rows = 0, t_free = 0, t_mark = tr_gemv ? globaltimer_ns() : 0;
      for (int it = r.n_main; it < r.n_items; it++) {
        const ItemDesc d = item_desc(p, lay, r, it);
        const uint8_t* wb = wait_item(it);
        if (tr_gemv) {
          const uint64_t now = globaltimer_ns();
          t_wait += now - t_mark;
          t_mark = now;
        }
        rows_2t(wb, d, aq, ad);  // ends with a CTA barrier: the item may be reused
        if (tr_gemv) {
          const uint64_t now = globaltimer_ns();
          t_rows += now - t_mark;
          t_mark = now;
        }
        free_item(it);
        if (tr_gemv) {
          const uint64_t now = globaltimer_ns();
          t_free += now - t_mark;
          t_mark = now;
        }
        const int r0 = 4 * d.g0[0];
        for (int i = tid; i < 4 * d.G[0]; i += kNT) {
          const int row = r0 + i;
          if (row >= p.V) continue;
          const float v = res[i];
          p.logits[row] = v;
          if (v > bv || bi == 0x7fffffff) {  // rows ascend per thread: first maximum
            bv = v;
            bi = row;
          }
        }
        __syncthreads();  // res is rewritten by the next chunk
        if (tr_gemv) t_mark = globaltimer_ns();
      }
      if (tr_gemv && p.trace) {
        p.trace[(size_t)(2 * p.n_layer) * kTracePoints + 4] = t_wait;
        p.trace[(size_t)(2 * p.n_layer) * kTracePoints + 5] = t_rows;
        p.trace[(size_t)(2 * p.n_layer) * kTracePoints + 6] = t_free;
        p.trace[(size_t)(2 * p.n_layer) * kTracePoints + 7] = (uint64_t)(r.n_items - r.n_main);
      }
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
        red_f[warp] = bv;
        red_i[warp] = bi;
      }
      __syncthreads();
      if (tid == 0) {
        for (int w = 1; w < kNW; w++)
          if (red_f[w] > bv || (red_f[w] == bv && red_i[w] < bi)) {
            bv = red_f[w];
            bi = red_i[w];
          }
        p.part_val[cta - p.n_attn] = bv;
        p.part_idx[cta - p.n_attn] = bi;
      }
      if (tr_gemv) pstamp(p, 2 * p.n_layer, 2);
    }
  }

  // ---- close the step: the last CTA to finish advances the state ----
  __syncthreads();
  if (tid == 0) {
    // items this CTA issued but did not consume (only after a time-out) get a
    // bounded chance to land before the shared memory is released
    for (int it = rs->freed; it < rs->next; it++)
      (void)mbar_wait_bounded(&bars[it % kQ], (uint32_t)((it / kQ) & 1), nullptr);
    __threadfence();
    s_ticket = atomicAdd(p.ticket, 1u);
  }
  __syncthreads();
  if (s_ticket == (uint32_t)G - 1 && tid == 0) {
    __threadfence();
    if (p.with_head) {
      // the first maximum over the projection CTAs, whose row ranges ascend
      float best = __ldcg(&p.part_val[0]);
      int32_t besti = __ldcg(&p.part_idx[0]);
      for (int c = 1; c < W; c++) {
        const float v = __ldcg(&p.part_val[c]);
        const int32_t i = __ldcg(&p.part_idx[c]);
        if (v > best || (v == best && i < besti)) {
          best = v;
          besti = i;
        }
      }
      *p.next_token = besti;
      if (*p.feedback && n_past + 1 < p.tokens_len) p.tokens[n_past + 1] = besti;
    }
    *p.pos = n_past + 1;
    *p.epoch = epoch + 1ull;
    *p.ticket = 0u;
    if (tr_gemv || tr_attn) pstamp(p, 2 * p.n_layer, 3);
  }
  // peers may still store into this CTA's shared memory (k / v hand-over)
  // until every CTA of the cluster is here
  cluster_arrive_relaxed();
  cluster_wait_acquire();
}

int g_optin = 0;

}  // namespace

cudaError_t prepare_persist_kernel(int optin) {
  // both instantiations (exact and fast mode) get the same dynamic budget
  cudaFuncAttributes f0{}, f1{};
  cudaError_t e = cudaFuncGetAttributes(&f0, persist_step_kernel<false>);
  if (e == cudaSuccess) e = cudaFuncGetAttributes(&f1, persist_step_kernel<true>);
  const int dyn = optin - (int)std::max(f0.sharedSizeBytes, f1.sharedSizeBytes);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(persist_step_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(persist_step_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(persist_step_kernel<false>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(persist_step_kernel<true>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e == cudaSuccess) g_optin = dyn;
  return e;
}

PersistPlan plan_persist(int64_t E, int32_t D, int32_t H, int32_t HKV, int64_t FF, int64_t V, int32_t n_layer,
                         int32_t n_ctx, int num_sms) {
  PersistPlan pl{};
  if (g_optin <= 0 || D < 32 || D > 128 || D % 32 != 0 || HKV <= 0 || H % HKV != 0 || E % 64 != 0 ||
      E > 1024 || E != (int64_t)H * D || FF % 64 != 0 || FF < 64 || V <= 0 || n_ctx <= 0)
    return pl;
  // one cluster for every head: n_kv_head * (n_rep + 1) CTAs, at most 16 (a
  // non-portable cluster size on B200)
  const int32_t n_rep = H / HKV, C = HKV * (n_rep + 1);
  if (C > 16) return pl;
  if (n_layer <= 0 || n_layer > kMaxLayers) return pl;
  const PSmem L = persist_smem(E, FF, n_layer);
  const size_t avail = (size_t)g_optin;
  if (avail <= L.ring + 4096) return pl;
  const size_t ring_gemv = (avail - L.ring) / 128 * 128;
  // query CTAs: a ring for the item of their q rows and the item of their O
  // rows, then the K / V tiles; k/v CTAs: the k and v rows and the O rows
  const int OG = (int)((E / 4 + C - 1) / C);
  if (OG * 4 > kMaxRes) return pl;
  const size_t ring_attn = groups_bytes(D / 4, E) + groups_bytes(OG, E);
  const size_t kv_item = 2 * groups_bytes(D / 4, E) + groups_bytes(OG, E);
  const size_t sc = n_ctx <= kScoresOnChipMax ? up16((size_t)n_ctx * 4) + kChainSlackBytes : 0;
  const size_t row = (size_t)(2 * D + 1) * 4;
  if (ring_gemv < kv_item || ring_gemv < ring_attn + sc + 32 * row) return pl;
  int64_t kt = (int64_t)((ring_gemv - ring_attn - sc) / row);
  kt = std::min<int64_t>(256, kt) / 32 * 32;
  // MI_CUDA_PERSIST_KV_TILE caps the K / V tile (positions, a multiple of 32),
  // so tests can make short contexts walk several tiles
  if (const char* e = std::getenv("MI_CUDA_PERSIST_KV_TILE"))
    if (std::atoi(e) >= 32) kt = std::min<int64_t>(kt, std::atoi(e) / 32 * 32);
  // clusters that can be resident at once: the whole grid must be
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kNT);
  cfg.dynamicSmemBytes = avail;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3((unsigned)(C * (num_sms / C)));
  // the grid must be resident at once in both modes (exact and fast)
  int n_clusters = 0, n_fast = 0;
  if (cudaOccupancyMaxActiveClusters(&n_clusters, persist_step_kernel<false>, &cfg) != cudaSuccess ||
      cudaOccupancyMaxActiveClusters(&n_fast, persist_step_kernel<true>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return pl;
  }
  n_clusters = std::min(n_clusters, n_fast);
  n_clusters = std::min(n_clusters, num_sms / C);
  const int32_t n_attn = C;
  const int32_t grid = C * n_clusters;
  const int32_t n_gemv = grid - n_attn;
  // every projection CTA keeps at most two 32-element FFN blocks (the ring
  // and kMaxRes hold 128 gate/up rows)
  if (n_gemv < 8 || (FF / 32 + n_gemv - 1) / n_gemv > 2 || (E / 4 + n_gemv - 1) / n_gemv * 4 > kMaxRes)
    return pl;
  // the largest item of a projection CTA must fit its ring
  const size_t gu_item = groups_bytes(16 * (int)((FF / 32 + n_gemv - 1) / n_gemv), E);
  const size_t dn_item = groups_bytes((int)((E / 4 + n_gemv - 1) / n_gemv), FF);
  if (gu_item > ring_gemv || dn_item > ring_gemv || groups_bytes(kHeadChunkGroups, E) > ring_gemv) return pl;
  pl.ok = true;
  pl.grid = grid;
  pl.cluster = C;
  pl.n_attn = n_attn;
  pl.n_gemv = n_gemv;
  pl.kv_tile = (int32_t)kt;
  pl.scores_in_smem = sc > 0 ? 1 : 0;
  pl.ring_gemv = (int32_t)ring_gemv;
  pl.ring_attn = (int32_t)ring_attn;
  pl.smem = avail;
  return pl;
}

cudaError_t launch_persist(const PersistParams& p, const PersistPlan& plan, cudaStream_t s) {
  if (!plan.ok) return cudaErrorInvalidValue;
  PersistParams q = p;
  q.n_attn = plan.n_attn;
  q.n_gemv = plan.n_gemv;
  q.kv_tile = plan.kv_tile;
  q.scores_in_smem = plan.scores_in_smem;
  q.ring_gemv = plan.ring_gemv;
  q.ring_attn = plan.ring_attn;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)plan.grid);
  cfg.blockDim = dim3(kNT);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)plan.cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return q.fast ? cudaLaunchKernelEx(&cfg, persist_step_kernel<true>, q)
                : cudaLaunchKernelEx(&cfg, persist_step_kernel<false>, q);
}

}  // namespace mi
