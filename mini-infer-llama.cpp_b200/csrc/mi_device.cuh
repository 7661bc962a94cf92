// Device-side building blocks shared by every kernel of the backend:
// PTX wrappers (mbarrier, bulk async copy, programmatic dependent launch),
// the libm-exact expf, and the exact-order arithmetic helpers.
//
// Exactness rule for every kernel: float arithmetic is written with the
// round-to-nearest intrinsics (__fadd_rn, __fmul_rn, __fdiv_rn, __fsqrt_rn,
// __fmaf_rn) in the reference's operation order, and the library is compiled
// with -fmad=false, so no multiply-add is ever contracted behind our back.
// __fmaf_rn appears only where the reference's AVX2 kernel issues an FMA.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdlib>

#include "mi_expf_core.h"
#include "mi_internal.h"

namespace mi {

// Iteration bound of every spin wait (each try_wait blocks for a while in
// hardware, so this is seconds, far beyond any legitimate wait).
constexpr uint32_t kSpinLimit = 1u << 22;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

// Global -> shared bulk copy (TMA engine, no tensor map). dst and src 16-byte
// aligned, bytes a multiple of 16; completion is counted on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// L2 policy for data read once per decode step (the weights): evict_first,
// so the weight stream does not displace what later steps read again (the KV
// cache rows, the activations, the expf exception table).
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// bulk_load with an L2 cache-policy hint (l2_evict_first_policy).
__device__ __forceinline__ void bulk_load_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                               uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
      "%4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on a phase of `bar`. On expiry records MI_CUDA_ERR_TIMEOUT in
// *err and returns false; the caller then skips its work and exits.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int32_t* err) {
  for (uint32_t it = 0; it < kSpinLimit; it++)
    if (mbar_try_wait(bar, parity)) return true;
  if (err) atomicExch(err, 5 /* MI_CUDA_ERR_TIMEOUT */);
  return false;
}

// Programmatic dependent launch: a kernel launched with programmatic stream
// serialization may start while its predecessor runs; pdl_wait() blocks until
// the predecessor grid has completed and its writes are visible. Both are
// no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// The CTA-wide form: one thread waits (the predecessor's writes become visible
// to the whole grid), the rest park on the CTA barrier, so a kernel launched
// early does not keep 256 threads polling beside the kernel it waits for.
__device__ __forceinline__ void pdl_wait_cta() {
  if (threadIdx.x == 0) pdl_wait();
  __syncthreads();
}
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// MI_CUDA_CARVEOUT=<percent> sets every decode kernel's preferred shared-memory
// carveout (cudaFuncAttributePreferredSharedMemoryCarveout); unset leaves the
// driver's choice. An SM changes its carveout only when idle, so a kernel whose
// CTAs need a large share can start beside its predecessor's CTAs only on SMs
// already configured that large.
template <typename F>
inline cudaError_t set_carveout(F* func) {
  const char* c = std::getenv("MI_CUDA_CARVEOUT");
  if (!c) return cudaSuccess;
  const int pct = std::atoi(c);
  if (pct < 0 || pct > 100) return cudaSuccess;
  return cudaFuncSetAttribute(func, cudaFuncAttributePreferredSharedMemoryCarveout, pct);
}

// ---------------------------------------------------------------------------
// Thread-block clusters: the hardware cluster barrier (every thread of every
// CTA arrives, then waits; exited threads do not count) and asynchronous
// stores into another CTA's shared memory (distributed shared memory).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The shared::cluster address of `p` (a variable of this CTA's shared memory)
// in the CTA of cluster rank `rank`.
__device__ __forceinline__ uint32_t dsmem_addr(const void* p, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_addr(p)), "r"(rank));
  return a;
}
// Four floats into another CTA's shared memory at `addr`, counted (16 bytes)
// on that CTA's mbarrier `bar` (both shared::cluster addresses from
// dsmem_addr); the receiver waits on its barrier like on a bulk copy.
__device__ __forceinline__ void dsmem_store_async(uint32_t addr, float4 v, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(addr),
               "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(bar)
               : "memory");
}

// One 32-bit word into another CTA's shared memory, counted (4 bytes) on its
// mbarrier `bar` (shared::cluster addresses, as dsmem_store_async).
__device__ __forceinline__ void dsmem_store_async_u32(uint32_t addr, uint32_t v, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(addr), "r"(v),
               "r"(bar)
               : "memory");
}

// ---------------------------------------------------------------------------
// Tensor-parallel exchange words: value bits | tag << 32, written with one
// 64-bit store (single-copy atomic), so a reader that sees the step's tag
// sees that step's value. Peer buffers are written through peer pointers
// (NVLink); readers poll their own copy with volatile loads.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t ll_load(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void ll_store(uint64_t* p, uint32_t bits, uint32_t tag) {
  const uint64_t v = ((uint64_t)tag << 32) | bits;
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// The value bits of *p once it carries `tag`. Bounded: after kSpinLimit polls
// it records MI_CUDA_ERR_TIMEOUT in *err, sets `dead` (later waits of the
// thread then return at once) and returns 0. It also gives up as soon as it
// sees *err set by another wait, so a stopped peer costs one time-out per
// step, not one per kernel.
__device__ __forceinline__ uint32_t ll_wait(const uint64_t* p, uint32_t tag, int32_t* err, bool& dead) {
  uint64_t v = ll_load(p);
  if ((uint32_t)(v >> 32) == tag) return (uint32_t)v;
  if (dead) return 0u;
  for (uint32_t it = 0; it < kSpinLimit; it++) {
    v = ll_load(p);
    if ((uint32_t)(v >> 32) == tag) return (uint32_t)v;
    if ((it & 1023u) == 1023u && err && *(volatile int32_t*)err != 0) {
      dead = true;
      return 0u;
    }
  }
  dead = true;
  if (err) atomicExch(err, 5 /* MI_CUDA_ERR_TIMEOUT */);
  return 0u;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Step trace: CTA 0 of a traced kernel stores globaltimer stamps at fixed
// points into its slot of kTracePoints entries: 0 entry, 1 dependency
// satisfied, 2 prologue done, 3 epilogue start; 4-7 kernel-specific phases.
constexpr int kTracePoints = 8;
__device__ __forceinline__ void trace_mark(uint64_t* trace, int32_t slot, int point) {
  if (trace && blockIdx.x == 0 && threadIdx.x == 0)
    trace[(size_t)slot * kTracePoints + point] = globaltimer_ns();
}

// libm-exact expf: the double-precision core plus one probe of the exception
// hash (two buckets of four (key, value) pairs, loaded as four independent
// 16-byte reads).
// Read-only 16-byte load whose line L2 keeps in preference to others
// (evict_last): the expf exception table is probed at random and would
// otherwise be evicted by the weight streams between uses.
__device__ __forceinline__ uint4 ldg_keep(const uint4* p) {
  uint64_t pol;
  asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  uint4 v;
  asm("ld.global.nc.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p), "l"(pol));
  return v;
}

__device__ __forceinline__ float expf_exact(float x, const ExpTab& t) {
  float y;
  if (x >= -110.0f && x <= 100.0f) {
    const double yd = mi_expf_core_wide(x);
    y = (float)yd;
    // results far from a rounding boundary are never exceptions (when the
    // table generator has verified that for this libm)
    if (t.filter && !mi_expf_near_tie(yd, MI_EXPF_TIE_PROBE)) return y;
  } else {
    y = mi_expf_core(x);
  }
  if (x == x) {
    uint32_t key = __float_as_uint(x);
    uint32_t b1 = mi_expf_bucket(key, t.mul1, t.log2b);
    uint32_t b2 = mi_expf_bucket(key, t.mul2, t.log2b);
    const uint4* p1 = t.buckets + 2 * (size_t)b1;
    const uint4* p2 = t.buckets + 2 * (size_t)b2;
    uint4 a0 = ldg_keep(p1), a1 = ldg_keep(p1 + 1), c0 = ldg_keep(p2), c1 = ldg_keep(p2 + 1);
    if (a0.x == key) y = __uint_as_float(a0.y);
    if (a0.z == key) y = __uint_as_float(a0.w);
    if (a1.x == key) y = __uint_as_float(a1.y);
    if (a1.z == key) y = __uint_as_float(a1.w);
    if (c0.x == key) y = __uint_as_float(c0.y);
    if (c0.z == key) y = __uint_as_float(c0.w);
    if (c1.x == key) y = __uint_as_float(c1.y);
    if (c1.z == key) y = __uint_as_float(c1.w);
  }
  return y;
}

// x / (1 + expf(-x)), ref src/ops_cpu.cpp:424.
__device__ __forceinline__ float silu_exact(float x, const ExpTab& t) {
  return __fdiv_rn(x, __fadd_rn(1.0f, expf_exact(-x, t)));
}

// Sequential float sum s = ((0 + a[0]) + a[1]) + ... + a[n-1] (one rounding
// per add, in order) for one thread, with the shared-memory loads issued 16
// elements ahead of the dependent adds so the chain runs at add latency.
// `a` is 16-byte aligned; any n.
__device__ __forceinline__ float ordered_sum_smem(const float* a, int n) {
  const float4* a4 = (const float4*)a;
  const int n4 = n >> 2;
  float s = 0.0f;
  float4 b0 = make_float4(0, 0, 0, 0), b1 = b0, b2 = b0, b3 = b0;
  if (n4 > 0) b0 = a4[0];
  if (n4 > 1) b1 = a4[1];
  if (n4 > 2) b2 = a4[2];
  if (n4 > 3) b3 = a4[3];
  int i = 0;
  for (; i + 4 <= n4; i += 4) {
    const float4 c0 = b0, c1 = b1, c2 = b2, c3 = b3;
    if (i + 4 < n4) b0 = a4[i + 4];
    if (i + 5 < n4) b1 = a4[i + 5];
    if (i + 6 < n4) b2 = a4[i + 6];
    if (i + 7 < n4) b3 = a4[i + 7];
    s = __fadd_rn(s, c0.x); s = __fadd_rn(s, c0.y); s = __fadd_rn(s, c0.z); s = __fadd_rn(s, c0.w);
    s = __fadd_rn(s, c1.x); s = __fadd_rn(s, c1.y); s = __fadd_rn(s, c1.z); s = __fadd_rn(s, c1.w);
    s = __fadd_rn(s, c2.x); s = __fadd_rn(s, c2.y); s = __fadd_rn(s, c2.z); s = __fadd_rn(s, c2.w);
    s = __fadd_rn(s, c3.x); s = __fadd_rn(s, c3.y); s = __fadd_rn(s, c3.z); s = __fadd_rn(s, c3.w);
  }
  for (; i < n4; i++) {
    const float4 c = a4[i];
    s = __fadd_rn(s, c.x); s = __fadd_rn(s, c.y); s = __fadd_rn(s, c.z); s = __fadd_rn(s, c.w);
  }
  for (int k = n4 * 4; k < n; k++) s = __fadd_rn(s, a[k]);
  return s;
}

// acc + v[0]*p[0] + v[vs]*p[1] + ... in order, each product and each sum
// rounded separately (no FMA), loads batched 16 ahead of the dependent adds.
__device__ __forceinline__ float ordered_dot(float acc, const float* v, int vs, const float* p, int n) {
  int t = 0;
  for (; t + 16 <= n; t += 16) {
    float a[16], b[16];
#pragma unroll
    for (int u = 0; u < 16; u++) {
      a[u] = v[(size_t)(t + u) * vs];
      b[u] = p[t + u];
    }
#pragma unroll
    for (int u = 0; u < 16; u++) acc = __fadd_rn(acc, __fmul_rn(a[u], b[u]));
  }
  for (; t < n; t++) acc = __fadd_rn(acc, __fmul_rn(v[(size_t)t * vs], p[t]));
  return acc;
}

// ordered_dot with the softmax normalization applied as the terms are used:
// acc + v[0]*(p[0]*s) + v[vs]*(p[1]*s) + ..., each product rounded separately
// (the same values as normalizing p first, src/ops_cpu.cpp:338-341, then
// accumulating, src/ops_cpu.cpp:402-406).
__device__ __forceinline__ float ordered_dot_scaled(float acc, const float* v, int vs, const float* p, float s,
                                                   int n) {
  int t = 0;
  for (; t + 16 <= n; t += 16) {
    float a[16], b[16];
#pragma unroll
    for (int u = 0; u < 16; u++) {
      a[u] = v[(size_t)(t + u) * vs];
      b[u] = __fmul_rn(p[t + u], s);
    }
#pragma unroll
    for (int u = 0; u < 16; u++) acc = __fadd_rn(acc, __fmul_rn(a[u], b[u]));
  }
  for (; t < n; t++) acc = __fadd_rn(acc, __fmul_rn(v[(size_t)t * vs], __fmul_rn(p[t], s)));
  return acc;
}

// ordered_dot_scaled with two 16-term register batches in ping-pong: the
// loads of the next batch are in flight while the current batch's dependent
// adds run. Same terms, same order, same roundings.
__device__ __forceinline__ float ordered_dot_scaled_pp(float acc, const float* v, int vs, const float* p, float s,
                                                      int n) {
  int t = 0;
  if (n >= 32) {
    float a0[16], b0[16], a1[16], b1[16];
#pragma unroll
    for (int u = 0; u < 16; u++) {
      a0[u] = v[(size_t)u * vs];
      b0[u] = __fmul_rn(p[u], s);
    }
    for (; t + 32 <= n; t += 32) {
#pragma unroll
      for (int u = 0; u < 16; u++) {
        a1[u] = v[(size_t)(t + 16 + u) * vs];
        b1[u] = __fmul_rn(p[t + 16 + u], s);
      }
#pragma unroll
      for (int u = 0; u < 16; u++) acc = __fadd_rn(acc, __fmul_rn(a0[u], b0[u]));
      if (t + 48 <= n) {
#pragma unroll
        for (int u = 0; u < 16; u++) {
          a0[u] = v[(size_t)(t + 32 + u) * vs];
          b0[u] = __fmul_rn(p[t + 32 + u], s);
        }
      }
#pragma unroll
      for (int u = 0; u < 16; u++) acc = __fadd_rn(acc, __fmul_rn(a1[u], b1[u]));
    }
  }
  return ordered_dot_scaled(acc, v + (size_t)t * vs, vs, p + t, s, n - t);
}

// One lane's accumulator chain of the Q8_0 dot over n blocks of a 4-row group
// held in shared memory in the packed layout (block i: quants gq[i*32 + lane],
// scales gd[i*4 + rr]) against the quantized activation (aq4 words, ad scales,
// both already offset to the chain's first block):
//   acc = fma((float)dp4a(w_i, a_i), fp16(w.d_i) * a.d_i, acc), i ascending.
// The operands of eight blocks are loaded before their dependent FMAs, so the
// chain runs at FMA latency rather than at shared-memory load latency.
__device__ __forceinline__ float lane_chain(float acc, const uint32_t* gq, const __half* gd, const int* aq4,
                                            const float* ad, int n, int lane, int j, int rr) {
  int i = 0;
  for (; i + 8 <= n; i += 8) {
    int w[8], a[8];
    float dx[8];
#pragma unroll
    for (int u = 0; u < 8; u++) {
      w[u] = (int)gq[(i + u) * 32 + lane];
      a[u] = aq4[(i + u) * 8 + j];
      dx[u] = __fmul_rn(__half2float(gd[(i + u) * 4 + rr]), ad[i + u]);
    }
#pragma unroll
    for (int u = 0; u < 8; u++) acc = __fmaf_rn(__int2float_rn(__dp4a(w[u], a[u], 0)), dx[u], acc);
  }
  if (i + 4 <= n) {
    int w[4], a[4];
    float dx[4];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      w[u] = (int)gq[(i + u) * 32 + lane];
      a[u] = aq4[(i + u) * 8 + j];
      dx[u] = __fmul_rn(__half2float(gd[(i + u) * 4 + rr]), ad[i + u]);
    }
#pragma unroll
    for (int u = 0; u < 4; u++) acc = __fmaf_rn(__int2float_rn(__dp4a(w[u], a[u], 0)), dx[u], acc);
    i += 4;
  }
  for (; i < n; i++)
    acc = __fmaf_rn(__int2float_rn(__dp4a((int)gq[i * 32 + lane], aq4[i * 8 + j], 0)),
                    __fmul_rn(__half2float(gd[i * 4 + rr]), ad[i]), acc);
  return acc;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Butterfly sum over a warp (tree order: only for the labelled fast mode,
// never on a path that must match the reference's sequential sums).
__device__ __forceinline__ float warp_sum_tree(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// C independent ordered chains over the same terms: s[c] = fl(s[c] + a[i]) for
// i in order. The chains interleave, so C of them cost about one chain's
// latency. `a` is 16-byte aligned shared memory that stays readable 8 floats
// past n: the loads run 8 terms ahead without bounds checks (the values read
// past n are never used).
template <int C>
__device__ __forceinline__ void ordered_chains(float (&s)[C], const float* a, int n) {
  const float4* a4 = (const float4*)a;
  const int n8 = n >> 3;
  float4 b0 = a4[0], b1 = a4[1];
  for (int i = 0; i < n8; i++) {
    const float4 c0 = b0, c1 = b1;
    b0 = a4[2 * i + 2];
    b1 = a4[2 * i + 3];
    const float v[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
    for (int u = 0; u < 8; u++)
#pragma unroll
      for (int c = 0; c < C; c++) s[c] = __fadd_rn(s[c], v[u]);
  }
  for (int k = n8 * 8; k < n; k++)
#pragma unroll
    for (int c = 0; c < C; c++) s[c] = __fadd_rn(s[c], a[k]);
}

// Bytes of slack a term buffer needs past its last element for ordered_chains.
constexpr int kChainSlackBytes = 32;

// ---------------------------------------------------------------------------
// Speculative parallel form of a one-accumulator float sum.
//
// The reference sums with one float accumulator, s = fl(s + t[i]) for i in
// order (rms_norm's sum of squares, src/ops_cpu.cpp:154-157; the softmax
// denominator, src/ops_cpu.cpp:331-336). The chain is serial, but it is a
// deterministic function of its start value. Here the CTA cuts t into NW
// contiguous segments (one per warp). Every warp sums its own segment
// (any order: it is only an estimate); warp w then estimates the chain's value
// at its segment's start as the sum of the preceding segments' sums and runs
// its segment from 32*C consecutive floats around that estimate at once (lane
// l, chain c starts from the bit pattern bits(estimate) - 16C + 32c + l).
// Thread 0 then walks the segments in order: with the exact chain value s at
// segment w's start known, the segment's end is the end of the candidate that
// started from exactly bits(s); if no candidate did, thread 0 runs that
// segment serially from s. Either way the result equals the serial chain bit
// for bit. The serial chain drifts from the exact prefix sum by a walk of
// rounding errors (up to a few tens of ulps at n in the thousands), so the
// fallback is rare and costs one segment when taken.
//
// Measured on B200 (one CTA, 8 warps, warm): n = 896 takes 2.6k cycles against
// 4.8k for one thread's chain, n = 3584 6.2k against 15.8k; below n of about
// 160 the serial chain is faster.
//
// Every thread of the CTA (NT of them) must call it: it synchronizes the CTA.
// `t` is 16-byte aligned shared memory readable kChainSlackBytes past n;
// `scratch` is shared memory of spec_sum_scratch_bytes(NT / 32, C) bytes,
// 4-byte aligned.
// ---------------------------------------------------------------------------
__host__ __device__ constexpr int spec_sum_scratch_bytes(int nw, int c) {
  return nw * 4 + nw * 32 * c * 4 + 16 + nw * 4;
}

template <int NT, int C>
__device__ __forceinline__ float spec_ordered_sum(const float* t, int n, uint8_t* scratch) {
  constexpr int NW = NT / 32;
  constexpr unsigned NC = 32u * C;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  unsigned* base = (unsigned*)scratch;
  float* ends = (float*)(scratch + NW * 4);
  float* result = ends + NW * NC;
  float* segsum = result + 4;
  const int S = (((n + NW - 1) / NW) + 7) & ~7;  // segment length, keeps 32-byte alignment
  const int b = warp * S;
  const int len = max(0, min(S, n - b));
  {
    float a0 = 0.0f, a1 = 0.0f;
    int i = lane;
    for (; i + 32 < len; i += 64) {
      a0 += t[b + i];
      a1 += t[b + i + 32];
    }
    if (i < len) a0 += t[b + i];
    float e = a0 + a1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) e += __shfl_xor_sync(0xffffffffu, e, o);
    if (lane == 0) segsum[warp] = e;
  }
  __syncthreads();
  if (len > 0) {
    if (warp == 0) {
      float s[1] = {0.0f};
      ordered_chains<1>(s, t, len);
      if (lane == 0) ends[0] = s[0];
    } else {
      float e = lane < warp ? segsum[lane] : 0.0f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) e += __shfl_xor_sync(0xffffffffu, e, o);
      const unsigned b0 = __float_as_uint(e) - 16u * C;
      float s[C];
#pragma unroll
      for (int c = 0; c < C; c++) s[c] = __uint_as_float(b0 + 32u * c + lane);
      ordered_chains<C>(s, t + b, len);
#pragma unroll
      for (int c = 0; c < C; c++) ends[warp * NC + 32 * c + lane] = s[c];
      if (lane == 0) base[warp] = b0;
    }
  }
  __syncthreads();
  if (tid == 0) {
    float s = n > 0 ? ends[0] : 0.0f;
    int miss = NW;
#pragma unroll
    for (int w = 1; w < NW; w++) {
      const bool live = w * S < n && miss == NW;
      const unsigned idx = __float_as_uint(s) - (live ? base[w] : 0u);
      const bool hit = live && idx < NC;
      if (live && !hit) miss = w;
      s = hit ? ends[w * NC + idx] : s;
    }
    // Serial from the first segment without a matching candidate; later
    // segments still take their candidate when one matches.
    for (int w = miss; w < NW && w * S < n; w++) {
      const unsigned idx = __float_as_uint(s) - base[w];
      if (w > miss && idx < NC) {
        s = ends[w * NC + idx];
      } else {
        float r[1] = {s};
        ordered_chains<1>(r, t + w * S, min(S, n - w * S));
        s = r[0];
      }
    }
    *result = s;
  }
  __syncthreads();
  return *result;
}

// One Q8_0_ACT block value: the reference's per-block quantizer
// (src/quant.cpp:199-218) for the element this lane holds; the warp holds the
// block's 32 elements. Returns q, writes d (same on every lane).
__device__ __forceinline__ int8_t quantize_lane(float v, float* d_out) {
  // max |v| over the block: the bit patterns of non-negative floats order like
  // their values, so one integer warp reduction gives the exact maximum.
  const float amax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v))));
  float d = __fdiv_rn(amax, 127.0f);
  float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
  int q = __float2int_rn(__fmul_rn(v, id));
  q = q > 127 ? 127 : (q < -127 ? -127 : q);
  *d_out = d;
  return (int8_t)q;
}

// Packed Q8_0 layout (see mi_cuda_q8_0_pack): qs plane of n_pad*K bytes, then
// the fp16 scale plane. Row r, block b:
//   qs at (r/4)*4K + b*128 + (r%4)*32, scale at plane + ((r/4)*nb + b)*4 + r%4.
__device__ __forceinline__ const int8_t* packed_qs(const uint8_t* w, int64_t K, int64_t r,
                                                   int64_t b) {
  return (const int8_t*)(w + (r >> 2) * 4 * K + b * 128 + (r & 3) * 32);
}
__device__ __forceinline__ float packed_scale(const uint8_t* w, int64_t K, int64_t n_pad,
                                              int64_t r, int64_t b) {
  const __half* d = (const __half*)(w + n_pad * K);
  return __half2float(d[((r >> 2) * (K / 32) + b) * 4 + (r & 3)]);
}

}  // namespace mi
