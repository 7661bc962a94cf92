// Batched-prefill Q8_0 GEMM on the 5th-generation tensor cores (tcgen05),
// bit-identical to the reference's per-(row, token) dot.
//
// The reference's dot (ref src/quant_avx2.cpp:170-181, called per output
// element by mul_mat, src/ops_cpu.cpp:226-237) keeps, per 32-element block,
// eight int32 lane partials p_j = sum_{e<4} w[4j+e] * a[4j+e], converts them
// to float and advances eight FMA chains acc_j = fma((float)p_j, d_w * d_a,
// acc_j); hsum_ps adds the lanes at the end as
// ((l0+l4)+(l1+l5))+((l2+l6)+(l3+l7)).
//
// A tensor-core MMA over the block returns sum_j p_j, which those chains
// cannot use. So the activation operand is lane-expanded: column (t, j) of B
// holds token t's elements 4j..4j+3 at their own K positions and zeros at the
// other 28, and D[r][(t, j)] = p_j(r, t) exactly. The MMA runs as kind::f16
// with f32 accumulation: int8 values are exact in fp16, every product is an
// integer of magnitude <= 16384, every partial sum an integer below 2^17, so
// nothing rounds, and the partials arrive in TMEM already as the floats the
// chains need. The chains -- the part whose rounding order is fixed -- run on
// the CUDA cores, two per instruction (fma.rn.f32x2).
//
// The lane split also halves the MMA work: lanes 0-3 read only elements 0-15
// of the block and lanes 4-7 only 16-31, so a block is two M128 x N128 x K16
// MMAs, one per half, each over its 16 K elements and its 128 (token, lane)
// columns.
//
// Weights use a prefill copy (made once at load by pack_tc_kernel from the
// decode layout): per 128-row tile and block, the 128 x 32 quants as fp16 in
// the MMA's K-major canonical layout (8 KB, copied into shared memory as is)
// and the 128 fp16 scales as floats.
//
// CTA tile: 128 weight rows x 32 tokens, the whole K loop; 20 warps (96
// registers each, five per register-file quadrant), specialised:
//   * warps 0-15, epilogue: warp w owns TMEM lanes 32(w%4)..
//     (32 rows) and tokens 8(w/4)..8(w/4)+7: 8 tokens x 8 lane chains per row
//     in registers. Per block: wait for the MMA, tcgen05.ld the partials,
//     advance the chains;
//   * warp 16, producer: stages of 4 blocks, four copies per stage -- the
//     weight tiles and their scales (one bulk copy each), the 32 tokens'
//     activation quants and scales (two 2-D tensor copies of the row-major
//     activation, 32 rows x 128 B and 32 rows x 4 floats; rows past the last
//     token and blocks past K arrive as zeros). When a row of scales is not a
//     multiple of 16 bytes (K % 128 != 0) the scales come by one 4-byte
//     cp.async per token and block instead;
//   * warps 17-18, B expansion: each block's activation int8 -> fp16 into its
//     lane-expanded layout (a ring of 4 buffers whose zeros are written once);
//   * warp 19, MMA issue (one thread), and TMEM allocation.
// TMEM holds two buffers of 256 columns: the MMAs of block b + 1 run while the
// epilogue reads block b. Every wait is bounded; on expiry the kernel records
// MI_CUDA_ERR_TIMEOUT, all roles stop, and TMEM is released.
#include <cuda.h>
#include <cuda_fp16.h>

#include "mi_device.cuh"

namespace mi {

namespace {

constexpr int kTcRows = 128;  // weight rows per CTA (MMA M)
constexpr int kTcTok = 32;    // tokens per CTA
constexpr int kTcG = 4;       // blocks per stage
constexpr int kTcStages = 4;
constexpr int kTcBx = 4;      // expanded-B ring
constexpr int kTcEpiWarps = 16;
constexpr int kTcThreads = (kTcEpiWarps + 4) * 32;
constexpr int kWarpProducer = 16, kWarpExpand0 = 17, kWarpMma = 19;
constexpr uint32_t kTcCols = 512;  // TMEM: two buffers x two halves x 128 columns

struct TcSmem {
  // staging ring: slot s holds stage i (blocks 4i..4i+3) for i % S == s
  static constexpr int wa = 0;                 // weight tiles, fp16 canonical, [4 blocks][8 KB]
  static constexpr int sw = wa + kTcG * 8192;  // weight scales, float [4][128]
  static constexpr int aq = sw + kTcG * 512;   // activation quants, [32 tokens][4 blocks x 32]
  static constexpr int da = aq + kTcTok * kTcG * 32;   // activation scales, float [32 tokens][4]
  static constexpr int stage = da + kTcTok * kTcG * 4;  // 39424
  static constexpr int bx0 = kTcStages * stage;  // expanded-B ring, 8 KB each: 2 halves x 16 column
                                                 // groups x 2 K chunks x 128 B
  static constexpr int bars = bx0 + kTcBx * 8192;
  // full[S], empty[S], bready[4], bfree[4], tfull[2], tempty[2]
  static constexpr int misc = bars + (2 * kTcStages + 2 * kTcBx + 4) * 8;
  // TMEM base, abort flag, stages issued, MMA blocks issued
  static constexpr int total = misc + 16 + 1024;  // + alignment slack of the base
};
static_assert(TcSmem::stage % 128 == 0 && TcSmem::aq % 128 == 0 && TcSmem::da % 128 == 0, "stage layout");
static_assert(kTcRows * 33 * 4 <= TcSmem::bx0, "gate/up exchange fits the staging ring");

// Shared-memory matrix descriptor, no swizzle, K-major: core matrices of 8
// rows x 16 B; lbo = byte distance between K-adjacent core matrices, sbo =
// between M/N-adjacent ones; bit 46 = descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)(lbo >> 4) << 16) |
         ((uint64_t)(sbo >> 4) << 32) | (1ull << 46);
}
// Instruction descriptor: D f32 (bit 4), A and B f16 (format 0), both K-major,
// N = 128 (N >> 3 at bit 17), M = 128 (M >> 4 at bit 24).
constexpr uint32_t kTcIdesc = (1u << 4) | ((128u >> 3) << 17) | ((128u >> 4) << 24);

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc) {
  const uint32_t zero = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kTcIdesc), "r"(zero), "r"(zero)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// tcgen05.wait::ld, with the loaded registers threaded through it so that no
// use of them can be scheduled before the wait.
__device__ __forceinline__ void tmem_wait_ld2(uint32_t (&r)[16], uint32_t (&s)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(s[0]), "+r"(s[1]), "+r"(s[2]), "+r"(s[3]), "+r"(s[4]), "+r"(s[5]), "+r"(s[6]),
                 "+r"(s[7]), "+r"(s[8]), "+r"(s[9]), "+r"(s[10]), "+r"(s[11]), "+r"(s[12]), "+r"(s[13]),
                 "+r"(s[14]), "+r"(s[15])
               :
               : "memory");
}

__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void mbar_arrive_one(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void cp_async4_tc(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
// Arrives on `bar` once this thread's earlier cp.async copies have landed (the
// arrival is part of the barrier's expected count).
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}
// 2-D tiled tensor copy global -> shared, completing on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int32_t x, int32_t y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

// try_wait that lets the thread sleep until the phase completes (or about a
// microsecond passes), so that waiting warps leave their issue slots to the
// warps that compute.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(1000u)
      : "memory");
  return ok != 0;
}

// Bounded wait of one thread: gives up when another role has flagged an
// abort, or after kSpinLimit polls (then it flags one).
__device__ __forceinline__ bool tc_wait1(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int32_t* err) {
  for (uint32_t it = 0;; it++) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    if ((it & 31u) == 31u && *abort_flag) return false;
    if (it >= kSpinLimit) {
      *abort_flag = 1;
      if (err) atomicExch(err, 5 /* MI_CUDA_ERR_TIMEOUT */);
      return false;
    }
  }
}
// The same for a whole warp (every lane polls, the warp leaves together).
// Re-polling a completed phase is safe: none of the barriers a warp waits on
// can complete its next phase without that warp's own arrival.
__device__ __forceinline__ bool tc_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                             int32_t* err) {
  for (uint32_t it = 0;; it++) {
    if (__all_sync(0xffffffffu, mbar_try_wait_sleep(bar, parity))) return true;
    if ((it & 31u) == 31u && __any_sync(0xffffffffu, *abort_flag != 0)) return false;
    if (it >= kSpinLimit) {
      *abort_flag = 1;
      if (err && (threadIdx.x & 31) == 0) atomicExch(err, 5 /* MI_CUDA_ERR_TIMEOUT */);
      return false;
    }
  }
}

}  // namespace

// Decode-layout Q8_0 rows -> the prefill GEMM's tile layout (see above).
// One thread per (row, block); rows at or beyond npad become zero rows.
__global__ void pack_tc_kernel(const uint8_t* w, int64_t K, int64_t npad, int64_t n_tc, uint8_t* wt, float* st) {
  const int64_t nb = K / 32;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n_tc * nb) return;
  const int64_t r = idx & (kTcRows - 1), tb = idx >> 7;  // tb = tile * nb + block
  const int64_t R = (tb / nb) * kTcRows + r, b = tb % nb;
  uint8_t* dst = wt + tb * 8192 + (r >> 3) * 512 + (r & 7) * 16;  // + K chunk * 128
  const int8_t* src = R < npad ? packed_qs(w, K, R, b) : nullptr;
#pragma unroll
  for (int kc = 0; kc < 4; kc++) {
    __align__(16) __half h[8];
#pragma unroll
    for (int e = 0; e < 8; e++) h[e] = __short2half_rn(src ? (short)src[kc * 8 + e] : (short)0);
    *(uint4*)(dst + kc * 128) = *(const uint4*)h;
  }
  st[idx] = src ? packed_scale(w, K, npad, R, b) : 0.0f;
}

cudaError_t launch_pack_tc(const uint8_t* w, int64_t K, int64_t npad, int64_t n_tc, uint8_t* wt, float* st,
                           cudaStream_t s) {
  if (K % 32 != 0 || n_tc % kTcRows != 0) return cudaErrorInvalidValue;
  const int64_t total = n_tc * (K / 32);
  if (total == 0) return cudaSuccess;
  pack_tc_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(w, K, npad, n_tc, wt, st);
  return cudaGetLastError();
}

int64_t tc_rows(int64_t npad) { return (npad + kTcRows - 1) / kTcRows * kTcRows; }
size_t tc_weight_bytes(int64_t n_tc, int64_t K) { return (size_t)n_tc * (size_t)K * 2; }

__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_tc_kernel(const GemmParams p, const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_d,
                   int da_tma) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // tensor-copy destinations want 128-byte alignment: align the base to 1 KB
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nb = (int)(p.K >> 5);
  const int n_st = (nb + kTcG - 1) / kTcG;
  const int64_t rt = blockIdx.x, T0 = (int64_t)blockIdx.y * kTcTok;
  const int n_tok = p.M - T0 < kTcTok ? (int)(p.M - T0) : kTcTok;
  uint64_t* full = (uint64_t*)(smem + TcSmem::bars);
  uint64_t* empty = full + kTcStages;
  uint64_t* bready = empty + kTcStages;
  uint64_t* bfree = bready + kTcBx;
  uint64_t* tfull = bfree + kTcBx;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_base = (uint32_t*)(smem + TcSmem::misc);
  volatile int* abort_flag = (volatile int*)(smem + TcSmem::misc + 4);
  volatile int* n_issued = (volatile int*)(smem + TcSmem::misc + 8);  // [0] stages, [1] MMA blocks

  if (tid == 0) {
    for (int s = 0; s < kTcStages; s++) {
      // the producer's expect-tx arrival (+ 32 cp.async arrivals when the
      // activation scales come by cp.async)
      mbar_init(&full[s], da_tma ? 1 : 33);
      mbar_init(&empty[s], kTcEpiWarps + 2);  // epilogue warps + the two expansion warps
    }
    for (int i = 0; i < kTcBx; i++) {
      mbar_init(&bready[i], 2);
      mbar_init(&bfree[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], kTcEpiWarps);
    }
    *abort_flag = 0;
    n_issued[0] = n_issued[1] = 0;
    fence_mbar_init();
  }
  // the expanded B buffers are zero except at the lanes' own K positions,
  // which every expansion rewrites: zero them once
  for (int i = tid; i < kTcBx * 512; i += kTcThreads)
    *(uint4*)(smem + TcSmem::bx0 + i * 16) = make_uint4(0, 0, 0, 0);
  if (warp == kWarpMma) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_base)),
                 "r"(kTcCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base;

  // acc[h][j'][u]: lane j = 4h + j' of tokens 8*tg + 2u (x) and 8*tg + 2u + 1 (y)
  float2 acc[2][4][4];
  const int q = warp & 3, tg = (warp >> 2) & 3;

  if (warp >= kTcEpiWarps) {
    if (warp == kWarpProducer) {
      // ---------------- producer ----------------
      const uint8_t* wt = p.wt + rt * (int64_t)nb * 8192;
      const float* stp = p.st + rt * (int64_t)nb * kTcRows;
      const int64_t d_stride = p.act_stride >> 5;
      for (int i = 0; i < n_st; i++) {
        const int s = i % kTcStages, b0 = i * kTcG, nv = min(kTcG, nb - b0);
        if (i >= kTcStages && !tc_wait_warp(&empty[s], ((i / kTcStages) + 1) & 1, abort_flag, p.err)) break;
        uint8_t* st = smem + s * TcSmem::stage;
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[s], (uint32_t)nv * (8192 + 512) + kTcTok * kTcG * 32 +
                                              (da_tma ? kTcTok * kTcG * 4 : 0));
          bulk_load(st + TcSmem::wa, wt + (int64_t)b0 * 8192, (uint32_t)nv * 8192, &full[s]);
          bulk_load(st + TcSmem::sw, stp + (int64_t)b0 * kTcRows, (uint32_t)nv * 512, &full[s]);
          tma_load_2d(st + TcSmem::aq, &tm_q, b0 * 32, (int32_t)T0, &full[s]);
          if (da_tma) tma_load_2d(st + TcSmem::da, &tm_d, b0, (int32_t)T0, &full[s]);
          n_issued[0] = i + 1;
        }
        if (!da_tma) {
          __syncwarp();
          if (lane < n_tok)
            for (int j = 0; j < nv; j++)
              cp_async4_tc(st + TcSmem::da + (lane * kTcG + j) * 4, p.act_d + (T0 + lane) * d_stride + b0 + j);
          cp_async_arrive_noinc(&full[s]);
        }
      }
    } else if (warp < kWarpMma) {
      // ---------------- B expansion: tokens 16e..16e+15 ----------------
      const int e = warp - kWarpExpand0;
      for (int b = 0; b < nb; b++) {
        const int i = b / kTcG, s = i % kTcStages, g = b % kTcG, c = b % kTcBx;
        if (g == 0 && !tc_wait_warp(&full[s], (i / kTcStages) & 1, abort_flag, p.err)) break;
        if (b >= kTcBx && !tc_wait_warp(&bfree[c], ((b / kTcBx) + 1) & 1, abort_flag, p.err)) break;
        const uint8_t* st = smem + s * TcSmem::stage;
        uint8_t* bx = smem + TcSmem::bx0 + c * 8192;
#pragma unroll
        for (int k = 0; k < 4; k++) {
          // lane j of token t: 4 int8 -> 4 fp16 at column (t/2)*8 + j'*2 + t%2 of half j/4
          const int pc = lane + 32 * k, t = 16 * e + (pc >> 3), j = pc & 7, h = j >> 2, jp = j & 3;
          const uint32_t a4 = *(const uint32_t*)(st + TcSmem::aq + t * (kTcG * 32) + g * 32 + j * 4);
          const __half2 kk = __halves2half2(__float2half_rn(1152.0f), __float2half_rn(1152.0f));
          uint32_t lo = __byte_perm(a4, 0x64646464u, 0x5140) ^ 0x00800080u;
          uint32_t hi = __byte_perm(a4, 0x64646464u, 0x7362) ^ 0x00800080u;
          __half2 l2 = __hsub2(*reinterpret_cast<const __half2*>(&lo), kk);
          __half2 h2 = __hsub2(*reinterpret_cast<const __half2*>(&hi), kk);
          *(uint2*)(bx + h * 4096 + (t >> 1) * 256 + (jp >> 1) * 128 + (jp * 2 + (t & 1)) * 16 + (jp & 1) * 8) =
              make_uint2(*reinterpret_cast<uint32_t*>(&l2), *reinterpret_cast<uint32_t*>(&h2));
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive_one(&bready[c]);
          if (g == kTcG - 1 || b == nb - 1) mbar_arrive_one(&empty[s]);
        }
      }
    } else if (lane == 0) {
      // ---------------- MMA issue ----------------
      // This thread's loop is on the critical path of every block, so it does
      // as little as possible: the descriptors are the first stage's plus the
      // operand's offset in 16-byte units (shared addresses stay below 2^18,
      // so the 14-bit address field never carries).
      const uint64_t a0 = umma_desc(smem_addr(smem + TcSmem::wa), 128, 512);
      const uint64_t b0 = umma_desc(smem_addr(smem + TcSmem::bx0), 128, 256);
      int s = 0, g = 0, c = 0;
      uint32_t pf = 0, pb = 0, pt = 0;  // phases of full[s], bready[c], tempty[d] to wait for
      for (int b = 0; b < nb; b++) {
        const int d = b & 1;
        if (g == 0 && !tc_wait1(&full[s], pf, abort_flag, p.err)) break;
        if (!tc_wait1(&bready[c], pb, abort_flag, p.err)) break;
        if (b >= 2 && !tc_wait1(&tempty[d], pt, abort_flag, p.err)) break;
        tc_fence_after();
        const uint64_t ad = a0 + (uint64_t)((s * TcSmem::stage + g * 8192) >> 4);
        const uint64_t bd = b0 + (uint64_t)((c * 8192) >> 4);
        const uint32_t dt = tmem + (uint32_t)d * 256;
        umma_f16(dt, ad, bd);
        umma_f16(dt + 128, ad + (256 >> 4), bd + (4096 >> 4));
        umma_commit(&tfull[d]);
        umma_commit(&bfree[c]);
        n_issued[1] = b + 1;
        // advance the ring positions and the phases they wait for
        if (d == 1 && b >= 2) pt ^= 1u;
        if (++c == kTcBx) {
          c = 0;
          pb ^= 1u;
        }
        if (++g == kTcG) {
          g = 0;
          if (++s == kTcStages) {
            s = 0;
            pf ^= 1u;
          }
        }
      }
    }
  } else {
    // ---------------- epilogue ----------------
#pragma unroll
    for (int h = 0; h < 2; h++)
#pragma unroll
      for (int j = 0; j < 4; j++)
#pragma unroll
        for (int u = 0; u < 4; u++) acc[h][j][u] = make_float2(0.0f, 0.0f);
    for (int b = 0; b < nb; b++) {
      const int i = b / kTcG, g = b % kTcG, d = b & 1;
      // (the stage's scales: landed long ago, but observed by this warp itself)
      if (g == 0 && !tc_wait_warp(&full[i % kTcStages], (i / kTcStages) & 1, abort_flag, p.err)) break;
      if (!tc_wait_warp(&tfull[d], (b >> 1) & 1, abort_flag, p.err)) break;
      tc_fence_after();
      // columns 32*tg .. +31 of each half: register c = token pair c/8, lane
      // j' = (c%8)/2, token parity c%2; loaded in four 16-column pieces
      const uint32_t tb = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)d * 256 + 32u * tg;
      uint32_t ra[16], rb[16];
      tmem_ld16(tb, ra);
      tmem_ld16(tb + 16, rb);
      const uint8_t* st = smem + (i % kTcStages) * TcSmem::stage;
      const float sw = ((const float*)(st + TcSmem::sw + g * 512))[32 * q + lane];
      const float* dab = (const float*)(st + TcSmem::da) + (8 * tg) * kTcG + g;
      const float2 sw2 = make_float2(sw, sw);
      float2 dp[4];
#pragma unroll
      for (int u = 0; u < 4; u++) dp[u] = __fmul2_rn(sw2, make_float2(dab[(2 * u) * kTcG], dab[(2 * u + 1) * kTcG]));
      tmem_wait_ld2(ra, rb);
#pragma unroll
      for (int hp = 0; hp < 2; hp++) {
        // columns 0-15 (ra: token pairs 0-1) and 16-31 (rb: token pairs 2-3) of half hp
#pragma unroll
        for (int c2 = 0; c2 < 8; c2++)
          acc[hp][c2 & 3][c2 >> 2] = __ffma2_rn(make_float2(__uint_as_float(ra[2 * c2]), __uint_as_float(ra[2 * c2 + 1])),
                                                dp[c2 >> 2], acc[hp][c2 & 3][c2 >> 2]);
        if (hp == 0) tmem_ld16(tb + 128, ra);
#pragma unroll
        for (int c2 = 0; c2 < 8; c2++)
          acc[hp][c2 & 3][2 + (c2 >> 2)] =
              __ffma2_rn(make_float2(__uint_as_float(rb[2 * c2]), __uint_as_float(rb[2 * c2 + 1])), dp[2 + (c2 >> 2)],
                         acc[hp][c2 & 3][2 + (c2 >> 2)]);
        if (hp == 0) {
          tmem_ld16(tb + 144, rb);
          tmem_wait_ld2(ra, rb);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_one(&tempty[d]);
        }
      }
      if (g == kTcG - 1 || b == nb - 1) {
        __syncwarp();
        if (lane == 0) mbar_arrive_one(&empty[i % kTcStages]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (tid == kWarpMma * 32) {
    // Before TMEM and shared memory are released, the last MMAs and any copies
    // still in flight must have landed (bounded; only an abort leaves any).
    const int n_mma = n_issued[1], n_loaded = n_issued[0];
    if (n_mma > 0) {
      const int b = n_mma - 1;
      for (uint32_t it = 0; it < kSpinLimit && !mbar_test(&tfull[b & 1], (b >> 1) & 1); it++) {
      }
    }
    for (int i = max(0, n_loaded - kTcStages); i < n_loaded; i++)
      for (uint32_t it = 0; it < kSpinLimit && !mbar_test(&full[i % kTcStages], (i / kTcStages) & 1); it++) {
      }
  }
  tc_fence_before();
  __syncthreads();
  if (*abort_flag == 0 && warp < kTcEpiWarps) {
    const int64_t row = rt * kTcRows + 32 * q + lane;
    // hsum_ps per (row, token)
    float2 dot[4];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const float2 s04 = __fadd2_rn(acc[0][0][u], acc[1][0][u]), s15 = __fadd2_rn(acc[0][1][u], acc[1][1][u]);
      const float2 s26 = __fadd2_rn(acc[0][2][u], acc[1][2][u]), s37 = __fadd2_rn(acc[0][3][u], acc[1][3][u]);
      dot[u] = __fadd2_rn(__fadd2_rn(s04, s15), __fadd2_rn(s26, s37));
    }
    if (p.epi == EPI_SILU_GATEUP_Q) {
      // The tile's 128 packed rows are the gate/up rows of two 32-element
      // blocks of the FFN activation: silu(gate) * up per element, then the
      // down projection's quantize node, per token.
      float* res = (float*)smem;  // [128 rows][33]
#pragma unroll
      for (int u = 0; u < 4; u++) {
        res[(32 * q + lane) * 33 + 8 * tg + 2 * u] = dot[u].x;
        res[(32 * q + lane) * 33 + 8 * tg + 2 * u + 1] = dot[u].y;
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kTcEpiWarps * 32) : "memory");
      const int64_t n_ffn = p.N >> 6;
      const int e = lane, lr = (e >> 2) * 8 + (e & 3);
      for (int item = warp; item < 2 * kTcTok; item += kTcEpiWarps) {
        const int fb = item / kTcTok, t = item % kTcTok;
        const int64_t blk = rt * 2 + fb;
        if (t >= n_tok || blk >= n_ffn) continue;
        const int64_t tok = T0 + t;
        const float v = __fmul_rn(silu_exact(res[(fb * 64 + lr) * 33 + t], p.et), res[(fb * 64 + lr + 4) * 33 + t]);
        float dq;
        const int8_t qv = quantize_lane(v, &dq);
        p.q_out[tok * p.q_stride + blk * 32 + e] = qv;
        if (e == 0) p.d_out[tok * (p.q_stride >> 5) + blk] = dq;
      }
    } else if (row < p.N) {
#pragma unroll
      for (int u = 0; u < 4; u++)
#pragma unroll
        for (int k = 0; k < 2; k++) {
          const int t = 8 * tg + 2 * u + k;
          if (t >= n_tok) continue;
          const int64_t tok = T0 + t;
          float v = k ? dot[u].y : dot[u].x;
          if (p.epi == EPI_BIAS) v = __fadd_rn(v, p.bias[row]);
          else if (p.epi == EPI_RESID) v = __fadd_rn(p.resid[tok * p.out_stride + row], v);
          p.out[tok * p.out_stride + row] = v;
        }
    }
  }
  if (warp == kWarpMma) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcCols));
  }
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against the driver library).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  return fn;
}

// A 2-D row-major [rows][cols] map with a [box_rows][box_cols] box;
// out-of-range elements read as zero.
bool make_map_2d(CUtensorMap* m, CUtensorMapDataType type, const void* base, int64_t cols, int64_t rows,
                 int64_t row_bytes, int box_cols, int box_rows) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, type, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t prepare_gemm_tc_kernel() {
  return cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TcSmem::total);
}

cudaError_t launch_gemm_tc(const GemmParams& p, cudaStream_t s) {
  if (p.M <= 0) return cudaSuccess;
  const int64_t n_tc = tc_rows(p.n_pad);
  if (p.K % 32 != 0 || !p.wt || !p.st || p.act_stride % 32 != 0 || p.act_stride < p.K ||
      (p.epi == EPI_SILU_GATEUP_Q && p.N % 64 != 0) || p.M > INT32_MAX)
    return cudaErrorInvalidValue;
  // activation quants [M][K] bytes (row stride act_stride), scales [M][K/32]
  // floats (row stride act_stride / 32 floats)
  CUtensorMap tq{}, td{};
  if (!make_map_2d(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, p.act_qs, p.K, p.M, p.act_stride, kTcG * 32, kTcTok))
    return cudaErrorInvalidValue;
  const int64_t d_row = (p.act_stride >> 5) * 4;
  const int da_tma =
      d_row % 16 == 0 && make_map_2d(&td, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, p.act_d, p.K >> 5, p.M, d_row, kTcG, kTcTok);
  dim3 grid((unsigned)(n_tc / kTcRows), (unsigned)((p.M + kTcTok - 1) / kTcTok));
  gemm_tc_kernel<<<grid, kTcThreads, TcSmem::total, s>>>(p, tq, td, da_tma);
  return cudaGetLastError();
}

}  // namespace mi
