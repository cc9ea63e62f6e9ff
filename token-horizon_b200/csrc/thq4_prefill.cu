// thq4_prefill.cu -- the prefill GEMM: y[m][n] = x[m][k] . dequant(W)[n][k]^T
// for m > 8 tokens, on the 5th-generation tensor cores (tcgen05, TMEM).
//
// Replaces the reference's prefill families AffineQpf (pf_tile / pf_tile_gu,
// engine/src/quant_kernel.rs:3930-5294), AffineQmppPrefill (:2068-2238,
// 3737-3928) and the dequant + dense GEMM fallback (AffineDequant + linear,
// :1743-1782, qwen35.rs:2035-2056).  Semantics are the reference CPU path's:
// every weight is dequantised to bf16(q * s + b) (qwen35.rs:110-134), the
// product accumulates in f32 over the whole of k, and the output is bf16
// (or f32).  The gate/up form applies the reference's SwiGLU epilogue,
// bf16(silu(bf16 g) * bf16 u) (qwen35.rs:711-884).
//
// Bound: tensor throughput (51.5 GFLOP per 512-token call of the BASELINE
// 12288 x 4096 shape against 28 MB of weights).  The tensor core's operand
// reads, the TMA fills and any dequantised tile written to shared memory all
// share the SM's 128 bytes/clock of shared-memory bandwidth, which a design
// with the bf16 weight tile in shared memory exhausts at ~55% of peak.  So:
//   - the weights are the A operand and live in TMEM: eight dequant warps
//     turn each raw slab-group (128 rows x 64 k: 4096 bytes of nibbles + 512
//     of scales, one bulk copy) into bf16 in registers and store it straight
//     into a TMEM ring (tcgen05.st, thread i -> row lane i).  A nibble
//     becomes an f32 by OR-ing it into the mantissa of 2^23 and subtracting
//     2^23 (exact); high nibbles stay in bits 4..7 and take s/16 (exact);
//     pairs go through packed f32x2 add / fma and one cvt to bf16x2;
//   - the activations are the B operand: x tiles of 256 (gate/up: 128)
//     tokens x 64 k, loaded by a 2-D TMA with 128-byte swizzle (zero fill
//     past m) into a shared-memory ring;
//   - a second producer warp streams the raw slab-groups into their own
//     ring, released as soon as the dequant warps have read a stage (not
//     when the MMA is done);
//   - one thread issues tcgen05.mma.kind::f16 (bf16 in, f32 accumulate in
//     TMEM), M = 128 output rows x N = 256 tokens per k-step of 16, and
//     commits each stage back to the producer;
//   - persistent CTAs (one per SM) walk tiles of one slab (128 rows) x 256
//     tokens, token tiles fastest, so a slab is fetched from HBM once and
//     re-read from L2; D has one or two TMEM buffers (two where TMEM has
//     room, so the next tile's MMAs overlap this tile's epilogue); eight
//     epilogue warps drain D (tcgen05.ld) -- a warp's
//     32 lanes hold 32 consecutive output rows, so each store of a token's
//     values is one contiguous 64-byte segment of y;
//   - every wait is bounded; a timeout raises kStatusTimeout, sets a CTA-wide
//     abort flag that ends every role's loop, and the CTA still frees TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "thq4_common.cuh"
#include "thq4_internal.h"

namespace thq4 {
namespace {

constexpr int kBN = 128;  // output rows per tile (one slab): the MMA's M
constexpr int kBK = 64;   // k per stage (one quant group)
constexpr int kDeqWarps = 8, kEpiWarps = 8;
// dequant warps are 0..7; the x producer, the MMA issuer and the weight producer follow the epilogue warps
constexpr int kWarpEpi0 = 8, kWarpProd = 16, kWarpMma = 17, kWarpRaw = 18;
constexpr int kPfThreads = 19 * 32;
constexpr uint32_t kXBox = 128 * kBK * 2;   // one 128-token x box, bytes
constexpr uint32_t kRawStage = 4096 + 512;  // one slab-group
constexpr int kAcolsPerStage = kBK / 2;     // TMEM columns of one stage's A (bf16 pairs)

struct PfArgs {
  const uint8_t *qw[2];  // gate (or the only) weight, up
  const uint8_t *sb[2];
  void *y;
  uint32_t *status;
  int m, n, ng;
  int m_tiles, tiles;
};

// One unit of work: output slab nt for activation rows [row0, row_end).
struct PfUnit {
  int nt, row0, row_end;
  const uint8_t *qw[2];
  const uint8_t *sb[2];
};
template <int BT>
__device__ __forceinline__ PfUnit pf_unit(const PfArgs &a, int u) {
  PfUnit x;
  const int mt = u % a.m_tiles;
  x.nt = u / a.m_tiles;
  x.row0 = mt * BT;
  x.row_end = a.m;
#pragma unroll
  for (int si = 0; si < 2; ++si) {
    x.qw[si] = a.qw[si];
    x.sb[si] = a.sb[si];
  }
  return x;
}

// NS weight streams (1, or 2 for gate/up), BT tokens per tile, S stages of
// x (shared memory) and of dequantised A (TMEM), RW stages of raw weights
// (shared memory), NB accumulator buffers in TMEM.  The raw ring is released
// as soon as the dequant warps have read a stage, so it can run far ahead of
// the tensor core: it is what keeps HBM requests in flight when a tile has
// few tokens.
template <int NS, int BT, int S, int RW, int NB>
struct PfCfg {
  static constexpr uint32_t x_stage = BT * kBK * 2;
  static constexpr uint32_t x_off = 0;
  static constexpr uint32_t raw_off = x_off + S * x_stage;
  // a bf16 output tile [BT tokens][128 rows], staged between TMEM and y
  static constexpr uint32_t y_off = raw_off + RW * NS * kRawStage;
  static constexpr uint32_t bar_off = y_off + BT * kBN * 2;
  // barriers: xfull[S], deq[S], empty[S], rawfull[RW], rawempty[RW],
  // accf[NB], acce[NB], yfull, ydone
  static constexpr int n_bars = 3 * S + 2 * RW + 2 * NB + 2;
  static constexpr uint32_t misc_off = bar_off + n_bars * 8;
  static constexpr int box_rows = BT < 128 ? BT : 128;  // x rows per TMA box
  static constexpr uint32_t bytes = misc_off + 16;
  static constexpr uint32_t alloc = bytes + 1024;  // room to align the base to 1024
  // TMEM: NB buffers of D (NS accumulators of BT columns each), then the A ring
  static constexpr int d_cols = NS * BT;
  static constexpr int a_col0 = NB * d_cols;
  static constexpr int cols = a_col0 + S * NS * kAcolsPerStage;
  static_assert(cols <= 512, "TMEM holds 512 columns");
  static_assert(alloc <= 227 * 1024, "shared memory");
  static_assert(RW >= S, "the raw ring is at least as deep as the A ring");
};

__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  // K-major, 128-byte swizzle: 8-row groups 1024 bytes apart (SBO), LBO 1
  // (unused by this layout), version 1, swizzle mode 2
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// kind::f16 instruction descriptor: bf16 A and B, f32 D, K-major, M = 128, N
constexpr uint32_t idesc_bf16(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// D[128 x N] (+)= A[128 x 16] . B[N x 16]^T with A in TMEM (lane = row, a
// 32-bit column = two consecutive k) and B in shared memory.
__device__ __forceinline__ void mma_bf16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(b), "r"(idesc), "r"(accumulate));
}
// 16 columns of this warp's 32 TMEM lanes from registers (thread i -> lane i)
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}
// 16 columns of this warp's 32 TMEM lanes into registers
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}

// Bounded wait that also gives up once another role has aborted the CTA.
__device__ __forceinline__ bool pf_wait(uint64_t *bar, uint32_t parity, volatile int *abort, uint32_t *status) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      *abort = 1;
      raise_status(status, kStatusTimeout);
      return false;
    }
  }
}

// After an abort: let copies or MMAs already issued finish before the CTA's
// shared memory and TMEM go away (bounded; the abort flag is not consulted).
__device__ __forceinline__ void drain_wait(uint64_t *bar, uint32_t parity) {
  (void)mbar_wait_bounded(bar, parity, kWaitLimitNs);
}

__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  uint64_t v;
  asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "f"(lo), "f"(hi));
  return v;
}
__device__ __forceinline__ uint64_t u2(uint32_t lo, uint32_t hi) {
  uint64_t v;
  asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "r"(lo), "r"(hi));
  return v;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// bf16x2 of the f32 pair {lo, hi}, round to nearest even
__device__ __forceinline__ uint32_t pack_bf16x2(uint64_t v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// (w & mask) | 0x4B000000: the f32 2^23 + (w & mask)
template <uint32_t MASK>
__device__ __forceinline__ uint32_t magic23(uint32_t w) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(r) : "r"(w), "n"(MASK), "n"(0x4B000000));
  return r;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&h);
}

template <int NS, int BT, int S, int RW, int NB, bool SF16, bool YF32>
__global__ void __launch_bounds__(kPfThreads, 1) prefill_kernel(const __grid_constant__ CUtensorMap xmap, const PfArgs a) {
  using C = PfCfg<NS, BT, S, RW, NB>;
  constexpr uint32_t kIdesc = idesc_bf16(BT);
  extern __shared__ unsigned char smem_raw[];
  unsigned char *sm = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + C::bar_off);
  uint64_t *xfull = bars, *deq = bars + S, *empty = bars + 2 * S;
  uint64_t *rawfull = bars + 3 * S, *rawempty = rawfull + RW;
  uint64_t *accf = rawempty + RW, *acce = accf + NB, *yfull = acce + NB, *ydone = yfull + 1;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(sm + C::misc_off);
  volatile int *abort = reinterpret_cast<volatile int *>(sm + C::misc_off + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&deq[s], kDeqWarps);
      mbar_init(&empty[s], 1);
    }
    for (int r = 0; r < RW; ++r) {
      mbar_init(&rawfull[r], 1);
      mbar_init(&rawempty[r], kDeqWarps);
    }
    for (int b = 0; b < NB; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], kEpiWarps);
    }
    mbar_init(yfull, kEpiWarps);
    mbar_init(ydone, kEpiWarps);
    *abort = 0;
  }
  if (warp == kWarpMma) {  // all of TMEM (one CTA per SM)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;\n" ::"r"(smem_addr(tmem_holder)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  fence_mbar_init();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int units = a.tiles;

  if (warp == kWarpProd) {
    // ---- x producer: TMA tiles of the activations ------------------------------
    if (lane == 0) {
      int it = 0, issued = 0;
      for (int tile = blockIdx.x; tile < units && !*abort; tile += gridDim.x) {
        const PfUnit un = pf_unit<BT>(a, tile);
        for (int g = 0; g < a.ng; ++g, ++it) {
          const int s = it % S;
          if (it >= S && !pf_wait(&empty[s], (uint32_t)(((it / S) - 1) & 1), abort, a.status)) break;
          unsigned char *xd = sm + C::x_off + (size_t)s * C::x_stage;
          mbar_arrive_expect_tx(&xfull[s], C::x_stage);
#pragma unroll
          for (int bx = 0; bx < BT / C::box_rows; ++bx)
            tma_load_2d(xd + bx * C::box_rows * kBK * 2, &xmap, g * kBK, un.row0 + bx * C::box_rows, &xfull[s]);
          issued = it + 1;
        }
      }
      if (*abort)
        for (int k = issued - S; k < issued; ++k)
          if (k >= 0) drain_wait(&xfull[k % S], (uint32_t)((k / S) & 1));
    }
  } else if (warp == kWarpRaw) {
    // ---- weight producer: one bulk copy per raw slab-group and stream ---------
    if (lane == 0) {
      const uint64_t pol = evict_first_policy();
      int it = 0, issued = 0;
      for (int tile = blockIdx.x; tile < units && !*abort; tile += gridDim.x) {
        const PfUnit un = pf_unit<BT>(a, tile);
        for (int g = 0; g < a.ng; ++g, ++it) {
          const int r = it % RW;
          if (it >= RW && !pf_wait(&rawempty[r], (uint32_t)(((it / RW) - 1) & 1), abort, a.status)) break;
          unsigned char *rd = sm + C::raw_off + (size_t)r * NS * kRawStage;
          const size_t sg = (size_t)un.nt * a.ng + g;
          mbar_arrive_expect_tx(&rawfull[r], NS * kRawStage);
#pragma unroll
          for (int si = 0; si < NS; ++si) {
            bulk_g2s(rd + si * kRawStage, un.qw[si] + sg * 4096, 4096, &rawfull[r], pol);
            bulk_g2s(rd + si * kRawStage + 4096, un.sb[si] + sg * 512, 512, &rawfull[r], pol);
          }
          issued = it + 1;
        }
      }
      if (*abort)
        for (int k = issued - RW; k < issued; ++k)
          if (k >= 0) drain_wait(&rawfull[k % RW], (uint32_t)((k / RW) & 1));
    }
  } else if (warp == kWarpMma) {
    // ---- MMA issuer ------------------------------------------------------------
    if (lane == 0) {
      int it = 0, local = 0, committed = 0;
      for (int tile = blockIdx.x; tile < units && !*abort; tile += gridDim.x, ++local) {
        const int b = local % NB;
        if (local >= NB && !pf_wait(&acce[b], (uint32_t)(((local / NB) - 1) & 1), abort, a.status)) break;
        tc_fence_after();
        const uint32_t dcol = (uint32_t)(b * C::d_cols);
        bool ok = true;
        for (int g = 0; g < a.ng; ++g, ++it) {
          const int s = it % S;
          const uint32_t par = (uint32_t)((it / S) & 1);
          if (!pf_wait(&xfull[s], par, abort, a.status) || !pf_wait(&deq[s], par, abort, a.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t xa = smem_addr(sm + C::x_off + (size_t)s * C::x_stage);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t bd = umma_desc_sw128(xa + kk * 32);
            const uint32_t acc = (g > 0 || kk > 0) ? 1u : 0u;
#pragma unroll
            for (int si = 0; si < NS; ++si)
              mma_bf16_ts(tmem + dcol + (uint32_t)(si * BT),
                          tmem + (uint32_t)(C::a_col0 + (s * NS + si) * kAcolsPerStage + kk * 8), bd, kIdesc, acc);
          }
          umma_commit(&empty[s]);  // frees x slot s and A slot s once these MMAs are done
          committed = it + 1;
        }
        if (!ok) break;
        umma_commit(&accf[b]);
      }
      if (*abort && committed > 0)
        drain_wait(&empty[(committed - 1) % S], (uint32_t)(((committed - 1) / S) & 1));
    }
  } else if (warp < kWarpEpi0) {
    // ---- dequant: raw slab-group -> bf16 A in TMEM -----------------------------
    // warp w: TMEM lane quarter q = w % 4 (rows 32q..32q+31, this thread row
    // 32q + lane) and k half kh = w / 4 (k 32kh..32kh+31 = A columns 16kh..)
    const int q = warp & 3, kh = warp >> 2;
    const int row = 32 * q + lane;  // 0..127
    const int tl = row >> 4, r = row & 7, hrow = (row >> 3) & 1;
    const uint64_t m23 = f2(-8388608.0f, -8388608.0f);
    int it = 0;
    for (int tile = blockIdx.x; tile < units && !*abort; tile += gridDim.x) {
      bool ok = true;
      for (int g = 0; g < a.ng; ++g, ++it) {
        const int s = it % S, rs = it % RW;
        // the raw stage has landed and the MMAs that read A slot s last are done
        if (!pf_wait(&rawfull[rs], (uint32_t)((it / RW) & 1), abort, a.status) ||
            (it >= S && !pf_wait(&empty[s], (uint32_t)(((it / S) - 1) & 1), abort, a.status))) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int si = 0; si < NS; ++si) {
          const unsigned char *raw = sm + C::raw_off + (size_t)(rs * NS + si) * kRawStage;
          const uint2 qd = *reinterpret_cast<const uint2 *>(raw + 4096 + tl * 64 + r * 8);
          const uint32_t sbw = hrow ? qd.y : qd.x;
          const float sv = sb_to_f32<SF16>(sbw & 0xffffu), bv = sb_to_f32<SF16>(sbw >> 16);
          // low nibbles take s, high nibbles (kept x16) take s / 16
          const uint64_t sc0 = f2(sv, sv), sc1 = f2(sv * 0.0625f, sv * 0.0625f), bb = f2(bv, bv);
          uint32_t v[16];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            // lane chunk (4r + c) of tile tl holds this row's k 2c, 2c+1 (+8,
            // +16, +24) of words j = 2kh, 2kh+1
            const uint2 wd = *reinterpret_cast<const uint2 *>(raw + tl * 512 + (4 * r + c) * 16 + kh * 8);
            const uint32_t ww[2] = {wd.x, wd.y};
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
              // this row's nibbles: byte hrow (k pair +0) and byte hrow + 2
              // (k pair +1), low half e = 0 (k + 0) and high half e = 1 (k + 16)
              const uint32_t lo = ww[jj] >> (8 * hrow), hi = ww[jj] >> (8 * hrow + 16);
              const uint64_t p0 = u2(magic23<0x0Fu>(lo), magic23<0x0Fu>(hi));
              const uint64_t p1 = u2(magic23<0xF0u>(lo), magic23<0xF0u>(hi));
              // k within the half: 8 jj + 16 e + 2c -> A column 4 jj + 8 e + c
              v[4 * jj + c] = pack_bf16x2(fma2(add2(p0, m23), sc0, bb));
              v[4 * jj + 8 + c] = pack_bf16x2(fma2(add2(p1, m23), sc1, bb));
            }
          }
          tmem_st16(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(C::a_col0 + (s * NS + si) * kAcolsPerStage + 16 * kh), v);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&rawempty[rs]);
          mbar_arrive(&deq[s]);
        }
      }
      if (!ok) break;
    }
  } else {
    // ---- epilogue: TMEM -> registers -> (bf16 tile in SMEM) -> y --------------
    // warp: TMEM lane quarter q (rows 32q..), token half th of the tile.  For
    // a bf16 y the accumulator is released as soon as it sits in the SMEM
    // tile, and y is then written in 16-byte pieces, a token's 128 values
    // (256 contiguous bytes) at a time; an f32 y is stored straight from
    // registers, a warp's 32 rows of one token being one contiguous segment.
    const int q = warp & 3, th = (warp - kWarpEpi0) >> 2;
    const int et = threadIdx.x - kWarpEpi0 * 32;  // 0..255
    uint16_t *ytile = reinterpret_cast<uint16_t *>(sm + C::y_off);
    int local = 0;
    for (int tile = blockIdx.x; tile < units && !*abort; tile += gridDim.x, ++local) {
      const PfUnit un = pf_unit<BT>(a, tile);
      const int nt = un.nt;
      const int b = local % NB;
      if (!pf_wait(&accf[b], (uint32_t)((local / NB) & 1), abort, a.status)) break;
      // the SMEM tile is free once every warp stored the previous one
      if (!YF32 && local >= 1 && !pf_wait(ydone, (uint32_t)((local - 1) & 1), abort, a.status)) break;
      tc_fence_after();
      const int nl = 32 * q + lane, n = nt * kBN + nl;
#pragma unroll 1
      for (int tc0 = th * (BT / 2); tc0 < (th + 1) * (BT / 2); tc0 += 16) {  // 16 tokens at a time
        const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * C::d_cols + tc0);
        uint32_t u[16];
        float v[16];
        tmem_ld16(taddr, u);
        if constexpr (NS == 2) {
          uint32_t uu[16];
          tmem_ld16(taddr + BT, uu);
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] = silu_mul(__uint_as_float(u[e]), __uint_as_float(uu[e]));
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] = __uint_as_float(u[e]);
        }
        if constexpr (YF32) {
          if (n < a.n) {
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const int t = un.row0 + tc0 + e;
              if (t < un.row_end) static_cast<float *>(a.y)[(size_t)t * a.n + n] = v[e];
            }
          }
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) ytile[(tc0 + e) * kBN + nl] = f32_to_bf16_bits(v[e]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[b]);  // the MMA may overwrite this D buffer from here on
      if constexpr (!YF32) {
        if (lane == 0) mbar_arrive(yfull);
        if (!pf_wait(yfull, (uint32_t)(local & 1), abort, a.status)) break;
        // BT token rows of 256 bytes; 256 threads, 16-byte pieces
        constexpr int kPer = BT * 16 / (kEpiWarps * 32);  // pieces per thread
        const bool vec = (a.n & 7) == 0 && nt * kBN + kBN <= a.n;
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
          const int piece = et + i * kEpiWarps * 32, tt = piece >> 4, col = (piece & 15) * 8;
          const int t = un.row0 + tt;
          if (t >= un.row_end) continue;
          const uint4 val = *reinterpret_cast<const uint4 *>(ytile + tt * kBN + col);
          uint16_t *dst = static_cast<uint16_t *>(a.y) + (size_t)t * a.n + nt * kBN + col;
          if (vec) {
            *reinterpret_cast<uint4 *>(dst) = val;
          } else {
            const uint16_t *h = reinterpret_cast<const uint16_t *>(&val);
#pragma unroll
            for (int e = 0; e < 8; ++e)
              if (nt * kBN + col + e < a.n) dst[e] = h[e];
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(ydone);
      }
    }
  }

  // every role is done with TMEM: free it (also after an abort)
  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;\n" ::"r"(tmem));
  }
}

template <int NS, int BT, int S, int RW, int NB, bool SF16, bool YF32>
cudaError_t prefill_launch_t(const CUtensorMap &map, const PfArgs &a, int grid, cudaStream_t stream) {
  auto *k = &prefill_kernel<NS, BT, S, RW, NB, SF16, YF32>;
  static DeviceOnce once;
  const size_t smem = PfCfg<NS, BT, S, RW, NB>::alloc;
  cudaError_t e = once.run([&] { return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); });
  if (e != cudaSuccess) return e;
  k<<<grid, kPfThreads, smem, stream>>>(map, a);
  return cudaGetLastError();
}

}  // namespace

namespace {

// The driver's tensor-map encoder, looked up through the runtime so the
// library needs no link-time driver dependency.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void *fn = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return encode;
}

}  // namespace

// x [rows][k] bf16 as a 2-D tensor (k innermost), 64 x box_rows boxes,
// 128-byte swizzle
cudaError_t make_xmap(const void *x, int k, int rows, int box_rows, CUtensorMap *map) {
  const auto encode = tensor_map_encoder();
  if (!encode) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)k * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult cr = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(x), dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return cr == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

namespace {

template <int NS, int BT, int S, int RW, int NB>
cudaError_t launch_cfg(const CUtensorMap &map, const PfArgs &a, int grid, bool f16, bool y_f32, cudaStream_t stream) {
  return f16 ? (y_f32 ? prefill_launch_t<NS, BT, S, RW, NB, true, true>(map, a, grid, stream)
                      : prefill_launch_t<NS, BT, S, RW, NB, true, false>(map, a, grid, stream))
             : (y_f32 ? prefill_launch_t<NS, BT, S, RW, NB, false, true>(map, a, grid, stream)
                      : prefill_launch_t<NS, BT, S, RW, NB, false, false>(map, a, grid, stream));
}

}  // namespace

bool prefill_supported(int m, bool x_f32) { return m > 8 && !x_f32; }

namespace {
// Token-tile width of the one-weight form: THQ4_PREFILL_BT=128 forces
// 128-token tiles with two D buffers (a tuning switch read once).  256 is
// the default: the dequant warps, not the tensor core, bound a tile, and a
// 128-token tile spends the same dequant work on half the product (at
// M = 512 it measured 1.5x slower despite the fuller last wave).
int prefill_bt(int m) {
  (void)m;
  static const int forced = [] {
    const char *s = std::getenv("THQ4_PREFILL_BT");
    const int v = s ? std::atoi(s) : 0;
    return v == 128 ? v : 0;
  }();
  return forced ? forced : 256;
}
}  // namespace

cudaError_t prefill_launch(const thq4_weight &w0, const thq4_weight *w1, const void *x, int m, void *y, bool y_f32,
                           cudaStream_t stream) {
  const bool gate_up = w1 != nullptr;
  const int bt = gate_up ? 128 : prefill_bt(m);
  CUtensorMap map;
  cudaError_t e = make_xmap(x, w0.in, m, 128, &map);
  if (e != cudaSuccess) return e;
  PfArgs a{};
  a.qw[0] = static_cast<const uint8_t *>(w0.qw);
  a.sb[0] = static_cast<const uint8_t *>(w0.sb);
  a.qw[1] = gate_up ? static_cast<const uint8_t *>(w1->qw) : nullptr;
  a.sb[1] = gate_up ? static_cast<const uint8_t *>(w1->sb) : nullptr;
  a.y = y;
  a.status = status_word();
  a.m = m;
  a.n = w0.out;
  a.ng = w0.in / kBK;
  a.m_tiles = (m + bt - 1) / bt;
  const long long tiles = (long long)a.m_tiles * row_slabs(w0.out);
  if (tiles >= (1ll << 31)) return cudaErrorInvalidValue;
  a.tiles = (int)tiles;
  const int grid = (int)std::min<long long>(tiles, device_sm_count());
  const bool f16 = w0.sb_dtype == THQ4_F16;
  if (gate_up) return launch_cfg<2, 128, 4, 4, 1>(map, a, grid, f16, y_f32, stream);
  if (bt == 128) return launch_cfg<1, 128, 8, 8, 2>(map, a, grid, f16, y_f32, stream);
  return launch_cfg<1, 256, 4, 4, 1>(map, a, grid, f16, y_f32, stream);
}

}  // namespace thq4
