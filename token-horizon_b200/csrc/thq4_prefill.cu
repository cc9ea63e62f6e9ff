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
// Warp roles.  DG groups of four dequant warps: warp w owns TMEM lane
// quarter w % 4 (32 rows) and the k-stages it with it % DG == w / 4, so DG
// stages are in work at once and four warps arrive per stage.  Then EW
// epilogue warps, the x producer, the MMA issuer and the raw-weight
// producer.
constexpr int kDeqPerStage = 4;
template <int DG, int EW>
struct PfWarps {
  static constexpr int epi0 = 4 * DG, prod = epi0 + EW, mma = prod + 1, raw = prod + 2;
  static constexpr int threads = (raw + 1) * 32;
};
constexpr uint32_t kXBox = 128 * kBK * 2;   // one 128-token x box, bytes
constexpr uint32_t kRawStage = 4096 + 512;  // one slab-group: nibbles, then scales
constexpr int kAcolsPerStage = kBK / 2;     // TMEM columns of one stage's A (bf16 pairs)

struct PfArgs {
  const uint8_t *qw[2];  // gate (or the only) weight, up
  const uint8_t *sb[2];
  void *y;
  uint32_t *status;
  int m, n, ng;
  int m_tiles, tiles;
  // stream-K split (sk != 0): CTA b takes the stage-units [b W / G, (b + 1)
  // W / G) of the tile-major (tile, k-stage) space, W = tiles * ng, G the
  // grid (W / G >= ng, so at most one boundary falls inside a tile).  The
  // tile cut by the boundary between CTAs b - 1 and b is finished through
  // part slot b and the claim / ready words sync[2b], sync[2b + 1].
  float *part;     // [G][BT tokens][128 rows] f32
  uint32_t *sync;  // [G][2], zero between calls
  int sk;
  long long work;
};

// The CTA's walk over its segments -- tile `tile`, k-stages [kb, ke) -- in
// order; every role takes the same walk.  Without the split: tiles
// blockIdx.x, blockIdx.x + G, ... whole.
struct PfWalk {
  long long s, s1;
  int tile;
};
__device__ __forceinline__ PfWalk pf_walk_begin(const PfArgs &a) {
  PfWalk w;
  w.s = a.sk ? (long long)blockIdx.x * a.work / gridDim.x : 0;
  w.s1 = a.sk ? (long long)(blockIdx.x + 1) * a.work / gridDim.x : 0;
  w.tile = blockIdx.x;
  return w;
}
__device__ __forceinline__ bool pf_walk_next(const PfArgs &a, PfWalk &w, int &tile, int &kb, int &ke) {
  if (a.sk) {
    if (w.s >= w.s1) return false;
    tile = (int)(w.s / a.ng);
    const long long t0 = (long long)tile * a.ng;
    const long long end = w.s1 < t0 + a.ng ? w.s1 : t0 + a.ng;
    kb = (int)(w.s - t0);
    ke = (int)(end - t0);
    w.s = end;
    return true;
  }
  if (w.tile >= a.tiles) return false;
  tile = w.tile;
  kb = 0;
  ke = a.ng;
  w.tile += gridDim.x;
  return true;
}

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
  // raw slab-groups: the nibbles (4096 bytes a stream, 128-byte swizzled by
  // the TMA, so 1024-aligned) and the scales (512 bytes a stream) in rings
  static constexpr uint32_t raw_off = x_off + S * x_stage;
  static constexpr uint32_t sb_off = raw_off + RW * NS * 4096;
  // a bf16 output tile [BT tokens][128 rows], staged between TMEM and y
  static constexpr uint32_t y_off = sb_off + RW * NS * 512;
  static constexpr uint32_t bar_off = y_off + BT * kBN * 2;
  // barriers: xfull[S], deq[S], empty[S], rawfull[RW], rawempty[RW],
  // accf[NB], acce[NB], yfull, ydone, claimed, parted (split tiles)
  static constexpr int n_bars = 3 * S + 2 * RW + 2 * NB + 4;
  static constexpr uint32_t misc_off = bar_off + n_bars * 8;
  // x rows per TMA box: 128-row boxes for 256 tokens, one box otherwise
  static constexpr int box_rows = BT <= 128 ? BT : (BT % 128 == 0 ? 128 : BT);
  static_assert(BT % 16 == 0 && BT <= 256 && BT % box_rows == 0, "token tile");
  static constexpr uint32_t bytes = misc_off + 16;
  static constexpr uint32_t alloc = bytes + 1024;  // room to align the base to 1024
  // TMEM: NB buffers of D (NS accumulators of BT columns each), then the A ring
  static constexpr int d_cols = NS * BT;
  static constexpr int a_col0 = NB * d_cols;
  static constexpr int cols = a_col0 + S * NS * kAcolsPerStage;
  static_assert(cols <= 512, "TMEM holds 512 columns");
  static_assert(alloc <= 227 * 1024, "shared memory");
  static_assert(RW >= S, "the raw ring is at least as deep as the A ring");
  static_assert(raw_off % 1024 == 0 && x_stage % 1024 == 0, "swizzled TMA destinations");
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
// 16 columns of this warp's 32 TMEM lanes from registers, not waited for
__device__ __forceinline__ void tmem_st16_async(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }
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

// 2-D TMA tile load with an L2 cache policy
__device__ __forceinline__ void tma_load_2d_hint(void *dst, const void *map, int c0, int c1, uint64_t *bar,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, %4}], "
      "[%2], %5;\n" ::"r"(smem_addr(dst)),
      "l"(map), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}
// explicit shared-space accesses (the aligned base pointer goes through an
// integer, so plain C++ accesses through it would be generic)
__device__ __forceinline__ uint2 lds_u2(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint4 lds_u4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ void sts_u16(uint32_t addr, uint16_t v) {
  asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"(v) : "memory");
}

// device-scope flag and partial-tile accesses of the split tiles
__device__ __forceinline__ uint32_t ld_acquire_gpu_u32(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu_u32(uint32_t *p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ float ld_relaxed_gpu_f32(const float *p) {
  float v;
  asm volatile("ld.relaxed.gpu.global.f32 %0, [%1];\n" : "=f"(v) : "l"(p) : "memory");
  return v;
}
// Bounded wait for a flag another CTA of this grid raises; false (and the
// CTA aborted, the status word set) on timeout.
__device__ __forceinline__ bool pf_poll_flag(const uint32_t *f, volatile int *abort, uint32_t *status) {
  if (ld_acquire_gpu_u32(f)) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    if (ld_acquire_gpu_u32(f)) return true;
    if (*abort) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      *abort = 1;
      raise_status(status, kStatusTimeout);
      return false;
    }
  }
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&h);
}

template <int NS, int BT, int S, int RW, int NB, int DG, int EW, bool SF16, bool YF32>
__global__ void __launch_bounds__(PfWarps<DG, EW>::threads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap0,
                   const __grid_constant__ CUtensorMap wmap1, const PfArgs a) {
  using C = PfCfg<NS, BT, S, RW, NB>;
  using W = PfWarps<DG, EW>;
  constexpr int kEpiWarps = EW;
  constexpr int kWarpEpi0 = W::epi0, kWarpProd = W::prod, kWarpMma = W::mma, kWarpRaw = W::raw;
  static_assert(EW == 4 || EW == 8, "one or two epilogue warps per TMEM lane quarter");
  static_assert((BT / (EW / 4)) % 16 == 0, "each epilogue warp takes its share of the tokens, 16 at a time");
  static_assert((BT * 16) % (EW * 32) == 0, "epilogue store pieces");
  constexpr uint32_t kIdesc = idesc_bf16(BT);
  extern __shared__ unsigned char smem_raw[];
  unsigned char *sm = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + C::bar_off);
  uint64_t *xfull = bars, *deq = bars + S, *empty = bars + 2 * S;
  uint64_t *rawfull = bars + 3 * S, *rawempty = rawfull + RW;
  uint64_t *accf = rawempty + RW, *acce = accf + NB, *yfull = acce + NB, *ydone = yfull + 1;
  uint64_t *claimed = ydone + 1, *parted = ydone + 2;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(sm + C::misc_off);
  volatile int *abort = reinterpret_cast<volatile int *>(sm + C::misc_off + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&deq[s], kDeqPerStage);
      mbar_init(&empty[s], 1);
    }
    for (int r = 0; r < RW; ++r) {
      mbar_init(&rawfull[r], 1);
      mbar_init(&rawempty[r], kDeqPerStage);
    }
    for (int b = 0; b < NB; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], kEpiWarps);
    }
    mbar_init(yfull, kEpiWarps);
    mbar_init(ydone, kEpiWarps);
    mbar_init(claimed, 1);
    mbar_init(parted, kEpiWarps);
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

  if (warp == kWarpProd) {
    // ---- x producer: TMA tiles of the activations ------------------------------
    if (lane == 0) {
      int it = 0, issued = 0, tile, kb, ke;
      PfWalk wk = pf_walk_begin(a);
      while (!*abort && pf_walk_next(a, wk, tile, kb, ke)) {
        const PfUnit un = pf_unit<BT>(a, tile);
        for (int g = kb; g < ke; ++g, ++it) {
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
      int it = 0, issued = 0, tile, kb, ke;
      PfWalk wk = pf_walk_begin(a);
      while (!*abort && pf_walk_next(a, wk, tile, kb, ke)) {
        const PfUnit un = pf_unit<BT>(a, tile);
        for (int g = kb; g < ke; ++g, ++it) {
          const int r = it % RW;
          if (it >= RW && !pf_wait(&rawempty[r], (uint32_t)(((it / RW) - 1) & 1), abort, a.status)) break;
          const size_t sg = (size_t)un.nt * a.ng + g;
          mbar_arrive_expect_tx(&rawfull[r], NS * kRawStage);
#pragma unroll
          for (int si = 0; si < NS; ++si) {
            // the nibbles as 32 lines of 128 bytes (the weight seen as a
            // [lines][128] byte matrix), 128-byte swizzled
            tma_load_2d_hint(sm + C::raw_off + (size_t)(r * NS + si) * 4096, si ? &wmap1 : &wmap0, 0,
                             (int)(sg * 32), &rawfull[r], pol);
            bulk_g2s(sm + C::sb_off + (size_t)(r * NS + si) * 512, un.sb[si] + sg * 512, 512, &rawfull[r], pol);
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
      int it = 0, local = 0, committed = 0, tile, kb, ke;
      PfWalk wk = pf_walk_begin(a);
      for (; !*abort && pf_walk_next(a, wk, tile, kb, ke); ++local) {
        const int b = local % NB;
        if (local >= NB && !pf_wait(&acce[b], (uint32_t)(((local / NB) - 1) & 1), abort, a.status)) break;
        tc_fence_after();
        const uint32_t dcol = (uint32_t)(b * C::d_cols);
        bool ok = true;
        for (int g = kb; g < ke; ++g, ++it) {
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
            const uint32_t acc = (g > kb || kk > 0) ? 1u : 0u;
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
    // 32q + lane), the whole 64 k of the stages it with it % DG == w / 4.
    // Chunk 4r + c of tile tl (16 bytes: words 0..3, this row's k pairs 2c,
    // 2c+1 (+8, +16, +24) with the row r + 8 of the tile) is 128-byte line
    // 4 tl + r / 2, chunk 4 (r % 2) + c before the swizzle, which moves
    // chunk ch of line L to ch ^ (L % 8): for one c the warp's sixteen
    // distinct chunks (tiles 2q and 2q + 1, r = 0..7) fill the 128-byte bank
    // window twice, the least two wavefronts can carry.
    const int q = warp & 3, grp = warp >> 2;
    const int row = 32 * q + lane;  // 0..127
    const int tl = row >> 4, r = row & 7, hrow = (row >> 3) & 1;
    uint32_t coff[4];
#pragma unroll
    for (int c = 0; c < 4; ++c)
      coff[c] = (uint32_t)(tl * 512 + (r >> 1) * 128 + (((4 * (r & 1) + c) ^ (4 * (tl & 1) + (r >> 1))) * 16));
    const uint32_t sboff = (uint32_t)(tl * 64 + r * 8);
    const uint32_t nib0 = smem_addr(sm + C::raw_off), sb0 = smem_addr(sm + C::sb_off);
    const uint64_t m23 = f2(-8388608.0f, -8388608.0f);
    int it = 0, tile, kb, ke;
    PfWalk wk = pf_walk_begin(a);
    while (!*abort && pf_walk_next(a, wk, tile, kb, ke)) {
      bool ok = true;
      for (int g = kb; g < ke; ++g, ++it) {
        if (it % DG != grp) continue;
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
          const uint32_t nib = nib0 + (uint32_t)(rs * NS + si) * 4096;
          const uint2 qd = lds_u2(sb0 + (uint32_t)(rs * NS + si) * 512 + sboff);
          const uint32_t sbw = hrow ? qd.y : qd.x;
          const float sv = sb_to_f32<SF16>(sbw & 0xffffu), bv = sb_to_f32<SF16>(sbw >> 16);
          // low nibbles take s, high nibbles (kept x16) take s / 16
          const uint64_t sc0 = f2(sv, sv), sc1 = f2(sv * 0.0625f, sv * 0.0625f), bb = f2(bv, bv);
          // k half kh: words 2 kh, 2 kh + 1 of each chunk -> A columns 16 kh..
#pragma unroll
          for (int kh = 0; kh < 2; ++kh) {
            uint32_t v[16];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const uint2 wd = lds_u2(nib + coff[c] + 8 * kh);
              const uint32_t ww[2] = {wd.x, wd.y};
#pragma unroll
              for (int jj = 0; jj < 2; ++jj) {
                // this row's nibbles: byte hrow (k pair +0) and byte hrow + 2
                // (k pair +1), low half e = 0 (k + 0) and high half e = 1 (k + 16)
                const uint32_t lo = ww[jj] >> (8 * hrow), hi = ww[jj] >> (8 * hrow + 16);
                const uint64_t p0 = u2(magic23<0x0Fu>(lo), magic23<0x0Fu>(hi));
                const uint64_t p1 = u2(magic23<0xF0u>(lo), magic23<0xF0u>(hi));
                // k = 32 kh + 8 jj + 16 e + 2c -> A column 16 kh + 4 jj + 8 e + c
                v[4 * jj + c] = pack_bf16x2(fma2(add2(p0, m23), sc0, bb));
                v[4 * jj + 8 + c] = pack_bf16x2(fma2(add2(p1, m23), sc1, bb));
              }
            }
            tmem_st16_async(tmem + ((uint32_t)(32 * q) << 16) +
                                (uint32_t)(C::a_col0 + (s * NS + si) * kAcolsPerStage + 16 * kh),
                            v);
          }
        }
        tmem_wait_st();
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
    constexpr int kTokPerWarp = BT / (EW / 4);  // tokens of the tile per warp
    const int q = warp & 3, th = (warp - kWarpEpi0) >> 2;  // token share th
    const int et = threadIdx.x - kWarpEpi0 * 32;  // 0 .. 32 EW - 1
    const uint32_t ytile = smem_addr(sm + C::y_off);
    volatile uint32_t *claim_word = reinterpret_cast<volatile uint32_t *>(sm + C::misc_off + 8);
    int local = 0, nsplit = 0, tile, kb, ke;
    PfWalk wk = pf_walk_begin(a);
    for (; !*abort && pf_walk_next(a, wk, tile, kb, ke); ++local) {
      const PfUnit un = pf_unit<BT>(a, tile);
      const int nt = un.nt;
      const int b = local % NB;
      if (!pf_wait(&accf[b], (uint32_t)((local / NB) & 1), abort, a.status)) break;
      // the SMEM tile is free once every warp stored the previous one
      if (!YF32 && local >= 1 && !pf_wait(ydone, (uint32_t)((local - 1) & 1), abort, a.status)) break;
      tc_fence_after();
      const int nl = 32 * q + lane, n = nt * kBN + nl;
      // A tile cut between two CTAs: the CTA that claims it first stores its
      // f32 part to the boundary's slot and raises the ready word; the second
      // waits for that word (its owner is already storing), adds the part to
      // its own sums (a + b == b + a, so the result does not depend on which
      // CTA came first) and finishes the tile.
      const bool split = NS == 1 && (kb > 0 || ke < a.ng);
      const int bnd = kb > 0 ? (int)blockIdx.x : (int)blockIdx.x + 1;
      const float *slot = split ? a.part + (size_t)bnd * (BT * kBN) : nullptr;
      bool first = false;
      if (split) {
        if (et == 0) {
          uint32_t *sy = a.sync + 2 * bnd;
          const uint32_t old = atom_add_acq_rel(sy, 1u);
          bool ok = true;
          if (old != 0) {
            ok = pf_poll_flag(sy + 1, abort, a.status);
            sy[0] = 0u;  // both CTAs have claimed: zero for the next call
            sy[1] = 0u;
          }
          *claim_word = (old == 0 ? 1u : 0u) | (ok ? 0u : 2u);
          mbar_arrive(claimed);
        }
        if (!pf_wait(claimed, (uint32_t)(nsplit & 1), abort, a.status)) break;
        const uint32_t cw = *claim_word;
        if (cw & 2u) break;
        first = (cw & 1u) != 0;
      }
#pragma unroll 1
      for (int tc0 = th * kTokPerWarp; tc0 < (th + 1) * kTokPerWarp; tc0 += 16) {  // 16 tokens at a time
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
        if (split) {
          // slot layout [token][128 rows]: a warp's 32 rows of one token are
          // one 128-byte segment
          float *sp = const_cast<float *>(slot) + (size_t)tc0 * kBN + nl;
          if (first) {
#pragma unroll
            for (int e = 0; e < 16; ++e) sp[(size_t)e * kBN] = v[e];
            continue;
          }
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] += ld_relaxed_gpu_f32(sp + (size_t)e * kBN);
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
          for (int e = 0; e < 16; ++e) sts_u16(ytile + (uint32_t)(((tc0 + e) * kBN + nl) * 2), f32_to_bf16_bits(v[e]));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[b]);  // the MMA may overwrite this D buffer from here on
      if (split) {
        // every warp has stored (or read) its share of the part: the first
        // CTA publishes it
        if (lane == 0) mbar_arrive(parted);
        if (et == 0) {
          if (!pf_wait(parted, (uint32_t)(nsplit & 1), abort, a.status)) break;
          if (first) {
            fence_acq_rel_gpu();
            st_release_gpu_u32(a.sync + 2 * bnd + 1, 1u);
          }
        }
        ++nsplit;
      }
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
          if (first || t >= un.row_end) continue;  // a first part has no output
          const uint4 val = lds_u4(ytile + (uint32_t)((tt * kBN + col) * 2));
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

template <int NS, int BT, int S, int RW, int NB, int DG, int EW, bool SF16, bool YF32>
cudaError_t prefill_launch_t(const CUtensorMap &map, const CUtensorMap *wm, const PfArgs &a, int grid,
                             cudaStream_t stream) {
  auto *k = &prefill_kernel<NS, BT, S, RW, NB, DG, EW, SF16, YF32>;
  static DeviceOnce once;
  const size_t smem = PfCfg<NS, BT, S, RW, NB>::alloc;
  cudaError_t e = once.run([&] { return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); });
  if (e != cudaSuccess) return e;
  k<<<grid, PfWarps<DG, EW>::threads, smem, stream>>>(map, wm[0], wm[1], a);
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

template <int NS, int BT, int S, int RW, int NB, int DG, int EW>
cudaError_t launch_cfg(const CUtensorMap &map, const CUtensorMap *wm, const PfArgs &a, int grid, bool f16, bool y_f32,
                       cudaStream_t stream) {
  return f16 ? (y_f32 ? prefill_launch_t<NS, BT, S, RW, NB, DG, EW, true, true>(map, wm, a, grid, stream)
                      : prefill_launch_t<NS, BT, S, RW, NB, DG, EW, true, false>(map, wm, a, grid, stream))
             : (y_f32 ? prefill_launch_t<NS, BT, S, RW, NB, DG, EW, false, true>(map, wm, a, grid, stream)
                      : prefill_launch_t<NS, BT, S, RW, NB, DG, EW, false, false>(map, wm, a, grid, stream));
}

// The nibbles of a frag weight (slab-groups of 4096 bytes, slab-major) as a
// [lines][128] byte matrix, read 32 lines (one slab-group) at a time with
// the 128-byte swizzle the dequant warps' conflict-free reads assume.
cudaError_t make_wmap(const void *qw, size_t bytes, CUtensorMap *map) {
  const auto encode = tensor_map_encoder();
  if (!encode) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {128, (cuuint64_t)(bytes / 128)};
  const cuuint64_t strides[1] = {128};
  const cuuint32_t box[2] = {128, 32};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult cr = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(qw), dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return cr == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace

bool prefill_supported(int m, bool x_f32) { return m > 8 && !x_f32; }

namespace {
// Token-tile width of the one-weight form.  The persistent grid takes
// ceil(tiles / SMs) rounds of tiles; a tile costs its BT MMA columns or the
// dequant's fixed pass over the slab, whichever is longer, plus a fixed cost
// (pipeline fill and the epilogue's hand-back of D).  The widest width of
// least cost wins, which fills the last wave where 256 would not: M = 512
// over the 96 slabs of a 12288-row weight runs as 3 x 96 tiles of 192
// tokens (1.95 waves on 148 SMs) instead of 2 x 96 of 256 (1.30 waves).
int prefill_plan(int m, int slabs, int sms) {
  constexpr int kWidths[] = {256, 192};
  constexpr int kDequantCols = 128, kTileCols = 32;
  int best = 256;
  long long best_cost = -1;
  for (const int bt : kWidths) {
    const long long tiles = (long long)((m + bt - 1) / bt) * slabs;
    const long long rounds = (tiles + sms - 1) / sms;
    const long long cost = rounds * (std::max(bt, kDequantCols) + kTileCols);
    if (best_cost < 0 || cost < best_cost) best_cost = cost, best = bt;
  }
  return best;
}

// THQ4_PREFILL_BT in {128, 192, 256} forces a width of whole tiles (a tuning
// switch read once; 128 runs with two D buffers and eight stages).
int prefill_forced_bt() {
  static const int forced = [] {
    const char *b = std::getenv("THQ4_PREFILL_BT");
    const int bt = b ? std::atoi(b) : 0;
    return (bt == 128 || bt == 192 || bt == 256) ? bt : 0;
  }();
  return forced;
}
// THQ4_PREFILL_SK=0 switches the stream-K split off (read once).
bool prefill_split_enabled() {
  static const bool on = [] {
    const char *e = std::getenv("THQ4_PREFILL_SK");
    return !(e && std::atoi(e) == 0);
  }();
  return on;
}

// Launch shape of one call.  Stream-K runs 256-token tiles (the best rate
// within a tile) when they outnumber the SMs but whole tiles would fill the
// waves to less than 80%: each CTA takes tiles x ng / SMs k-stages, so the
// last wave is as full as the others.  With every SM busy a k-stage takes
// longer than in a part-empty last wave, so a nearly full last wave runs
// faster whole (measured: M = 512 over 96 slabs, waves 65% full, 58.0 us
// split against 63.7 whole; M = 4096, 94% full, 423 against 399).
// Otherwise whole tiles of the planned width.
struct PfPlan {
  int bt;
  bool sk;
  long long tiles;
  int grid;
};
PfPlan prefill_plan_on(int out, int m, bool gate_up, int sms) {
  const int slabs = row_slabs(out);
  PfPlan p{};
  const int forced = prefill_forced_bt();
  if (gate_up) {
    p.bt = 128;
  } else if (forced) {
    p.bt = forced;
  } else {
    const long long t256 = (long long)((m + 255) / 256) * slabs;
    const long long rounds = (t256 + sms - 1) / sms;
    p.sk = prefill_split_enabled() && t256 > sms && t256 * 5 < rounds * sms * 4;
    p.bt = p.sk ? 256 : prefill_plan(m, slabs, sms);
  }
  p.tiles = (long long)((m + p.bt - 1) / p.bt) * slabs;
  p.grid = (int)std::min<long long>(p.tiles, sms);
  return p;
}
PfPlan prefill_plan_for(const thq4_weight &w0, int m, bool gate_up) {
  return prefill_plan_on(w0.out, m, gate_up, device_sm_count());
}
// Workspace layout of a split call: [decode region][claim words][parts].
size_t round256(size_t v) { return (v + 255) & ~(size_t)255; }
size_t split_sync_off(const thq4_weight &w0) { return round256(gemv_workspace_bytes(w0.out)); }
size_t split_part_off(const thq4_weight &w0, int grid) {
  return split_sync_off(w0) + round256((size_t)grid * 2 * sizeof(uint32_t));
}
}  // namespace

PrefillPlanInfo prefill_debug_plan(int out, int m, bool gate_up, int sms) {
  const PfPlan p = prefill_plan_on(out, m, gate_up, sms);
  PrefillPlanInfo r{p.bt, p.sk, p.tiles, p.grid, 0};
  if (p.sk) {
    thq4_weight w{};
    w.out = out;
    r.split_bytes = split_part_off(w, p.grid) + (size_t)p.grid * p.bt * kBN * sizeof(float);
  }
  return r;
}

size_t prefill_workspace_bytes(const thq4_weight &w0, int m) {
  if (!prefill_supported(m, false)) return 0;
  const PfPlan p = prefill_plan_for(w0, m, false);
  if (!p.sk) return 0;
  return split_part_off(w0, p.grid) + (size_t)p.grid * p.bt * kBN * sizeof(float);
}

cudaError_t prefill_launch(const thq4_weight &w0, const thq4_weight *w1, const void *x, int m, void *y, bool y_f32,
                           void *workspace, size_t workspace_bytes, cudaStream_t stream) {
  const bool gate_up = w1 != nullptr;
  PfPlan plan = prefill_plan_for(w0, m, gate_up);
  if (plan.sk && (!workspace || workspace_bytes < prefill_workspace_bytes(w0, m) ||
                  reinterpret_cast<uintptr_t>(workspace) % 256 != 0)) {
    // no room for the parts (or not the aligned workspace the split's
    // claim words and parts assume): whole tiles
    plan.sk = false;
    plan.bt = prefill_plan(m, row_slabs(w0.out), device_sm_count());
    plan.tiles = (long long)((m + plan.bt - 1) / plan.bt) * row_slabs(w0.out);
    plan.grid = (int)std::min<long long>(plan.tiles, device_sm_count());
  }
  const int bt = plan.bt;
  CUtensorMap map, wm[2];
  cudaError_t e = make_xmap(x, w0.in, m, bt <= 128 ? bt : (bt % 128 == 0 ? 128 : bt), &map);
  if (e != cudaSuccess) return e;
  const size_t nib_bytes = (size_t)row_slabs(w0.out) * (size_t)(w0.in / kBK) * 4096;
  e = make_wmap(w0.qw, nib_bytes, &wm[0]);
  if (e != cudaSuccess) return e;
  wm[1] = wm[0];
  if (gate_up && (e = make_wmap(w1->qw, nib_bytes, &wm[1])) != cudaSuccess) return e;
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
  const long long tiles = plan.tiles;
  if (tiles >= (1ll << 31)) return cudaErrorInvalidValue;
  a.tiles = (int)tiles;
  const int grid = plan.grid;
  if (plan.sk) {
    unsigned char *ws = static_cast<unsigned char *>(workspace);
    a.sk = 1;
    a.work = tiles * a.ng;
    a.sync = reinterpret_cast<uint32_t *>(ws + split_sync_off(w0));
    a.part = reinterpret_cast<float *>(ws + split_part_off(w0, grid));
  }
  const bool f16 = w0.sb_dtype == THQ4_F16;
  if (gate_up) return launch_cfg<2, 128, 4, 4, 1, 2, 8>(map, wm, a, grid, f16, y_f32, stream);
  if (bt == 128) return launch_cfg<1, 128, 8, 8, 2, 2, 8>(map, wm, a, grid, f16, y_f32, stream);
  if (bt == 192) return launch_cfg<1, 192, 4, 4, 2, 2, 8>(map, wm, a, grid, f16, y_f32, stream);
  return launch_cfg<1, 256, 4, 4, 1, 2, 8>(map, wm, a, grid, f16, y_f32, stream);
}

}  // namespace thq4
