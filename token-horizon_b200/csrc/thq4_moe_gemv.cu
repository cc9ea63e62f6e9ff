// thq4_moe_gemv.cu -- the MoE expert products: for every group tile (up to
// 32 routed activation rows of one expert), y = x . expert^T, gate/up fused
// with the SwiGLU epilogue, then down.
//
// Replaces the expert-tile kernels of Splash's MoE (moe.metal moe_expert_tile /
// q4_mpp_tile, docs/splash/runtime/metal/kernels/shared/moe.metal:453-640).
//
// At T = 256 tokens, k = 8 of E = 128 experts a tile holds ~16 live rows, so
// the product is bound by streaming every touched expert's weights from HBM
// once (0.5625 bytes per weight), like the decode GEMV, not by the tensor
// core.  A dense-tile design (dequantise every weight to bf16, tcgen05 MMA)
// spends ~3 ALU operations per weight on the exact dequant and runs at a
// quarter of HBM speed here.  This kernel instead:
//   - keeps the weights as the A operand of mma.m16n8k16 in registers: one
//     LOP3 per register turns a nibble pair into the bf16 pair (128 + q0,
//     128 + q1) (exact: bf16 has 8 significant bits), 7 operations per 8
//     weights, shared by every token of the tile;
//   - takes the activations as they are: bf16 B operands, loaded by a 2-D TMA
//     with 128-byte swizzle (one 32-row x 64-k box per group) and read with
//     ldmatrix, conflict-free;
//   - folds the offset and the group's affine parameters into a per-group
//     epilogue: y += s * acc + (b - 128 s) * sum(x), with sum(x) per (row,
//     group) computed once where the activations are produced (the gather
//     kernel; this kernel's own gate/up epilogue for the down projection);
//   - runs one persistent CTA per SM: a producer warp streams (tile, slab)
//     units, four groups per stage (x boxes, nibbles, scales, sums) into a
//     ring with bulk copies; eight consumer warps own one 16-row tile of the
//     slab each and compute only as many 8-token column blocks as the tile
//     has live rows, that count being a compile-time constant of the
//     unrolled body (no branches inside a group); the finished 32 x 128
//     output tile is staged in shared memory and written with 16-byte stores.
// Every mbarrier wait is bounded (kStatusTimeout, no hang).
#include <cuda.h>

#include <algorithm>

#include "thq4_common.cuh"
#include "thq4_internal.h"

namespace thq4 {
namespace {

// One consumer warp per 16-row tile of a slab, then the producer warp.
constexpr int kMgConsumers = kSlabTiles;
constexpr int kMgThreads = (kMgConsumers + 1) * 32;
constexpr int kMgCB = 4;                         // groups per stage
constexpr int kMgMaxStages = 8;
constexpr uint32_t kXBox = kMoeTileRows * 128;   // one group's x box: 32 rows x 64 bf16
constexpr uint32_t kOutTile = kMoeTileRows * 128 * 2;

struct MgArgs {
  const uint8_t *qw[2];  // gate (or the only) experts, up experts: expert e at + e * stride
  const uint8_t *sb[2];
  uint64_t qw_stride[2], sb_stride[2];
  const uint8_t *shq[2], *shsb[2];  // the shared expert's, which tiles of id n_experts run
  int n_experts;
  const uint32_t *tiles;   // [2 gt]: expert, [2 gt + 1]: live rows
  const uint32_t *ntiles;  // group tiles in use (device)
  const float *xsum;       // [tile][ng][32]: sum of each row's group of x
  uint16_t *y;             // [rows][n] bf16
  float *ysum;             // [tile][n / 64][32] sums of y's groups, or null
  uint32_t *status;
  int n, ng, n_slabs, max_units, stages;
};

template <int NS>
struct MgStage {
  static constexpr uint32_t x_off = 0;  // kMgCB boxes, 1024-byte aligned (swizzle)
  static constexpr uint32_t nib_off = kMgCB * kXBox;
  static constexpr uint32_t sb_off = nib_off + NS * kMgCB * 4096;
  static constexpr uint32_t xs_off = sb_off + NS * kMgCB * 512;
  static constexpr uint32_t bytes = (xs_off + kMgCB * 128 + 1023) / 1024 * 1024;
};
template <int NS>
constexpr size_t mg_smem(int stages) {
  return 1024 /* alignment slack */ + 1024 /* barriers */ + (size_t)stages * MgStage<NS>::bytes + kOutTile;
}

__device__ __forceinline__ void bulk_g2s_plain(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                   smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
// D = A * B (+ D), bf16 inputs, f32 accumulate, m16n8k16 (register-only, so
// not volatile: the compiler may interleave independent chains)
__device__ __forceinline__ void mma_bf16_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// (v & 0x000F000F) | 0x43004300: the bf16 pair (128 + q0, 128 + q1) of the
// nibbles in bits 0..3 and 16..19, exact
__device__ __forceinline__ uint32_t nib_bf16x2(uint32_t v) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(r) : "r"(v), "n"(0x000F000F), "n"(0x43004300));
  return r;
}
__device__ __forceinline__ uint64_t pk2(float lo, float hi) {
  uint64_t v;
  asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "f"(lo), "f"(hi));
  return v;
}
__device__ __forceinline__ void unpk2(uint64_t v, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
// a * b + c on both f32 lanes, round to nearest (one instruction)
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// Shared-space accesses by 32-bit address (the ring's base is aligned through
// an integer, so C++ accesses through it would be generic, 64-bit).
__device__ __forceinline__ uint4 mg_lds4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint2 mg_lds2(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}
__device__ __forceinline__ void mg_sts16(uint32_t addr, uint16_t v) {
  asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"(v) : "memory");
}
__device__ __forceinline__ void mg_consumer_sync() {
  asm volatile("bar.sync 1, %0;\n" ::"r"(kMgConsumers * 32) : "memory");
}

// Group j of stage `st` for the NL (compile-time) 8-row column blocks that
// hold live rows: A from the nibbles, B from the swizzled x box, then
// y += s * acc + (b - 128 s) * sum(x) per output.
template <int NS, int NL, bool SF16>
__device__ __forceinline__ void mg_group(uint32_t st, int j, int tile, int lane, float (&y)[NS][4][4]) {
  using St = MgStage<NS>;
  const int r = lane >> 2, c = lane & 3;
  // A of every stream first (k-step 2p: nibbles 0/4 (rows r) and 2/6 (rows
  // r + 8) of words 2p, 2p+1; k-step 2p+1: nibbles 1/5 and 3/7; frag
  // layout), then one 8-row block of B at a time, shared by the streams
  uint32_t av[NS][16];
  float sr[NS], s8[NS], cr[NS], c8[NS];
#pragma unroll
  for (int si = 0; si < NS; ++si) {
    const uint4 w = mg_lds4(st + St::nib_off + (uint32_t)((si * kMgCB + j) * 4096 + tile * 512 + lane * 16));
    av[si][0] = nib_bf16x2(w.x), av[si][1] = nib_bf16x2(w.x >> 8);
    av[si][2] = nib_bf16x2(w.y), av[si][3] = nib_bf16x2(w.y >> 8);
    av[si][4] = nib_bf16x2(w.x >> 4), av[si][5] = nib_bf16x2(w.x >> 12);
    av[si][6] = nib_bf16x2(w.y >> 4), av[si][7] = nib_bf16x2(w.y >> 12);
    av[si][8] = nib_bf16x2(w.z), av[si][9] = nib_bf16x2(w.z >> 8);
    av[si][10] = nib_bf16x2(w.w), av[si][11] = nib_bf16x2(w.w >> 8);
    av[si][12] = nib_bf16x2(w.z >> 4), av[si][13] = nib_bf16x2(w.z >> 12);
    av[si][14] = nib_bf16x2(w.w >> 4), av[si][15] = nib_bf16x2(w.w >> 12);
    const uint2 q = mg_lds2(st + St::sb_off + (uint32_t)((si * kMgCB + j) * 512 + tile * 64 + r * 8));
    sr[si] = sb_to_f32<SF16>(q.x & 0xffffu), s8[si] = sb_to_f32<SF16>(q.y & 0xffffu);
    cr[si] = fmaf(-128.0f, sr[si], sb_to_f32<SF16>(q.x >> 16));
    c8[si] = fmaf(-128.0f, s8[si], sb_to_f32<SF16>(q.y >> 16));
  }
  // B: x rows 8 nb + (lane & 7); k-steps 0/1 from 16-byte chunks 0..3,
  // k-steps 2/3 from chunks 4..7 (swizzled by row & 7)
  const uint32_t xb = st + St::x_off + (uint32_t)j * kXBox;
  const uint32_t xs = st + St::xs_off + (uint32_t)j * 128;
  uint32_t bq[NL][8];
  float2 sx[NL];
#pragma unroll
  for (int nb = 0; nb < NL; ++nb) {
    const int row = nb * 8 + (lane & 7), mat = lane >> 3;
    uint32_t t[4];
    ldsm_x4(t, xb + row * 128 + (((0 + mat) ^ (row & 7)) << 4));
    bq[nb][0] = t[0], bq[nb][1] = t[1], bq[nb][2] = t[2], bq[nb][3] = t[3];
    ldsm_x4(t, xb + row * 128 + (((4 + mat) ^ (row & 7)) << 4));
    bq[nb][4] = t[0], bq[nb][5] = t[1], bq[nb][6] = t[2], bq[nb][7] = t[3];
    const uint2 sv = mg_lds2(xs + (uint32_t)(nb * 8 + 2 * c) * 4);
    sx[nb] = make_float2(__uint_as_float(sv.x), __uint_as_float(sv.y));
  }
  // k-step by k-step over every (stream, block) accumulator: NS x NL
  // independent chains in flight
  float acc[NS][NL][4];
#pragma unroll
  for (int ks = 0; ks < 4; ++ks)
#pragma unroll
    for (int si = 0; si < NS; ++si)
#pragma unroll
      for (int nb = 0; nb < NL; ++nb) {
        const uint32_t *A = &av[si][4 * ks];
        if (ks == 0)
          mma_bf16_z(acc[si][nb], A[0], A[1], A[2], A[3], bq[nb][0], bq[nb][1]);
        else
          mma_bf16(acc[si][nb], A[0], A[1], A[2], A[3], bq[nb][2 * ks], bq[nb][2 * ks + 1]);
      }
  // the same two FMAs per output, in packed f32x2 form: {y0, y1} (row r,
  // tokens 2c and 2c + 1) and {y2, y3} (row r + 8)
#pragma unroll
  for (int si = 0; si < NS; ++si) {
    const uint64_t srr = pk2(sr[si], sr[si]), crr = pk2(cr[si], cr[si]);
    const uint64_t s88 = pk2(s8[si], s8[si]), c88 = pk2(c8[si], c8[si]);
#pragma unroll
    for (int nb = 0; nb < NL; ++nb) {
      const uint64_t xs2 = pk2(sx[nb].x, sx[nb].y);
      uint64_t lo = pk2(y[si][nb][0], y[si][nb][1]), hi = pk2(y[si][nb][2], y[si][nb][3]);
      lo = ffma2(srr, pk2(acc[si][nb][0], acc[si][nb][1]), ffma2(crr, xs2, lo));
      hi = ffma2(s88, pk2(acc[si][nb][2], acc[si][nb][3]), ffma2(c88, xs2, hi));
      unpk2(lo, y[si][nb][0], y[si][nb][1]);
      unpk2(hi, y[si][nb][2], y[si][nb][3]);
    }
  }
}

// The groups of a stage holding `cnt` groups.
template <int NS, int NL, bool SF16>
__device__ __forceinline__ void mg_stage(uint32_t st, int cnt, int tile, int lane, float (&y)[NS][4][4]) {
  if (cnt == kMgCB) {
#pragma unroll
    for (int j = 0; j < kMgCB; ++j) mg_group<NS, NL, SF16>(st, j, tile, lane, y);
  } else {
    for (int j = 0; j < cnt; ++j) mg_group<NS, NL, SF16>(st, j, tile, lane, y);
  }
}

template <int NS, bool SF16>
__global__ void __launch_bounds__(kMgThreads, 1) moe_gemv_kernel(const __grid_constant__ CUtensorMap xmap, const MgArgs a) {
  using St = MgStage<NS>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char *sm = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t *full = reinterpret_cast<uint64_t *>(sm);
  uint64_t *empty = full + kMgMaxStages;
  unsigned char *ring = sm + 1024;
  const int R = a.stages;
  uint16_t *otile = reinterpret_cast<uint16_t *>(ring + (size_t)R * St::bytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < R; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kMgConsumers);
    }
  }
  fence_mbar_init();
  __syncthreads();
  pdl_wait();  // the tiles, rows and sums come from the preceding kernels
  pdl_launch_dependents();
  const int units = min(a.max_units, (int)(*a.ntiles) * a.n_slabs);
  const int cpu = (a.ng + kMgCB - 1) / kMgCB;  // stages per unit

  if (warp == kMgConsumers) {
    // ---- producer ------------------------------------------------------------
    if (lane != 0) return;
    const uint64_t pol = evict_first_policy();
    int it = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      const int gt = u / a.n_slabs, sl = u - gt * a.n_slabs;
      uint32_t e = a.tiles[2 * gt];
      const bool shared = e == (uint32_t)a.n_experts && a.shq[0] != nullptr;
      if (e >= (uint32_t)a.n_experts && !shared) {  // never produced by the grouping kernel
        raise_status(a.status, kStatusBadExpert);
        e = 0;
      }
      for (int c = 0; c < cpu; ++c, ++it) {
        const int s = it % R;
        if (it >= R && !mbar_wait_bounded(&empty[s], (uint32_t)(((it / R) - 1) & 1), kWaitLimitNs)) {
          raise_status(a.status, kStatusTimeout);
          for (int q = it - R; q < it; ++q) (void)mbar_wait_bounded(&full[q % R], (uint32_t)((q / R) & 1), kWaitLimitNs);
          return;
        }
        const int g0 = c * kMgCB, cnt = min(kMgCB, a.ng - g0);
        unsigned char *st = ring + (size_t)s * St::bytes;
        mbar_arrive_expect_tx(&full[s], (uint32_t)cnt * (kXBox + NS * (4096 + 512) + 128));
        for (int j = 0; j < cnt; ++j) tma_load_2d(st + St::x_off + j * kXBox, &xmap, (g0 + j) * 64, gt * kMoeTileRows, &full[s]);
        const size_t sg = (size_t)sl * a.ng + g0;
#pragma unroll
        for (int si = 0; si < NS; ++si) {
          const uint8_t *qb = shared ? a.shq[si] : a.qw[si] + e * a.qw_stride[si];
          const uint8_t *sbb = shared ? a.shsb[si] : a.sb[si] + e * a.sb_stride[si];
          bulk_g2s(st + St::nib_off + si * kMgCB * 4096, qb + sg * 4096, cnt * 4096, &full[s], pol);
          bulk_g2s(st + St::sb_off + si * kMgCB * 512, sbb + sg * 512, cnt * 512, &full[s], pol);
        }
        bulk_g2s_plain(st + St::xs_off, a.xsum + ((size_t)gt * a.ng + g0) * kMoeTileRows, cnt * 128, &full[s]);
      }
    }
    return;
  }

  // ---- consumers: warp `tile` owns rows [16 tile, 16 tile + 16) of the slab
  const int tile = warp;
  const int r = lane >> 2, c = lane & 3;
  bool aborted = false;
  int it = 0;
  for (int u = blockIdx.x; u < units; u += gridDim.x) {
    const int gt = u / a.n_slabs, sl = u - gt * a.n_slabs;
    const int live = (int)a.tiles[2 * gt + 1];
    const int nlive = (live + 7) >> 3;  // 8-row column blocks holding live rows
    float y[NS][4][4];
#pragma unroll
    for (int si = 0; si < NS; ++si)
#pragma unroll
      for (int nb = 0; nb < 4; ++nb)
#pragma unroll
        for (int e = 0; e < 4; ++e) y[si][nb][e] = 0.0f;
    for (int cc = 0; cc < cpu; ++cc, ++it) {
      const int s = it % R;
      if (!aborted && !mbar_wait_bounded(&full[s], (uint32_t)((it / R) & 1), kWaitLimitNs)) {
        raise_status(a.status, kStatusTimeout);
        aborted = true;
      }
      if (!aborted) {
        const uint32_t st = smem_addr(ring) + (uint32_t)s * St::bytes;
        const int cnt = min(kMgCB, a.ng - cc * kMgCB);
        switch (nlive) {
          case 1: mg_stage<NS, 1, SF16>(st, cnt, tile, lane, y); break;
          case 2: mg_stage<NS, 2, SF16>(st, cnt, tile, lane, y); break;
          case 3: mg_stage<NS, 3, SF16>(st, cnt, tile, lane, y); break;
          default: mg_stage<NS, 4, SF16>(st, cnt, tile, lane, y); break;
        }
      }
      __syncwarp();
      if (lane == 0 && !aborted) mbar_arrive(&empty[s]);
    }

    mg_consumer_sync();  // every warp is done with the previous tile
    // ---- the unit's 32 x 128 output tile: registers -> shared -> y ----------
#pragma unroll
    for (int nb = 0; nb < 4; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float v = NS == 2 ? silu_mul(y[0][nb][e], y[NS - 1][nb][e]) : y[0][nb][e];
        const int tok = nb * 8 + 2 * c + (e & 1), row = tile * 16 + r + 8 * (e >> 1);
        mg_sts16(smem_addr(otile) + (uint32_t)(tok * 128 + row) * 2, f32_to_bf16_bits(v));
      }
    mg_consumer_sync();
    const int tid = threadIdx.x;  // 0 .. 255
    // rows past `live` are written too for gate/up (they are 0: their x rows
    // are 0), so the down projection reads defined values
    const int rows_out = NS == 2 ? kMoeTileRows : live;
    for (int p = tid; p < kMoeTileRows * 16; p += kMgConsumers * 32) {
      const int tok = p >> 4, col = (p & 15) * 8;
      if (tok < rows_out && sl * 128 + col < a.n && !aborted)
        *reinterpret_cast<uint4 *>(a.y + ((size_t)gt * kMoeTileRows + tok) * a.n + sl * 128 + col) =
            mg_lds4(smem_addr(otile) + (uint32_t)(tok * 128 + col) * 2);
    }
    if (a.ysum) {
      // sums of the bf16 values over each token's two 64-row groups: four
      // threads per (token, group), 16 values each, a fixed shuffle tree
      const int qi = tid >> 2, part = tid & 3, tok = qi >> 1, hg = qi & 1;
      const uint32_t src = smem_addr(otile) + (uint32_t)(tok * 128 + hg * 64 + part * 16) * 2;
      float sum = 0.0f;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint4 v = mg_lds4(src + 16 * h);
        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) sum += __uint_as_float(wv[e] << 16) + __uint_as_float(wv[e] & 0xffff0000u);
      }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      if (part == 0 && sl * 128 + hg * 64 < a.n && !aborted) a.ysum[((size_t)gt * (a.n / 64) + sl * 2 + hg) * kMoeTileRows + tok] = sum;
    }
  }
}

template <int NS, bool SF16>
cudaError_t mg_launch_t(const CUtensorMap &map, const MgArgs &a, int grid, size_t smem, cudaStream_t stream) {
  auto *k = &moe_gemv_kernel<NS, SF16>;
  static DeviceOnce once;
  cudaError_t e = once.run([&] { return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvMaxSmem); });
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kMgThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = gemv_pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, map, a);
}

}  // namespace

cudaError_t moe_expert_launch(const MoeExperts &g, cudaStream_t stream) {
  const bool gate_up = g.w1 != nullptr;
  if (g.w0->in % 64 != 0 || g.w0->out % 64 != 0) return cudaErrorInvalidValue;
  CUtensorMap map;
  cudaError_t e = make_xmap(g.x, g.w0->in, g.max_tiles * kMoeTileRows, kMoeTileRows, &map);
  if (e != cudaSuccess) return e;
  MgArgs a{};
  a.qw[0] = static_cast<const uint8_t *>(g.w0->qw);
  a.sb[0] = static_cast<const uint8_t *>(g.w0->sb);
  a.qw[1] = gate_up ? static_cast<const uint8_t *>(g.w1->qw) : nullptr;
  a.sb[1] = gate_up ? static_cast<const uint8_t *>(g.w1->sb) : nullptr;
  a.qw_stride[0] = g.w0->qw_stride;
  a.sb_stride[0] = g.w0->sb_stride;
  a.qw_stride[1] = gate_up ? g.w1->qw_stride : 0;
  a.sb_stride[1] = gate_up ? g.w1->sb_stride : 0;
  a.n_experts = g.n_experts > 0 ? g.n_experts : g.w0->experts;
  a.shq[0] = g.sw0 ? static_cast<const uint8_t *>(g.sw0->qw) : nullptr;
  a.shsb[0] = g.sw0 ? static_cast<const uint8_t *>(g.sw0->sb) : nullptr;
  a.shq[1] = g.sw1 ? static_cast<const uint8_t *>(g.sw1->qw) : nullptr;
  a.shsb[1] = g.sw1 ? static_cast<const uint8_t *>(g.sw1->sb) : nullptr;
  if (gate_up && (a.shq[0] != nullptr) != (a.shq[1] != nullptr)) return cudaErrorInvalidValue;
  a.tiles = g.tiles;
  a.ntiles = g.count;
  a.xsum = g.xsum;
  a.y = static_cast<uint16_t *>(g.y);
  a.ysum = g.ysum;
  a.status = status_word();
  a.n = g.w0->out;
  a.ng = g.w0->in / 64;
  a.n_slabs = row_slabs(g.w0->out);
  const long long units = (long long)g.max_tiles * a.n_slabs;
  if (units >= (1ll << 31)) return cudaErrorInvalidValue;
  a.max_units = (int)units;
  const int grid = (int)std::min<long long>(units, device_sm_count());
  const bool f16 = g.w0->sb_dtype == THQ4_F16;
  if (gate_up) {
    a.stages = 4;
    const size_t smem = mg_smem<2>(a.stages);
    return f16 ? mg_launch_t<2, true>(map, a, grid, smem, stream) : mg_launch_t<2, false>(map, a, grid, smem, stream);
  }
  a.stages = 6;
  const size_t smem = mg_smem<1>(a.stages);
  return f16 ? mg_launch_t<1, true>(map, a, grid, smem, stream) : mg_launch_t<1, false>(map, a, grid, smem, stream);
}

}  // namespace thq4
