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
// 12288 x 4096 shape against 28 MB of weights).  Design:
//   - persistent CTAs (one per SM) walk output tiles of 256 tokens x 128
//     output rows (one frag slab); consecutive tiles share the slab, so the
//     weight is fetched from HBM once and re-read from L2;
//   - per 64-k stage (one quant group): a producer warp loads the x tile with
//     a 2-D TMA (two 128-row boxes, 128-byte swizzle, zero fill past m) and
//     the raw slab-group (4608 bytes of nibbles + scales) with one bulk copy;
//   - four dequant warps turn the slab-group into the bf16 B tile in the
//     K-major 128-byte-swizzled layout tcgen05 reads (each 4-byte store lands
//     in a distinct bank), fence it to the async proxy and arrive;
//   - one thread issues tcgen05.mma.kind::f16 (bf16 in, f32 accumulate in
//     TMEM): per k-step of 16, two M=128 x N=128 MMAs (the two token halves)
//     sharing the B tile, and commits the stage back to the producer;
//   - the accumulator is double-buffered in TMEM (2 x 256 of its 512
//     columns), so four epilogue warps drain tile i (tcgen05.ld, convert,
//     store) while tile i+1 accumulates; the gate/up form keeps gate and up
//     accumulators side by side (all 512 columns) and drains between tiles;
//   - every wait is bounded; a timeout raises kStatusTimeout, sets a CTA-wide
//     abort flag that ends every role's loop, and the CTA still frees TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "thq4_common.cuh"
#include "thq4_internal.h"

namespace thq4 {
namespace {

constexpr int kBM = 256;  // tokens per tile (two M = 128 MMAs)
constexpr int kBN = 128;  // output rows per tile (one slab)
constexpr int kBK = 64;   // k per stage (one quant group)
constexpr int kDeqWarps = 4, kEpiWarps = 4;
constexpr int kWarpEpi0 = 4, kWarpProd = 8, kWarpMma = 9;  // dequant warps are 0..3
constexpr int kPfThreads = 10 * 32;
constexpr uint32_t kXBox = 128 * kBK * 2;        // one 128-row x box, bytes
constexpr uint32_t kXStage = 2 * kXBox;          // 32 KB
constexpr uint32_t kWStage = kBN * kBK * 2;      // bf16 B tile, 16 KB
constexpr uint32_t kRawStage = 4096 + 512;       // one slab-group

struct PfArgs {
  const uint8_t *qw[2];  // gate (or the only) weight, up
  const uint8_t *sb[2];
  void *y;
  uint32_t *status;
  int m, n, ng;
  int m_tiles, tiles;
  int yf32;
};

template <int NS, int S>
struct PfSmem {
  static constexpr uint32_t x_off = 0;
  static constexpr uint32_t w_off = x_off + S * kXStage;
  static constexpr uint32_t raw_off = w_off + S * NS * kWStage;
  static constexpr uint32_t bar_off = raw_off + S * NS * kRawStage;
  // barriers: xfull[S], rawfull[S], deq[S], empty[S], accf[2], acce[2]
  static constexpr uint32_t misc_off = bar_off + (4 * S + 4) * 8;
  static constexpr uint32_t bytes = misc_off + 16;
  static constexpr uint32_t alloc = bytes + 1024;  // room to align the base to 1024
};

__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  // K-major, 128-byte swizzle: 8-row groups 1024 bytes apart (SBO), LBO 1
  // (unused by this layout), version 1, swizzle mode 2
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// kind::f16 instruction descriptor: bf16 A and B, f32 D, K-major, M = 128, N = kBN
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);

__device__ __forceinline__ void mma_bf16_ss(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(kIdesc), "r"(accumulate));
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
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int c0, int c1, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];\n" ::"r"(
          smem_addr(dst)),
      "l"(map), "r"(smem_addr(bar)), "r"(c0), "r"(c1)
      : "memory");
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

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&h);
}

// Stores 32 consecutive outputs of one token row.
__device__ __forceinline__ void store_row32(const PfArgs &a, int token, int col, const float (&v)[32]) {
  if (token >= a.m || col >= a.n) return;
  const bool full = col + 32 <= a.n;
  if (a.yf32) {
    float *dst = static_cast<float *>(a.y) + (size_t)token * a.n + col;
    if (full && (a.n & 3) == 0) {
#pragma unroll
      for (int e = 0; e < 32; e += 4) *reinterpret_cast<float4 *>(dst + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e)
        if (col + e < a.n) dst[e] = v[e];
    }
  } else {
    uint16_t *dst = static_cast<uint16_t *>(a.y) + (size_t)token * a.n + col;
    if (full && (a.n & 7) == 0) {
#pragma unroll
      for (int e = 0; e < 32; e += 8)
        *reinterpret_cast<uint4 *>(dst + e) = make_uint4(pack_bf16(v[e], v[e + 1]), pack_bf16(v[e + 2], v[e + 3]),
                                                         pack_bf16(v[e + 4], v[e + 5]), pack_bf16(v[e + 6], v[e + 7]));
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e)
        if (col + e < a.n) dst[e] = f32_to_bf16_bits(v[e]);
    }
  }
}

template <int NS, int S, bool SF16>
__global__ void __launch_bounds__(kPfThreads, 1) prefill_kernel(const __grid_constant__ CUtensorMap xmap, const PfArgs a) {
  using L = PfSmem<NS, S>;
  constexpr bool kDB = NS == 1;  // double-buffered accumulator
  extern __shared__ unsigned char smem_raw[];
  unsigned char *sm = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + L::bar_off);
  uint64_t *xfull = bars, *rawfull = bars + S, *deq = bars + 2 * S, *empty = bars + 3 * S;
  uint64_t *accf = bars + 4 * S, *acce = accf + 2;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(sm + L::misc_off);
  volatile int *abort = reinterpret_cast<volatile int *>(sm + L::misc_off + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&rawfull[s], 1);
      mbar_init(&deq[s], kDeqWarps);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], kEpiWarps);
    }
    *abort = 0;
  }
  if (warp == kWarpMma) {  // the whole of TMEM: two 256-column accumulators
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;\n" ::"r"(smem_addr(tmem_holder)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  fence_mbar_init();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == kWarpProd) {
    // ---- producer ------------------------------------------------------------
    if (lane == 0) {
      const uint64_t pol = evict_first_policy();
      int it = 0, issued = 0;
      for (int tile = blockIdx.x; tile < a.tiles && !*abort; tile += gridDim.x) {
        const int mt = tile % a.m_tiles, nt = tile / a.m_tiles;
        for (int g = 0; g < a.ng; ++g, ++it) {
          const int s = it % S;
          if (it >= S && !pf_wait(&empty[s], (uint32_t)(((it / S) - 1) & 1), abort, a.status)) break;
          unsigned char *xd = sm + L::x_off + (size_t)s * kXStage;
          mbar_arrive_expect_tx(&xfull[s], kXStage);
          tma_load_2d(xd, &xmap, g * kBK, mt * kBM, &xfull[s]);
          tma_load_2d(xd + kXBox, &xmap, g * kBK, mt * kBM + 128, &xfull[s]);
          unsigned char *rd = sm + L::raw_off + (size_t)s * NS * kRawStage;
          const size_t sg = (size_t)nt * a.ng + g;
          mbar_arrive_expect_tx(&rawfull[s], NS * kRawStage);
#pragma unroll
          for (int si = 0; si < NS; ++si) {
            bulk_g2s(rd + si * kRawStage, a.qw[si] + sg * 4096, 4096, &rawfull[s], pol);
            bulk_g2s(rd + si * kRawStage + 4096, a.sb[si] + sg * 512, 512, &rawfull[s], pol);
          }
          issued = it + 1;
        }
      }
      if (*abort)
        for (int k = issued - S; k < issued; ++k)
          if (k >= 0) {
            drain_wait(&xfull[k % S], (uint32_t)((k / S) & 1));
            drain_wait(&rawfull[k % S], (uint32_t)((k / S) & 1));
          }
    }
  } else if (warp == kWarpMma) {
    // ---- MMA issuer ------------------------------------------------------------
    if (lane == 0) {
      int it = 0, local = 0, committed = 0;
      for (int tile = blockIdx.x; tile < a.tiles && !*abort; tile += gridDim.x, ++local) {
        const int b = kDB ? (local & 1) : 0;
        const int use = kDB ? (local >> 1) : local;  // earlier uses of accumulator b
        if (use >= 1 && !pf_wait(&acce[b], (uint32_t)((use - 1) & 1), abort, a.status)) break;
        tc_fence_after();
        bool ok = true;
        for (int g = 0; g < a.ng; ++g, ++it) {
          const int s = it % S;
          const uint32_t par = (uint32_t)((it / S) & 1);
          if (!pf_wait(&xfull[s], par, abort, a.status) || !pf_wait(&deq[s], par, abort, a.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t xa = smem_addr(sm + L::x_off + (size_t)s * kXStage);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t a0 = umma_desc_sw128(xa + kk * 32), a1 = umma_desc_sw128(xa + kXBox + kk * 32);
#pragma unroll
            for (int si = 0; si < NS; ++si) {
              const uint64_t bd = umma_desc_sw128(smem_addr(sm + L::w_off + (size_t)(s * NS + si) * kWStage) + kk * 32);
              const uint32_t col = (uint32_t)((b * NS + si) * 2 * kBN);
              const uint32_t acc = (g > 0 || kk > 0) ? 1u : 0u;
              mma_bf16_ss(tmem + col, a0, bd, acc);
              mma_bf16_ss(tmem + col + kBN, a1, bd, acc);
            }
          }
          umma_commit(&empty[s]);  // frees the stage once these MMAs are done
          committed = it + 1;
        }
        if (!ok) break;
        umma_commit(&accf[b]);
      }
      if (*abort && committed > 0)
        drain_wait(&empty[(committed - 1) % S], (uint32_t)(((committed - 1) / S) & 1));
    }
  } else if (warp < kWarpEpi0) {
    // ---- dequant: raw slab-group -> bf16 B tile (K-major, 128-byte swizzle) ----
    const int t = threadIdx.x;  // 0..127
    int it = 0;
    for (int tile = blockIdx.x; tile < a.tiles && !*abort; tile += gridDim.x) {
      bool ok = true;
      for (int g = 0; g < a.ng; ++g, ++it) {
        const int s = it % S;
        if (!pf_wait(&rawfull[s], (uint32_t)((it / S) & 1), abort, a.status)) {
          ok = false;
          break;
        }
#pragma unroll
        for (int si = 0; si < NS; ++si) {
          const unsigned char *raw = sm + L::raw_off + (size_t)(s * NS + si) * kRawStage;
          unsigned char *wt = sm + L::w_off + (size_t)(s * NS + si) * kWStage;
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            const int ch = t + half * 128, tl = ch >> 5, ln = ch & 31, r = ln >> 2, c = ln & 3;
            const uint4 w4 = *reinterpret_cast<const uint4 *>(raw + ch * 16);
            const uint2 q = *reinterpret_cast<const uint2 *>(raw + 4096 + tl * 64 + r * 8);
            const float s0 = sb_to_f32<SF16>(q.x & 0xffffu), b0 = sb_to_f32<SF16>(q.x >> 16);
            const float s8 = sb_to_f32<SF16>(q.y & 0xffffu), b8 = sb_to_f32<SF16>(q.y >> 16);
            const uint32_t wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int hi8 = (i >> 1) & 1;
                const float sc = hi8 ? s8 : s0, bi = hi8 ? b8 : b0;
                const float v0 = fmaf((float)((wv[j] >> (4 * i)) & 0xFu), sc, bi);
                const float v1 = fmaf((float)((wv[j] >> (4 * i + 16)) & 0xFu), sc, bi);
                const int row = tl * 16 + r + 8 * hi8;                        // 0..127
                const int chunk = 4 * (j >> 1) + (j & 1) + 2 * (i & 1);      // 16-byte column of the row
                *reinterpret_cast<uint32_t *>(wt + (row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4) +
                                              4 * c) = pack_bf16(v0, v1);
              }
            }
          }
        }
        fence_proxy_async_smem();  // generic-proxy writes -> tcgen05 reads
        __syncwarp();
        if (lane == 0) mbar_arrive(&deq[s]);
      }
      if (!ok) break;
    }
  } else {
    // ---- epilogue: TMEM -> registers -> y --------------------------------------
    const int q4 = warp & 3;  // this warp's TMEM lane quarter
    int local = 0;
    for (int tile = blockIdx.x; tile < a.tiles && !*abort; tile += gridDim.x, ++local) {
      const int mt = tile % a.m_tiles, nt = tile / a.m_tiles;
      const int b = kDB ? (local & 1) : 0;
      const int use = kDB ? (local >> 1) : local;
      if (!pf_wait(&accf[b], (uint32_t)(use & 1), abort, a.status)) break;
      tc_fence_after();
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        const int token = mt * kBM + h * 128 + q4 * 32 + lane;
#pragma unroll 1
        for (int cc = 0; cc < kBN / 32; ++cc) {
          const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
          uint32_t u[32];
          float v[32];
          tmem_ld32(tmem + lane_base + (uint32_t)(b * NS * 2 * kBN + h * kBN + cc * 32), u);
          if constexpr (NS == 2) {
            uint32_t uu[32];
            tmem_ld32(tmem + lane_base + (uint32_t)(2 * kBN + h * kBN + cc * 32), uu);
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = silu_mul(__uint_as_float(u[e]), __uint_as_float(uu[e]));
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(u[e]);
          }
          store_row32(a, token, nt * kBN + cc * 32, v);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[b]);
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

template <int NS, int S, bool SF16>
cudaError_t prefill_launch_t(const CUtensorMap &map, const PfArgs &a, int grid, cudaStream_t stream) {
  auto *k = &prefill_kernel<NS, S, SF16>;
  static DeviceOnce once;
  const size_t smem = PfSmem<NS, S>::alloc;
  cudaError_t e = once.run([&] { return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); });
  if (e != cudaSuccess) return e;
  k<<<grid, kPfThreads, smem, stream>>>(map, a);
  return cudaGetLastError();
}

}  // namespace

bool prefill_supported(int m, bool x_f32) { return m > 8 && !x_f32; }

cudaError_t prefill_launch(const thq4_weight &w0, const thq4_weight *w1, const void *x, int m, void *y, bool y_f32,
                           cudaStream_t stream) {
  // x [m][k] bf16 as a 2-D tensor (k innermost), 64 x 128 boxes, 128-byte swizzle
  // the driver's tensor-map encoder, looked up through the runtime so the
  // library needs no link-time driver dependency
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void *fn = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!encode) return cudaErrorNotSupported;
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)w0.in, (cuuint64_t)m};
  const cuuint64_t strides[1] = {(cuuint64_t)w0.in * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kBK, 128};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult cr = encode(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(x), dims,
                                             strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return cudaErrorInvalidValue;
  PfArgs a{};
  const bool gate_up = w1 != nullptr;
  a.qw[0] = static_cast<const uint8_t *>(w0.qw);
  a.sb[0] = static_cast<const uint8_t *>(w0.sb);
  a.qw[1] = gate_up ? static_cast<const uint8_t *>(w1->qw) : nullptr;
  a.sb[1] = gate_up ? static_cast<const uint8_t *>(w1->sb) : nullptr;
  a.y = y;
  a.status = status_word();
  a.m = m;
  a.n = w0.out;
  a.ng = w0.in / kBK;
  a.m_tiles = (m + kBM - 1) / kBM;
  const long long tiles = (long long)a.m_tiles * row_slabs(w0.out);
  if (tiles >= (1ll << 31)) return cudaErrorInvalidValue;
  a.tiles = (int)tiles;
  a.yf32 = y_f32 ? 1 : 0;
  const int grid = (int)std::min<long long>(tiles, device_sm_count());
  const bool f16 = w0.sb_dtype == THQ4_F16;
  if (gate_up)
    return f16 ? prefill_launch_t<2, 3, true>(map, a, grid, stream) : prefill_launch_t<2, 3, false>(map, a, grid, stream);
  return f16 ? prefill_launch_t<1, 4, true>(map, a, grid, stream) : prefill_launch_t<1, 4, false>(map, a, grid, stream);
}

}  // namespace thq4
