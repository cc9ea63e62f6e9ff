// thq4_gemv.cu -- decode (m = 1) and spec-verify (m <= 8) Q4 projections.
//
// Replaces the reference's m = 1 matvec AffineQmvT / qmvt<RPL,NSG,GateUp>
// (engine/src/quant_kernel.rs:2768-3136) and its m <= 8 decode/verify families
// AffineQmpp (th_mpp_tile, :1793-2569), AffineQsg (:1149-1632) and AffineQmm
// (:1634-1740), with one kernel.
//
// The path is bound by HBM bandwidth (0.5625 bytes per weight, each read once),
// so the design goal is to keep enough bytes in flight and to spend few issue
// slots per weight:
//   - each warp owns one 16-row tile and a contiguous range of quant groups;
//     per group a lane issues one 16-byte streaming load of nibbles (the warp
//     reads one contiguous 512-byte chunk) and one 8-byte scale/bias load,
//     two stages of U groups ahead;
//   - the multiply runs on the tensor cores with the weight as the A operand
//     (16 rows) and the m tokens as N (8 columns): mma.m16n8k16 bf16 with f32
//     accumulation.  A nibble pair becomes a bf16 pair (128 + q) by one shift
//     and one LOP3 -- exact -- and the 128 offset is removed per group in the
//     epilogue together with the bias, following the per-group form of the
//     reference kernels (quant_kernel.rs:1994-2001, 2887-2890):
//         y += s * sum((128+q) x) + (b - 128 s) * sum(x)
//            = s * sum(q x) + b * sum(x);
//   - an f32 activation is split into bf16 hi + lo parts that occupy two of
//     the eight N columns, so an f32 GEMV keeps ~16 significant bits of x at
//     no extra weight traffic;
//   - the activation is staged once per CTA in shared memory in B-fragment
//     order (one 16-byte LDS per lane per two k-steps), with its per-group
//     sums;
//   - K may be split over the warps of a CTA (split-K); partial sums are
//     reduced through shared memory in a fixed slice order, so results are
//     bitwise deterministic (the reference asserts the same,
//     qwen35.rs:6986-6988), and no cross-CTA synchronisation exists.
#include "thq4_common.cuh"
#include "thq4_internal.h"

#include <type_traits>

namespace thq4 {

namespace {

constexpr int kStages = 2;  // register double-buffering of U-group stages

struct GemvArgs {
  const uint4 *qw0;  // gate (or the only) weight: frag16 nibbles
  const uint2 *sb0;
  const uint4 *qw1;  // up weight (gate/up only)
  const uint2 *sb1;
  const void *x;     // [m][in]
  void *y;           // [m][out]
  int m;             // tokens in this launch
  int in, ng, out, rtiles;
  int ks;            // K slices per row tile (warps sharing a tile)
  int rt_per_cta;    // row tiles per CTA
  int gps;           // groups per slice
  int mcols;         // B columns in use: m (bf16 x) or 2m (f32 x)
};

// Shared memory: xs (fragment-order activation), xsum, then the split-K
// reduction buffer.
__host__ __device__ inline size_t xs_bytes(int ng, int mcols) { return (size_t)ng * 2 * mcols * 64; }
__host__ __device__ inline size_t xsum_bytes(int ng) { return (size_t)ng * 8 * sizeof(float); }
__host__ __device__ inline size_t red_bytes(int ks, int rt, bool gate_up) {
  return (size_t)(ks > 1 ? ks - 1 : 0) * rt * 32 * 4 * sizeof(float) * (gate_up ? 2 : 1);
}

// Stage x into shared memory in B-fragment order.  Column r of the B operand
// is token r (bf16 x) or token r/2's hi (r even) / lo (r odd) part (f32 x).
// Entry ((g*2 + h)*mcols + r)*4 + c holds, for k-steps j = 2h and 2h+1 of
// group g, the pairs {x[2c], x[2c+1]} and {x[2c+8], x[2c+9]} (k relative to
// 64 g + 16 j).  Per-(group, column) sums go to xsum[g*8 + r] (zero for
// unused columns).  Each thread takes 8 consecutive k of one token; the 8
// threads of a group reduce their sums with a fixed shuffle tree.
template <bool XF32>
__device__ void stage_x(const GemvArgs &a, uint16_t *xs16, float *xsum) {
  const int kb8 = a.in / 8;  // 8-element blocks per token
  const int total = a.m * kb8;
  // zero xsum for unused columns (and all when m < 8)
  for (int i = threadIdx.x; i < a.ng * 8; i += blockDim.x) xsum[i] = 0.0f;
  __syncthreads();
  // round up so every lane of a warp takes part in the shuffles
  const int span = (total + 31) / 32 * 32;
  for (int idx = threadIdx.x; idx < span; idx += blockDim.x) {
    const bool live = idx < total;
    const int t = live ? idx / kb8 : 0;
    const int k0 = live ? (idx % kb8) * 8 : 0;
    float v[2][8];  // [part][element]
    if (live) {
      if constexpr (XF32) {
        const float4 *xp = reinterpret_cast<const float4 *>(
            static_cast<const float *>(a.x) + (size_t)t * a.in + k0);
        const float4 p0 = xp[0], p1 = xp[1];
        const float f[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float hi = round_bf16(f[e]);
          v[0][e] = hi;
          v[1][e] = round_bf16(f[e] - hi);
        }
      } else {
        const uint4 p = *reinterpret_cast<const uint4 *>(
            static_cast<const uint16_t *>(a.x) + (size_t)t * a.in + k0);
        const uint32_t w[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          v[0][2 * e] = __uint_as_float(w[e] << 16);
          v[0][2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) v[1][e] = 0.0f;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[0][e] = v[1][e] = 0.0f;
    }
    const int g = k0 / 64, kk = k0 % 64;  // kk in {0, 8, ..., 56}
    const int j = kk / 16, hi8 = (kk % 16) / 8;  // k-step; second half of the step
    const int h = j >> 1, comp = (j & 1) * 2 + hi8;
    constexpr int parts = XF32 ? 2 : 1;
#pragma unroll
    for (int p = 0; p < parts; ++p) {
      const int col = XF32 ? 2 * t + p : t;
      if (live) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int c = e >> 1, half = e & 1;
          const size_t entry = ((size_t)(g * 2 + h) * a.mcols + col) * 4 + c;
          xs16[entry * 8 + comp * 2 + half] = f32_to_bf16_bits(v[p][e]);
        }
      }
      float s = ((v[p][0] + v[p][1]) + (v[p][2] + v[p][3])) + ((v[p][4] + v[p][5]) + (v[p][6] + v[p][7]));
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      s += __shfl_xor_sync(0xffffffffu, s, 4);
      if (live && (idx & 7) == 0) xsum[g * 8 + col] = s;
    }
  }
  __syncthreads();
}

template <bool XF32, bool SF16, bool GATE_UP, bool YF32>
__global__ void __launch_bounds__(512) gemv_kernel(const GemvArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  uint16_t *xs16 = reinterpret_cast<uint16_t *>(smem);
  float *xsum = reinterpret_cast<float *>(smem + xs_bytes(a.ng, a.mcols));
  float *red = xsum + a.ng * 8;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r = lane >> 2, c = lane & 3;
  const int ks = warp % a.ks, rtl = warp / a.ks;
  const int rt = blockIdx.x * a.rt_per_cta + rtl;
  const bool tile_live = rt < a.rtiles;
  const int g0 = min(a.ng, ks * a.gps), g1 = min(a.ng, g0 + a.gps);
  const uint64_t pol = evict_first_policy();

  const uint4 *q0 = a.qw0 + ((size_t)(tile_live ? rt : 0) * a.ng) * 32 + lane;
  const uint2 *s0 = a.sb0 + ((size_t)(tile_live ? rt : 0) * a.ng) * 8 + r;
  const uint4 *q1 = GATE_UP ? a.qw1 + ((size_t)(tile_live ? rt : 0) * a.ng) * 32 + lane : nullptr;
  const uint2 *s1 = GATE_UP ? a.sb1 + ((size_t)(tile_live ? rt : 0) * a.ng) * 8 + r : nullptr;
  constexpr int NS = GATE_UP ? 2 : 1;
  // quant groups per register stage (gate/up streams two weights at once)
  constexpr int kU = GATE_UP ? 2 : 4;

  uint4 qv[kStages][kU][NS];
  uint2 sv[kStages][kU][NS];
  // ST is a template argument so the register arrays stay in registers
  auto issue = [&](auto stage, int gb) {
    constexpr int ST = decltype(stage)::value;
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int g = gb + u;
      if (tile_live && g < g1) {
        qv[ST][u][0] = ld_stream_v4(q0 + (size_t)g * 32, pol);
        sv[ST][u][0] = ld_stream_v2(s0 + (size_t)g * 8, pol);
        if constexpr (GATE_UP) {
          qv[ST][u][1] = ld_stream_v4(q1 + (size_t)g * 32, pol);
          sv[ST][u][1] = ld_stream_v2(s1 + (size_t)g * 8, pol);
        }
      }
    }
  };
  // start streaming weights before staging x: the loads overlap the prologue
  issue(std::integral_constant<int, 0>{}, g0);
  stage_x<XF32>(a, xs16, xsum);

  float y[NS][4];
#pragma unroll
  for (int s = 0; s < NS; ++s)
#pragma unroll
    for (int i = 0; i < 4; ++i) y[s][i] = 0.0f;

  const uint4 *xs4 = reinterpret_cast<const uint4 *>(xs16);
  const bool col_live = r < a.mcols;
  auto compute = [&](auto stage, int gb) {
    constexpr int ST = decltype(stage)::value;
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int g = gb + u;
      if (!tile_live || g >= g1) break;
      uint4 xa = make_uint4(0, 0, 0, 0), xb = make_uint4(0, 0, 0, 0);
      if (col_live) {
        xa = xs4[((size_t)(g * 2 + 0) * a.mcols + r) * 4 + c];
        xb = xs4[((size_t)(g * 2 + 1) * a.mcols + r) * 4 + c];
      }
      const float2 xsm = *reinterpret_cast<const float2 *>(xsum + g * 8 + 2 * c);
#pragma unroll
      for (int s = 0; s < NS; ++s) {
        const uint4 w = qv[ST][u][s];
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        mma_bf16_16816(acc, nib_bf16x2(w.x, 0), nib_bf16x2(w.x, 4), nib_bf16x2(w.x, 8),
                       nib_bf16x2(w.x, 12), xa.x, xa.y);
        mma_bf16_16816(acc, nib_bf16x2(w.y, 0), nib_bf16x2(w.y, 4), nib_bf16x2(w.y, 8),
                       nib_bf16x2(w.y, 12), xa.z, xa.w);
        mma_bf16_16816(acc, nib_bf16x2(w.z, 0), nib_bf16x2(w.z, 4), nib_bf16x2(w.z, 8),
                       nib_bf16x2(w.z, 12), xb.x, xb.y);
        mma_bf16_16816(acc, nib_bf16x2(w.w, 0), nib_bf16x2(w.w, 4), nib_bf16x2(w.w, 8),
                       nib_bf16x2(w.w, 12), xb.z, xb.w);
        const uint2 q = sv[ST][u][s];
        const float sr = sb_to_f32<SF16>(q.x & 0xffffu);
        const float br = sb_to_f32<SF16>(q.x >> 16);
        const float sr8 = sb_to_f32<SF16>(q.y & 0xffffu);
        const float br8 = sb_to_f32<SF16>(q.y >> 16);
        const float bpr = fmaf(-128.0f, sr, br), bpr8 = fmaf(-128.0f, sr8, br8);
        y[s][0] = fmaf(bpr, xsm.x, fmaf(sr, acc[0], y[s][0]));
        y[s][1] = fmaf(bpr, xsm.y, fmaf(sr, acc[1], y[s][1]));
        y[s][2] = fmaf(bpr8, xsm.x, fmaf(sr8, acc[2], y[s][2]));
        y[s][3] = fmaf(bpr8, xsm.y, fmaf(sr8, acc[3], y[s][3]));
      }
    }
  };
  // two register stages: while one stage's groups are multiplied, the next
  // stage's loads are in flight
  for (int gb = g0; gb < g1; gb += 2 * kU) {
    if (gb + kU < g1) issue(std::integral_constant<int, 1>{}, gb + kU);
    compute(std::integral_constant<int, 0>{}, gb);
    if (gb + kU >= g1) break;
    if (gb + 2 * kU < g1) issue(std::integral_constant<int, 0>{}, gb + 2 * kU);
    compute(std::integral_constant<int, 1>{}, gb + kU);
  }

  // split-K: slices 1..ks-1 hand their partials to slice 0, which adds them
  // in slice order
  if (a.ks > 1) {
    if (ks > 0) {
      float *dst = red + ((size_t)((ks - 1) * a.rt_per_cta + rtl) * 32 + lane) * 4 * NS;
#pragma unroll
      for (int s = 0; s < NS; ++s)
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[s * 4 + i] = y[s][i];
    }
    __syncthreads();
    if (ks > 0) return;
    for (int k = 1; k < a.ks; ++k) {
      const float *src = red + ((size_t)((k - 1) * a.rt_per_cta + rtl) * 32 + lane) * 4 * NS;
#pragma unroll
      for (int s = 0; s < NS; ++s)
#pragma unroll
        for (int i = 0; i < 4; ++i) y[s][i] += src[s * 4 + i];
    }
  }
  if (!tile_live) return;

  // y[s][0..3] = rows (r, r, r+8, r+8) x columns (2c, 2c+1, 2c, 2c+1)
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int row = rt * 16 + r + 8 * half;
    if (row >= a.out) continue;
    if constexpr (XF32) {
      // columns 2c (hi) and 2c+1 (lo) are the two parts of token c
      const int t = c;
      if (t >= a.m) continue;
      float v = y[0][2 * half] + y[0][2 * half + 1];
      if constexpr (GATE_UP) v = silu_mul(v, y[1][2 * half] + y[1][2 * half + 1]);
      if constexpr (YF32)
        static_cast<float *>(a.y)[(size_t)t * a.out + row] = v;
      else
        static_cast<uint16_t *>(a.y)[(size_t)t * a.out + row] = f32_to_bf16_bits(v);
    } else {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = 2 * c + e;
        if (t >= a.m) continue;
        float v = y[0][2 * half + e];
        if constexpr (GATE_UP) v = silu_mul(v, y[1][2 * half + e]);
        if constexpr (YF32)
          static_cast<float *>(a.y)[(size_t)t * a.out + row] = v;
        else
          static_cast<uint16_t *>(a.y)[(size_t)t * a.out + row] = f32_to_bf16_bits(v);
      }
    }
  }
}

template <bool XF32, bool SF16, bool GATE_UP, bool YF32>
cudaError_t launch_one(const GemvArgs &a, int threads, size_t smem, cudaStream_t stream) {
  auto *k = &gemv_kernel<XF32, SF16, GATE_UP, YF32>;
  static DeviceOnce once;
  cudaError_t e = once.run([&] {
    return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvMaxSmem);
  });
  if (e != cudaSuccess) return e;
  const int grid = (a.rtiles + a.rt_per_cta - 1) / a.rt_per_cta;
  k<<<grid, threads, smem, stream>>>(a);
  return cudaGetLastError();
}

template <bool XF32, bool SF16>
cudaError_t dispatch_y(const GemvArgs &a, bool gate_up, bool yf32, int threads, size_t smem,
                       cudaStream_t s) {
  if (gate_up)
    return yf32 ? launch_one<XF32, SF16, true, true>(a, threads, smem, s)
                : launch_one<XF32, SF16, true, false>(a, threads, smem, s);
  return yf32 ? launch_one<XF32, SF16, false, true>(a, threads, smem, s)
              : launch_one<XF32, SF16, false, false>(a, threads, smem, s);
}

}  // namespace

GemvPlan gemv_plan(int out, int in, int m, bool x_f32, bool gate_up) {
  GemvPlan p{};
  const int rtiles = row_tiles(out), ng = in / kGroup;
  const int sms = device_sm_count();
  // tokens per launch: B has 8 columns; f32 x takes two per token.  Shrink the
  // pass further if the staged activation would not fit in shared memory.
  int per = x_f32 ? 4 : 8;
  if (per > m) per = m;
  GemvCfg cfg = gemv_cfg_override();
  int ks;
  if (cfg.ks > 0) {
    ks = cfg.ks;
  } else {
    // enough warps to keep ~24 resident per SM streaming, at least 4 groups
    // per warp, at most 16 slices
    ks = 1;
    while (ks < 16 && (long)rtiles * ks < (long)sms * 24 && (ng + 2 * ks - 1) / (2 * ks) >= 4) ks *= 2;
  }
  if (ks > ng) ks = ng;
  int warps = cfg.warps > 0 ? cfg.warps : (ks >= 16 ? 16 : 8);
  if (warps < ks) warps = ks;
  int rt = warps / ks;
  if (rt < 1) rt = 1;
  for (;;) {
    const int mcols = x_f32 ? 2 * per : per;
    const size_t smem = xs_bytes(ng, mcols) + xsum_bytes(ng) + red_bytes(ks, rt, gate_up);
    if (smem <= (size_t)kGemvMaxSmem || per == 1) {
      p.smem = smem;
      break;
    }
    per = (per + 1) / 2;
  }
  p.tokens_per_pass = per;
  p.ks = ks;
  p.rt_per_cta = rt;
  p.threads = 32 * ks * rt;
  p.gps = (ng + ks - 1) / ks;
  p.grid = (rtiles + rt - 1) / rt;
  p.ok = p.smem <= (size_t)kGemvMaxSmem;
  return p;
}

cudaError_t gemv_launch(const thq4_weight &w0, const thq4_weight *w1, const void *x, bool x_f32,
                        int m, void *y, bool y_f32, cudaStream_t stream) {
  const bool gate_up = w1 != nullptr;
  const GemvPlan p = gemv_plan(w0.out, w0.in, m, x_f32, gate_up);
  if (!p.ok) return cudaErrorInvalidConfiguration;
  const int xb = x_f32 ? 4 : 2, yb = y_f32 ? 4 : 2;
  for (int t0 = 0; t0 < m; t0 += p.tokens_per_pass) {
    const int mt = min(p.tokens_per_pass, m - t0);
    GemvArgs a{};
    a.qw0 = static_cast<const uint4 *>(w0.qw);
    a.sb0 = static_cast<const uint2 *>(w0.sb);
    a.qw1 = gate_up ? static_cast<const uint4 *>(w1->qw) : nullptr;
    a.sb1 = gate_up ? static_cast<const uint2 *>(w1->sb) : nullptr;
    a.x = static_cast<const char *>(x) + (size_t)t0 * w0.in * xb;
    a.y = static_cast<char *>(y) + (size_t)t0 * w0.out * yb;
    a.m = mt;
    a.in = w0.in;
    a.ng = w0.in / kGroup;
    a.out = w0.out;
    a.rtiles = row_tiles(w0.out);
    a.ks = p.ks;
    a.rt_per_cta = p.rt_per_cta;
    a.gps = p.gps;
    a.mcols = x_f32 ? 2 * mt : mt;
    const size_t smem = xs_bytes(a.ng, a.mcols) + xsum_bytes(a.ng) + red_bytes(p.ks, p.rt_per_cta, gate_up);
    const bool f16 = w0.sb_dtype == THQ4_F16;
    cudaError_t e;
    if (x_f32)
      e = f16 ? dispatch_y<true, true>(a, gate_up, y_f32, p.threads, smem, stream)
              : dispatch_y<true, false>(a, gate_up, y_f32, p.threads, smem, stream);
    else
      e = f16 ? dispatch_y<false, true>(a, gate_up, y_f32, p.threads, smem, stream)
              : dispatch_y<false, false>(a, gate_up, y_f32, p.threads, smem, stream);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace thq4
