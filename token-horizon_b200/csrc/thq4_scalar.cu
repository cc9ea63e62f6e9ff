// thq4_scalar.cu -- the scalar GPU reference product (thq4_linear_scalar).
//
// Replaces the reference's scalar Metal kernels AffineQmv / AffineQmm
// (engine/src/quant_kernel.rs:1026-1147 affine_qmv, :1634-1740 affine_qmm;
// ops :2686-2766, :5766-5834): a plain product with nothing tuned, against
// which the reference's tests check the tuned kernels on the same device
// (scalar_ref, qwen35.rs:6928-6938, used by the qmvt tests :6963-7008).
//
// Arithmetic, as affine_qmm's: every weight is dequantised in f32,
// w = q * s + b (one fused multiply-add, as Metal contracts
// `float(q) * sc + bi`), and the products accumulate in f32.  The order is
// fixed, so the kernel is deterministic: one warp per output row; lane l
// takes the eight consecutive k at 8 l, 8 l + 256, 8 l + 512, ... and adds
// w * x in k order into one f32 accumulator per token (fused), then the 32
// lanes combine by xor butterfly (partners 16, 8, 4, 2, 1).  It reads the
// frag layout (thq4_common.cuh) one 16-bit half-word pair at a time; speed
// is not its purpose.
#include "thq4_common.cuh"
#include "thq4_internal.h"

namespace thq4 {
namespace {

constexpr int kScalarRowsPerCta = 8;   // one warp per row
constexpr int kScalarMaxTokens = 8;    // affine_qmm's M <= 8 accumulators

template <bool SF16>
__global__ void __launch_bounds__(kScalarRowsPerCta * 32) scalar_kernel(const uint32_t *qw, const uint16_t *sb,
                                                                          int out, int in, const void *x, int xf32,
                                                                          int m, void *y, int yf32) {
  const int lane = threadIdx.x & 31;
  const int n = blockIdx.x * kScalarRowsPerCta + (threadIdx.x >> 5);
  if (n >= out) return;  // whole warps leave together
  const int ng = in / kGroup;
  const int slab = n / kSlabRows, t = (n % kSlabRows) / kTileRows, rr = n % kTileRows, r = rr % 8, irow = rr / 8;
  float acc[kScalarMaxTokens];
#pragma unroll
  for (int tk = 0; tk < kScalarMaxTokens; ++tk) acc[tk] = 0.0f;
  for (int k0 = 8 * lane; k0 < in; k0 += 256) {
    // the eight k share one word j and one row half; the pair (2c, 2c + 1)
    // sits at bits 4i and 4i + 16 of the word of lane column c
    const int g = k0 / kGroup, kk = k0 % kGroup;
    const int j = 2 * ((kk >> 5) & 1) + ((kk >> 3) & 1);
    const int i = ((kk >> 4) & 1) + 2 * irow;
    const size_t chunk = ((size_t)slab * ng + g) * kSlabTiles + t;
    const uint2 quad = reinterpret_cast<const uint2 *>(sb)[chunk * 8 + r];
    const uint32_t qd = irow ? quad.y : quad.x;
    const float s = sb_to_f32<SF16>(qd & 0xffffu), b = sb_to_f32<SF16>(qd >> 16);
    float w[8];
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      const uint32_t word = qw[(chunk * 32 + 4 * r + cc) * 4 + j];
      w[2 * cc] = fmaf((float)((word >> (4 * i)) & 0xFu), s, b);
      w[2 * cc + 1] = fmaf((float)((word >> (4 * i + 16)) & 0xFu), s, b);
    }
#pragma unroll
    for (int tk = 0; tk < kScalarMaxTokens; ++tk) {
      if (tk >= m) break;
      float xv[8];
      if (xf32) {
        const float4 *p = reinterpret_cast<const float4 *>(static_cast<const float *>(x) + (size_t)tk * in + k0);
        const float4 u0 = p[0], u1 = p[1];
        xv[0] = u0.x, xv[1] = u0.y, xv[2] = u0.z, xv[3] = u0.w, xv[4] = u1.x, xv[5] = u1.y, xv[6] = u1.z,
        xv[7] = u1.w;
      } else {
        const uint4 u = *reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(x) + (size_t)tk * in + k0);
        const uint32_t wv[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          xv[2 * e] = __uint_as_float(wv[e] << 16);
          xv[2 * e + 1] = __uint_as_float(wv[e] & 0xffff0000u);
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[tk] = fmaf(w[e], xv[e], acc[tk]);
    }
  }
#pragma unroll
  for (int tk = 0; tk < kScalarMaxTokens; ++tk) {
    float v = acc[tk];
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    acc[tk] = v;
  }
  if (lane == 0)
    for (int tk = 0; tk < m; ++tk) {
      if (yf32)
        static_cast<float *>(y)[(size_t)tk * out + n] = acc[tk];
      else
        static_cast<uint16_t *>(y)[(size_t)tk * out + n] = f32_to_bf16_bits(acc[tk]);
    }
}

}  // namespace

cudaError_t scalar_launch(const thq4_weight &w, const void *x, bool x_f32, int m, void *y, bool y_f32,
                          cudaStream_t stream) {
  const int grid = (w.out + kScalarRowsPerCta - 1) / kScalarRowsPerCta;
  const int xb = x_f32 ? 4 : 2, yb = y_f32 ? 4 : 2;
  for (int t0 = 0; t0 < m; t0 += kScalarMaxTokens) {
    const int mt = m - t0 < kScalarMaxTokens ? m - t0 : kScalarMaxTokens;
    const void *xp = static_cast<const char *>(x) + (size_t)t0 * w.in * xb;
    void *yp = static_cast<char *>(y) + (size_t)t0 * w.out * yb;
    if (w.sb_dtype == THQ4_F16)
      scalar_kernel<true><<<grid, kScalarRowsPerCta * 32, 0, stream>>>(
          static_cast<const uint32_t *>(w.qw), static_cast<const uint16_t *>(w.sb), w.out, w.in, xp, x_f32, mt, yp,
          y_f32);
    else
      scalar_kernel<false><<<grid, kScalarRowsPerCta * 32, 0, stream>>>(
          static_cast<const uint32_t *>(w.qw), static_cast<const uint16_t *>(w.sb), w.out, w.in, xp, x_f32, mt, yp,
          y_f32);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace thq4
