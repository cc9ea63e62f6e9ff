// thq4_repack.cu -- load-time repack of the reference's Q4 formats into the
// frag layout, and the dequantise-to-bf16 kernel.
//
// Replaces QLin::tiled's host-thread repack (engine/src/qwen35.rs:629-697)
// with a device kernel, and reads every layout the reference stores:
//   MLX row-major    wq [out][in/8] + sb [out][2 ng]   (qwen35.rs:249-300)
//   QLin::tiled      [tile][group][col][8] + planar sb  (qwen35.rs:629-697,
//                    addressing quant_kernel.rs:1085-1101)
//   Splash slab      [weights][scales][biases]          (moe_expert_slab.h:15-28)
// AffineDequant (quant_kernel.rs:1765-1781) becomes dequant_kernel below.
#include "thq4_common.cuh"
#include "thq4_internal.h"

namespace thq4 {
namespace {

struct RepackArgs {
  int layout;
  const uint32_t *w;   // source words (MLX / tiled) or slab bytes
  const uint16_t *sb;  // source scale/bias (MLX / tiled)
  int src_out, in, ng, row_begin, rows, slabs;
  uint32_t *dq;        // frag nibbles
  uint16_t *dsb;       // frag quads
};

// The 8 words of source row `row`, group g (zeros for rows past `rows`).
__device__ inline void load_row_group(const RepackArgs &a, int local_row, int g, uint32_t (&wv)[8],
                                      uint16_t &s, uint16_t &b) {
  if (local_row >= a.rows) {
#pragma unroll
    for (int i = 0; i < 8; ++i) wv[i] = 0;
    s = b = 0;
    return;
  }
  const int row = a.row_begin + local_row;
  if (a.layout == THQ4_SRC_MLX) {
    const uint4 *p = reinterpret_cast<const uint4 *>(a.w + (size_t)row * a.ng * 8 + (size_t)g * 8);
    const uint4 lo = p[0], hi = p[1];
    wv[0] = lo.x, wv[1] = lo.y, wv[2] = lo.z, wv[3] = lo.w;
    wv[4] = hi.x, wv[5] = hi.y, wv[6] = hi.z, wv[7] = hi.w;
    s = a.sb[(size_t)row * 2 * a.ng + g];
    b = a.sb[(size_t)row * 2 * a.ng + a.ng + g];
    return;
  }
  // tiled and slab share the word order [tile][group][col][8]
  const size_t t = (size_t)row / 256, col = (size_t)row % 256;
  const uint4 *p = reinterpret_cast<const uint4 *>(a.w + t * a.ng * 2048 + (size_t)g * 2048 + col * 8);
  const uint4 lo = p[0], hi = p[1];
  wv[0] = lo.x, wv[1] = lo.y, wv[2] = lo.z, wv[3] = lo.w;
  wv[4] = hi.x, wv[5] = hi.y, wv[6] = hi.z, wv[7] = hi.w;
  const size_t prm = (t * a.ng + g) * 256 + col;
  if (a.layout == THQ4_SRC_TILED) {
    const size_t tiles = ((size_t)a.src_out + 255) / 256;
    s = a.sb[prm];
    b = a.sb[prm + tiles * a.ng * 256];
  } else {  // slab: scales at elements/2 bytes, biases elements/32 bytes later
    const size_t elements = (size_t)a.src_out * a.in;
    const uint16_t *sc = reinterpret_cast<const uint16_t *>(reinterpret_cast<const char *>(a.w) + elements / 2);
    const uint16_t *bi = reinterpret_cast<const uint16_t *>(reinterpret_cast<const char *>(a.w) + elements / 2 + elements / 32);
    s = sc[prm];
    b = bi[prm];
  }
}

// One thread per (chunk, lane): four output words and, for c == 0, the quad
// of rows r and r+8.  Chunk (slab * ng + g) * 8 + t is tile t of the slab.
__global__ void repack_kernel(const RepackArgs a) {
  const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t total = (size_t)a.slabs * a.ng * kSlabTiles * 32;
  if (tid >= total) return;
  const int lane = (int)(tid % 32);
  const size_t chunk = tid / 32;
  const int t = (int)(chunk % kSlabTiles);
  const size_t sg = chunk / kSlabTiles;
  const int g = (int)(sg % a.ng), slab = (int)(sg / a.ng);
  const int r = lane >> 2, c = lane & 3;
  const int row0 = slab * kSlabRows + t * kTileRows;
  uint32_t w0[8], w1[8];
  uint16_t s0, b0, s1, b1;
  load_row_group(a, row0 + r, g, w0, s0, b0);
  load_row_group(a, row0 + r + 8, g, w1, s1, b1);
  auto nib = [&](int which, int k) -> uint32_t {  // k within the group
    const uint32_t word = which ? w1[k >> 3] : w0[k >> 3];
    return (word >> (4 * (k & 7))) & 0xFu;
  };
  uint32_t out[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t word = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      word |= nib((i >> 1) & 1, frag_k(j, i, c)) << (4 * i);
    out[j] = word;
  }
  reinterpret_cast<uint4 *>(a.dq)[tid] = make_uint4(out[0], out[1], out[2], out[3]);
  if (c == 0) {
    uint2 q;
    q.x = (uint32_t)s0 | ((uint32_t)b0 << 16);
    q.y = (uint32_t)s1 | ((uint32_t)b1 << 16);
    reinterpret_cast<uint2 *>(a.dsb)[chunk * 8 + r] = q;
  }
}

// Copies an already packed frag weight (rows must cover whole tiles).
__global__ void copy_kernel(const uint4 *src, uint4 *dst, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = src[i];
}

// y[n][k] = bf16(q * s + b), one thread per 8 consecutive k of a row.
template <bool SF16>
__global__ void dequant_kernel(const uint32_t *qw, const uint16_t *sb, int out, int in, uint4 *y) {
  const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int kb8 = in / 8, ng = in / 64;
  if (tid >= (size_t)out * kb8) return;
  const int n = (int)(tid / kb8), k0 = (int)(tid % kb8) * 8;
  const int slab = n / kSlabRows, t = (n % kSlabRows) / kTileRows, rr = n % kTileRows, r = rr % 8, irow = rr / 8;
  // eight consecutive k share the word (j) and the nibble row-half; element
  // pair (2c', 2c'+1) sits at bits 4i and 4i+16 of lane column c'
  const int g = k0 / 64, kk = k0 % 64, j = 2 * ((kk >> 5) & 1) + ((kk >> 3) & 1);
  const int i = ((kk >> 4) & 1) + 2 * irow;
  const size_t chunk = ((size_t)slab * ng + g) * kSlabTiles + t;
  const uint2 quad = reinterpret_cast<const uint2 *>(sb)[chunk * 8 + r];
  const uint32_t qd = irow ? quad.y : quad.x;
  const float s = sb_to_f32<SF16>(qd & 0xffffu), b = sb_to_f32<SF16>(qd >> 16);
  uint32_t o[4];
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    const uint32_t word = qw[(chunk * 32 + 4 * r + cc) * 4 + j];
    const float v0 = fmaf((float)((word >> (4 * i)) & 0xFu), s, b);
    const float v1 = fmaf((float)((word >> (4 * i + 16)) & 0xFu), s, b);
    o[cc] = (uint32_t)f32_to_bf16_bits(v0) | ((uint32_t)f32_to_bf16_bits(v1) << 16);
  }
  y[tid] = make_uint4(o[0], o[1], o[2], o[3]);
}

}  // namespace

cudaError_t repack_launch(int layout, const void *src_w, const void *src_sb, int src_out, int in,
                          int row_begin, int rows, void *dst_qw, void *dst_sb, cudaStream_t stream) {
  const int ng = in / kGroup, slabs = row_slabs(rows);
  if (layout == THQ4_SRC_FRAG) {
    // a frag source is copied as is (row_begin must be 0 and rows whole)
    const size_t nq = (size_t)slabs * ng * kSlabTiles * kChunkBytes / 16;
    const size_t ns = (size_t)slabs * ng * kSlabTiles * kQuadBytes / 16;
    copy_kernel<<<1024, 256, 0, stream>>>(static_cast<const uint4 *>(src_w), static_cast<uint4 *>(dst_qw), nq);
    copy_kernel<<<256, 256, 0, stream>>>(static_cast<const uint4 *>(src_sb), static_cast<uint4 *>(dst_sb), ns);
    return cudaGetLastError();
  }
  RepackArgs a{};
  a.layout = layout;
  a.w = static_cast<const uint32_t *>(src_w);
  a.sb = static_cast<const uint16_t *>(src_sb);
  a.src_out = src_out;
  a.in = in;
  a.ng = ng;
  a.row_begin = row_begin;
  a.rows = rows;
  a.slabs = slabs;
  a.dq = static_cast<uint32_t *>(dst_qw);
  a.dsb = static_cast<uint16_t *>(dst_sb);
  const size_t total = (size_t)slabs * ng * kSlabTiles * 32;
  const unsigned blocks = (unsigned)((total + 255) / 256);
  repack_kernel<<<blocks, 256, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t dequant_launch(const thq4_weight &w, void *y, cudaStream_t stream) {
  const size_t total = (size_t)w.out * (w.in / 8);
  const unsigned blocks = (unsigned)((total + 255) / 256);
  if (w.sb_dtype == THQ4_F16)
    dequant_kernel<true><<<blocks, 256, 0, stream>>>(static_cast<const uint32_t *>(w.qw),
                                                     static_cast<const uint16_t *>(w.sb), w.out, w.in,
                                                     static_cast<uint4 *>(y));
  else
    dequant_kernel<false><<<blocks, 256, 0, stream>>>(static_cast<const uint32_t *>(w.qw),
                                                      static_cast<const uint16_t *>(w.sb), w.out, w.in,
                                                      static_cast<uint4 *>(y));
  return cudaGetLastError();
}

}  // namespace thq4
