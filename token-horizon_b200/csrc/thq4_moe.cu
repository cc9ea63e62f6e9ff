// thq4_moe.cu -- the MoE layer: routing, grouping, the grouped expert
// products and the weighted combine.
//
// Replaces Splash's MoE::add (docs/splash/runtime/ops/MoE.cpp:119-231) and
// its kernels (docs/splash/runtime/metal/kernels/shared/moe.metal):
//   select   moe_route_select_q8 (:270-361): per token the top k experts by
//            descending score, lowest id first among equal scores, weights
//            exp(s_r - s_0) / sum_selected exp(s_o - s_0) rounded to bf16;
//   group    moe_group_routes (:368-449): a counting sort of the T*k routes
//            by expert into tiles of kMoeTileRows rows ({expert, live rows}
//            descriptors, MoeTileDescriptor abi/MoE.h:26-29), padding rows
//            ~0u, and the inverse map route -> grouped row.  The reference's
//            atomic cursors leave the order of routes within an expert open;
//            this library fixes it to ascending route index, so the
//            permutation is bit-exact and reproducible;
//   experts  moe_gather_rows + moe_expert_tile / q4_mpp_tile (:453-640): the
//            gathered rows (with their 64-group sums) go through the grouped
//            small-tile kernel of thq4_moe_gemv.cu (gate/up with the SwiGLU
//            epilogue, then down), bf16 at each boundary;
//   combine  moe_combine (:642-664): y = residual + sum over the k slots in
//            slot order of w * d, in f32 (separate multiply and add), one bf16
//            rounding.
//
//   router   moe_route_scores_q8_m8 / _m32 (:34-262): the Q8 router's scores
//            as the sum over eight K slices, in order, of per-group terms
//            fma(dot, scale, sum * bias); the slices run in separate CTAs
//            and the select adds them in slice order;
//   shared   the shared expert (moe_route_select_q8's scalar gate :297-322,
//            its tiles after the routed ones :429-448): a last route per
//            token with weight sigmoid(x . gate row 0).
//
// The router and the shared gate run on CUDA cores in a fixed summation
// order (documented at each kernel) so that the scores -- and so the expert
// selection -- are bit-identical to the CPU oracle's; the tensor pipe's
// accumulation order is not specified.  Select runs one warp per token;
// group runs in one CTA (a two-pass stable counting sort over warp segments
// of the routes); gather and combine move 16-byte pieces.  All of it is
// negligible next to the expert products, which stream every touched
// expert's weights from HBM once per group tile.
#include <algorithm>

#include "thq4_common.cuh"
#include "thq4_internal.h"

namespace thq4 {
namespace {

constexpr uint32_t kPad = 0xFFFFFFFFu;

__device__ __forceinline__ float bf16f(uint16_t v) { return __uint_as_float((uint32_t)v << 16); }

// One warp per token.  Repeated arg-max over the warp: candidates are the
// experts not yet taken whose score is not -inf; ties go to the lower id; a
// token without a candidate takes expert 0 (the oracle's rule).
__global__ void select_kernel(const uint16_t *logits, int T, int E, int k, uint32_t *ids, uint16_t *weights) {
  pdl_wait();
  pdl_launch_dependents();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= T) return;
  const uint16_t *row = logits + (size_t)warp * E;
  float top[32];
  uint32_t taken = 0;  // bit j: this lane's expert lane + 32 j is taken (E <= 1024)
  for (int r = 0; r < k; ++r) {
    float bv = 0.0f;
    int bi = -1;
    for (int j = 0, e = lane; e < E; ++j, e += 32) {
      if ((taken >> j) & 1u) continue;
      const float v = bf16f(row[e]);
      if (v == -INFINITY) continue;
      if (bi < 0 || v > bv) bv = v, bi = e;  // ascending e within the lane
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) bv = ov, bi = oi;
    }
    const int best = bi < 0 ? 0 : bi;
    if (bi >= 0 && (best & 31) == lane) taken |= 1u << (best >> 5);
    if (lane == 0) ids[(size_t)warp * k + r] = (uint32_t)best;
    // without a candidate every remaining score is -inf, expert 0's included
    top[r & 31] = bi < 0 ? -INFINITY : bv;
  }
  if (lane == 0) {
    float den = 0.0f;
    for (int o = 0; o < k; ++o) den = __fadd_rn(den, expf(__fsub_rn(top[o], top[0])));
    for (int r = 0; r < k; ++r)
      weights[(size_t)warp * k + r] = f32_to_bf16_bits(__fdiv_rn(expf(__fsub_rn(top[r], top[0])), den));
  }
}

// ---- the Q8 router -------------------------------------------------------------
constexpr int kRouteRows = 32, kRouteCols = 64, kRouteThreads = 128;

__device__ __forceinline__ float u8f(uint32_t word, int i) {
  return __uint_as_float(0x4B000000u | ((word >> (8 * i)) & 0xFFu)) - 8388608.0f;  // exact
}

// One CTA: 32 tokens x 64 router columns x one K slice (blockIdx.z).  Per
// group of the slice the CTA stages x as f32 [k][token] and q as f32
// [k][column] in shared memory (the next group's bytes are loaded into
// registers while this one computes), each warp forms the group sums of 8
// tokens (pairs x[l] + x[l+32] combined by xor butterfly), and each thread
// accumulates a 4 x 4 block: dot = sum over k in order of x * q (each
// product exact in f32), then slice += fma(dot, scale, sum * bias).
// partial[(s*T + t)*ncols + n] = slice s's sum.
__global__ void __launch_bounds__(kRouteThreads) route_scores_kernel(const uint16_t *__restrict__ x, int T, int H,
                                                                     const uint8_t *__restrict__ q,
                                                                     const uint16_t *__restrict__ scales,
                                                                     const uint16_t *__restrict__ biases, int ncols,
                                                                     float *__restrict__ partial) {
  __shared__ __align__(16) float xs[64][kRouteRows];
  __shared__ __align__(16) float qs[64][kRouteCols];
  __shared__ float sums[kRouteRows], ss[kRouteCols], bs[kRouteCols];
  pdl_wait();
  pdl_launch_dependents();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row0 = blockIdx.x * kRouteRows, col0 = blockIdx.y * kRouteCols, sl = blockIdx.z;
  const int G = H / 64, g0 = sl * G / kRouteSlices, g1 = (sl + 1) * G / kRouteSlices;
  const int tr = tid >> 4, tc = tid & 15;  // tokens 4tr.., columns 4tc..
  float acc[4][4];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[r][c] = 0.0f;
  // staging: x piece p (tid, tid + 128): token p & 31, k (p >> 5) * 8 .. +8;
  // q piece p: column p & 63, k (p >> 6) * 16 .. +16; the group-sum pairs
  // of warp w's tokens 8w .. 8w+7 at k = lane and lane + 32.
  uint4 xr[2], qr[2];
  uint32_t pair[8];
  uint16_t prm = 0;
  auto load = [&](int g) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int p = tid + 128 * i;
      const int t = row0 + (p & 31);
      xr[i] = t < T ? *reinterpret_cast<const uint4 *>(x + (size_t)t * H + 64 * g + (p >> 5) * 8)
                    : make_uint4(0, 0, 0, 0);
      const int n = col0 + (p & 63);
      qr[i] = n < ncols ? *reinterpret_cast<const uint4 *>(q + ((size_t)g * 256 + n) * 64 + (p >> 6) * 16)
                        : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int rr = 0; rr < 8; ++rr) {
      const int t = row0 + 8 * warp + rr;
      const uint16_t *xp = x + (size_t)t * H + 64 * g + lane;
      pair[rr] = t < T ? (uint32_t)xp[0] | ((uint32_t)xp[32] << 16) : 0u;
    }
    const int n = col0 + (tid & 63);
    prm = n < ncols ? (tid < 64 ? scales : biases)[(size_t)g * 256 + n] : (uint16_t)0;
  };
  if (g0 < g1) load(g0);
  for (int g = g0; g < g1; ++g) {
    __syncthreads();  // the previous group's reads of the staging buffers are done
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int p = tid + 128 * i;
      const uint32_t w[4] = {xr[i].x, xr[i].y, xr[i].z, xr[i].w};
#pragma unroll
      for (int e = 0; e < 8; ++e) xs[(p >> 5) * 8 + e][p & 31] = bf16f((uint16_t)(w[e >> 1] >> (16 * (e & 1))));
      const uint32_t b[4] = {qr[i].x, qr[i].y, qr[i].z, qr[i].w};
#pragma unroll
      for (int e = 0; e < 16; ++e) qs[(p >> 6) * 16 + e][p & 63] = u8f(b[e >> 2], e & 3);
    }
    (tid < 64 ? ss : bs)[tid & 63] = bf16f(prm);
#pragma unroll
    for (int rr = 0; rr < 8; ++rr) {
      float v = bf16f((uint16_t)(pair[rr] & 0xFFFFu)) + bf16f((uint16_t)(pair[rr] >> 16));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
      if (lane == 0) sums[8 * warp + rr] = v;
    }
    __syncthreads();
    if (g + 1 < g1) load(g + 1);
    float dot[4][4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) dot[r][c] = 0.0f;
#pragma unroll 8
    for (int j = 0; j < 64; ++j) {
      const float4 xv = *reinterpret_cast<const float4 *>(&xs[j][4 * tr]);
      const float4 qv = *reinterpret_cast<const float4 *>(&qs[j][4 * tc]);
      const float xa[4] = {xv.x, xv.y, xv.z, xv.w}, qa[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) dot[r][c] = __fmaf_rn(xa[r], qa[c], dot[r][c]);
    }
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c)
        acc[r][c] = __fadd_rn(acc[r][c], __fmaf_rn(dot[r][c], ss[4 * tc + c], __fmul_rn(sums[4 * tr + r], bs[4 * tc + c])));
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int t = row0 + 4 * tr + r;
    if (t >= T) continue;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int n = col0 + 4 * tc + c;
      if (n < ncols) partial[((size_t)sl * T + t) * ncols + n] = acc[r][c];
    }
  }
}

// scores[t*ld + n] = bf16 of the slice sums added in slice order.
__global__ void scores_kernel(const float *partial, int T, int ncols, uint16_t *scores, int ld) {
  pdl_wait();
  pdl_launch_dependents();
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)T * ncols) return;
  float total = 0.0f;
#pragma unroll
  for (int s = 0; s < kRouteSlices; ++s) total = __fadd_rn(total, partial[(size_t)s * T * ncols + i]);
  scores[(i / ncols) * ld + i % ncols] = f32_to_bf16_bits(total);
}

// moe_route_select_q8 from the router partials, one warp per token (E <= 256):
// scores = bf16 of the slice sums, top k as select_kernel; with a shared
// gate, route k of the token is expert E with weight bf16(1 / (1 + exp(-g))):
// virtual thread v = 32w + lane of 256 accumulates g over k = v, v + 256, ...
// by fma of x and fma(q, scale, bias) (row 0, group k/64), each virtual warp
// combines by xor butterfly, the eight warp sums add in order.
__global__ void select_q8_kernel(const float *partial, int T, int E, int k, int rpr, const uint16_t *x, int H,
                                 const uint8_t *sq, const uint16_t *ssc, const uint16_t *sbi, uint32_t *ids,
                                 uint16_t *weights) {
  pdl_wait();
  pdl_launch_dependents();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= T) return;
  float sc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int e = lane + 32 * j;
    sc[j] = -INFINITY;
    if (e < E) {
      float total = 0.0f;
#pragma unroll
      for (int s = 0; s < kRouteSlices; ++s) total = __fadd_rn(total, partial[((size_t)s * T + warp) * E + e]);
      sc[j] = bf16f(f32_to_bf16_bits(total));
    }
  }
  float top[32];
  uint32_t taken = 0;
  for (int r = 0; r < k; ++r) {
    float bv = 0.0f;
    int bi = -1;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = lane + 32 * j;
      if (e >= E || ((taken >> j) & 1u)) continue;
      const float v = sc[j];
      if (v == -INFINITY) continue;
      if (bi < 0 || v > bv) bv = v, bi = e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) bv = ov, bi = oi;
    }
    const int best = bi < 0 ? 0 : bi;
    if (bi >= 0 && (best & 31) == lane) taken |= 1u << (best >> 5);
    if (lane == 0) ids[(size_t)warp * rpr + r] = (uint32_t)best;
    top[r & 31] = bi < 0 ? -INFINITY : bv;
  }
  if (lane == 0) {
    float den = 0.0f;
    for (int o = 0; o < k; ++o) den = __fadd_rn(den, expf(__fsub_rn(top[o], top[0])));
    for (int r = 0; r < k; ++r)
      weights[(size_t)warp * rpr + r] = f32_to_bf16_bits(__fdiv_rn(expf(__fsub_rn(top[r], top[0])), den));
  }
  if (rpr == k) return;
  const uint16_t *row = x + (size_t)warp * H;
  float g = 0.0f;
  for (int w = 0; w < 8; ++w) {
    float a = 0.0f;
    for (int d = 32 * w + lane; d < H; d += 256) {
      const size_t p = (size_t)(d >> 6) * 256;
      const float deq = __fmaf_rn((float)sq[p * 64 + (d & 63)], bf16f(ssc[p]), bf16f(sbi[p]));
      a = __fmaf_rn(bf16f(row[d]), deq, a);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, o));
    g = __fadd_rn(g, a);
  }
  if (lane == 0) {
    ids[(size_t)warp * rpr + k] = (uint32_t)E;
    weights[(size_t)warp * rpr + k] = f32_to_bf16_bits(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g))));
  }
}

// Warps of the grouping kernel: each owns a contiguous segment of the routes
// and one row of per-expert counters in shared memory.
__host__ __device__ inline int group_warps(int E) { return E <= 512 ? 32 : 16; }

// One CTA.  A stable counting sort of the routes by expert:
//   1. every warp counts its segment's routes per expert (32 routes at a
//      time; lanes holding the same expert find each other with match.any);
//   2. per expert, the warps' counts become exclusive prefixes in warp order
//      and the expert's total; the experts' tile counts are scanned into
//      their first tile;
//   3. every warp walks its segment again and places each route after the
//      earlier ones of its expert (its rank among the 32 plus the running
//      count), so routes stay in ascending order within an expert.
// Routes whose expert id is out of range are dropped (combine skips them).
// Experts [e0, e0 + E) of E_all are grouped (local ids e - e0); routes to
// other valid experts are dropped silently (another rank computes them).
// Each token has rpr routes; slots k.. (the shared expert's) are not sorted:
// with shared_local, ceil(T/32) tiles of local id E after the routed ones
// hold every token's shared route in token order (moe.metal:429-448),
// otherwise those routes are dropped.
__global__ void group_kernel(const uint32_t *ids, int T, int k, int rpr, int E_all, int e0, int E, int shared_local,
                             int max_tiles, uint32_t *tiles, uint32_t *grouped, uint32_t *route_rows, uint32_t *ntiles,
                             uint32_t *status) {
  pdl_wait();
  pdl_launch_dependents();
  const int R = T * rpr;
  extern __shared__ uint32_t sm[];
  const int W = blockDim.x >> 5;
  uint32_t *cw = sm;            // [W][E]: counts, then each warp's running base
  uint32_t *off = sm + W * E;   // [E + 1]: first tile of each expert, tiles in use
  uint32_t *tot = off + E + 1;  // [E + 1]: routes of each expert, then all tiles
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t lt = (1u << lane) - 1u;
  for (int i = threadIdx.x; i < W * E; i += blockDim.x) cw[i] = 0;
  __syncthreads();
  const int seg = (R + W - 1) / W;
  const int r0 = min(R, warp * seg), r1 = min(R, r0 + seg);
  auto routed = [&](int r) { return rpr == k || r % rpr < k; };
  auto expert_of = [&](int r) -> uint32_t {
    if (r >= r1 || !routed(r)) return kPad;
    const uint32_t e = ids[r] - (uint32_t)e0;  // wraps for e < e0
    return e < (uint32_t)E ? e : kPad;
  };
  for (int b = r0; b < r1; b += 32) {
    const int r = b + lane;
    const uint32_t e = expert_of(r);
    if (r < r1 && e == kPad) {
      if (routed(r) && ids[r] >= (uint32_t)E_all) raise_status(status, kStatusBadExpert);
      route_rows[r] = kPad;
    }
    const uint32_t peers = __match_any_sync(0xffffffffu, e);
    if (e != kPad && (peers & lt) == 0) cw[warp * E + e] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    uint32_t acc = 0;
    for (int w = 0; w < W; ++w) {
      const uint32_t c = cw[w * E + e];
      cw[w * E + e] = acc;
      acc += c;
    }
    tot[e] = acc;
  }
  __syncthreads();
  if (warp == 0) {
    uint32_t carry = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      const uint32_t nt = e < E ? (tot[e] + kMoeTileRows - 1) / kMoeTileRows : 0u;
      uint32_t v = nt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
      }
      if (e < E) off[e] = carry + v - nt;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
    if (lane == 0) {
      const uint32_t total = carry + (shared_local ? (uint32_t)(T + kMoeTileRows - 1) / kMoeTileRows : 0u);
      off[E] = carry;
      tot[E] = total;
      *ntiles = total <= (uint32_t)max_tiles ? total : 0u;
      if (total > (uint32_t)max_tiles) raise_status(status, kStatusBounds);
    }
  }
  __syncthreads();
  if (tot[E] > (uint32_t)max_tiles) return;
  if (shared_local) {
    const uint32_t base = off[E], nst = tot[E] - base;
    for (uint32_t i = threadIdx.x; i < nst; i += blockDim.x) {
      tiles[2 * (base + i)] = (uint32_t)E;
      tiles[2 * (base + i) + 1] = min((uint32_t)kMoeTileRows, (uint32_t)T - i * kMoeTileRows);
    }
    for (uint32_t t = threadIdx.x; t < nst * kMoeTileRows; t += blockDim.x) {
      const uint32_t row = base * kMoeTileRows + t;
      if (t < (uint32_t)T) {
        grouped[row] = t * (uint32_t)rpr + (uint32_t)k;
        route_rows[t * rpr + k] = row;
      } else {
        grouped[row] = kPad;
      }
    }
  }
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const uint32_t t0 = off[e], c = tot[e], nt = (c + kMoeTileRows - 1) / kMoeTileRows;
    for (uint32_t t = 0; t < nt; ++t) {
      tiles[2 * (t0 + t)] = (uint32_t)e;
      tiles[2 * (t0 + t) + 1] = min((uint32_t)kMoeTileRows, c - t * kMoeTileRows);
    }
    for (uint32_t row = t0 * kMoeTileRows + c; row < (t0 + nt) * kMoeTileRows; ++row) grouped[row] = kPad;
  }
  for (int b = r0; b < r1; b += 32) {
    const int r = b + lane;
    const uint32_t e = expert_of(r);
    const uint32_t peers = __match_any_sync(0xffffffffu, e);
    uint32_t base = 0;
    if (e != kPad) {
      base = cw[warp * E + e];
      const uint32_t row = off[e] * kMoeTileRows + base + __popc(peers & lt);
      grouped[row] = (uint32_t)r;
      route_rows[r] = row;
    }
    __syncwarp();
    if (e != kPad && (peers & lt) == 0) cw[warp * E + e] = base + __popc(peers);
    __syncwarp();
  }
}

// xg[row] = x[route / rpr] for the live rows of the live tiles, zero for
// padding, and xsum[tile][g][row % 32] = the sum of the row's 64-group g in
// f32.  One thread per 16-byte piece (8 values, summed in order); the 8
// pieces of a group are 8 aligned lanes, which add their sums with a fixed
// shuffle tree (deterministic).
__global__ void gather_kernel(const uint16_t *x, int H, int rpr, const uint32_t *grouped, const uint32_t *ntiles,
                              uint16_t *xg, float *xsum) {
  pdl_wait();
  pdl_launch_dependents();
  const int pieces = H / 8;
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t row = i / pieces;
  if (row >= (size_t)(*ntiles) * kMoeTileRows) return;  // whole 8-lane groups leave together
  const int p = (int)(i % pieces);
  const uint32_t route = grouped[row];
  uint4 v = make_uint4(0, 0, 0, 0);
  if (route != kPad) v = reinterpret_cast<const uint4 *>(x + (size_t)(route / rpr) * H)[p];
  reinterpret_cast<uint4 *>(xg + row * H)[p] = v;
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  float sum = 0.0f;
#pragma unroll
  for (int e = 0; e < 4; ++e) sum = (sum + bf16f((uint16_t)(w[e] & 0xffffu))) + bf16f((uint16_t)(w[e] >> 16));
  const unsigned lane = threadIdx.x & 31, gmask = 0xFFu << (lane & ~7u);
  sum += __shfl_xor_sync(gmask, sum, 1);
  sum += __shfl_xor_sync(gmask, sum, 2);
  sum += __shfl_xor_sync(gmask, sum, 4);
  if ((p & 7) == 0) xsum[((row / kMoeTileRows) * (H / 64) + p / 8) * kMoeTileRows + row % kMoeTileRows] = sum;
}

// y[t] = residual[t] + sum_s w[t][s] * d[route_rows[t*rpr + s]] over the
// rpr slots in order (the shared expert's last), f32.
// F32: y is f32 (an expert shard's partial, summed over the ranks later).
template <bool F32>
__global__ void combine_kernel(const uint16_t *d, const uint16_t *weights, const uint32_t *route_rows,
                               const uint16_t *residual, int T, int H, int rpr, void *y) {
  pdl_wait();
  pdl_launch_dependents();
  const int pieces = H / 8;
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)T * pieces) return;
  const int t = (int)(i / pieces), p = (int)(i % pieces);
  float v[8];
  if (residual) {
    const uint4 r = reinterpret_cast<const uint4 *>(residual + (size_t)t * H)[p];
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = bf16f((uint16_t)(w[e >> 1] >> (16 * (e & 1))));
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = 0.0f;
  }
  // four slots at a time: their row indices, then their rows, are requested
  // together; the sums still run in slot order
  constexpr int kB = 4;
  for (int s0 = 0; s0 < rpr; s0 += kB) {
    uint32_t row[kB];
    float ws[kB];
    uint4 dv[kB];
#pragma unroll
    for (int j = 0; j < kB; ++j) {
      const int s = s0 + j;
      row[j] = s < rpr ? route_rows[(size_t)t * rpr + s] : kPad;
      ws[j] = s < rpr ? bf16f(weights[(size_t)t * rpr + s]) : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < kB; ++j)
      dv[j] = row[j] != kPad ? reinterpret_cast<const uint4 *>(d + (size_t)row[j] * H)[p] : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int j = 0; j < kB; ++j) {
      if (row[j] == kPad) continue;
      const uint32_t w[4] = {dv[j].x, dv[j].y, dv[j].z, dv[j].w};
#pragma unroll
      for (int e = 0; e < 8; ++e)
        v[e] = __fadd_rn(v[e], __fmul_rn(ws[j], bf16f((uint16_t)(w[e >> 1] >> (16 * (e & 1))))));
    }
  }
  if constexpr (F32) {
    float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(y) + (size_t)t * H) + 2 * p;
    dst[0] = make_float4(v[0], v[1], v[2], v[3]);
    dst[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e)
      o[e] = (uint32_t)f32_to_bf16_bits(v[2 * e]) | ((uint32_t)f32_to_bf16_bits(v[2 * e + 1]) << 16);
    reinterpret_cast<uint4 *>(static_cast<uint16_t *>(y) + (size_t)t * H)[p] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

size_t align256(size_t b) { return (b + 255) / 256 * 256; }

// Every kernel of the MoE chain starts with griddepcontrol.wait (before it
// touches global memory) and launches with programmatic stream
// serialization, so its launch and set-up overlap its predecessor's tail.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = gemv_pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...);
}

}  // namespace

uint32_t moe_max_tiles(int T, int E, int k, bool shared) {
  const uint64_t routed = (uint64_t)T * (uint64_t)k;
  const uint64_t bound = routed / kMoeTileRows + (uint64_t)E;
  return (uint32_t)std::min(bound, routed) + (shared ? (uint32_t)((T + kMoeTileRows - 1) / kMoeTileRows) : 0u);
}

size_t moe_group_smem(int R, int E) {
  (void)R;  // the routes are read from global memory twice, never staged
  return ((size_t)group_warps(E) * E + 2 * (size_t)E + 2) * 4;
}

size_t moe_scores_bytes(int T, int ncols) { return (size_t)kRouteSlices * T * ncols * sizeof(float); }

cudaError_t moe_scores_launch(const void *x, int T, int H, const thq4_q8_weight &router, int ncols, float *partial,
                              uint16_t *scores, int ld, cudaStream_t stream) {
  const dim3 grid((T + kRouteRows - 1) / kRouteRows, (ncols + kRouteCols - 1) / kRouteCols, kRouteSlices);
  cudaError_t e = launch_pdl(route_scores_kernel, grid, dim3(kRouteThreads), 0, stream, static_cast<const uint16_t *>(x),
                             T, H, static_cast<const uint8_t *>(router.q), static_cast<const uint16_t *>(router.scales),
                             static_cast<const uint16_t *>(router.biases), ncols, partial);
  if (e != cudaSuccess || !scores) return e;
  const size_t n = (size_t)T * ncols;
  return launch_pdl(scores_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, stream, partial, T, ncols, scores,
                    ld);
}

cudaError_t moe_route_launch(const MoeRouting &rt, int T, int E, int k, uint32_t *ids, uint16_t *weights,
                             uint32_t *tiles, uint32_t *grouped, uint32_t *route_rows, uint32_t *ntiles, int max_tiles,
                             cudaStream_t stream, int e0, int e1) {
  if (e1 < 0) e1 = E;
  const int threads = 256, warps = threads / 32;
  const int rpr = k + (rt.shared_gate ? 1 : 0);
  cudaError_t e;
  const dim3 sgrid((T + warps - 1) / warps);
  if (rt.logits) {
    e = launch_pdl(select_kernel, sgrid, dim3(threads), 0, stream, rt.logits, T, E, k, ids, weights);
  } else {
    if ((e = moe_scores_launch(rt.x, T, rt.H, *rt.router, E, rt.partial, nullptr, 0, stream)) != cudaSuccess) return e;
    const thq4_q8_weight *sg = rt.shared_gate;
    e = launch_pdl(select_q8_kernel, sgrid, dim3(threads), 0, stream, static_cast<const float *>(rt.partial), T, E, k,
                   rpr, static_cast<const uint16_t *>(rt.x), rt.H,
                   sg ? static_cast<const uint8_t *>(sg->q) : nullptr,
                   sg ? static_cast<const uint16_t *>(sg->scales) : nullptr,
                   sg ? static_cast<const uint16_t *>(sg->biases) : nullptr, ids, weights);
  }
  if (e != cudaSuccess) return e;
  const int E_loc = e1 - e0;
  const size_t smem = moe_group_smem(T * rpr, E_loc);
  static DeviceOnce once;
  e = once.run([] { return cudaFuncSetAttribute(group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024); });
  if (e != cudaSuccess) return e;
  return launch_pdl(group_kernel, dim3(1), dim3(group_warps(E_loc) * 32), smem, stream,
                    static_cast<const uint32_t *>(ids), T, k, rpr, E, e0, E_loc,
                    rt.shared_gate && rt.shared_local ? 1 : 0, max_tiles, tiles, grouped, route_rows, ntiles,
                    status_word());
}

MoeWorkspace moe_workspace(int T, int H, int I, int E, int k, void *base, int rpr, bool shared_local,
                           int router_cols) {
  if (rpr < 0) rpr = k;
  MoeWorkspace w{};
  const size_t R = (size_t)T * rpr, mt = moe_max_tiles(T, E, k, shared_local), rows = mt * kMoeTileRows;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o += align256(bytes);
    return base ? static_cast<char *>(base) + at : nullptr;
  };
  w.ids = reinterpret_cast<uint32_t *>(take(R * 4));
  w.weights = reinterpret_cast<uint16_t *>(take(R * 2));
  w.tiles = reinterpret_cast<uint32_t *>(take(mt * 8));
  w.grouped = reinterpret_cast<uint32_t *>(take(rows * 4));
  w.route_rows = reinterpret_cast<uint32_t *>(take(R * 4));
  w.ntiles = reinterpret_cast<uint32_t *>(take(4));
  w.xg = reinterpret_cast<uint16_t *>(take(rows * H * 2));
  w.h = reinterpret_cast<uint16_t *>(take(rows * I * 2));
  w.d = reinterpret_cast<uint16_t *>(take(rows * H * 2));
  w.xsum = reinterpret_cast<float *>(take(rows * (H / 64) * 4));
  w.hsum = reinterpret_cast<float *>(take(rows * (I / 64) * 4));
  w.partial = router_cols > 0 ? reinterpret_cast<float *>(take(moe_scores_bytes(T, router_cols))) : nullptr;
  w.bytes = o;
  w.max_tiles = (int)mt;
  return w;
}

cudaError_t moe_launch(const void *x, const void *residual, const MoeRouting &rt, int T, int H, int I, int E, int k,
                       const MoeSets &sets, void *y, const MoeWorkspace &w, cudaStream_t stream, int e0, int e1,
                       bool y_f32) {
  if (e1 < 0) e1 = E;
  const int rpr = k + (rt.shared_gate ? 1 : 0);
  cudaError_t e = moe_route_launch(rt, T, E, k, w.ids, w.weights, w.tiles, w.grouped, w.route_rows, w.ntiles,
                                   w.max_tiles, stream, e0, e1);
  if (e != cudaSuccess) return e;
  const size_t rows = (size_t)w.max_tiles * kMoeTileRows;
  {
    const size_t n = rows * (H / 8);
    e = launch_pdl(gather_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, stream,
                   static_cast<const uint16_t *>(x), H, rpr, static_cast<const uint32_t *>(w.grouped),
                   static_cast<const uint32_t *>(w.ntiles), w.xg, w.xsum);
    if (e != cudaSuccess) return e;
  }
  const bool sh = rt.shared_gate && rt.shared_local;
  MoeExperts g{};
  g.x = w.xg;
  g.y = w.h;
  g.w0 = sets.gate;
  g.w1 = sets.up;
  g.sw0 = sh ? sets.sgate : nullptr;
  g.sw1 = sh ? sets.sup : nullptr;
  g.n_experts = e1 - e0;
  g.tiles = w.tiles;
  g.count = w.ntiles;
  g.xsum = w.xsum;
  g.ysum = w.hsum;
  g.max_tiles = w.max_tiles;
  if ((e = moe_expert_launch(g, stream)) != cudaSuccess) return e;
  g.x = w.h;
  g.y = w.d;
  g.w0 = sets.down;
  g.w1 = nullptr;
  g.sw0 = sh ? sets.sdown : nullptr;
  g.sw1 = nullptr;
  g.xsum = w.hsum;
  g.ysum = nullptr;
  if ((e = moe_expert_launch(g, stream)) != cudaSuccess) return e;
  const size_t n = (size_t)T * (H / 8);
  const unsigned blocks = (unsigned)((n + 255) / 256);
  const uint16_t *res = static_cast<const uint16_t *>(residual);
  const uint16_t *dd = w.d, *wts = w.weights;
  const uint32_t *rr = w.route_rows;
  return launch_pdl(y_f32 ? combine_kernel<true> : combine_kernel<false>, dim3(blocks), dim3(256), 0, stream, dd, wts,
                    rr, res, T, H, rpr, y);
}

}  // namespace thq4
