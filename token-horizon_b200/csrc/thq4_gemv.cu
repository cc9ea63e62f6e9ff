// thq4_gemv.cu -- decode (m = 1) and spec-verify (m <= 8) Q4 projections.
//
// Replaces the reference's m = 1 matvec AffineQmvT / qmvt<RPL,NSG,GateUp>
// (engine/src/quant_kernel.rs:2768-3136) and its m <= 8 decode/verify families
// AffineQmpp (th_mpp_tile, :1793-2569), AffineQsg (:1149-1632) and AffineQmm
// (:1634-1740), with one kernel.
//
// The path is bound by HBM bandwidth (0.5625 bytes per weight, each read once).
// Measured on B200: a warp-per-run stream of 16-byte loads tops out near
// 4 TB/s whatever its depth (each warp tracks only a few loads), while
// one-dimensional bulk copies of 16 KB stream at ~5.8 TB/s from 148 CTAs.
// Hence:
//   - the weight is a stream of "slab-groups" (SG): 128 rows x 64 k, 4096
//     bytes of nibbles + 512 bytes of scale/bias, slab-major, so any run of
//     SGs is one contiguous byte range of the frag layout.  A persistent grid
//     (one or two CTAs per SM) gives every CTA an equal contiguous run of
//     SGs; a run may start and end inside a slab;
//   - one producer warp per CTA streams the run into a ring of shared-memory
//     stages with bulk copies (cp.async.bulk, evict-first in L2, no
//     multicast) of ~16 KB, completing on a "full" mbarrier per stage; the
//     first stages are requested before the kernel waits for its input;
//   - eight consumer warps each own one 16-row tile of every SG, so their
//     output rows are disjoint and no reduction crosses warps.  Per SG a warp
//     runs four mma.m16n8k16 with the weight as the A operand (16 rows) and
//     the m tokens as N (8 columns), bf16 with f32 accumulation.  A nibble
//     pair becomes the bf16 pair (128 + q) by one shift and one LOP3 --
//     exact -- and the 128 offset is removed per group in the epilogue
//     together with the bias, the per-group form of the reference kernels
//     (quant_kernel.rs:1994-2001, 2887-2890):
//         y += s * sum((128+q) x) + (b - 128 s) * sum(x)
//            = s * sum(q x) + b * sum(x),
//     then releases the stage on an "empty" mbarrier.  Every mbarrier wait is
//     bounded in time and reports kStatusTimeout instead of hanging;
//   - an f32 activation is split into bf16 hi + lo parts that occupy two of
//     the eight N columns, so an f32 GEMV keeps ~16 significant bits of x at
//     no extra weight traffic;
//   - the activation is staged once per CTA in shared memory in B-fragment
//     order, with its per-group sums;
//   - a slab split between CTAs (only a CTA's first and last slab can be) is
//     finished per tile by the warp that arrives last ("last arriver
//     reduces", the reference's split-K scheme, quant_kernel.rs:1299-1332):
//     each writes its partial to the caller's workspace and bumps the
//     (slab, tile) counter; the last one adds the partials in CTA order, so
//     results are bitwise deterministic (qwen35.rs:6986-6988) with no
//     waiting, and resets the counter;
//   - CTAs stay within half an SM when the activation allows, and the kernel
//     uses programmatic dependent launch: the next projection's CTA can become
//     resident and request its weights while this one finishes; griddepcontrol
//     .wait guards only the activation reads and the output writes.
#include "thq4_common.cuh"
#include "thq4_internal.h"

namespace thq4 {

namespace {

constexpr int kConsumers = kSlabTiles;  // one consumer warp per tile of a slab
constexpr int kThreads = (kConsumers + 1) * 32;
constexpr int kSgBytes = kSlabTiles * (kChunkBytes + kQuadBytes);  // 4608
constexpr int kMaxStages = 8;

struct GemvArgs {
  const uint8_t *qw0;  // gate (or the only) weight: frag nibbles
  const uint8_t *sb0;
  const uint8_t *qw1;  // up weight (gate/up only)
  const uint8_t *sb1;
  const void *x;       // [m][in]
  void *y;             // [m][out]
  uint32_t *status;    // device status word
  float *part;         // workspace: partials [cta][2 sides][8 tiles][NS][32 lanes][4]
  uint32_t *count;     // workspace: arrivals per (slab, tile) (zero between calls)
  long long sgs;       // slab-groups in the weight (slabs * ng)
  int m;               // tokens in this launch
  int in, ng, out;
  int mcols;           // B columns in use: m (bf16 x) or 2m (f32 x)
  int stages;          // ring stages
  int cb;              // slab-groups per stage
};

__host__ __device__ inline size_t xs_bytes(int ng, int mcols) { return (size_t)ng * 2 * mcols * 64; }
__host__ __device__ inline size_t xsum_bytes(int ng) { return (size_t)ng * 8 * sizeof(float); }
__host__ __device__ inline size_t stage_bytes(int cb, bool gate_up) { return (size_t)(gate_up ? 2 : 1) * cb * kSgBytes; }
__host__ __device__ inline size_t gemv_smem(int stages, int cb, bool gate_up, int ng, int mcols) {
  return 128 + (size_t)stages * stage_bytes(cb, gate_up) + xs_bytes(ng, mcols) + xsum_bytes(ng);
}
// floats of one CTA side's partial: 8 tiles x NS x 32 lanes x 4
__host__ __device__ inline int side_floats(bool gate_up) { return kSlabTiles * (gate_up ? 2 : 1) * 32 * 4; }
__device__ __forceinline__ long long run_begin(long long i, long long total, long long parts) {
  return i * total / parts;
}
// The run holding offset o (0 <= o < total): the largest i with
// run_begin(i) <= o, which is never an empty run.
__device__ __forceinline__ long long run_of(long long o, long long total, long long parts) {
  return ((o + 1) * parts + total - 1) / total - 1;
}
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;\n" ::"r"(kConsumers * 32) : "memory");
}

// ---- packed f32x2 arithmetic (sm_100) ---------------------------------------
__device__ __forceinline__ uint64_t pk(float lo, float hi) {
  uint64_t v;
  asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "f"(lo), "f"(hi));
  return v;
}
__device__ __forceinline__ void upk(uint64_t v, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// Stage x into shared memory in B-fragment order (consumer warps only):
// entry ((g*2 + h)*mcols + col)*4 + c (16 bytes) holds, for k-steps
// j = 2h, 2h+1 of group g, the bf16 pairs {x[2c], x[2c+1]} and
// {x[2c+8], x[2c+9]} (k relative to 64 g + 16 j) of B column col: token col
// (bf16 x), or token col/2's hi (even col) or lo (odd col) part (f32 x).  One
// thread builds one entry with one 16-byte store; the 8 threads holding
// (g, col)'s 8 entries reduce the group sum xsum[g*8 + col] with a fixed
// shuffle tree.  Columns >= mcols have sum 0.
template <bool XF32>
__device__ void stage_x(const GemvArgs &a, uint4 *xs4, float *xsum) {
  const int tid = threadIdx.x, nthr = kConsumers * 32;
  for (int i = tid; i < a.ng * 8; i += nthr)
    if ((i & 7) >= a.mcols) xsum[i] = 0.0f;  // disjoint from the sums below
  const int entries = a.ng * a.mcols * 8;   // (g, col, h, c)
  const int span = (entries + 31) / 32 * 32;
  for (int idx = tid; idx < span; idx += nthr) {
    const bool live = idx < entries;
    const int e = live ? idx : 0;
    const int c = e & 3, h = (e >> 2) & 1, gc = e >> 3;
    const int col = gc % a.mcols, g = gc / a.mcols;
    const int t = XF32 ? col >> 1 : col, part = XF32 ? col & 1 : 0;
    float v[8];
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
      const int k = g * 64 + 16 * (2 * h + jj) + 2 * c;
#pragma unroll
      for (int hi8 = 0; hi8 < 2; ++hi8) {
        float p0 = 0.0f, p1 = 0.0f;
        if (live) {
          if constexpr (XF32) {
            const float2 f = *reinterpret_cast<const float2 *>(static_cast<const float *>(a.x) + (size_t)t * a.in +
                                                              k + 8 * hi8);
            const float h0 = round_bf16(f.x), h1 = round_bf16(f.y);
            p0 = part ? round_bf16(f.x - h0) : h0;
            p1 = part ? round_bf16(f.y - h1) : h1;
          } else {
            const uint32_t w = *reinterpret_cast<const uint32_t *>(static_cast<const uint16_t *>(a.x) +
                                                                   (size_t)t * a.in + k + 8 * hi8);
            p0 = __uint_as_float(w << 16);
            p1 = __uint_as_float(w & 0xffff0000u);
          }
        }
        v[jj * 4 + hi8 * 2] = p0;
        v[jj * 4 + hi8 * 2 + 1] = p1;
      }
    }
    if (live) {
      uint4 o;
      o.x = (uint32_t)f32_to_bf16_bits(v[0]) | ((uint32_t)f32_to_bf16_bits(v[1]) << 16);
      o.y = (uint32_t)f32_to_bf16_bits(v[2]) | ((uint32_t)f32_to_bf16_bits(v[3]) << 16);
      o.z = (uint32_t)f32_to_bf16_bits(v[4]) | ((uint32_t)f32_to_bf16_bits(v[5]) << 16);
      o.w = (uint32_t)f32_to_bf16_bits(v[6]) | ((uint32_t)f32_to_bf16_bits(v[7]) << 16);
      xs4[((size_t)(g * 2 + h) * a.mcols + col) * 4 + c] = o;
    }
    float s = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    s += __shfl_xor_sync(0xffffffffu, s, 4);
    if (live && (idx & 7) == 0) xsum[g * 8 + col] = s;
  }
  consumer_sync();
}

// One tile-group's contribution: four mma.m16n8k16 (two independent chains,
// started from a zero C) on the dequantised nibbles, then the per-group
// scale / bias epilogue.  y[0..3] = rows (r, r, r+8, r+8) x columns (2c,
// 2c+1, 2c, 2c+1); with ONE_COL only column 0 (m = 1, bf16 x) is kept.
template <bool SF16, bool ONE_COL>
__device__ __forceinline__ void gt_step(float (&y)[4], const uint4 w, const uint2 q, const uint4 xa, const uint4 xb,
                                        const float2 xsm) {
  float a0[4], a1[4];
  mma_bf16_16816_z(a0, nib_bf16x2_mh(w.x, 0), nib_bf16x2_mh(w.x, 4), nib_bf16x2_mh(w.x, 8),
                   nib_bf16x2_mh(w.x, 12), xa.x, xa.y);
  mma_bf16_16816_z(a1, nib_bf16x2_mh(w.z, 0), nib_bf16x2_mh(w.z, 4), nib_bf16x2_mh(w.z, 8),
                   nib_bf16x2_mh(w.z, 12), xb.x, xb.y);
  mma_bf16_16816(a0, nib_bf16x2_mh(w.y, 0), nib_bf16x2_mh(w.y, 4), nib_bf16x2_mh(w.y, 8), nib_bf16x2_mh(w.y, 12),
                 xa.z, xa.w);
  mma_bf16_16816(a1, nib_bf16x2_mh(w.w, 0), nib_bf16x2_mh(w.w, 4), nib_bf16x2_mh(w.w, 8), nib_bf16x2_mh(w.w, 12),
                 xb.z, xb.w);
  const float sr = sb_to_f32<SF16>(q.x & 0xffffu), br = sb_to_f32<SF16>(q.x >> 16);
  const float sr8 = sb_to_f32<SF16>(q.y & 0xffffu), br8 = sb_to_f32<SF16>(q.y >> 16);
  const float bpr = fmaf(-128.0f, sr, br), bpr8 = fmaf(-128.0f, sr8, br8);
  y[0] = fmaf(sr, a1[0], fmaf(sr, a0[0], fmaf(bpr, xsm.x, y[0])));
  y[2] = fmaf(sr8, a1[2], fmaf(sr8, a0[2], fmaf(bpr8, xsm.x, y[2])));
  if constexpr (!ONE_COL) {
    y[1] = fmaf(sr, a1[1], fmaf(sr, a0[1], fmaf(bpr, xsm.y, y[1])));
    y[3] = fmaf(sr8, a1[3], fmaf(sr8, a0[3], fmaf(bpr8, xsm.y, y[3])));
  }
}

// Final values of one 16-row tile; gate/up combines streams 0 and 1.
template <bool XF32, bool GATE_UP, bool YF32>
__device__ __forceinline__ void store_tile(const GemvArgs &a, int rt, int lane, const float *y0, const float *y1) {
  const int r = lane >> 2, c = lane & 3;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int row = rt * 16 + r + 8 * half;
    if (row >= a.out) continue;
    if constexpr (XF32) {
      const int t = c;  // columns 2c (hi) and 2c+1 (lo) are the parts of token c
      if (t >= a.m) continue;
      float v = y0[2 * half] + y0[2 * half + 1];
      if constexpr (GATE_UP) v = silu_mul(v, y1[2 * half] + y1[2 * half + 1]);
      if constexpr (YF32)
        static_cast<float *>(a.y)[(size_t)t * a.out + row] = v;
      else
        static_cast<uint16_t *>(a.y)[(size_t)t * a.out + row] = f32_to_bf16_bits(v);
    } else {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = 2 * c + e;
        if (t >= a.m) continue;
        float v = y0[2 * half + e];
        if constexpr (GATE_UP) v = silu_mul(v, y1[2 * half + e]);
        if constexpr (YF32)
          static_cast<float *>(a.y)[(size_t)t * a.out + row] = v;
        else
          static_cast<uint16_t *>(a.y)[(size_t)t * a.out + row] = f32_to_bf16_bits(v);
      }
    }
  }
}

template <int CB, bool ONE_COL, bool XF32, bool SF16, bool GATE_UP, bool YF32>
__global__ void __launch_bounds__(kThreads, 2) gemv_kernel(const GemvArgs a) {
  constexpr int NS = GATE_UP ? 2 : 1;
  extern __shared__ __align__(128) unsigned char smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int R = a.stages;
  constexpr size_t SB = (size_t)NS * CB * kSgBytes;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem);
  uint64_t *empty = full + kMaxStages;
  unsigned char *ring = smem + 128;
  unsigned char *tail = ring + (size_t)R * SB;
  uint4 *xs4 = reinterpret_cast<uint4 *>(tail);
  float *xsum = reinterpret_cast<float *>(tail + xs_bytes(a.ng, a.mcols));

  // this CTA's run of slab-groups, in chunks of CB
  const long long F0 = run_begin(blockIdx.x, a.sgs, gridDim.x), F1 = run_begin(blockIdx.x + 1, a.sgs, gridDim.x);
  const int nch = (int)((F1 - F0 + CB - 1) / CB);

  if (threadIdx.x == 0) {
    for (int s = 0; s < R; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumers);
    }
  }
  fence_mbar_init();
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kConsumers) {
    // ---- producer: one elected lane streams the run -------------------------
    if (lane != 0) return;
    const uint64_t pol = evict_first_policy();
    for (int n = 0; n < nch; ++n) {
      const int s = n % R;
      if (n >= R && !mbar_wait_bounded(&empty[s], (uint32_t)(((n / R) - 1) & 1), kWaitLimitNs)) {
        raise_status(a.status, kStatusTimeout);
        // copies already issued must land before the CTA's memory is reused
        for (int k = n - R; k < n; ++k)
          if (k >= 0) (void)mbar_wait_bounded(&full[k % R], (uint32_t)((k / R) & 1), kWaitLimitNs);
        return;
      }
      const long long fb = F0 + (long long)n * CB;
      const int cnt = (int)min((long long)CB, F1 - fb);
      unsigned char *dst = ring + (size_t)s * SB;
      mbar_arrive_expect_tx(&full[s], (uint32_t)(NS * cnt * kSgBytes));
      bulk_g2s(dst, a.qw0 + fb * 4096, cnt * 4096, &full[s], pol);
      bulk_g2s(dst + (size_t)NS * CB * 4096, a.sb0 + fb * 512, cnt * 512, &full[s], pol);
      if constexpr (GATE_UP) {
        bulk_g2s(dst + (size_t)CB * 4096, a.qw1 + fb * 4096, cnt * 4096, &full[s], pol);
        bulk_g2s(dst + (size_t)NS * CB * 4096 + CB * 512, a.sb1 + fb * 512, cnt * 512, &full[s], pol);
      }
    }
    // the consumers wait for every chunk before they release it
    return;
  }

  // ---- consumers: warp `warp` owns tile `warp` of every slab-group ----------
  const int r = lane >> 2, c = lane & 3;
  pdl_wait();
  stage_x<XF32>(a, xs4, xsum);
  const bool col_live = r < a.mcols;
  // this lane's B-fragment entries and group sums, advanced per group
  const int xstride = 2 * a.mcols * 4;  // uint4 entries per group
  const uint4 *xl = xs4 + r * 4 + c;
  const float *xsl = xsum + 2 * c;

  float y[NS][4], yfirst[NS][4];
#pragma unroll
  for (int s = 0; s < NS; ++s)
#pragma unroll
    for (int e = 0; e < 4; ++e) y[s][e] = yfirst[s][e] = 0.0f;
  int slab = (int)(F0 / a.ng), g = (int)(F0 % a.ng);
  long long seg0 = F0;
  bool have_first = false;
  int first_slab = slab;

  auto step = [&](const unsigned char *wq_u, const unsigned char *sb_u, int gg) {
    uint4 xa = make_uint4(0, 0, 0, 0), xb = make_uint4(0, 0, 0, 0);
    if (col_live) {
      xa = xl[(size_t)gg * xstride];
      xb = xl[(size_t)gg * xstride + a.mcols * 4];
    }
    const float2 xsm = *reinterpret_cast<const float2 *>(xsl + gg * 8);
#pragma unroll
    for (int si = 0; si < NS; ++si) {
      const uint4 w = *reinterpret_cast<const uint4 *>(wq_u + (size_t)si * CB * 4096);
      const uint2 q = *reinterpret_cast<const uint2 *>(sb_u + (size_t)si * CB * 512);
      gt_step<SF16, ONE_COL>(y[si], w, q, xa, xb, xsm);
    }
  };

  long long f = F0;
  for (int n = 0; n < nch; ++n) {
    const int s = n % R;
    if (!mbar_wait_bounded(&full[s], (uint32_t)((n / R) & 1), kWaitLimitNs)) {
      // the producer then times out on this stage's release and stops;
      // outputs of this call are undefined and the status word says so
      raise_status(a.status, kStatusTimeout);
      return;
    }
    const unsigned char *stw = ring + (size_t)s * SB + warp * 512 + lane * 16;
    const unsigned char *sts = ring + (size_t)s * SB + (size_t)NS * CB * 4096 + warp * 64 + r * 8;
    const int cnt = (int)min((long long)CB, F1 - f);
    if (cnt == CB && a.ng - g > CB) {
      // no slab boundary in this chunk
#pragma unroll
      for (int u = 0; u < CB; ++u) step(stw + u * 4096, sts + u * 512, g + u);
      g += CB;
      f += CB;
    } else {
      for (int u = 0; u < cnt; ++u, ++f) {
        step(stw + u * 4096, sts + u * 512, g);
        if (++g == a.ng) {  // slab boundary
          const long long s0 = (long long)slab * a.ng;
          if (seg0 == s0) {
            store_tile<XF32, GATE_UP, YF32>(a, slab * kSlabTiles + warp, lane, y[0], y[NS - 1]);
          } else {  // the run's first segment, partial: kept for the hand-over
            have_first = true;
            first_slab = slab;
#pragma unroll
            for (int si = 0; si < NS; ++si)
#pragma unroll
              for (int e = 0; e < 4; ++e) yfirst[si][e] = y[si][e];
          }
#pragma unroll
          for (int si = 0; si < NS; ++si)
#pragma unroll
            for (int e = 0; e < 4; ++e) y[si][e] = 0.0f;
          g = 0;
          ++slab;
          seg0 = f + 1;
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  // The run's partial slabs: its first (if it began inside a slab) and its
  // last (if it ended inside one).  Publish this CTA's part; the CTA that
  // arrives last adds every part in CTA order and stores the tile.
  auto hand_over = [&](int sl, int side, float (&v)[NS][4]) {
    float *gslot = a.part + (((size_t)blockIdx.x * 2 + side) * kSlabTiles + warp) * (NS * 128) + lane * 4;
#pragma unroll
    for (int si = 0; si < NS; ++si)
#pragma unroll
      for (int e = 0; e < 4; ++e) gslot[si * 128 + e] = v[si][e];
    __threadfence();
    __syncwarp();
    const long long t0 = (long long)sl * a.ng, t1 = t0 + a.ng;
    const long long clo = run_of(t0, a.sgs, gridDim.x), chi = run_of(t1 - 1, a.sgs, gridDim.x);
    uint32_t old = 0;
    uint32_t *cnt = &a.count[(size_t)sl * kSlabTiles + warp];
    if (lane == 0) old = atomicAdd(cnt, 1u);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old + 1 != (uint32_t)(chi - clo + 1)) return;
    __threadfence();
    float acc[NS][4];
#pragma unroll
    for (int si = 0; si < NS; ++si)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[si][e] = 0.0f;
    for (long long q = clo; q <= chi; ++q) {
      const int qs = (q == clo && run_begin(q, a.sgs, gridDim.x) < t0) ? 1 : 0;
      const volatile float *src = a.part + (((size_t)q * 2 + qs) * kSlabTiles + warp) * (NS * 128) + lane * 4;
#pragma unroll
      for (int si = 0; si < NS; ++si)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[si][e] += src[si * 128 + e];
    }
    if (lane == 0) *cnt = 0;  // ready for the next call
    store_tile<XF32, GATE_UP, YF32>(a, sl * kSlabTiles + warp, lane, acc[0], acc[NS - 1]);
  };
  if (have_first) hand_over(first_slab, 0, yfirst);
  // a last segment that did not end on a slab boundary (it is also the first
  // segment when the whole run lies inside one slab)
  if (F1 > F0 && seg0 < F1) hand_over(slab, seg0 == F0 ? 0 : 1, y);
}

template <int CB, bool ONE_COL, bool XF32, bool SF16, bool GATE_UP, bool YF32>
cudaError_t launch_one(const GemvArgs &a, int grid, size_t smem, cudaStream_t stream) {
  auto *k = &gemv_kernel<CB, ONE_COL, XF32, SF16, GATE_UP, YF32>;
  static DeviceOnce once;
  cudaError_t e = once.run([&] {
    return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvMaxSmem);
  });
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = gemv_pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, a);
}

template <bool XF32, bool SF16>
cudaError_t dispatch(const GemvArgs &a, bool gate_up, bool yf32, int grid, size_t smem, cudaStream_t s) {
  // chunk of slab-groups per stage: 2 per stream for gate/up, 4 otherwise
  // (a forced 1, 2 or 4 is honoured for the plain projection)
  if (gate_up)
    return yf32 ? launch_one<2, false, XF32, SF16, true, true>(a, grid, smem, s)
                : launch_one<2, false, XF32, SF16, true, false>(a, grid, smem, s);
  const bool one = !XF32 && a.mcols == 1;
#define THQ4_PLAIN(CB_)                                                                         \
  if (a.cb == CB_) {                                                                            \
    if (one)                                                                                    \
      return yf32 ? launch_one<CB_, true, XF32, SF16, false, true>(a, grid, smem, s)            \
                  : launch_one<CB_, true, XF32, SF16, false, false>(a, grid, smem, s);          \
    return yf32 ? launch_one<CB_, false, XF32, SF16, false, true>(a, grid, smem, s)             \
                : launch_one<CB_, false, XF32, SF16, false, false>(a, grid, smem, s);           \
  }
  THQ4_PLAIN(4)
  THQ4_PLAIN(2)
  THQ4_PLAIN(1)
#undef THQ4_PLAIN
  return cudaErrorInvalidValue;
}

}  // namespace

size_t gemv_workspace_bytes(int rows) {
  // one partial per CTA side (at most two CTAs per SM), sized for gate and
  // up, then one counter per (slab, tile)
  const size_t ctas = (size_t)device_sm_count() * 2;
  return ctas * 2 * side_floats(true) * sizeof(float) +
         ((size_t)row_slabs(rows) * kSlabTiles * 4 + 255) / 256 * 256;
}

GemvPlan gemv_plan(int out, int in, int m, bool x_f32, bool gate_up) {
  GemvPlan p{};
  const int ng = in / kGroup;
  const int sms = device_sm_count();
  const GemvCfg cfg = gemv_cfg_override();
  int per = x_f32 ? 4 : 8;  // tokens per launch: 8 B columns, two per f32 token
  if (per > m) per = m;
  const long long sgs = (long long)row_slabs(out) * ng;
  // ~16 KB of nibbles per stage: 4 slab-groups, or 2 per stream for gate/up
  const int cb = gate_up ? 2 : (cfg.warps > 0 ? cfg.warps : 4);
  p.ok = false;
  int per_sm = 2;
  for (;;) {
    const int mcols = x_f32 ? 2 * per : per;
    int st = 0;
    if (cfg.depth > 0) {
      if (gemv_smem(cfg.depth, cb, gate_up, ng, mcols) <= (size_t)kGemvMaxSmem) st = cfg.depth;
      per_sm = st && gemv_smem(st, cb, gate_up, ng, mcols) <= (size_t)kGemvHalfSmem ? 2 : 1;
    } else {
      // two CTAs per SM with the deepest ring that fits half an SM (up to 6),
      // else one CTA per SM
      for (int t = 6; t >= 2 && !st; --t)
        if (gemv_smem(t, cb, gate_up, ng, mcols) <= (size_t)kGemvHalfSmem) st = t;
      per_sm = 2;
      if (!st) {
        per_sm = 1;
        for (int t = kMaxStages; t >= 2 && !st; --t)
          if (gemv_smem(t, cb, gate_up, ng, mcols) <= (size_t)kGemvMaxSmem) st = t;
      }
    }
    if (st) {
      p.ok = true;
      p.stages = st;
      p.smem = gemv_smem(st, cb, gate_up, ng, mcols);
      break;
    }
    if (per == 1) break;
    per = (per + 1) / 2;
  }
  long long grid = cfg.grid > 0 ? cfg.grid : (long long)sms * per_sm;
  if (grid > (long long)sms * 2) grid = (long long)sms * 2;
  if (sgs < grid) grid = sgs;  // every CTA run holds at least one slab-group
  p.grid = (int)grid;
  p.threads = kThreads;
  p.pieces = (int)grid;
  p.tokens_per_pass = per;
  p.ch = cb;
  return p;
}

cudaError_t gemv_launch(const thq4_weight &w0, const thq4_weight *w1, const void *x, bool x_f32, int m, void *y,
                        bool y_f32, void *workspace, cudaStream_t stream) {
  const bool gate_up = w1 != nullptr;
  const GemvPlan p = gemv_plan(w0.out, w0.in, m, x_f32, gate_up);
  if (!p.ok) return cudaErrorInvalidConfiguration;
  const int xb = x_f32 ? 4 : 2, yb = y_f32 ? 4 : 2;
  const int ng = w0.in / kGroup;
  const size_t part_bytes =
      gemv_workspace_bytes(w0.out) - ((size_t)row_slabs(w0.out) * kSlabTiles * 4 + 255) / 256 * 256;
  for (int t0 = 0; t0 < m; t0 += p.tokens_per_pass) {
    const int mt = min(p.tokens_per_pass, m - t0);
    GemvArgs a{};
    a.qw0 = static_cast<const uint8_t *>(w0.qw);
    a.sb0 = static_cast<const uint8_t *>(w0.sb);
    a.qw1 = gate_up ? static_cast<const uint8_t *>(w1->qw) : nullptr;
    a.sb1 = gate_up ? static_cast<const uint8_t *>(w1->sb) : nullptr;
    a.x = static_cast<const char *>(x) + (size_t)t0 * w0.in * xb;
    a.y = static_cast<char *>(y) + (size_t)t0 * w0.out * yb;
    a.status = status_word();
    a.part = static_cast<float *>(workspace);
    a.count = reinterpret_cast<uint32_t *>(static_cast<char *>(workspace) + part_bytes);
    a.sgs = (long long)row_slabs(w0.out) * ng;
    a.m = mt;
    a.in = w0.in;
    a.ng = ng;
    a.out = w0.out;
    a.mcols = x_f32 ? 2 * mt : mt;
    a.stages = p.stages;
    a.cb = p.ch;
    const size_t smem = gemv_smem(p.stages, p.ch, gate_up, ng, a.mcols);
    const bool f16 = w0.sb_dtype == THQ4_F16;
    cudaError_t e;
    if (x_f32)
      e = f16 ? dispatch<true, true>(a, gate_up, y_f32, p.grid, smem, stream)
              : dispatch<true, false>(a, gate_up, y_f32, p.grid, smem, stream);
    else
      e = f16 ? dispatch<false, true>(a, gate_up, y_f32, p.grid, smem, stream)
              : dispatch<false, false>(a, gate_up, y_f32, p.grid, smem, stream);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace thq4
