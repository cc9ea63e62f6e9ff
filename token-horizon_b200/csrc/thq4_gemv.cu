// thq4_gemv.cu -- decode (m = 1) and spec-verify (m <= 8) Q4 projections.
//
// Replaces the reference's m = 1 matvec AffineQmvT / qmvt<RPL,NSG,GateUp>
// (engine/src/quant_kernel.rs:2768-3136) and its m <= 8 decode/verify families
// AffineQmpp (th_mpp_tile, :1793-2569), AffineQsg (:1149-1632) and AffineQmm
// (:1634-1740), with one kernel.
//
// The path is bound by HBM bandwidth (0.5625 bytes per weight, each read
// once), and on B200 the instruction budget per streamed byte is tight: at
// full bandwidth an SM has ~25 cycles for each 16x64 tile-group (576 bytes).
// Hence:
//   - the weight is a stream of "slab-groups" (SG): 128 rows x 64 k, 4096
//     bytes of nibbles + 512 bytes of scale/bias, slab-major, so any run of
//     SGs is one contiguous byte range of the frag layout.  A persistent grid
//     (one CTA per SM) gives every CTA an equal run of "chunks" (CB = 8, or 4,
//     consecutive SGs of one slab, CB-aligned); a run may start and end
//     inside a slab.  Where whole slabs per CTA still fill >= 85% of the SMs
//     the grid is the slab count instead, and nothing is split;
//   - one producer warp per CTA streams the run into a ring of shared-memory
//     stages with bulk copies (cp.async.bulk, evict-first in L2, no
//     multicast) of one chunk each, completing on a "full" mbarrier per stage;
//     the first stages are requested before the kernel waits for its input;
//   - eight consumer warps each own one 16-row tile of every SG, so their
//     output rows are disjoint and no reduction crosses warps (sixteen, two
//     per tile, measured no faster: the LOP3 work of the in-register dequant
//     fills the ALU pipe either way).  Per SG a warp
//     runs four mma.m16n8k16 (fp16 x fp16 -> f32) with the weight as the A
//     operand (16 rows) and activation columns as N (8).  unpack_word
//     (thq4_common.cuh) turns a frag word into the four A registers: the
//     even k-steps' nibble pairs as the exact fp16 q (a LOP3 gives 1024 + q,
//     an f16x2 subtraction removes the 1024), the odd k-steps' as 64 + q (a
//     LOP3 on the nibbles in mantissa bits 4..7).  Two independent chains
//     (k-steps 0, 2 and 1, 3) meet in the epilogue as acc0 + acc1 - off,
//     off = 64 * (sum of x over the odd k-steps) computed when x is staged.
//     The group's value is then the reference's per-group form
//     (quant_kernel.rs:1994-2001, 2887-2890):  s * sum(q x) + b * sum(x).
//     (Offsets cost accumulator bits: 1024 + q would carry the offset at
//     1024x the size of the q signal, so it is removed exactly before the
//     MMA; 64 + q costs six bits on half the products);
//   - with few tokens most of the 8 columns are free, so consecutive groups
//     share one accumulator: in a "window" of GW groups (4 when a group
//     needs <= 2 columns), group j's activation sits in columns
//     [8j/GW, 8(j+1)/GW) and is zero elsewhere.  After the window each lane
//     holds the sums of exactly one group (its own columns), so the scale /
//     bias epilogue runs once per window with every lane busy -- 4x fewer
//     epilogue instructions for a matvec.  Windows never cross a chunk, so
//     the epilogue reads its scales from the stage still held;
//   - the activation is converted to fp16 per (group, token) with a power-of-
//     two scale 2^e that puts the group's largest |x| in [2^14, 2^15): exact
//     for bf16 input over 31 binades below the group maximum, no overflow at
//     any magnitude; e is undone in the epilogue.  An f32 activation is split
//     into fp16 hi + lo parts in two columns (22 significant bits);
//   - a slab split between CTAs (only a CTA's first and last slab can be) is
//     finished per tile by the warp that arrives last ("last arriver
//     reduces", the reference's split-K scheme, quant_kernel.rs:1299-1332):
//     each writes its partial to the caller's workspace and bumps the
//     (slab, tile) counter; the last one adds the partials in CTA order, so
//     results are bitwise deterministic (qwen35.rs:6986-6988) with no
//     waiting, and resets the counter;
//   - the kernel uses programmatic dependent launch: the next projection's
//     CTA can become resident and request its weights while this one
//     finishes; griddepcontrol.wait guards only the activation reads and the
//     output writes.  Every mbarrier wait is bounded in time and reports
//     kStatusTimeout instead of hanging.
#include <algorithm>
#include <atomic>
#include <mutex>

#include "thq4_common.cuh"
#include "thq4_internal.h"

namespace thq4 {

namespace {

constexpr int kConsumers = kSlabTiles;  // chain kernel: one consumer warp per tile of a slab
constexpr int kThreads = (kConsumers + 1) * 32;
// The decode/verify kernel has two consumer warps per 16-row tile; all
// sixteen stage the activation.  For a single weight both also stream:
// warp t + 8h takes the run's chunks n with n % 2 == h for tile t, and the
// pair adds its partial sums at every slab end -- twice the warps to cover
// the latency of the in-register dequant and of the MMA chains (one-weight
// launches measured 6-15% faster).  In the fused gate/up only warp t
// streams (gemv_wpt = 1): its 73.7 KB stages fill the ring in two, and with
// both stages being consumed at once nothing would be in flight (measured
// 23% slower).
constexpr int kGemvConsumers = 2 * kSlabTiles;
constexpr int kGemvThreads = (kGemvConsumers + 1) * 32;
__host__ __device__ constexpr int gemv_wpt(bool gate_up) { return gate_up ? 1 : 2; }
constexpr int kSgBytes = kSlabTiles * (kChunkBytes + kQuadBytes);  // 4608
constexpr int kMaxStages = 8;

struct GemvArgs {
  const uint8_t *qw0;  // gate (or the only) weight: frag nibbles
  const uint8_t *sb0;
  const uint8_t *qw1;  // up weight (gate/up only)
  const uint8_t *sb1;
  const void *x;       // [m][in], bf16 or f32
  void *y;             // [m][out], bf16 or f32
  uint32_t *status;    // device status word
  float *part;         // workspace: partials [cta][2 sides][8 tiles][NS][32 lanes][4]
  uint32_t *count;     // workspace: arrivals per (slab, tile) (zero between calls)
  int chunks;          // slabs * cps: the units CTA runs are cut in
  int run_base, run_rem;  // chunks / grid, chunks % grid: run i holds base + (i < rem)
  int cps;             // chunks per slab, ceil(ng / cb)
  int m, in, ng, out;
  int P;               // B columns in use: m (bf16 x) or 2m (f32 x)
  int xf32, yf32;
  int stages;          // ring stages
  int xcap;            // activation groups staged per CTA
  int pre;             // stages requested before x is staged (0: all)
  int cl_j;            // > 1: slab-split mode, j CTAs per slab in one cluster
  // fused exchange of shards (g_mode 0: none).  g_mode 1 (gather): the
  // first g_rows outputs also go to full[t * g_stride + g_off + row] on
  // every rank; g_mode 2 (reduce): every output, in f32, goes to slot g_rank
  // of every rank's reduction buffer instead of y.  Then the grid's last CTA
  // raises this rank's flag on every peer.  g_wait: wait for the peers'
  // flags before reading x.  g_mode 3 (low-latency reduce): as 2, but every
  // output is one 8-byte word {f32 bits, this exchange's number} that the
  // reader polls for; no fence and no flag.
  uint16_t *const *g_dst;
  uint32_t *const *g_flags;
  uint32_t *g_count, *g_arrive;
  int g_mode, g_world, g_rank, g_rows, g_off, g_stride, g_wait;
  long long g_slot;
  // xparts > 0: x is xparts f32 partials (x + p * xslot floats, [m][in]),
  // summed in order and rounded to bf16 as they are staged
  int xparts;
  long long xslot;
  // x_ll: the partials are low-latency words (g_mode 3's layout: 8 bytes
  // {f32 bits, exchange number}, x + p * xslot words); each is waited for
  // until it carries this exchange's number
  int x_ll;
  // x is a presum block: its f32 sums [ng][8] (the bias term's sum(x) of
  // group g, token t at xsum[g * 8 + t]); nullptr otherwise
  const float *xsum;
  // phase trace (testing hook; nullptr = off): a record of 8 header words
  // then 8 %globaltimer stamps per CTA (thq4_debug_set_trace)
  unsigned long long *trace;
};

// Phase stamps of the trace, taken by thread 0 (consumer warp 0).
enum : int {
  kTrEntry = 0,    // CTA running, barriers initialised
  kTrPdl = 1,      // griddepcontrol.wait returned: the predecessor completed
  kTrPeer = 2,     // the peers' exchange flags seen (= kTrPdl without a wait)
  kTrStaged = 3,   // activation staged in shared memory
  kTrFirst = 4,    // the first weight stage has landed
  kTrStreamed = 5, // every stage consumed
  kTrStored = 6,   // outputs stored (after any split-K or cluster combine)
  kTrDone = 7,     // exchange signalled; the CTA exits
  kTrFenced = 8,   // exchange: this CTA's stores fenced at system scope, arrival counted
  kTrFlagged = 9,  // exchange: the peers' flags written (the grid's last CTA only)
};
constexpr int kTrStamps = 10;
__device__ __forceinline__ void trace_stamp(const GemvArgs &a, int i) {
  if (a.trace && threadIdx.x == 0) a.trace[8 + (size_t)blockIdx.x * kTrStamps + i] = global_timer_ns();
}

// columns with per-group metadata: P rounded up to even (lanes own pairs)
__host__ __device__ inline int meta_cols(int P) { return (P + 1) & ~1; }
// fp16 B fragments [slot][P][2][4] x 16 B, a 128-byte zero block, then per
// (slot, column) {xs, f, off, 0}: the column's sum(x), its scale 2^e and
// the magic-number offset 64 sum(x') over the group's odd k-steps
__host__ __device__ inline size_t xstage_bytes(int xcap, int P) {
  return (size_t)xcap * P * 128 + 128 + (size_t)xcap * meta_cols(P) * 16;
}
__host__ __device__ inline size_t stage_bytes(int cb, bool gate_up) { return (size_t)(gate_up ? 2 : 1) * cb * kSgBytes; }
// two buffers of one warp's partial sums per (tile, stream) for the warp
// pairs' slab-end exchange (two consumer warps per tile)
__host__ __device__ inline size_t pair_bytes(bool gate_up) {
  return gemv_wpt(gate_up) == 2 ? (size_t)2 * kSlabTiles * (gate_up ? 2 : 1) * 32 * 16 : 0;
}
__host__ __device__ inline size_t gemv_smem(int stages, int cb, bool gate_up, int xcap, int P) {
  return 256 + (size_t)stages * stage_bytes(cb, gate_up) + xstage_bytes(xcap, P) + pair_bytes(gate_up);
}
// floats of one CTA side's partial: 8 tiles x NS x 32 lanes x 4
__host__ __device__ inline int side_floats(bool gate_up) { return kSlabTiles * (gate_up ? 2 : 1) * 32 * 4; }
// First chunk of run i: runs hold base + 1 chunks for i < rem, base after.
template <class A>
__device__ __forceinline__ int run_begin(const A &a, int i) { return i * a.run_base + min(i, a.run_rem); }
// The run holding chunk o (every run is non-empty: base >= 1).
template <class A>
__device__ __forceinline__ int run_of(const A &a, int o) {
  const int big = a.run_rem * (a.run_base + 1);
  return o < big ? o / (a.run_base + 1) : a.run_rem + (o - big) / a.run_base;
}
// slab-groups before chunk C
__device__ __forceinline__ int sgs_before(int C, int cps, int ng, int cb) {
  const int sl = C / cps;
  return sl * ng + min((C - sl * cps) * cb, ng);
}
template <int NC = kConsumers>
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;\n" ::"r"(NC * 32) : "memory");
}

// Eight consecutive low-latency words (four 16-byte loads, each 8-byte word
// read whole): their f32 values once every word carries `seq`.  Words that
// do not yet are read again until the deadline, after which `late` is set and
// the values read last are used (the status word then says kStatusTimeout).
__device__ __forceinline__ void ll_wait8(const uint4 *w4, uint32_t seq, uint64_t deadline, bool &late, float (&d)[8]) {
  uint4 q[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) q[i] = ld_volatile_v4(w4 + i);
  for (;;) {
    bool ok = true;
#pragma unroll
    for (int i = 0; i < 4; ++i) ok = ok && q[i].y == seq && q[i].w == seq;
    if (ok || late) break;
    if (global_timer_ns() > deadline) {
      late = true;
      break;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (q[i].y != seq || q[i].w != seq) q[i] = ld_volatile_v4(w4 + i);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    d[2 * i] = __uint_as_float(q[i].x);
    d[2 * i + 1] = __uint_as_float(q[i].z);
  }
}

// Stage the activation groups [gs, gs + xcnt) (mod ng) of the m tokens into
// shared memory (consumer warps only).  Fragment entry ((slot*P + q)*2 + h)*4
// + c (16 bytes) holds, for k-steps 2h and 2h+1 of the group, the fp16 pairs
// {x'[2c], x'[2c+1]}, {x'[2c+8], x'[2c+9]} (k relative to the k-step) of
// column q: token q (bf16 x) or token q/2's hi (even q) or lo (odd q) part
// (f32 x), with x' = x 2^-e.  One item = 8 consecutive k of one (slot,
// column), read with one vector load; the 8 items of a (slot, column) are 8
// adjacent lanes, which reduce the group's max |x| and sum with a fixed
// shuffle tree (deterministic).  Up to four items per thread are requested
// before any is used.
template <bool PARTS, int NC = kConsumers, class A>
__device__ __forceinline__ void stage_x(const A &a, int gs, int xcnt, uint4 *xf, uint4 *zero, float4 *mx) {
  const int tid = threadIdx.x, nthr = NC * 32;
  const int P = a.P, P8 = meta_cols(P);
  constexpr int kU = 4;
  if (tid < 8) zero[tid] = make_uint4(0, 0, 0, 0);
  if (P & 1)  // the unused column of the last pair contributes nothing
    for (int i = tid; i < xcnt; i += nthr) mx[i * P8 + P] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  uint32_t *xw = reinterpret_cast<uint32_t *>(xf);
  const int items = xcnt * P * 8;
  // low-latency partials: this exchange's number (this rank's count, final
  // once the previous launch completed) and one deadline for every wait
  uint32_t ll_seq = 0;
  uint64_t ll_deadline = 0;
  bool ll_late = false;
  if constexpr (PARTS) {
    if (a.x_ll) {
      ll_seq = *reinterpret_cast<const volatile uint32_t *>(a.g_count);
      ll_deadline = global_timer_ns() + kWaitLimitNs;
    }
  }
  const int span = (items + 31) / 32 * 32;  // whole warps: every lane takes part in the shuffles
  // An item slot whose whole warp lies past `span` is skipped (the test is
  // warp-uniform: nthr and span are multiples of 32), so a warp does the
  // conversion work of the items it holds and no more.
  const int wfirst = tid & ~31;
  for (int base = tid; base < span; base += kU * nthr) {
    float v[kU][8];
#pragma unroll
    for (int it = 0; it < kU; ++it) {
      const int idx = base + it * nthr;
#pragma unroll
      for (int e = 0; e < 8; ++e) v[it][e] = 0.0f;
      if (idx >= items) continue;
      const int h8 = idx & 7, sq = idx >> 3, q = P == 1 ? 0 : sq % P, slot = P == 1 ? sq : sq / P;
      int g = gs + slot;
      if (g >= a.ng) g -= a.ng;
      const int t = a.xf32 ? q >> 1 : q;
      const size_t at = (size_t)t * a.in + (size_t)g * kGroup + 8 * h8;
      if constexpr (PARTS) {  // the all-reduce's last step: sum the ranks' partials in order, one bf16 rounding
        if (a.x_ll) {
#pragma unroll 1
          for (int pp = 0; pp < a.xparts; ++pp) {
            const uint4 *w4 =
                reinterpret_cast<const uint4 *>(static_cast<const unsigned long long *>(a.x) + (size_t)pp * a.xslot + at);
            float d[8];
            ll_wait8(w4, ll_seq, ll_deadline, ll_late, d);
#pragma unroll
            for (int e = 0; e < 8; ++e) v[it][e] += d[e];
          }
        } else {
#pragma unroll 1
          for (int pp = 0; pp < a.xparts; ++pp) {
            const float4 *p4 =
                reinterpret_cast<const float4 *>(static_cast<const float *>(a.x) + (size_t)pp * a.xslot + at);
            const float4 u0 = p4[0], u1 = p4[1];
            v[it][0] += u0.x, v[it][1] += u0.y, v[it][2] += u0.z, v[it][3] += u0.w;
            v[it][4] += u1.x, v[it][5] += u1.y, v[it][6] += u1.z, v[it][7] += u1.w;
          }
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) v[it][e] = __uint_as_float((uint32_t)f32_to_bf16_bits(v[it][e]) << 16);
      } else if (a.xf32) {
        const float4 *p4 = reinterpret_cast<const float4 *>(static_cast<const float *>(a.x) + at);
        const float4 u0 = p4[0], u1 = p4[1];
        v[it][0] = u0.x, v[it][1] = u0.y, v[it][2] = u0.z, v[it][3] = u0.w;
        v[it][4] = u1.x, v[it][5] = u1.y, v[it][6] = u1.z, v[it][7] = u1.w;
      } else {
        const uint4 u = *reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(a.x) + at);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          v[it][2 * e] = __uint_as_float(w[e] << 16);
          v[it][2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
        }
      }
    }
    // all kU items go through the shuffle trees together (independent
    // chains); an item past `span` is a whole warp's, whose results are dropped
#pragma unroll
    for (int it = 0; it < kU; ++it) {
      const int idx = base + it * nthr;
      if ((base - tid + wfirst) + it * nthr >= span) break;  // this warp holds no item here or later
      const bool live = idx < items;
      const int h8 = idx & 7, sq = live ? idx >> 3 : 0, q = P == 1 ? 0 : sq % P, slot = P == 1 ? sq : sq / P;
      const int part = a.xf32 ? q & 1 : 0;
      float amax = 0.0f;
#pragma unroll
      for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(v[it][e]));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
      // 2^e with the group max in [2^14, 2^15); e = 0 for an all-zero group
      const int ex = (__float_as_int(amax) >> 23) & 0xff;
      const int e2 = ex == 0 ? 0 : min(max(ex - 127 - 14, -110), 114);
      const float dn = __int_as_float((127 - e2) << 23), f = __int_as_float((127 + e2) << 23);
      float sum = 0.0f;
      uint32_t hv[4];
#pragma unroll
      for (int pr = 0; pr < 4; ++pr) {
        uint32_t bits = 0;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const float xs = v[it][2 * pr + hh] * dn;
          const __half hi = __float2half_rn(xs);
          const __half val = part ? __float2half_rn(xs - __half2float(hi)) : hi;
          sum += __half2float(val);
          bits |= (uint32_t)__half_as_ushort(val) << (16 * hh);
        }
        hv[pr] = bits;
      }
      if (live) {
        // k = 8 h8 + 2 pr + {0, 1}: k-step kp = h8 / 2, lane column pr, word
        // 2 (kp & 1) + (h8 & 1) of entry ((slot*P + q)*2 + kp/2)*4 + pr
        const int kp = h8 >> 1, wd = 2 * (kp & 1) + (h8 & 1);
        const int e0 = ((slot * P + q) * 2 + (kp >> 1)) * 4;
#pragma unroll
        for (int pr = 0; pr < 4; ++pr) xw[(e0 + pr) * 4 + wd] = hv[pr];
      }
      // the odd k-steps' values meet the weights as 64 + q (unpack_word):
      // their sum is the offset the epilogue takes back out
      float osum = (h8 & 2) ? sum : 0.0f;
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      sum += __shfl_xor_sync(0xffffffffu, sum, 4);
      osum += __shfl_xor_sync(0xffffffffu, osum, 1);
      osum += __shfl_xor_sync(0xffffffffu, osum, 2);
      osum += __shfl_xor_sync(0xffffffffu, osum, 4);
      if (live && h8 == 0) {
        // the bias term's sum(x): the producer's (presum block) or this one;
        // the offset term always uses the sum of the fp16 values multiplied
        int g = gs + slot;
        if (g >= a.ng) g -= a.ng;
        const float bsum = a.xsum ? a.xsum[g * 8 + q] : f * sum;
        mx[slot * P8 + q] = make_float4(bsum, f, 64.0f * osum, 0.0f);
      }
    }
  }
  if constexpr (PARTS) {
    if (ll_late) raise_status(a.status, kStatusTimeout);
  }
  consumer_sync<NC>();
}

// Final values of one 16-row tile from lanes holding reduced column pairs;
// gate/up combines streams 0 and 1.
template <int GW, bool GATE_UP, class A>
__device__ __forceinline__ void store_tile(const A &a, int rt, int lane, const float *y0, const float *y1,
                                           uint32_t seq = 0) {
  constexpr int LPJ = 4 / GW;
  const int r = lane >> 2, c = lane & 3;
  if (c >= LPJ) return;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int row = rt * 16 + r + 8 * half;
    if (row >= a.out) continue;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      int t;
      float v, u = 0.0f;
      if (a.xf32) {  // columns 2c (hi) and 2c + 1 (lo) are the parts of token c
        if (e) break;
        t = c;
        v = y0[2 * half] + y0[2 * half + 1];
        if (GATE_UP) u = y1[2 * half] + y1[2 * half + 1];
      } else {
        t = 2 * c + e;
        v = y0[2 * half + e];
        if (GATE_UP) u = y1[2 * half + e];
      }
      if (t >= a.m) continue;
      if constexpr (GATE_UP) v = silu_mul(v, u);
      if (a.g_mode == 2) {  // this rank's partial of the output, into its slot on every rank (NVLink stores)
        for (int rk = 0; rk < a.g_world; ++rk)
          reinterpret_cast<float *>(a.g_dst[rk])[(size_t)a.g_rank * a.g_slot + (size_t)t * a.g_stride + row] = v;
      } else if (a.g_mode == 3) {  // the same as one 8-byte word {value, exchange number} the reader polls for
        const unsigned long long word = ((unsigned long long)seq << 32) | __float_as_uint(v);
        for (int rk = 0; rk < a.g_world; ++rk)
          st_volatile_u64(reinterpret_cast<unsigned long long *>(a.g_dst[rk]) + (size_t)a.g_rank * a.g_slot +
                              (size_t)t * a.g_stride + row,
                          word);
      } else if (a.yf32) {
        static_cast<float *>(a.y)[(size_t)t * a.out + row] = v;
      } else {
        const uint16_t bits = f32_to_bf16_bits(v);
        static_cast<uint16_t *>(a.y)[(size_t)t * a.out + row] = bits;
        if (a.g_mode == 1 && row < a.g_rows)  // the shard's slice of the full vector, on every rank (NVLink stores)
          for (int rk = 0; rk < a.g_world; ++rk) a.g_dst[rk][(size_t)t * a.g_stride + a.g_off + row] = bits;
      }
    }
  }
}

// Until every peer has completed as many gathers as this rank (its own
// count is final: the previous projection on this stream has completed), or
// kWaitLimitNs, after which the status word says kStatusTimeout.
__device__ void peer_wait(uint32_t *const *flags, const uint32_t *count, int world, int rank, uint32_t *status) {
  const uint32_t target = *reinterpret_cast<const volatile uint32_t *>(count);
  const uint32_t *mine = flags[rank];
  const uint64_t t0 = global_timer_ns();
  for (int rk = 0; rk < world; ++rk) {
    if (rk == rank) continue;
    while ((int32_t)(ld_acquire_sys(mine + rk) - target) < 0) {
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        raise_status(status, kStatusTimeout);
        return;
      }
    }
  }
}
// After every consumer warp's stores: the grid's last CTA bumps this rank's
// gather count and writes it into this rank's slot of every peer's flags.
template <int NC>
__device__ void peer_signal(const GemvArgs &a) {
  consumer_sync<NC>();
  if (threadIdx.x != 0) return;
  if (a.g_mode == 3) {
    // low-latency words need no fence or flag: the grid's last CTA only
    // counts the exchange (every CTA read the count before its stores)
    if (atom_add_acq_rel(a.g_arrive, 1u) + 1u == gridDim.x) {
      *a.g_arrive = 0;
      *a.g_count = *a.g_count + 1u;
    }
    trace_stamp(a, kTrFenced);
    return;
  }
  fence_acq_rel_sys();  // this CTA's stores, local and remote, before its arrival
  const bool last = atom_add_acq_rel(a.g_arrive, 1u) + 1u == gridDim.x;
  trace_stamp(a, kTrFenced);
  if (!last) return;
  *a.g_arrive = 0;
  const uint32_t c = *a.g_count + 1u;  // only the last CTA of each launch touches it
  *a.g_count = c;
  // Each flag store is a system-scope release: it orders before the flag
  // everything this thread has observed, including every other CTA's stores,
  // which each CTA fenced at system scope before its arrival that the
  // counter's acquire read (release is cumulative), so no second fence.
  for (int rk = 0; rk < a.g_world; ++rk)
    if (rk != a.g_rank) st_release_sys(a.g_flags[rk] + a.g_rank, c);
  trace_stamp(a, kTrFlagged);
}

__global__ void peer_wait_kernel(uint32_t *const *flags, const uint32_t *count, int world, int rank, uint32_t *status) {
  if (threadIdx.x == 0) peer_wait(flags, count, world, rank, status);
}

// The producer lane: streams the run's nch chunks from chunk C0 into the
// ring.  On a timeout it waits (bounded) for the copies it issued and stops.
template <int CB, bool GATE_UP>
__device__ __forceinline__ bool produce_run(const GemvArgs &a, int C0, int nch, int R, uint64_t *full, uint64_t *empty,
                                            uint64_t *xready, unsigned char *ring) {
  constexpr int NS = GATE_UP ? 2 : 1;
  constexpr size_t SB = (size_t)NS * CB * kSgBytes;
  const uint64_t pol = evict_first_policy();
  int sl = C0 / a.cps;  // slab and chunk-in-slab of chunk C0 + n
  int cg = C0 - sl * a.cps;
  int s = 0;
  uint32_t par = 0;  // parity of this use of stage s
  for (int n = 0; n < nch; ++n, ++cg) {
    if (cg == a.cps) cg = 0, ++sl;
    // Only the first a.pre stages go out before the consumers have staged
    // x: the activation loads then do not queue behind the whole ring's
    // weight burst.  (A timeout here only delays the stream.)
    if (n == a.pre && a.pre > 0) (void)mbar_wait_bounded(xready, 0, kWaitLimitNs);
    if (n >= R && !mbar_wait_bounded(&empty[s], par ^ 1u, kWaitLimitNs)) {
      raise_status(a.status, kStatusTimeout);
      // copies already issued must land before the CTA's memory is reused
      for (int k = n - R; k < n; ++k) (void)mbar_wait_bounded(&full[k % R], (uint32_t)((k / R) & 1), kWaitLimitNs);
      return false;
    }
    const int g0c = cg * CB, cnt = min(CB, a.ng - g0c);
    const long long sg = (long long)sl * a.ng + g0c;
    unsigned char *dst = ring + (size_t)s * SB;
    mbar_arrive_expect_tx(&full[s], (uint32_t)(NS * cnt * kSgBytes));
    bulk_g2s(dst, a.qw0 + sg * 4096, cnt * 4096, &full[s], pol);
    bulk_g2s(dst + (size_t)NS * CB * 4096, a.sb0 + sg * 512, cnt * 512, &full[s], pol);
    if constexpr (GATE_UP) {
      bulk_g2s(dst + (size_t)CB * 4096, a.qw1 + sg * 4096, cnt * 4096, &full[s], pol);
      bulk_g2s(dst + (size_t)NS * CB * 4096 + CB * 512, a.sb1 + sg * 512, cnt * 512, &full[s], pol);
    }
    if (++s == R) s = 0, par ^= 1u;
  }
  // the consumers wait for every chunk before they release it
  return true;
}

template <int CB, int GW, bool ONE, bool SF16, bool GATE_UP, bool PARTS>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(const GemvArgs a) {
  constexpr int WPT = gemv_wpt(GATE_UP), NC = kGemvConsumers;
  constexpr int NS = GATE_UP ? 2 : 1;
  constexpr int CPG = 8 / GW;  // B columns per window position
  constexpr int LPJ = 4 / GW;  // lanes (c) per window position
  extern __shared__ __align__(128) unsigned char smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int R = a.stages;
  constexpr size_t SB = (size_t)NS * CB * kSgBytes;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem);
  uint64_t *empty = full + kMaxStages;
  uint64_t *xready = empty + kMaxStages;  // the consumers have staged x
  // set by any warp of this CTA that gave up on a wait (read by the other
  // CTAs of a cluster before they exchange tile sums)
  volatile uint32_t *abort_word = reinterpret_cast<volatile uint32_t *>(smem + 240);
  unsigned char *ring = smem + 256;
  unsigned char *xt = ring + (size_t)R * SB;
  const int P = a.P, P8 = meta_cols(P);
  uint4 *xf = reinterpret_cast<uint4 *>(xt);
  uint4 *zero = reinterpret_cast<uint4 *>(xt + (size_t)a.xcap * P * 128);
  float4 *mx = reinterpret_cast<float4 *>(xt + (size_t)a.xcap * P * 128 + 128);
  // the warp pairs' slab-end exchange: [2 buffers][8 tiles][NS][32 lanes]
  float4 *pairbuf = reinterpret_cast<float4 *>(xt + xstage_bytes(a.xcap, P));

  // this CTA's run of chunks: an equal share of the flattened chunk space,
  // or (slab-split mode) part `part` of the chunks of slab blockIdx / j
  const bool clustered = a.cl_j > 1;
  const int part = clustered ? (int)(blockIdx.x % (unsigned)a.cl_j) : 0;
  int C0, C1;
  if (clustered) {
    const int slab = blockIdx.x / a.cl_j;
    C0 = slab * a.cps + part * a.cps / a.cl_j;
    C1 = slab * a.cps + (part + 1) * a.cps / a.cl_j;
  } else {
    C0 = run_begin(a, blockIdx.x);
    C1 = run_begin(a, blockIdx.x + 1);
  }
  const int nch = C1 - C0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < R; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kSlabTiles);  // one warp per tile consumes each stage
    }
    mbar_init(xready, 1);
    *abort_word = 0u;
  }
  fence_mbar_init();
  __syncthreads();
  pdl_launch_dependents();
  trace_stamp(a, kTrEntry);
  if (a.trace && blockIdx.x == 0 && threadIdx.x == 0) {
    a.trace[0] = 0x7468713474726163ull;  // record magic
    a.trace[1] = gridDim.x;
    a.trace[2] = (unsigned long long)a.out;
    a.trace[3] = (unsigned long long)a.in;
    a.trace[4] = (unsigned long long)(GATE_UP ? 1 : 0) | ((unsigned long long)a.cl_j << 8) |
                 ((unsigned long long)a.g_mode << 16) | ((unsigned long long)a.g_wait << 24);
    a.trace[5] = (unsigned long long)a.m;
    a.trace[6] = (unsigned long long)CB | ((unsigned long long)a.stages << 8);
    a.trace[7] = 0;
  }

  if (warp == NC) {
    // ---- producer: one elected lane streams the run -------------------------
    // (in slab-split mode the whole warp stays for the final cluster barrier)
    if (lane == 0 && !produce_run<CB, GATE_UP>(a, C0, nch, R, full, empty, xready, ring)) *abort_word = 1u;
    __syncwarp();
    if (clustered) {  // the consumers' two cluster barriers (below)
      cluster_sync_all();
      cluster_sync_all();
    }
    return;
  }
  // ---- consumers: warp tile + 8 half owns tile `tile` of the slab-groups
  // of the run's chunks n with n % 2 == half (one weight), or of every
  // chunk when half == 0 (gate/up: warps 8..15 only stage x)
  const int tile = warp % kSlabTiles, half = warp / kSlabTiles;
  pdl_wait();
  trace_stamp(a, kTrPdl);
  // a low-latency exchange's number: this rank's count + 1 (final once the
  // previous launch completed; the grid's last CTA raises the count)
  const uint32_t wseq = a.g_mode == 3 ? *reinterpret_cast<const volatile uint32_t *>(a.g_count) + 1u : 0u;
  if (a.g_wait) {  // x holds the peers' slices or partials: wait until they have landed
    if (threadIdx.x == 0) peer_wait(a.g_flags, a.g_count, a.g_world, a.g_rank, a.status);
    consumer_sync<NC>();
  }
  trace_stamp(a, kTrPeer);
  const int sl0 = C0 / a.cps, cg0 = C0 - sl0 * a.cps;
  const int gs = cg0 * CB;
  const int xcnt =
      min(a.ng, sgs_before(C1, a.cps, a.ng, CB) - sgs_before(C0, a.cps, a.ng, CB));
  stage_x<PARTS, NC>(a, gs, xcnt, xf, zero, mx);
  if (threadIdx.x == 0) mbar_arrive(xready);
  trace_stamp(a, kTrStaged);

  const int r = lane >> 2, c = lane & 3;
  const int jr = r / CPG, qr = r % CPG;  // this lane's B column: window position jr, column qr
  const int jc = c / LPJ, cp = c % LPJ;  // this lane's D columns 2c, 2c+1: position jc, pair cp
  const bool colv = 2 * cp < P;          // the pair holds a column in use
  const int xoff = qr * 8 + c;           // B entry of column qr within a slot
  bool bsel[GW];                         // B of window position j is this lane's column
#pragma unroll
  for (int j = 0; j < GW; ++j) bsel[j] = jr == j && qr < P;
  auto slot_of = [&](int g) { return g >= gs ? g - gs : g + a.ng - gs; };

  float lo[NS][4], hi[NS][4], y[NS][4];
#pragma unroll
  for (int s = 0; s < NS; ++s)
#pragma unroll
    for (int e = 0; e < 4; ++e) lo[s][e] = hi[s][e] = y[s][e] = 0.0f;
  bool seg_whole = cg0 == 0;  // the current slab segment began at the slab's start
  bool finished_any = false;

  // Group u of the chunk; `live`: this lane's B column holds it; `first`:
  // the window's first group, which starts both chains from zero.
  auto group = [&](const unsigned char *nib, const uint4 *xc, int u, bool live, bool first) {
    const uint4 *bp = live ? xc + u * P * 8 : zero + c;
    const uint4 xa = bp[0], xb = bp[4];
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      const uint4 w = *reinterpret_cast<const uint4 *>(nib + (size_t)(s * CB + u) * 4096 + tile * 512 + lane * 16);
      // k-step 2p rows r / r+8: bits 0..3 / 8..11 of each half (exact q);
      // k-step 2p+1: bits 4..7 / 12..15 (64 + q)
      uint32_t a00, a01, a02, a03, a10, a11, a12, a13, a20, a21, a22, a23, a30, a31, a32, a33;
      unpack_word(w.x, a00, a01, a10, a11);
      unpack_word(w.y, a02, a03, a12, a13);
      unpack_word(w.z, a20, a21, a30, a31);
      unpack_word(w.w, a22, a23, a32, a33);
      if (first) {
        mma_f16_16816_z(lo[s], a00, a01, a02, a03, xa.x, xa.y);
        mma_f16_16816_z(hi[s], a10, a11, a12, a13, xa.z, xa.w);
      } else {
        mma_f16_16816(lo[s], a00, a01, a02, a03, xa.x, xa.y);
        mma_f16_16816(hi[s], a10, a11, a12, a13, xa.z, xa.w);
      }
      mma_f16_16816(lo[s], a20, a21, a22, a23, xb.x, xb.y);
      mma_f16_16816(hi[s], a30, a31, a32, a33, xb.z, xb.w);
    }
  };
  // Epilogue of the window starting at chunk group w0: this lane's group is
  // w0 + jc; its scales come from the stage, its activation sums from mc.
  auto close_window = [&](const unsigned char *scl, const float4 *mc, int w0, bool valid) {
    if (!valid) return;
    const int gu = w0 + jc;
    const float4 m0 = mc[gu * P8];
    const float4 m1 = ONE ? m0 : mc[gu * P8 + 1];
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      const uint2 q = *reinterpret_cast<const uint2 *>(scl + (size_t)(s * CB + gu) * 512 + tile * 64 + r * 8);
      const float sr = sb_to_f32<SF16>(q.x & 0xffffu), br = sb_to_f32<SF16>(q.x >> 16);
      const float s8 = sb_to_f32<SF16>(q.y & 0xffffu), b8 = sb_to_f32<SF16>(q.y >> 16);
      y[s][0] = fmaf(sr * m0.y, (lo[s][0] + hi[s][0]) - m0.z, fmaf(br, m0.x, y[s][0]));
      y[s][2] = fmaf(s8 * m0.y, (lo[s][2] + hi[s][2]) - m0.z, fmaf(b8, m0.x, y[s][2]));
      if constexpr (!ONE) {
        y[s][1] = fmaf(sr * m1.y, (lo[s][1] + hi[s][1]) - m1.z, fmaf(br, m1.x, y[s][1]));
        y[s][3] = fmaf(s8 * m1.y, (lo[s][3] + hi[s][3]) - m1.z, fmaf(b8, m1.x, y[s][3]));
      }
    }
  };
  // The two warps of a tile hold sums over different chunks of the same
  // outputs: the second stores its sums to shared memory, the pair meets at
  // the tile's named barrier, the first adds them (always in this order).
  // Buffers alternate, so one barrier per exchange suffices: a warp writes
  // a buffer again only after passing the next exchange's barrier, which
  // the first warp reaches after reading it.
  int pair_phase = 0;
  auto pair_combine = [&]() {
    if constexpr (WPT == 2) {
      float4 *pb = pairbuf + (size_t)(pair_phase * kSlabTiles + tile) * NS * 32 + lane;
      if (half == 1) {
#pragma unroll
        for (int si = 0; si < NS; ++si) pb[si * 32] = make_float4(y[si][0], y[si][1], y[si][2], y[si][3]);
      }
      asm volatile("bar.sync %0, 64;\n" ::"r"(2 + tile) : "memory");
      if (half == 0) {
#pragma unroll
        for (int si = 0; si < NS; ++si) {
          const float4 v = pb[si * 32];
          y[si][0] += v.x, y[si][1] += v.y, y[si][2] += v.z, y[si][3] += v.w;
        }
      }
      pair_phase ^= 1;
    }
  };
  // lanes of one column pair but different window positions hold disjoint
  // groups of the same outputs: add them (every such lane gets the same sum)
  auto reduce_y = [&]() {
#pragma unroll
    for (int s = 0; s < NS; ++s)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v = y[s][e];
        if constexpr (GW == 4) {
          v += __shfl_xor_sync(0xffffffffu, v, 1);
          v += __shfl_xor_sync(0xffffffffu, v, 2);
        } else if constexpr (GW == 2) {
          v += __shfl_xor_sync(0xffffffffu, v, 2);
        }
        y[s][e] = v;
      }
  };

  // The run's partial slabs: its first (if it began inside a slab) and its
  // last (if it ended inside one).  This CTA's part of each is stored to the
  // workspace as soon as it is complete (side 0: the run's first segment,
  // side 1: its last) with plain stores; at the end of the run one
  // acquire-release increment per partial slab publishes them, and the CTA
  // whose increment completes the count adds every part in CTA order and
  // stores the tile.  Nothing waits; one release fence before the (relaxed)
  // increments and one acquire fence in the completing CTA order the parts.
  auto publish = [&](int side, const float (&v)[NS][4]) {
    float *gslot = a.part + (((size_t)blockIdx.x * 2 + side) * kSlabTiles + tile) * (NS * 128) + lane * 4;
#pragma unroll
    for (int si = 0; si < NS; ++si)
      *reinterpret_cast<float4 *>(gslot + si * 128) = make_float4(v[si][0], v[si][1], v[si][2], v[si][3]);
  };
  auto contributors = [&](int sl, int &clo, int &chi) {
    const int t0 = sl * a.cps;
    clo = run_of(a, t0);
    chi = run_of(a, t0 + a.cps - 1);
  };
  auto combine = [&](int sl) {
    int clo, chi;
    contributors(sl, clo, chi);
    const int t0 = sl * a.cps;
    float acc[NS][4];
#pragma unroll
    for (int si = 0; si < NS; ++si)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[si][e] = 0.0f;
    // up to kBatch contributors' parts are requested before any is added,
    // so the loads overlap; the sum still runs in CTA order
    constexpr int kBatch = 8 / NS;
    for (int q0 = clo; q0 <= chi; q0 += kBatch) {
      float4 v[kBatch][NS];
#pragma unroll
      for (int i = 0; i < kBatch; ++i) {
        const int q = q0 + i;
        if (q > chi) break;
        const int qs = (q == clo && run_begin(a, q) < t0) ? 1 : 0;
        const float *src = a.part + (((size_t)q * 2 + qs) * kSlabTiles + tile) * (NS * 128) + lane * 4;
#pragma unroll
        for (int si = 0; si < NS; ++si) v[i][si] = ld_relaxed_f4(src + si * 128);
      }
#pragma unroll
      for (int i = 0; i < kBatch; ++i) {
        if (q0 + i > chi) break;
#pragma unroll
        for (int si = 0; si < NS; ++si)
          acc[si][0] += v[i][si].x, acc[si][1] += v[i][si].y, acc[si][2] += v[i][si].z, acc[si][3] += v[i][si].w;
      }
    }
    if (lane == 0) a.count[(size_t)sl * kSlabTiles + tile] = 0;  // ready for the next call
    store_tile<GW, GATE_UP>(a, sl * kSlabTiles + tile, lane, acc[0], acc[NS - 1], wseq);
  };
  int first_slab = -1;
  int sl = sl0, cg = cg0 - 1, s = R - 1;
  uint32_t par = 1;  // (stage, parity) of chunk n, kept incrementally
  // A warp whose wait times out stops computing and releasing stages; the
  // producer then times out on the stage's release and stops.  Outputs of
  // the call are undefined and the status word says so.
  bool aborted = false;
  for (int n = 0; n < nch; ++n) {
    if (++cg == a.cps) cg = 0, ++sl;
    if (++s == R) s = 0, par ^= 1u;
    if (WPT == 1 ? half == 0 : (n & 1) == half) {  // this warp's chunk
    if (!aborted && !mbar_wait_bounded(&full[s], par, kWaitLimitNs)) {
      raise_status(a.status, kStatusTimeout);
      aborted = true;
      *abort_word = 1u;
    }
    if (n == 0) trace_stamp(a, kTrFirst);
    const int g0c = cg * CB, cnt = min(CB, a.ng - g0c);
    const unsigned char *nib = ring + (size_t)s * SB;
    const unsigned char *scl = nib + (size_t)NS * CB * 4096;
    // the chunk's groups are consecutive slots (gs is chunk-aligned)
    const int slot0 = slot_of(g0c);
    const uint4 *xc = xf + (size_t)slot0 * P * 8 + xoff;
    const float4 *mc = mx + (size_t)slot0 * P8 + 2 * cp;
    if (aborted) {
    } else if (cnt == CB) {
#pragma unroll
      for (int u = 0; u < CB; ++u) {
        group(nib, xc, u, bsel[u % GW], u % GW == 0);
        if (u % GW == GW - 1) close_window(scl, mc, u - (GW - 1), colv);
      }
    } else {  // the slab's last chunk when ng is not a multiple of CB
      for (int u = 0; u < cnt; ++u) {
        const int j = u % GW;
        group(nib, xc, u, jr == j && qr < P, j == 0);
        if (j == GW - 1 || u == cnt - 1) close_window(scl, mc, u - j, colv && u - j + jc < cnt);
      }
    }
    __syncwarp();
    if (lane == 0 && !aborted) mbar_arrive(&empty[s]);
    }  // this warp's chunk
    if (!clustered && cg == a.cps - 1) {  // slab end
      pair_combine();
      reduce_y();
      if (aborted || half != 0) {
      } else if (seg_whole) {
        store_tile<GW, GATE_UP>(a, sl * kSlabTiles + tile, lane, y[0], y[NS - 1], wseq);
      } else {  // the run's first segment, partial
        publish(0, y);
      }
      if (!seg_whole) first_slab = sl;
#pragma unroll
      for (int si = 0; si < NS; ++si)
#pragma unroll
        for (int e = 0; e < 4; ++e) y[si][e] = 0.0f;
      seg_whole = true;
      finished_any = true;
    }
  }

  trace_stamp(a, kTrStreamed);
  if (clustered) {
    // Slab-split mode: this CTA holds part `part` of one slab.  Once every
    // CTA of the cluster is past its stream (barrier 1) the leader's ring is
    // free; the other parts go there through DSMEM (barrier 2), and the
    // leader adds them in part order and stores the tile.
    // If any CTA of the cluster gave up on a wait (its copies may still be
    // landing in its ring), nobody writes into the leader's ring and nothing
    // is stored; every CTA still passes both barriers.
    pair_combine();
    reduce_y();
    float4 *xb = reinterpret_cast<float4 *>(ring);
    cluster_sync_all();
    uint32_t gave_up = 0;
    if (lane == 0)
      for (int pp = 0; pp < a.cl_j; ++pp)
        gave_up |= ld_cluster_u32(cluster_map(smem_addr(const_cast<uint32_t *>(abort_word)), (uint32_t)pp));
    gave_up = __shfl_sync(0xffffffffu, gave_up, 0);
    if (part > 0 && !gave_up && half == 0) {
#pragma unroll
      for (int si = 0; si < NS; ++si) {
        const uint32_t at = smem_addr(xb + (((size_t)part * kSlabTiles + tile) * NS + si) * 32 + lane);
        st_cluster_f4(cluster_map(at, 0), make_float4(y[si][0], y[si][1], y[si][2], y[si][3]));
      }
    }
    cluster_sync_all();
    if (part == 0 && !gave_up && half == 0) {
      for (int pp = 1; pp < a.cl_j; ++pp)
#pragma unroll
        for (int si = 0; si < NS; ++si) {
          const float4 v = xb[(((size_t)pp * kSlabTiles + tile) * NS + si) * 32 + lane];
          y[si][0] += v.x, y[si][1] += v.y, y[si][2] += v.z, y[si][3] += v.w;
        }
      store_tile<GW, GATE_UP>(a, (C0 / a.cps) * kSlabTiles + tile, lane, y[0], y[NS - 1], wseq);
    }
    trace_stamp(a, kTrStored);
    if (a.g_mode) peer_signal<NC>(a);
    trace_stamp(a, kTrDone);
    return;
  }

  int last_slab = -1;
  if (nch > 0 && cg != a.cps - 1) {  // the run ended inside a slab
    pair_combine();
    reduce_y();
    if (!aborted && half == 0) publish(finished_any ? 1 : 0, y);
    last_slab = sl;
  }
  if (!aborted && half == 0 && (first_slab >= 0 || last_slab >= 0)) {
    // the lanes' stores above happen before lane 0's release fence; one
    // fence covers both increments, which are then in flight together
    __syncwarp();
    uint32_t done = 0;  // bit 0: first slab complete, bit 1: last slab complete
    if (lane == 0) {
      uint32_t o0 = 0, o1 = 0;
      int clo, chi;
      fence_acq_rel_gpu();
      if (first_slab >= 0) o0 = atom_add_relaxed(&a.count[(size_t)first_slab * kSlabTiles + tile], 1u);
      if (last_slab >= 0) o1 = atom_add_relaxed(&a.count[(size_t)last_slab * kSlabTiles + tile], 1u);
      if (first_slab >= 0) {
        contributors(first_slab, clo, chi);
        if (o0 + 1 == (uint32_t)(chi - clo + 1)) done |= 1u;
      }
      if (last_slab >= 0) {
        contributors(last_slab, clo, chi);
        if (o1 + 1 == (uint32_t)(chi - clo + 1)) done |= 2u;
      }
      if (done) fence_acq_rel_gpu();  // acquire: every other part is visible
    }
    done = __shfl_sync(0xffffffffu, done, 0);
    // lane 0's acquire happens before the other lanes' loads
    __syncwarp();
    if (done & 1u) combine(first_slab);
    if (done & 2u) combine(last_slab);
  }
  trace_stamp(a, kTrStored);
  if (a.g_mode) peer_signal<NC>(a);  // every consumer warp gets here
  trace_stamp(a, kTrDone);
}

// ---------------------------------------------------------------------------
// Chains: dependent projections in one persistent launch (thq4_linear_chain)
// ---------------------------------------------------------------------------
// Within one launch of a single projection the weight stream stops at every
// launch boundary: a launch's CTAs start only as the predecessor's leave the
// SMs, then wait for the predecessor's output before staging x.  A chain
// runs ops 0..n-1 in one cooperative launch (one CTA per SM): the producer
// warp streams the weights of op after op into the ring without ever
// waiting for activations (weights do not depend on them), while the
// consumer warps finish op p, meet the other CTAs at a grid barrier (op p's
// outputs complete and visible), stage op p + 1's x and go on with stages
// that are already in shared memory.  Every stage holds 8 slab-groups of
// one weight or 4 of gate and 4 of up (the same 36,864 bytes), so ops of
// either kind share one ring.  Each op's slab-groups are split over the CTAs
// as in the single launch (whole slabs per CTA where they fill >= 85% of
// the SMs, else equal runs of chunks whose split slabs finish by the last
// arriver); CTAs without a run in an op only pass its barrier, while their
// producer already streams the next op.
constexpr int kMaxChainOps = 112;
constexpr int kChainStageBytes = 8 * kSgBytes;

struct ChainOp {
  const uint8_t *qw0, *sb0, *qw1, *sb1;
  const void *x;
  void *y;
  int out, in, ng, cps;
  int chunks, run_base, run_rem, active;  // CTAs 0 .. active-1 hold a run of the op
  int gate_up, yf32;
};

struct ChainArgs {
  uint32_t *status;
  float *part;     // split-K partials, as GemvArgs::part
  uint32_t *count; // arrivals per (slab, tile), as GemvArgs::count
  uint32_t *bar;   // [0] barrier arrivals, [1] exits (zero between launches)
  int n, m, P, xf32, stages, xcap;
  // phase trace (thq4_debug_set_trace; nullptr = off): 8 header words, then
  // per (op, CTA) 4 %globaltimer stamps: op begun (barrier passed), x
  // staged, stream consumed, outputs stored
  unsigned long long *trace;
  ChainOp ops[kMaxChainOps];
};

// One op of a chain through the members the GEMV helpers read (no exchange).
// The consumers keep the current op's view in shared memory: held in
// registers across the chunk loop it would crowd out the loop's own.
struct OpView {
  const void *x;
  void *y;
  int m, in, ng, out, P, xf32, yf32;
  int run_base, run_rem, cps, active, gate_up, index;
  int g_mode, g_world, g_rank, g_rows, g_off, g_stride;
  long long g_slot;
  uint16_t *const *g_dst;
  int xparts;
  long long xslot;
  const float *xsum;
};
constexpr int kViewOffset = 256;  // the view's place in shared memory, after the barriers
static_assert(sizeof(OpView) <= 256, "the op view fits its slot");

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void chain_stamp(const ChainArgs &a, int p, int i) {
  if (a.trace && threadIdx.x == 0) a.trace[8 + ((size_t)p * gridDim.x + blockIdx.x) * 4 + i] = global_timer_ns();
}

// Thread 0 writes op p's view; the consumers see it after their barrier.
__device__ __forceinline__ void chain_set_view(const ChainArgs &a, int p, OpView *vs) {
  if (threadIdx.x == 0) {
    const ChainOp &op = a.ops[p];
    OpView v;
    v.x = op.x;
    v.y = op.y;
    v.m = a.m;
    v.in = op.in;
    v.ng = op.ng;
    v.out = op.out;
    v.P = a.P;
    v.xf32 = a.xf32;
    v.yf32 = op.yf32;
    v.run_base = op.run_base;
    v.run_rem = op.run_rem;
    v.cps = op.cps;
    v.active = op.active;
    v.gate_up = op.gate_up;
    v.index = p;
    v.g_mode = v.g_world = v.g_rank = v.g_rows = v.g_off = v.g_stride = 0;
    v.g_slot = 0;
    v.g_dst = nullptr;
    v.xparts = 0;
    v.xslot = 0;
    v.xsum = nullptr;
    *vs = v;
  }
  consumer_sync();
}

// The producer lane's stream of one op: its run's chunks into the ring, whose
// cursor (stage s, parity par, chunks issued so far) carries over between
// ops.  False after a timeout (the copies in flight have been waited for).
template <int CB, bool GATE_UP>
__device__ __forceinline__ bool chain_produce_op(const ChainOp &op, int C0, int nch, int R, uint64_t *full,
                                                uint64_t *empty, unsigned char *ring, uint32_t *status, int &s,
                                                uint32_t &par, long long &issued, uint64_t pol) {
  constexpr int NS = GATE_UP ? 2 : 1;
  static_assert(NS * CB * kSgBytes == kChainStageBytes, "chain stages are uniform");
  int sl = C0 / op.cps, cg = C0 - sl * op.cps;
  for (int n = 0; n < nch; ++n, ++cg) {
    if (cg == op.cps) cg = 0, ++sl;
    if (issued >= R && !mbar_wait_bounded(&empty[s], par ^ 1u, kWaitLimitNs)) {
      raise_status(status, kStatusTimeout);
      for (long long k = issued - R; k < issued; ++k)
        (void)mbar_wait_bounded(&full[k % R], (uint32_t)((k / R) & 1), kWaitLimitNs);
      return false;
    }
    const int g0c = cg * CB, cnt = min(CB, op.ng - g0c);
    const long long sg = (long long)sl * op.ng + g0c;
    unsigned char *dst = ring + (size_t)s * kChainStageBytes;
    mbar_arrive_expect_tx(&full[s], (uint32_t)(NS * cnt * kSgBytes));
    bulk_g2s(dst, op.qw0 + sg * 4096, cnt * 4096, &full[s], pol);
    bulk_g2s(dst + (size_t)NS * CB * 4096, op.sb0 + sg * 512, cnt * 512, &full[s], pol);
    if constexpr (GATE_UP) {
      bulk_g2s(dst + (size_t)CB * 4096, op.qw1 + sg * 4096, cnt * 4096, &full[s], pol);
      bulk_g2s(dst + (size_t)NS * CB * 4096 + CB * 512, op.sb1 + sg * 512, cnt * 512, &full[s], pol);
    }
    ++issued;
    if (++s == R) s = 0, par ^= 1u;
  }
  return true;
}

// Every CTA's consumers are done with op p - 1 (outputs stored, split slabs
// finished): one arrival per CTA on the launch's counter, then a bounded wait
// for all of them.  A timeout marks the CTA aborted (status kStatusTimeout).
__device__ __forceinline__ void chain_barrier(const ChainArgs &a, int p, volatile uint32_t *abort_word) {
  consumer_sync();
  if (threadIdx.x == 0) {
    fence_acq_rel_gpu();  // this CTA's outputs (ordered before by the bar.sync) before its arrival
    atom_add_relaxed(a.bar, 1u);
    const uint32_t target = (uint32_t)p * gridDim.x;
    const uint64_t t0 = global_timer_ns();
    while ((int32_t)(ld_acquire_gpu(a.bar) - target) < 0) {
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        raise_status(a.status, kStatusTimeout);
        *abort_word = 1u;
        break;
      }
    }
  }
  consumer_sync();
}

// The consumers' place in the ring (the stage of the last chunk taken and its
// parity) and whether this warp gave up on a wait, carried from op to op.
struct RingCursor {
  int s;
  uint32_t par;
  int aborted;
};

// The consumers' share of one op: stage its x, consume the run's chunks from
// the ring, store whole slabs and finish split ones by the last arriver --
// the same arithmetic as gemv_kernel.  Not inlined: each kind of op (one
// weight, gate/up) gets the kernel's register budget for its own loop.
template <int CB, int GW, bool ONE, bool SF16, bool GATE_UP>
__device__ __noinline__ RingCursor chain_consume_op(const ChainArgs &a, const OpView &v, int R, uint64_t *full,
                                                    uint64_t *empty, unsigned char *ring, uint4 *xf, uint4 *zero,
                                                    float4 *mx, volatile uint32_t *abort_word, RingCursor cur) {
  constexpr int NS = GATE_UP ? 2 : 1;
  constexpr int CPG = 8 / GW;
  constexpr int LPJ = 4 / GW;
  const int lane = threadIdx.x & 31, tile = threadIdx.x >> 5;
  chain_stamp(a, v.index, 0);
  if ((int)blockIdx.x >= v.active) return cur;  // no run in this op (every consumer warp alike)
  int s = cur.s;
  uint32_t par = cur.par;
  bool aborted = cur.aborted != 0;
  const int C0 = run_begin(v, blockIdx.x), C1 = run_begin(v, blockIdx.x + 1);
  const int nch = C1 - C0;
  const int P = a.P, P8 = meta_cols(P);
  const int sl0 = C0 / v.cps, cg0 = C0 - sl0 * v.cps;
  const int gs = cg0 * CB;
  const int xcnt = min(v.ng, sgs_before(C1, v.cps, v.ng, CB) - sgs_before(C0, v.cps, v.ng, CB));
  stage_x<false>(v, gs, xcnt, xf, zero, mx);
  chain_stamp(a, v.index, 1);

  const int r = lane >> 2, c = lane & 3;
  const int jr = r / CPG, qr = r % CPG;
  const int jc = c / LPJ, cp = c % LPJ;
  const bool colv = 2 * cp < P;
  const int xoff = qr * 8 + c;
  bool bsel[GW];
#pragma unroll
  for (int j = 0; j < GW; ++j) bsel[j] = jr == j && qr < P;
  auto slot_of = [&](int g) { return g >= gs ? g - gs : g + v.ng - gs; };

  float lo[NS][4], hi[NS][4], y[NS][4];
#pragma unroll
  for (int si = 0; si < NS; ++si)
#pragma unroll
    for (int e = 0; e < 4; ++e) lo[si][e] = hi[si][e] = y[si][e] = 0.0f;
  bool seg_whole = cg0 == 0;
  bool finished_any = false;

  auto group = [&](const unsigned char *nib, const uint4 *xc, int u, bool live, bool first) {
    const uint4 *bp = live ? xc + u * P * 8 : zero + c;
    const uint4 xa = bp[0], xb = bp[4];
#pragma unroll
    for (int si = 0; si < NS; ++si) {
      const uint4 w = *reinterpret_cast<const uint4 *>(nib + (size_t)(si * CB + u) * 4096 + tile * 512 + lane * 16);
      uint32_t a00, a01, a02, a03, a10, a11, a12, a13, a20, a21, a22, a23, a30, a31, a32, a33;
      unpack_word(w.x, a00, a01, a10, a11);
      unpack_word(w.y, a02, a03, a12, a13);
      unpack_word(w.z, a20, a21, a30, a31);
      unpack_word(w.w, a22, a23, a32, a33);
      if (first) {
        mma_f16_16816_z(lo[si], a00, a01, a02, a03, xa.x, xa.y);
        mma_f16_16816_z(hi[si], a10, a11, a12, a13, xa.z, xa.w);
      } else {
        mma_f16_16816(lo[si], a00, a01, a02, a03, xa.x, xa.y);
        mma_f16_16816(hi[si], a10, a11, a12, a13, xa.z, xa.w);
      }
      mma_f16_16816(lo[si], a20, a21, a22, a23, xb.x, xb.y);
      mma_f16_16816(hi[si], a30, a31, a32, a33, xb.z, xb.w);
    }
  };
  auto close_window = [&](const unsigned char *scl, const float4 *mc, int w0, bool valid) {
    if (!valid) return;
    const int gu = w0 + jc;
    const float4 m0 = mc[gu * P8];
    const float4 m1 = ONE ? m0 : mc[gu * P8 + 1];
#pragma unroll
    for (int si = 0; si < NS; ++si) {
      const uint2 q = *reinterpret_cast<const uint2 *>(scl + (size_t)(si * CB + gu) * 512 + tile * 64 + r * 8);
      const float sr = sb_to_f32<SF16>(q.x & 0xffffu), br = sb_to_f32<SF16>(q.x >> 16);
      const float s8 = sb_to_f32<SF16>(q.y & 0xffffu), b8 = sb_to_f32<SF16>(q.y >> 16);
      y[si][0] = fmaf(sr * m0.y, (lo[si][0] + hi[si][0]) - m0.z, fmaf(br, m0.x, y[si][0]));
      y[si][2] = fmaf(s8 * m0.y, (lo[si][2] + hi[si][2]) - m0.z, fmaf(b8, m0.x, y[si][2]));
      if constexpr (!ONE) {
        y[si][1] = fmaf(sr * m1.y, (lo[si][1] + hi[si][1]) - m1.z, fmaf(br, m1.x, y[si][1]));
        y[si][3] = fmaf(s8 * m1.y, (lo[si][3] + hi[si][3]) - m1.z, fmaf(b8, m1.x, y[si][3]));
      }
    }
  };
  auto reduce_y = [&]() {
#pragma unroll
    for (int si = 0; si < NS; ++si)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float t = y[si][e];
        if constexpr (GW == 4) {
          t += __shfl_xor_sync(0xffffffffu, t, 1);
          t += __shfl_xor_sync(0xffffffffu, t, 2);
        } else if constexpr (GW == 2) {
          t += __shfl_xor_sync(0xffffffffu, t, 2);
        }
        y[si][e] = t;
      }
  };
  auto publish = [&](int side, const float (&pv)[NS][4]) {
    float *gslot = a.part + (((size_t)blockIdx.x * 2 + side) * kSlabTiles + tile) * (NS * 128) + lane * 4;
#pragma unroll
    for (int si = 0; si < NS; ++si)
      *reinterpret_cast<float4 *>(gslot + si * 128) = make_float4(pv[si][0], pv[si][1], pv[si][2], pv[si][3]);
  };
  auto contributors = [&](int sl, int &clo, int &chi) {
    const int t0 = sl * v.cps;
    clo = run_of(v, t0);
    chi = run_of(v, t0 + v.cps - 1);
  };
  auto combine = [&](int sl) {
    int clo, chi;
    contributors(sl, clo, chi);
    const int t0 = sl * v.cps;
    float acc[NS][4];
#pragma unroll
    for (int si = 0; si < NS; ++si)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[si][e] = 0.0f;
    constexpr int kBatch = 8 / NS;
    for (int q0 = clo; q0 <= chi; q0 += kBatch) {
      float4 pv[kBatch][NS];
#pragma unroll
      for (int i = 0; i < kBatch; ++i) {
        const int q = q0 + i;
        if (q > chi) break;
        const int qs = (q == clo && run_begin(v, q) < t0) ? 1 : 0;
        const float *src = a.part + (((size_t)q * 2 + qs) * kSlabTiles + tile) * (NS * 128) + lane * 4;
#pragma unroll
        for (int si = 0; si < NS; ++si) pv[i][si] = ld_relaxed_f4(src + si * 128);
      }
#pragma unroll
      for (int i = 0; i < kBatch; ++i) {
        if (q0 + i > chi) break;
#pragma unroll
        for (int si = 0; si < NS; ++si)
          acc[si][0] += pv[i][si].x, acc[si][1] += pv[i][si].y, acc[si][2] += pv[i][si].z, acc[si][3] += pv[i][si].w;
      }
    }
    if (lane == 0) a.count[(size_t)sl * kSlabTiles + tile] = 0;
    store_tile<GW, GATE_UP>(v, sl * kSlabTiles + tile, lane, acc[0], acc[NS - 1]);
  };

  int first_slab = -1;
  int sl = sl0, cg = cg0 - 1;
  for (int n = 0; n < nch; ++n) {
    if (++cg == v.cps) cg = 0, ++sl;
    if (++s == R) s = 0, par ^= 1u;
    if (!aborted && !mbar_wait_bounded(&full[s], par, kWaitLimitNs)) {
      raise_status(a.status, kStatusTimeout);
      aborted = true;
      *abort_word = 1u;
    }
    const int g0c = cg * CB, cnt = min(CB, v.ng - g0c);
    const unsigned char *nib = ring + (size_t)s * kChainStageBytes;
    const unsigned char *scl = nib + (size_t)NS * CB * 4096;
    const int slot0 = slot_of(g0c);
    const uint4 *xc = xf + (size_t)slot0 * P * 8 + xoff;
    const float4 *mc = mx + (size_t)slot0 * P8 + 2 * cp;
    if (aborted) {
    } else if (cnt == CB) {
#pragma unroll
      for (int u = 0; u < CB; ++u) {
        group(nib, xc, u, bsel[u % GW], u % GW == 0);
        if (u % GW == GW - 1) close_window(scl, mc, u - (GW - 1), colv);
      }
    } else {
      for (int u = 0; u < cnt; ++u) {
        const int j = u % GW;
        group(nib, xc, u, jr == j && qr < P, j == 0);
        if (j == GW - 1 || u == cnt - 1) close_window(scl, mc, u - j, colv && u - j + jc < cnt);
      }
    }
    __syncwarp();
    if (lane == 0 && !aborted) mbar_arrive(&empty[s]);
    if (cg == v.cps - 1) {
      reduce_y();
      if (aborted) {
      } else if (seg_whole) {
        store_tile<GW, GATE_UP>(v, sl * kSlabTiles + tile, lane, y[0], y[NS - 1]);
      } else {
        publish(0, y);
      }
      if (!seg_whole) first_slab = sl;
#pragma unroll
      for (int si = 0; si < NS; ++si)
#pragma unroll
        for (int e = 0; e < 4; ++e) y[si][e] = 0.0f;
      seg_whole = true;
      finished_any = true;
    }
  }
  chain_stamp(a, v.index, 2);
  int last_slab = -1;
  if (nch > 0 && cg != v.cps - 1) {
    reduce_y();
    if (!aborted) publish(finished_any ? 1 : 0, y);
    last_slab = sl;
  }
  if (!aborted && (first_slab >= 0 || last_slab >= 0)) {
    __syncwarp();
    uint32_t done = 0;
    if (lane == 0) {
      uint32_t o0 = 0, o1 = 0;
      int clo, chi;
      fence_acq_rel_gpu();
      if (first_slab >= 0) o0 = atom_add_relaxed(&a.count[(size_t)first_slab * kSlabTiles + tile], 1u);
      if (last_slab >= 0) o1 = atom_add_relaxed(&a.count[(size_t)last_slab * kSlabTiles + tile], 1u);
      if (first_slab >= 0) {
        contributors(first_slab, clo, chi);
        if (o0 + 1 == (uint32_t)(chi - clo + 1)) done |= 1u;
      }
      if (last_slab >= 0) {
        contributors(last_slab, clo, chi);
        if (o1 + 1 == (uint32_t)(chi - clo + 1)) done |= 2u;
      }
      if (done) fence_acq_rel_gpu();
    }
    done = __shfl_sync(0xffffffffu, done, 0);
    __syncwarp();
    if (done & 1u) combine(first_slab);
    if (done & 2u) combine(last_slab);
  }
  chain_stamp(a, v.index, 3);
  return RingCursor{s, par, aborted ? 1 : 0};
}

template <int GW, bool ONE, bool SF16>
__global__ void __launch_bounds__(kThreads, 1) chain_kernel(const __grid_constant__ ChainArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int R = a.stages;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem);
  uint64_t *empty = full + kMaxStages;
  volatile uint32_t *abort_word = reinterpret_cast<volatile uint32_t *>(smem + 240);
  OpView *view = reinterpret_cast<OpView *>(smem + kViewOffset);
  unsigned char *ring = smem + 512;
  unsigned char *xt = ring + (size_t)R * kChainStageBytes;
  uint4 *xf = reinterpret_cast<uint4 *>(xt);
  uint4 *zero = reinterpret_cast<uint4 *>(xt + (size_t)a.xcap * a.P * 128);
  float4 *mx = reinterpret_cast<float4 *>(xt + (size_t)a.xcap * a.P * 128 + 128);
  if (threadIdx.x == 0) {
    for (int s = 0; s < R; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumers);
    }
    *abort_word = 0u;
  }
  fence_mbar_init();
  __syncthreads();

  if (warp == kConsumers) {
    // ---- producer: every op's run, back to back ----------------------------
    if (lane == 0) {
      const uint64_t pol = evict_first_policy();
      int s = 0;
      uint32_t par = 0;
      long long issued = 0;
      for (int p = 0; p < a.n; ++p) {
        const ChainOp &op = a.ops[p];
        if ((int)blockIdx.x >= op.active) continue;
        const int C0 = blockIdx.x * op.run_base + min((int)blockIdx.x, op.run_rem);
        const int C1 = C0 + op.run_base + ((int)blockIdx.x < op.run_rem ? 1 : 0);
        const bool ok = op.gate_up
                            ? chain_produce_op<4, true>(op, C0, C1 - C0, R, full, empty, ring, a.status, s, par,
                                                        issued, pol)
                            : chain_produce_op<8, false>(op, C0, C1 - C0, R, full, empty, ring, a.status, s, par,
                                                         issued, pol);
        if (!ok) {
          *abort_word = 1u;
          break;
        }
      }
    }
    return;
  }
  // ---- consumers ------------------------------------------------------------
  if (a.trace && blockIdx.x == 0 && threadIdx.x == 0) {
    a.trace[0] = 0x7468713463686e21ull;  // chain record magic
    a.trace[1] = gridDim.x;
    a.trace[2] = (unsigned long long)a.n;
    a.trace[3] = (unsigned long long)a.stages;
    for (int i = 4; i < 8; ++i) a.trace[i] = 0;
  }
  RingCursor cur{R - 1, 1u, 0};
  for (int p = 0; p < a.n; ++p) {
    if (p > 0) {
      chain_barrier(a, p, abort_word);
      if (*abort_word != 0u) cur.aborted = 1;
    }
    chain_set_view(a, p, view);
    cur = view->gate_up
              ? chain_consume_op<4, GW, ONE, SF16, true>(a, *view, R, full, empty, ring, xf, zero, mx, abort_word, cur)
              : chain_consume_op<8, GW, ONE, SF16, false>(a, *view, R, full, empty, ring, xf, zero, mx, abort_word,
                                                         cur);
  }
  // the last CTA out leaves the barrier words zero for the next launch
  consumer_sync();
  if (threadIdx.x == 0) {
    fence_acq_rel_gpu();
    if (atom_add_acq_rel(a.bar + 1, 1u) + 1u == gridDim.x) {
      a.bar[0] = 0u;
      a.bar[1] = 0u;
    }
  }
}

template <int CB, int GW, bool ONE, bool SF16, bool GATE_UP, bool PARTS>
cudaError_t launch_one(const GemvArgs &a, int grid, size_t smem, cudaStream_t stream) {
  auto *k = &gemv_kernel<CB, GW, ONE, SF16, GATE_UP, PARTS>;
  static DeviceOnce once;
  cudaError_t e = once.run([&] {
    return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvMaxSmem);
  });
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = gemv_pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (a.cl_j > 1) {  // the j CTAs of a slab form one cluster
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)a.cl_j;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
    // all clusters must be resident at once (one wave): how many fit depends
    // on how the SMs group into GPCs; asked once per (device, instance,
    // size, smem).  One word per device holds the question and its answer,
    // so concurrent callers never pair one footprint's answer with another's
    // key; a failed query is not remembered.
    static std::atomic<uint64_t> cached[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    const uint64_t want = ((uint64_t)smem << 8) | (uint64_t)a.cl_j;  // < 2^40
    int n = 0;
    const uint64_t c = cached[dev].load(std::memory_order_relaxed);
    if (c != 0 && (c >> 20) == want) {
      n = (int)(c & 0xFFFFFu);
    } else if (cudaOccupancyMaxActiveClusters(&n, k, &cfg) == cudaSuccess) {
      cached[dev].store((want << 20) | (uint64_t)std::min(std::max(n, 0), 0xFFFFF), std::memory_order_relaxed);
    } else {
      (void)cudaGetLastError();
      n = 0;
    }
    if (n * a.cl_j < grid) return cudaErrorCooperativeLaunchTooLarge;  // the caller re-plans without clusters
  }
  return cudaLaunchKernelEx(&cfg, k, a);
}

template <int CB, bool SF16, bool GATE_UP, bool PARTS>
cudaError_t dispatch_gw_t(const GemvArgs &a, int gw, int grid, size_t smem, cudaStream_t s) {
  if (gw == 4)
    return a.P == 1 ? launch_one<CB, 4, true, SF16, GATE_UP, PARTS>(a, grid, smem, s)
                    : launch_one<CB, 4, false, SF16, GATE_UP, PARTS>(a, grid, smem, s);
  if (gw == 2) return launch_one<CB, 2, false, SF16, GATE_UP, PARTS>(a, grid, smem, s);
  return launch_one<CB, 1, false, SF16, GATE_UP, PARTS>(a, grid, smem, s);
}

// x partials (the end of a fused all-reduce) have their own instances, only
// for the default 8-group chunks: the extra staging code would otherwise
// weigh on the register allocation of every kernel.
template <int CB, bool SF16, bool GATE_UP>
cudaError_t dispatch_gw(const GemvArgs &a, int gw, int grid, size_t smem, cudaStream_t s) {
  if (a.xparts) {
    if constexpr (CB == 8) return dispatch_gw_t<CB, SF16, GATE_UP, true>(a, gw, grid, smem, s);
    return cudaErrorInvalidValue;
  }
  return dispatch_gw_t<CB, SF16, GATE_UP, false>(a, gw, grid, smem, s);
}

template <bool SF16>
cudaError_t dispatch(const GemvArgs &a, bool gate_up, int cb, int gw, int grid, size_t smem, cudaStream_t s) {
  if (gate_up)
    return cb == 8 ? dispatch_gw<8, SF16, true>(a, gw, grid, smem, s) : dispatch_gw<4, SF16, true>(a, gw, grid, smem, s);
  return cb == 8 ? dispatch_gw<8, SF16, false>(a, gw, grid, smem, s)
                 : dispatch_gw<4, SF16, false>(a, gw, grid, smem, s);
}

int window_groups(int P) { return P <= 2 ? 4 : (P <= 4 ? 2 : 1); }

}  // namespace

// Clusters of j CTAs (one CTA per SM, the GEMV's footprint) that can be
// resident at once: it depends on how the SMs group into GPCs.  Asked once
// per device and j.
int cluster_capacity(int j) {
  static std::mutex mu;
  static int cache[64][9];
  int dev = 0;
  if (j < 2 || j > 8 || cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev][j]) return cache[dev][j] - 1;
  auto *k = &gemv_kernel<8, 4, true, true, false, false>;
  int n = 0;
  bool ok = false;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvMaxSmem) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(j * 64);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = 150 * 1024;  // any footprint that allows one CTA per SM
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)j;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    ok = cudaOccupancyMaxActiveClusters(&n, k, &cfg) == cudaSuccess;
  }
  (void)cudaGetLastError();
  if (!ok) return 0;  // not remembered: asked again next time
  cache[dev][j] = n + 1;
  return n;
}

size_t gemv_workspace_bytes(int rows) {
  // one partial per CTA side, sized for gate and up (room for two CTAs per
  // SM; the grid is at most one per SM), then one counter per (slab, tile)
  const size_t ctas = (size_t)device_sm_count() * 2;
  return ctas * 2 * side_floats(true) * sizeof(float) +
         ((size_t)row_slabs(rows) * kSlabTiles * 4 + 255) / 256 * 256;
}

GemvPlan gemv_plan(int out, int in, int m, bool x_f32, bool gate_up) {
  return gemv_plan_for(out, in, m, x_f32, gate_up, device_sm_count(), cluster_capacity);
}

GemvPlan gemv_plan_for(int out, int in, int m, bool x_f32, bool gate_up, int sms, const ClusterCapacity &capacity) {
  GemvPlan p{};
  p.ok = false;
  const int ng = in / kGroup;
  const GemvCfg cfg = gemv_cfg_override();
  const int cb = cfg.warps > 0 ? cfg.warps : 8;
  const int cps = (ng + cb - 1) / cb;
  const long long chunks = (long long)row_slabs(out) * cps;
  // run arithmetic on the device is 32-bit
  if ((long long)row_slabs(out) * ng >= (1ll << 31)) return p;
  int per = x_f32 ? 4 : 8;  // tokens per launch: 8 B columns, two per f32 token
  if (per > m) per = m;
  for (;;) {
    const int P = x_f32 ? 2 * per : per;
    // one CTA per SM with a deep ring of 8-group chunks measured best for
    // every decode shape
    {
      // one CTA per SM (a CTA holds 17 warps and most of the shared memory)
      long long grid = cfg.grid > 0 ? std::min(cfg.grid, 2 * sms) : (long long)sms;
      // Whole slabs per CTA when that still fills >= 85% of the SMs: no
      // slab is split, so there is no split-K fix-up at the end of the run
      // (the fused gate/up of a 17408-wide MLP: 136 slabs on 148 SMs).
      // Otherwise, with fewer slabs than SMs, each slab is split among j
      // CTAs of one cluster when that fills >= 75% of the SMs: the parts
      // meet in shared memory (DSMEM) instead of the workspace (hidden-5120
      // q/k/v: 56 slabs x 2; o and down: 40 slabs x 3).
      p.cl_j = 1;
      if (cfg.grid <= 0) {
        const int slabs = row_slabs(out);
        const int j = (slabs + sms - 1) / sms;
        if (slabs % j == 0 && (long long)(slabs / j) * 100 >= (long long)sms * 85) {
          grid = slabs / j;
        } else if (slabs < sms) {
          // the largest j whose clusters all fit at once and fill >= 75%
          for (int jc = std::min(std::min(8, sms / slabs), cps); jc >= 2; --jc) {
            if ((long long)slabs * jc * 100 < (long long)sms * 75) break;
            if (capacity(jc) >= slabs) {
              grid = (long long)slabs * jc;
              p.cl_j = jc;
              break;
            }
          }
          // When even the flat split cannot fill the SMs (at most one chunk
          // per CTA, every slab split anyway), clusters combine the parts in
          // DSMEM instead of the workspace fix-up, whatever their fill (the
          // small shards of a tensor-parallel layer).
          if (p.cl_j == 1 && chunks <= sms)
            for (int jc = std::min(std::min(8, sms / slabs), cps); jc >= 2; --jc)
              if (capacity(jc) >= slabs) {
                grid = (long long)slabs * jc;
                p.cl_j = jc;
                break;
              }
        }
      }
      if (chunks < grid) grid = chunks;  // every CTA run holds at least one chunk
      const long long max_run = (chunks + grid - 1) / grid;
      const int xcap = (int)std::min<long long>(ng, max_run * cb);
      const size_t limit = (size_t)kGemvMaxSmem;
      // the deepest ring that fits, up to a forced depth
      int st = 0;
      for (int t = cfg.depth > 0 ? cfg.depth : 5; t >= 2 && !st; --t)
        if (gemv_smem(t, cb, gate_up, xcap, P) <= limit) st = t;
      if (st) {
        p.ok = true;
        p.stages = st;
        p.grid = (int)grid;
        p.xcap = xcap;
        p.smem = gemv_smem(st, cb, gate_up, xcap, P);
      }
    }
    if (p.ok) break;
    if (per == 1) return p;
    per = (per + 1) / 2;
  }
  p.threads = kGemvThreads;
  p.pieces = p.grid;
  p.tokens_per_pass = per;
  p.ch = cb;
  p.cps = cps;
  p.chunks = chunks;
  return p;
}

namespace {
// The phase trace buffer (thq4_debug_set_trace): records are reserved in
// launch order on the host.
std::mutex g_trace_mu;
unsigned long long *g_trace = nullptr;
size_t g_trace_words = 0, g_trace_next = 0;

unsigned long long *trace_record_words(size_t need) {
  std::lock_guard<std::mutex> lock(g_trace_mu);
  if (!g_trace) return nullptr;
  if (g_trace_next + need + 8 > g_trace_words) return nullptr;  // keep room for the end marker
  unsigned long long *r = g_trace + g_trace_next;
  g_trace_next += need;
  return r;
}
unsigned long long *trace_record(int grid) { return trace_record_words(8 + (size_t)grid * kTrStamps); }
}  // namespace

void gemv_set_trace(void *buf, size_t bytes) {
  std::lock_guard<std::mutex> lock(g_trace_mu);
  g_trace = static_cast<unsigned long long *>(buf);
  g_trace_words = buf ? bytes / 8 : 0;
  g_trace_next = 0;
}

cudaError_t gemv_launch(const thq4_weight &w0, const thq4_weight *w1, const void *x, bool x_f32, int m, void *y,
                        bool y_f32, void *workspace, cudaStream_t stream, const PeerGather *peer, bool x_presum) {
  const bool gate_up = w1 != nullptr;
  const GemvPlan p = gemv_plan(w0.out, w0.in, m, x_f32, gate_up);
  if (!p.ok) return cudaErrorInvalidConfiguration;
  // a gathered call is one launch (one signal per call)
  if (peer && (m > p.tokens_per_pass || y_f32)) return cudaErrorInvalidValue;
  const int xb = x_f32 ? 4 : 2, yb = y_f32 ? 4 : 2;
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
    a.chunks = (int)p.chunks;
    a.run_base = (int)(p.chunks / p.grid);
    a.run_rem = (int)(p.chunks % p.grid);
    a.cps = p.cps;
    a.m = mt;
    a.in = w0.in;
    a.ng = w0.in / kGroup;
    a.out = w0.out;
    a.P = x_f32 ? 2 * mt : mt;
    a.xf32 = x_f32 ? 1 : 0;
    a.yf32 = y_f32 ? 1 : 0;
    // a presum block is one pass (m <= 8): its sums follow the 8 rows
    a.xsum = x_presum ? reinterpret_cast<const float *>(static_cast<const uint16_t *>(x) + (size_t)8 * w0.in) + t0
                      : nullptr;
    a.stages = p.stages;
    a.xcap = p.xcap;
    a.pre = gemv_cfg_override().pre;
    a.cl_j = p.cl_j;
    if (peer) {
      a.g_dst = peer->dst;
      a.g_flags = peer->flags;
      a.g_count = peer->count;
      a.g_arrive = peer->arrive;
      a.g_mode = peer->mode;
      a.g_world = peer->world;
      a.g_rank = peer->rank;
      a.g_rows = peer->rows;
      a.g_off = peer->offset;
      a.g_stride = peer->stride;
      a.g_wait = peer->wait;
      a.g_slot = peer->slot;
      a.xparts = peer->x_parts;
      a.xslot = peer->x_slot;
      a.x_ll = peer->x_ll;
    }
    a.trace = trace_record(p.grid);
    // a last pass with fewer tokens fits in the footprint planned for more
    const size_t smem = gemv_smem(p.stages, p.ch, gate_up, p.xcap, a.P);
    const int gw = window_groups(a.P);
    cudaError_t e = w0.sb_dtype == THQ4_F16 ? dispatch<true>(a, gate_up, p.ch, gw, p.grid, smem, stream)
                                            : dispatch<false>(a, gate_up, p.ch, gw, p.grid, smem, stream);
    if (e == cudaErrorCooperativeLaunchTooLarge && a.cl_j > 1) {
      // the clusters do not fit in one wave: one CTA per SM with split-K
      const int grid = (int)std::min<long long>(p.chunks, device_sm_count());
      a.cl_j = 1;
      if (a.trace && grid > p.grid) a.trace = nullptr;  // the record holds p.grid CTAs
      a.run_base = (int)(p.chunks / grid);
      a.run_rem = (int)(p.chunks % grid);
      e = w0.sb_dtype == THQ4_F16 ? dispatch<true>(a, gate_up, p.ch, gw, grid, smem, stream)
                                  : dispatch<false>(a, gate_up, p.ch, gw, grid, smem, stream);
    }
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

size_t chain_workspace_bytes(int max_rows) { return gemv_workspace_bytes(max_rows) + 256; }

int chain_max_ops() { return kMaxChainOps; }

namespace {
template <int GW, bool ONE, bool SF16>
cudaError_t chain_launch_t(const ChainArgs &a, int grid, size_t smem, cudaStream_t stream) {
  auto *k = &chain_kernel<GW, ONE, SF16>;
  static DeviceOnce once;
  cudaError_t e = once.run([&] {
    return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvMaxSmem);
  });
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kThreads, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorCooperativeLaunchTooLarge;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  // every CTA is resident at once: the grid barrier between ops relies on it
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, a);
}
}  // namespace

cudaError_t chain_launch(const ChainSpec *ops, int n, bool x_f32, int m, void *workspace, size_t workspace_bytes,
                         cudaStream_t stream) {
  if (n < 1 || n > kMaxChainOps) return cudaErrorInvalidValue;
  const int grid = device_sm_count();
  ChainArgs a{};
  a.status = status_word();
  a.n = n;
  a.m = m;
  a.P = x_f32 ? 2 * m : m;
  a.xf32 = x_f32 ? 1 : 0;
  int max_rows = 0, xcap = 1;
  for (int i = 0; i < n; ++i) {
    const ChainSpec &c = ops[i];
    ChainOp &o = a.ops[i];
    const bool gu = c.up != nullptr;
    const int cb = gu ? 4 : 8;
    o.qw0 = static_cast<const uint8_t *>(c.w->qw);
    o.sb0 = static_cast<const uint8_t *>(c.w->sb);
    o.qw1 = gu ? static_cast<const uint8_t *>(c.up->qw) : nullptr;
    o.sb1 = gu ? static_cast<const uint8_t *>(c.up->sb) : nullptr;
    o.x = c.x;
    o.y = c.y;
    o.out = c.w->out;
    o.in = c.w->in;
    o.ng = c.w->in / kGroup;
    o.cps = (o.ng + cb - 1) / cb;
    const int slabs = row_slabs(o.out);
    if ((long long)slabs * o.ng >= (1ll << 31)) return cudaErrorInvalidValue;
    o.chunks = slabs * o.cps;
    // whole slabs per CTA where that fills >= 85% of the SMs, else equal runs
    const int j = (slabs + grid - 1) / grid;
    if (slabs % j == 0 && (long long)(slabs / j) * 100 >= (long long)grid * 85) {
      o.active = slabs / j;
      o.run_base = j * o.cps;
      o.run_rem = 0;
    } else {
      o.active = std::min(o.chunks, grid);
      o.run_base = o.chunks / o.active;
      o.run_rem = o.chunks % o.active;
    }
    o.gate_up = gu ? 1 : 0;
    o.yf32 = c.y_f32 ? 1 : 0;
    const int max_run = o.run_base + (o.run_rem ? 1 : 0);
    xcap = std::max(xcap, std::min(o.ng, max_run * cb));
    max_rows = std::max(max_rows, o.out);
  }
  if (workspace_bytes < chain_workspace_bytes(max_rows)) return cudaErrorInvalidValue;
  const size_t part_bytes =
      gemv_workspace_bytes(max_rows) - ((size_t)row_slabs(max_rows) * kSlabTiles * 4 + 255) / 256 * 256;
  a.part = static_cast<float *>(workspace);
  a.count = reinterpret_cast<uint32_t *>(static_cast<char *>(workspace) + part_bytes);
  a.bar = reinterpret_cast<uint32_t *>(static_cast<char *>(workspace) + gemv_workspace_bytes(max_rows));
  a.xcap = xcap;
  a.trace = trace_record_words(8 + (size_t)n * grid * 4);
  int st = 0;
  for (int t = 5; t >= 2 && !st; --t)
    if (512 + (size_t)t * kChainStageBytes + xstage_bytes(xcap, a.P) <= (size_t)kGemvMaxSmem) st = t;
  if (!st) return cudaErrorInvalidConfiguration;
  a.stages = st;
  const size_t smem = 512 + (size_t)st * kChainStageBytes + xstage_bytes(xcap, a.P);
  const int gw = window_groups(a.P);
  const bool f16 = ops[0].w->sb_dtype == THQ4_F16;
  if (gw == 4)
    return a.P == 1 ? (f16 ? chain_launch_t<4, true, true>(a, grid, smem, stream)
                           : chain_launch_t<4, true, false>(a, grid, smem, stream))
                    : (f16 ? chain_launch_t<4, false, true>(a, grid, smem, stream)
                           : chain_launch_t<4, false, false>(a, grid, smem, stream));
  if (gw == 2)
    return f16 ? chain_launch_t<2, false, true>(a, grid, smem, stream) : chain_launch_t<2, false, false>(a, grid, smem, stream);
  return f16 ? chain_launch_t<1, false, true>(a, grid, smem, stream) : chain_launch_t<1, false, false>(a, grid, smem, stream);
}

cudaError_t peer_wait_launch(const PeerGather &g, cudaStream_t stream) {
  peer_wait_kernel<<<1, 32, 0, stream>>>(g.flags, g.count, g.world, g.rank, status_word());
  return cudaGetLastError();
}

}  // namespace thq4
