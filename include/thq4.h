/*
 * thq4.h -- C ABI of the B200 (sm_100a) Q4 affine quantized-matmul path.
 *
 * This is the drop-in boundary for th-engine's quant-linear operator.  The
 * reference reaches its kernels through candle custom ops on (wq: U32,
 * sb: BF16, x: BF16) behind QLin (engine/src/qwen35.rs:398 linear_ps, :711
 * gate_up_act_ps, :918 lin_apply_ps; ops engine/src/quant_kernel.rs:2686-2766,
 * 3040-3135, 3514-3735, 4860-5084) and, for MoE, through Splash's
 * MoE::add (docs/splash/runtime/ops/MoE.cpp:119-231).  Each entry point below
 * names the reference interface it replaces.
 *
 * Conventions
 *   - Every data pointer is a DEVICE pointer unless stated otherwise; `stream`
 *     is a cudaStream_t passed as void* (NULL = the legacy default stream).
 *   - Every call validates its arguments on the host before launching anything
 *     and returns a thq4_status; on failure nothing was launched and
 *     thq4_last_error() holds a message (per host thread).  This mirrors the
 *     reference's bail!-before-encode checks (quant_kernel.rs:2671-2684,
 *     qwen35.rs:405-411) and MoE::add's throw-before-encode
 *     (MoE.cpp:119-144).
 *   - Inputs are read-only; outputs never alias inputs; weights are immutable
 *     after repack.  No entry point allocates device memory: scratch comes
 *     from the caller's workspace.  Calls on distinct streams are thread-safe.
 *   - Launches are asynchronous; a kernel-side status (bad expert id, etc.) is
 *     reported by thq4_device_status().
 */
#ifndef THQ4_H
#define THQ4_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define THQ4_ABI_VERSION 2

typedef enum thq4_status {
  THQ4_OK = 0,
  THQ4_ERR_INVALID_ARGUMENT = 1, /* shape/dtype/pointer/alignment mismatch */
  THQ4_ERR_UNSUPPORTED = 2,      /* valid request this build does not serve */
  THQ4_ERR_WORKSPACE = 3,        /* workspace missing or too small */
  THQ4_ERR_CUDA = 4,             /* a CUDA runtime call failed */
  THQ4_ERR_NCCL = 5              /* a collective failed */
} thq4_status;

typedef enum thq4_dtype {
  THQ4_BF16 = 0,
  THQ4_F16 = 1,
  THQ4_F32 = 2,
  /* x of thq4_linear / thq4_gate_up given as a presum block (m <= 8): see
   * thq4_presum_block_bytes */
  THQ4_PRESUM = 3
} thq4_dtype;

/* Source layouts thq4_repack accepts (the reference's formats, plus ours). */
typedef enum thq4_src_layout {
  /* MLX affine: w u32 [out][in/8] nibbles LSB first, sb [out][2*ng] = a row's
   * ng scales then its ng biases (qwen35.rs:249-300, quant_kernel.rs:14-15). */
  THQ4_SRC_MLX = 0,
  /* QLin::tiled (qwen35.rs:629-697): words [tile][group][col][8] over rows
   * padded to 256; sb planar, scales then biases at + padded*ng. */
  THQ4_SRC_TILED = 1,
  /* Splash expert slab (moe_expert_slab.h:15-28): [weights][scales][biases]
   * in StorageN=256 order, out % 256 == 0; `sb` is ignored. */
  THQ4_SRC_SLAB = 2,
  /* This library's frag layout (a device copy of an already packed weight). */
  THQ4_SRC_FRAG = 3
} thq4_src_layout;

/* One packed projection in the frag layout (documented in
 * token-horizon_b200/csrc/thq4_common.cuh): rows pad to 128, one 4096-byte
 * nibble chunk and one 512-byte scale/bias chunk per (128-row slab, group).
 * Replaces QLin {wq, sb, out, inp, gs, tiled} (qwen35.rs:303-325). */
typedef struct thq4_weight {
  int32_t out;      /* logical output rows */
  int32_t in;       /* input size K, a multiple of 64 */
  int32_t gs;       /* quant group size; 64 */
  int32_t sb_dtype; /* THQ4_BF16 (reference format) or THQ4_F16 */
  const void *qw;   /* nibbles, 16-byte aligned, thq4_weight_bytes() long */
  const void *sb;   /* scale/bias quads, 16-byte aligned */
} thq4_weight;

/* A set of experts with identical shape, packed back to back in the frag layout
 * (replaces Splash ExpertQ4Projection, docs/splash/runtime/ops/Linear.hpp:
 * 37-43).  Expert e's nibbles start at qw + e*qw_stride bytes, its scales at
 * sb + e*sb_stride bytes. */
typedef struct thq4_experts {
  int32_t experts;
  int32_t out;
  int32_t in;
  int32_t gs;
  int32_t sb_dtype;
  int32_t reserved;
  const void *qw;
  const void *sb;
  uint64_t qw_stride;
  uint64_t sb_stride;
} thq4_experts;

/* ---- library ------------------------------------------------------------ */

/* "thq4 <semver> sm_100a" -- a static string. */
const char *thq4_version(void);
/* Copies the calling thread's last error message (NUL-terminated, truncated to
 * `cap`); returns its full length. */
size_t thq4_last_error(char *buf, size_t cap);
/* Reads and clears the device-side status word of the current device (bad
 * expert ids and similar conditions a kernel skipped instead of faulting).
 * Synchronises `stream`.  *status_out = 0 when clean. */
thq4_status thq4_device_status(uint32_t *status_out, void *stream);

/* ---- weights (replaces Weights::get_lin + QLin::tiled, qwen35.rs:249-300,
 * 629-697, and the Splash package loader's slab view) -------------------- */

/* Bytes of the frag buffers for `rows` x `in` (either pointer may be NULL).
 * Returns the total. */
size_t thq4_weight_bytes(int rows, int in, int gs, size_t *qw_bytes,
                         size_t *sb_bytes);
/* Repacks rows [row_begin, row_begin + rows) of a `src_out` x `in` weight in
 * `src_layout` into the frag layout.  All pointers are device pointers.  Row ranges
 * let one call cut a column shard or the gate/up halves of a fused
 * [gate | up] weight (fuse_lins, qwen35.rs:1581-1610). */
thq4_status thq4_repack(int src_layout, const void *src_w, const void *src_sb,
                        int src_out, int in, int gs, int sb_dtype,
                        int row_begin, int rows, void *dst_qw,
                        size_t dst_qw_bytes, void *dst_sb, size_t dst_sb_bytes,
                        void *stream);
/* Fills a thq4_weight after checking alignment and shape. */
thq4_status thq4_weight_init(thq4_weight *w, int out, int in, int gs,
                             int sb_dtype, const void *qw, const void *sb);

/* ---- projections ---------------------------------------------------------
 * x [m][in] (x_dtype THQ4_BF16 or THQ4_F32), y [m][out] (y_dtype THQ4_BF16
 * or THQ4_F32).  m = 1 runs the decode GEMV, 2..8 the verify kernel, larger
 * m the prefill GEMM: the row-count routing of QLin::linear_ps
 * (qwen35.rs:398-617).  Output element (t, n) = sum over groups of
 * s * sum(q*x) + b * sum(x), accumulated in f32 (decode/verify), or the
 * bf16-dequantised weight times x accumulated in f32 (prefill). */

/* Replaces QLin::linear_ps / AffineQmvT / AffineQmpp / AffineQsg / AffineQmm
 * / AffineQpf / AffineQmppPrefill (qwen35.rs:398-617). */
thq4_status thq4_linear(const thq4_weight *w, const void *x, int x_dtype, int m,
                        void *y, int y_dtype, void *workspace,
                        size_t workspace_bytes, void *stream);
/* Replaces QLin::gate_up_act_ps (qwen35.rs:711-884): y [m][gate.out] =
 * bf16(silu(bf16 g) * bf16 u) with g = gate x, u = up x.  gate and up are
 * the two halves of the fused weight (same out, in, sb_dtype).  Both calls
 * return THQ4_ERR_WORKSPACE without a large enough workspace. */
thq4_status thq4_gate_up(const thq4_weight *gate, const thq4_weight *up,
                         const void *x, int x_dtype, int m, void *y,
                         int y_dtype, void *workspace, size_t workspace_bytes,
                         void *stream);
/* Replaces the scalar reference kernels AffineQmv / AffineQmm
 * (quant_kernel.rs:1026-1147, 1634-1740; ops :2686-2766, 5766-5834), which the
 * reference's tests use to check the tuned kernels on the device (scalar_ref,
 * qwen35.rs:6928-6938).  y [m][out] = x [m][in] . W^T with every weight
 * dequantised in f32 as fma(q, s, b) and the products accumulated in f32:
 * one warp per output row, lane l adding the 8 consecutive k at 8l, 8l + 256,
 * ... in k order, the lanes combined by xor butterfly (16, 8, 4, 2, 1); any
 * m >= 1 (passes of 8 tokens), x and y as thq4_linear.  Deterministic, not
 * tuned; no workspace. */
thq4_status thq4_linear_scalar(const thq4_weight *w, const void *x, int x_dtype, int m, void *y, int y_dtype,
                               void *stream);
/* Workspace bytes thq4_linear / thq4_gate_up need for this weight at m rows
 * (for thq4_gate_up pass the gate half).  The decode/verify kernel splits
 * tiles over warps and finishes each split tile in the warp that arrives
 * last: the workspace holds the partial sums and one arrival counter per
 * 16-row tile.  At m > 8 (bf16 x) the figure can be larger: thq4_linear's
 * prefill then splits the k-stages of its 128-row x 256-token tiles evenly
 * over the SMs (stream-K) and needs, after the decode region, one claim word
 * pair and one f32 part tile (128 KB) per SM.  Given less, no workspace or
 * one that is not 256-byte aligned, the prefill runs whole tiles instead,
 * which is slower when the tiles do not fill whole waves.  The workspace must be 256-byte aligned and
 * zero-filled before its first use; every call leaves its counters and
 * claim words zeroed (the parts need no clearing), so one allocation serves
 * every later call.  Calls that may overlap on the GPU need separate
 * workspaces. */
size_t thq4_linear_workspace_bytes(const thq4_weight *w, int m);
/* A chain of dependent projections in one persistent launch.  No single
 * reference counterpart: it runs what consecutive QLin::linear_ps /
 * gate_up_act_ps calls (qwen35.rs:398, 711) would, e.g. an MLP's gate/up and
 * then its down projection (lin_apply_ps, :918), or a decode layer's
 * projections, with op i seeing every output of ops 0 .. i-1.  Each op is
 * thq4_linear (up == NULL) or thq4_gate_up (w = gate half, up = up half) on
 * x [m][w->in] -> y [m][w->out] with the arithmetic of that call.  One
 * cooperative launch with one CTA per SM streams the weights of op after op
 * without pausing at op boundaries; a grid-wide barrier orders each op's
 * outputs before the next op reads them. */
typedef struct thq4_chain_op {
  const thq4_weight *w;  /* the projection (the gate half of a gate/up op) */
  const thq4_weight *up; /* the up half, or NULL */
  const void *x;         /* device, [m][w->in] of the chain's x_dtype (may be an earlier op's y) */
  void *y;               /* device, [m][w->out], y_dtype; never this op's x */
  int32_t y_dtype;       /* THQ4_BF16 or THQ4_F32 */
  int32_t reserved;      /* 0 */
} thq4_chain_op;
/* Workspace bytes of thq4_linear_chain: split-K partials, arrival counters
 * and the grid barrier's words.  256-byte aligned and zero-filled before its
 * first use; every completed call leaves the counters and barrier words at
 * zero again (unless it timed out), so one allocation serves later calls. */
size_t thq4_linear_chain_workspace_bytes(const thq4_chain_op *ops, int n);
/* 1 <= n <= 112 ops, one scale dtype, m <= 8 tokens of bf16 x (4 of f32 x).
 * Calls that may overlap on the GPU need separate workspaces. */
thq4_status thq4_linear_chain(const thq4_chain_op *ops, int n, int x_dtype, int m, void *workspace,
                              size_t workspace_bytes, void *stream);
/* thq4_linear without a workspace argument.  No reference counterpart: the
 * reference's ops take scratch from candle's buffer pool.  It routes by row
 * count exactly as thq4_linear does (the prefill kernel for m > 8 bf16 rows,
 * which needs no scratch; the decode/verify kernel otherwise), so both entry
 * points give the same numbers.  The decode/verify kernel's split-K scratch
 * (partial sums and arrival counters) comes from one 6 MiB buffer the library
 * keeps in device memory per device, so the call allocates nothing and needs
 * only the weight, x and y.
 *
 * For callers that cannot allocate or own device memory where they run a
 * projection: a binding that only receives tensors from its host and has no
 * device allocator of its own, or a serving loop whose device memory is fixed
 * before the first request (a cudaMalloc there would also synchronise the
 * device).
 *
 *   - The first call on a device, with that device current, looks up the
 *     buffer's address once (cudaGetSymbolAddress); make that first call
 *     before any stream capture.  Neither it nor any later call allocates:
 *     no cudaMalloc / cudaFree and no allocating library call.
 *   - A weight whose workspace (thq4_linear_workspace_bytes) is larger than
 *     the buffer is rejected with THQ4_ERR_UNSUPPORTED before anything is
 *     launched (at 148 SMs: above about 5.7 million rows).
 *   - Must start at zero: the arrival counters.  The buffer is zero when the
 *     library's module loads on a device, and every completed call leaves the
 *     counters zero again.  A call whose kernel reported kStatusTimeout
 *     (thq4_device_status) may leave them set, and nothing in this ABI clears
 *     the buffer: after a timeout, restart the process before calling this
 *     entry point again (thq4_linear's caller can re-zero its own
 *     workspace instead).
 *   - Every call on a device shares the one buffer: calls that can overlap on
 *     the GPU (streams not ordered with each other) race and produce wrong
 *     results.  Order them on one stream, or use thq4_linear with a workspace
 *     per stream. */
thq4_status thq4_linear_noalloc(const thq4_weight *w, const void *x, int x_dtype,
                                int m, void *y, int y_dtype, void *stream);
/* ---- presum blocks (replaces the K45 presum machinery, quant_kernel.rs:
 * 265-318, 2544-2568, 3355-3440, 3642-3657) ------------------------------
 * A presum block of width `in` is a decode / verify activation of m <= 8
 * rows laid out as 8 bf16 rows [8][in] (rows >= m zero) followed by the f32
 * sums [in/64][8]: sums[g * 8 + t] is row t's group g summed in the
 * reference's lane pattern (lane l adds x[64g + l] + x[64g + 32 + l] in f32,
 * the 32 lanes combine by xor butterfly 16, 8, 4, 2, 1).  Passed as x with
 * x_dtype THQ4_PRESUM, thq4_linear and thq4_gate_up use the block's sums for
 * each group's bias term b * sum(x) instead of computing them; the block must
 * be thq4_presum_block_bytes(in) bytes long and 16-byte aligned (the
 * reference's "presum block missing" check, quant_kernel.rs:3642-3657). */
/* 8 * in * 2 + (in / 64) * 8 * 4 (presum_block_bytes, quant_kernel.rs:
 * 265-273); 0 when in is not a positive multiple of 64. */
size_t thq4_presum_block_bytes(int in);
/* Q4AttachSums (quant_kernel.rs:3355-3440): block = x [m][in] bf16 as a
 * presum block (rows m..7 zero) with its sums.  1 <= m <= 8. */
thq4_status thq4_presum_attach(const void *x, int m, int in, void *block, void *stream);
/* AddRmsNorm { sums } (engine/src/gdn_kernel.rs:1851-1866, 1919-1962):
 * res bf16 [T][C] = bf16(x + r) and block = the presum block of
 * bf16(bf16(res) * inv * w) (rows T..7 zero), inv = 1 / sqrt(ss / C + eps),
 * ss = sum of (x + r)^2 in f32, lane l accumulating columns l, l + 32, ...
 * in order, the 32 lanes combined by the butterfly; 1 / sqrt is correctly
 * rounded here where the reference's Metal rsqrt is approximate.  x, r, w
 * bf16; 1 <= T <= 8; C a multiple of 64, at most 32768. */
thq4_status thq4_add_rms_norm(const void *x, const void *r, const void *w, int T, int C, float eps, void *res,
                              void *block, void *stream);

/* Replaces AffineDequant (quant_kernel.rs:1743-1782, 5836-5899): y bf16
 * [out][in] = bf16(q * s + b). */
thq4_status thq4_dequant(const thq4_weight *w, void *y, void *stream);

/* ---- MoE (replaces Splash MoE::add, docs/splash/runtime/ops/MoE.cpp:119-231,
 * and its kernels in docs/splash/runtime/metal/kernels/shared/moe.metal) ---- */

/* Group tiles (of 32 routes each) the routing of T tokens to k of E experts
 * can produce: min(T*k/32 + E, T*k) (moeMaximumTiles, MoE.hpp:72-77, without
 * a shared expert). */
uint32_t thq4_moe_max_tiles(int T, int E, int k);
/* Routing on the device (moe_route_select_q8 + moe_group_routes,
 * moe.metal:270-449).  logits bf16 [T][E]; outputs: ids u32 [T][k] (experts by
 * descending score, lowest id first among equal scores), weights bf16 [T][k]
 * (softmax over the k selected scores), tiles u32 [max_tiles][2] = {expert,
 * live rows}, grouped_routes u32 [max_tiles*32] (route t*k+slot, padding
 * 0xFFFFFFFF), route_rows u32 [T*k] (the inverse map), ntiles u32 [1].  Within
 * an expert, routes ascend by route index: the permutation is deterministic
 * and bit-exact.  max_tiles >= thq4_moe_max_tiles(T, E, k); E <= 1024,
 * 1 <= k <= min(E, 32). */
thq4_status thq4_moe_route(const void *logits, int T, int E, int k, uint32_t *ids, void *weights,
                           uint32_t *tiles, uint32_t *grouped_routes, uint32_t *route_rows,
                           uint32_t *ntiles, int max_tiles, void *stream);
/* Workspace bytes of thq4_moe (routing tables, the gathered rows and the
 * per-route intermediates). */
size_t thq4_moe_workspace_bytes(int T, int H, int I, int E, int k);
/* One MoE layer: y bf16 [T][H] = residual (optional, bf16 [T][H]) + sum over
 * the k routes of each token, in slot order, of w * down(bf16(silu(bf16 g) *
 * bf16 u)), g = gate x, u = up x, accumulated in f32 (moe_combine,
 * moe.metal:642-664).  x bf16 [T][H], logits bf16 [T][E]; gate and up:
 * E experts of I x H, down: E experts of H x I, one scale dtype.  All sizes
 * are checked before anything is launched (MoE::add throws the same way,
 * MoE.cpp:119-144). */
thq4_status thq4_moe(const void *x, const void *residual, const void *logits, int T, int H, int I,
                     int E, int k, const thq4_experts *gate, const thq4_experts *up,
                     const thq4_experts *down, void *y, void *workspace, size_t workspace_bytes,
                     void *stream);

/* ---- the Splash MoE layer with its Q8 router and shared expert ---------- */

/* An 8-bit affine projection in Splash's StorageN = 256 order (replaces
 * Q8Projection, docs/splash/runtime/ops/Linear.hpp:27-33): output n < 256 of
 * input k has its byte q at ((k/64)*256 + n)*64 + k%64 and its bf16 scale and
 * bias at (k/64)*256 + n, value q * scale + bias.  out is 256; in % 64 == 0;
 * q, scales and biases 16-byte aligned. */
typedef struct thq4_q8_weight {
  int32_t out;
  int32_t in;
  const void *q;
  const void *scales;
  const void *biases;
} thq4_q8_weight;

/* All weights of one sparse MoE block (replaces MoeWeights, MoE.hpp:35-44):
 * the router (scores of experts 0..E-1 are its rows 0..E-1), E routed experts,
 * and the shared expert -- three one-expert projections of the routed
 * shapes, weighted per token by the sigmoid of row 0 of
 * shared_expert_gate.  A layer without a shared expert passes
 * shared_gate.qw == NULL and shared_expert_gate.q == NULL. */
typedef struct thq4_moe_weights {
  thq4_q8_weight router;
  thq4_experts gate, up, down;
  thq4_experts shared_gate, shared_up, shared_down;
  thq4_q8_weight shared_expert_gate;
} thq4_moe_weights;

/* Router scores (moe_route_scores_q8_m8 / _m32, moe.metal:34-262): scores
 * bf16 [T][ld] columns 0..ncols-1 = bf16 of, over eight K slices in order
 * (slice s: groups [s*G/8, (s+1)*G/8) of G = in/64), the sum in group order
 * of fma(dot, scale, sum * bias); dot = sum over the group's 64 k in k order
 * of x * q (f32), sum = the group's 64 x as 32 pairs (x[l] + x[l+32])
 * combined by xor butterfly (partners 16, 8, 4, 2, 1).  x bf16 [T][in],
 * 16-byte aligned; 1 <= ncols <= 256, ld >= ncols.  Workspace:
 * thq4_moe_scores_workspace_bytes(T, ncols) (the eight slices' f32 sums). */
size_t thq4_moe_scores_workspace_bytes(int T, int ncols);
thq4_status thq4_moe_scores_q8(const void *x, int T, const thq4_q8_weight *router, int ncols, void *scores, int ld,
                               void *workspace, size_t workspace_bytes, void *stream);

/* Group tiles of MoE::add for T tokens, k of E experts, plus ceil(T/32)
 * tiles of the shared expert when shared != 0 (moeMaximumTiles, MoE.hpp:
 * 72-77). */
uint32_t thq4_moe_add_max_tiles(int T, int E, int k, int shared);
/* The routing of MoE::add on the device (the router, moe_route_select_q8 and
 * moe_group_routes, moe.metal:34-449): scores as thq4_moe_scores_q8, top k
 * by descending score (lowest id first among equal scores) with softmax
 * weights; with a shared expert gate (not NULL) a last route per token holds
 * expert E with weight bf16(1 / (1 + exp(-g))), g = x . row 0 of the gate
 * dequantised (thread v of 256 accumulates k = v, v + 256, ... by fma, warps
 * by xor butterfly, the eight warp sums in order).  rpr = k (+1 with the
 * shared expert) routes per token: ids u32 [T][rpr], weights bf16 [T][rpr],
 * tiles u32 [max_tiles][2], grouped_routes u32 [max_tiles*32], route_rows
 * u32 [T*rpr], ntiles u32 [1]; the shared expert's tiles follow the routed
 * ones and hold every token in order.  Workspace:
 * thq4_moe_scores_workspace_bytes(T, E). */
thq4_status thq4_moe_route_q8(const void *x, int T, int E, int k, const thq4_q8_weight *router,
                              const thq4_q8_weight *shared_expert_gate, uint32_t *ids, void *weights, uint32_t *tiles,
                              uint32_t *grouped_routes, uint32_t *route_rows, uint32_t *ntiles, int max_tiles,
                              void *workspace, size_t workspace_bytes, void *stream);
/* Workspace bytes of thq4_moe_add (shared: the block has a shared expert). */
size_t thq4_moe_add_workspace_bytes(int T, int H, int I, int E, int k, int shared);
/* One MoE block (replaces MoE::add, MoE.cpp:119-231): routing as
 * thq4_moe_route_q8, then y bf16 [T][H] = residual (optional) + the sum over
 * each token's routes in slot order (the shared expert last) of
 * w * down(bf16(silu(bf16 g) * bf16 u)), f32, one bf16 rounding.  Checked
 * before anything is launched as MoE::add validates (MoE.cpp:43-58):
 * H and I multiples of 256, 1 <= k <= E <= 256, router and shared gate
 * 256 x H, experts E x I x H (gate, up) and E x H x I (down), the shared
 * projections one expert each. */
thq4_status thq4_moe_add(const void *x, const void *residual, int T, int H, int I, int E, int k,
                         const thq4_moe_weights *w, void *y, void *workspace, size_t workspace_bytes, void *stream);

/* ---- multi-GPU shards ------------------------------------------------------
 * The reference engine is single-device; these entry points are the sharded
 * extension, one process per GPU.
 *
 * Column shards (out_mode 0, gather): each rank holds a contiguous range of a
 * projection's output rows; instead of an all-gather after the projection,
 * the GEMV's epilogue stores its rows straight into every rank's copy of the
 * full vector (NVLink stores through IPC mappings).
 *
 * Row shards (out_mode 1, reduce): each rank holds a contiguous range of a
 * projection's input columns and computes an f32 partial of every output;
 * the epilogue stores it into slot `rank` of every rank's reduction buffer
 * (dst[r] + rank * slot floats, [t][stride]).  The all-reduce finishes on
 * read: a projection with x_parts = world reads x as the sum of the partials
 * in rank order, rounded once to bf16 -- a column-then-row-sharded pair (an
 * MLP's gate/up then down) exchanges one vector instead of two.
 *
 * Low-latency reduce (out_mode 3): as reduce, but every output is one
 * aligned 8-byte word {f32 value, exchange number} in the reduction buffer
 * (slot and x_slot then count words); the exchange number is this rank's
 * completed-exchange count + 1, the same on every rank.  The writer neither
 * fences nor raises flags; a projection reading such partials (x_parts with
 * x_ll = 1, wait = 0) polls each word in its own memory until it carries the
 * exchange number (bounded; kStatusTimeout).  No NVLink round trip is on the
 * writer's path: the values themselves are the signal.
 *
 * Reuse: a rank may write a reduction or gather buffer of a peer again only
 * after that peer's reader of its previous contents has completed, which the
 * writer must have observed: e.g. o and down writing two buffers in turn,
 * where a rank's next o follows its q/k/v that read the peers' down words,
 * written after each peer's gate/up had read the previous o's; or a host
 * barrier between uses.
 *
 * After its stores the grid's last CTA writes this rank's completed-exchange
 * count into its slot of every peer's flag words (system-scope release).  A
 * projection whose x comes from such an exchange waits (wait = 1, before it
 * reads x; bounded, kStatusTimeout bit 2 of thq4_device_status) until every
 * peer's flag has reached this rank's own count.  out_mode 2 (local) neither
 * exchanges nor signals (a column shard whose output stays local).  Every
 * rank must make the same sequence of calls.  The flag and count words live
 * in memory every rank maps (thq4_ipc_alloc / thq4_ipc_open) and start at 0. */
typedef struct thq4_peer_gather {
  int32_t world;           /* ranks, 1 .. 8 */
  int32_t rank;
  int32_t rows;            /* gather: the first `rows` outputs of the call are gathered ... */
  int32_t offset;          /* ... to full[t * stride + offset + row] on every rank */
  int32_t stride;          /* full-vector length per token (reduce: >= out) */
  int32_t wait;            /* 1: wait for the peers' exchanges before reading x */
  void *const *dst;        /* device array [world]: rank r's full vector (bf16) or reduction buffer (f32) */
  uint32_t *const *flags;  /* device array [world]: rank r's flag words (u32 [world]), as mapped here */
  uint32_t *count;         /* this rank's completed-exchange count (one device word) */
  uint32_t *arrive;        /* this rank's CTA arrival counter (one device word, left at 0) */
  int32_t out_mode;        /* 0 gather, 1 reduce, 2 local, 3 low-latency reduce */
  int32_t x_parts;         /* > 0: x (THQ4_F32) is x_parts partials, x + p * x_slot floats, each [m][in] */
  int64_t slot;            /* reduce: floats (3: words) between the ranks' partials in a reduction buffer (>= m * stride) */
  int64_t x_slot;          /* floats (x_ll: words) between the partials of x (>= m * in) */
  int32_t x_ll;            /* 1: the partials of x are low-latency words (written by out_mode 3) */
  int32_t reserved;        /* 0 */
} thq4_peer_gather;

/* thq4_linear (up == NULL) or thq4_gate_up with the exchange fused in; y is
 * bf16 [m][out] (the local rows; ignored, may be NULL, in reduce mode), m <= 8
 * for bf16 x or x partials (4 for f32 x). */
thq4_status thq4_linear_peer(const thq4_weight *w, const thq4_weight *up, const void *x, int x_dtype, int m,
                             void *y, void *workspace, size_t workspace_bytes, const thq4_peer_gather *g,
                             void *stream);
/* On `stream`, waits until every peer has completed as many exchanges as this
 * rank (for an exchanged vector read by something other than thq4_linear_peer). */
thq4_status thq4_peer_wait(const thq4_peer_gather *g, void *stream);

/* Expert-sharded MoE: this rank holds experts [e0, e1) of E (gate, up and
 * down describe just those, e1 - e0 experts each).  Routing runs over all E
 * experts, bit-identical on every rank given the same logits; only the
 * routes to local experts are computed.  y_part f32 [T][H] = residual (if
 * not NULL; pass it on one rank only) + the sum over each token's local
 * routes, in slot order, of w * down(bf16(silu(bf16 g) * bf16 u)).  Summing
 * y_part over the ranks (one all-reduce) and rounding once to bf16 gives the
 * layer's output.  Workspace: thq4_moe_workspace_bytes(T, H, I, e1 - e0, k). */
thq4_status thq4_moe_partial(const void *x, const void *residual, const void *logits, int T, int H, int I, int E,
                             int k, int e0, int e1, const thq4_experts *gate, const thq4_experts *up,
                             const thq4_experts *down, float *y_part, void *workspace, size_t workspace_bytes,
                             void *stream);

/* Workspace bytes of thq4_moe_add_partial for a shard holding experts
 * [e0, e1) of E; shared_route: the layer has a shared expert (every token k +
 * 1 routes); runs_shared: this shard runs it. */
size_t thq4_moe_add_partial_workspace_bytes(int T, int H, int I, int E, int k, int e0, int e1, int shared_route,
                                            int runs_shared);
/* thq4_moe_add for an expert shard: w holds routed experts [e0, e1) of E
 * (gate, up, down: e1 - e0 experts), the full router and, when
 * shared_expert_gate.q is not NULL, the layer's shared expert gate (every
 * token then has k + 1 routes); the shard runs the shared expert when
 * w->shared_gate.qw is not NULL (one rank of the group).  y_part f32 [T][H]
 * as thq4_moe_partial.  Workspace: thq4_moe_add_partial_workspace_bytes. */
thq4_status thq4_moe_add_partial(const void *x, const void *residual, int T, int H, int I, int E, int k, int e0,
                                 int e1, const thq4_moe_weights *w, float *y_part, void *workspace,
                                 size_t workspace_bytes, void *stream);

#define THQ4_IPC_HANDLE_BYTES 64
/* Device memory another process of this node can map: cudaMalloc'd, zeroed,
 * with its IPC handle (THQ4_IPC_HANDLE_BYTES bytes) written to `handle`. */
thq4_status thq4_ipc_alloc(size_t bytes, void **ptr, void *handle);
thq4_status thq4_ipc_open(const void *handle, void **ptr);
thq4_status thq4_ipc_close(void *ptr);
thq4_status thq4_ipc_free(void *ptr);
/* Stream-ordered copy between any two addresses (cudaMemcpyAsync, default kind). */
thq4_status thq4_copy(void *dst, const void *src, size_t bytes, void *stream);

/* ---- testing hooks -------------------------------------------------------
 * Forces the decode/verify kernel's launch shape for every later call in this
 * process: slab-groups per streamed stage (4 or 8), stages in the
 * shared-memory ring (2 .. 8; an upper bound, lowered to what fits) and CTAs
 * in the grid (1 .. 2x SM count: up to two CTAs per SM); 0 leaves a field to
 * the policy, all zeros restore it.  The reference's tests
 * run every instantiated tile config the same way (qwen35.rs:6963-6989).
 * Returns THQ4_ERR_INVALID_ARGUMENT for other values; `reserved` must be 0. */
thq4_status thq4_debug_set_gemv(int chunk, int stages, int grid, int reserved);
/* Phase trace of the decode/verify kernel for every later launch in this
 * process (NULL turns it off; each call starts over at the buffer's start).
 * `buf` is zero-filled device memory.  Each launch that fits appends a record:
 * 8 header words {0x7468713474726163, CTAs, out, in, gate_up | cluster size
 * << 8 | exchange mode << 16 | waits << 24, tokens, chunk | stages << 8, 0}
 * then, per CTA, 10 %globaltimer stamps (ns): running, predecessor complete,
 * peers' flags seen, activation staged, first weight stage landed, stream
 * consumed, outputs stored, exchange signalled, and for an exchanging launch
 * its stores fenced at system scope (every CTA) and the peers' flags written
 * (the last CTA; 0 elsewhere).  A chain launch (thq4_linear_chain) appends
 * 8 header words {0x7468713463686e21, CTAs, ops, stages, 0...} then, per
 * (op, CTA), 4 stamps: op begun, x staged, stream consumed, outputs
 * stored.  A launch captured in a CUDA
 * graph keeps its record; replays overwrite it.  No reference counterpart
 * (the reference times its kernels with Metal's GPU counters). */
thq4_status thq4_debug_set_trace(void *buf, size_t bytes);
/* The decode/verify launch plan for an out x in weight and m tokens (x_f32,
 * gate_up as thq4_linear / thq4_gate_up would pass them) on a GPU with `sms`
 * SMs on which cluster_fit[j] clusters of j one-CTA-per-SM CTAs can be
 * resident at once (j = 2..8; cluster_fit may be NULL: no clusters).  Fills
 * plan[8] = {planned (0/1), CTAs, cluster size (1: none), ring stages,
 * tokens per launch, chunks per 128-row slab, slab-groups per chunk,
 * dynamic shared memory bytes}.  Host only; the reference's tests pin their
 * dispatch tables the same way (quant_kernel.rs:5914-5973). */
thq4_status thq4_debug_gemv_plan(int out, int in, int m, int x_f32, int gate_up, int sms, const int *cluster_fit,
                                 int64_t *plan);
/* The prefill's launch plan for an out x in weight and m > 8 bf16 tokens
 * (gate_up: the two-weight form) on a GPU with `sms` SMs.  Fills plan[5] =
 * {tokens per tile, stream-K split (0/1), tiles, CTAs, bytes of the split's
 * workspace region after the decode kernel's (0 for whole tiles)}; the split
 * runs only when the caller's workspace holds that much.  Host only; pins the
 * prefill's dispatch policy the way thq4_debug_gemv_plan pins the decode
 * kernel's (the reference pins its own tables, quant_kernel.rs:5914-5973). */
thq4_status thq4_debug_prefill_plan(int out, int in, int m, int gate_up, int sms, int64_t *plan);

#ifdef __cplusplus
}
#endif
#endif /* THQ4_H */
