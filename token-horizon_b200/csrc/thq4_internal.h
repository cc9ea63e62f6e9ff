// thq4_internal.h -- declarations shared by the thq4 translation units.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <mutex>
#include <functional>
#include <string>

#include "../../include/thq4.h"

struct CUtensorMap_st;  // cuda.h's tensor map (only pointers to it cross files)

namespace thq4 {

// Dynamic shared memory the GEMV may use per CTA (B200: 227 KB opt-in).
constexpr int kGemvMaxSmem = 227 * 1024;

// Runs `fn` once per device (e.g. a cudaFuncSetAttribute), remembering
// success; a failure is returned and retried on the next call.
class DeviceOnce {
 public:
  template <class Fn>
  cudaError_t run(Fn &&fn) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    const uint64_t bit = 1ull << dev;
    if (done_.load(std::memory_order_acquire) & bit) return cudaSuccess;
    std::lock_guard<std::mutex> lock(mu_);
    if (done_.load(std::memory_order_relaxed) & bit) return cudaSuccess;
    e = fn();
    if (e == cudaSuccess) done_.fetch_or(bit, std::memory_order_release);
    return e;
  }

 private:
  std::atomic<uint64_t> done_{0};
  std::mutex mu_;
};

int device_sm_count();
// Device address of the status word on the current device (nullptr on error).
uint32_t *status_word();

// ---- GEMV / verify ---------------------------------------------------------
struct GemvCfg {
  int warps = 0;  // forced slab-groups per ring stage, 4 or 8 (0 = policy)
  int depth = 0;  // forced ring stages (0 = policy)
  int grid = 0;   // forced CTAs (0 = policy)
  int pre = 0;    // ring stages requested before x is staged (0 = all)
};
// The testing hook's forced shape, else THQ4_GEMV (read once), else none.
GemvCfg gemv_cfg_override();

struct GemvPlan {
  bool ok;
  int threads, grid, pieces, tokens_per_pass, ch, stages;
  int cps, xcap;     // chunks per slab, activation groups staged per CTA
  int cl_j;          // > 1: each slab split among cl_j CTAs of one cluster
  long long chunks;  // chunks in the weight
  size_t smem;
};
// Workspace the decode/verify kernel needs for a weight of `rows` rows:
// partial-sum slots for every warp plus one counter per 16-row tile.  It
// must be zero-filled before first use; every call leaves it zeroed.
size_t gemv_workspace_bytes(int rows);
// Programmatic dependent launch for the GEMV and the MoE chain (THQ4_PDL=0
// disables; read once).
bool gemv_pdl_enabled();
GemvPlan gemv_plan(int out, int in, int m, bool x_f32, bool gate_up);
// The same plan for a given SM count and cluster capacity (clusters of j
// one-CTA-per-SM CTAs resident at once); gemv_plan passes the device's.
using ClusterCapacity = std::function<int(int)>;
GemvPlan gemv_plan_for(int out, int in, int m, bool x_f32, bool gate_up, int sms, const ClusterCapacity &capacity);
int cluster_capacity(int j);
// The all-gather of column shards fused into the projection (thq4_peer_gather).
struct PeerGather {
  uint16_t *const *dst;     // device array [world]: each rank's full-vector (bf16) or reduction (f32) buffer
  uint32_t *const *flags;   // device array [world]: each rank's flag words [world]
  uint32_t *count, *arrive;
  int world, rank, rows, offset, stride, wait;
  int mode;                 // 0: no exchange, 1: gather, 2: reduce, 3: low-latency reduce
  long long slot;           // reduce: floats (mode 3: 8-byte words) between the ranks' partials
  int x_parts;              // > 0: x is this many f32 partials, summed as staged
  long long x_slot;         // floats (x_ll: 8-byte words) between the partials of x
  int x_ll = 0;             // the partials of x are low-latency words
};
cudaError_t gemv_launch(const thq4_weight &w0, const thq4_weight *w1, const void *x, bool x_f32,
                        int m, void *y, bool y_f32, void *workspace, cudaStream_t stream,
                        const PeerGather *peer = nullptr, bool x_presum = false);
// A chain of dependent projections in one persistent launch (thq4_linear_chain).
struct ChainSpec {
  const thq4_weight *w, *up;  // up: the second half of a gate/up op, or nullptr
  const void *x;
  void *y;
  bool y_f32;
};
int chain_max_ops();
size_t chain_workspace_bytes(int max_rows);
cudaError_t chain_launch(const ChainSpec *ops, int n, bool x_f32, int m, void *workspace, size_t workspace_bytes,
                         cudaStream_t stream);
// The GEMV's phase trace buffer (device memory, nullptr = off); records are
// taken from the start of the buffer again after every call.
void gemv_set_trace(void *buf, size_t bytes);
// Waits (one thread, bounded) until every peer has completed as many gathers
// as this rank, then returns; used where a gathered vector is consumed by
// something other than the next projection.
cudaError_t peer_wait_launch(const PeerGather &g, cudaStream_t stream);

// The scalar reference product (thq4_linear_scalar): f32 dequant, f32
// accumulate, one warp per row, any m in passes of 8 tokens.
cudaError_t scalar_launch(const thq4_weight &w, const void *x, bool x_f32, int m, void *y, bool y_f32,
                          cudaStream_t stream);

// ---- prefill GEMM (tcgen05) -------------------------------------------------
// The tensor-core path serves m > 8 tokens of bf16 x.  With a workspace of at
// least prefill_workspace_bytes(w0, m) bytes (the decode kernel's region
// first, untouched, then the split tiles' claim words and f32 parts) the
// one-weight form splits the k-stages evenly over the CTAs (stream-K);
// without one (workspace null or smaller) it runs whole tiles.
bool prefill_supported(int m, bool x_f32);
size_t prefill_workspace_bytes(const thq4_weight &w0, int m);
// The prefill's launch shape for an out-row weight and m tokens on `sms` SMs
// (host only): token-tile width, stream-K or whole tiles, tiles, CTAs, and
// the workspace bytes a split call asks for (0 for whole tiles).
struct PrefillPlanInfo {
  int bt;
  bool split;
  long long tiles;
  int grid;
  size_t split_bytes;
};
PrefillPlanInfo prefill_debug_plan(int out, int m, bool gate_up, int sms);
cudaError_t prefill_launch(const thq4_weight &w0, const thq4_weight *w1, const void *x, int m, void *y, bool y_f32,
                           void *workspace, size_t workspace_bytes, cudaStream_t stream);

// bf16 x [rows][k] (k innermost) as a 2-D tensor map with 64 x box_rows
// boxes and 128-byte swizzle; `map` points to a CUtensorMap.
cudaError_t make_xmap(const void *x, int k, int rows, int box_rows, ::CUtensorMap_st *map);

// ---- MoE -------------------------------------------------------------------
// Routes are grouped by expert into tiles of this many activation rows.
constexpr int kMoeTileRows = 32;

// The expert products for small group tiles (csrc/thq4_moe_gemv.cu): for
// every group tile gt < *count, y rows [gt*32, gt*32 + 32) = x rows .
// expert(tiles[2gt])^T (w1: the fused SwiGLU with w0 = gate, w1 = up).
// xsum [tile][in/64][32] holds the sum of each x row's 64-groups; ysum
// (optional) receives the same for y.  x, y: [max_tiles*32][in], [..][out].
// Tiles of expert id n_experts run the shared expert (sw0, sw1: one expert each).
struct MoeExperts {
  const void *x;
  void *y;
  const thq4_experts *w0, *w1;
  const thq4_experts *sw0, *sw1;
  int n_experts;
  const uint32_t *tiles, *count;
  const float *xsum;
  float *ysum;
  int max_tiles;
};
cudaError_t moe_expert_launch(const MoeExperts &g, cudaStream_t stream);

// Upper bound on group tiles for T tokens routed to k of E experts, plus
// ceil(T/32) tiles of a shared expert.
uint32_t moe_max_tiles(int T, int E, int k, bool shared = false);
// Shared memory of the grouping kernel for R routes and E experts.
size_t moe_group_smem(int R, int E);
// Eight K slices of router partial sums per (token, column).
constexpr int kRouteSlices = 8;
size_t moe_scores_bytes(int T, int ncols);

// Where a layer's routing comes from: bf16 logits [T][E], or the Q8 router
// applied to x (partial: [8][T][E] f32 scratch).  With a shared expert gate
// every token gets a last route (id E); shared_local: this call runs the
// shared expert (its tiles carry the local id e1 - e0), otherwise that route
// is dropped here.
struct MoeRouting {
  const uint16_t *logits;
  const void *x;
  int H;
  const thq4_q8_weight *router;
  const thq4_q8_weight *shared_gate;
  bool shared_local;
  float *partial;
};
// Router partial sums and, when scores is not null, the bf16 scores.
cudaError_t moe_scores_launch(const void *x, int T, int H, const thq4_q8_weight &router, int ncols, float *partial,
                              uint16_t *scores, int ld, cudaStream_t stream);
// Select (top-k, softmax weights, the shared route) and group (stable
// counting sort) on the device.  Experts [e0, e1) of E are grouped (e1 < 0:
// all); the tiles hold local ids.
cudaError_t moe_route_launch(const MoeRouting &r, int T, int E, int k, uint32_t *ids, uint16_t *weights,
                             uint32_t *tiles, uint32_t *grouped, uint32_t *route_rows, uint32_t *ntiles, int max_tiles,
                             cudaStream_t stream, int e0 = 0, int e1 = -1);
// The MoE layer's scratch, carved from one caller buffer (nullptr: sizes only).
// rpr routes per token (k, or k + 1 with a shared expert); shared_local adds
// the shared expert's tiles; router_cols > 0 reserves the router's partials.
struct MoeWorkspace {
  uint32_t *ids, *tiles, *grouped, *route_rows, *ntiles;
  uint16_t *weights, *xg, *h, *d;
  float *xsum, *hsum;  // group sums of xg and h: [tile][groups][32]
  float *partial;      // router partials [8][T][router_cols]
  size_t bytes;
  int max_tiles;
};
MoeWorkspace moe_workspace(int T, int H, int I, int E, int k, void *base, int rpr = -1, bool shared_local = false,
                           int router_cols = 0);
// The expert sets of one call: routed (gate, up, down) and, optionally, the
// shared expert's (one expert each).
struct MoeSets {
  const thq4_experts *gate, *up, *down;
  const thq4_experts *sgate, *sup, *sdown;
};
// The layer (y bf16) or, for an expert shard [e0, e1), its f32 partial.
cudaError_t moe_launch(const void *x, const void *residual, const MoeRouting &r, int T, int H, int I, int E, int k,
                       const MoeSets &sets, void *y, const MoeWorkspace &w, cudaStream_t stream, int e0 = 0,
                       int e1 = -1, bool y_f32 = false);

// ---- presum blocks ----------------------------------------------------------
// [8][in] bf16 rows then f32 sums [in/64][8] (thq4_presum.cu).
size_t presum_block_bytes(int in);
// add_rms_norm keeps a row of f32 x + r in shared memory
constexpr int kAddRmsNormMaxC = 32768;
cudaError_t add_rms_norm_launch(const void *x, const void *r, const void *w, int T, int C, float eps, void *res,
                                void *block, cudaStream_t stream);
cudaError_t presum_attach_launch(const void *x, int m, int in, void *block, cudaStream_t stream);

// ---- repack / dequant ------------------------------------------------------
cudaError_t repack_launch(int src_layout, const void *src_w, const void *src_sb, int src_out, int in,
                          int row_begin, int rows, void *dst_qw, void *dst_sb, cudaStream_t stream);
cudaError_t dequant_launch(const thq4_weight &w, void *y, cudaStream_t stream);

// ---- errors ----------------------------------------------------------------
thq4_status set_error(thq4_status s, const std::string &msg);
thq4_status cuda_error(cudaError_t e, const char *what);

}  // namespace thq4
