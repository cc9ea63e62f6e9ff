// thq4_api.cu -- the C ABI: argument validation, routing and error reporting.
//
// Host-side mirror of the reference's operator layer: QLin::linear_ps's
// row-count routing (engine/src/qwen35.rs:398-617), gate_up_act_ps
// (:711-884) and the candle op checks that bail before anything is encoded
// (check3, quant_kernel.rs:2671-2684; presum length check :3642-3657).
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "thq4_common.cuh"
#include "thq4_internal.h"

namespace thq4 {

__device__ uint32_t g_status = 0;

uint32_t *status_word() {
  static DeviceOnce once;
  static uint32_t *addr[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  once.run([&] { return cudaGetSymbolAddress(reinterpret_cast<void **>(&addr[dev]), g_status); });
  return addr[dev];
}

namespace {
thread_local std::string t_last_error;

bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
}  // namespace

thq4_status set_error(thq4_status s, const std::string &msg) {
  t_last_error = msg;
  return s;
}

thq4_status cuda_error(cudaError_t e, const char *what) {
  return set_error(THQ4_ERR_CUDA, std::string(what) + ": " + cudaGetErrorName(e) + " (" +
                                      cudaGetErrorString(e) + ")");
}

int device_sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

namespace {
std::atomic<int> g_force_warps{0}, g_force_depth{0}, g_force_grid{0};
}  // namespace

bool gemv_pdl_enabled() {
  static const bool on = [] {
    const char *e = std::getenv("THQ4_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

GemvCfg gemv_cfg_override() {
  GemvCfg c;
  c.warps = g_force_warps.load(std::memory_order_relaxed);
  c.depth = g_force_depth.load(std::memory_order_relaxed);
  c.grid = g_force_grid.load(std::memory_order_relaxed);
  if (c.warps || c.depth || c.grid) return c;
  // THQ4_GEMV="chunk,stages,grid,pre", read once (the reference reads its TH_QMVT /
  // TH_Q4_POLICY switches once the same way, quant_kernel.rs:41-78, 367-432)
  static const GemvCfg env = [] {
    GemvCfg e;
    const char *s = std::getenv("THQ4_GEMV");
    if (s && *s) {
      int w = 0, d = 0, g = 0, pre = 0;
      if (std::sscanf(s, "%d,%d,%d,%d", &w, &d, &g, &pre) >= 1) {
        if (w == 4 || w == 8) e.warps = w;
        if (d >= 2 && d <= 8) e.depth = d;
        if (g > 0) e.grid = g;
        if (pre > 0 && pre <= 8) e.pre = pre;
      }
    }
    return e;
  }();
  return env;
}

namespace {

thq4_status check_weight(const thq4_weight *w, const char *who) {
  if (!w) return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": weight is NULL");
  if (w->out <= 0 || w->in <= 0)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": weight has out " +
                                                    std::to_string(w->out) + ", in " + std::to_string(w->in));
  if (w->gs != kGroup)
    return set_error(THQ4_ERR_UNSUPPORTED, std::string(who) + ": group size " + std::to_string(w->gs) +
                                               " (only 64 is packed)");
  if (w->in % kGroup != 0)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": in " + std::to_string(w->in) +
                                                    " is not a multiple of 64");
  if (w->sb_dtype != THQ4_BF16 && w->sb_dtype != THQ4_F16)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": scale dtype must be bf16 or f16");
  if (!w->qw || !w->sb || !aligned(w->qw, 16) || !aligned(w->sb, 16))
    return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": weight buffers must be non-NULL and "
                                                                   "16-byte aligned");
  return THQ4_OK;
}

thq4_status check_io(const void *x, int x_dtype, int m, const void *y, int y_dtype, const char *who) {
  if (m < 1) return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": m must be >= 1");
  if (x_dtype != THQ4_BF16 && x_dtype != THQ4_F32)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": x dtype must be bf16 or f32");
  if (y_dtype != THQ4_BF16 && y_dtype != THQ4_F32)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": y dtype must be bf16 or f32");
  if (!x || !y) return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": x and y must be non-NULL");
  // the kernels read x as 16-byte vectors (the reference rejects a
  // misaligned x the same way, qwen35.rs:366, 7034-7037)
  if (!aligned(x, 16))
    return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": x must be 16-byte aligned");
  if (!aligned(y, y_dtype == THQ4_F32 ? 4 : 2))
    return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": y is misaligned");
  return THQ4_OK;
}

thq4_status check_workspace(void *ws, size_t have, size_t need, const char *who) {
  if (need == 0) return THQ4_OK;
  if (!ws || have < need || !aligned(ws, 256))
    return set_error(THQ4_ERR_WORKSPACE, std::string(who) + ": needs a 256-byte aligned, zero-filled workspace of " +
                                             std::to_string(need) + " bytes (thq4_linear_workspace_bytes), got " +
                                             std::to_string(have));
  return THQ4_OK;
}

}  // namespace
}  // namespace thq4

namespace thq4 {
namespace {

// Scratch of thq4_linear_noalloc (the split-K partials and arrival counters
// thq4_linear takes from its workspace argument): one buffer per device,
// zero when the module loads; calls leave the counters zeroed.
constexpr size_t kNoAllocScratchBytes = 6u << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on the current device, looked up once
// per device (nullptr and *err set when the lookup fails).
void *noalloc_scratch(cudaError_t *err) {
  static DeviceOnce once;
  static void *addr[64] = {nullptr};
  int dev = 0;
  *err = cudaGetDevice(&dev);
  if (*err != cudaSuccess) return nullptr;
  if (dev < 0 || dev >= 64) {
    *err = cudaErrorInvalidDevice;
    return nullptr;
  }
  *err = once.run([&] { return cudaGetSymbolAddress(&addr[dev], g_noalloc_scratch); });
  return *err == cudaSuccess ? addr[dev] : nullptr;
}

}  // namespace
}  // namespace thq4

using namespace thq4;

extern "C" {

const char *thq4_version(void) { return "thq4 " THQ4_SEMVER " sm_100a"; }

size_t thq4_last_error(char *buf, size_t cap) {
  const std::string &s = t_last_error;
  if (buf && cap) {
    const size_t n = s.size() < cap - 1 ? s.size() : cap - 1;
    std::memcpy(buf, s.data(), n);
    buf[n] = '\0';
  }
  return s.size();
}

thq4_status thq4_device_status(uint32_t *status_out, void *stream) {
  if (!status_out) return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_device_status: status_out is NULL");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t zero = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(status_out, g_status, sizeof(uint32_t), 0, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaMemcpyToSymbolAsync(g_status, &zero, sizeof(uint32_t), 0, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_error(e, "thq4_device_status");
  return THQ4_OK;
}

size_t thq4_weight_bytes(int rows, int in, int gs, size_t *qw_bytes, size_t *sb_bytes) {
  size_t q = 0, s = 0;
  if (rows > 0 && in > 0 && gs == kGroup && in % kGroup == 0) {
    const size_t chunks = (size_t)row_slabs(rows) * kSlabTiles * (size_t)(in / kGroup);
    q = chunks * kChunkBytes;
    s = chunks * kQuadBytes;
  }
  if (qw_bytes) *qw_bytes = q;
  if (sb_bytes) *sb_bytes = s;
  return q + s;
}

thq4_status thq4_repack(int src_layout, const void *src_w, const void *src_sb, int src_out, int in, int gs,
                        int sb_dtype, int row_begin, int rows, void *dst_qw, size_t dst_qw_bytes, void *dst_sb,
                        size_t dst_sb_bytes, void *stream) {
  const char *who = "thq4_repack";
  if (src_layout < THQ4_SRC_MLX || src_layout > THQ4_SRC_FRAG)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_repack: unknown source layout");
  if (gs != kGroup) return set_error(THQ4_ERR_UNSUPPORTED, "thq4_repack: only group size 64 is packed");
  if (sb_dtype != THQ4_BF16 && sb_dtype != THQ4_F16)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_repack: scale dtype must be bf16 or f16");
  if (src_out <= 0 || in <= 0 || in % kGroup != 0)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": bad shape " + std::to_string(src_out) +
                                                    " x " + std::to_string(in));
  if (rows <= 0 || row_begin < 0 || row_begin + rows > src_out)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": row range [" + std::to_string(row_begin) +
                                                    ", " + std::to_string(row_begin + rows) + ") outside " +
                                                    std::to_string(src_out) + " rows");
  if (src_layout == THQ4_SRC_SLAB && src_out % 256 != 0)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_repack: a slab needs out % 256 == 0 (StorageN=256)");
  if (src_layout == THQ4_SRC_FRAG && (row_begin != 0 || rows != src_out))
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_repack: a frag source is copied whole");
  if (!src_w || (src_layout != THQ4_SRC_SLAB && !src_sb))
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_repack: source pointers must be non-NULL");
  if (!aligned(src_w, 16) || (src_sb && !aligned(src_sb, 2)) ||
      (src_layout == THQ4_SRC_FRAG && !aligned(src_sb, 16)))
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_repack: source weights must be 16-byte aligned");
  size_t need_q = 0, need_s = 0;
  thq4_weight_bytes(rows, in, gs, &need_q, &need_s);
  if (!dst_qw || !dst_sb || !aligned(dst_qw, 16) || !aligned(dst_sb, 16))
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_repack: destination buffers must be 16-byte aligned");
  if (dst_qw_bytes < need_q || dst_sb_bytes < need_s)
    return set_error(THQ4_ERR_INVALID_ARGUMENT,
                     std::string(who) + ": destination too small (need " + std::to_string(need_q) + " + " +
                         std::to_string(need_s) + " bytes)");
  cudaError_t e = repack_launch(src_layout, src_w, src_sb, src_out, in, row_begin, rows, dst_qw, dst_sb,
                                static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, who);
  return THQ4_OK;
}

thq4_status thq4_weight_init(thq4_weight *w, int out, int in, int gs, int sb_dtype, const void *qw,
                             const void *sb) {
  if (!w) return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_weight_init: w is NULL");
  thq4_weight t{out, in, gs, sb_dtype, qw, sb};
  thq4_status s = check_weight(&t, "thq4_weight_init");
  if (s != THQ4_OK) return s;
  *w = t;
  return THQ4_OK;
}

size_t thq4_linear_workspace_bytes(const thq4_weight *w, int m) {
  if (!w || w->out <= 0 || w->in <= 0) return 0;
  return std::max(gemv_workspace_bytes(w->out), prefill_workspace_bytes(*w, m));
}

namespace {
// x given as a presum block (x_dtype THQ4_PRESUM): m <= 8 rows of bf16 in an
// [8][in] block followed by its sums; the checks of quant_kernel.rs:3642-3657
// that the host can make (the block's length is the caller's to provide:
// thq4_presum_block_bytes).
thq4_status check_presum_x(const void *x, int m, const void *y, int y_dtype, const char *who) {
  thq4_status s = check_io(x, THQ4_BF16, m, y, y_dtype, who);
  if (s != THQ4_OK) return s;
  if (m > 8)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": a presum block holds at most 8 rows (m " +
                                                    std::to_string(m) + ")");
  return THQ4_OK;
}
}  // namespace

thq4_status thq4_linear(const thq4_weight *w, const void *x, int x_dtype, int m, void *y, int y_dtype,
                        void *workspace, size_t workspace_bytes, void *stream) {
  thq4_status s = check_weight(w, "thq4_linear");
  if (s != THQ4_OK) return s;
  if (x_dtype == THQ4_PRESUM) {
    if ((s = check_presum_x(x, m, y, y_dtype, "thq4_linear")) != THQ4_OK) return s;
    if ((s = check_workspace(workspace, workspace_bytes, gemv_workspace_bytes(w->out), "thq4_linear")) != THQ4_OK)
      return s;
    const cudaError_t e = gemv_launch(*w, nullptr, x, false, m, y, y_dtype == THQ4_F32, workspace,
                                      static_cast<cudaStream_t>(stream), nullptr, true);
    if (e != cudaSuccess) return cuda_error(e, "thq4_linear (presum)");
    return THQ4_OK;
  }
  s = check_io(x, x_dtype, m, y, y_dtype, "thq4_linear");
  if (s != THQ4_OK) return s;
  if (prefill_supported(m, x_dtype == THQ4_F32)) {
    const cudaError_t e = prefill_launch(*w, nullptr, x, m, y, y_dtype == THQ4_F32, workspace, workspace_bytes,
                                         static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_error(e, "thq4_linear (prefill)");
    return THQ4_OK;
  }
  s = check_workspace(workspace, workspace_bytes, gemv_workspace_bytes(w->out), "thq4_linear");
  if (s != THQ4_OK) return s;
  cudaError_t e = gemv_launch(*w, nullptr, x, x_dtype == THQ4_F32, m, y, y_dtype == THQ4_F32, workspace,
                              static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, "thq4_linear");
  return THQ4_OK;
}

thq4_status thq4_linear_noalloc(const thq4_weight *w, const void *x, int x_dtype, int m, void *y, int y_dtype,
                                void *stream) {
  const char *who = "thq4_linear_noalloc";
  thq4_status s = check_weight(w, who);
  if (s != THQ4_OK) return s;
  s = check_io(x, x_dtype, m, y, y_dtype, who);
  if (s != THQ4_OK) return s;
  // the same row-count routing as thq4_linear: the prefill kernel needs no
  // scratch at all
  if (prefill_supported(m, x_dtype == THQ4_F32)) {
    const cudaError_t e =
        prefill_launch(*w, nullptr, x, m, y, y_dtype == THQ4_F32, nullptr, 0, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_error(e, "thq4_linear_noalloc (prefill)");
    return THQ4_OK;
  }
  const size_t need = gemv_workspace_bytes(w->out);
  if (need > kNoAllocScratchBytes)
    return set_error(THQ4_ERR_UNSUPPORTED, std::string(who) + ": a " + std::to_string(w->out) +
                                               "-row weight needs " + std::to_string(need) +
                                               " bytes of scratch, above the built-in " +
                                               std::to_string(kNoAllocScratchBytes) + "; use thq4_linear");
  cudaError_t e = cudaSuccess;
  void *scratch = noalloc_scratch(&e);
  if (!scratch) return cuda_error(e, "thq4_linear_noalloc: cudaGetSymbolAddress");
  e = gemv_launch(*w, nullptr, x, x_dtype == THQ4_F32, m, y, y_dtype == THQ4_F32, scratch,
                  static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, who);
  return THQ4_OK;
}

thq4_status thq4_linear_scalar(const thq4_weight *w, const void *x, int x_dtype, int m, void *y, int y_dtype,
                               void *stream) {
  const char *who = "thq4_linear_scalar";
  thq4_status s = check_weight(w, who);
  if (s != THQ4_OK) return s;
  if ((s = check_io(x, x_dtype, m, y, y_dtype, who)) != THQ4_OK) return s;
  const cudaError_t e = scalar_launch(*w, x, x_dtype == THQ4_F32, m, y, y_dtype == THQ4_F32,
                                      static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, who);
  return THQ4_OK;
}

size_t thq4_linear_chain_workspace_bytes(const thq4_chain_op *ops, int n) {
  if (!ops || n < 1) return 0;
  int rows = 0;
  for (int i = 0; i < n; ++i)
    if (ops[i].w && ops[i].w->out > rows) rows = ops[i].w->out;
  return rows > 0 ? chain_workspace_bytes(rows) : 0;
}

thq4_status thq4_linear_chain(const thq4_chain_op *ops, int n, int x_dtype, int m, void *workspace,
                              size_t workspace_bytes, void *stream) {
  const char *who = "thq4_linear_chain";
  if (!ops || n < 1 || n > chain_max_ops())
    return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": need 1 <= n <= " +
                                                    std::to_string(chain_max_ops()) + " ops");
  const int per = x_dtype == THQ4_F32 ? 4 : 8;
  if (m < 1 || m > per)
    return set_error(THQ4_ERR_UNSUPPORTED, std::string(who) + ": m " + std::to_string(m) + " outside 1.." +
                                               std::to_string(per) + " (one decode/verify pass per op)");
  ChainSpec spec[128];
  int rows = 0;
  for (int i = 0; i < n; ++i) {
    const thq4_chain_op &o = ops[i];
    const std::string at = std::string(who) + " op " + std::to_string(i);
    thq4_status s = check_weight(o.w, at.c_str());
    if (s != THQ4_OK) return s;
    if (o.up) {
      if ((s = check_weight(o.up, at.c_str())) != THQ4_OK) return s;
      if (o.w->out != o.up->out || o.w->in != o.up->in || o.w->sb_dtype != o.up->sb_dtype)
        return set_error(THQ4_ERR_INVALID_ARGUMENT, at + ": gate and up halves differ in shape or dtype");
    }
    if (o.w->sb_dtype != ops[0].w->sb_dtype)
      return set_error(THQ4_ERR_INVALID_ARGUMENT, at + ": every op of a chain has the same scale dtype");
    if (o.reserved != 0) return set_error(THQ4_ERR_INVALID_ARGUMENT, at + ": reserved must be 0");
    if ((s = check_io(o.x, x_dtype, m, o.y, o.y_dtype, at.c_str())) != THQ4_OK) return s;
    if (o.x == o.y) return set_error(THQ4_ERR_INVALID_ARGUMENT, at + ": y aliases x");
    spec[i] = ChainSpec{o.w, o.up, o.x, o.y, o.y_dtype == THQ4_F32};
    rows = std::max(rows, (int)o.w->out);
  }
  thq4_status s = check_workspace(workspace, workspace_bytes, chain_workspace_bytes(rows), who);
  if (s != THQ4_OK) return s;
  const cudaError_t e =
      chain_launch(spec, n, x_dtype == THQ4_F32, m, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, who);
  return THQ4_OK;
}

thq4_status thq4_gate_up(const thq4_weight *gate, const thq4_weight *up, const void *x, int x_dtype, int m,
                         void *y, int y_dtype, void *workspace, size_t workspace_bytes, void *stream) {
  thq4_status s = check_weight(gate, "thq4_gate_up");
  if (s != THQ4_OK) return s;
  s = check_weight(up, "thq4_gate_up");
  if (s != THQ4_OK) return s;
  if (gate->out != up->out || gate->in != up->in || gate->sb_dtype != up->sb_dtype)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_gate_up: gate and up halves differ in shape or dtype");
  if (x_dtype == THQ4_PRESUM) {
    if ((s = check_presum_x(x, m, y, y_dtype, "thq4_gate_up")) != THQ4_OK) return s;
    if ((s = check_workspace(workspace, workspace_bytes, gemv_workspace_bytes(gate->out), "thq4_gate_up")) != THQ4_OK)
      return s;
    const cudaError_t e = gemv_launch(*gate, up, x, false, m, y, y_dtype == THQ4_F32, workspace,
                                      static_cast<cudaStream_t>(stream), nullptr, true);
    if (e != cudaSuccess) return cuda_error(e, "thq4_gate_up (presum)");
    return THQ4_OK;
  }
  s = check_io(x, x_dtype, m, y, y_dtype, "thq4_gate_up");
  if (s != THQ4_OK) return s;
  if (prefill_supported(m, x_dtype == THQ4_F32)) {
    const cudaError_t e =
        prefill_launch(*gate, up, x, m, y, y_dtype == THQ4_F32, nullptr, 0, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_error(e, "thq4_gate_up (prefill)");
    return THQ4_OK;
  }
  s = check_workspace(workspace, workspace_bytes, gemv_workspace_bytes(gate->out), "thq4_gate_up");
  if (s != THQ4_OK) return s;
  cudaError_t e = gemv_launch(*gate, up, x, x_dtype == THQ4_F32, m, y, y_dtype == THQ4_F32, workspace,
                              static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, "thq4_gate_up");
  return THQ4_OK;
}

namespace {
thq4_status check_peer(const thq4_peer_gather *g, const char *who) {
  const std::string pre = std::string(who) + ": ";
  if (!g) return set_error(THQ4_ERR_INVALID_ARGUMENT, pre + "peer gather is NULL");
  if (g->world < 1 || g->world > 8 || g->rank < 0 || g->rank >= g->world)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, pre + "need 1 <= world <= 8 and 0 <= rank < world (world " +
                                                    std::to_string(g->world) + ", rank " + std::to_string(g->rank) + ")");
  if (g->out_mode < 0 || g->out_mode > 3)
    return set_error(THQ4_ERR_INVALID_ARGUMENT,
                     pre + "out_mode must be 0 (gather), 1 (reduce), 2 (local) or 3 (low-latency reduce)");
  if (g->x_ll != 0 && g->x_ll != 1) return set_error(THQ4_ERR_INVALID_ARGUMENT, pre + "x_ll must be 0 or 1");
  if (g->x_ll && (g->x_parts < 1 || g->wait))
    return set_error(THQ4_ERR_INVALID_ARGUMENT, pre + "x_ll needs x_parts > 0 and wait 0 (the words are the signal)");
  if (g->reserved != 0) return set_error(THQ4_ERR_INVALID_ARGUMENT, pre + "reserved must be 0");
  if (g->wait != 0 && g->wait != 1) return set_error(THQ4_ERR_INVALID_ARGUMENT, pre + "wait must be 0 or 1");
  if (!g->flags || !g->count || (g->out_mode != 2 && (!g->dst || !g->arrive)))
    return set_error(THQ4_ERR_INVALID_ARGUMENT, pre + "dst, flags, count and arrive must be device pointers");
  if (g->x_parts < 0 || g->x_parts > 8)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, pre + "x_parts must be 0 .. 8");
  return THQ4_OK;
}

PeerGather peer_of(const thq4_peer_gather *g) {
  PeerGather pg{reinterpret_cast<uint16_t *const *>(g->dst), g->flags, g->count, g->arrive, g->world, g->rank,
                g->rows, g->offset, g->stride, g->wait};
  pg.mode = g->out_mode == 0 ? 1 : g->out_mode == 1 ? 2 : g->out_mode == 3 ? 3 : 0;
  pg.slot = g->slot;
  pg.x_parts = g->x_parts;
  pg.x_slot = g->x_slot;
  pg.x_ll = g->x_ll;
  return pg;
}
}  // namespace

thq4_status thq4_linear_peer(const thq4_weight *w, const thq4_weight *up, const void *x, int x_dtype, int m, void *y,
                             void *workspace, size_t workspace_bytes, const thq4_peer_gather *g, void *stream) {
  const char *who = "thq4_linear_peer";
  thq4_status s = check_weight(w, who);
  if (s != THQ4_OK) return s;
  if (up) {
    if ((s = check_weight(up, who)) != THQ4_OK) return s;
    if (w->out != up->out || w->in != up->in || w->sb_dtype != up->sb_dtype)
      return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_linear_peer: gate and up halves differ in shape or dtype");
  }
  if ((s = check_peer(g, who)) != THQ4_OK) return s;
  const bool reduce = g->out_mode == 1 || g->out_mode == 3;
  // reduce mode stores no y: check the rest of the I/O against x alone
  if ((s = check_io(x, x_dtype, m, reduce ? x : y, THQ4_BF16, who)) != THQ4_OK) return s;
  const bool parts = g->x_parts > 0;
  if (parts && x_dtype != THQ4_F32)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_linear_peer: x partials are f32 (x_dtype THQ4_F32)");
  const int per = x_dtype == THQ4_F32 && !parts ? 4 : 8;
  if (m > per)
    return set_error(THQ4_ERR_UNSUPPORTED, "thq4_linear_peer: m " + std::to_string(m) + " > " + std::to_string(per) +
                                               " (one decode/verify launch per exchanged call)");
  if (parts && (g->x_slot < (long long)m * w->in || g->x_slot % 4))
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_linear_peer: x_slot must be >= m * in and a multiple of 4");
  if (g->out_mode == 0 &&
      (g->rows < 0 || g->rows > w->out || g->offset < 0 || g->stride < 1 || (long long)g->offset + g->rows > g->stride))
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_linear_peer: need 0 <= rows <= out and offset + rows <= stride");
  if (reduce && (g->rows != w->out || g->offset != 0 || g->stride < w->out || g->slot < (long long)m * g->stride))
    return set_error(THQ4_ERR_INVALID_ARGUMENT,
                     "thq4_linear_peer: reduce needs rows == out, offset 0, stride >= out and slot >= m * stride");
  if (reduce && up)
    return set_error(THQ4_ERR_UNSUPPORTED, "thq4_linear_peer: a gate/up pair is column-sharded (no reduce)");
  if ((s = check_workspace(workspace, workspace_bytes, gemv_workspace_bytes(w->out), who)) != THQ4_OK) return s;
  const PeerGather pg = peer_of(g);
  const cudaError_t e = gemv_launch(*w, up, x, x_dtype == THQ4_F32 && !parts, m, reduce ? nullptr : y, false,
                                    workspace, static_cast<cudaStream_t>(stream), &pg);
  if (e != cudaSuccess) return cuda_error(e, who);
  return THQ4_OK;
}

thq4_status thq4_peer_wait(const thq4_peer_gather *g, void *stream) {
  thq4_status s = check_peer(g, "thq4_peer_wait");
  if (s != THQ4_OK) return s;
  const PeerGather pg = peer_of(g);
  const cudaError_t e = peer_wait_launch(pg, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, "thq4_peer_wait");
  return THQ4_OK;
}

thq4_status thq4_ipc_alloc(size_t bytes, void **ptr, void *handle) {
  if (!ptr || !handle || bytes == 0) return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_ipc_alloc: bad arguments");
  static_assert(sizeof(cudaIpcMemHandle_t) == THQ4_IPC_HANDLE_BYTES, "IPC handle size");
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_error(e, "thq4_ipc_alloc");
  if ((e = cudaMemset(p, 0, bytes)) != cudaSuccess || (e = cudaDeviceSynchronize()) != cudaSuccess) {
    cudaFree(p);
    return cuda_error(e, "thq4_ipc_alloc");
  }
  cudaIpcMemHandle_t h;
  if ((e = cudaIpcGetMemHandle(&h, p)) != cudaSuccess) {
    cudaFree(p);
    return cuda_error(e, "thq4_ipc_alloc");
  }
  std::memcpy(handle, &h, sizeof h);
  *ptr = p;
  return THQ4_OK;
}

thq4_status thq4_ipc_open(const void *handle, void **ptr) {
  if (!ptr || !handle) return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_ipc_open: bad arguments");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof h);
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_error(e, "thq4_ipc_open");
  return THQ4_OK;
}

thq4_status thq4_ipc_close(void *ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return cuda_error(e, "thq4_ipc_close");
  return THQ4_OK;
}

thq4_status thq4_ipc_free(void *ptr) {
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return cuda_error(e, "thq4_ipc_free");
  return THQ4_OK;
}

thq4_status thq4_copy(void *dst, const void *src, size_t bytes, void *stream) {
  if ((!dst || !src) && bytes) return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_copy: NULL pointer");
  const cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, "thq4_copy");
  return THQ4_OK;
}

thq4_status thq4_dequant(const thq4_weight *w, void *y, void *stream) {
  thq4_status s = check_weight(w, "thq4_dequant");
  if (s != THQ4_OK) return s;
  if (!y || !aligned(y, 16)) return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_dequant: y must be 16-byte aligned");
  cudaError_t e = dequant_launch(*w, y, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, "thq4_dequant");
  return THQ4_OK;
}

uint32_t thq4_moe_max_tiles(int T, int E, int k) {
  if (T <= 0 || E <= 0 || k <= 0) return 0;
  return moe_max_tiles(T, E, k);
}

namespace {
thq4_status check_route_args(int T, int E, int k, const char *who) {
  if (T < 1 || E < 1 || E > 1024 || k < 1 || k > E || k > 32)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": need T >= 1, 1 <= E <= 1024, 1 <= k <= min(E, 32) "
                                                                   "(T " + std::to_string(T) + ", E " +
                                                    std::to_string(E) + ", k " + std::to_string(k) + ")");
  if (moe_group_smem(T * k, E) > 200 * 1024)
    return set_error(THQ4_ERR_UNSUPPORTED, std::string(who) + ": " + std::to_string((long long)T * k) +
                                               " routes exceed the grouping kernel's shared memory");
  return THQ4_OK;
}
thq4_status check_experts(const thq4_experts *w, int E, int out, int in, const char *what, const char *who) {
  const std::string pre = std::string(who) + ": " + what;
  if (!w) return set_error(THQ4_ERR_INVALID_ARGUMENT, pre + " experts are NULL");
  if (w->experts != E || w->out != out || w->in != in)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, pre + " experts are " + std::to_string(w->experts) + " x " +
                                                    std::to_string(w->out) + " x " + std::to_string(w->in) +
                                                    ", expected " + std::to_string(E) + " x " + std::to_string(out) +
                                                    " x " + std::to_string(in));
  if (w->gs != kGroup) return set_error(THQ4_ERR_UNSUPPORTED, pre + ": only group size 64 is packed");
  if (w->sb_dtype != THQ4_BF16 && w->sb_dtype != THQ4_F16)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, pre + ": scale dtype must be bf16 or f16");
  size_t qb = 0, sbb = 0;
  thq4_weight_bytes(out, in, kGroup, &qb, &sbb);
  if (!w->qw || !w->sb || !aligned(w->qw, 16) || !aligned(w->sb, 16) || w->qw_stride % 16 || w->sb_stride % 16 ||
      w->qw_stride < qb || w->sb_stride < sbb)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, pre + ": buffers must be 16-byte aligned with per-expert strides >= " +
                                                    std::to_string(qb) + " / " + std::to_string(sbb) + " bytes");
  return THQ4_OK;
}
}  // namespace

thq4_status thq4_moe_route(const void *logits, int T, int E, int k, uint32_t *ids, void *weights, uint32_t *tiles,
                           uint32_t *grouped_routes, uint32_t *route_rows, uint32_t *ntiles, int max_tiles,
                           void *stream) {
  const char *who = "thq4_moe_route";
  thq4_status s = check_route_args(T, E, k, who);
  if (s != THQ4_OK) return s;
  if (!logits || !ids || !weights || !tiles || !grouped_routes || !route_rows || !ntiles)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_moe_route: pointers must be non-NULL");
  if (!aligned(logits, 2) || !aligned(weights, 2) || !aligned(ids, 4) || !aligned(tiles, 4) ||
      !aligned(grouped_routes, 4) || !aligned(route_rows, 4) || !aligned(ntiles, 4))
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_moe_route: misaligned buffer");
  if (max_tiles < (int)moe_max_tiles(T, E, k))
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_moe_route: max_tiles below thq4_moe_max_tiles(T, E, k) = " +
                                                    std::to_string(moe_max_tiles(T, E, k)));
  MoeRouting rt{};
  rt.logits = static_cast<const uint16_t *>(logits);
  cudaError_t e = moe_route_launch(rt, T, E, k, ids, static_cast<uint16_t *>(weights), tiles, grouped_routes, route_rows,
                                   ntiles, max_tiles, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, who);
  return THQ4_OK;
}

size_t thq4_moe_workspace_bytes(int T, int H, int I, int E, int k) {
  if (T <= 0 || H <= 0 || I <= 0 || E <= 0 || k <= 0) return 0;
  return moe_workspace(T, H, I, E, k, nullptr).bytes;
}

thq4_status thq4_moe(const void *x, const void *residual, const void *logits, int T, int H, int I, int E, int k,
                     const thq4_experts *gate, const thq4_experts *up, const thq4_experts *down, void *y,
                     void *workspace, size_t workspace_bytes, void *stream) {
  const char *who = "thq4_moe";
  thq4_status s = check_route_args(T, E, k, who);
  if (s != THQ4_OK) return s;
  if (H <= 0 || I <= 0 || H % kGroup || I % kGroup)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_moe: H and I must be positive multiples of 64");
  if ((s = check_experts(gate, E, I, H, "gate", who)) != THQ4_OK) return s;
  if ((s = check_experts(up, E, I, H, "up", who)) != THQ4_OK) return s;
  if ((s = check_experts(down, E, H, I, "down", who)) != THQ4_OK) return s;
  if (gate->sb_dtype != up->sb_dtype || gate->sb_dtype != down->sb_dtype)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_moe: gate, up and down differ in scale dtype");
  if (!x || !y || !logits || !aligned(x, 16) || !aligned(y, 16) || !aligned(logits, 2) ||
      (residual && !aligned(residual, 16)))
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_moe: x, y (and residual) must be 16-byte aligned, logits non-NULL");
  const MoeWorkspace need = moe_workspace(T, H, I, E, k, nullptr);
  if (!workspace || workspace_bytes < need.bytes || !aligned(workspace, 256))
    return set_error(THQ4_ERR_WORKSPACE, "thq4_moe: needs a 256-byte aligned workspace of " + std::to_string(need.bytes) +
                                             " bytes (thq4_moe_workspace_bytes), got " + std::to_string(workspace_bytes));
  const MoeWorkspace w = moe_workspace(T, H, I, E, k, workspace);
  MoeRouting rt{};
  rt.logits = static_cast<const uint16_t *>(logits);
  const MoeSets sets{gate, up, down, nullptr, nullptr, nullptr};
  cudaError_t e = moe_launch(x, residual, rt, T, H, I, E, k, sets, y, w, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, who);
  return THQ4_OK;
}

thq4_status thq4_moe_partial(const void *x, const void *residual, const void *logits, int T, int H, int I, int E,
                             int k, int e0, int e1, const thq4_experts *gate, const thq4_experts *up,
                             const thq4_experts *down, float *y_part, void *workspace, size_t workspace_bytes,
                             void *stream) {
  const char *who = "thq4_moe_partial";
  thq4_status s = check_route_args(T, E, k, who);
  if (s != THQ4_OK) return s;
  if (e0 < 0 || e1 <= e0 || e1 > E)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_moe_partial: need 0 <= e0 < e1 <= E (e0 " + std::to_string(e0) +
                                                    ", e1 " + std::to_string(e1) + ", E " + std::to_string(E) + ")");
  if (H <= 0 || I <= 0 || H % kGroup || I % kGroup)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_moe_partial: H and I must be positive multiples of 64");
  const int El = e1 - e0;
  if ((s = check_experts(gate, El, I, H, "gate", who)) != THQ4_OK) return s;
  if ((s = check_experts(up, El, I, H, "up", who)) != THQ4_OK) return s;
  if ((s = check_experts(down, El, H, I, "down", who)) != THQ4_OK) return s;
  if (gate->sb_dtype != up->sb_dtype || gate->sb_dtype != down->sb_dtype)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_moe_partial: gate, up and down differ in scale dtype");
  if (!x || !y_part || !logits || !aligned(x, 16) || !aligned(y_part, 16) || !aligned(logits, 2) ||
      (residual && !aligned(residual, 16)))
    return set_error(THQ4_ERR_INVALID_ARGUMENT,
                     "thq4_moe_partial: x, y_part (and residual) must be 16-byte aligned, logits non-NULL");
  const MoeWorkspace need = moe_workspace(T, H, I, El, k, nullptr);
  if (!workspace || workspace_bytes < need.bytes || !aligned(workspace, 256))
    return set_error(THQ4_ERR_WORKSPACE, "thq4_moe_partial: needs a 256-byte aligned workspace of " +
                                             std::to_string(need.bytes) +
                                             " bytes (thq4_moe_workspace_bytes with E = e1 - e0), got " +
                                             std::to_string(workspace_bytes));
  const MoeWorkspace w = moe_workspace(T, H, I, El, k, workspace);
  MoeRouting rt{};
  rt.logits = static_cast<const uint16_t *>(logits);
  const MoeSets sets{gate, up, down, nullptr, nullptr, nullptr};
  cudaError_t e = moe_launch(x, residual, rt, T, H, I, E, k, sets, y_part, w, static_cast<cudaStream_t>(stream), e0,
                             e1, true);
  if (e != cudaSuccess) return cuda_error(e, who);
  return THQ4_OK;
}

// ---- the Splash MoE block: Q8 router, shared expert --------------------------

namespace {
thq4_status check_q8(const thq4_q8_weight *w, int in, const char *what, const char *who) {
  const std::string pre = std::string(who) + ": " + what;
  if (!w) return set_error(THQ4_ERR_INVALID_ARGUMENT, pre + " is NULL");
  if (w->out != 256 || w->in != in)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, pre + " is " + std::to_string(w->out) + " x " + std::to_string(w->in) +
                                                    ", expected 256 x " + std::to_string(in));
  if (!w->q || !w->scales || !w->biases || !aligned(w->q, 16) || !aligned(w->scales, 2) || !aligned(w->biases, 2))
    return set_error(THQ4_ERR_INVALID_ARGUMENT, pre + ": q must be 16-byte aligned, scales and biases non-NULL");
  return THQ4_OK;
}

bool has_shared(const thq4_moe_weights *w) { return w->shared_expert_gate.q != nullptr; }
bool runs_shared(const thq4_moe_weights *w) { return w->shared_gate.qw != nullptr; }

// MoE::add's validate (MoE.cpp:14-58) for a call holding experts [e0, e1) of E.
thq4_status check_moe_add(int T, int H, int I, int E, int k, int e0, int e1, const thq4_moe_weights *w,
                          const char *who) {
  if (!w) return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": weights are NULL");
  if (T < 1 || H <= 0 || H % 256 || I <= 0 || I % 256 || E < 1 || E > 256 || k < 1 || k > E || k > 32)
    return set_error(THQ4_ERR_INVALID_ARGUMENT,
                     std::string(who) + ": MoE weights do not match execution shape (need T >= 1, H and I multiples "
                                        "of 256, 1 <= k <= E <= 256, k <= 32; T " + std::to_string(T) + ", H " +
                         std::to_string(H) + ", I " + std::to_string(I) + ", E " + std::to_string(E) + ", k " +
                         std::to_string(k) + ")");
  if (e0 < 0 || e1 <= e0 || e1 > E)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": need 0 <= e0 < e1 <= E");
  const int El = e1 - e0, rpr = k + (has_shared(w) ? 1 : 0);
  if (moe_group_smem(T * rpr, El) > 200 * 1024)
    return set_error(THQ4_ERR_UNSUPPORTED, std::string(who) + ": " + std::to_string((long long)T * rpr) +
                                               " routes exceed the grouping kernel's shared memory");
  thq4_status s;
  if ((s = check_q8(&w->router, H, "router", who)) != THQ4_OK) return s;
  if ((s = check_experts(&w->gate, El, I, H, "gate", who)) != THQ4_OK) return s;
  if ((s = check_experts(&w->up, El, I, H, "up", who)) != THQ4_OK) return s;
  if ((s = check_experts(&w->down, El, H, I, "down", who)) != THQ4_OK) return s;
  const int dt = w->gate.sb_dtype;
  if (w->up.sb_dtype != dt || w->down.sb_dtype != dt)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": expert scale dtypes differ");
  if (runs_shared(w) && !has_shared(w))
    return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": a shared expert needs its shared_expert_gate");
  if (has_shared(w) && (s = check_q8(&w->shared_expert_gate, H, "shared_expert_gate", who)) != THQ4_OK) return s;
  if (runs_shared(w)) {
    if ((s = check_experts(&w->shared_gate, 1, I, H, "shared gate", who)) != THQ4_OK) return s;
    if ((s = check_experts(&w->shared_up, 1, I, H, "shared up", who)) != THQ4_OK) return s;
    if ((s = check_experts(&w->shared_down, 1, H, I, "shared down", who)) != THQ4_OK) return s;
    if (w->shared_gate.sb_dtype != dt || w->shared_up.sb_dtype != dt || w->shared_down.sb_dtype != dt)
      return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": expert scale dtypes differ");
  }
  return THQ4_OK;
}

thq4_status moe_add_common(const void *x, const void *residual, int T, int H, int I, int E, int k, int e0, int e1,
                           const thq4_moe_weights *w, void *y, bool y_f32, void *workspace, size_t workspace_bytes,
                           void *stream, const char *who) {
  thq4_status s = check_moe_add(T, H, I, E, k, e0, e1, w, who);
  if (s != THQ4_OK) return s;
  if (!x || !y || !aligned(x, 16) || !aligned(y, 16) || (residual && !aligned(residual, 16)))
    return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": x, y (and residual) must be 16-byte aligned");
  const int El = e1 - e0, rpr = k + (has_shared(w) ? 1 : 0);
  const MoeWorkspace need = moe_workspace(T, H, I, El, k, nullptr, rpr, runs_shared(w), E);
  if (!workspace || workspace_bytes < need.bytes || !aligned(workspace, 256))
    return set_error(THQ4_ERR_WORKSPACE, std::string(who) + ": MoE grouped scratch is smaller than its bound (needs a "
                                                            "256-byte aligned workspace of " +
                                             std::to_string(need.bytes) + " bytes; got " +
                                             std::to_string(workspace_bytes) + ")");
  const MoeWorkspace ws = moe_workspace(T, H, I, El, k, workspace, rpr, runs_shared(w), E);
  MoeRouting rt{};
  rt.x = x;
  rt.H = H;
  rt.router = &w->router;
  rt.shared_gate = has_shared(w) ? &w->shared_expert_gate : nullptr;
  rt.shared_local = runs_shared(w);
  rt.partial = ws.partial;
  const MoeSets sets{&w->gate, &w->up, &w->down, &w->shared_gate, &w->shared_up, &w->shared_down};
  cudaError_t e = moe_launch(x, residual, rt, T, H, I, E, k, sets, y, ws, static_cast<cudaStream_t>(stream), e0, e1,
                             y_f32);
  if (e != cudaSuccess) return cuda_error(e, who);
  return THQ4_OK;
}
}  // namespace

size_t thq4_moe_scores_workspace_bytes(int T, int ncols) {
  if (T <= 0 || ncols <= 0) return 0;
  return moe_scores_bytes(T, ncols);
}

thq4_status thq4_moe_scores_q8(const void *x, int T, const thq4_q8_weight *router, int ncols, void *scores, int ld,
                               void *workspace, size_t workspace_bytes, void *stream) {
  const char *who = "thq4_moe_scores_q8";
  if (!router) return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_moe_scores_q8: router is NULL");
  if (T < 1 || ncols < 1 || ncols > 256 || ld < ncols || router->in <= 0 || router->in % kGroup)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_moe_scores_q8: need T >= 1, 1 <= ncols <= 256, ld >= ncols, "
                                                "router input a positive multiple of 64");
  thq4_status s = check_q8(router, router->in, "router", who);
  if (s != THQ4_OK) return s;
  if (!x || !scores || !aligned(x, 16) || !aligned(scores, 2))
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_moe_scores_q8: x must be 16-byte aligned, scores non-NULL");
  if (!workspace || workspace_bytes < moe_scores_bytes(T, ncols) || !aligned(workspace, 16))
    return set_error(THQ4_ERR_WORKSPACE, "thq4_moe_scores_q8: needs a 16-byte aligned workspace of " +
                                             std::to_string(moe_scores_bytes(T, ncols)) + " bytes");
  cudaError_t e = moe_scores_launch(x, T, router->in, *router, ncols, static_cast<float *>(workspace),
                                    static_cast<uint16_t *>(scores), ld, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, who);
  return THQ4_OK;
}

uint32_t thq4_moe_add_max_tiles(int T, int E, int k, int shared) {
  if (T <= 0 || E <= 0 || k <= 0) return 0;
  return moe_max_tiles(T, E, k, shared != 0);
}

thq4_status thq4_moe_route_q8(const void *x, int T, int E, int k, const thq4_q8_weight *router,
                              const thq4_q8_weight *shared_expert_gate, uint32_t *ids, void *weights, uint32_t *tiles,
                              uint32_t *grouped_routes, uint32_t *route_rows, uint32_t *ntiles, int max_tiles,
                              void *workspace, size_t workspace_bytes, void *stream) {
  const char *who = "thq4_moe_route_q8";
  if (T < 1 || E < 1 || E > 256 || k < 1 || k > E || k > 32)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_moe_route_q8: need T >= 1, 1 <= k <= E <= 256, k <= 32");
  if (!router) return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_moe_route_q8: router is NULL");
  const int H = router->in;
  if (H <= 0 || H % kGroup)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_moe_route_q8: router input must be a positive multiple of 64");
  thq4_status s = check_q8(router, H, "router", who);
  if (s != THQ4_OK) return s;
  if (shared_expert_gate && (s = check_q8(shared_expert_gate, H, "shared_expert_gate", who)) != THQ4_OK) return s;
  const int rpr = k + (shared_expert_gate ? 1 : 0);
  if (moe_group_smem(T * rpr, E) > 200 * 1024)
    return set_error(THQ4_ERR_UNSUPPORTED, "thq4_moe_route_q8: too many routes for the grouping kernel");
  if (!x || !ids || !weights || !tiles || !grouped_routes || !route_rows || !ntiles || !aligned(x, 16) ||
      !aligned(weights, 2) || !aligned(ids, 4) || !aligned(tiles, 4) || !aligned(grouped_routes, 4) ||
      !aligned(route_rows, 4) || !aligned(ntiles, 4))
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_moe_route_q8: NULL or misaligned buffer");
  const uint32_t need_tiles = moe_max_tiles(T, E, k, shared_expert_gate != nullptr);
  if (max_tiles < (int)need_tiles)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_moe_route_q8: max_tiles below thq4_moe_add_max_tiles = " +
                                                    std::to_string(need_tiles));
  if (!workspace || workspace_bytes < moe_scores_bytes(T, E) || !aligned(workspace, 16))
    return set_error(THQ4_ERR_WORKSPACE, "thq4_moe_route_q8: needs a 16-byte aligned workspace of " +
                                             std::to_string(moe_scores_bytes(T, E)) + " bytes");
  MoeRouting rt{};
  rt.x = x;
  rt.H = H;
  rt.router = router;
  rt.shared_gate = shared_expert_gate;
  rt.shared_local = true;
  rt.partial = static_cast<float *>(workspace);
  cudaError_t e = moe_route_launch(rt, T, E, k, ids, static_cast<uint16_t *>(weights), tiles, grouped_routes,
                                   route_rows, ntiles, max_tiles, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, who);
  return THQ4_OK;
}

size_t thq4_moe_add_workspace_bytes(int T, int H, int I, int E, int k, int shared) {
  if (T <= 0 || H <= 0 || I <= 0 || E <= 0 || k <= 0) return 0;
  return moe_workspace(T, H, I, E, k, nullptr, k + (shared ? 1 : 0), shared != 0, E).bytes;
}

size_t thq4_moe_add_partial_workspace_bytes(int T, int H, int I, int E, int k, int e0, int e1, int shared_route,
                                            int runs_shared) {
  if (T <= 0 || H <= 0 || I <= 0 || E <= 0 || k <= 0 || e0 < 0 || e1 <= e0 || e1 > E) return 0;
  return moe_workspace(T, H, I, e1 - e0, k, nullptr, k + (shared_route ? 1 : 0), runs_shared != 0, E).bytes;
}

thq4_status thq4_moe_add(const void *x, const void *residual, int T, int H, int I, int E, int k,
                         const thq4_moe_weights *w, void *y, void *workspace, size_t workspace_bytes, void *stream) {
  const char *who = "thq4_moe_add";
  if (w && has_shared(w) != runs_shared(w))
    return set_error(THQ4_ERR_INVALID_ARGUMENT,
                     "thq4_moe_add: MoE weights do not match execution shape (shared expert and its gate go together)");
  return moe_add_common(x, residual, T, H, I, E, k, 0, E, w, y, false, workspace, workspace_bytes, stream, who);
}

thq4_status thq4_moe_add_partial(const void *x, const void *residual, int T, int H, int I, int E, int k, int e0,
                                 int e1, const thq4_moe_weights *w, float *y_part, void *workspace,
                                 size_t workspace_bytes, void *stream) {
  return moe_add_common(x, residual, T, H, I, E, k, e0, e1, w, y_part, true, workspace, workspace_bytes, stream,
                        "thq4_moe_add_partial");
}

size_t thq4_presum_block_bytes(int in) {
  if (in <= 0 || in % kGroup) return 0;
  return presum_block_bytes(in);
}

thq4_status thq4_presum_attach(const void *x, int m, int in, void *block, void *stream) {
  const char *who = "thq4_presum_attach";
  if (m < 1 || m > 8 || in <= 0 || in % kGroup)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": need 1 <= m <= 8 and in a positive multiple "
                                                                   "of 64 (m " + std::to_string(m) + ", in " +
                                                    std::to_string(in) + ")");
  if (!x || !block || !aligned(x, 16) || !aligned(block, 16))
    return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": x and block must be 16-byte aligned");
  const cudaError_t e = presum_attach_launch(x, m, in, block, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, who);
  return THQ4_OK;
}

thq4_status thq4_add_rms_norm(const void *x, const void *r, const void *w, int T, int C, float eps, void *res,
                              void *block, void *stream) {
  const char *who = "thq4_add_rms_norm";
  if (T < 1 || T > 8 || C <= 0 || C % kGroup || C > kAddRmsNormMaxC)
    return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": need 1 <= T <= 8 and C a multiple of 64 up "
                                                                   "to " + std::to_string(kAddRmsNormMaxC) +
                                                    " (T " + std::to_string(T) + ", C " + std::to_string(C) + ")");
  if (!x || !r || !w || !res || !block || !aligned(block, 16) || !aligned(x, 2) || !aligned(r, 2) ||
      !aligned(w, 2) || !aligned(res, 2))
    return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": NULL or misaligned buffer (block 16-byte aligned)");
  if (!(eps >= 0.0f)) return set_error(THQ4_ERR_INVALID_ARGUMENT, std::string(who) + ": eps must be >= 0");
  const cudaError_t e = add_rms_norm_launch(x, r, w, T, C, eps, res, block, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(e, who);
  return THQ4_OK;
}

thq4_status thq4_debug_set_gemv(int chunk, int stages, int grid, int reserved) {
  if (!(chunk == 0 || chunk == 4 || chunk == 8) || stages < 0 || stages == 1 || stages > 8 ||
      grid < 0 || grid > 2 * device_sm_count() || reserved != 0)
    return set_error(THQ4_ERR_INVALID_ARGUMENT,
                     "thq4_debug_set_gemv: chunk 0/4/8, stages 0 or 2..8, grid 0..2x SM count, reserved 0");
  g_force_warps.store(chunk, std::memory_order_relaxed);
  g_force_depth.store(stages, std::memory_order_relaxed);
  g_force_grid.store(grid, std::memory_order_relaxed);
  return THQ4_OK;
}

thq4_status thq4_debug_set_trace(void *buf, size_t bytes) {
  if (buf && (bytes < 256 || reinterpret_cast<uintptr_t>(buf) % 16))
    return set_error(THQ4_ERR_INVALID_ARGUMENT, "thq4_debug_set_trace: a 16-byte aligned buffer of >= 256 bytes");
  gemv_set_trace(buf, bytes);
  return THQ4_OK;
}

thq4_status thq4_debug_gemv_plan(int out, int in, int m, int x_f32, int gate_up, int sms, const int *cluster_fit,
                                 int64_t *plan) {
  if (out < 1 || in < kGroup || in % kGroup || m < 1 || sms < 1 || sms > 1024 || !plan)
    return set_error(THQ4_ERR_INVALID_ARGUMENT,
                     "thq4_debug_gemv_plan: need out >= 1, in a positive multiple of 64, m >= 1, 1 <= sms <= 1024, "
                     "plan non-NULL");
  const GemvPlan p = gemv_plan_for(out, in, m, x_f32 != 0, gate_up != 0, sms, [cluster_fit](int j) {
    return cluster_fit && j >= 2 && j <= 8 ? cluster_fit[j] : 0;
  });
  const int64_t v[8] = {p.ok ? 1 : 0, p.grid, p.cl_j > 1 ? p.cl_j : 1, p.stages, p.tokens_per_pass, p.cps, p.ch,
                        (int64_t)p.smem};
  for (int i = 0; i < 8; ++i) plan[i] = p.ok || i == 0 ? v[i] : 0;
  return THQ4_OK;
}

thq4_status thq4_debug_prefill_plan(int out, int in, int m, int gate_up, int sms, int64_t *plan) {
  if (out < 1 || in < kGroup || in % kGroup || m <= 8 || sms < 1 || sms > 1024 || !plan)
    return set_error(THQ4_ERR_INVALID_ARGUMENT,
                     "thq4_debug_prefill_plan: need out >= 1, in a positive multiple of 64, m > 8 (the prefill's "
                     "rows), 1 <= sms <= 1024, plan non-NULL");
  const PrefillPlanInfo p = prefill_debug_plan(out, m, gate_up != 0, sms);
  plan[0] = p.bt;
  plan[1] = p.split ? 1 : 0;
  plan[2] = p.tiles;
  plan[3] = p.grid;
  plan[4] = (int64_t)p.split_bytes;
  return THQ4_OK;
}

}  // extern "C"
