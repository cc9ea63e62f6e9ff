// thq4_common.cuh -- shared device/host helpers of the thq4 library (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/thq4.h"

#define THQ4_SEMVER "0.1.0"

// ---------------------------------------------------------------------------
// frag weight layout
// ---------------------------------------------------------------------------
// Rows pad to slabs of 128 = eight 16-row tiles (a tile is the M of one
// mma.m16n8k16).  K splits into quant groups of 64.  Chunk
// ch = (slab * ng + g) * 8 + t covers tile t of the slab for group g:
//
//   nibbles: 512 bytes at byte offset ch * 512.  Lane l of a warp owns bytes
//            [16 l, 16 l + 16): four u32 words.  With r = l / 4, c = l % 4,
//            the nibble at bits 4i..4i+3 (i = 0..7) of word j holds
//                row = 128 slab + 16 t + r + 8 ((i >> 1) & 1)
//                k   = 64 g + 32 (j >> 1) + 8 (j & 1) + 16 (i & 1) + 2 c + (i >> 2)
//            (frag_k below).  So for word w of k-step pair p = j >> 1,
//            with the nibble moved to bits 4..7 of each 16-bit half:
//              (w << 4) & 0x00F000F0  rows r   / k-step 2p
//              (w >> 4) & 0x00F000F0  rows r+8 / k-step 2p
//              w        & 0x00F000F0  rows r   / k-step 2p+1
//              (w >> 8) & 0x00F000F0  rows r+8 / k-step 2p+1
//            each a pair of adjacent k (2c, 2c+1) in the two halves: exactly
//            the A-fragment registers of mma.m16n8k16 (words j = 2p and
//            2p+1 give the k and k+8 halves).  OR-ing 0x54005400 makes each
//            half the fp16 number 64 + q -- exact (the unit in the last place
//            of [64, 128) is 1/16).  The decode kernel takes the even
//            k-steps' nibbles from bits 0..3 in place instead (unpack_word).
//   scales:  64 bytes at byte offset ch * 64: eight quads
//            {s_r, b_r, s_r+8, b_r+8} (16-bit, bf16 or f16), quad r at + 8 r.
//
// One (slab, group) -- a "slab-group" (SG), the unit the kernels stream -- is
// 4096 contiguous nibble bytes and 512 contiguous scale bytes, and slab-groups
// follow each other slab-major, so any run of them is one contiguous byte
// range, fetched with large bulk copies.  Padding rows have zero nibbles,
// scales and biases.  Per weight the layout stores exactly 0.5 + 4/64 =
// 0.5625 bytes, the same as the reference's formats; only the order differs.
namespace thq4 {

constexpr int kGroup = 64;
constexpr int kTileRows = 16;
constexpr int kSlabTiles = 8;
constexpr int kSlabRows = kSlabTiles * kTileRows;
constexpr int kChunkBytes = 512;  // nibbles per (tile, group)
constexpr int kQuadBytes = 64;    // scale/bias per (tile, group)

// k (within the group) of the nibble at bits 4i..4i+3 of word j, lane column c
__host__ __device__ constexpr int frag_k(int j, int i, int c) {
  return 32 * (j >> 1) + 8 * (j & 1) + 16 * (i & 1) + 2 * c + (i >> 2);
}

__host__ __device__ inline int row_slabs(int rows) { return (rows + kSlabRows - 1) / kSlabRows; }
__host__ __device__ inline int row_tiles(int rows) { return (rows + 15) / 16; }

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------

// Streaming 16-byte load: read-only path, no L1 allocation, evict-first in L2
// (each weight byte is used exactly once per call).
__device__ __forceinline__ uint4 ld_stream_v4(const void *p, uint64_t policy) {
  uint4 v;
  asm volatile(
      "ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;\n"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p), "l"(policy));
  return v;
}
__device__ __forceinline__ uint2 ld_stream_v2(const void *p, uint64_t policy) {
  uint2 v;
  asm volatile(
      "ld.global.nc.L1::no_allocate.L2::cache_hint.v2.u32 {%0,%1}, [%2], %3;\n"
      : "=r"(v.x), "=r"(v.y)
      : "l"(p), "l"(policy));
  return v;
}
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(p));
  return p;
}

// (w & 0x00F000F0) | 0x54005400 as one LOP3: the fp16 pair (64 + q0,
// 64 + q1) of the nibbles in bits 4..7 and 20..23, exact.
template <uint32_t MASK>
__device__ __forceinline__ uint32_t nib_f16x2(uint32_t w) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xea;\n" : "=r"(r) : "r"(w), "n"(MASK), "n"(0x54005400));
  return r;
}

// The four mma.m16n8k16 A registers one frag word holds (see the layout
// above): k-step 2p rows r / r + 8 (nibbles at bits 0..3 / 8..11 of each
// half) as the exact fp16 q -- (w & 0x000F000F) | 0x64006400 is 1024 + q
// (unit in the last place 1), less 1024 on the fp16 pipe -- and k-step
// 2p + 1 rows r / r + 8 (bits 4..7 / 12..15) as 64 + q.  One shift, four
// LOP3 and two f16x2 subtractions: five operations on the integer pipe per
// eight weights instead of seven with a shift per register.
__device__ __forceinline__ void unpack_word(uint32_t w, uint32_t &e_r, uint32_t &e_r8, uint32_t &o_r,
                                            uint32_t &o_r8) {
  const uint32_t t = w >> 8;
  uint32_t u0, u1;
  asm("lop3.b32 %0, %1, %2, %3, 0xea;\n" : "=r"(u0) : "r"(w), "n"(0x000F000F), "n"(0x64006400));
  asm("lop3.b32 %0, %1, %2, %3, 0xea;\n" : "=r"(u1) : "r"(t), "n"(0x000F000F), "n"(0x64006400));
  asm("sub.rn.f16x2 %0, %1, %2;\n" : "=r"(e_r) : "r"(u0), "r"(0x64006400));
  asm("sub.rn.f16x2 %0, %1, %2;\n" : "=r"(e_r8) : "r"(u1), "r"(0x64006400));
  o_r = nib_f16x2<0x00F000F0u>(w);
  o_r8 = nib_f16x2<0x00F000F0u>(t);
}

// D = A * B (C = 0), fp16 inputs, f32 accumulate, m16n8k16.
__device__ __forceinline__ void mma_f16_16816_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
}

// D = A * B + C, fp16 inputs, f32 accumulate, m16n8k16.
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Device-scope acquire-release atomic add (orders this thread's earlier
// writes before it, and later reads after it).
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;\n" ::: "memory"); }
__device__ __forceinline__ uint32_t atom_add_relaxed(uint32_t *p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.relaxed.gpu.global.add.u32 %0, [%1], %2;\n" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
// Thread-block clusters: every thread of every CTA of the cluster arrives
// (release) and waits (acquire); DSMEM stores into another CTA's shared
// memory at the same offset (mapa).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_map(uint32_t smem_addr_local, uint32_t cta_rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(smem_addr_local), "r"(cta_rank));
  return r;
}
__device__ __forceinline__ void st_cluster_f4(uint32_t addr, float4 v) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};\n" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}
__device__ __forceinline__ uint32_t ld_cluster_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];\n" : "=r"(v) : "r"(addr) : "memory");
  return v;
}
// Volatile (relaxed, system scope) 16-byte load / 8-byte store: each aligned
// 8-byte word is read or written whole, the low-latency exchange's unit.
__device__ __forceinline__ uint4 ld_volatile_v4(const uint4 *p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ void st_volatile_u64(unsigned long long *p, unsigned long long v) {
  asm volatile("st.volatile.global.u64 [%0], %1;\n" ::"l"(p), "l"(v) : "memory");
}
// System-scope ordering for flags that other GPUs read over NVLink.
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;\n" ::: "memory"); }
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t atom_add_acq_rel(uint32_t *p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;\n" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
// Device-scope relaxed 16-byte load (not served from a stale L1 line).
__device__ __forceinline__ float4 ld_relaxed_f4(const float *p) {
  float4 v;
  asm volatile("ld.relaxed.gpu.global.v4.f32 {%0,%1,%2,%3}, [%4];\n"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// ---- mbarrier / bulk-copy / PDL wrappers --------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(count));
}
// Makes mbarrier initialisation visible to the async proxy (the bulk copies).
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
// One-dimensional bulk copy global -> shared (no multicast), completing on
// `bar` with its byte count; evict-first in L2.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;\n" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}
// 2-D tiled TMA load of the box at (c0 innermost, c1) into shared memory,
// completing on `bar` (c0 * element size must be a multiple of 16 bytes).
__device__ __forceinline__ void tma_load_2d(void *dst, const void *map, int c0, int c1, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];\n" ::"r"(
          smem_addr(dst)),
      "l"(map), "r"(smem_addr(bar)), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;\n" : "=l"(t));
  return t;
}
// Waits for phase `parity` of `bar` for at most `limit_ns`; false on timeout.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > limit_ns) return false;
  }
  return true;
}
// Programmatic dependent launch: wait for the preceding grid's results /
// allow the next grid to start its prologue.  No-ops without the launch
// attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t lo16) {
  return __uint_as_float(lo16 << 16);
}
__device__ __forceinline__ float f16_bits_to_f32(uint32_t lo16) {
  return __half2float(__ushort_as_half((unsigned short)lo16));
}
template <bool F16>
__device__ __forceinline__ float sb_to_f32(uint32_t lo16) {
  if constexpr (F16)
    return f16_bits_to_f32(lo16);
  else
    return bf16_bits_to_f32(lo16);
}
__device__ __forceinline__ float round_bf16(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float v) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}

// silu(bf16 g) * bf16 u in f32, the reference's gate/up epilogue
// (quant_kernel.rs:2039-2046): gate / (1 + exp(-gate)) * up.
__device__ __forceinline__ float silu_mul(float gate, float up) {
  const float g = round_bf16(gate), u = round_bf16(up);
  return g / (1.0f + expf(-g)) * u;
}

// Kernels record conditions they skip instead of faulting (bad ids, bounds)
// by OR-ing these bits into the device status word whose address the host
// passes in; thq4_device_status reads and clears it.
enum : uint32_t {
  kStatusBadExpert = 1u << 0,
  kStatusBounds = 1u << 1,
  kStatusTimeout = 1u << 2,  // an mbarrier wait ran out of time
};
// Bound on any single wait for an in-flight copy (a healthy one completes in
// microseconds).
constexpr uint64_t kWaitLimitNs = 2000000000ull;
__device__ __forceinline__ void raise_status(uint32_t *status, uint32_t bit) {
  if (status) atomicOr(status, bit);
}

}  // namespace thq4
