// thq4_presum.cu -- presum blocks: a decode / verify projection's activation
// as 8 zero-padded bf16 rows followed by its f32 per-(group, row) sums, and
// the two producers of the reference that emit them.
//
// Block of width `in` (engine/src/quant_kernel.rs:265-273,
// presum_block_bytes): rows [8][in] bf16 (rows >= m are zero), then sums
// f32 [in/64][8], sums[g * 8 + t] = the sum of row t's group g taken in the
// reference's lane pattern: lane l of a warp adds x[64g + l] and
// x[64g + 32 + l] in f32, then the 32 lanes combine (quant_kernel.rs:
// 1864-1884; gdn_kernel.rs:1922-1962).  The lanes combine here by xor
// butterfly with partners 16, 8, 4, 2, 1; that order is the oracle's too.
//
// Producers: AddRmsNorm { sums } (gdn_kernel.rs:1851-1866, 1919-1962):
// res = bf16(x + r) and the normed plane bf16(bf16(res) * inv * w) as a
// presum block, inv = 1 / sqrt(ss / C + eps) with ss accumulated per lane
// over columns lane, lane + 32, ... in order and combined by the butterfly;
// and Q4AttachSums: an activation copied into a block with its sums.
#include "thq4_common.cuh"
#include "thq4_internal.h"

namespace thq4 {

namespace {

__device__ __forceinline__ float lane_butterfly(float s) {
  s += __shfl_xor_sync(0xffffffffu, s, 16);
  s += __shfl_xor_sync(0xffffffffu, s, 8);
  s += __shfl_xor_sync(0xffffffffu, s, 4);
  s += __shfl_xor_sync(0xffffffffu, s, 2);
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  return s;
}

// One CTA per block row t (8 CTAs): rows t < T hold rms_norm(x + r) * w,
// rows T..7 and their sums are zero.  tv: the row's f32 x + r in shared memory.
__global__ void __launch_bounds__(256) add_rms_norm_kernel(const uint16_t *x, const uint16_t *r, const uint16_t *w,
                                                           int T, int C, float eps, uint16_t *res, uint16_t *block) {
  extern __shared__ float tv[];
  __shared__ float s_inv;
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint16_t *nrm = block + (size_t)t * C;
  float *sums = reinterpret_cast<float *>(block + (size_t)8 * C);
  const int ng = C / kGroup;
  if (t >= T) {
    for (int c = tid; c < C; c += blockDim.x) nrm[c] = 0;
    for (int g = tid; g < ng; g += blockDim.x) sums[g * 8 + t] = 0.0f;
    return;
  }
  for (int c = tid; c < C; c += blockDim.x) {
    const float v = __fadd_rn(bf16_bits_to_f32(x[(size_t)t * C + c]), bf16_bits_to_f32(r[(size_t)t * C + c]));
    res[(size_t)t * C + c] = f32_to_bf16_bits(v);
    tv[c] = v;
  }
  __syncthreads();
  if (warp == 0) {
    float ss = 0.0f;
    for (int c = lane; c < C; c += 32) ss = __fadd_rn(ss, __fmul_rn(tv[c], tv[c]));
    ss = lane_butterfly(ss);
    // correctly rounded: 1 / sqrt, each step IEEE
    if (lane == 0) s_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)C), eps)));
  }
  __syncthreads();
  const float inv = s_inv;
  // groups g = warp, warp + 8, ...: the lane pattern needs one warp per group
  for (int g = warp; g < ng; g += blockDim.x / 32) {
    const int c0 = g * kGroup + lane;
    const uint16_t a = f32_to_bf16_bits(__fmul_rn(__fmul_rn(round_bf16(tv[c0]), inv), bf16_bits_to_f32(w[c0])));
    const uint16_t b =
        f32_to_bf16_bits(__fmul_rn(__fmul_rn(round_bf16(tv[c0 + 32]), inv), bf16_bits_to_f32(w[c0 + 32])));
    nrm[c0] = a;
    nrm[c0 + 32] = b;
    const float s = lane_butterfly(__fadd_rn(bf16_bits_to_f32(a), bf16_bits_to_f32(b)));
    if (lane == 0) sums[g * 8 + t] = s;
  }
}

// One CTA (8 warps) per group g: warp t copies row t's 64 values of the group
// into the block (zero for t >= m) and writes their sum.
__global__ void __launch_bounds__(256) presum_attach_kernel(const uint16_t *x, int m, int in, uint16_t *block) {
  const int g = blockIdx.x, t = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c0 = g * kGroup + lane;
  uint16_t a = 0, b = 0;
  if (t < m) {
    a = x[(size_t)t * in + c0];
    b = x[(size_t)t * in + c0 + 32];
  }
  block[(size_t)t * in + c0] = a;
  block[(size_t)t * in + c0 + 32] = b;
  const float s = lane_butterfly(__fadd_rn(bf16_bits_to_f32(a), bf16_bits_to_f32(b)));
  if (lane == 0) reinterpret_cast<float *>(block + (size_t)8 * in)[g * 8 + t] = s;
}

}  // namespace

size_t presum_block_bytes(int in) { return (size_t)8 * in * 2 + (size_t)(in / kGroup) * 8 * 4; }

cudaError_t add_rms_norm_launch(const void *x, const void *r, const void *w, int T, int C, float eps, void *res,
                                void *block, cudaStream_t stream) {
  const size_t smem = (size_t)C * sizeof(float);
  static DeviceOnce once;
  cudaError_t e = once.run([&] {
    return cudaFuncSetAttribute(add_rms_norm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)(kAddRmsNormMaxC * sizeof(float)));
  });
  if (e != cudaSuccess) return e;
  add_rms_norm_kernel<<<8, 256, smem, stream>>>(static_cast<const uint16_t *>(x), static_cast<const uint16_t *>(r),
                                                static_cast<const uint16_t *>(w), T, C, eps,
                                                static_cast<uint16_t *>(res), static_cast<uint16_t *>(block));
  return cudaGetLastError();
}

cudaError_t presum_attach_launch(const void *x, int m, int in, void *block, cudaStream_t stream) {
  presum_attach_kernel<<<in / kGroup, 256, 0, stream>>>(static_cast<const uint16_t *>(x), m, in,
                                                        static_cast<uint16_t *>(block));
  return cudaGetLastError();
}

}  // namespace thq4
