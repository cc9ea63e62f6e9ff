/*
 * q4_oracle.h -- CPU restatement of th-engine's Q4 affine quantized-matmul path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA path is
 * compared against; it is never linked into, loaded by or called from the
 * product library (libthq4.so).  Only tests/, __graft_entry__.smoke() and the
 * CPU-baseline / reference legs of bench.py load it.
 *
 * Parity status: PARTIALLY PINNED.  The reference implements this path in Rust
 * (candle custom ops) and Metal shaders, neither of which can be built or run
 * here, and it ships no golden vectors for it.  The bf16 rounding, the split-K
 * tolerance and the MoE tile bound are pinned against the reference's own C++
 * (docs/splash/dev/tuning/LinearNumerics.hpp, docs/splash/runtime/ops/MoE.hpp)
 * compiled from its sources by oracle/Makefile into oracle/_ref/.  The matmul,
 * layout and routing arithmetic below are restatements of the cited reference
 * lines and are otherwise unpinned.
 *
 * Conventions (all from engine/src/qwen35.rs and engine/src/quant_kernel.rs):
 *   - MLX affine Q4, group size gs (64): wq is u32 [out][in/8], nibble e of a
 *     word is element 8*word+e, LSB first (qwen35.rs:105-134);
 *   - sb is 16-bit [out][2*ng]: the ng scales of a row, then its ng biases
 *     (quant_kernel.rs:14-15, qwen35.rs:249-300);
 *   - dequantised weight w = q * s + b (qwen35.rs:126-128).
 *   sb_dtype selects the 16-bit scale/bias format: 0 = bf16 (the reference's
 *   format), 1 = f16 (the benchmark configurations).
 */
#ifndef Q4_ORACLE_H
#define Q4_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { Q4O_SB_BF16 = 0, Q4O_SB_F16 = 1 };

/* ---- scalar conversions (round to nearest even) ------------------------ */
uint16_t q4o_f32_to_bf16(float v);
float q4o_bf16_to_f32(uint16_t v);
uint16_t q4o_f32_to_f16(float v);
float q4o_f16_to_f32(uint16_t v);
float q4o_sb_to_f32(uint16_t v, int sb_dtype);
void q4o_f32_to_bf16_n(const float *src, uint16_t *dst, size_t n);
void q4o_bf16_to_f32_n(const uint16_t *src, float *dst, size_t n);

/* ---- deterministic generators ------------------------------------------ */
/* The reference tests' LCG (qwen35.rs:6889-6892, moe_metal_test.mm:69-73):
 * state = state * 6364136223846793005 + 1442695040888963407; out = state >> 33. */
uint64_t q4o_lcg(uint64_t *state);
/* rand_qlin of qwen35.rs:6896-6915: random words and (scale, bias) per group,
 * bf16, MLX row-major.  Consumes the LCG in the reference's order. */
void q4o_rand_qlin(int out, int in, uint64_t seed, uint32_t *wq, uint16_t *sb);
/* rand_x of qwen35.rs:6917-6923 as bf16 bits. */
void q4o_rand_x(int in, uint64_t seed, uint16_t *x);

/* pf_vec_matches_legacy_bitwise (quant_kernel.rs:5428-5466): its LCG returns
 * (state >> 32) and one state runs through all cases.  Writes a reference
 * tiled-layout weight of `total_out` rows (words tw [padded*ng*8], planar
 * sb tsb [2*padded*ng]: scales 0.002 + 0.01u then biases -0.05 + 0.02u,
 * u = (lcg % 1000) / 1000) and x bf16 [m][in] = (lcg % 2000) / 500 - 2. */
void q4o_rand_pf_case(int total_out, int in, int m, uint64_t *state,
                      uint32_t *tw, uint16_t *tsb, uint16_t *x);

/* ---- quantiser (this repository's own; the reference loads checkpoints that
 * arrive pre-quantised, qwen35.rs:5-7) ------------------------------------ */
/* Per (row, group of gs): s = (max - min) / 15, b = min, both rounded to
 * sb_dtype; q = clamp(round((w - b) / s), 0, 15) against the rounded s, b. */
void q4o_quantize(const float *w, int out, int in, int gs, int sb_dtype,
                  uint32_t *wq, uint16_t *sb, int nthreads);

/* ---- layouts ------------------------------------------------------------ */
/* Reference tiled layout, QLin::tiled (qwen35.rs:629-697): rows pad to 256,
 * words [tile][group][col][8], scales [(tile*ng+g)*256+col], biases at
 * + padded*ng.  tw holds tiles*ng*2048 words, tsb 2*padded*ng entries. */
void q4o_mlx_to_tiled(const uint32_t *wq, const uint16_t *sb, int out, int in,
                      uint32_t *tw, uint16_t *tsb);
void q4o_tiled_to_mlx(const uint32_t *tw, const uint16_t *tsb, int out, int in,
                      uint32_t *wq, uint16_t *sb);
/* Splash expert slab (moe_expert_slab.h:15-28, packer moe_metal_test.mm:
 * 126-145): [weights][scales][biases], StorageN=256 order, out % 256 == 0.
 * Size q4PackedBytes = out*in/16*9 (WeightStore.cpp:57-60). */
size_t q4o_slab_bytes(int out, int in);
void q4o_mlx_to_slab(const uint32_t *wq, const uint16_t *sb, int out, int in,
                     uint8_t *slab);
void q4o_slab_to_mlx(const uint8_t *slab, int out, int in, uint32_t *wq,
                     uint16_t *sb);
/* This repository's B200 layout ("frag"), described in full in
 * token-horizon_b200/csrc/thq4_common.cuh: rows pad to slabs of 16*ts rows
 * (ts tiles of 16; the library uses ts = 8); fq holds slabs*ts*ng*128 words
 * and fsb slabs*ts*ng*32 entries. */
size_t q4o_frag_qw_bytes(int out, int in, int ts);
size_t q4o_frag_sb_bytes(int out, int in, int ts);
void q4o_mlx_to_frag(const uint32_t *wq, const uint16_t *sb, int out, int in, int ts,
                     uint32_t *fq, uint16_t *fsb);
void q4o_frag_to_mlx(const uint32_t *fq, const uint16_t *fsb, int out, int in, int ts,
                     uint32_t *wq, uint16_t *sb);

/* ---- products ----------------------------------------------------------- */
/* Kernel semantics of every reference GPU family (qmvt quant_kernel.rs:
 * 2887-2890, MPP tile :1994-2001, prefill tile :4111-4122): per row and
 * group, acc += s * sum_k(q*x) + b * sum_k(x).  Accumulated in fp64 and
 * returned unrounded: y [m][out], x [m][in] as float values. */
void q4o_linear_group(const uint32_t *wq, const uint16_t *sb, int sb_dtype,
                      int out, int in, const float *x, int m, double *y,
                      int nthreads);
/* The reference CPU path (QLin::cpu_dequant + linear, qwen35.rs:327-352 and
 * dequant_affine :110-134): w = bf16(q*s + b) computed in f64, then the dot
 * product accumulated in fp64.  y [m][out] unrounded. */
void q4o_linear_dequant(const uint32_t *wq, const uint16_t *sb, int sb_dtype,
                        int out, int in, const float *x, int m, double *y,
                        int nthreads);
/* Dequantised bf16 weight [out][in], the AffineDequant output
 * (quant_kernel.rs:1765-1781) with dequant_affine's f64 arithmetic. */
void q4o_dequant_bf16(const uint32_t *wq, const uint16_t *sb, int sb_dtype,
                      int out, int in, uint16_t *w);
/* The gate/up epilogue (quant_kernel.rs:2039-2046, 2921-2926): gate and up
 * rounded to bf16, silu(gate) * up in f32, rounded to bf16. */
uint16_t q4o_silu_mul_bf16(float gate, float up);
/* Fused [gate | up] projection: rows [0, half) gate, [up_row, up_row+half)
 * up.  out_bf16 [m][half]. */
void q4o_gate_up(const uint32_t *wq, const uint16_t *sb, int sb_dtype, int out,
                 int in, int up_row, int half, const float *x, int m,
                 uint16_t *out_bf16, int nthreads);

/* ---- MoE (Splash docs/splash/runtime/metal/kernels/shared/moe.metal) ---- */
/* Top-k per token, descending score then ascending expert id, weights
 * exp(s_r - s_0) / sum_topk exp(s_o - s_0) rounded to bf16 (moe.metal:
 * 323-360).  logits bf16 [T][E]; ids [T][k]; weights bf16 [T][k]. */
void q4o_moe_select(const uint16_t *logits, int T, int E, int k, uint32_t *ids,
                    uint16_t *weights);
/* Upper bound on grouped tiles (MoE.hpp:72-77 without the shared expert). */
uint32_t q4o_moe_max_tiles(int T, int E, int k, int tile_rows);
/* Counting sort of the T*k routes by expert (moe.metal:368-449) into tiles of
 * tile_rows rows.  Canonical order: within an expert, routes ascend by route
 * index (t*k + slot); the reference's atomic cursors leave that order open.
 * tiles [max_tiles][2] = {expert, live rows}; grouped_routes
 * [max_tiles*tile_rows] (padding 0xFFFFFFFF); route_rows [T*k].  Returns the
 * tile count, or -1 if max_tiles is too small. */
int q4o_moe_group(const uint32_t *ids, int T, int k, int E, int tile_rows,
                  int max_tiles, uint32_t *tiles, uint32_t *grouped_routes,
                  uint32_t *route_rows);
/* One MoE layer on MLX row-major expert weights.  gate_up_w: E weights of
 * [2*I][H] ([gate | up] rows, stride gu_stride words/sb entries per expert);
 * down_w: E weights of [H][I].  x bf16 [T][H]; residual bf16 [T][H] or NULL;
 * h_out bf16 [T*k][I] per route (optional); y bf16 [T][H].
 * h = silu(bf16 g)*bf16 u per route (bf16); d = down(h) rounded to bf16;
 * y = residual + sum_slot w * d in slot order, f32, rounded to bf16
 * (moe_combine, moe.metal:642-664). */
void q4o_moe_forward(const uint16_t *x, const uint16_t *residual, int T, int H,
                     int I, int E, int k, const uint32_t *ids,
                     const uint16_t *weights, const uint32_t *gu_wq,
                     const uint16_t *gu_sb, const uint32_t *dn_wq,
                     const uint16_t *dn_sb, int sb_dtype, uint16_t *h_out,
                     uint16_t *d_out, uint16_t *y, int nthreads);

/* q4o_moe_forward with a shared expert: ids [T][k] hold routed experts and,
 * in any slot, expert id E for the shared expert, whose weights are the sh_*
 * arguments (MLX row-major like the routed ones; NULL: no shared expert). */
void q4o_moe_forward_shared(const uint16_t *x, const uint16_t *residual, int T, int H, int I, int E, int k,
                            const uint32_t *ids, const uint16_t *weights, const uint32_t *gu_wq,
                            const uint16_t *gu_sb, const uint32_t *dn_wq, const uint16_t *dn_sb,
                            const uint32_t *sh_gu_wq, const uint16_t *sh_gu_sb, const uint32_t *sh_dn_wq,
                            const uint16_t *sh_dn_sb, int sb_dtype, uint16_t *h_out, uint16_t *d_out,
                            uint16_t *y, int nthreads);
/* Router scores of a Q8 projection in StorageN = 256 order (moe.metal:34-262),
 * bf16 [T][ncols]; the fixed summation order is documented in q4_oracle.c. */
void q4o_moe_scores_q8(const uint16_t *x, int T, int H, const uint8_t *q, const uint16_t *scales,
                       const uint16_t *biases, int ncols, uint16_t *scores, int nthreads);
/* The shared expert's routing weight (moe.metal:297-322): bf16 [T] sigmoid of
 * the scalar gate (row 0 of a Q8 projection); logit [T] optional. */
void q4o_moe_shared_gate(const uint16_t *x, int T, int H, const uint8_t *q, const uint16_t *scales,
                         const uint16_t *biases, uint16_t *weights, float *logit);
/* Grouping with a shared slot last in each token's rpr = k + 1 routes
 * (moe.metal:368-449); rpr == k: as q4o_moe_group. */
int q4o_moe_group_shared(const uint32_t *ids, int T, int k, int rpr, int E, int tile_rows, int max_tiles,
                         uint32_t *tiles, uint32_t *grouped_routes, uint32_t *route_rows);
/* The reference MoE test's fixture (moe_metal_test.mm:46-271): Splash slabs
 * (q4o_slab_bytes each) of E gate, up and down experts and the shared
 * expert's three projections, inputs and residuals bf16 [rows][H]. */
void q4o_splash_moe_fixture(int H, int I, int E, int rows, uint64_t seed, uint8_t *gate, uint8_t *up,
                            uint8_t *down, uint8_t *shared_gate, uint8_t *shared_up, uint8_t *shared_down,
                            uint16_t *x, uint16_t *residual);

/* ---- CPU baseline (the reference arm of bench.py) ---------------------- */
/* The reference CPU semantics (dequantise on the fly, accumulate in f32),
 * vectorised and threaded over output rows.  y [m][out] f32.  Returns the
 * thread count used. */
int q4o_cpu_linear(const uint32_t *wq, const uint16_t *sb, int sb_dtype,
                   int out, int in, const float *x, int m, float *y,
                   int nthreads);

#ifdef __cplusplus
}
#endif
#endif
