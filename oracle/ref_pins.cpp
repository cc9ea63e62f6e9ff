// ref_pins.cpp -- exports a few of the reference's own C++ helpers through a C
// ABI so the oracle's arithmetic can be pinned against them.
//
// TEST INFRASTRUCTURE ONLY.  Compiled by oracle/Makefile against the
// reference's headers where they lie (REF_ROOT/docs/splash/...); nothing of
// the reference is copied into this repository.  The output goes to
// oracle/_ref/ and is only loaded by tests.
//
//   docs/splash/dev/tuning/LinearNumerics.hpp:17-23   bf16 <-> f32
//   docs/splash/dev/tuning/LinearNumerics.hpp:29-36   ulpBf16
//   docs/splash/dev/tuning/LinearNumerics.hpp:57-59   reassociationSlack
//   docs/splash/dev/tuning/LinearNumerics.hpp:112-126 splitTolerance
//   docs/splash/runtime/ops/MoE.hpp:72-77             moeMaximumTiles
//   docs/splash/runtime/metal/abi/MoE.h:26-29         MoeTileDescriptor
#include "tuning/LinearNumerics.hpp"
#include "ops/MoE.hpp"
#include "metal/abi/MoE.h"

#include <cstdint>

namespace tn = splash::ops::tuning;

extern "C" {

uint16_t ref_float_to_bf16(float v) { return tn::floatToBf16(v); }
float ref_bf16_to_float(uint16_t v) { return tn::bf16ToFloat(v); }
float ref_ulp_bf16(float v) { return tn::ulpBf16(v); }
float ref_silu(float v) { return tn::silu(v); }
float ref_reassociation_slack(uint32_t input_size, float max_abs_reference) {
  return tn::reassociationSlack(input_size, max_abs_reference);
}
// epilogue: 0 None, 1 Residual, 2 GateUp (LinearEpilogue order, Linear.hpp)
float ref_split_tolerance(int epilogue, float value, float residual, float gate,
                          float up, float slack) {
  tn::SplitReference r;
  r.value = value;
  r.residual = residual;
  r.gate = gate;
  r.up = up;
  return tn::splitTolerance(static_cast<splash::ops::LinearEpilogue>(epilogue), r, slack);
}
uint32_t ref_moe_maximum_tiles(uint32_t rows, uint32_t hidden, uint32_t experts,
                               uint32_t top_k, uint32_t intermediate,
                               uint32_t tile_rows) {
  splash::ops::MoeShape s{hidden, experts, top_k, intermediate};
  return splash::ops::moeMaximumTiles(rows, s, tile_rows);
}
uint32_t ref_moe_tile_descriptor_bytes(void) { return sizeof(MoeTileDescriptor); }

}  // extern "C"
