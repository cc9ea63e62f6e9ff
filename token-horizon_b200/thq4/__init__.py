"""thq4 -- B200 (sm_100a) Q4 affine quantized-matmul path of th-engine.

The operators live in libthq4.so (C ABI: include/thq4.h); this package is the
host-side mirror of the reference's operator API on top of it.
"""
from ._lib import (BF16, F16, F32, SRC_FRAG, SRC_MLX, SRC_SLAB, SRC_TILED, Thq4Error, check, last_error,
                   lib, version)
from .qlin import (LinearChain, MoeWeights, PackedExperts, PackedWeight, Q8Projection, QLin, fuse_lins, lin_apply, lin_apply_ps,
                   maybe_tiled, moe, moe_add, add_rms_norm, presum_block, presum_block_bytes, moe_add_partial, moe_partial, moe_route, moe_route_q8, moe_scores_q8)

__all__ = ["BF16", "F16", "F32", "SRC_FRAG", "SRC_MLX", "SRC_SLAB", "SRC_TILED", "Thq4Error", "check",
           "last_error", "lib", "version", "PackedWeight", "QLin", "fuse_lins", "lin_apply", "lin_apply_ps",
           "maybe_tiled", "PackedExperts", "moe", "moe_partial", "moe_route", "Q8Projection", "MoeWeights",
           "moe_add", "moe_add_partial", "moe_route_q8", "moe_scores_q8", "LinearChain", "add_rms_norm", "presum_block",
           "presum_block_bytes"]
