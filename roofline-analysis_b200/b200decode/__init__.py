"""b200decode — B200-native (sm_100a) paged decode attention.

Host layer over libb2d.so (hand-written CUDA kernels behind a C ABI,
include/b2d_decode.h).  Public API:

    decode(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale)
        -> (out, lse)
    decode_mla(q, kv_cache, cache_seqlens, block_table, softmax_scale)
        -> (out, lse)
    append_kv(key, value, k_cache, v_cache, slot_mapping)     (reshape_and_cache)
    GqaDecoder(...).run() / .capture() / .replay()           (plan once, CUDA graphs)
    cluster_decode.cluster_decode_forward(q, k, v, config)   (the reference's own
        dense decode entry point)
    python -m b200decode.decodebench [mla] ...               (decodebench backend)

There is no CPU or library fallback: calling either without the compiled
library or without a CUDA device raises.
"""
from .api import (  # noqa: F401
    B2DError,
    append_kv,
    DecodeWorkspace,
    GqaDecoder,
    check_device_status,
    decode,
    decode_mla,
    gqa_plan,
    library_path,
)

from . import cluster_decode  # noqa: F401,E402

__version__ = "0.1.0"
