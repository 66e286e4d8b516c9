"""The reference's CPU decode path, for timing and cross-checks — TEST
INFRASTRUCTURE ONLY (imported by tests/ and bench.py's CPU legs).

The reference's decode math on a host is
`torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=False,
enable_gqa=Hq != Hkv)` (decodebench/torch_sdpa_benchmark.py:95-102) on dense
[B, H, S, D] tensors.  Paged caches are first gathered into dense
per-sequence tensors (untimed, like the reference's own dense setup); each
sequence is then one SDPA call, since lengths differ.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def gather_dense(k_cache, v_cache, cache_seqlens, block_table, k_scale=None, v_scale=None,
                 dtype=None):
    """Paged NHD caches -> list of (k [1, Hkv, L, D], v [1, Hkv, L, D]).

    FP8 caches are dequantised with their per-KV-head scales into `dtype`
    (fp32 by default for FP8, the cache dtype otherwise)."""
    page = k_cache.shape[1]
    out = []
    for b, length in enumerate(cache_seqlens.tolist()):
        n = (length + page - 1) // page
        idx = block_table[b, :n].long()
        k = k_cache[idx].reshape(n * page, *k_cache.shape[2:])[:length]
        v = v_cache[idx].reshape(n * page, *v_cache.shape[2:])[:length]
        if k_cache.dtype == torch.float8_e4m3fn:
            tgt = dtype or torch.float32
            k = k.to(tgt) * (k_scale.to(tgt)[None, :, None] if k_scale is not None else 1)
            v = v.to(tgt) * (v_scale.to(tgt)[None, :, None] if v_scale is not None else 1)
        elif dtype is not None:
            k, v = k.to(dtype), v.to(dtype)
        out.append((k.permute(1, 0, 2).unsqueeze(0).contiguous(),
                    v.permute(1, 0, 2).unsqueeze(0).contiguous()))
    return out


def sdpa_decode(q, dense_kv, softmax_scale):
    """q [B, Hq, D]; dense_kv from gather_dense -> out [B, Hq, D] (q dtype
    unless the KV were upcast)."""
    outs = []
    for b, (k, v) in enumerate(dense_kv):
        qb = q[b:b + 1, :, None, :].to(k.dtype)
        o = F.scaled_dot_product_attention(qb, k, v, is_causal=False, scale=softmax_scale,
                                           enable_gqa=qb.shape[1] != k.shape[1])
        outs.append(o[:, :, 0, :])
    return torch.cat(outs, 0)
