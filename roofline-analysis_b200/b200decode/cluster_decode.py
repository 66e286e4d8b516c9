"""Drop-in for the reference's own decode entry points:
`cluster_decode_forward` / `cluster_decode_split_forward` over dense,
contiguous q [B, H, 1, 128], k/v [B, H, S, 128]
(cute_attention/cluster_decode/cluster_decode.py:114-147,
cluster_decode_split.py:160-200), with the same config record
(common.py:86-96) and the same input checks and messages
(common.py:111-130).

Both run this library's split-KV decode: each sequence's [H, S, D] block is
read in place as one page of an HND cache ([pages = B, Hkv = H, P = S, D]),
so nothing is copied; `cluster_size` and `num_threads` are accepted for
interface parity (the kernels choose their own split).  The outputs follow
the reference's semantics: o = softmax(q k^T * scale) v in q's dtype
(cluster_decode.py:103-111).
"""
from __future__ import annotations

import dataclasses
import math
from typing import Optional

import torch

from . import api


@dataclasses.dataclass
class ClusterDecodeConfig:
    """The reference's config record (common.py:86-96)."""
    softmax_scale: Optional[float] = None
    num_threads: int = 128
    cluster_size: int = 2

    def resolve_scale(self, head_dim: int) -> float:
        return self.softmax_scale if self.softmax_scale is not None else 1.0 / math.sqrt(head_dim)


def validate_decode_qkv(q, k, v, config: ClusterDecodeConfig) -> None:
    """Same checks, order and messages as common.py:111-130."""
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("Expected q, k, v to have shape (batch, heads, seqlen, headdim).")
    if q.shape[0] != k.shape[0] or q.shape[0] != v.shape[0]:
        raise ValueError("q, k, v must have the same batch size.")
    if q.shape[1] != k.shape[1] or q.shape[1] != v.shape[1]:
        raise ValueError("cluster_decode v0 only supports MHA with matching q/k/v heads.")
    if q.shape[2] != 1:
        raise ValueError("cluster_decode v0 only supports decode q_len=1.")
    if q.shape[-1] != k.shape[-1] or q.shape[-1] != v.shape[-1]:
        raise ValueError("cluster_decode v0 requires q, k, v to have the same head_dim.")
    if q.shape[-1] != 128:
        raise ValueError("cluster_decode v0 is scoped to head_dim=128.")
    if config.cluster_size not in (2, 4):
        raise ValueError("cluster_decode v0 supports cluster_size 2 or 4.")
    if not q.is_cuda or not k.is_cuda or not v.is_cuda:
        raise ValueError("cluster_decode targets CUDA tensors only.")
    if not q.is_contiguous() or not k.is_contiguous() or not v.is_contiguous():
        raise ValueError("q, k, v must be contiguous.")


def _dense_decode(q, k, v, config: Optional[ClusterDecodeConfig]):
    config = config or ClusterDecodeConfig()
    validate_decode_qkv(q, k, v, config)
    if k.shape != v.shape:
        raise ValueError("k and v must have the same shape.")
    batch, heads, _, head_dim = q.shape
    seq_len = k.shape[2]
    out = torch.empty_like(q)
    if seq_len == 0:
        out.zero_()
        return out
    dev = q.device
    # one page per sequence: [pages = B, Hkv = H, P = S, D] is k's own memory
    block_table = torch.arange(batch, dtype=torch.int32, device=dev).view(batch, 1)
    seqlens = torch.full((batch,), seq_len, dtype=torch.int32, device=dev)
    api.decode(q[:, :, 0], k, v, seqlens, block_table, config.resolve_scale(head_dim),
               out=out[:, :, 0], kv_layout="HND")
    return out


def cluster_decode_forward(q, k, v, config: Optional[ClusterDecodeConfig] = None):
    """cluster_decode.py:114-147: returns o [B, H, 1, 128] in q's dtype."""
    return _dense_decode(q, k, v, config)


def cluster_decode_split_forward(q, k, v, config: Optional[ClusterDecodeConfig] = None):
    """cluster_decode_split.py:160-200 (split-KV over a cluster there; the
    same split-KV decode here): returns o [B, H, 1, 128] in q's dtype."""
    return _dense_decode(q, k, v, config)
