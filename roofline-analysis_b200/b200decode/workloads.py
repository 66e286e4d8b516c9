"""Seeded synthetic inputs for the BASELINE configurations.

The reference builds its decodebench inputs with unseeded torch.randn and a
uniform context length with identity page order
(decodebench/flashinfer_kernel.py:65-92).  The configurations here restate
BASELINE's five configs as concrete, seeded tensors: per-sequence lengths
drawn uniformly from [seqlen_lo, seqlen_hi], a page pool of exactly
sum(ceil(L_b / P)) pages, and block-table rows that index a random
permutation of that pool (rows are padded with page 0, never read).
"""
from __future__ import annotations

import dataclasses
import math
from typing import Optional

import torch

_TORCH_DT = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp8": torch.float8_e4m3fn}


@dataclasses.dataclass(frozen=True)
class GqaWorkload:
    name: str
    batch: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    page_size: int
    kv_dtype: str            # "bf16" | "fp16" | "fp8"
    seqlen_lo: int
    seqlen_hi: int
    q_dtype: str = "bf16"
    seed: int = 0
    page_perm: bool = True
    kv_scale_range: Optional[tuple] = None   # fp8: per-KV-head scales ~ U[lo, hi]
    value_std: float = 1.0

    @property
    def softmax_scale(self) -> float:
        return 1.0 / math.sqrt(self.head_dim)

    def scaled(self, **kw) -> "GqaWorkload":
        return dataclasses.replace(self, **kw)


@dataclasses.dataclass(frozen=True)
class MlaWorkload:
    name: str
    batch: int
    num_heads: int
    head_dim_qk: int
    head_dim_v: int
    page_size: int
    seqlen_lo: int
    seqlen_hi: int
    seed: int = 0
    value_std: float = 0.5   # "values ~ N(0, 0.5)" read as standard deviation 0.5

    @property
    def softmax_scale(self) -> float:
        return 1.0 / math.sqrt(192.0)   # qk_nope 128 + qk_rope 64

    def scaled(self, **kw) -> "MlaWorkload":
        return dataclasses.replace(self, **kw)


# BASELINE.json configs, in order.
CFG1_MHA_CPU = GqaWorkload("cfg1_mha_dense_s2048", 1, 16, 16, 128, 2048, "fp16", 2048, 2048,
                           q_dtype="fp16", page_perm=False)
CFG2_GQA_PAGED = GqaWorkload("cfg2_gqa_paged_b64_p16", 64, 32, 8, 128, 16, "bf16", 1024, 8192)
CFG3_LONG_SPLITKV = GqaWorkload("cfg3_long_splitkv_b4_s131072", 4, 64, 8, 128, 64, "bf16",
                                131072, 131072)
CFG4_MLA = MlaWorkload("cfg4_mla_b128_p64", 128, 128, 576, 512, 64, 2048, 16384)
CFG5_FP8 = GqaWorkload("cfg5_fp8_b256_p16", 256, 32, 8, 128, 16, "fp8", 2048, 8192,
                       kv_scale_range=(0.01, 0.1))

CONFIGS = {w.name: w for w in (CFG1_MHA_CPU, CFG2_GQA_PAGED, CFG3_LONG_SPLITKV, CFG4_MLA, CFG5_FP8)}
ALIASES = {"cfg1": CFG1_MHA_CPU.name, "cfg2": CFG2_GQA_PAGED.name, "cfg3": CFG3_LONG_SPLITKV.name,
           "cfg4": CFG4_MLA.name, "cfg5": CFG5_FP8.name}


def get(name: str):
    return CONFIGS[ALIASES.get(name, name)]


def draw_seqlens(batch: int, lo: int, hi: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed * 7919 + 17)
    return torch.randint(lo, hi + 1, (batch,), generator=g, dtype=torch.int64)


def make_block_table(seqlens: torch.Tensor, page_size: int, perm: bool, seed: int):
    """-> (block_table int32 [B, max_pages], num_pages)."""
    npages = [(int(l) + page_size - 1) // page_size for l in seqlens.tolist()]
    total = max(1, sum(npages))
    maxp = max(1, max(npages) if npages else 1)
    g = torch.Generator().manual_seed(seed * 104729 + 3)
    pool = torch.randperm(total, generator=g) if perm else torch.arange(total)
    bt = torch.zeros(len(npages), maxp, dtype=torch.int32)
    off = 0
    for b, n in enumerate(npages):
        bt[b, :n] = pool[off:off + n].to(torch.int32)
        off += n
    return bt, total


def _randn(shape, gen, device, std=1.0):
    return torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std


def make_gqa_inputs(w: GqaWorkload, device="cpu", seqlens: Optional[torch.Tensor] = None):
    """Inputs for decode(): dict with q, k_cache, v_cache (NHD), cache_seqlens,
    block_table, k_scale, v_scale, softmax_scale.  Given `seqlens`, the batch
    is len(seqlens)."""
    device = torch.device(device)
    if seqlens is None:
        seqlens = draw_seqlens(w.batch, w.seqlen_lo, w.seqlen_hi, w.seed)
    w = w.scaled(batch=len(seqlens))
    bt, npages = make_block_table(seqlens, w.page_size, w.page_perm, w.seed)
    gen = torch.Generator(device=device).manual_seed(w.seed * 31 + 1)
    qdt = _TORCH_DT[w.q_dtype]
    q = _randn((w.batch, w.num_q_heads, w.head_dim), gen, device, w.value_std).to(qdt)
    shape = (npages, w.page_size, w.num_kv_heads, w.head_dim)
    k_scale = v_scale = None
    if w.kv_dtype == "fp8":
        lo, hi = w.kv_scale_range or (1.0, 1.0)
        sg = torch.Generator().manual_seed(w.seed * 13 + 5)
        k_scale = (lo + (hi - lo) * torch.rand(w.num_kv_heads, generator=sg)).to(device)
        v_scale = (lo + (hi - lo) * torch.rand(w.num_kv_heads, generator=sg)).to(device)
        k_cache = torch.empty(shape, dtype=torch.float8_e4m3fn, device=device)
        v_cache = torch.empty(shape, dtype=torch.float8_e4m3fn, device=device)
        # Fill block by block to bound the fp32 temporary.  Values are
        # saturated to the e4m3 range (+-448) before the cast, as a quantiser
        # does: torch's cast turns out-of-range values into the NaN code
        # (N(0,1) / 0.01 exceeds 448 a few times per config-5 cache).
        step = max(1, (1 << 26) // (w.page_size * w.num_kv_heads * w.head_dim))
        for p0 in range(0, npages, step):
            p1 = min(npages, p0 + step)
            sub = (p1 - p0,) + shape[1:]
            k_cache[p0:p1] = (_randn(sub, gen, device, w.value_std)
                              / k_scale[None, None, :, None]).clamp_(-448.0, 448.0).to(torch.float8_e4m3fn)
            v_cache[p0:p1] = (_randn(sub, gen, device, w.value_std)
                              / v_scale[None, None, :, None]).clamp_(-448.0, 448.0).to(torch.float8_e4m3fn)
    else:
        kdt = _TORCH_DT[w.kv_dtype]
        k_cache = torch.empty(shape, dtype=kdt, device=device)
        v_cache = torch.empty(shape, dtype=kdt, device=device)
        step = max(1, (1 << 27) // (w.page_size * w.num_kv_heads * w.head_dim))
        for p0 in range(0, npages, step):
            p1 = min(npages, p0 + step)
            sub = (p1 - p0,) + shape[1:]
            k_cache[p0:p1] = _randn(sub, gen, device, w.value_std).to(kdt)
            v_cache[p0:p1] = _randn(sub, gen, device, w.value_std).to(kdt)
    return dict(q=q, k_cache=k_cache, v_cache=v_cache,
                cache_seqlens=seqlens.to(torch.int32).to(device), block_table=bt.to(device),
                k_scale=k_scale, v_scale=v_scale, softmax_scale=w.softmax_scale)


def to_vllm_layout(k_cache: torch.Tensor, v_cache: torch.Tensor):
    """NHD caches [pages, P, Hkv, D] -> vLLM paged_attention's layout
    (decodebench/vllm_paged_kernel.py:102-123): K [pages, Hkv, D/x, P, x]
    with x = 16 bytes of elements, V [pages, Hkv, D, P]."""
    pages, P, hkv, d = k_cache.shape
    x = 16 // k_cache.element_size()
    k = k_cache.reshape(pages, P, hkv, d // x, x).permute(0, 2, 3, 1, 4).contiguous()
    v = v_cache.permute(0, 2, 3, 1).contiguous()
    return k, v


def make_mla_inputs(w: MlaWorkload, device="cpu", seqlens: Optional[torch.Tensor] = None,
                    page_perm: bool = True):
    """Inputs for decode_mla(): q [B, H, 576], kv_cache [pages, P, 576]."""
    device = torch.device(device)
    if seqlens is None:
        seqlens = draw_seqlens(w.batch, w.seqlen_lo, w.seqlen_hi, w.seed)
    w = w.scaled(batch=len(seqlens))
    bt, npages = make_block_table(seqlens, w.page_size, page_perm, w.seed)
    gen = torch.Generator(device=device).manual_seed(w.seed * 31 + 2)
    q = _randn((w.batch, w.num_heads, w.head_dim_qk), gen, device, w.value_std).to(torch.bfloat16)
    kv = torch.empty((npages, w.page_size, w.head_dim_qk), dtype=torch.bfloat16, device=device)
    step = max(1, (1 << 27) // (w.page_size * w.head_dim_qk))
    for p0 in range(0, npages, step):
        p1 = min(npages, p0 + step)
        kv[p0:p1] = _randn((p1 - p0, w.page_size, w.head_dim_qk), gen, device,
                           w.value_std).to(torch.bfloat16)
    return dict(q=q, kv_cache=kv, cache_seqlens=seqlens.to(torch.int32).to(device),
                block_table=bt.to(device), softmax_scale=w.softmax_scale)


def gqa_algorithmic_bytes(w: GqaWorkload, seqlens: torch.Tensor) -> int:
    """Compulsory HBM bytes of one decode step: exact-token K+V, q, out,
    lse, block-table entries and seqlens (split partials not counted)."""
    es = 1 if w.kv_dtype == "fp8" else 2
    tokens = int(seqlens.sum())
    kv = tokens * w.num_kv_heads * w.head_dim * es * 2
    qo = len(seqlens) * w.num_q_heads * w.head_dim * 2 * 2
    lse = len(seqlens) * w.num_q_heads * 4
    pages = sum((int(l) + w.page_size - 1) // w.page_size for l in seqlens.tolist())
    meta = pages * 4 + len(seqlens) * 4 + (w.num_kv_heads * 8 if w.kv_dtype == "fp8" else 0)
    return kv + qo + lse + meta


def gqa_flops(w: GqaWorkload, seqlens: torch.Tensor) -> int:
    return 4 * w.num_q_heads * w.head_dim * int(seqlens.sum())


def gqa_kv_bytes_reference(w: GqaWorkload, seqlens: torch.Tensor) -> int:
    """decodebench's approx_kv_bytes_read (flashinfer_kernel.py:26-28), with
    the per-sequence lengths summed instead of B * context_len."""
    es = 1 if w.kv_dtype == "fp8" else 2
    return int(seqlens.sum()) * w.num_kv_heads * w.head_dim * 2 * es


def mla_algorithmic_bytes(w: MlaWorkload, seqlens: torch.Tensor) -> int:
    tokens = int(seqlens.sum())
    b = len(seqlens)
    pages = sum((int(l) + w.page_size - 1) // w.page_size for l in seqlens.tolist())
    return (tokens * w.head_dim_qk * 2 + b * w.num_heads * (w.head_dim_qk + w.head_dim_v) * 2
            + b * w.num_heads * 4 + pages * 4 + b * 4)


def mla_flops(w: MlaWorkload, seqlens: torch.Tensor) -> int:
    return 2 * w.num_heads * (w.head_dim_qk + w.head_dim_v) * int(seqlens.sum())
