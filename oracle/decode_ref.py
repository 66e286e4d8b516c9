"""CPU oracle for paged decode attention — TEST INFRASTRUCTURE ONLY.

This module is the checker the parity tests compare the CUDA kernels
against.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
--impl reference legs may import it; the shipped decode path never does.

It restates, in numpy float64, the decode math the reference relies on:

* Dense decode attention, the call decodebench/torch_sdpa_benchmark.py:100-102
  makes (`F.scaled_dot_product_attention(q, k, v, is_causal=False,
  enable_gqa=Hq != Hkv)`): query head h reads KV head h // (Hq // Hkv).
* Paged caches gathered through a block table as flash_attn_with_kvcache
  reads them (decodebench/flashattn_kvcache_kernel.py:150-169): sequence b's
  token t lives at page block_table[b, t // P], slot t % P.
* Split-KV partials and their LSE merge, following
  cute_attention/cluster_decode/cluster_decode_reduce.py:16-64
  (split_kv_decode_partials) and :67-91 (merge_split_kv_decode_partials).
* lse = ln sum_t exp(s_t), the natural-log log-sum-exp the merge defines
  (M + ln L).
* FP8-e4m3 K/V dequantised as e4m3 * scale[kv_head] (
  the reference itself stores FP8 with unit scales, flashinfer_kernel.py:79-82).
* Absorbed MLA (decodebench/trtllm_mla_kernel.py:115-132): one latent KV head
  of width 576; scores use all 576 columns, V is the first 512.

Pinned by tests/test_oracle.py against fixtures the reference itself
produced (tests/golden/make_golden.py).  Arrays are numpy; 16-bit and 8-bit
inputs are passed as their raw bit patterns so that the oracle owns every
conversion.
"""
from __future__ import annotations

import numpy as np

# ---------------------------------------------------------------------------
# element formats (from their bit-level definitions)
# ---------------------------------------------------------------------------


def bf16_bits_to_f64(bits: np.ndarray) -> np.ndarray:
    """bf16 is the upper half of an IEEE binary32."""
    u32 = bits.astype(np.uint32) << 16
    return u32.view(np.float32).astype(np.float64)


def f16_bits_to_f64(bits: np.ndarray) -> np.ndarray:
    return bits.astype(np.uint16).view(np.float16).astype(np.float64)


def _e4m3_table() -> np.ndarray:
    """OCP FP8 E4M3 ("fn"): 1 sign, 4 exponent (bias 7), 3 mantissa bits;
    no infinities, S.1111.111 is NaN, subnormals m * 2^-9."""
    tab = np.empty(256, dtype=np.float64)
    for code in range(256):
        s = -1.0 if code & 0x80 else 1.0
        e = (code >> 3) & 0xF
        m = code & 0x7
        if e == 0xF and m == 0x7:
            tab[code] = np.nan
        elif e == 0:
            tab[code] = s * m * 2.0 ** -9
        else:
            tab[code] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return tab


E4M3_TABLE = _e4m3_table()


def e4m3_bits_to_f64(bits: np.ndarray) -> np.ndarray:
    return E4M3_TABLE[bits.astype(np.uint8)]


def f64_to_e4m3_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even quantisation to e4m3fn with saturation at 448;
    the sign is kept, also when the result rounds to zero (-0 is 0x80), as
    torch's float8_e4m3fn cast does for finite inputs within range."""
    x = np.asarray(x, dtype=np.float64)
    pos = np.sort(np.unique(E4M3_TABLE[np.isfinite(E4M3_TABLE) & (E4M3_TABLE >= 0)]))
    codes_pos = np.array([int(np.where(E4M3_TABLE == v)[0][0]) for v in pos], dtype=np.int64)
    a = np.minimum(np.abs(x), 448.0)
    idx = np.clip(np.searchsorted(pos, a), 1, len(pos) - 1)
    lo, hi = pos[idx - 1], pos[idx]
    dlo, dhi = a - lo, hi - a
    take_hi = (dhi < dlo) | ((dhi == dlo) & ((codes_pos[idx] & 1) == 0))
    code = np.where(take_hi, codes_pos[idx], codes_pos[idx - 1])
    code = np.where(a <= 0.0, 0, code)
    sign = np.where(np.signbit(x), 0x80, 0)
    return (code | sign).astype(np.uint8)


# ---------------------------------------------------------------------------
# dense decode (torch_sdpa_benchmark.py:100-102)
# ---------------------------------------------------------------------------


def dense_decode(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float):
    """q [Hq, D], k/v [Hkv, S, Dk/Dv] float64 -> out [Hq, Dv], lse [Hq].

    Query head h uses KV head h // (Hq // Hkv) (SDPA enable_gqa).  S == 0
    gives out = 0 and lse = -inf (the library's defined empty-sequence
    result)."""
    hq = q.shape[0]
    hkv = k.shape[0]
    group = hq // hkv
    out = np.zeros((hq, v.shape[-1]), dtype=np.float64)
    lse = np.full((hq,), -np.inf, dtype=np.float64)
    if k.shape[1] == 0:
        return out, lse
    for g in range(hkv):   # the `group` query heads of KV head g at once
        hs = slice(g * group, (g + 1) * group)
        s = (q[hs] @ k[g].T) * scale            # [group, S]
        m = s.max(axis=1, keepdims=True)
        e = np.exp(s - m)
        den = e.sum(axis=1)
        out[hs] = (e @ v[g]) / den[:, None]
        lse[hs] = m[:, 0] + np.log(den)
    return out, lse


# ---------------------------------------------------------------------------
# paged decode (flashattn_kvcache_kernel.py:150-169 semantics)
# ---------------------------------------------------------------------------


def gather_pages(cache: np.ndarray, block_table_row: np.ndarray, length: int, page_size: int):
    """cache [num_pages, P, Hkv, D] -> [Hkv, length, D] for one sequence."""
    npages = (length + page_size - 1) // page_size
    pages = block_table_row[:npages]
    toks = cache[pages].reshape(npages * page_size, *cache.shape[2:])[:length]
    return np.transpose(toks, (1, 0, 2))


def paged_decode(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale,
                 k_scale=None, v_scale=None):
    """All inputs float64 numpy (already converted).

    q [B, Hq, D]; k_cache/v_cache [num_pages, P, Hkv, D] (NHD);
    cache_seqlens [B]; block_table [B, max_pages]; k_scale/v_scale [Hkv] or
    None.  Returns out [B, Hq, D], lse [B, Hq] (natural log)."""
    bsz, hq, _ = q.shape
    page = k_cache.shape[1]
    out = np.zeros((bsz, hq, v_cache.shape[-1]), dtype=np.float64)
    lse = np.full((bsz, hq), -np.inf, dtype=np.float64)
    for b in range(bsz):
        length = int(cache_seqlens[b])
        k = gather_pages(k_cache, block_table[b], length, page)
        v = gather_pages(v_cache, block_table[b], length, page)
        if k_scale is not None:
            k = k * np.asarray(k_scale, dtype=np.float64)[:, None, None]
        if v_scale is not None:
            v = v * np.asarray(v_scale, dtype=np.float64)[:, None, None]
        out[b], lse[b] = dense_decode(q[b], k, v, softmax_scale)
    return out, lse


def paged_decode_mla(q, kv_cache, cache_seqlens, block_table, softmax_scale, head_dim_v=512):
    """Absorbed MLA (trtllm_mla_kernel.py:115-132): q [B, H, 576],
    kv_cache [num_pages, P, 576]; K = all columns, V = first head_dim_v."""
    kv4 = kv_cache[:, :, None, :]
    bsz, h, _ = q.shape
    out = np.zeros((bsz, h, head_dim_v))
    lse = np.full((bsz, h), -np.inf)
    for b in range(bsz):
        length = int(cache_seqlens[b])
        kv = gather_pages(kv4, block_table[b], length, kv_cache.shape[1])
        out[b], lse[b] = dense_decode(q[b], kv, kv[:, :, :head_dim_v], softmax_scale)
    return out, lse


# ---------------------------------------------------------------------------
# split-KV partials + merge (cluster_decode_reduce.py:16-91)
# ---------------------------------------------------------------------------


def split_partials(q, k, v, num_splits: int, scale: float):
    """q [BH, D], k/v [BH, S, D] -> (m [BH, n], l [BH, n], o [BH, n, D]):
    slice r covers tokens [r*ceil(S/n), (r+1)*ceil(S/n)) and holds its own
    max, sum of exp(s - max) and unnormalised exp-weighted V sum; empty
    slices keep m = -inf, l = 0, o = 0 (cluster_decode_reduce.py:16-64)."""
    bh, s_len, _ = k.shape
    m = np.full((bh, num_splits), -np.inf)
    l = np.zeros((bh, num_splits))
    o = np.zeros((bh, num_splits, v.shape[-1]))
    per = (s_len + num_splits - 1) // num_splits
    for r in range(num_splits):
        a, b = r * per, min((r + 1) * per, s_len)
        if a >= b:
            continue
        sc = np.einsum("hd,hsd->hs", q, k[:, a:b]) * scale
        mx = sc.max(axis=1)
        e = np.exp(sc - mx[:, None])
        m[:, r] = mx
        l[:, r] = e.sum(axis=1)
        o[:, r] = np.einsum("hs,hsd->hd", e, v[:, a:b])
    return m, l, o


def merge_partials(m, l, o):
    """M = max m_i; L = sum l_i e^(m_i - M); O = sum O_i e^(m_i - M) / L
    (cluster_decode_reduce.py:67-91).  Returns (out, lse = M + ln L)."""
    big = m.max(axis=1)
    w = np.where(np.isfinite(m), np.exp(m - big[:, None]), 0.0)
    den = (l * w).sum(axis=1)
    num = (o * w[:, :, None]).sum(axis=1)
    return num / den[:, None], big + np.log(den)


# ---------------------------------------------------------------------------
# KV-cache append (vllm_paged_kernel.py:160-172, reshape_and_cache)
# ---------------------------------------------------------------------------


def append_kv(cache, rows, slots, page_size, scale=None, fp8=False):
    """Reference for b2d_append_kv on one cache (numpy, in place).

    cache: [num_pages, P, H, D] array of stored values (uint8 e4m3 codes when
    fp8, else float); rows: [T, H, D] float32 source values; slots: [T] int
    (negative = skip, >= num_pages * P = skip and counted).  FP8 stores
    e4m3(x * (1 / scale)) computed in float32, round-to-nearest-even,
    saturated.  Returns the number of out-of-range slots."""
    cap = cache.shape[0] * page_size
    bad = 0
    for t, slot in enumerate(np.asarray(slots).tolist()):
        if slot < 0:
            continue
        if slot >= cap:
            bad += 1
            continue
        page, off = divmod(slot, page_size)
        x = np.asarray(rows[t], dtype=np.float32)
        if fp8:
            inv = (np.float32(1.0) / np.asarray(scale, dtype=np.float32))[:, None]
            cache[page, off] = f64_to_e4m3_bits((x * inv).astype(np.float32).astype(np.float64))
        else:
            cache[page, off] = x
    return bad
