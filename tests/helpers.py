"""Shared test helpers: torch tensors -> oracle inputs, tolerance checks."""
from __future__ import annotations

import numpy as np
import torch

from oracle import decode_ref as R

# Parity bar: out max-abs 2e-2 with rtol 1e-2, lse 1e-3 (absolute, natural log).
OUT_ATOL, OUT_RTOL, LSE_ATOL = 2e-2, 1e-2, 1e-3


def to_oracle(t: torch.Tensor) -> np.ndarray:
    """Any bf16/fp16/fp8/fp32 tensor -> float64 numpy through the oracle's own
    bit-level conversions."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return R.bf16_bits_to_f64(t.view(torch.int16).numpy().view(np.uint16))
    if t.dtype == torch.float16:
        return R.f16_bits_to_f64(t.view(torch.int16).numpy().view(np.uint16))
    if t.dtype == torch.float8_e4m3fn:
        return R.e4m3_bits_to_f64(t.view(torch.uint8).numpy())
    return t.double().numpy()


def oracle_gqa(x, rows=None):
    """Oracle out/lse for a make_gqa_inputs() dict (optionally only the
    sequences `rows`)."""
    q = to_oracle(x["q"])
    kc, vc = to_oracle(x["k_cache"]), to_oracle(x["v_cache"])
    sl = x["cache_seqlens"].cpu().numpy()
    bt = x["block_table"].cpu().numpy()
    ks = None if x.get("k_scale") is None else x["k_scale"].cpu().double().numpy()
    vs = None if x.get("v_scale") is None else x["v_scale"].cpu().double().numpy()
    if rows is not None:
        q, sl, bt = q[rows], sl[rows], bt[rows]
    return R.paged_decode(q, kc, vc, sl, bt, x["softmax_scale"], ks, vs)


def assert_parity(out, lse, ref_out, ref_lse, rows=None, atol=OUT_ATOL, rtol=OUT_RTOL,
                  lse_atol=LSE_ATOL):
    o = to_oracle(out)
    l = lse.detach().cpu().double().numpy()
    if rows is not None:
        o, l = o[rows], l[rows]
    o = o.reshape(ref_out.shape)
    err = np.abs(o - ref_out)
    bad = ~(err <= atol + rtol * np.abs(ref_out))
    assert not bad.any(), (f"out mismatch: max abs err {np.nanmax(err):.3e} at "
                           f"{np.unravel_index(np.nanargmax(err), err.shape)}")
    fin = np.isfinite(ref_lse)
    assert np.array_equal(np.isneginf(l), np.isneginf(ref_lse)), "lse -inf pattern differs"
    lerr = np.abs(l[fin] - ref_lse[fin]) if fin.any() else np.zeros(1)
    assert lerr.max() <= lse_atol, f"lse mismatch: max abs err {lerr.max():.3e}"
    return float(err.max()), float(lerr.max())


def _compact_pages(x, rows, cache_keys):
    """Only the pages that sequences `rows` use, gathered on the device and
    converted for the oracle, with a block table renumbered to match."""
    page = x[cache_keys[0]].shape[1]
    sl = x["cache_seqlens"][rows].cpu().numpy()
    bt = x["block_table"][rows]
    npg = [(int(l) + page - 1) // page for l in sl]
    idx = [bt[j, :n].long() for j, n in enumerate(npg) if n]
    pages = torch.cat(idx) if idx else torch.zeros(1, dtype=torch.long, device=bt.device)
    caches = [to_oracle(x[k][pages]) for k in cache_keys]
    new_bt = np.zeros((len(rows), max(1, max(npg))), dtype=np.int64)
    off = 0
    for j, n in enumerate(npg):
        new_bt[j, :n] = np.arange(off, off + n)
        off += n
    return caches, sl, new_bt


def oracle_gqa_streamed(x, rows=None, chunk=8):
    """oracle_gqa over sequences `rows` (default: all), `chunk` sequences at
    a time, converting only the pages they use (full-size caches do not fit
    in host memory as float64)."""
    bsz = x["q"].shape[0]
    rows = list(range(bsz)) if rows is None else list(rows)
    q = to_oracle(x["q"])
    ks = None if x.get("k_scale") is None else x["k_scale"].cpu().double().numpy()
    vs = None if x.get("v_scale") is None else x["v_scale"].cpu().double().numpy()
    outs, lses = [], []
    for i in range(0, len(rows), chunk):
        rr = rows[i:i + chunk]
        (kc, vc), sl, bt = _compact_pages(x, rr, ("k_cache", "v_cache"))
        o, l = R.paged_decode(q[rr], kc, vc, sl, bt, x["softmax_scale"], ks, vs)
        outs.append(o)
        lses.append(l)
    return np.concatenate(outs), np.concatenate(lses)


def oracle_mla_streamed(x, rows=None, chunk=8):
    """The MLA oracle over sequences `rows` (default: all), chunked likewise."""
    bsz = x["q"].shape[0]
    rows = list(range(bsz)) if rows is None else list(rows)
    q = to_oracle(x["q"])
    outs, lses = [], []
    for i in range(0, len(rows), chunk):
        rr = rows[i:i + chunk]
        (kv,), sl, bt = _compact_pages(x, rr, ("kv_cache",))
        o, l = R.paged_decode_mla(q[rr], kv, sl, bt, x["softmax_scale"])
        outs.append(o)
        lses.append(l)
    return np.concatenate(outs), np.concatenate(lses)
