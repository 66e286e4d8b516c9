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
