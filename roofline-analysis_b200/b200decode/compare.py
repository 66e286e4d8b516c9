"""Same-box comparison with the reference's sm_100 bars.

The reference (decodebench/) publishes decode timings of third-party B200
kernels measured on another machine.  This module times this library and
those kernels, as installed here, on the SAME inputs on the SAME GPU:

* TRT-LLM-gen paged decode, flashinfer.decode.trtllm_batch_decode_with_kv_cache
  (the call of decodebench/trtllm_decode_kernel.py:102-113), given this
  library's own NHD caches as a (k_cache, v_cache) tuple, so both kernels
  read identical memory;
* TRT-LLM-gen MLA, flashinfer.decode.trtllm_batch_decode_with_kv_cache_mla
  (decodebench/trtllm_mla_kernel.py:115-132) on the same latent cache;
* cuDNN SDPA on dense caches, torch SDPA under the cuDNN backend
  (decodebench/torch_sdpa_benchmark.py:95-106).

Timing follows the reference: warm-up calls, then one CUDA-event pair per
call and the p50 (decodebench/flashinfer_benchmark.py:17-35,
matrix_b200.py:9-13).  Every row also reports the largest difference
between the two outputs.  The vendor kernels are comparators only: nothing
in the library calls them.

    python -m b200decode.compare [--rows published|configs|all] [--json out.jsonl]
"""
from __future__ import annotations

import argparse
import json
import math
import sys
from typing import Callable, Optional

import torch

from . import api
from . import workloads as W

WARMUP, REPEAT = 20, 100


def _p50_us(fn: Callable, warmup: int = WARMUP, repeat: int = REPEAT) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(repeat)]
    for a, b in evs:
        a.record()
        fn()
        b.record()
    torch.cuda.synchronize()
    t = sorted(a.elapsed_time(b) for a, b in evs)
    return t[len(t) // 2] * 1e3


def _gqa_row(name: str, w: W.GqaWorkload, published: Optional[tuple]) -> dict:
    dev = torch.device("cuda")
    x = W.make_gqa_inputs(w, dev)
    kc, vc = x["k_cache"], x["v_cache"]
    fp8 = kc.dtype == torch.float8_e4m3fn
    ours = api.GqaDecoder(x["q"], kc, vc, x["cache_seqlens"], x["block_table"],
                          x["softmax_scale"], k_scale=x["k_scale"], v_scale=x["v_scale"])
    row = {"row": name, "kind": "gqa", "batch": w.batch, "hq": w.num_q_heads,
           "hkv": w.num_kv_heads, "head_dim": w.head_dim, "page": w.page_size,
           "kv_dtype": w.kv_dtype, "seqlen": [w.seqlen_lo, w.seqlen_hi]}
    row["b2d_us"] = _p50_us(ours.run)
    out_ours = ours.run()[0].float().clone()
    kv_bytes = W.gqa_kv_bytes_reference(w, x["cache_seqlens"].cpu())
    row["b2d_kv_gbs"] = kv_bytes / (row["b2d_us"] * 1e3)
    try:
        import flashinfer
        ws = torch.zeros(1 << 30, dtype=torch.int8, device=dev)
        out = torch.empty_like(x["q"])
        scale = x["softmax_scale"]
        k_s = float(x["k_scale"][0]) if fp8 and x["k_scale"] is not None else 1.0
        v_s = float(x["v_scale"][0]) if fp8 and x["v_scale"] is not None else 1.0
        max_len = int(x["cache_seqlens"].max())

        def vendor():
            return flashinfer.decode.trtllm_batch_decode_with_kv_cache(
                query=x["q"], kv_cache=(kc, vc), workspace_buffer=ws,
                block_tables=x["block_table"], seq_lens=x["cache_seqlens"],
                max_seq_len=max_len, bmm1_scale=scale * k_s, bmm2_scale=v_s, out=out,
                kv_layout="NHD")

        row["vendor"] = "flashinfer trtllm_batch_decode_with_kv_cache"
        row["vendor_us"] = _p50_us(vendor)
        vendor()
        torch.cuda.synchronize()
        row["max_abs_diff"] = float((out.float() - out_ours).abs().max())
        row["speedup"] = row["vendor_us"] / row["b2d_us"]
    except Exception as e:  # an unsupported shape is a result, not a failure
        row["vendor"] = "flashinfer trtllm_batch_decode_with_kv_cache"
        row["vendor_error"] = f"{type(e).__name__}: {str(e).splitlines()[0][:200]}"
    if published:
        row["published_us"], row["published_backend"] = published
    return row


def _mla_row(name: str, w: W.MlaWorkload, published: Optional[tuple]) -> dict:
    dev = torch.device("cuda")
    x = W.make_mla_inputs(w, dev)
    out_o = torch.empty(w.batch, w.num_heads, w.head_dim_v, dtype=torch.bfloat16, device=dev)
    lse_o = torch.empty(w.batch, w.num_heads, dtype=torch.float32, device=dev)

    def ours():
        return api.decode_mla(x["q"], x["kv_cache"], x["cache_seqlens"], x["block_table"],
                              x["softmax_scale"], out=out_o, lse=lse_o)

    row = {"row": name, "kind": "mla", "batch": w.batch, "heads": w.num_heads,
           "page": w.page_size, "seqlen": [w.seqlen_lo, w.seqlen_hi]}
    row["b2d_us"] = _p50_us(ours)
    ours()
    out_ours = out_o.float().clone()
    kv_bytes = int(x["cache_seqlens"].sum()) * w.head_dim_qk * 2
    row["b2d_kv_gbs"] = kv_bytes / (row["b2d_us"] * 1e3)
    try:
        import flashinfer
        ws = torch.zeros(64 << 20, dtype=torch.uint8, device=dev)
        q4 = x["q"][:, None]
        out = torch.empty(w.batch, 1, w.num_heads, w.head_dim_v, dtype=torch.bfloat16, device=dev)
        max_len = int(x["cache_seqlens"].max())

        def vendor():
            return flashinfer.decode.trtllm_batch_decode_with_kv_cache_mla(
                query=q4, kv_cache=x["kv_cache"], workspace_buffer=ws,
                qk_nope_head_dim=128, kv_lora_rank=512, qk_rope_head_dim=64,
                block_tables=x["block_table"], seq_lens=x["cache_seqlens"], max_seq_len=max_len,
                out=out, bmm1_scale=x["softmax_scale"], bmm2_scale=1.0)

        row["vendor"] = "flashinfer trtllm_batch_decode_with_kv_cache_mla"
        row["vendor_us"] = _p50_us(vendor)
        vendor()
        torch.cuda.synchronize()
        row["max_abs_diff"] = float((out[:, 0].float() - out_ours).abs().max())
        row["speedup"] = row["vendor_us"] / row["b2d_us"]
    except Exception as e:
        row["vendor"] = "flashinfer trtllm_batch_decode_with_kv_cache_mla"
        row["vendor_error"] = f"{type(e).__name__}: {str(e).splitlines()[0][:200]}"
    if published:
        row["published_us"], row["published_backend"] = published
    return row


def _dense_row(name: str, batch: int, heads: int, seqlen: int, published: Optional[tuple]) -> dict:
    """Dense MHA decode: cuDNN SDPA vs this library reading each dense
    [H, S, D] block in place (b200decode.cluster_decode)."""
    from torch.nn.attention import SDPBackend, sdpa_kernel
    from . import cluster_decode
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(1)
    q = torch.randn(batch, heads, 1, 128, generator=g, device=dev, dtype=torch.bfloat16)
    k = torch.randn(batch, heads, seqlen, 128, generator=g, device=dev, dtype=torch.bfloat16)
    v = torch.randn(batch, heads, seqlen, 128, generator=g, device=dev, dtype=torch.bfloat16)
    row = {"row": name, "kind": "dense", "batch": batch, "heads": heads, "seqlen": seqlen}
    ours = lambda: cluster_decode.cluster_decode_forward(q, k, v)
    row["b2d_us"] = _p50_us(ours)
    o1 = ours().float()
    row["b2d_kv_gbs"] = 2 * batch * heads * seqlen * 128 * 2 / (row["b2d_us"] * 1e3)
    try:
        def vendor():
            with sdpa_kernel(SDPBackend.CUDNN_ATTENTION):
                return torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=False)
        row["vendor"] = "torch SDPA, cuDNN backend"
        row["vendor_us"] = _p50_us(vendor)
        row["max_abs_diff"] = float((vendor().float() - o1).abs().max())
        row["speedup"] = row["vendor_us"] / row["b2d_us"]
    except Exception as e:
        row["vendor"] = "torch SDPA, cuDNN backend"
        row["vendor_error"] = f"{type(e).__name__}: {str(e).splitlines()[0][:200]}"
    if published:
        row["published_us"], row["published_backend"] = published
    return row


def _uniform(name, batch, hq, hkv, ctx, page, dt):
    return W.GqaWorkload(name, batch, hq, hkv, 128, page, dt, ctx, ctx, page_perm=False)


# The reference's published decodebench rows (uniform length, identity page
# order, unit FP8 scales), with the best published backend and p50.
PUBLISHED = [
    ("gqa bf16 B=128 ctx8k p64", _uniform("r1", 128, 32, 8, 8192, 64, "bf16"), (600.1, "trtllm-gen")),
    ("gqa bf16 B=64 ctx4k p64", _uniform("r2", 64, 32, 8, 4096, 64, "bf16"), (171.1, "trtllm-gen")),
    ("gqa bf16 B=64 ctx4k p16", _uniform("r3", 64, 32, 8, 4096, 16, "bf16"), (226.8, "FA4")),
    ("gqa bf16 B=1 ctx128k p64", _uniform("r4", 1, 32, 8, 131072, 64, "bf16"), (98.8, "trtllm-gen")),
    ("gqa fp8 B=128 ctx8k p64", _uniform("r5", 128, 32, 8, 8192, 64, "fp8"), (510.9, "trtllm-gen")),
    ("gqa fp8 B=32 ctx32k p64", _uniform("r6", 32, 32, 8, 32768, 64, "fp8"), (580.7, "trtllm-gen")),
    ("gqa fp8 B=1 ctx128k p64", _uniform("r7", 1, 32, 8, 131072, 64, "fp8"), (88.8, "trtllm-gen")),
    ("mha bf16 B=16 ctx4k p64", _uniform("r8", 16, 32, 32, 4096, 64, "bf16"), (168.9, "trtllm-gen")),
    ("gqa bf16 B=1 ctx4k p64", _uniform("r9", 1, 32, 8, 4096, 64, "bf16"), (25.1, "trtllm-gen")),
]
PUBLISHED_MLA = [
    ("mla bf16 B=32 ctx32k p64", W.MlaWorkload("m1", 32, 128, 576, 512, 64, 32768, 32768), (265.1, "trtllm-gen mla")),
    ("mla bf16 B=64 ctx4k p64", W.MlaWorkload("m2", 64, 128, 576, 512, 64, 4096, 4096), (84.1, "trtllm-gen mla")),
]
PUBLISHED_DENSE = [
    ("dense mha bf16 B=64 H=32 ctx4k", 64, 32, 4096, (176.7, "torch_sdpa_cudnn (gqa 32/8)")),
]


def unit_scales(w: W.GqaWorkload) -> W.GqaWorkload:
    """The comparators take one scalar K and V scale: same-box FP8 rows use
    unit per-head scales."""
    return w.scaled(kv_scale_range=None) if w.kv_dtype == "fp8" else w


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--rows", choices=["published", "configs", "all"], default="all")
    ap.add_argument("--json", default=None, help="write one JSON line per row here")
    args = ap.parse_args(argv)
    rows = []
    if args.rows in ("published", "all"):
        for name, w, pub in PUBLISHED:
            rows.append(_gqa_row(name, w, pub))
        for name, w, pub in PUBLISHED_MLA:
            rows.append(_mla_row(name, w, pub))
        for name, b, h, s, pub in PUBLISHED_DENSE:
            rows.append(_dense_row(name, b, h, s, pub))
    if args.rows in ("configs", "all"):
        rows.append(_gqa_row("BASELINE cfg2", W.CFG2_GQA_PAGED, None))
        rows.append(_gqa_row("BASELINE cfg3", W.CFG3_LONG_SPLITKV, None))
        rows.append(_gqa_row("BASELINE cfg5 (unit scales)", unit_scales(W.CFG5_FP8), None))
        rows.append(_mla_row("BASELINE cfg4", W.CFG4_MLA, None))
    out = open(args.json, "w") if args.json else None
    for r in rows:
        line = json.dumps(r)
        print(line, flush=True)
        if out:
            out.write(line + "\n")
    print(f"{'row':34s} {'b2d us':>9s} {'vendor us':>10s} {'speedup':>8s} {'maxdiff':>8s} {'published':>10s}",
          file=sys.stderr)
    for r in rows:
        print(f"{r['row']:34s} {r['b2d_us']:9.1f} {r.get('vendor_us', float('nan')):10.1f} "
              f"{r.get('speedup', float('nan')):8.3f} {r.get('max_abs_diff', float('nan')):8.4f} "
              f"{r.get('published_us', float('nan')):10.1f} {r.get('vendor_error', '')}", file=sys.stderr)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
