"""Regenerates the golden fixtures in this folder from the reference itself.

Run in a checkout where the reference repository is available:

    python tests/golden/make_golden.py /path/to/Roofline-Analysis

Fixtures written:

* split_merge_bh3_s129_d128.npz — inputs and outputs of the reference's own
  split-KV contract, cute_attention/cluster_decode/cluster_decode_reduce.py
  (split_kv_decode_partials :16-64, merge_split_kv_decode_partials :67-91,
  split_kv_decode_reference :94-97) at the shape of its test
  cute_attention/cluster_decode/tests/test_correctness.py:34-46
  (batch_heads=3, seq_len=129, head_dim=128, cluster sizes 2 and 4), plus
  the test's fp32 decode_reference (:24-27).
* sdpa_paged_gqa.npz — a small paged GQA decode (bf16 inputs, ragged
  lengths including 1 and a partial last page, permuted pages) answered by
  the reference's decode call, F.scaled_dot_product_attention(..., is_causal=
  False, enable_gqa=True) (decodebench/torch_sdpa_benchmark.py:100-102), run
  in fp32 on the gathered pages; lse from torch.logsumexp of the same scores.
* sdpa_paged_mla.npz — a small absorbed-MLA decode whose geometry comes
  from the reference's own shape record, decodebench/trtllm_mla_kernel.py:
  7-26 (TRTLLMMLADecodeShape: latent row = kv_lora_rank + qk_rope_head_dim
  columns, V = the first kv_lora_rank of them, softmax scale 1/sqrt(
  head_dim_qk) as at :77), answered by the same SDPA call with one shared
  KV head (enable_gqa) on the gathered latent pages.

Nothing under tests/ or the package imports the reference at run time; the
tests read only the .npz files.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent


def split_merge_fixture(ref_root: Path) -> None:
    sys.path.insert(0, str(ref_root / "cute_attention"))
    from cluster_decode.cluster_decode_reduce import (  # noqa: E402
        leader_reduce_payload_floats, merge_split_kv_decode_partials, split_kv_decode_partials,
        split_kv_decode_reference)

    torch.manual_seed(1234)
    bh, s, d = 3, 129, 128
    scale = d ** -0.5
    q = torch.randn(bh, 1, d, dtype=torch.float32)
    k = torch.randn(bh, s, d, dtype=torch.float32)
    v = torch.randn(bh, s, d, dtype=torch.float32)
    scores = torch.matmul(q, k.transpose(-2, -1)) * scale
    dense = torch.matmul(torch.softmax(scores, dim=-1), v)
    rec = dict(q=q.numpy(), k=k.numpy(), v=v.numpy(), scale=np.float64(scale),
               dense_out=dense.numpy(), payload_floats=np.int64(leader_reduce_payload_floats(d)))
    for cs in (2, 4):
        pm, ps, po = split_kv_decode_partials(q, k, v, cs, scale)
        rec[f"m_{cs}"] = pm.numpy()
        rec[f"l_{cs}"] = ps.numpy()
        rec[f"o_{cs}"] = po.numpy()
        rec[f"merged_{cs}"] = merge_split_kv_decode_partials(pm, ps, po).numpy()
        rec[f"split_ref_{cs}"] = split_kv_decode_reference(q, k, v, cs, scale).numpy()
    np.savez_compressed(HERE / "split_merge_bh3_s129_d128.npz", **rec)


def sdpa_paged_fixture() -> None:
    g = torch.Generator().manual_seed(99)
    b, hq, hkv, d, page = 3, 8, 2, 64, 16
    lens = [1, 37, 100]
    npg = [(l + page - 1) // page for l in lens]
    total = sum(npg)
    perm = torch.randperm(total, generator=g)
    bt = torch.zeros(b, max(npg), dtype=torch.int32)
    off = 0
    for i, n in enumerate(npg):
        bt[i, :n] = perm[off:off + n].int()
        off += n
    q = torch.randn(b, hq, d, generator=g).to(torch.bfloat16)
    kc = torch.randn(total, page, hkv, d, generator=g).to(torch.bfloat16)
    vc = torch.randn(total, page, hkv, d, generator=g).to(torch.bfloat16)
    scale = d ** -0.5
    outs, lses = [], []
    for i, l in enumerate(lens):
        idx = bt[i, :npg[i]].long()
        k = kc[idx].reshape(-1, hkv, d)[:l].permute(1, 0, 2).float()[None]
        v = vc[idx].reshape(-1, hkv, d)[:l].permute(1, 0, 2).float()[None]
        qq = q[i:i + 1, :, None, :].float()
        o = F.scaled_dot_product_attention(qq, k, v, is_causal=False, scale=scale, enable_gqa=True)
        outs.append(o[0, :, 0].numpy())
        kk = k[0].repeat_interleave(hq // hkv, dim=0)
        sc = torch.einsum("hd,hsd->hs", qq[0, :, 0], kk) * scale
        lses.append(torch.logsumexp(sc, dim=-1).numpy())
    np.savez_compressed(
        HERE / "sdpa_paged_gqa.npz",
        q_bits=q.view(torch.int16).numpy(), k_bits=kc.view(torch.int16).numpy(),
        v_bits=vc.view(torch.int16).numpy(), block_table=bt.numpy(),
        seqlens=np.array(lens, dtype=np.int32), scale=np.float64(scale),
        out=np.stack(outs), lse=np.stack(lses))


def sdpa_paged_mla_fixture(ref_root: Path) -> None:
    sys.path.insert(0, str(ref_root / "decodebench"))
    from trtllm_mla_kernel import TRTLLMMLADecodeShape  # noqa: E402

    shape = TRTLLMMLADecodeShape(batch_size=2, context_len=70, num_q_heads=8, num_kv_heads=1,
                                 qk_nope_head_dim=128, kv_lora_rank=512, qk_rope_head_dim=64,
                                 kv_dtype="bf16", page_size=64)
    width = shape.kv_lora_rank + shape.qk_rope_head_dim
    dv = shape.kv_lora_rank
    scale = 1.0 / (shape.head_dim_qk ** 0.5)
    g = torch.Generator().manual_seed(7)
    lens = [1, shape.context_len]
    page = shape.page_size
    npg = [(l + page - 1) // page for l in lens]
    total = sum(npg)
    perm = torch.randperm(total, generator=g)
    bt = torch.zeros(shape.batch_size, max(npg), dtype=torch.int32)
    off = 0
    for i, n in enumerate(npg):
        bt[i, :n] = perm[off:off + n].int()
        off += n
    q = (0.5 * torch.randn(shape.batch_size, shape.num_q_heads, width, generator=g)).to(torch.bfloat16)
    kv = (0.5 * torch.randn(total, page, width, generator=g)).to(torch.bfloat16)
    outs, lses = [], []
    for i, l in enumerate(lens):
        rows = kv[bt[i, :npg[i]].long()].reshape(-1, width)[:l].float()
        k = rows[None, None]
        v = rows[None, None, :, :dv]
        qq = q[i:i + 1, :, None, :].float()
        o = F.scaled_dot_product_attention(qq, k, v, is_causal=False, scale=scale, enable_gqa=True)
        outs.append(o[0, :, 0].numpy())
        sc = (qq[0, :, 0] @ rows.T) * scale
        lses.append(torch.logsumexp(sc, dim=-1).numpy())
    np.savez_compressed(
        HERE / "sdpa_paged_mla.npz",
        q_bits=q.view(torch.int16).numpy(), kv_bits=kv.view(torch.int16).numpy(),
        block_table=bt.numpy(), seqlens=np.array(lens, dtype=np.int32), scale=np.float64(scale),
        head_dim_v=np.int64(dv), out=np.stack(outs), lse=np.stack(lses))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/Roofline-Analysis")
    root = Path(sys.argv[1])
    split_merge_fixture(root)
    sdpa_paged_fixture()
    sdpa_paged_mla_fixture(root)
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))
