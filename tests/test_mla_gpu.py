"""GPU parity of the absorbed-MLA tcgen05 decode kernel against the CPU
oracle (decodebench/trtllm_mla_kernel.py:115-132 semantics), through the C ABI
(b200decode.decode_mla -> libb2d.so)."""
import numpy as np
import pytest
import torch

import b200decode
from b200decode import workloads as W
from helpers import assert_parity, oracle_mla_streamed, to_oracle
from oracle import decode_ref as R

pytestmark = pytest.mark.gpu

SMALL = W.MlaWorkload("mla_small", 3, 128, 576, 512, 64, 1, 300, seed=5)


def _inputs(cuda, w, lens=None):
    sl = None if lens is None else torch.tensor(lens, dtype=torch.int64)
    return W.make_mla_inputs(w, cuda, seqlens=sl)


def _oracle(x, rows=None):
    q = to_oracle(x["q"])
    kv = to_oracle(x["kv_cache"])
    sl = x["cache_seqlens"].cpu().numpy()
    bt = x["block_table"].cpu().numpy()
    if rows is not None:
        q, sl, bt = q[rows], sl[rows], bt[rows]
    return R.paged_decode_mla(q, kv, sl, bt, x["softmax_scale"])


def _run(x, **kw):
    out, lse = b200decode.decode_mla(x["q"], x["kv_cache"], x["cache_seqlens"], x["block_table"],
                                     x["softmax_scale"], **kw)
    torch.cuda.synchronize()
    b200decode.check_device_status()
    return out, lse


def test_mla_single_short_sequence(cuda):
    x = _inputs(cuda, SMALL, lens=[40])
    out, lse = _run(x)
    assert_parity(out, lse, *_oracle(x))


def test_mla_ragged_batch(cuda):
    x = _inputs(cuda, SMALL, lens=[1, 33, 64, 65, 300, 0, 17])
    out, lse = _run(x)
    assert_parity(out, lse, *_oracle(x))


@pytest.mark.parametrize("num_ctas", [2, 6, 64, 296])
def test_mla_split_counts_agree(cuda, num_ctas):
    x = _inputs(cuda, SMALL.scaled(seqlen_lo=100, seqlen_hi=3000), lens=None)
    out, lse = _run(x, num_ctas=num_ctas)
    assert_parity(out, lse, *_oracle(x))


def test_mla_nan_in_page_tail_is_ignored(cuda):
    x = _inputs(cuda, SMALL, lens=[5, 70])
    bt = x["block_table"].cpu()
    for b, l in enumerate([5, 70]):
        last = bt[b, (l - 1) // 64].item()
        x["kv_cache"][last, l % 64:] = float("nan")
    out, lse = _run(x)
    assert torch.isfinite(out.float()).all()
    assert_parity(out, lse, *_oracle(x))


def test_mla_large_scores_trigger_rescale(cuda):
    """Scores that grow along the sequence force the lazy rescale path."""
    x = _inputs(cuda, SMALL, lens=[600])
    L = 600
    pages = x["block_table"][0, : (L + 63) // 64].long()
    ramp = torch.linspace(0.2, 4.0, L, device=cuda)
    kv = x["kv_cache"][pages].reshape(-1, 576)[:L].float()
    kv *= ramp[:, None]
    x["kv_cache"][pages] = torch.cat([kv, torch.zeros(len(pages) * 64 - L, 576, device=cuda)]).reshape(
        len(pages), 64, 576).to(torch.bfloat16)
    out, lse = _run(x)
    assert_parity(out, lse, *_oracle(x))


def test_mla_cfg4_full(cuda):
    """Config 4 at full size: every sequence and head against the oracle."""
    x = _inputs(cuda, W.CFG4_MLA)
    out, lse = _run(x)
    assert_parity(out, lse, *oracle_mla_streamed(x))


def test_mla_batch_larger_than_one_launch(cuda):
    """More sequences than one launch's row table (384): the host slices the
    batch, offsetting q, lengths, block table, out and lse per slice."""
    rng = np.random.default_rng(11)
    lens = rng.integers(1, 140, size=400).tolist()
    lens[5] = 0
    lens[390] = 0
    x = _inputs(cuda, SMALL.scaled(batch=400), lens=lens)
    out, lse = _run(x)
    rows = [0, 5, 17, 383, 384, 385, 390, 399]
    ro, rl = _oracle(x, rows=rows)
    assert_parity(out[rows], lse[rows], ro, rl)


def test_mla_rejects_unsupported_shapes(cuda):
    x = _inputs(cuda, SMALL, lens=[10])
    with pytest.raises(b200decode.B2DError):
        b200decode.decode_mla(x["q"][:, :64].contiguous(), x["kv_cache"], x["cache_seqlens"],
                              x["block_table"])


def test_decodebench_mla_adapter(cuda, tmp_path):
    """`python -m b200decode.decodebench mla ...` (trtllm_mla_benchmark.py's
    flags and record); the adapter's run() output matches the oracle."""
    import json
    from b200decode import decodebench
    shape = decodebench.MlaDecodeShape(2, 300, 128, 1, 128, 512, 64, "bf16", 64)
    k = decodebench.B2DMlaKernel(shape, seed=1)
    out, lse = k.run()
    torch.cuda.synchronize()
    x = dict(k.x, softmax_scale=k.scale)
    assert_parity(out, lse, *_oracle(x))
    with pytest.raises(ValueError):
        decodebench.B2DMlaKernel(decodebench.MlaDecodeShape(2, 300, 64, 1, 128, 512, 64, "bf16", 64))
    path = tmp_path / "m.json"
    rc = decodebench.main(["mla", "--batch-size", "4", "--context-len", "1000", "--num-q-heads",
                           "128", "--kv-dtype", "bf16", "--page-size", "64", "--warmup-steps", "2",
                           "--repeat", "5", "--output", str(path)])
    assert rc == 0
    d = json.loads(path.read_text())
    assert d["attention"] == "MLA" and d["approx_kv_bytes_read"] == 4 * 1000 * 576 * 2
    for key in ("kernel_latency_p50_us", "approx_effective_kv_bandwidth_gb_s", "fallback"):
        assert key in d
