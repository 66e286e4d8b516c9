"""GPU parity of the split-KV GQA decode kernel against the CPU oracle,
called through the C ABI (b200decode.decode -> libb2d.so)."""
import numpy as np
import pytest
import torch

import b200decode
from b200decode import workloads as W
from helpers import assert_parity, oracle_gqa, oracle_gqa_streamed, to_oracle
from oracle import decode_ref as R

pytestmark = pytest.mark.gpu


def _run(x, **kw):
    out, lse = b200decode.decode(x["q"], x["k_cache"], x["v_cache"], x["cache_seqlens"],
                                 x["block_table"], x["softmax_scale"], k_scale=x["k_scale"],
                                 v_scale=x["v_scale"], **kw)
    torch.cuda.synchronize()
    b200decode.check_device_status()
    return out, lse


def _inputs(cuda, w, lens=None):
    sl = None if lens is None else torch.tensor(lens, dtype=torch.int64)
    return W.make_gqa_inputs(w, cuda, seqlens=sl)


SMALL = W.GqaWorkload("small", 5, 8, 2, 128, 16, "bf16", 1, 300, seed=3)


@pytest.mark.parametrize("hq,hkv", [(8, 8), (8, 4), (8, 2), (16, 2), (32, 4), (32, 1), (6, 2), (3, 1)])
def test_group_sizes(cuda, hq, hkv):
    x = _inputs(cuda, SMALL.scaled(num_q_heads=hq, num_kv_heads=hkv))
    out, lse = _run(x)
    assert_parity(out, lse, *oracle_gqa(x))


@pytest.mark.parametrize("d", [64, 128, 256])
@pytest.mark.parametrize("dt", ["bf16", "fp16", "fp8"])
def test_head_dims_and_dtypes(cuda, d, dt):
    qdt = "fp16" if dt == "fp16" else "bf16"
    w = SMALL.scaled(head_dim=d, kv_dtype=dt, q_dtype=qdt,
                     kv_scale_range=(0.01, 0.1) if dt == "fp8" else None)
    x = _inputs(cuda, w)
    out, lse = _run(x)
    assert_parity(out, lse, *oracle_gqa(x))


@pytest.mark.parametrize("dt", ["bf16", "fp16"])
@pytest.mark.parametrize("hq,hkv,page", [(8, 2, 16), (32, 2, 64), (16, 16, 32)])
def test_head_dim_192(cuda, dt, hq, hkv, page):
    """head_dim 192 (tensor-core path, 16-bit caches)."""
    w = SMALL.scaled(head_dim=192, kv_dtype=dt, q_dtype=dt, num_q_heads=hq, num_kv_heads=hkv,
                     page_size=page)
    x = _inputs(cuda, w, lens=[1, page + 3, 5 * page, 300, 0])
    out, lse = _run(x)
    assert_parity(out, lse, *oracle_gqa(x))


@pytest.mark.parametrize("kw", [dict(kv_dtype="fp8", kv_scale_range=(0.01, 0.1)),
                                dict(page_size=8)])
def test_head_dim_192_unsupported_combinations(cuda, kw):
    """fp8 at head_dim 192, or a page size that is not a multiple of 16,
    is refused with B2D_ERR_UNSUPPORTED rather than computed wrongly."""
    x = _inputs(cuda, SMALL.scaled(head_dim=192, **kw))
    with pytest.raises(b200decode.B2DError, match="(?i)unsupported"):
        _run(x)


# Extended sweep (decodebench matrix_b200_extended.py:28-40 and
# matrix_b200.py:214-228 shapes, at test sizes): GQA ratios 2-16, MQA
# (group 32), head_dim 64 and 128, page 128.
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("hq,hkv", [(16, 8), (32, 8), (32, 4), (32, 2), (32, 1)])
def test_extended_sweep_page128(cuda, d, hq, hkv):
    w = SMALL.scaled(head_dim=d, num_q_heads=hq, num_kv_heads=hkv, page_size=128)
    x = _inputs(cuda, w, lens=[1, 127, 128, 129, 700])
    out, lse = _run(x)
    assert_parity(out, lse, *oracle_gqa(x))


@pytest.mark.parametrize("page", [1, 4, 8, 16, 32, 64, 128, 48])
def test_page_sizes(cuda, page):
    w = SMALL.scaled(page_size=page)
    x = _inputs(cuda, w, lens=[1, page - 1 if page > 1 else 2, page, page + 1, 3 * page + 5])
    out, lse = _run(x)
    assert_parity(out, lse, *oracle_gqa(x))


def test_empty_and_tiny_sequences(cuda):
    x = _inputs(cuda, SMALL, lens=[0, 1, 0, 2, 17])
    out, lse = _run(x)
    assert_parity(out, lse, *oracle_gqa(x))
    assert torch.all(out[0] == 0) and torch.all(torch.isneginf(lse[0]))


def test_all_empty_batch(cuda):
    x = _inputs(cuda, SMALL, lens=[0, 0, 0])
    out, lse = _run(x)
    assert torch.all(out == 0) and torch.all(torch.isneginf(lse))


@pytest.mark.parametrize("num_ctas", [1, 2, 3, 7, 64, 296, 1000])
def test_split_counts_agree(cuda, num_ctas):
    """Every CTA count partitions the same work differently (whole rows,
    split rows, rows over many CTAs, more CTAs than chunks); all must match."""
    x = _inputs(cuda, SMALL.scaled(batch=4, seqlen_lo=1, seqlen_hi=2000))
    out, lse = _run(x, num_ctas=num_ctas)
    assert_parity(out, lse, *oracle_gqa(x))


def test_hnd_layout_and_strided_views(cuda):
    """TRT-LLM-style HND cache [pages, 2, Hkv, P, D] passed as K/V views."""
    x = _inputs(cuda, SMALL.scaled(page_size=64))
    kc, vc = x["k_cache"], x["v_cache"]
    both = torch.stack([kc.permute(0, 2, 1, 3), vc.permute(0, 2, 1, 3)], dim=1).contiguous()
    out, lse = b200decode.decode(x["q"], both[:, 0], both[:, 1], x["cache_seqlens"],
                                 x["block_table"], x["softmax_scale"], kv_layout="HND")
    torch.cuda.synchronize()
    assert_parity(out, lse, *oracle_gqa(x))


@pytest.mark.parametrize("dt", ["bf16", "fp16"])
@pytest.mark.parametrize("d,hq,hkv,page", [(128, 32, 8, 16), (128, 8, 2, 64), (64, 16, 4, 32),
                                           (256, 8, 1, 16), (192, 8, 2, 16), (128, 32, 32, 16)])
def test_vllm_cache_layout(cuda, dt, d, hq, hkv, page):
    """vLLM paged_attention's own cache layout (K [blocks, Hkv, D/x, P, x],
    V [blocks, Hkv, D, P]; decodebench/vllm_paged_kernel.py:102-123) gives
    the same decode as the NHD copy of the same cache."""
    w = SMALL.scaled(head_dim=d, kv_dtype=dt, q_dtype=dt, num_q_heads=hq, num_kv_heads=hkv,
                     page_size=page)
    x = _inputs(cuda, w, lens=[1, page - 1, 3 * page + 5, 300, 0])
    kv, vv = W.to_vllm_layout(x["k_cache"], x["v_cache"])
    out, lse = b200decode.decode(x["q"], kv, vv, x["cache_seqlens"], x["block_table"],
                                 x["softmax_scale"], kv_layout="vllm")
    torch.cuda.synchronize()
    b200decode.check_device_status()
    assert_parity(out, lse, *oracle_gqa(x))


def test_vllm_cache_layout_decoder_and_refusals(cuda):
    x = _inputs(cuda, SMALL.scaled(num_q_heads=16, num_kv_heads=4))
    kv, vv = W.to_vllm_layout(x["k_cache"], x["v_cache"])
    dec = b200decode.GqaDecoder(x["q"], kv, vv, x["cache_seqlens"], x["block_table"],
                                x["softmax_scale"], kv_layout="vllm")
    dec.capture()
    out, lse = dec.replay()
    torch.cuda.synchronize()
    assert_parity(out, lse, *oracle_gqa(x))
    # page size 8 is not a multiple of 16: refused, not computed wrongly
    x8 = _inputs(cuda, SMALL.scaled(page_size=8))
    k8, v8 = W.to_vllm_layout(x8["k_cache"], x8["v_cache"])
    with pytest.raises(b200decode.B2DError, match="(?i)unsupported"):
        b200decode.decode(x8["q"], k8, v8, x8["cache_seqlens"], x8["block_table"],
                          kv_layout="vllm")
    with pytest.raises(ValueError):
        b200decode.decode(x["q"], kv[:, :, :, :, :4], vv, x["cache_seqlens"], x["block_table"],
                          kv_layout="vllm")


def test_q_with_token_axis_and_preallocated_outputs(cuda):
    x = _inputs(cuda, SMALL)
    q4 = x["q"][:, None]
    out = torch.full_like(q4, float("nan"))
    lse = torch.full((q4.shape[0], q4.shape[2]), float("nan"), device=cuda)
    o2, l2 = b200decode.decode(q4, x["k_cache"], x["v_cache"], x["cache_seqlens"],
                               x["block_table"], x["softmax_scale"], out=out, lse=lse)
    torch.cuda.synchronize()
    assert o2 is out and l2 is lse
    assert_parity(out[:, 0], lse, *oracle_gqa(x))


def test_nan_in_page_tail_is_ignored(cuda):
    """Slots past a sequence's length (same page) hold garbage; they must not
    leak into the result."""
    x = _inputs(cuda, SMALL, lens=[5, 19])
    bt = x["block_table"].cpu()
    for b, l in enumerate([5, 19]):
        last = bt[b, (l - 1) // 16].item()
        x["k_cache"][last, l % 16:] = float("nan")
        x["v_cache"][last, l % 16:] = float("inf")
    out, lse = _run(x)
    assert torch.isfinite(out.float()).all()
    assert_parity(out, lse, *oracle_gqa(x))


def test_batch_larger_than_one_launch(cuda):
    """More than 2048 rows: the host slices the batch into launches."""
    w = SMALL.scaled(batch=2100, num_q_heads=4, num_kv_heads=1, head_dim=64, seqlen_lo=1, seqlen_hi=40)
    x = _inputs(cuda, w)
    out, lse = _run(x)
    rows = np.r_[0:5, 2040:2060, 2095:2100]
    ref_out, ref_lse = oracle_gqa(x, rows=rows)
    assert_parity(out, lse, ref_out, ref_lse, rows=rows)


def test_deterministic(cuda):
    x = _inputs(cuda, SMALL.scaled(batch=8, seqlen_hi=3000))
    o1, l1 = _run(x)
    o2, l2 = _run(x)
    assert torch.equal(o1, o2) and torch.equal(l1, l2)


def test_out_of_range_page_id_is_reported(cuda):
    """The kernel clamps a bad page id to page 0 (no out-of-bounds access)
    and records it in the status word."""
    x = _inputs(cuda, SMALL, lens=[20, 20])
    x["block_table"][1, 0] = x["k_cache"].shape[0] + 5
    b200decode.decode(x["q"], x["k_cache"], x["v_cache"], x["cache_seqlens"], x["block_table"])
    with pytest.raises(b200decode.B2DError, match="out of range"):
        b200decode.check_device_status()
    b200decode.check_device_status()  # cleared


def test_errors_surface_as_exceptions(cuda):
    x = _inputs(cuda, SMALL)
    with pytest.raises(ValueError):
        b200decode.decode(x["q"].float(), x["k_cache"], x["v_cache"], x["cache_seqlens"], x["block_table"])
    with pytest.raises(ValueError):
        b200decode.decode(x["q"], x["k_cache"], x["v_cache"], x["cache_seqlens"].long(), x["block_table"])


# ---------------- BASELINE configurations at full size ----------------

def test_cfg1_mha_dense(cuda):
    x = _inputs(cuda, W.CFG1_MHA_CPU)
    out, lse = _run(x)
    assert_parity(out, lse, *oracle_gqa(x))


def test_cfg2_gqa_paged_full(cuda):
    """Config 2 at full size, every sequence and head against the oracle."""
    x = _inputs(cuda, W.CFG2_GQA_PAGED)
    out, lse = _run(x)
    assert_parity(out, lse, *oracle_gqa_streamed(x))


def test_cfg5_fp8_full(cuda):
    """Config 5 (FP8 KV, per-head scales) at full size, every sequence."""
    x = _inputs(cuda, W.CFG5_FP8)
    out, lse = _run(x)
    assert_parity(out, lse, *oracle_gqa_streamed(x))


def test_cfg3_long_context_full(cuda):
    """B=4 x 131072 tokens: every sequence and every KV head (all 64 query
    heads) against the oracle, one (sequence, KV head) at a time, plus
    invariance of the result under a very different split count."""
    w = W.CFG3_LONG_SPLITKV
    x = _inputs(cuda, w)
    out, lse = _run(x)
    g = w.num_q_heads // w.num_kv_heads
    for b in range(w.batch):
        L = int(x["cache_seqlens"][b])
        pages = x["block_table"][b, : (L + w.page_size - 1) // w.page_size].long()
        for h in range(w.num_kv_heads):
            k = to_oracle(x["k_cache"][pages][:, :, h].reshape(-1, w.head_dim)[:L])[None]
            v = to_oracle(x["v_cache"][pages][:, :, h].reshape(-1, w.head_dim)[:L])[None]
            q = to_oracle(x["q"][b, h * g:(h + 1) * g])
            ro, rl = R.dense_decode(q, k, v, w.softmax_scale)
            assert_parity(out[b, h * g:(h + 1) * g], lse[b, h * g:(h + 1) * g], ro, rl)
    out2, lse2 = _run(x, num_ctas=37)
    assert (out2.float() - out.float()).abs().max().item() < 1e-2
    assert (lse2 - lse).abs().max().item() < 1e-4


def test_wait_timeout_is_reported_and_recovers(cuda):
    """The bounded-wait path: with B2D_FLAG_TEST_NO_LOADS the producer
    issues no copies, so every consumer wait runs out after 1 ms, records a
    timeout in the status word and returns (nothing is in flight).  The
    status read-back raises it; a normal decode on the same workspace then
    passes parity."""
    from b200decode import _lib
    x = _inputs(cuda, SMALL.scaled(batch=8, seqlen_hi=600))
    ws = b200decode.DecodeWorkspace(cuda)
    kw = dict(k_scale=x["k_scale"], v_scale=x["v_scale"], workspace=ws)
    args = (x["q"], x["k_cache"], x["v_cache"], x["cache_seqlens"], x["block_table"],
            x["softmax_scale"])
    b200decode.decode(*args, flags=_lib.B2D_FLAG_TEST_NO_LOADS, wait_limit_us=1000, **kw)
    torch.cuda.synchronize()
    with pytest.raises(b200decode.B2DError) as e:
        b200decode.check_device_status(ws)
    assert e.value.code == -6   # B2D_ERR_DEVICE_TIMEOUT
    b200decode.check_device_status(ws)   # cleared by the read above
    out, lse = b200decode.decode(*args, **kw)
    torch.cuda.synchronize()
    b200decode.check_device_status(ws)
    assert_parity(out, lse, *oracle_gqa(x))


def test_decoder_plan_run_and_graph_replay(cuda):
    """Plan/run object and its CUDA-graph replay give the decode() result,
    and pick up in-place refills of q and the lengths."""
    x = _inputs(cuda, SMALL.scaled(batch=6, seqlen_hi=900))
    dec = b200decode.GqaDecoder(x["q"], x["k_cache"], x["v_cache"], x["cache_seqlens"],
                                x["block_table"], x["softmax_scale"])
    out, lse = dec.run()
    torch.cuda.synchronize()
    assert_parity(out, lse, *oracle_gqa(x))
    dec.capture()
    x["q"].copy_(torch.randn_like(x["q"], dtype=torch.float32).to(x["q"].dtype))
    x["cache_seqlens"].copy_(torch.clamp(x["cache_seqlens"] - 7, min=0))
    out, lse = dec.replay()
    torch.cuda.synchronize()
    assert_parity(out, lse, *oracle_gqa(x))


def test_decodebench_adapter_writes_reference_schema(cuda, tmp_path):
    import json
    from b200decode import decodebench
    out = tmp_path / "r.json"
    rc = decodebench.main(["--batch-size", "8", "--context-len", "1000", "--num-q-heads", "32",
                           "--num-kv-heads", "8", "--head-dim", "128", "--kv-dtype", "bf16",
                           "--page-size", "16", "--warmup-steps", "2", "--repeat", "5",
                           "--output", str(out), "--cuda-graph"])
    assert rc == 0
    d = json.loads(out.read_text())
    for k in ("backend", "compare_latency_us", "kernel_latency_p50_us", "approx_kv_bytes_read",
              "approx_effective_kv_bandwidth_gb_s", "fallback", "attention"):
        assert k in d
    assert d["backend"] == "b2d_decode" and d["approx_kv_bytes_read"] == 8 * 1000 * 8 * 128 * 4
