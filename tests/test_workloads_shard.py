"""Host logic: seeded workloads, block tables, byte accounting, sharding
(including a world-size-2 gloo all-gather on CPU)."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from b200decode import shard
from b200decode import workloads as W


def test_block_table_is_a_permutation_of_the_pool():
    sl = W.draw_seqlens(64, 1024, 8192, 0)
    bt, n = W.make_block_table(sl, 16, True, 0)
    used = torch.cat([bt[b, : (int(l) + 15) // 16] for b, l in enumerate(sl.tolist())])
    assert n == sum((int(l) + 15) // 16 for l in sl.tolist())
    assert sorted(used.tolist()) == list(range(n))
    assert used.tolist() != list(range(n))  # permuted


def test_seeded_and_bounded():
    a = W.draw_seqlens(64, 1024, 8192, 0)
    assert torch.equal(a, W.draw_seqlens(64, 1024, 8192, 0))
    assert int(a.min()) >= 1024 and int(a.max()) <= 8192


def test_algorithmic_bytes_cfg2_near_survey_figure():
    sl = W.draw_seqlens(64, 1024, 8192, 0)
    b = W.gqa_algorithmic_bytes(W.CFG2_GQA_PAGED, sl)
    kv = W.gqa_kv_bytes_reference(W.CFG2_GQA_PAGED, sl)
    assert kv == int(sl.sum()) * 8 * 128 * 2 * 2
    assert 0 < b - kv < 2_000_000
    assert W.gqa_algorithmic_bytes(W.CFG3_LONG_SPLITKV, torch.full((4,), 131072)) > 2_147_483_648


def test_balance_sequences_covers_each_once_and_balances():
    sl = W.draw_seqlens(256, 2048, 8192, 0).tolist()
    parts = shard.balance_sequences(sl, 8)
    flat = sorted(i for p in parts for i in p)
    assert flat == list(range(256))
    loads = [sum(sl[i] for i in p) for p in parts]
    assert max(loads) - min(loads) <= max(sl)


def test_head_shard():
    assert shard.head_shard(32, 8, 8, 3) == (slice(12, 16), slice(3, 4))
    with pytest.raises(ValueError):
        shard.head_shard(32, 8, 3, 0)


def test_slice_by_batch_keeps_only_own_pages():
    x = W.make_gqa_inputs(W.CFG2_GQA_PAGED.scaled(batch=6, seqlen_lo=3, seqlen_hi=50), "cpu")
    y = shard.slice_gqa_inputs_by_batch(x, [1, 4])
    assert y["k_cache"].shape[0] == sum((int(l) + 15) // 16 for l in y["cache_seqlens"].tolist())
    for j, b in enumerate([1, 4]):
        n = (int(x["cache_seqlens"][b]) + 15) // 16
        assert torch.equal(y["k_cache"][y["block_table"][j, :n].long()],
                           x["k_cache"][x["block_table"][b, :n].long()])


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _gather_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        b, hq, d = 3, 8, 4
        full = torch.arange(b * hq * d, dtype=torch.float32).view(b, hq, d)
        lse_full = torch.arange(b * hq, dtype=torch.float32).view(b, hq)
        qs, _ = shard.head_shard(hq, 4, world, rank)
        out, lse = shard.gather_heads(full[:, qs].contiguous(), lse_full[:, qs].contiguous())
        ok = bool(torch.equal(out, full) and torch.equal(lse, lse_full))
        # the preallocated packed form, twice (buffers are reused per step)
        hg = shard.HeadGather(b, hq // world, d, torch.float32, "cpu")
        for k in range(2):
            hg.out_local.copy_(full[:, qs] + k)
            hg.lse_local.copy_(lse_full[:, qs] - k)
            out, lse = hg.gather()
            ok = ok and bool(torch.equal(out, full + k) and torch.equal(lse, lse_full - k))
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tp_head_gather_layout_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_gather_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(60)
    res = dict(q.get(timeout=10) for _ in range(world))
    assert res == {r: True for r in range(world)}


def test_decodebench_shape_matches_reference_record():
    from b200decode.decodebench import DecodeShape
    s = DecodeShape(64, 4096, 32, 8, 128, "bf16", 16)
    assert s.attention == "GQA" and s.kv_bytes == 64 * 4096 * 8 * 128 * 2 * 2
    assert DecodeShape(1, 10, 8, 8, 64, "fp8", 16).kv_bytes == 10 * 8 * 64 * 2
    assert DecodeShape(1, 10, 8, 1, 64, "fp16", 16).attention == "MQA"


def test_to_vllm_layout_element_mapping():
    """K [blocks, Hkv, D/x, P, x] (x = 16 bytes of elements), V [blocks, Hkv, D, P]
    (decodebench/vllm_paged_kernel.py:102-123) hold the NHD cache's values."""
    pages, P, H, D = 3, 16, 2, 64
    k = torch.randn(pages, P, H, D).to(torch.bfloat16)
    v = torch.randn(pages, P, H, D).to(torch.bfloat16)
    kv, vv = W.to_vllm_layout(k, v)
    x = 8
    assert kv.shape == (pages, H, D // x, P, x) and vv.shape == (pages, H, D, P)
    assert kv.is_contiguous() and vv.is_contiguous()
    for (pg, t, h, d) in [(0, 0, 0, 0), (2, 15, 1, 63), (1, 7, 0, 9), (2, 3, 1, 40)]:
        assert kv[pg, h, d // x, t, d % x] == k[pg, t, h, d]
        assert vv[pg, h, d, t] == v[pg, t, h, d]


def test_decodebench_mla_cli_defaults_match_reference_flags():
    """`decodebench mla` takes trtllm_mla_benchmark.py's flags and defaults."""
    from b200decode import decodebench
    a = decodebench.parse_mla_args(["--batch-size", "2", "--context-len", "10",
                                    "--num-q-heads", "128", "--kv-dtype", "bf16",
                                    "--output", "x.json"])
    assert (a.num_kv_heads, a.qk_nope_head_dim, a.kv_lora_rank, a.qk_rope_head_dim,
            a.page_size, a.warmup_steps, a.repeat) == (1, 128, 512, 64, 64, 10, 50)
    shape = decodebench.MlaDecodeShape(32, 32768, 128, 1, 128, 512, 64, "bf16", 64)
    assert shape.head_dim_qk == 192 and shape.kv_bytes == 32 * 32768 * 576 * 2
    g = decodebench.parse_args(["--batch-size", "1", "--context-len", "5", "--num-q-heads", "8",
                                "--num-kv-heads", "8", "--head-dim", "128", "--kv-dtype", "bf16",
                                "--page-size", "16", "--output", "y.json", "--kv-layout", "vllm"])
    assert g.kv_layout == "vllm"


def test_fp8_cache_generation_saturates_instead_of_nan():
    """Config-5 style FP8 caches (scales down to 0.01, so N(0,1)/scale can
    exceed 448) hold no e4m3 NaN code: values are saturated like a quantiser."""
    from b200decode import workloads as W
    w = W.CFG5_FP8.scaled(batch=8, seqlen_lo=2000, seqlen_hi=4000, kv_scale_range=(0.01, 0.011))
    x = W.make_gqa_inputs(w, "cpu")
    for c in (x["k_cache"], x["v_cache"]):
        bits = c.view(torch.uint8)
        assert int(((bits & 0x7F) == 0x7F).sum()) == 0
        assert int(((bits & 0x7F) == 0x7E).sum()) > 0   # some values did saturate to 448
