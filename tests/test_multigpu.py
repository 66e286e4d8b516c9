"""Multi-GPU sharding over NCCL (one process per GPU): batch-sharded (DP)
and KV-head-sharded (TP, all-gather of out/lse) decodes must match the
single-GPU decode of the whole batch within the parity tolerance (the split
plan, hence the fp32 merge order, depends on the shard's shape).  Skips with
fewer than 2 GPUs."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, mode, q):
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parent.parent
    sys.path[:0] = [str(repo), str(repo / "roofline-analysis_b200")]
    import b200decode
    from b200decode import shard
    from b200decode import workloads as W
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        w = W.CFG5_FP8.scaled(batch=24, seqlen_lo=100, seqlen_hi=2000, seed=7)
        x = W.make_gqa_inputs(w, dev)
        full_out, full_lse = b200decode.decode(x["q"], x["k_cache"], x["v_cache"], x["cache_seqlens"],
                                               x["block_table"], x["softmax_scale"],
                                               k_scale=x["k_scale"], v_scale=x["v_scale"])
        if mode == "tp":
            y = shard.slice_gqa_inputs_by_heads(x, world, rank)
            o, l = b200decode.decode(y["q"], y["k_cache"], y["v_cache"], y["cache_seqlens"],
                                     y["block_table"], y["softmax_scale"], k_scale=y["k_scale"],
                                     v_scale=y["v_scale"])
            o, l = shard.gather_heads(o, l)
            ok = bool(((o.float() - full_out.float()).abs() <= 2e-2 + 1e-2 * full_out.float().abs()).all()
                      and ((l - full_lse).abs() <= 1e-3).all())
        else:
            rows = shard.balance_sequences(x["cache_seqlens"].tolist(), world)[rank]
            y = shard.slice_gqa_inputs_by_batch(x, rows)
            o, l = b200decode.decode(y["q"], y["k_cache"], y["v_cache"], y["cache_seqlens"],
                                     y["block_table"], y["softmax_scale"], k_scale=y["k_scale"],
                                     v_scale=y["v_scale"])
            idx = torch.as_tensor(rows, device=dev)
            ok = bool(((o.float() - full_out[idx].float()).abs() <= 2e-2 + 1e-2 * full_out[idx].float().abs()).all()
                      and ((l - full_lse[idx]).abs() <= 1e-3).all())
        torch.cuda.synchronize()
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["tp", "dp"])
def test_two_gpu_sharding_matches_single_gpu(mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
    res = dict(q.get(timeout=30) for _ in range(2))
    assert res == {0: True, 1: True}
