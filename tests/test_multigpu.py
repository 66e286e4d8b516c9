"""Multi-GPU sharding over NCCL (one process per GPU): batch-sharded (DP)
and KV-head-sharded (TP, packed all-gather of out/lse) decodes are compared
with the CPU oracle of the whole batch within the parity tolerance.  Skips
with fewer than 2 GPUs.  NVLS is off (NCCL_NVLS_ENABLE=0) and every process
group has a bounded timeout."""
import datetime
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
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        sys.path.insert(0, str(repo / "tests"))
        from helpers import OUT_ATOL, OUT_RTOL, LSE_ATOL, oracle_gqa_streamed, to_oracle
        import numpy as np
        w = W.CFG5_FP8.scaled(batch=24, seqlen_lo=100, seqlen_hi=2000, seed=7)
        x = W.make_gqa_inputs(w, dev)
        ref_out, ref_lse = oracle_gqa_streamed(x)

        def close(o, l, ro, rl):
            o = to_oracle(o).reshape(ro.shape)
            l = l.detach().cpu().double().numpy()
            return bool((np.abs(o - ro) <= OUT_ATOL + OUT_RTOL * np.abs(ro)).all()
                        and (np.abs(l - rl) <= LSE_ATOL).all())

        if mode == "tp":
            y = shard.slice_gqa_inputs_by_heads(x, world, rank)
            hg = shard.HeadGather(w.batch, w.num_q_heads // world, w.head_dim, x["q"].dtype, dev)
            ok = True
            for _ in range(2):   # the gather buffers are reused step after step
                b200decode.decode(y["q"], y["k_cache"], y["v_cache"], y["cache_seqlens"],
                                  y["block_table"], y["softmax_scale"], k_scale=y["k_scale"],
                                  v_scale=y["v_scale"], out=hg.out_local, lse=hg.lse_local)
                o, l = hg.gather()
                ok = ok and close(o, l, ref_out, ref_lse)
        else:
            rows = shard.balance_sequences(x["cache_seqlens"].tolist(), world)[rank]
            y = shard.slice_gqa_inputs_by_batch(x, rows, seed=rank)
            o, l = b200decode.decode(y["q"], y["k_cache"], y["v_cache"], y["cache_seqlens"],
                                     y["block_table"], y["softmax_scale"], k_scale=y["k_scale"],
                                     v_scale=y["v_scale"])
            ok = close(o, l, ref_out[rows], ref_lse[rows])
        b200decode.check_device_status()
        torch.cuda.synchronize()
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["tp", "dp"])
def test_two_gpu_sharding_matches_oracle(mode):
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
