"""decodebench backend "b2d_decode": the adapter pair the reference's harness
expects (decodebench/<x>_kernel.py + <x>_benchmark.py), for this library.

GQA/MHA/MQA:

Kernel side mirrors decodebench/flashinfer_kernel.py:41-116: the constructor
builds q, the paged caches, the lengths and the block table for a shape (the
reference's DecodeShape fields, decodebench/flashinfer_kernel.py:8-28), and
run() is the single timed call.  Benchmark side mirrors
decodebench/flashinfer_benchmark.py:17-103: warm-up, one CUDA-event pair per
run(), p50/p95/avg, and the same JSON record, extended with this library's
fields (lengths distribution, seed, roofline figures).

    python -m b200decode.decodebench --batch-size 64 --context-len 4096 \\
        --num-q-heads 32 --num-kv-heads 8 --head-dim 128 --kv-dtype bf16 \\
        --page-size 16 --output result.json [--seqlen-lo 1024 --seqlen-hi 8192]

Absorbed MLA (mirrors decodebench/trtllm_mla_kernel.py:7-25 and
trtllm_mla_benchmark.py:13-94; same shape fields, same record):

    python -m b200decode.decodebench mla --batch-size 32 --context-len 32768 \\
        --num-q-heads 128 --kv-dtype bf16 --page-size 64 --output result.json
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import math
import os
from datetime import datetime, timezone
from pathlib import Path
from typing import Optional

import torch

from . import api
from . import workloads as W


@dataclasses.dataclass(frozen=True)
class DecodeShape:
    """Field-for-field the reference's record (flashinfer_kernel.py:8-28)."""
    batch_size: int
    context_len: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    kv_dtype: str
    page_size: int

    @property
    def attention(self) -> str:
        if self.num_q_heads == self.num_kv_heads:
            return "MHA"
        if self.num_kv_heads == 1:
            return "MQA"
        return "GQA"

    @property
    def kv_bytes(self) -> int:
        dtype_bytes = 1 if self.kv_dtype == "fp8" else 2
        return (self.batch_size * self.context_len * self.num_kv_heads * self.head_dim * 2
                * dtype_bytes)


class B2DDecodeKernel:
    """Kernel(shape).run() adapter.  Lengths default to context_len for every
    sequence with identity page order (the reference's inputs); seqlen_lo /
    seqlen_hi / page_perm / seed select BASELINE-style distributions."""

    def __init__(self, shape: DecodeShape, seqlen_lo: Optional[int] = None,
                 seqlen_hi: Optional[int] = None, page_perm: bool = False, seed: int = 0,
                 kv_scale_range=None, use_graph: bool = False, kv_layout: str = "NHD"):
        if not torch.cuda.is_available():
            raise RuntimeError("CUDA is required")
        self.shape = shape
        lo = seqlen_lo if seqlen_lo is not None else shape.context_len
        hi = seqlen_hi if seqlen_hi is not None else shape.context_len
        fp8 = shape.kv_dtype == "fp8"
        self.workload = W.GqaWorkload(
            "decodebench", shape.batch_size, shape.num_q_heads, shape.num_kv_heads,
            shape.head_dim, shape.page_size, shape.kv_dtype, lo, hi,
            q_dtype="fp16" if shape.kv_dtype == "fp16" else "bf16", seed=seed,
            page_perm=page_perm, kv_scale_range=(kv_scale_range or ((1.0, 1.0) if fp8 else None)))
        self.x = W.make_gqa_inputs(self.workload, torch.device("cuda"))
        x = self.x
        kc, vc = x["k_cache"], x["v_cache"]
        if kv_layout == "HND":
            kc, vc = kc.transpose(1, 2).contiguous(), vc.transpose(1, 2).contiguous()
        elif kv_layout == "vllm":
            kc, vc = W.to_vllm_layout(kc, vc)
        elif kv_layout != "NHD":
            raise ValueError(f"unknown kv_layout {kv_layout!r}")
        self.kv_layout = kv_layout
        self.decoder = api.GqaDecoder(x["q"], kc, vc, x["cache_seqlens"], x["block_table"],
                                      x["softmax_scale"], k_scale=x["k_scale"],
                                      v_scale=x["v_scale"], kv_layout=kv_layout)
        self.use_graph = use_graph
        if use_graph:
            self.decoder.capture()

    def run(self):
        return self.decoder.replay() if self.use_graph else self.decoder.run()

    @property
    def algorithmic_bytes(self) -> int:
        return W.gqa_algorithmic_bytes(self.workload, self.x["cache_seqlens"].cpu())

    @property
    def kv_bytes_exact(self) -> int:
        return W.gqa_kv_bytes_reference(self.workload, self.x["cache_seqlens"].cpu())


@dataclasses.dataclass(frozen=True)
class MlaDecodeShape:
    """Field-for-field the reference's TRTLLMMLADecodeShape
    (decodebench/trtllm_mla_kernel.py:7-25)."""
    batch_size: int
    context_len: int
    num_q_heads: int
    num_kv_heads: int
    qk_nope_head_dim: int
    kv_lora_rank: int
    qk_rope_head_dim: int
    kv_dtype: str
    page_size: int

    @property
    def head_dim_qk(self) -> int:
        return self.qk_nope_head_dim + self.qk_rope_head_dim

    @property
    def kv_bytes(self) -> int:
        return self.batch_size * self.context_len * (self.kv_lora_rank + self.qk_rope_head_dim) * 2


class B2DMlaKernel:
    """Kernel(shape).run() adapter for absorbed MLA.  The shapes the library
    builds: 128 query heads, one latent KV head of kv_lora_rank 512 + rope 64,
    bf16, page size a multiple of 64.  softmax_scale = 1/sqrt(nope + rope), as
    the reference passes as bmm1_scale (trtllm_mla_kernel.py:71)."""

    def __init__(self, shape: MlaDecodeShape, seqlen_lo: Optional[int] = None,
                 seqlen_hi: Optional[int] = None, page_perm: bool = False, seed: int = 0):
        if not torch.cuda.is_available():
            raise RuntimeError("CUDA is required")
        if (shape.num_q_heads != 128 or shape.num_kv_heads != 1 or shape.kv_lora_rank != 512
                or shape.qk_rope_head_dim != 64 or shape.kv_dtype != "bf16"
                or shape.page_size % 64 != 0):
            raise ValueError("b2d MLA decode is built for 128 heads, kv_lora_rank 512, rope 64, "
                             "bf16, page size a multiple of 64")
        self.shape = shape
        lo = seqlen_lo if seqlen_lo is not None else shape.context_len
        hi = seqlen_hi if seqlen_hi is not None else shape.context_len
        self.workload = W.MlaWorkload("decodebench_mla", shape.batch_size, shape.num_q_heads,
                                      shape.kv_lora_rank + shape.qk_rope_head_dim,
                                      shape.kv_lora_rank, shape.page_size, lo, hi, seed=seed)
        dev = torch.device("cuda")
        self.x = W.make_mla_inputs(self.workload, dev, page_perm=page_perm)
        self.scale = 1.0 / math.sqrt(shape.head_dim_qk)
        self.out = torch.empty(shape.batch_size, shape.num_q_heads, shape.kv_lora_rank,
                               dtype=torch.bfloat16, device=dev)
        self.lse = torch.empty(shape.batch_size, shape.num_q_heads, dtype=torch.float32,
                               device=dev)
        self.workspace = api.DecodeWorkspace(dev)

    def run(self):
        x = self.x
        return api.decode_mla(x["q"], x["kv_cache"], x["cache_seqlens"], x["block_table"],
                              self.scale, head_dim_v=self.shape.kv_lora_rank, out=self.out,
                              lse=self.lse, workspace=self.workspace)

    @property
    def algorithmic_bytes(self) -> int:
        return W.mla_algorithmic_bytes(self.workload, self.x["cache_seqlens"].cpu())


def cuda_time_ms(fn, repeat: int) -> list:
    """One CUDA-event pair per call, synchronised (flashinfer_benchmark.py:17-27)."""
    times = []
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    for _ in range(repeat):
        start.record()
        fn()
        end.record()
        torch.cuda.synchronize()
        times.append(start.elapsed_time(end))
    return times


def percentile(values, pct: float) -> float:
    values = sorted(values)
    if not values:
        return float("nan")
    index = min(len(values) - 1, max(0, math.ceil(pct / 100 * len(values)) - 1))
    return values[index]


def parse_args(argv=None) -> argparse.Namespace:
    ap = argparse.ArgumentParser(description="Benchmark the b2d paged decode kernel.")
    ap.add_argument("--batch-size", type=int, required=True)
    ap.add_argument("--context-len", type=int, required=True)
    ap.add_argument("--num-q-heads", type=int, required=True)
    ap.add_argument("--num-kv-heads", type=int, required=True)
    ap.add_argument("--head-dim", type=int, required=True)
    ap.add_argument("--kv-dtype", required=True, choices=["bf16", "fp16", "fp8"])
    ap.add_argument("--page-size", type=int, required=True)
    ap.add_argument("--warmup-steps", type=int, default=20)
    ap.add_argument("--repeat", type=int, default=100)
    ap.add_argument("--output", type=Path, required=True)
    ap.add_argument("--seqlen-lo", type=int, default=None)
    ap.add_argument("--seqlen-hi", type=int, default=None)
    ap.add_argument("--page-perm", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cuda-graph", action="store_true")
    ap.add_argument("--kv-scale-range", type=float, nargs=2, default=None, metavar=("LO", "HI"),
                    help="fp8 only: per-KV-head dequantisation scales ~ U[LO, HI] "
                         "(default: unit scales, as the reference)")
    ap.add_argument("--ncu", action="store_true",
                    help="re-run once under Nsight Compute and merge DRAM bytes, traffic ratio "
                         "and tensor-pipe utilisation of the split-KV kernel into the record "
                         "(small cases only)")
    ap.add_argument("--num-gpus", type=int, default=1,
                    help="shard the batch (--shard dp) or the KV heads (--shard tp) over this "
                         "many GPUs, one process each (NCCL)")
    ap.add_argument("--shard", choices=["dp", "tp"], default="dp")
    ap.add_argument("--kv-layout", default="NHD", choices=["NHD", "HND", "vllm"],
                    help="cache layout handed to the kernel (vllm = paged_attention's "
                         "K [blocks, Hkv, D/8, P, 8], V [blocks, Hkv, D, P])")
    return ap.parse_args(argv)


def parse_mla_args(argv=None) -> argparse.Namespace:
    """Same flags and defaults as decodebench/trtllm_mla_benchmark.py:13-27."""
    ap = argparse.ArgumentParser(description="Benchmark the b2d absorbed-MLA decode kernel.")
    ap.add_argument("--batch-size", type=int, required=True)
    ap.add_argument("--context-len", type=int, required=True)
    ap.add_argument("--num-q-heads", type=int, required=True)
    ap.add_argument("--num-kv-heads", type=int, default=1)
    ap.add_argument("--qk-nope-head-dim", type=int, default=128)
    ap.add_argument("--kv-lora-rank", type=int, default=512)
    ap.add_argument("--qk-rope-head-dim", type=int, default=64)
    ap.add_argument("--kv-dtype", required=True, choices=["bf16", "fp16"])
    ap.add_argument("--page-size", type=int, default=64, choices=[64, 128])
    ap.add_argument("--warmup-steps", type=int, default=10)
    ap.add_argument("--repeat", type=int, default=50)
    ap.add_argument("--output", type=Path, required=True)
    ap.add_argument("--seqlen-lo", type=int, default=None)
    ap.add_argument("--seqlen-hi", type=int, default=None)
    ap.add_argument("--page-perm", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--ncu", action="store_true",
                    help="re-run once under Nsight Compute and merge the MLA kernel's counters "
                         "into the record (small cases only)")
    return ap.parse_args(argv)


def _child_argv(argv, mla: bool):
    """The same adapter command without --ncu (what ncu re-runs)."""
    a = [x for x in argv if x != "--ncu"]
    return (["mla"] if mla else []) + a


def main_mla(argv=None) -> int:
    import sys
    argv = sys.argv[2:] if argv is None else list(argv)
    args = parse_mla_args(argv)
    shape = MlaDecodeShape(args.batch_size, args.context_len, args.num_q_heads,
                           args.num_kv_heads, args.qk_nope_head_dim, args.kv_lora_rank,
                           args.qk_rope_head_dim, args.kv_dtype, args.page_size)
    kernel = B2DMlaKernel(shape, args.seqlen_lo, args.seqlen_hi, args.page_perm, args.seed)
    for _ in range(args.warmup_steps):
        kernel.run()
    torch.cuda.synchronize()
    times_ms = cuda_time_ms(kernel.run, args.repeat)
    avg_ms = sum(times_ms) / len(times_ms)
    p50_ms = percentile(times_ms, 50)
    p95_ms = percentile(times_ms, 95)
    alg = kernel.algorithmic_bytes
    result = {
        "run_id": os.environ.get("DECODEBENCH_RUN_ID"),
        "timestamp": datetime.now(timezone.utc).isoformat(),
        "gpu": torch.cuda.get_device_name(),
        "backend": "b2d_mla_decode",
        "kernel_path": "b2d mla_decode_kernel (sm_100a, tcgen05) via libb2d.so",
        "layer": "kernel",
        "workload_id": os.environ.get("DECODEBENCH_WORKLOAD_ID"),
        "attention": "MLA",
        "kv_dtype": shape.kv_dtype,
        "page_size": shape.page_size,
        "batch_size": shape.batch_size,
        "context_len": shape.context_len,
        "decode_steps": 1,
        "kernel_latency_avg_us": avg_ms * 1000.0,
        "kernel_latency_p50_us": p50_ms * 1000.0,
        "kernel_latency_p95_us": p95_ms * 1000.0,
        "approx_kv_bytes_read": shape.kv_bytes,
        "approx_effective_kv_bandwidth_gb_s": shape.kv_bytes / (p50_ms * 1e6),
        "peak_allocated_gb": torch.cuda.max_memory_allocated() / 1e9,
        "selected_backend": "b2d_mla_decode",
        "fallback": False,
        "fallback_reason": None,
        "notes": "Absorbed-MLA decode through b200decode.decode_mla (one C-ABI call per run).",
        "roofline_bytes": alg,
        "achieved_tb_s": alg / (p50_ms * 1e-3) / 1e12,
        "seqlen_lo": kernel.workload.seqlen_lo,
        "seqlen_hi": kernel.workload.seqlen_hi,
        "seed": args.seed,
        "page_perm": args.page_perm,
    }
    if args.ncu:
        from . import ncu_harness
        result["ncu"] = ncu_harness.capture(_child_argv(argv, True), "mla", skip=args.warmup_steps,
                                            count=min(3, args.repeat), algorithmic_bytes=alg)
    args.output.parent.mkdir(parents=True, exist_ok=True)
    args.output.write_text(json.dumps(result, indent=2) + "\n", encoding="utf-8")
    print(json.dumps(result))
    return 0


def main(argv=None) -> int:
    import sys
    argv = sys.argv[1:] if argv is None else list(argv)
    if argv and argv[0] == "mla":
        return main_mla(argv[1:])
    args = parse_args(argv)
    shape = DecodeShape(args.batch_size, args.context_len, args.num_q_heads, args.num_kv_heads,
                        args.head_dim, args.kv_dtype, args.page_size)
    if args.num_gpus > 1:
        return main_multi_gpu(args, shape)
    kernel = B2DDecodeKernel(shape, args.seqlen_lo, args.seqlen_hi, args.page_perm, args.seed,
                             kv_scale_range=(tuple(args.kv_scale_range) if args.kv_scale_range
                                             else None),
                             use_graph=args.cuda_graph, kv_layout=args.kv_layout)
    for _ in range(args.warmup_steps):
        kernel.run()
    torch.cuda.synchronize()
    times_ms = cuda_time_ms(kernel.run, args.repeat)
    avg_ms = sum(times_ms) / len(times_ms)
    p50_ms = percentile(times_ms, 50)
    p95_ms = percentile(times_ms, 95)
    kv_bytes = kernel.kv_bytes_exact
    alg = kernel.algorithmic_bytes
    result = {
        "run_id": os.environ.get("DECODEBENCH_RUN_ID"),
        "timestamp": datetime.now(timezone.utc).isoformat(),
        "gpu": torch.cuda.get_device_name(),
        "backend": "b2d_decode",
        "kernel_path": "b2d gqa_mma_kernel (sm_100a) via libb2d.so",
        "layer": "kernel",
        "workload_id": os.environ.get("DECODEBENCH_WORKLOAD_ID"),
        "attention": shape.attention,
        "kv_dtype": shape.kv_dtype,
        "page_size": shape.page_size,
        "batch_size": shape.batch_size,
        "context_len": shape.context_len,
        "decode_steps": 1,
        "compare_latency_us": p50_ms * 1000.0,
        "kernel_latency_avg_us": avg_ms * 1000.0,
        "kernel_latency_p50_us": p50_ms * 1000.0,
        "kernel_latency_p95_us": p95_ms * 1000.0,
        "approx_kv_bytes_read": kv_bytes,
        "approx_effective_kv_bandwidth_gb_s": kv_bytes / (p50_ms * 1e6),
        "peak_allocated_gb": torch.cuda.max_memory_allocated() / 1e9,
        "selected_backend": "b2d_decode",
        "fallback": False,
        "fallback_reason": None,
        "notes": "Paged decode through b200decode.GqaDecoder.run (one C-ABI call per run).",
        "roofline_bytes": alg,
        "achieved_tb_s": alg / (p50_ms * 1e-3) / 1e12,
        "seqlen_lo": kernel.workload.seqlen_lo,
        "seqlen_hi": kernel.workload.seqlen_hi,
        "seed": args.seed,
        "page_perm": args.page_perm,
        "cuda_graph": args.cuda_graph,
        "kv_layout": args.kv_layout,
        "kv_scale_range": args.kv_scale_range,
    }
    if args.ncu:
        from . import ncu_harness
        # -k selects the split-KV kernel: one launch per run, plus the one
        # run that records the CUDA graph
        result["ncu"] = ncu_harness.capture(_child_argv(argv, False), "gqa",
                                            skip=args.warmup_steps + (1 if args.cuda_graph else 0),
                                            count=min(3, args.repeat), algorithmic_bytes=alg)
    args.output.parent.mkdir(parents=True, exist_ok=True)
    args.output.write_text(json.dumps(result, indent=2) + "\n", encoding="utf-8")
    print(json.dumps(result))
    return 0


def _mg_worker(rank: int, world: int, port: int, args, shape: DecodeShape, q):
    """One rank of a sharded decodebench run: build the whole batch (same
    seed on every rank), keep this rank's shard, time its decode (plus the
    head all-gather under TP) with one CUDA-event pair per run, and send the
    p50 and the shard's bytes to rank 0."""
    import datetime as _dt
    import torch.distributed as dist
    from . import shard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=_dt.timedelta(seconds=120))
    try:
        k = B2DDecodeKernel(shape, args.seqlen_lo, args.seqlen_hi, args.page_perm, args.seed,
                            kv_scale_range=(tuple(args.kv_scale_range) if args.kv_scale_range
                                            else None))
        x, w = k.x, k.workload
        if args.shard == "dp":
            rows = shard.balance_sequences(x["cache_seqlens"].tolist(), world)[rank]
            y = shard.slice_gqa_inputs_by_batch(x, rows, seed=args.seed + rank)
            wl = w.scaled(batch=len(rows))
            hg = None
        else:
            y = shard.slice_gqa_inputs_by_heads(x, world, rank)
            wl = w.scaled(num_q_heads=w.num_q_heads // world, num_kv_heads=w.num_kv_heads // world)
            hg = shard.HeadGather(w.batch, wl.num_q_heads, w.head_dim, x["q"].dtype, dev)
        del k, x
        dec = api.GqaDecoder(y["q"], y["k_cache"], y["v_cache"], y["cache_seqlens"],
                             y["block_table"], y["softmax_scale"], k_scale=y["k_scale"],
                             v_scale=y["v_scale"], out=None if hg is None else hg.out_local,
                             lse=None if hg is None else hg.lse_local)

        def step():
            dec.run()
            if hg is not None:
                hg.gather()

        for _ in range(args.warmup_steps):
            step()
        torch.cuda.synchronize()
        dist.barrier()
        times = cuda_time_ms(step, args.repeat)
        sl = y["cache_seqlens"].cpu()
        mine = {"rank": rank, "p50_ms": percentile(times, 50), "p95_ms": percentile(times, 95),
                "kv_bytes": W.gqa_kv_bytes_reference(wl, sl),
                "alg_bytes": W.gqa_algorithmic_bytes(wl, sl), "sequences": int(sl.numel()),
                "tokens": int(sl.sum())}
        allr = [None] * world
        dist.all_gather_object(allr, mine)
        if rank == 0:
            q.put(allr)
    finally:
        dist.destroy_process_group()


def main_multi_gpu(args, shape: DecodeShape) -> int:
    """--num-gpus N: one process per GPU (NCCL), batch- or head-sharded; the
    record's latency is the slowest rank's p50 and its bandwidth is all
    ranks' bytes over that latency."""
    import socket
    import torch.multiprocessing as mp
    world = args.num_gpus
    if torch.cuda.device_count() < world:
        raise RuntimeError(f"--num-gpus {world} needs {world} GPUs, found {torch.cuda.device_count()}")
    if args.shard == "tp" and shape.num_kv_heads % world:
        raise ValueError("--shard tp needs num_kv_heads divisible by --num-gpus")
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_mg_worker, args=(r, world, port, args, shape, q))
             for r in range(world)]
    for p in procs:
        p.start()
    ranks = q.get(timeout=900)
    for p in procs:
        p.join(120)
    worst = max(ranks, key=lambda r: r["p50_ms"])
    kv = sum(r["kv_bytes"] for r in ranks)
    alg = sum(r["alg_bytes"] for r in ranks)
    result = {
        "run_id": os.environ.get("DECODEBENCH_RUN_ID"),
        "timestamp": datetime.now(timezone.utc).isoformat(),
        "gpu": torch.cuda.get_device_name(),
        "backend": "b2d_decode",
        "kernel_path": f"b2d gqa_mma_kernel (sm_100a) via libb2d.so, {args.shard}{world}",
        "layer": "kernel",
        "workload_id": os.environ.get("DECODEBENCH_WORKLOAD_ID"),
        "attention": shape.attention,
        "kv_dtype": shape.kv_dtype,
        "page_size": shape.page_size,
        "batch_size": shape.batch_size,
        "context_len": shape.context_len,
        "decode_steps": 1,
        "num_gpus": world,
        "shard": args.shard,
        "compare_latency_us": worst["p50_ms"] * 1000.0,
        "kernel_latency_p50_us": worst["p50_ms"] * 1000.0,
        "kernel_latency_p95_us": max(r["p95_ms"] for r in ranks) * 1000.0,
        "approx_kv_bytes_read": kv,
        "approx_effective_kv_bandwidth_gb_s": kv / (worst["p50_ms"] * 1e6),
        "fallback": False,
        "fallback_reason": None,
        "notes": ("one process per GPU over NCCL; latency = slowest rank's p50"
                  + ("; TP step includes the packed out/lse all-gather" if args.shard == "tp" else "")),
        "roofline_bytes": alg,
        "achieved_tb_s": alg / (worst["p50_ms"] * 1e-3) / 1e12,
        "per_rank": ranks,
        "seqlen_lo": args.seqlen_lo,
        "seqlen_hi": args.seqlen_hi,
        "seed": args.seed,
        "page_perm": args.page_perm,
    }
    args.output.parent.mkdir(parents=True, exist_ok=True)
    args.output.write_text(json.dumps(result, indent=2) + "\n", encoding="utf-8")
    print(json.dumps(result))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
