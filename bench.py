#!/usr/bin/env python
"""Decode-attention benchmark: one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg2]
                    [--shard dp|tp] [--scaling weak|strong] [--impl b2d|reference]

A step is one decode of the workload's whole batch.  The default workload
is BASELINE config 5, the one the metric is quoted on at 1/2/4/8 GPUs: FP8
KV GQA, B=256, Hq=32, Hkv=8, D=128, e4m3 K/V with per-KV-head fp32 scales,
lengths ~ U[2048, 8192], page 16, permuted pages.  Other workloads by flag
(--workload cfg1|cfg2|cfg3|cfg4).  For N > 1 the script runs under
torch.distributed.run, one process per GPU over NCCL:

* --scaling strong --shard dp (default): the one batch is split across
  ranks by a greedy length balance; no collective inside the step.
* --scaling strong --shard tp: KV heads are split across ranks and the
  outputs are all-gathered over NCCL inside the step.
* --scaling weak: every rank decodes its own full batch (seed + rank).

Timing: W warm-up steps, then K steps between CUDA events on the launching
stream, bracketed by barrier + synchronize, max over ranks.  The KV cache of
one step (2.7 GB for config 5, 1.2 GB for config 2) is 10-20x the 126 MB
L2, so no flush is needed between steps at N=1; at N=8 each rank's share
(~335 MB) is still ~2.7x L2.  `value` is achieved HBM TB/s over all ranks (algorithmic
bytes / step time); `roofline` times the split-KV kernel alone.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import platform
import statistics
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "roofline-analysis_b200"))
sys.path.insert(0, str(REPO))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "decode attention µs/step and achieved HBM TB/s (% of roofline) at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b2d", "reference"], default="b2d")
    ap.add_argument("--workload", default="cfg5")
    ap.add_argument("--shard", choices=["dp", "tp"], default="dp")
    ap.add_argument("--scaling", choices=["weak", "strong"], default="strong")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="CPU work budget of the cpu_baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--sustained-s", type=float, default=1.0,
                    help="seconds of the extra sustained loop (power-capped steady state)")
    ap.add_argument("--no-other-workloads", action="store_true",
                    help="skip the short cfg2 / cfg4 lines that an N=1 cfg5 run adds")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the workload's batch (smaller profiling cases)")
    return ap.parse_args()


# --------------------------------------------------------------------------
# environment helpers
# --------------------------------------------------------------------------

def measured_hbm_peak():
    try:
        d = json.loads((REPO / "MEASURED_PEAKS.json").read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def committed_traffic(workload: str, bytes_per_launch: int):
    """(traffic, tensor_pipe_pct, source) of the split-KV kernel from the
    committed ncu records (profiles/traffic.json, written from `decodebench
    --ncu` captures): the captured case's DRAM / algorithmic ratio times this
    launch's algorithmic bytes."""
    try:
        d = json.loads((REPO / "profiles" / "traffic.json").read_text()).get(workload)
    except Exception:
        d = None
    if not d or not d.get("traffic_ratio"):
        return None, None, None
    ratio = d["traffic_ratio"]
    return (int(ratio * bytes_per_launch), d.get("tensor_pipe_pct"),
            f"ncu capture ({d.get('captured', '')}), DRAM/algorithmic {ratio:.4f} scaled to this launch")


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML while running."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4,
        "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
        "display_clock_setting": 0x100,
    }

    def __init__(self, index: int):
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _sample(self):
        try:
            self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
            self.reasons |= self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        except Exception:
            pass

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(0.001)

    def __enter__(self):
        if self.nv is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t is not None:
            self._t.join()

    def summary(self):
        if self.nv is None or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml unavailable"]}
        names = [n for n, bit in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples)}


def dist_setup():
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def other_workloads(args):
    """At N=1, short lines of the other BASELINE GPU configurations (GQA bf16
    config 2 and MLA config 4), each from its own bench.py process, so one
    driver run also times MLA."""
    if args.no_other_workloads or args.workload not in ("cfg5", "cfg5_fp8_b256_p16") or args.batch:
        return None
    import subprocess
    res = {}
    for wl in ("cfg2", "cfg4"):
        cmd = [sys.executable, str(REPO / "bench.py"), "--workload", wl, "--steps", str(args.steps),
               "--warmup", str(max(3, args.warmup)), "--no-cpu-baseline", "--no-e2e",
               "--no-other-workloads", "--sustained-s", "0.2"]
        try:
            out = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
            d = json.loads(out.stdout.strip().splitlines()[-1])
            r = d["roofline"]
            res[wl] = {"workload": d["config"]["workload"], "us_per_step": d["us_per_step"],
                       "value": d["value"], "unit": d["unit"], "roofline_bound": r["bound"],
                       "kernel_achieved": r["achieved"], "frac": r["frac"],
                       "tensor": r.get("tensor"), "sustained_us_per_step": d["sustained"]["us_per_step"],
                       "clocks": d["clocks"]}
        except Exception as e:
            res[wl] = {"error": f"{type(e).__name__}: {e}"[:300]}
    return res


def gather_rows(vals, world: int, device):
    """All ranks' lists of floats, in rank order (host-side, after timing)."""
    if world == 1:
        return [list(vals)]
    t = torch.tensor(vals, dtype=torch.float64, device=device)
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [o.tolist() for o in out]


def reduce_over_ranks(x: float, world: int, device, op) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=op)
    return float(t.item())


# --------------------------------------------------------------------------
# CPU baseline: the reference's SDPA call on host cores
# --------------------------------------------------------------------------

def cpu_sample_inputs(w, x, n_seqs):
    """The first n sequences of the workload as dense CPU tensors (gather not
    timed) -> (q, dense_kv, algorithmic bytes, n)."""
    from oracle.sdpa_cpu import gather_dense
    from b200decode import workloads as W
    n = max(1, min(n_seqs, x["q"].shape[0]))
    sl = x["cache_seqlens"][:n].cpu()
    bt = x["block_table"][:n].cpu()
    page = x["k_cache"].shape[1]
    used = torch.unique(torch.cat([bt[i, : (int(l) + page - 1) // page]
                                   for i, l in enumerate(sl.tolist())]).long())
    kc = torch.zeros(tuple(x["k_cache"].shape), dtype=x["k_cache"].dtype)
    vc = torch.zeros_like(kc)
    kc[used] = x["k_cache"][used.to(x["k_cache"].device)].cpu()
    vc[used] = x["v_cache"][used.to(x["v_cache"].device)].cpu()
    ks = None if x.get("k_scale") is None else x["k_scale"].cpu()
    vs = None if x.get("v_scale") is None else x["v_scale"].cpu()
    dense = gather_dense(kc, vc, sl, bt, ks, vs)
    q = x["q"][:n].cpu()
    return q, dense, W.gqa_algorithmic_bytes(w.scaled(batch=n), sl), n


def time_cpu_sdpa(q, dense, scale, seconds):
    """Median seconds per pass of the SDPA decode over the sample, repeating
    passes for about `seconds` of CPU work (at least 3 passes)."""
    from oracle.sdpa_cpu import sdpa_decode
    torch.set_num_threads(os.cpu_count() or 1)
    sdpa_decode(q, dense, scale)  # warm-up
    times = []
    t_end = time.perf_counter() + seconds
    while len(times) < 3 or time.perf_counter() < t_end:
        t0 = time.perf_counter()
        sdpa_decode(q, dense, scale)
        times.append(time.perf_counter() - t0)
        if len(times) >= 200:
            break
    return statistics.median(times), len(times)


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor()


# --------------------------------------------------------------------------
# main
# --------------------------------------------------------------------------

def main():
    args = parse_args()
    world, rank, local = dist_setup()
    from b200decode import workloads as W

    w0 = W.get(args.workload)
    if args.batch:
        w0 = w0.scaled(batch=args.batch)
    if args.impl == "reference":
        return run_reference_arm(args, world, rank, w0)
    if isinstance(w0, W.MlaWorkload):
        return run_mla(args, world, rank, local, w0)

    import b200decode
    from b200decode import _lib, shard

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    SUM, MAX = dist.ReduceOp.SUM, dist.ReduceOp.MAX

    # ---- inputs ----
    tp = args.scaling == "strong" and args.shard == "tp" and world > 1
    if args.scaling == "weak" or world == 1:
        w = w0.scaled(seed=w0.seed + rank) if world > 1 else w0
        x = W.make_gqa_inputs(w, dev)
        par = f"dp{world}-weak" if world > 1 else "single"
    else:
        xg = W.make_gqa_inputs(w0, dev)
        if args.shard == "dp":
            rows = shard.balance_sequences(xg["cache_seqlens"].tolist(), world)[rank]
            x = shard.slice_gqa_inputs_by_batch(xg, rows, seed=rank)
            w = w0.scaled(batch=len(rows))
        else:
            x = shard.slice_gqa_inputs_by_heads(xg, world, rank)
            w = w0.scaled(num_kv_heads=w0.num_kv_heads // world,
                          num_q_heads=w0.num_q_heads // world)
        del xg
        torch.cuda.empty_cache()
        par = f"{args.shard}{world}"
    sl = x["cache_seqlens"].cpu()
    local_bytes = W.gqa_algorithmic_bytes(w, sl)

    def make_decoder(flags=0, **kw):
        # plan once, run every step (GqaDecoder is decode() with the argument
        # checks hoisted out of the loop)
        return b200decode.GqaDecoder(x["q"], x["k_cache"], x["v_cache"], x["cache_seqlens"],
                                     x["block_table"], x["softmax_scale"], k_scale=x["k_scale"],
                                     v_scale=x["v_scale"], flags=flags, **kw)

    hgather = (shard.HeadGather(w.batch, w.num_q_heads, w.head_dim, x["q"].dtype, dev)
               if tp else None)
    decoder = (make_decoder(out=hgather.out_local, lse=hgather.lse_local) if tp
               else make_decoder())

    def step():
        out, lse = decoder.run()
        if tp:   # one packed all-gather into preallocated buffers
            out, lse = hgather.gather()
        return out, lse

    # launches of our kernels per step, as the library counts them (the
    # split-KV kernel per batch slice, plus a combine kernel when the merge
    # is not done in-kernel)
    n_ctas, chunk, hk_cta = b200decode.gqa_plan(x["q"], x["k_cache"], x["v_cache"],
                                                x["cache_seqlens"], x["block_table"])
    launches_per_step = decoder.launches_per_run()

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    b200decode.check_device_status()

    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with sampler:
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    local_ms = ev0.elapsed_time(ev1) / args.steps
    ms = reduce_over_ranks(local_ms, world, dev, MAX)
    total_bytes = reduce_over_ranks(local_bytes, world, dev, SUM)
    total_flops = reduce_over_ranks(W.gqa_flops(w, sl), world, dev, SUM)
    total_kv_ref = reduce_over_ranks(W.gqa_kv_bytes_reference(w, sl), world, dev, SUM)
    total_tokens = reduce_over_ranks(int(sl.sum()), world, dev, SUM)
    tbs = total_bytes / (ms * 1e-3) / 1e12

    # ---- the split-KV kernel and the combine kernel alone ----
    def timed(flag, n):
        d = make_decoder(flag)
        for _ in range(3):
            d.run()
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(n):
            d.run()
        ev1.record(stream)
        torch.cuda.synchronize()
        return ev0.elapsed_time(ev1) / n

    kk = max(5, args.steps)
    graph_ms = None
    sampler_k = ClockSampler(local)
    sampler_k.__enter__()
    if not tp:
        gdec = make_decoder().capture()
        for _ in range(3):
            gdec.replay()
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(kk):
            gdec.replay()
        ev1.record(stream)
        torch.cuda.synchronize()
        graph_ms = ev0.elapsed_time(ev1) / kk
    kern_ms = timed(_lib.B2D_FLAG_SKIP_COMBINE, kk)
    combine_ms = timed(_lib.B2D_FLAG_COMBINE_ONLY, kk) if launches_per_step > 1 else 0.0
    sampler_k.__exit__()
    peak, peak_kind = measured_hbm_peak()
    # When a step is one launch of the split-KV kernel (merge in-kernel, no
    # collective), the timed region itself times that kernel: its per-step
    # time is the launch duration plus the gap to the next launch.
    roof_from_step = launches_per_step == 1 and not tp
    roof_ms = local_ms if roof_from_step else kern_ms
    achieved_gbs = local_bytes / (roof_ms * 1e-3) / 1e9

    # ---- sustained: the same step for about a second, under the power cap ----
    # sized from the max-over-ranks step time, the same on every rank: under
    # TP each step is a collective, so every rank must run the same count
    sus_steps = max(args.steps, int(math.ceil(args.sustained_s * 1e3 / max(ms, 1e-3))))
    sampler_s = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with sampler_s:
        ev0.record(stream)
        for _ in range(sus_steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
    sus_ms = reduce_over_ranks(ev0.elapsed_time(ev1) / sus_steps, world, dev, MAX)

    # ---- end to end through the public API with host buffers ----
    e2e = None
    if not args.no_e2e:
        # Every step copies its inputs (q, lengths, block table) from pinned
        # host memory and reads out/lse back.  Two input/output buffer sets
        # and a copy stream let step k+1's copies overlap step k's decode.
        qh = x["q"].cpu().pin_memory()
        slh = x["cache_seqlens"].cpu().pin_memory()
        bth = x["block_table"].cpu().pin_memory()
        hq_out = w0.num_q_heads if tp else w.num_q_heads
        sets = []
        for _ in range(2):
            qd, sld, btd = (torch.empty_like(x["q"]), torch.empty_like(x["cache_seqlens"]),
                            torch.empty_like(x["block_table"]))
            hg_j = (shard.HeadGather(w.batch, w.num_q_heads, w.head_dim, x["q"].dtype, dev)
                    if tp else None)
            dec_j = b200decode.GqaDecoder(qd, x["k_cache"], x["v_cache"], sld, btd,
                                          x["softmax_scale"], k_scale=x["k_scale"],
                                          v_scale=x["v_scale"],
                                          out=hg_j.out_local if tp else None,
                                          lse=hg_j.lse_local if tp else None)
            out_h = torch.empty((w.batch, hq_out, w.head_dim), dtype=x["q"].dtype).pin_memory()
            lse_h = torch.empty((w.batch, hq_out), dtype=torch.float32).pin_memory()
            sets.append(dict(q=qd, sl=sld, bt=btd, dec=dec_j, hg=hg_j, out_h=out_h, lse_h=lse_h,
                             ready=torch.cuda.Event(), done=torch.cuda.Event(),
                             free=torch.cuda.Event()))
        h2d_stream, d2h_stream = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

        def e2e_step(k):
            st = sets[k % 2]
            with torch.cuda.stream(h2d_stream):
                h2d_stream.wait_event(st["free"])      # previous use of this set read back
                st["q"].copy_(qh, non_blocking=True)
                st["sl"].copy_(slh, non_blocking=True)
                st["bt"].copy_(bth, non_blocking=True)
                st["ready"].record(h2d_stream)
            stream.wait_event(st["ready"])
            out, lse = st["dec"].run()
            if tp:
                out, lse = st["hg"].gather()
            st["done"].record(stream)
            with torch.cuda.stream(d2h_stream):
                d2h_stream.wait_event(st["done"])
                st["out_h"].copy_(out, non_blocking=True)
                st["lse_h"].copy_(lse, non_blocking=True)
                st["free"].record(d2h_stream)

        for k in range(4):
            e2e_step(k)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ev0.record(stream)
        h2d_stream.wait_event(ev0)
        for k in range(args.steps):
            e2e_step(k)
        tail = torch.cuda.Event()
        tail.record(d2h_stream)
        stream.wait_event(tail)
        ev1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = reduce_over_ranks(ev0.elapsed_time(ev1) / args.steps, world, dev, MAX)
        h2d = qh.numel() * qh.element_size() + slh.numel() * 4 + bth.numel() * 4
        d2h = sets[0]["out_h"].numel() * sets[0]["out_h"].element_size() + sets[0]["lse_h"].numel() * 4
        e2e = {"value": round(total_bytes / (e2e_ms * 1e-3) / 1e12, 4), "unit": "TB/s",
               "us_per_step": round(e2e_ms * 1e3, 2),
               "h2d_bytes_per_step": int(reduce_over_ranks(h2d, world, dev, SUM)),
               "d2h_bytes_per_step": int(reduce_over_ranks(d2h, world, dev, SUM)),
               "overlap": "double-buffered inputs/outputs; H2D and D2H on their own streams"}

    # ---- per-rank numbers (the slowest rank sets the step time) ----
    per_rank = gather_rows([local_ms * 1e3, float(sl.sum()), float(w.batch), kern_ms * 1e3,
                            (graph_ms or 0.0) * 1e3], world, dev)

    # ---- CPU baseline (rank 0, N = 1) ----
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        q_s, dense, sbytes, n = cpu_sample_inputs(w, x, min(4, w.batch))
        sec, reps = time_cpu_sdpa(q_s, dense, x["softmax_scale"], args.cpu_seconds)
        cpu = {"value": round(sbytes / sec / 1e12, 6), "unit": "TB/s",
               "cores": torch.get_num_threads(), "kind": "reference",
               "sample": (f"torch.nn.functional.scaled_dot_product_attention on CPU (the call of "
                          f"decodebench/torch_sdpa_benchmark.py:100-102, enable_gqa) over the "
                          f"first {n} of {w.batch} sequences ({int(sl[:n].sum())} tokens), pages "
                          f"gathered untimed; median of {reps} passes, {sec * 1e3:.1f} ms each; "
                          f"TB/s = the sample's algorithmic bytes / its time"),
               "extrapolated": n < w.batch,
               "cpu_model": cpu_model(), "os_cpu_count": os.cpu_count()}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(tbs, 4), "unit": "TB/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": round(ms, 5),
            "us_per_step": round(ms * 1e3, 2), "higher_is_better": True,
            "scaling": "weak" if (args.scaling == "weak" or world == 1) else "strong",
            "vs_baseline": None,
            "pct_hbm_roofline": round(100 * tbs / (peak * world / 1e3), 2),
            "dtype": "fp8_e4m3" if w0.kv_dtype == "fp8" else w0.kv_dtype,
            "accumulate": "fp32",
            "data": ("synthetic: seeded N(0,1) q/K/V, lengths ~ U[%d,%d], random page permutation"
                     % (w0.seqlen_lo, w0.seqlen_hi)),
            "config": {"workload": w0.name, "batch": w0.batch, "num_q_heads": w0.num_q_heads,
                       "num_kv_heads": w0.num_kv_heads, "head_dim": w0.head_dim,
                       "page_size": w0.page_size, "kv_dtype": w0.kv_dtype, "parallelism": par,
                       "tokens_per_step": int(total_tokens),
                       "algorithmic_bytes_per_step": int(total_bytes),
                       "approx_kv_bytes_read": int(total_kv_ref),
                       "flops_per_step": int(total_flops),
                       "l2": "each step reads >1 GB of KV (> 126 MB L2); no flush between steps",
                       "num_ctas": n_ctas, "chunk_tokens": chunk, "kv_heads_per_cta": hk_cta},
            "roofline": {"bound": "hbm",
                         "kernel": "b2d::gqa_mma_kernel" if w0.page_size % 16 == 0 and not (
                             w0.kv_dtype == "fp8" and w0.head_dim < 128) else "b2d::gqa_decode_kernel",
                         "achieved": round(achieved_gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved_gbs / peak, 4), "peak_source": peak_kind,
                         "timed_from": ("the timed region (one launch per step)" if roof_from_step
                                        else "a loop of the split-KV kernel alone"),
                         "traffic": committed_traffic(w0.name, local_bytes)[0],
                         "traffic_source": committed_traffic(w0.name, local_bytes)[2],
                         "tensor_pipe_pct": committed_traffic(w0.name, local_bytes)[1],
                         "kernel_us": round(kern_ms * 1e3, 2),
                         "combine_us": round(combine_ms * 1e3, 2),
                         "cuda_graph_step_us": None if graph_ms is None else round(graph_ms * 1e3, 2),
                         "bytes_per_launch": int(local_bytes)},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches_per_step * args.steps,
            "launches_per_step": launches_per_step,
            "clocks": sampler.summary(),
            "clocks_kernel_loops": sampler_k.summary(),
            "sustained": {"us_per_step": round(sus_ms * 1e3, 2), "steps": sus_steps,
                          "value": round(total_bytes / (sus_ms * 1e-3) / 1e12, 4), "unit": "TB/s",
                          "clocks": sampler_s.summary(),
                          "note": "the same step repeated for about a second; the power cap "
                                  "(sw_power_cap) lowers SM clocks after ~50-100 ms of FP8 decode"},
            "other_workloads": other_workloads(args) if world == 1 else None,
            "per_rank": [{"rank": r, "us_per_step": round(v[0], 2), "tokens": int(v[1]),
                          "sequences": int(v[2]), "kernel_us": round(v[3], 2),
                          "cuda_graph_step_us": round(v[4], 2) if v[4] else None}
                         for r, v in enumerate(per_rank)],
            "slowest_rank": int(max(range(len(per_rank)), key=lambda r: per_rank[r][0])),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def measured_bf16_peak():
    try:
        d = json.loads((REPO / "MEASURED_PEAKS.json").read_text())
        return float(d["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def mla_cpu_sample(x, n, scale):
    """First n MLA sequences as dense CPU tensors -> (q [n,128,576], [(kv [1,1,L,576])])."""
    sl = x["cache_seqlens"][:n].cpu().tolist()
    bt = x["block_table"][:n].cpu()
    page = x["kv_cache"].shape[1]
    dense = []
    for b, length in enumerate(sl):
        npg = (length + page - 1) // page
        kv = x["kv_cache"][bt[b, :npg].long().to(x["kv_cache"].device)].reshape(-1, 576)[:length]
        dense.append(kv.cpu()[None, None])
    return x["q"][:n].cpu(), dense


def mla_cpu_decode(q, dense, scale):
    import torch.nn.functional as F
    outs = []
    for b, kv in enumerate(dense):
        qb = q[b:b + 1, :, None, :]
        o = F.scaled_dot_product_attention(qb, kv, kv[..., :512], is_causal=False, scale=scale,
                                           enable_gqa=True)
        outs.append(o[:, :, 0])
    return torch.cat(outs)


def run_mla(args, world, rank, local, w0):
    """Absorbed-MLA decode; weak scaling across ranks."""
    import b200decode
    from b200decode import _lib
    from b200decode import workloads as W
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    SUM, MAX = dist.ReduceOp.SUM, dist.ReduceOp.MAX
    w = w0.scaled(seed=w0.seed + rank) if world > 1 else w0
    x = W.make_mla_inputs(w, dev)
    sl = x["cache_seqlens"].cpu()
    local_bytes = W.mla_algorithmic_bytes(w, sl)
    local_flops = W.mla_flops(w, sl)
    out = torch.empty(w.batch, w.num_heads, w.head_dim_v, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(w.batch, w.num_heads, dtype=torch.float32, device=dev)

    def dec(flags=0, q=None, seqlens=None, bt=None):
        return b200decode.decode_mla(x["q"] if q is None else q, x["kv_cache"],
                                     x["cache_seqlens"] if seqlens is None else seqlens,
                                     x["block_table"] if bt is None else bt, x["softmax_scale"],
                                     out=out, lse=lse, flags=flags)

    for _ in range(max(3, args.warmup)):
        dec()
    torch.cuda.synchronize()
    b200decode.check_device_status()
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with sampler:
        ev0.record(stream)
        for _ in range(args.steps):
            dec()
        ev1.record(stream)
        torch.cuda.synchronize()
    ms = reduce_over_ranks(ev0.elapsed_time(ev1) / args.steps, world, dev, MAX)

    def timed(flag):
        for _ in range(3):
            dec(flag)
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(args.steps):
            dec(flag)
        ev1.record(stream)
        torch.cuda.synchronize()
        return ev0.elapsed_time(ev1) / args.steps

    kern_ms = timed(_lib.B2D_FLAG_SKIP_COMBINE)
    combine_ms = timed(_lib.B2D_FLAG_COMBINE_ONLY)
    # sustained: the same step for about a second
    sus_steps = max(args.steps, int(math.ceil(args.sustained_s * 1e3 / max(ms, 1e-3))))
    sampler_s = ClockSampler(local)
    torch.cuda.synchronize()
    with sampler_s:
        ev0.record(stream)
        for _ in range(sus_steps):
            dec()
        ev1.record(stream)
        torch.cuda.synchronize()
    sus_ms = reduce_over_ranks(ev0.elapsed_time(ev1) / sus_steps, world, dev, MAX)
    total_bytes = reduce_over_ranks(local_bytes, world, dev, SUM)
    total_flops = reduce_over_ranks(local_flops, world, dev, SUM)
    hbm_peak, hbm_kind = measured_hbm_peak()
    tc_peak, tc_kind = measured_bf16_peak()
    ach_gbs = local_bytes / (kern_ms * 1e-3) / 1e9
    ach_tfs = local_flops / (kern_ms * 1e-3) / 1e12
    t_hbm = local_bytes / (hbm_peak * 1e9)
    t_tc = local_flops / (tc_peak * 1e12)
    bound = "hbm" if t_hbm >= t_tc else "tensor"

    e2e = None
    if not args.no_e2e:
        # As for GQA: two input/output buffer sets, H2D and D2H copies on
        # their own streams, so step k+1's copies overlap step k's decode.
        qh = x["q"].cpu().pin_memory()
        slh = x["cache_seqlens"].cpu().pin_memory()
        bth = x["block_table"].cpu().pin_memory()
        sets = []
        for _ in range(2):
            sets.append(dict(q=torch.empty_like(x["q"]), sl=torch.empty_like(x["cache_seqlens"]),
                             bt=torch.empty_like(x["block_table"]), out=torch.empty_like(out),
                             lse=torch.empty_like(lse),
                             out_h=torch.empty(out.shape, dtype=out.dtype).pin_memory(),
                             lse_h=torch.empty(lse.shape, dtype=lse.dtype).pin_memory(),
                             ready=torch.cuda.Event(), done=torch.cuda.Event(),
                             free=torch.cuda.Event()))
        h2d_stream, d2h_stream = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        out_h, lse_h = sets[0]["out_h"], sets[0]["lse_h"]

        def e2e_step(k):
            st = sets[k % 2]
            with torch.cuda.stream(h2d_stream):
                h2d_stream.wait_event(st["free"])
                st["q"].copy_(qh, non_blocking=True)
                st["sl"].copy_(slh, non_blocking=True)
                st["bt"].copy_(bth, non_blocking=True)
                st["ready"].record(h2d_stream)
            stream.wait_event(st["ready"])
            b200decode.decode_mla(st["q"], x["kv_cache"], st["sl"], st["bt"], x["softmax_scale"],
                                  out=st["out"], lse=st["lse"])
            st["done"].record(stream)
            with torch.cuda.stream(d2h_stream):
                d2h_stream.wait_event(st["done"])
                st["out_h"].copy_(st["out"], non_blocking=True)
                st["lse_h"].copy_(st["lse"], non_blocking=True)
                st["free"].record(d2h_stream)

        for k in range(4):
            e2e_step(k)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ev0.record(stream)
        h2d_stream.wait_event(ev0)
        for k in range(args.steps):
            e2e_step(k)
        tail = torch.cuda.Event()
        tail.record(d2h_stream)
        stream.wait_event(tail)
        ev1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = reduce_over_ranks(ev0.elapsed_time(ev1) / args.steps, world, dev, MAX)
        h2d = qh.numel() * 2 + slh.numel() * 4 + bth.numel() * 4
        d2h = out_h.numel() * 2 + lse_h.numel() * 4
        e2e = {"value": round(total_bytes / (e2e_ms * 1e-3) / 1e12, 4), "unit": "TB/s",
               "us_per_step": round(e2e_ms * 1e3, 2),
               "h2d_bytes_per_step": int(reduce_over_ranks(h2d, world, dev, SUM)),
               "d2h_bytes_per_step": int(reduce_over_ranks(d2h, world, dev, SUM)),
               "overlap": "double-buffered inputs/outputs; H2D and D2H on their own streams"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        q_s, dense = mla_cpu_sample(x, 1, x["softmax_scale"])
        torch.set_num_threads(os.cpu_count() or 1)
        mla_cpu_decode(q_s, dense, x["softmax_scale"])
        times = []
        t_end = time.perf_counter() + args.cpu_seconds
        while len(times) < 3 or (time.perf_counter() < t_end and len(times) < 200):
            t0 = time.perf_counter()
            mla_cpu_decode(q_s, dense, x["softmax_scale"])
            times.append(time.perf_counter() - t0)
        sec = statistics.median(times)
        sb = W.mla_algorithmic_bytes(w.scaled(batch=1), sl[:1])
        cpu = {"value": round(sb / sec / 1e12, 6), "unit": "TB/s", "cores": torch.get_num_threads(),
               "kind": "reference",
               "sample": (f"torch SDPA on CPU (the decode call of decodebench/torch_sdpa_benchmark.py:"
                          f"100-102 with enable_gqa, one 576-wide latent KV head, V = first 512 "
                          f"columns) over the first of {w.batch} sequences ({int(sl[0])} tokens); "
                          f"median of {len(times)} passes, {sec * 1e3:.1f} ms each"),
               "cpu_model": cpu_model(), "os_cpu_count": os.cpu_count()}

    if rank == 0:
        tbs = total_bytes / (ms * 1e-3) / 1e12
        line = {
            "metric": METRIC, "value": round(tbs, 4), "unit": "TB/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": round(ms, 5),
            "us_per_step": round(ms * 1e3, 2), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None,
            "pct_hbm_roofline": round(100 * tbs / (hbm_peak * world / 1e3), 2),
            "dtype": "bf16",
            "accumulate": "fp32 (tcgen05, TMEM)",
            "data": "synthetic: seeded N(0, 0.5) q and latent cache, lengths ~ U[%d,%d], random page permutation" % (w0.seqlen_lo, w0.seqlen_hi),
            "config": {"workload": w0.name, "batch": w0.batch, "num_heads": w0.num_heads,
                       "head_dim_qk": w0.head_dim_qk, "head_dim_v": w0.head_dim_v,
                       "page_size": w0.page_size, "parallelism": f"dp{world}-weak" if world > 1 else "single",
                       "tokens_per_step": int(reduce_over_ranks(int(sl.sum()), world, dev, SUM)),
                       "algorithmic_bytes_per_step": int(total_bytes), "flops_per_step": int(total_flops),
                       "l2": "each step reads >1 GB of latent cache (> 126 MB L2); no flush"},
            "roofline": {"bound": bound, "kernel": "b2d::mla_decode_kernel",
                         "achieved": round(ach_gbs, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(max(t_hbm, t_tc) / (kern_ms * 1e-3), 4),
                         "peak_source": hbm_kind,
                         "tensor": {"achieved": round(ach_tfs, 1), "peak": tc_peak, "unit": "TFLOP/s",
                                    "frac": round(ach_tfs / tc_peak, 4), "peak_source": tc_kind},
                         "traffic": committed_traffic(w0.name, local_bytes)[0],
                         "traffic_source": committed_traffic(w0.name, local_bytes)[2],
                         "tensor_pipe_pct": committed_traffic(w0.name, local_bytes)[1],
                         "kernel_us": round(kern_ms * 1e3, 2),
                         "combine_us": round(combine_ms * 1e3, 2), "bytes_per_launch": int(local_bytes)},
            "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": 2 * args.steps,
            "clocks": sampler.summary(),
            "sustained": {"us_per_step": round(sus_ms * 1e3, 2), "steps": sus_steps,
                          "value": round(total_bytes / (sus_ms * 1e-3) / 1e12, 4), "unit": "TB/s",
                          "clocks": sampler_s.summary()},
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_reference_arm(args, world, rank, w0):
    """The reference's CPU decode path (torch SDPA on host cores), timed on
    rank 0 only, each step a bounded sample of the same workload."""
    if rank != 0:
        return
    from b200decode import workloads as W
    from oracle.sdpa_cpu import sdpa_decode
    mla = isinstance(w0, W.MlaWorkload)
    torch.set_num_threads(os.cpu_count() or 1)
    seqlens = W.draw_seqlens(w0.batch, w0.seqlen_lo, w0.seqlen_hi, w0.seed)
    budget = max(0.2, 120.0 / (args.steps + max(3, args.warmup)))

    def sample_inputs(n):
        """The first n sequences as dense CPU tensors, the pass that decodes
        them, and their algorithmic bytes."""
        ws = w0.scaled(batch=n)
        if mla:   # one 576-wide latent head, V = its first 512 columns
            xs = W.make_mla_inputs(ws, "cpu", seqlens=seqlens[:n])
            q, dense = mla_cpu_sample(xs, n, xs["softmax_scale"])
            return (lambda: mla_cpu_decode(q, dense, xs["softmax_scale"]),
                    W.mla_algorithmic_bytes(ws, seqlens[:n]))
        xs = W.make_gqa_inputs(ws, "cpu", seqlens=seqlens[:n])
        q, dense, nbytes, _ = cpu_sample_inputs(ws, xs, n)
        return (lambda: sdpa_decode(q, dense, ws.softmax_scale)), nbytes

    n = 1
    while True:   # grow the sample while one pass stays under a quarter of the budget
        run_pass, nbytes = sample_inputs(n)
        t0 = time.perf_counter()
        run_pass()
        dt = time.perf_counter() - t0
        if dt * 4 > budget or n >= w0.batch:
            break
        n = min(w0.batch, n * 2)
    for _ in range(max(3, args.warmup)):
        run_pass()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        run_pass()
        times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    tbs = nbytes / sec / 1e12
    what = ("the absorbed-MLA decode (one 576-wide latent KV head, V = its first 512 columns)"
            if mla else "the decode")
    sample = (f"torch SDPA (decodebench/torch_sdpa_benchmark.py:100-102) on CPU, {what}, over "
              f"{n} of {w0.batch} sequences ({int(seqlens[:n].sum())} tokens) per step, pages "
              f"gathered untimed")
    line = {"impl": "reference", "metric": METRIC, "value": float(f"{tbs:.4g}"), "unit": "TB/s",
            "n_gpus": world, "steps": args.steps, "warmup": max(3, args.warmup),
            "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16" if mla else ("fp8_e4m3" if w0.kv_dtype == "fp8" else w0.kv_dtype),
            "data": "synthetic",
            "config": {"workload": w0.name, "batch": w0.batch, "parallelism": "host cores",
                       "sample_sequences": n},
            "cpu_baseline": {"value": float(f"{tbs:.4g}"), "unit": "TB/s",
                             "cores": torch.get_num_threads(), "kind": "reference",
                             "sample": sample, "cpu_model": cpu_model()},
            "e2e": {"value": float(f"{tbs:.4g}"), "unit": "TB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
