"""Roofline counters from Nsight Compute, merged into a decodebench record.

The reference wraps a benchmark run in `ncu --csv --page raw` and merges the
counters it parses into its JSON result (decodebench/run_matrix.py:372-411,
ncu_utils.py:9-30,94-188, profile_ncu.py:47-128).  This module does the same
for this library's kernels: it re-runs the adapter command once under ncu,
on one kernel (-k), after the warm-up launches (-s), for a few launches (-c),
with the clocks left alone (--clock-control none), and reports per launch:

* gpu_time_us          gpu__time_duration.sum
* dram_bytes           dram__bytes_read.sum + dram__bytes_write.sum
* traffic_ratio        dram_bytes / the launch's algorithmic bytes (1.0 means
                       every byte moved once; more means re-reads)
* tensor_pipe_pct      sm__pipe_tensor_cycles_active, % of peak over the launch
* dram_throughput_pct  gpu__dram_throughput, % of peak

Counters from a replayed launch are cold-cache and serialised: use them for
traffic and utilisation, not as the timing (the adapter's CUDA-event p50 is
the timing).  Keep the captured case small (a few GB of device memory at
most): ncu replays the launch once per counter pass.
"""
from __future__ import annotations

import csv
import io
import os
import shutil
import subprocess
import sys
from typing import Dict, List, Optional

METRICS = [
    "gpu__time_duration.sum",
    "dram__bytes_read.sum",
    "dram__bytes_write.sum",
    "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed",
    "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed",
]

# Kernel-name patterns of this library's split-KV kernels.
KERNEL_REGEX = {"gqa": "regex:gqa_(mma|decode)_kernel", "mla": "regex:mla_decode_kernel"}


def ncu_path() -> Optional[str]:
    for p in (shutil.which("ncu"), "/usr/local/cuda/bin/ncu"):
        if p and os.path.exists(p):
            return p
    return None


def parse_raw_csv(text: str) -> List[Dict[str, str]]:
    """Rows of `ncu --csv --page raw` output (one per captured launch); the
    line after the header carries units and is skipped."""
    lines = [l for l in text.splitlines() if l.startswith('"')]
    if len(lines) < 2:
        return []
    reader = csv.reader(io.StringIO("\n".join(lines)))
    header = next(reader)
    rows = []
    for i, row in enumerate(reader):
        if i == 0 and row and row[0] == "":
            continue   # units line
        rows.append(dict(zip(header, row)))
    return rows


def _num(v: str) -> float:
    try:
        return float(v.replace(",", ""))
    except (AttributeError, ValueError):
        return float("nan")


def summarise(rows: List[Dict[str, str]], algorithmic_bytes: int) -> Dict:
    """Per-launch averages of the captured launches."""
    if not rows:
        return {"error": "no launch captured"}
    n = len(rows)
    avg = lambda k: sum(_num(r.get(k, "nan")) for r in rows) / n
    t_ns = avg("gpu__time_duration.sum")
    dram = avg("dram__bytes_read.sum") + avg("dram__bytes_write.sum")
    return {
        "kernel": rows[0].get("Kernel Name", ""),
        "launches": n,
        "gpu_time_us": t_ns / 1e3,
        "dram_bytes": dram,
        "algorithmic_bytes": algorithmic_bytes,
        "traffic_ratio": dram / algorithmic_bytes if algorithmic_bytes else None,
        "tensor_pipe_pct": avg("sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed"),
        "dram_throughput_pct": avg("gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed"),
    }


def capture(child_argv: List[str], kind: str, skip: int, count: int = 3,
            algorithmic_bytes: int = 0) -> Dict:
    """Run `python -m b200decode.decodebench <child_argv>` under ncu and
    summarise the captured launches of this library's split-KV kernel.  The
    capture is given no time limit: an ncu killed in mid-capture can leave the
    GPU unusable, so the case must be small enough to end by itself."""
    ncu = ncu_path()
    if ncu is None:
        return {"error": "ncu not found"}
    import tempfile
    with tempfile.TemporaryDirectory() as td:
        log = os.path.join(td, "ncu.csv")
        cmd = [ncu, "--clock-control", "none", "-k", KERNEL_REGEX[kind], "-s", str(skip),
               "-c", str(count), "--metrics", ",".join(METRICS), "--csv", "--page", "raw",
               "--log-file", log, sys.executable, "-m", "b200decode.decodebench", *child_argv]
        pkg_root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        env = dict(os.environ)
        env["PYTHONPATH"] = pkg_root + (os.pathsep + env["PYTHONPATH"] if env.get("PYTHONPATH") else "")
        res = subprocess.run(cmd, capture_output=True, text=True, env=env)
        text = open(log).read() if os.path.exists(log) else ""
    out = summarise(parse_raw_csv(text), algorithmic_bytes)
    out["command"] = " ".join(cmd[:-len(child_argv) - 3] + ["python -m b200decode.decodebench"]
                              + child_argv)
    if res.returncode != 0:
        out["error"] = f"ncu exited {res.returncode}: {res.stderr.strip().splitlines()[-1:]}"
    return out
