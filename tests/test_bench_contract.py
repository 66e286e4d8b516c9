"""bench.py's reference arm runs on host cores alone, so its JSON-line
contract can be checked without a GPU (the GPU arm's line is checked by the
GPU runs)."""
import json
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference",
                        "--workload", "cfg1", "--steps", "2", "--warmup", "1"],
                       capture_output=True, text=True, timeout=600, cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "TB/s" and d["value"] > 0
    assert d["higher_is_better"] is True and d["steps"] == 2 and d["warmup"] >= 3
    assert d["config"]["workload"].startswith("cfg1")
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == d["value"]
    e = d["e2e"]
    assert e["value"] == d["value"] and e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0


def test_roofline_traffic_comes_from_committed_ncu_records():
    """`roofline.traffic` is the captured case's DRAM / algorithmic ratio
    (profiles/traffic.json, from decodebench --ncu) scaled to the launch."""
    sys.path.insert(0, str(REPO))
    import importlib
    bench = importlib.import_module("bench")
    rec = json.loads((REPO / "profiles" / "traffic.json").read_text())
    for wl in ("cfg5_fp8_b256_p16", "cfg4_mla_b128_p64", "cfg2_gqa_paged_b64_p16"):
        traffic, tensor_pct, src = bench.committed_traffic(wl, 10 ** 9)
        assert traffic == int(rec[wl]["traffic_ratio"] * 10 ** 9)
        assert 1.0 <= rec[wl]["traffic_ratio"] < 1.05 and src
    assert bench.committed_traffic("no_such_workload", 1) == (None, None, None)
