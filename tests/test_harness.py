"""Host-side pieces of the measurement harness (no GPU): the Nsight Compute
CSV parsing and per-launch summary that decodebench --ncu merges into its
record, and the adapter's multi-GPU / ncu flags."""
import pytest

from b200decode import decodebench, ncu_harness

RAW = '''==PROF== Connected to process 1
"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream","Block Size","Grid Size","Device","CC","Section Name","dram__bytes_read.sum","dram__bytes_write.sum","gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed","gpu__time_duration.sum","sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed"
"","","","","","","","","","","","","byte","byte","%","ns","%"
"0","1","python","h","void b2d::gqa_mma_kernel<128>(CUtensorMap_st, CUtensorMap_st, b2d::GqaParams)","1","7","(288, 1, 1)","(148, 1, 1)","0","10.0","","1,000,000","24,000","91.5","200,000","12.5"
"1","1","python","h","void b2d::gqa_mma_kernel<128>(CUtensorMap_st, CUtensorMap_st, b2d::GqaParams)","1","7","(288, 1, 1)","(148, 1, 1)","0","10.0","","1,002,000","26,000","92.5","202,000","13.5"
'''


def test_parse_and_summarise_raw_csv():
    rows = ncu_harness.parse_raw_csv(RAW)
    assert len(rows) == 2
    s = ncu_harness.summarise(rows, algorithmic_bytes=1_000_000)
    assert s["launches"] == 2
    assert s["gpu_time_us"] == pytest.approx(201.0)
    assert s["dram_bytes"] == pytest.approx(1_026_000)
    assert s["traffic_ratio"] == pytest.approx(1.026)
    assert s["tensor_pipe_pct"] == pytest.approx(13.0)
    assert s["dram_throughput_pct"] == pytest.approx(92.0)
    assert "gqa_mma_kernel" in s["kernel"]


def test_summarise_without_launches_reports_it():
    assert "error" in ncu_harness.summarise([], 1)


def test_adapter_flags():
    a = decodebench.parse_args(["--batch-size", "8", "--context-len", "100", "--num-q-heads", "32",
                                "--num-kv-heads", "8", "--head-dim", "128", "--kv-dtype", "fp8",
                                "--page-size", "16", "--output", "x.json", "--num-gpus", "4",
                                "--shard", "tp", "--ncu"])
    assert (a.num_gpus, a.shard, a.ncu) == (4, "tp", True)
    assert decodebench._child_argv(["--a", "--ncu", "--b"], False) == ["--a", "--b"]
    assert decodebench._child_argv(["--a", "--ncu"], True) == ["mla", "--a"]
    m = decodebench.parse_mla_args(["--batch-size", "2", "--context-len", "64", "--num-q-heads",
                                    "128", "--kv-dtype", "bf16", "--output", "m.json", "--ncu"])
    assert m.ncu
