"""The benchmark's JSON-line contract for the reference arm, which runs on the
host cores alone: one line with the metric, value, unit, the CPU baseline's
description and an e2e block; configs without a CPU counterpart print an
``unavailable`` line and exit 0."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _run(*args):
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True,
                         timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    return json.loads(lines[0])


def test_reference_arm_prints_one_contract_line():
    line = _run("--impl", "reference", "--config", "c2", "--steps", "3", "--warmup", "3")
    assert line["impl"] == "reference"
    if "unavailable" in line:  # the reference runtime is not built here
        return
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["value"] > 0 and line["unit"] == "images/s" and line["higher_is_better"] is True
    cpu = line["cpu_baseline"]
    assert cpu["kind"] == "reference" and cpu["cores"] >= 1 and cpu["value"] == line["value"] and cpu["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_latency_config_has_no_cpu_arm():
    line = _run("--impl", "reference", "--config", "latency")
    assert line["impl"] == "reference" and line["unavailable"]


def test_rank_to_gpu_map_alternates_host_bridge_halves():
    import importlib.util

    spec = importlib.util.spec_from_file_location("bench_mod", ROOT / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    halves = [bench.device_map("halves", r, 4, 8) for r in range(4)]
    assert halves == [0, 4, 1, 5]
    assert [bench.device_map("halves", r, 2, 8) for r in range(2)] == [0, 4]
    assert [bench.device_map("halves", r, 8, 8) for r in range(8)] == list(range(8))  # every GPU in use
    assert [bench.device_map("identity", r, 4, 8) for r in range(4)] == [0, 1, 2, 3]
    assert bench.device_map("halves", 0, 1, 1) == 0


def test_job_clock_record_is_the_slowest_gpu_with_every_reason():
    import importlib.util

    spec = importlib.util.spec_from_file_location("bench_mod", ROOT / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    merged = bench._merge_clocks([{"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": []},
                                  {"sm_mhz": 1800.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"]}])
    assert merged["sm_mhz"] == 1800.0 and merged["sm_max_mhz"] == 1965.0
    assert merged["reasons"] == ["sw_power_cap"] and len(merged["per_gpu"]) == 2


def _bench_module():
    import importlib.util

    spec = importlib.util.spec_from_file_location("bench_mod", ROOT / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    return bench


def test_c2_batch_scales_the_case_and_names_the_workload():
    bench = _bench_module()
    base = bench._config_case("c2")
    small = bench._config_case("c2", c2_batch=4)
    assert base["workload"] == "c2_nchw_to_nhwc_pad4_f16" and base["shape"] == [64, 3, 224, 224]
    assert small["workload"] == "c2_nchw_to_nhwc_pad4_f16_batch4" and small["shape"] == [4, 3, 224, 224]
    assert small["src"].shape == (4, 3, 224, 224) and small["unit_per_step"] == 4
    assert small["kernel_bytes"] == 20 * 4 * 224 * 224 and small["dst_bytes"] == 8 * 4 * 224 * 224
    assert base["kernel_bytes"] == 16 * small["kernel_bytes"]


def test_reference_arm_takes_the_c2_batch():
    line = _run("--impl", "reference", "--config", "c2", "--c2-batch", "2", "--steps", "3", "--warmup", "3")
    if "unavailable" in line:
        return
    assert line["config"]["workload"].endswith("_batch2") and line["config"]["shape"][0] == 2


def test_int8_tile_kernel_name_follows_the_library_switch(monkeypatch):
    bench = _bench_module()
    monkeypatch.delenv("SYM_B200_TMA_TALL", raising=False)
    assert bench.int8_tile_kernel() == "k_tma_tall"
    monkeypatch.setenv("SYM_B200_TMA_TALL", "0")
    assert bench.int8_tile_kernel() == "k_tma_tile"
