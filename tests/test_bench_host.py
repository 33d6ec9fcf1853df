"""Host-side pieces of bench.py that need no GPU: the clock sampler against a
stand-in NVML module (read-only queries; it sets nothing on any GPU), the
roofline's algorithmic byte counts and committed traffic, and the reference
arm's JSON line."""
import os
import sys
import time
import types

import bench


def test_clock_sampler_reports_median_max_and_reasons(monkeypatch):
    clocks = iter([1900.0, 1905.0, 1910.0] + [1905.0] * 10000)
    fake = types.SimpleNamespace(
        NVML_CLOCK_SM=0,
        nvmlInit=lambda: None,
        nvmlDeviceGetHandleByIndex=lambda i: ("gpu", i),
        nvmlDeviceGetMaxClockInfo=lambda h, c: 1965,
        nvmlDeviceGetClockInfo=lambda h, c: next(clocks),
        # sw_power_cap | hw_slowdown, plus a bit the sampler does not name
        nvmlDeviceGetCurrentClocksEventReasons=lambda h: 0x4 | 0x8 | 0x1,
    )
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    with bench.Clocks(0, period_s=0.001) as c:
        time.sleep(0.02)
    s = c.summary()
    assert s["sm_max_mhz"] == 1965.0
    assert s["samples"] >= 1 and 1900.0 <= s["sm_mhz"] <= 1910.0
    assert s["reasons"] == ["hw_slowdown", "sw_power_cap"]


def test_clock_sampler_without_nvml(monkeypatch):
    """No NVML: the bench still runs and reports no clock samples."""
    monkeypatch.setitem(sys.modules, "pynvml", None)  # import raises ImportError
    with bench.Clocks(0) as c:
        pass
    s = c.summary()
    assert s["samples"] == 0 and s["sm_mhz"] is None and s["reasons"] == []


def test_gpt2_step_bytes_is_the_algorithmic_count():
    """The roofline numerator: every GPT-2 Small weight once (per layer
    q|k|v, attention output and fc as Q4_K, fc2 as Q6_K: 4,589,568 B; the
    Q6_K lm_head: 31,661,910 B), the fp32 norms and biases, one embedding
    row, and 73,728 B of fp32 K/V rows per cached position."""
    D, F, L = 768, 3072, 12
    vectors = L * 4 * (2 * D + 3 * D + D + F + D + 2 * D) + 4 * 2 * D  # ln1/ln2, biases; ln_f
    embed_row = 3 * 210 + 4 * D  # three Q6_K blocks of wte, one fp32 row of wpe
    assert bench.gpt2_step_bytes(0) == L * 4_589_568 + 31_661_910 + vectors + embed_row
    assert bench.gpt2_step_bytes(101) - bench.gpt2_step_bytes(100) == 2 * L * D * 4 == 73_728


def test_committed_step_traffic_is_one_read_of_the_algorithmic_bytes():
    """The ncu DRAM bytes of the step kernel in profiles/ over the
    algorithmic bytes at the capture's context: every byte read about once
    (no re-reads, nothing skipped)."""
    tr = bench.step_traffic("k_step")
    assert tr is not None and "ctx" in tr
    ratio = tr["bytes"] / bench.gpt2_step_bytes(tr["ctx"])
    assert 1.0 <= ratio < 1.03, ratio


def _run_bench(args, env_extra, tmp_path):
    import json
    import os
    import subprocess
    env = dict(os.environ, LMC_BENCH_CACHE=str(tmp_path), **env_extra)
    r = subprocess.run([sys.executable, os.path.join(bench.ROOT, "bench.py")] + args, env=env, cwd=bench.ROOT,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    return [json.loads(ln) for ln in lines]


def test_reference_arm_prints_the_contract_line(tmp_path):
    """`bench.py --impl reference` times LMc's own model_forward (compiled
    from its sources) on the host cores for the GPU arm's metric and
    workload, and prints one JSON line with the reference arm's keys; under
    torchrun the ranks other than 0 print nothing and exit 0."""
    import pytest
    from oracle import ref_library_path
    if not os.path.exists(ref_library_path()):
        pytest.skip("LMc reference build (oracle/_ref) not present")
    (line,) = _run_bench(["--impl", "reference", "--steps", "8", "--warmup", "0"], {}, tmp_path)
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == bench.UNIT and line["higher_is_better"] is True
    assert line["config"]["workload"] == bench.WORKLOAD
    assert line["value"] > 0 and line["warmup"] >= 3 and line["n_gpus"] == 1
    cb = line["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == line["value"] and cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": bench.UNIT, "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert _run_bench(["--impl", "reference", "--gpus", "2"], {"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"},
                      tmp_path) == []


def test_cpu_reference_times_a_llama_prompt(tmp_path):
    """The model workloads' CPU baseline: LMc's model_forward on a LLaMA
    file with the caller's prompt ids (not the GPT-2 prompt)."""
    import pytest
    from oracle import ref_library_path
    from lmc_b200 import synth
    if not os.path.exists(ref_library_path()):
        pytest.skip("LMc reference build (oracle/_ref) not present")
    path = synth.cached_model("llama", str(tmp_path), L=1, D=96, H=6, Hkv=3, F=192, S=16, V=64, seed=1)
    rate, feed, threads, sample = bench.cpu_reference(path, 2, reps=1, prompt=[1, 2, 63])
    assert rate > 0 and feed > 0 and threads >= 1
    assert "3-token prompt then 2 greedy decode tokens" in sample


def test_cpu_matmul_times_every_sweep_format():
    """The gemv / sweep lines' LMc column: matmul_vec on the dequantized
    weights of any format, including rows that start inside a block."""
    import pytest
    from oracle import ref_library_path
    from lmc_b200 import synth
    if not os.path.exists(ref_library_path()):
        pytest.skip("LMc reference build (oracle/_ref) not present")
    names = {v: k for k, v in synth.NAMES.items()}
    for tn in bench.SWEEP_TYPES:
        s = bench.cpu_matmul(names[tn], 64, 1600, reps=4)  # K = 1600: blocks straddle rows
        assert 0 < s < 1.0, (tn, s)
