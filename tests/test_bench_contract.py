"""bench.py's one-line JSON contract: the keys the round-end driver reads, for the
reference arm (host cores, runs here) and for this repository's arm (GPU)."""
import json
import subprocess
import sys

import pytest

from conftest import REPO

BASE_KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
             "scaling", "vs_baseline", "dtype", "data", "config"}


def _run_bench(args, timeout):
    r = subprocess.run([sys.executable, "bench.py", *args], cwd=REPO, capture_output=True, text=True, timeout=timeout)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, r.stdout[-2000:]  # exactly one JSON line on stdout
    return json.loads(lines[0])


def test_profile_traffic_lines():
    import bench

    for key in ("flash_bwd:c3", "flash_fwd:c3"):
        t = bench.profile_traffic(key)
        assert t is not None and t > 1e8, key


def test_reference_arm_json_contract():
    d = _run_bench(["--impl", "reference", "--steps", "1", "--warmup", "1"], timeout=600)
    assert BASE_KEYS <= set(d), BASE_KEYS - set(d)
    assert d["impl"] == "reference"
    assert d["config"]["workload"].startswith("c3")
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


@pytest.mark.gpu
def test_bench_json_contract_gpu():
    d = _run_bench(["--steps", "3", "--warmup", "3", "--no-lm", "--no-cpu", "--lm-steps", "1"], timeout=900)
    assert BASE_KEYS <= set(d), BASE_KEYS - set(d)
    assert d["config"]["kernel_path"] == "sm100" and d["value"] > 0
    rf = d["roofline"]
    assert rf["bound"] in ("hbm", "tensor") and rf["peak"] > 0 and 0 < rf["frac"] == pytest.approx(rf["achieved"] / rf["peak"], rel=1e-2)
    e2e = d["e2e"]
    assert e2e["h2d_bytes_per_step"] == 4 * 8 * 8 * 4096 * 64 * 2 and e2e["d2h_bytes_per_step"] == 4 * 8 * 8 * 4096 * 64 * 2 + 4
    # the host link's own floor: the step's copies alone, and the e2e step no faster than them
    hl = e2e["host_link"]
    assert hl["h2d_gbs"] > 0 and hl["d2h_gbs"] > 0 and hl["both_ms"] > 0
    assert hl["frac"] == pytest.approx(hl["both_ms"] / e2e["ms_per_step"], rel=1e-2) and hl["frac"] < 1.2
    assert d["gpu_launches"] > 0 and "sm_mhz" in d["clocks"] and "reasons" in d["clocks"]
    assert d["fir"]["c5_k_8x16384x2048"]["GB/s"] > 0 and d["fir"]["lm_k_32x512x256"]["device_GB/s"] > 0
    lk = d["lm_kernels"]
    for k in ("head_xent", "add_layernorm_fwd", "add_layernorm_bwd", "gelu_bwd_colsum", "gelu_fwd"):
        assert lk[k]["us"] > 0 and 0 < lk[k]["frac_of_hbm"] < 1.2, (k, lk[k])
    assert rf["traffic"] > 1e8 and "profiles/" in rf["traffic_source"]
    # config 3's tau sweep: silence only at +0.5, where about half the causal tiles skip
    sw = d["tau_sweep"]
    assert set(sw) >= {"-0.5", "+0.0", "+0.5"}
    assert sw["-0.5"]["tiles_silent_frac"] == 0.0 and 0.3 < sw["+0.5"]["tiles_silent_frac"] < 0.7
    assert sw["+0.5"]["ms_per_step"] < sw["+0.0"]["ms_per_step"]
    assert d["deterministic"]["value"] > 0
    c5 = d["c5"]
    assert c5["heads_per_rank"] == 128 and c5["value"] > 0 and c5["roofline"]["frac"] > 0


@pytest.mark.gpu
def test_bench_lm_section_gpu():
    """Config 4's LM step in the bench line: the graph-captured step (headline)
    and the eager one, same losses from the same weights and batches."""
    d = _run_bench(["--steps", "3", "--warmup", "3", "--no-e2e", "--no-fir", "--no-sweep", "--no-c5", "--no-cpu",
                    "--no-triton", "--no-lm-kernels", "--lm-steps", "2"], timeout=900)
    lm = d["lm"]
    assert lm["tokens_per_s"] > 0 and lm["tokens_per_s_eager"] > 0 and lm["params"] == 13383174
    assert lm["global_batch"] == 32 and lm["seq_len"] == 512
    assert abs(lm["loss"] - lm["loss_eager"]) < 1e-2 * abs(lm["loss_eager"])


@pytest.mark.gpu
def test_reference_arm_times_reference_triton_on_gpu():
    """On a GPU the reference arm also times the reference's own Triton Flash kernels
    (staged unchanged in oracle/_ref) at the config-3 tau sweep."""
    from oracle import stage_ref

    if stage_ref.staged() is None:
        pytest.skip("the reference package was not staged into oracle/_ref (no reference checkout at build time)")
    d = _run_bench(["--impl", "reference", "--steps", "2", "--warmup", "1"], timeout=900)
    t = d["triton_b200"]
    assert "unavailable" not in t, t
    for k in ("+0.0", "-0.5", "+0.5"):
        assert t[k]["value"] > 0 and t[k]["ms_per_step"] > 0
