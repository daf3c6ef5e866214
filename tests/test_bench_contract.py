"""The JSON line `bench.py` prints: the keys and relations every arm must carry.

The reference arm runs on the host cores (the reference's own `sample_token`,
compiled from its sources), so it is checked on the CPU; the CUDA arm is checked
through the lines kept under `profiles/` here, and on a short run on the GPU in
`test_z_full_size_gpu.py`.
"""
import json
import math
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

COMMON = ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
          "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config", "e2e")


def last_json_line(text: str) -> dict:
    lines = [l for l in text.splitlines() if l.startswith("{")]
    assert lines, f"no JSON line in the output:\n{text[-2000:]}"
    return json.loads(lines[-1])


def check_common(d: dict) -> None:
    for k in COMMON:
        assert k in d, k
    assert d["value"] > 0 and math.isfinite(d["value"])
    assert d["unit"] == "codes/s"
    assert d["higher_is_better"] is True
    assert d["scaling"] == "weak"
    assert d["warmup"] >= 3
    assert d["vs_baseline"] is None
    assert d["data"] == "synthetic"
    assert isinstance(d["config"], dict) and d["config"].get("workload")
    e = d["e2e"]
    for k in ("value", "unit", "h2d_bytes_per_step", "d2h_bytes_per_step"):
        assert k in e, k
    assert e["unit"] == d["unit"] and e["value"] > 0


def check_ours(d: dict) -> None:
    check_common(d)
    assert "impl" not in d or d["impl"] == "ours"
    r = d["roofline"]
    for k in ("bound", "achieved", "peak", "unit", "frac", "traffic"):
        assert k in r, k
    assert r["bound"] == "hbm" and r["unit"] == "GB/s"
    assert r["frac"] == pytest.approx(r["achieved"] / r["peak"], rel=1e-9)
    # achieved = algorithmic bytes of one launch / the launch's mean time
    assert r["achieved"] == pytest.approx(
        r["bytes_per_launch"] / (r["kernel_ms"] / 1e3) / 1e9, rel=1e-9)
    # value = rows of every rank / the timed steps' time
    rows = d["config"]["streams_per_gpu"] * d["config"]["codebooks"] * d["n_gpus"]
    assert d["value"] == pytest.approx(rows / (d["ms_per_step"] / 1e3), rel=1e-6)
    # the host copies are counted from the logits and the codes of a step
    per_gpu = d["config"]["streams_per_gpu"] * d["config"]["codebooks"]
    assert d["e2e"]["h2d_bytes_per_step"] == 4 * per_gpu * d["config"]["vocab"]
    assert d["e2e"]["d2h_bytes_per_step"] > 0
    assert d["gpu_launches"] >= d["steps"]
    c = d["clocks"]
    assert c is not None and {"sm_mhz", "sm_max_mhz", "reasons"} <= set(c)
    cpu = d["cpu_baseline"]
    if cpu is not None:
        assert {"value", "unit", "cores", "kind", "sample"} <= set(cpu)
        assert cpu["kind"] in ("reference", "port")


def check_reference(d: dict) -> None:
    check_common(d)
    assert d["impl"] == "reference"
    cpu = d["cpu_baseline"]
    assert {"value", "unit", "cores", "kind", "sample"} <= set(cpu)
    assert cpu["kind"] in ("reference", "port") and cpu["cores"] >= 1
    assert cpu["value"] == d["value"]
    assert d["e2e"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0


@pytest.mark.parametrize("name", ["bench_line_1gpu.json", "bench_line_2gpu.json",
                                  "bench_line_8gpu.json"])
def test_kept_lines_keep_the_contract(name):
    path = os.path.join(REPO, "profiles", name)
    with open(path) as f:
        d = json.loads(f.read().strip().splitlines()[-1])
    check_ours(d)
    if d["n_gpus"] == 1:
        assert d["cpu_baseline"] is not None and d["cpu_baseline"]["value"] > 0


def test_reference_arm_line():
    """One full step of the reference arm (about 10 s on 8 host threads)."""
    p = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1",
                        "--warmup", "0"], cwd=REPO, capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr[-2000:]
    d = last_json_line(p.stdout)
    if "unavailable" in d:
        pytest.skip(d["unavailable"])
    check_reference(d)
    assert d["steps"] == 1 and d["n_gpus"] == 1
