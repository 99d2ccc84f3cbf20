"""The reference arm of bench.py keeps the one-JSON-line contract the
round-end runner reads; it needs no GPU.  With the reference installed in
baseline/_ref the arm runs the reference's own LazyMoE.forward (kind
"reference"), else the oracle restatement (kind "port")."""

import json
import subprocess
import sys

import pytest

from conftest import REPO


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "0", "--tokens", "4"], capture_output=True, text=True, timeout=600, cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["cpu_baseline"]["kind"] in ("reference", "port") and d["cpu_baseline"]["cores"] >= 1
    if d["cpu_baseline"]["kind"] == "reference":
        assert d["config"]["same_config"] is True and d["cpu_baseline"]["err_vs_oracle_rms"] <= 2e-2
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["unit"] == d["unit"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["config"]["workload"] == "decode_moe_layer"


def test_reference_layer_is_the_oracle_layer():
    """The reference arm's layer (the reference's LazyMoE with the CPU Gate /
    Expert stand-ins, experts materialized by its packed store and compiled
    loader) computes the oracle's layer: bf16 products in fp32 against the
    oracle's float64 sums, here on the small configuration."""
    from oracle import reference_runtime as R
    from spark_b200.synthetic import CONFIGS, make_layer

    try:
        R.import_reference()
    except RuntimeError as exc:
        pytest.skip(str(exc))
    layer = make_layer(CONFIGS["cpu_ref"], seed=0, device="cpu")
    ref = R.ReferenceLayer(layer)
    try:
        assert R.layer_matches_oracle(ref, layer, tokens=4) <= 2e-2
        assert ref.cache.snapshot()["packed_loads"] > 0  # experts came through the reference's packed store
    finally:
        ref.close()
