"""The reference arm of bench.py on the host (no GPU): its JSON line carries
the contract's keys, from glm.c's own code (oracle/_ref) when that was built,
else from the oracle's C restatement with kind "port"."""
import argparse
import contextlib
import io
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _check_line(line: dict, kind: str) -> None:
    assert line["impl"] == "reference"
    assert line["unit"] == "GB/s" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["cpu_baseline"]["value"] == line["value"]
    assert line["cpu_baseline"]["kind"] == kind and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    import bench

    # the repo arm's exact workload dict (here with the small test stack)
    assert line["config"] == bench.workload_config(1, 2)


def test_reference_arm_json_line():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    if not oracle.ref_available():
        pytest.skip("oracle/_ref not built here")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "3", "--layers", "2"], capture_output=True, text=True, timeout=600,
                       cwd=ROOT, env=dict(os.environ, OMP_NUM_THREADS="2"))
    assert r.returncode == 0, r.stderr[-2000:]
    _check_line(json.loads(r.stdout.strip().splitlines()[-1]), "reference")


def test_reference_arm_falls_back_to_the_oracle_port(monkeypatch):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import bench
    import oracle

    monkeypatch.setattr(oracle, "ref_available", lambda: False)
    out = io.StringIO()
    with contextlib.redirect_stdout(out):
        bench.run_reference(argparse.Namespace(steps=1, warmup=3, layers=2, seed=42))
    line = json.loads(out.getvalue().strip().splitlines()[-1])
    _check_line(line, "port")
    assert line["cpu_baseline"]["cores"] == 1 and line["kind"] == "port" and "note" in line


def test_cpu_baseline_port_fallback(monkeypatch):
    """The bench's cpu_baseline object without oracle/_ref: the oracle port,
    one thread, on the same config-0 layer."""
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import bench
    import oracle
    from __graft_entry__ import load_package

    synth = load_package().synth
    monkeypatch.setattr(oracle, "ref_available", lambda: False)
    cb = bench.cpu_baseline(argparse.Namespace(layers=2, seed=3, cpu_budget_s=0.3), synth)
    assert cb["kind"] == "port" and cb["cores"] == 1 and cb["value"] > 0 and cb["cpu_model"]


def test_cpu_baseline_every_config():
    """With glm.c compiled: the config-0 line plus the 1-thread line, the
    config-1 matvec shapes and the config-3/4 token loops (config 2's full
    decoder is skipped here: it needs ~33 GB of host memory)."""
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import bench
    import oracle
    from __graft_entry__ import load_package

    if not oracle.ref_available():
        pytest.skip("oracle/_ref not built here")
    synth = load_package().synth
    args = argparse.Namespace(layers=2, seed=3, cpu_budget_s=0.3, prefill_tokens=16, ep_layers=2, no_decode=True)
    cb = bench.cpu_baseline(args, synth)
    assert cb["kind"] == "reference" and cb["value"] > 0 and cb["one_thread"]["value"] > 0
    assert set(cb["matvec"]) == {f"{r}x{c}" for r, c in bench.MATVEC_SHAPES}
    assert cb["prefill"]["tok_s"] > 0 and cb["ep_prefill"]["tok_s"] > 0
