"""The benchmark's CPU reference arm (the driver runs `bench.py --impl
reference`): it must print one JSON line with the contract's keys, time the
reference's CPU path on all of this host's cores, and need no GPU.  Run the
way torchrun runs it too (OMP_NUM_THREADS=1 exported)."""
import json
import os
import subprocess
import sys

from conftest import ROOT


def test_reference_arm_prints_contract_line():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "1"], capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    # the reference's own kv_quant + SDPA when baseline/_ref holds the reference
    # install, else the oracle port; always on every host core
    want = "reference" if os.path.exists(os.path.join(ROOT, "baseline", "_ref", "kv_quant.py")) else "port"
    assert d["cpu_baseline"]["kind"] == want and d["cpu_baseline"]["cores"] == len(os.sched_getaffinity(0))
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert "workload" in d["config"]
