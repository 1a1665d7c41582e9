"""LoRA shrink kernels: the tensor-core shrink (tcgen05, every distinct tenant of a
128-row tile stacked into one B operand) against the per-warp mma.sync shrink.

STAGEML_SHRINK (read once per process) picks the kernel: "mma" for every shrink,
"tc" (default) for rows already in the GEMM layout, "tc_all" for gathered rows too.
Each mode runs in a child process; every case must match the oracle within the
16-bit tolerance, and the modes agree far closer than that (they differ only in the
fp32 summation order of the partial dot products before the 16-bit rounding of S).
"""

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL16 = 1e-2
MODES = ("mma", "tc", "tc_all")
HERE = Path(__file__).resolve().parent


def _run(mode: str, out: Path) -> dict:
    env = dict(os.environ, STAGEML_SHRINK=mode)
    r = subprocess.run([sys.executable, str(HERE / "shrink_modes_child.py"), str(out)], env=env, capture_output=True,
                       text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-3000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


@pytest.fixture(scope="module")
def results(tmp_path_factory):
    d = tmp_path_factory.mktemp("shrink_modes")
    res = {}
    for m in MODES:
        res[m] = _run(m, d / f"{m}.pt")
        res[m]["_y"] = torch.load(d / f"{m}.pt")
    return res


@pytest.mark.parametrize("mode", MODES)
def test_shrink_mode_matches_oracle(results, mode):
    res = results[mode]
    assert res["status"] == 0
    for name, v in res.items():
        if name in ("status", "_y"):
            continue
        assert v["rel_l2"] < TOL16, (mode, name, v)


@pytest.mark.parametrize("mode", ["tc", "tc_all"])
def test_tensor_core_shrink_agrees_with_warp_shrink(results, mode):
    for name, y in results["mma"]["_y"].items():
        z = results[mode]["_y"][name]
        rel = float((z - y).norm() / y.norm())
        assert rel < 2e-3, (mode, name, rel)
