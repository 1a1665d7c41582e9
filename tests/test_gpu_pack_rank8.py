"""Rank-8 LoRA expand on the one-CTA grouped GEMM: two tenant runs per K = 16 step.

The shrink reduce writes S by the parity of each row's run in its 128-row tile (values
in columns 0-7 or 8-15 of each 16-column group, zeros in the other), and one masked MMA
over the rows of runs 2q and 2q+1 multiplies it with both runs' B rows side by side.
STAGEML_PACK_RANK8=0 keeps one masked K = 16 step per run (B's other 8 columns zero).
Both run in child processes with STAGEML_GEMM_PAIRS=0 (every GEMM on the one-CTA
kernel); both must match the oracle, and they are the same bits: each row's K = 16
step multiplies the same eight nonzero products.
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
HERE = Path(__file__).resolve().parent
MODES = {"pack": {"STAGEML_GEMM_PAIRS": "0"},
         "nopack": {"STAGEML_GEMM_PAIRS": "0", "STAGEML_PACK_RANK8": "0"}}


def _run(env_extra: dict, out: Path) -> dict:
    env = dict(os.environ, **env_extra)
    r = subprocess.run([sys.executable, str(HERE / "shrink_modes_child.py"), str(out)], env=env, capture_output=True,
                       text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-3000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


@pytest.fixture(scope="module")
def results(tmp_path_factory):
    d = tmp_path_factory.mktemp("pack_rank8")
    res = {}
    for m, env in MODES.items():
        res[m] = _run(env, d / f"{m}.pt")
        res[m]["_y"] = torch.load(d / f"{m}.pt")
    return res


@pytest.mark.parametrize("mode", list(MODES))
def test_one_cta_lora_matches_oracle(results, mode):
    res = results[mode]
    assert res["status"] == 0
    for name, v in res.items():
        if name not in ("status", "_y"):
            assert v["rel_l2"] < TOL16, (mode, name, v)


def test_packed_rank8_same_bits_as_one_run_per_step(results):
    for name, y in results["nopack"]["_y"].items():
        assert torch.equal(results["pack"]["_y"][name], y), name
