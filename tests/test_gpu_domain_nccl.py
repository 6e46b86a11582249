"""Spatial domains on real ranks: one process per GPU, exchanges over NCCL
(torch.distributed), against the whole-cell prediction at the fp32 parity
bar.  Needs at least two GPUs (skipped otherwise)."""
import json
import os
import subprocess
import sys

import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [2, 4, 8])
def test_nccl_domains_match_whole_cell(world, model_file, tmp_path):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    path = model_file("pet-oam-l", 9)
    out = str(tmp_path / "result.json")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes", "1",
           "--nproc-per-node", str(world), "--master-addr", "127.0.0.1", "--master-port", str(29400 + world),
           os.path.join(ROOT, "tests", "domain_nccl_rank.py"), path, out]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    run = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert run.returncode == 0, run.stdout[-3000:] + run.stderr[-3000:]
    r = json.load(open(out))
    assert r["de_per_atom"] <= 1e-5 and r["df"] <= 1e-4 and r["ds"] <= 1e-4, r
    assert r["stats"]["token_rows_in"] > 0 and r["stats"]["ghosts"] > 0
