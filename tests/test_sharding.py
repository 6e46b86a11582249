"""Batches of independent structures sharded over ranks
(mlip.cpp_b200/sharding.py): the split, and a 2-rank gloo run whose
gathered results equal the single-process float64 oracle."""
import os
import socket

import numpy as np
import pytest
import torch

import conftest  # noqa: F401  (registers mlipcpp_b200, also in spawned ranks)
from mlipcpp_b200 import sharding as sh
from mlipcpp_b200 import workloads as wl
from oracle import pet_oracle as po


def test_shard_covers_every_structure_once_and_balances():
    rng = np.random.default_rng(0)
    n = rng.integers(10, 61, size=512)
    costs = [sh.structure_cost(int(k)) for k in n]
    for world in (1, 2, 3, 8):
        parts = sh.shard(costs, world)
        assert sorted(i for p in parts for i in p) == list(range(512))
        loads = [sum(costs[i] for i in p) for p in parts]
        # LPT: the heaviest rank exceeds the mean by at most the largest item
        assert max(loads) <= sum(costs) / world + max(costs)


def oracle_eval(orc):
    def run(structs):
        return [(r["energy_f64"], r["forces"], r.get("stress")) for r in orc.predict(structs)]
    return run


def _rank(rank, world, port, path, out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    orc = po.load_oracle(path, torch.float64)
    mols = wl.molecules(12, n_min=4, n_max=14, seed=5)
    res = sh.BatchRunner(oracle_eval(orc), world=world, rank=rank).run(mols)
    if rank == 0:
        np.savez(out, e=np.array([r[0] for r in res]), **{f"f{i}": r[1] for i, r in enumerate(res)})
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_match_one_process(model_file, tmp_path):
    import torch.multiprocessing as mp
    path = model_file("tiny", 11, cutoff=3.0, cutoff_width=0.5)
    mols = wl.molecules(12, n_min=4, n_max=14, seed=5)
    ref = po.load_oracle(path, torch.float64).predict(mols)
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        port = sock.getsockname()[1]
    out = str(tmp_path / "r.npz")
    mp.start_processes(_rank, args=(2, port, path, out), nprocs=2, start_method="spawn")
    r = np.load(out)
    np.testing.assert_allclose(r["e"], [x["energy_f64"] for x in ref], rtol=0, atol=1e-9)
    for i, x in enumerate(ref):
        np.testing.assert_allclose(r[f"f{i}"], x["forces"], rtol=0, atol=1e-9)


@pytest.mark.gpu
def test_gpu_sharded_batch_matches_one_batch(model_file):
    """Two shards evaluated one after the other with the GPU library give
    the results of one batched call."""
    import mlipcpp_b200 as mb
    pred = mb.Predictor(model_file("pet-mad-s", 12))
    mols = wl.molecules(40, seed=12)
    whole = pred.predict_batch(mols)
    ev = sh.predictor_batch_eval(pred)
    parts = sh.shard([sh.structure_cost(m.n_atoms) for m in mols], 2)
    got = {}
    for p in parts:
        for i, r in zip(p, ev([mols[i] for i in p])):
            got[i] = r
    for i, w in enumerate(whole):
        assert abs(got[i][0] - w.energy) / mols[i].n_atoms <= 1e-5
        assert np.abs(got[i][1] - w.forces).max() <= 1e-4
