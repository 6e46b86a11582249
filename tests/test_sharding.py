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


def test_packed_batch_layout():
    mols = wl.molecules(9, n_min=4, n_max=14, seed=3)
    b = sh.PackedBatch.pack(mols)
    assert len(b) == 9 and b.first[-1] == sum(m.n_atoms for m in mols)
    for k, m in enumerate(b.structures()):
        np.testing.assert_array_equal(m.positions, mols[k].positions)
        np.testing.assert_array_equal(m.numbers, mols[k].numbers)
    idx = [7, 2, 5]
    sub = b.take(idx)
    np.testing.assert_array_equal(sub.n_atoms, [mols[i].n_atoms for i in idx])
    np.testing.assert_array_equal(sub.positions, np.concatenate([mols[i].positions for i in idx]))
    np.testing.assert_array_equal(b.positions[b.atom_index(idx)], sub.positions)
    assert b.take(range(9)) is b
    cells = [wl.si_diamond(1, seed=s) for s in (1, 2)]
    pc = sh.PackedBatch.pack(cells)
    assert pc.cells.shape == (2, 9) and pc.pbc.all()
    with pytest.raises(ValueError):
        sh.PackedBatch.pack([mols[0], cells[0]])


def oracle_packed_eval(orc):
    def run(batch):
        res = orc.predict(batch.structures())
        return (np.array([r["energy_f64"] for r in res]),
                np.concatenate([np.asarray(r["forces"]) for r in res]), None)
    return run


def _rank_packed(rank, world, port, path, out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    orc = po.load_oracle(path, torch.float64)
    b = sh.PackedBatch.pack(wl.molecules(12, n_min=4, n_max=14, seed=5))
    e, f, st = sh.PackedBatchRunner(oracle_packed_eval(orc), world=world, rank=rank).run(b)
    assert st is None
    if rank == 0:
        np.savez(out, e=e, f=f)
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_packed_match_one_process(model_file, tmp_path):
    import torch.multiprocessing as mp
    path = model_file("tiny", 11, cutoff=3.0, cutoff_width=0.5)
    mols = wl.molecules(12, n_min=4, n_max=14, seed=5)
    ref = po.load_oracle(path, torch.float64).predict(mols)
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        port = sock.getsockname()[1]
    out = str(tmp_path / "p.npz")
    mp.start_processes(_rank_packed, args=(2, port, path, out), nprocs=2, start_method="spawn")
    r = np.load(out)
    np.testing.assert_allclose(r["e"], [x["energy_f64"] for x in ref], rtol=0, atol=1e-9)
    np.testing.assert_allclose(r["f"], np.concatenate([x["forces"] for x in ref]), rtol=0, atol=1e-9)


@pytest.mark.gpu
def test_gpu_packed_batch_matches_batch(model_file):
    """predict_packed equals predict_batch (same kernels, same grouping),
    for molecules and for periodic cells, and the packed runner's one-rank
    path is the same call."""
    import mlipcpp_b200 as mb
    pred = mb.Predictor(model_file("pet-mad-s", 12))
    mols = wl.molecules(40, seed=13)
    whole = pred.predict_batch(mols)
    b = sh.PackedBatch.pack(mols)
    r = pred.predict_packed(b.positions, b.numbers, b.n_atoms)
    assert r.stress is None
    for k, w in enumerate(whole):
        assert r.energies[k] == np.float32(w.energy)
        np.testing.assert_array_equal(r.forces[b.first[k]:b.first[k + 1]], w.forces)
    e, f, _ = sh.PackedBatchRunner(sh.predictor_packed_eval(pred)).run(b)
    np.testing.assert_array_equal(e, r.energies)
    np.testing.assert_array_equal(f, r.forces)
    cells = [wl.si_diamond(2, seed=s) for s in (1, 2)]
    pc = sh.PackedBatch.pack(cells)
    rp = pred.predict_packed(pc.positions, pc.numbers, pc.n_atoms, pc.cells, pc.pbc, compute_stress=True)
    for k, c in enumerate(cells):
        one = pred.predict(c.positions, c.numbers, c.cell, compute_stress=True)
        assert rp.energies[k] == np.float32(one.energy)
        np.testing.assert_array_equal(rp.forces[pc.first[k]:pc.first[k + 1]], one.forces)
        np.testing.assert_array_equal(rp.stress[k], one.stress)
    # energy only: forces not asked for, not returned
    eo = pred.predict_packed(b.positions, b.numbers, b.n_atoms, compute_forces=False)
    assert eo.forces is None and eo.energies.shape == (40,)
    with pytest.raises(mb.MLIPError) as ei:
        pred.predict_packed(b.positions[:3], b.numbers[:3], [3, 0])
    assert ei.value.code == mb.INVALID_PARAMETER


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


def _rank_packed_small(rank, world, port, out):
    """More ranks than structures: some shares are empty."""
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    b = sh.PackedBatch.pack(wl.molecules(2, n_min=3, n_max=6, seed=8))

    def ev(sub):  # energy = sum of Z, force = the positions, stress = 1..6 per structure
        e = np.array([float(s.numbers.sum()) for s in sub.structures()])
        return e, sub.positions.astype(np.float64), np.tile(np.arange(1, 7, dtype=np.float32), (len(sub), 1))
    e, f, st = sh.PackedBatchRunner(ev, world=world, rank=rank).run(b)
    if rank == 0:
        np.savez(out, e=e, f=f, st=st)
    dist.barrier()
    dist.destroy_process_group()


def test_three_gloo_ranks_with_empty_shares(tmp_path):
    import torch.multiprocessing as mp
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        port = sock.getsockname()[1]
    out = str(tmp_path / "s.npz")
    mp.start_processes(_rank_packed_small, args=(3, port, out), nprocs=3, start_method="spawn")
    r = np.load(out)
    b = sh.PackedBatch.pack(wl.molecules(2, n_min=3, n_max=6, seed=8))
    np.testing.assert_array_equal(r["e"], [float(s.numbers.sum()) for s in b.structures()])
    assert r["f"].dtype == np.float64 and r["st"].dtype == np.float32
    np.testing.assert_array_equal(r["f"], b.positions)
    np.testing.assert_array_equal(r["st"], np.tile(np.arange(1, 7), (2, 1)))


def test_packed_runner_plan_inverts_the_rank_order_and_is_kept():
    """The exchange plan of a 3-rank runner: the gathered shares, in rank
    order, go back to input order through its inverse permutations; the plan
    is reused while the sizes repeat and remade when they change."""
    mols = wl.molecules(10, n_min=3, n_max=9, seed=11)
    b = sh.PackedBatch.pack(mols)
    r = sh.PackedBatchRunner(None, world=3, rank=1)
    P = r._plan(b, None)
    assert sorted(i for p in P["parts"] for i in p) == list(range(10))
    s_cat = np.concatenate([np.asarray(p) for p in P["parts"]])
    np.testing.assert_array_equal(s_cat[P["s_inv"]], np.arange(10))
    a_cat = np.concatenate(P["rows"])
    np.testing.assert_array_equal(a_cat[P["a_inv"]], np.arange(b.positions.shape[0]))
    assert r._plan(sh.PackedBatch.pack(mols), None) is P
    other = sh.PackedBatch.pack(wl.molecules(10, n_min=3, n_max=9, seed=12))
    assert r._plan(other, None) is not P
