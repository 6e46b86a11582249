"""Spatial domain decomposition (mlip.cpp_b200/domain.py) on CPU: the
partition, the ghost shells, and the cross-rank sums over a 2-rank gloo
group.  The per-domain evaluation here is the float64 oracle restricted to
the owned atoms' energy; the GPU evaluator is tested in test_gpu_domain.py."""
import os

import numpy as np
import pytest
import torch

import conftest  # noqa: F401  (registers mlipcpp_b200, also in spawned ranks)
from mlipcpp_b200 import domain as dd
from mlipcpp_b200 import workloads as wl
from oracle import pet_oracle as po


def test_grid_for():
    assert dd.grid_for(1) == (1, 1, 1)
    assert dd.grid_for(2) == (1, 1, 2)
    assert dd.grid_for(4) == (1, 2, 2)
    assert dd.grid_for(8) == (2, 2, 2)


@pytest.mark.parametrize("grid", [(1, 1, 2), (1, 2, 2), (2, 2, 2)])
def test_partition_owns_once_and_ghosts_complete(grid):
    s = wl.si_diamond(3, seed=1)
    rc = 3.0
    n_dom = int(np.prod(grid))
    owners = np.zeros(s.n_atoms, int)
    cell = s.cell.astype(np.float64)
    for r in range(n_dom):
        d = dd.partition(s.positions, cell, rc, grid, r)
        owners[d.index[:d.n_owned]] += 1
        assert d.pbc == tuple(g == 1 for g in grid)
        split = np.array([g > 1 for g in grid])
        local = s.positions[d.index].astype(np.float64) + d.shift @ cell
        # images are told apart only along split axes (the local system is
        # periodic along the others)
        key = lambda i, sh: (int(i), *(int(x) if sp else 0 for x, sp in zip(sh, split)))  # noqa: E731
        keys = {key(i, sh) for i, sh in zip(d.index, d.shift)}
        assert len(keys) == d.n_local  # no duplicate images
        own = local[:d.n_owned]
        # every image of every atom within 2 rc of an owned atom is local, and
        # within rc of an owned atom it is in the layer-0 set
        shifts = np.array(np.meshgrid(*([(-2, -1, 0, 1, 2)] * 3), indexing="ij")).reshape(3, -1).T
        frac = s.positions.astype(np.float64) @ np.linalg.inv(cell)
        base = -np.floor(frac)
        lay0 = {key(i, sh) for i, sh in zip(d.index[:d.n_layer0], d.shift[:d.n_layer0])}
        for sh in shifts:
            img_shift = base + sh
            pos_img = s.positions.astype(np.float64) + img_shift @ cell
            dmin = np.min(np.linalg.norm(pos_img[:, None, :] - own[None, :, :], axis=2), axis=1)
            for i in np.nonzero(dmin < 2 * rc)[0]:
                assert key(i, img_shift[i]) in keys
            for i in np.nonzero(dmin < rc)[0]:
                assert key(i, img_shift[i]) in lay0
    assert np.all(owners == 1)


def oracle_local_eval(orc):
    """Owned-atom energy, its forces on every local atom, and the local
    virial, from the float64 oracle on the open local system."""
    h = orc.h

    def run(d, local_pos, numbers, forces_out):
        st = wl.Structure(local_pos.numpy().astype(np.float32), np.asarray(numbers, np.int32), d.cell, d.pbc)
        b = po.prepare_batch([st], h.cutoff, h.cutoff_width, orc.species_to_index)
        vec = torch.tensor(b.vec, dtype=torch.float64, requires_grad=True)
        e = orc.atomic_energies(b, vec)[:d.n_owned].sum()
        (g,) = torch.autograd.grad(e, vec)
        g = g.numpy()
        valid = b.pad > 0.5
        ci = np.repeat(np.arange(b.n_atoms), b.max_nb).reshape(b.n_atoms, b.max_nb)
        F = np.zeros((b.n_atoms, 3))
        np.add.at(F, ci[valid], g[valid])
        np.add.at(F, b.nbr[valid], -g[valid])
        ev, gv = b.vec[valid].astype(np.float64), g[valid]
        vir = np.array([np.sum(ev[:, 0] * gv[:, 0]), np.sum(ev[:, 1] * gv[:, 1]), np.sum(ev[:, 2] * gv[:, 2]),
                        0.5 * np.sum(ev[:, 1] * gv[:, 2] + ev[:, 2] * gv[:, 1]),
                        0.5 * np.sum(ev[:, 0] * gv[:, 2] + ev[:, 2] * gv[:, 0]),
                        0.5 * np.sum(ev[:, 0] * gv[:, 1] + ev[:, 1] * gv[:, 0])])
        comp = sum(orc.composition.get(int(z), 0.0) for z in numbers[:d.n_owned])
        forces_out.copy_(torch.from_numpy(F.astype(np.float32)))
        return float(e.detach()) + comp, vir
    return run


def _system(model_file):
    orc = po.load_oracle(model_file("tiny", 3, cutoff=3.0, cutoff_width=0.5), torch.float64)
    return orc, wl.si_diamond(3, seed=2)


def test_emulated_domains_match_full_oracle(model_file):
    orc, s = _system(model_file)
    full = orc.predict([s])[0]
    for n_dom in (2, 8):
        run = dd.DomainRunner(oracle_local_eval(orc), s.numbers, s.cell, orc.h.cutoff, emulate=n_dom, device="cpu")
        e, F, vir = run.step(torch.from_numpy(s.positions))
        assert abs(e - full["energy_f64"]) / s.n_atoms < 1e-6
        np.testing.assert_allclose(F.numpy(), full["forces"], atol=2e-5)
        np.testing.assert_allclose(run.stress(vir), full["stress"], atol=2e-6)


def _rank(rank, world, port, path, out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    orc = po.load_oracle(path, torch.float64)
    s = wl.si_diamond(3, seed=2)
    run = dd.DomainRunner(oracle_local_eval(orc), s.numbers, s.cell, orc.h.cutoff, world=world, rank=rank,
                           device="cpu")
    e, F, vir = run.step(torch.from_numpy(s.positions))
    if rank == 0:
        np.savez(out, e=e, F=F.numpy(), S=run.stress(vir))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_match_full_oracle(model_file, tmp_path):
    import socket
    import torch.multiprocessing as mp
    orc, s = _system(model_file)
    full = orc.predict([s])[0]
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        port = sock.getsockname()[1]
    out = str(tmp_path / "r.npz")
    mp.start_processes(_rank, args=(2, port, model_file("tiny", 3, cutoff=3.0, cutoff_width=0.5), out),
                       nprocs=2, start_method="spawn")
    r = np.load(out)
    assert abs(float(r["e"]) - full["energy_f64"]) / s.n_atoms < 1e-6
    np.testing.assert_allclose(r["F"], full["forces"], atol=2e-5)
    np.testing.assert_allclose(r["S"], full["stress"], atol=2e-6)
