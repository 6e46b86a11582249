"""Spatial domain decomposition on the GPU (csrc/domain.cu through the C ABI
mlipcpp_b200_domain_*): several ranks emulated on one GPU, one thread, model
and engine each, exchanging through in-process collectives.  Their summed
energy, gathered forces and stress must equal the whole-cell evaluation and
the float64 oracle.  Tolerances are the fp32 parity bar (|dE|/N <= 1e-5 eV,
|dF| <= 1e-4 eV/A, |dsigma| <= 1e-4 eV/A^3)."""
import numpy as np
import pytest
import torch

import mlipcpp_b200 as mb
from mlipcpp_b200 import domain as dd
from mlipcpp_b200 import workloads as wl
from oracle import pet_oracle as po

pytestmark = pytest.mark.gpu
TOL_E, TOL_F, TOL_S = 1e-5, 1e-4, 1e-4


def check(e, F, S, ref_e, ref_F, ref_S, n):
    assert abs(e - ref_e) / n <= TOL_E, (e, ref_e)
    assert np.abs(F - ref_F).max() <= TOL_F, np.abs(F - ref_F).max()
    assert np.abs(S - ref_S).max() <= TOL_S, np.abs(S - ref_S).max()


def stress(virial, cell):
    return np.asarray(virial) / abs(np.linalg.det(np.asarray(cell, np.float64)))


@pytest.mark.parametrize("grid", [(1, 1, 1), (1, 1, 2), (1, 2, 2), (2, 2, 2)])
def test_domains_match_whole_cell(grid, model_file):
    path = model_file("pet-mad-s", 5)
    s = wl.si_diamond(4, seed=61)
    full = mb.Predictor(path).predict(s.positions, s.numbers, s.cell, s.pbc, compute_stress=True)
    e, F, vir, st = dd.run_emulated(lambda: mb.Predictor(path), s, grid)
    check(e, F, stress(vir, s.cell), full.energy, full.forces, full.stress, s.n_atoms)
    if grid != (1, 1, 1):
        assert all(x["ghosts"] > 0 and x["token_rows_in"] > 0 for x in st)
        # every requested token was found by its owner: rows sent == rows
        # requested, summed over the ranks
        assert sum(x["token_rows_in"] for x in st) == sum(x["token_rows_out"] for x in st)


def test_domains_match_oracle_triclinic(model_file):
    path = model_file("pet-oam-l", 7)
    s = wl.fcc_alloy(10, seed=62)
    ref = po.load_oracle(path, torch.float64).predict([s])[0]
    e, F, vir, _ = dd.run_emulated(lambda: mb.Predictor(path), s, (2, 2, 2))
    check(e, F, stress(vir, s.cell), ref["energy_f64"], ref["forces"], ref["stress"], s.n_atoms)


def test_domains_unwrapped_positions_skin_and_repeat(model_file):
    # positions moved by whole cell vectors, a skin, and two steps in a row:
    # the same cell, the same answer from step to step
    path = model_file("pet-mad-s", 8)
    s = wl.si_diamond(4, seed=63)
    rng = np.random.default_rng(5)
    moved = wl.Structure((s.positions + rng.integers(-3, 4, size=(s.n_atoms, 3)) @ s.cell).astype(np.float32),
                         s.numbers, s.cell, s.pbc)
    # the reference sees the same float32 positions (moving by cell vectors
    # rounds them by ~1e-5 A at |x| ~ 65 A, which moves forces by ~1e-4)
    full = mb.Predictor(path).predict(moved.positions, s.numbers, s.cell, s.pbc, compute_stress=True)
    e1, F1, v1, _ = dd.run_emulated(lambda: mb.Predictor(path), moved, (1, 2, 2), skin=0.4, steps=1)
    e2, F2, v2, _ = dd.run_emulated(lambda: mb.Predictor(path), moved, (1, 2, 2), skin=0.4, steps=2)
    check(e1, F1, stress(v1, s.cell), full.energy, full.forces, full.stress, s.n_atoms)
    # energy and virial are deterministic sums; forces on ghosts are
    # accumulated with atomic adds (edges whose reverse is on another rank),
    # so repeated steps agree to rounding
    assert e1 == e2 and np.array_equal(v1, v2)
    assert np.abs(F1 - F2).max() <= 2e-6


def test_domain_rejects_too_small_cell(model_file):
    pred = mb.Predictor(model_file("pet-mad-s", 5))
    s = wl.si_diamond(2, seed=64)  # 10.9 A: a slab of 5.4 A is thinner than 2 cutoffs
    comm = dd.LocalComm(2)
    with pytest.raises(mb.MLIPError) as ei:
        dd.Domain(pred, s.cell, (1, 1, 2), 0, comm.for_rank(0))
    assert ei.value.code == mb.INVALID_PARAMETER
    assert "slab" in str(ei.value)


class AbandoningComm(dd.LocalComm):
    """Rank `bad` abandons one exchange of the step (the `at`-th alltoallv,
    or the final all-reduce for at = 0): it reports an error without
    joining the others, as a rank that dies or never posts its halo would.
    The failure is made on the host; no kernel is made to fault or wait."""

    def __init__(self, world, bad, at):
        super().__init__(world, timeout=30.0)
        self.bad, self.at, self.calls = bad, at, 0

    def _alltoallv(self, rank, *args):
        if rank == self.bad:
            self.calls += 1
            if self.calls == self.at:
                return 1
        return super()._alltoallv(rank, *args)

    def _allreduce(self, rank, *args):
        if rank == self.bad and self.at == 0:
            return 1
        return super()._allreduce(rank, *args)


@pytest.mark.parametrize("at", [1, 4, 5, 6, 7, 0])
def test_domain_exchange_failure_is_reported_and_ranks_recover(at, model_file):
    """A failed exchange at any point of the step (halo counts, requests,
    the layer-0 tokens inside the forward pass, their gradients inside the
    backward, the force halo, the final sum) ends every rank's step with
    MLIPCPP_ERROR_COMPUTATION instead of a hang; the same models then give
    the result of a clean step again."""
    path = model_file("pet-mad-s", 9)
    s = wl.si_diamond(4, seed=64)
    preds = [mb.Predictor(path), mb.Predictor(path)]
    grid = (1, 1, 2)

    def run(comm=None):
        it = iter(preds)
        return dd.run_emulated(lambda: next(it), s, grid, comm=comm)

    e0, F0, v0, _ = run()
    with pytest.raises(mb.MLIPError) as ei:
        run(AbandoningComm(2, bad=1, at=at))
    assert ei.value.code == mb.COMPUTATION
    assert "domain exchange" in str(ei.value)
    e1, F1, v1, _ = run()
    assert e1 == e0
    np.testing.assert_allclose(F1, F0, rtol=0, atol=2e-6)
    np.testing.assert_allclose(np.asarray(v1), np.asarray(v0), rtol=0, atol=1e-9 * max(1.0, np.abs(v0).max()))
