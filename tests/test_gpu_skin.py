"""Verlet neighbour lists kept across calls (mlipcpp_b200_set_neighbor_skin).

A model with a skin keeps its cutoff + skin list while no atom has moved
more than skin / 2 since the build, modulo the cell, and refreshes the
pair vectors from the new positions.  Its results must equal those of a
model that builds a fresh list every call, as the reference does
(PETModel::predict_batch, src/models/pet/pet.cpp:125-694), to rounding:
the extra pairs sit beyond the cutoff where f_c = 0 and the key mask is
-inf, like the reference's padding slots; only the order of the kept pairs
and the last bit of a refreshed vector differ."""
import numpy as np
import pytest
import torch  # noqa: F401  (md keeps its state in torch tensors)

import mlipcpp_b200 as mb
from mlipcpp_b200 import md
from mlipcpp_b200 import workloads as wl

pytestmark = pytest.mark.gpu

SKIN = 0.6


def close(a, b, n):
    assert abs(a.energy - b.energy) / n <= 5e-6
    np.testing.assert_allclose(a.forces, b.forces, rtol=0, atol=5e-5)
    if b.stress.size:
        np.testing.assert_allclose(a.stress, b.stress, rtol=0, atol=5e-5)


@pytest.fixture(scope="module")
def pair(model_file):
    path = model_file("pet-mad-s", 21)
    kept, fresh = mb.Predictor(path), mb.Predictor(path)
    kept.set_neighbor_skin(SKIN)
    return kept, fresh


def test_gpu_kept_list_matches_fresh_lists(pair):
    kept, fresh = pair
    s = wl.si_diamond(3, seed=31)
    n = s.n_atoms
    cell = np.asarray(s.cell, np.float32).reshape(3, 3)
    b0 = kept.neighbor_builds()
    pos = s.positions.copy()
    rng = np.random.default_rng(5)
    for step in range(4):  # moves well inside skin / 2 from the build
        if step:
            pos = s.positions + rng.uniform(-0.12, 0.12, s.positions.shape).astype(np.float32)
        close(kept.predict(pos, s.numbers, s.cell, compute_stress=True),
              fresh.predict(pos, s.numbers, s.cell, compute_stress=True), n)
    assert kept.neighbor_builds() == b0 + 1

    # an atom wrapped by a lattice vector has not moved
    wrapped = pos.copy()
    wrapped[0] += cell[0]
    wrapped[5] -= cell[2]
    close(kept.predict(wrapped, s.numbers, s.cell, compute_stress=True),
          fresh.predict(pos, s.numbers, s.cell, compute_stress=True), n)
    assert kept.neighbor_builds() == b0 + 1

    # a move beyond skin / 2 rebuilds
    far = pos.copy()
    far[7] += np.float32([0.5, 0.0, 0.0])
    close(kept.predict(far, s.numbers, s.cell, compute_stress=True),
          fresh.predict(far, s.numbers, s.cell, compute_stress=True), n)
    assert kept.neighbor_builds() == b0 + 2

    # another cell rebuilds
    t = wl.si_diamond(2, seed=32)
    close(kept.predict(t.positions, t.numbers, t.cell, compute_stress=True),
          fresh.predict(t.positions, t.numbers, t.cell, compute_stress=True), t.n_atoms)
    assert kept.neighbor_builds() == b0 + 3


def test_gpu_kept_list_open_system_and_batches(pair):
    kept, fresh = pair
    mol = wl.molecules(1, seed=41)[0]
    rng = np.random.default_rng(6)
    b0 = kept.neighbor_builds()
    for step in range(3):
        pos = mol.positions + (rng.uniform(-0.1, 0.1, mol.positions.shape).astype(np.float32) if step else 0)
        close(kept.predict(pos, mol.numbers), fresh.predict(pos, mol.numbers), mol.n_atoms)
    assert kept.neighbor_builds() == b0 + 1
    # a batch call builds its own list; the next single call builds again
    kept.predict_batch(wl.molecules(3, seed=42))
    b1 = kept.neighbor_builds()
    assert b1 > b0 + 1
    close(kept.predict(mol.positions, mol.numbers), fresh.predict(mol.positions, mol.numbers), mol.n_atoms)
    assert kept.neighbor_builds() == b1 + 1


def test_gpu_md_with_kept_list(model_file):
    """The device-resident MD loop from the same start with and without the
    kept list (the reference rebuilds every step): the trajectories agree,
    and the kept list is rebuilt on few steps although the integrator wraps
    positions into the cell every step."""
    path = model_file("tiny", 23)
    kept, fresh = mb.Predictor(path), mb.Predictor(path)
    kept.set_neighbor_skin(SKIN)
    s = wl.si_diamond(2, seed=23)
    m = md.masses_of(s.numbers)
    v0 = md.maxwell_boltzmann(m, 300.0, seed=4)
    runs = []
    for pred in (kept, fresh):
        b0 = pred.neighbor_builds()
        vv = md.VelocityVerlet(md.predictor_forces(pred, s.numbers, s.cell), s.positions, m, 0.5, cell=s.cell,
                               velocities=v0, device="cuda")
        vv.step(20)
        runs.append((vv.x.cpu().numpy(), vv.energy, pred.neighbor_builds() - b0))
    (xk, ek, bk), (xf, ef, bf) = runs
    np.testing.assert_allclose(xk, xf, rtol=0, atol=1e-4)
    assert ek == pytest.approx(ef, abs=1e-4)
    assert bf == 21 and bk < bf, (bk, bf)


def test_gpu_skin_argument_checks(pair):
    kept, _ = pair
    for bad in (-0.1, float("nan"), float("inf")):
        with pytest.raises(mb.MLIPError) as ei:
            kept.set_neighbor_skin(bad)
        assert ei.value.code == mb.INVALID_PARAMETER
    kept.set_neighbor_skin(SKIN)
