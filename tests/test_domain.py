"""Spatial domain decomposition (mlip.cpp_b200/domain.py, csrc/domain.cu) on
CPU: the grid, the ownership of atoms, and the halo geometry.  The halo test
is a float64 restatement of the engine's (every atom within the cutoff of an
owned atom must reach the local system exactly once, images included); the
engine itself runs in test_gpu_domain.py."""
import numpy as np
import pytest

import conftest  # noqa: F401  (registers mlipcpp_b200)
from mlipcpp_b200 import domain as dd
from mlipcpp_b200 import workloads as wl


def test_grid_for():
    assert dd.grid_for(1) == (1, 1, 1)
    assert dd.grid_for(2) == (1, 1, 2)
    assert dd.grid_for(4) == (1, 2, 2)
    assert dd.grid_for(8) == (2, 2, 2)


@pytest.mark.parametrize("grid", [(1, 1, 2), (1, 2, 2), (2, 2, 2), (1, 1, 3)])
def test_every_atom_owned_once(grid):
    s = wl.fcc_alloy(10, seed=2)
    # some atoms outside the cell (unwrapped coordinates)
    shift = np.random.default_rng(3).integers(-2, 3, size=(s.n_atoms, 3)) @ s.cell.astype(np.float64)
    pos = s.positions.astype(np.float64) + shift
    own = dd.owners(pos, s.cell, grid)
    assert own.min() >= 0 and own.max() < np.prod(grid)
    assert np.array_equal(own, dd.owners(s.positions, s.cell, grid))
    assert len(np.unique(own)) == np.prod(grid)


def _local_system(pos, cell, grid, rank, width):
    """Owned atoms (wrapped) and received copies of rank `rank`: global
    atom, image shift (cell vectors), position."""
    cell = np.asarray(cell, np.float64)
    frac = pos @ np.linalg.inv(cell)
    W = -np.floor(frac)
    own = np.nonzero(dd.owners(pos, cell, grid) == rank)[0]
    atoms = [(int(i), tuple(W[i].astype(int))) for i in own]
    for src in range(int(np.prod(grid))):
        for i, s in dd.halo_copies(pos, cell, grid, src, rank, width):
            atoms.append((i, tuple((W[i] + np.array(s)).astype(int))))
    return atoms, len(own)


@pytest.mark.parametrize("grid", [(1, 1, 2), (1, 2, 2), (2, 2, 2)])
def test_halo_reaches_every_neighbour_once(grid):
    s = wl.si_diamond(4, seed=1)
    rc = 4.5
    cell = s.cell.astype(np.float64)
    pos = s.positions.astype(np.float64)
    split = np.array([g > 1 for g in grid])
    for r in range(int(np.prod(grid))):
        atoms, n_own = _local_system(pos, cell, grid, r, rc)
        # images are told apart only along split axes (the local system is
        # periodic along the others)
        key = lambda i, sh: (i, *(int(x) if sp else 0 for x, sp in zip(sh, split)))  # noqa: E731
        keys = [key(i, sh) for i, sh in atoms]
        assert len(set(keys)) == len(keys)  # no atom image twice
        present = set(keys)
        owned = atoms[:n_own]
        opos = np.array([pos[i] + np.array(sh) @ cell for i, sh in owned])
        frac = pos @ np.linalg.inv(cell)
        base = -np.floor(frac)
        shifts = np.array(np.meshgrid(*([(-1, 0, 1)] * 3), indexing="ij")).reshape(3, -1).T
        for sh in shifts:
            img = base + sh
            pimg = pos + img @ cell
            dmin = np.min(np.linalg.norm(pimg[:, None, :] - opos[None, :, :], axis=2), axis=1)
            for i in np.nonzero(dmin < rc)[0]:
                assert key(int(i), img[i].astype(int)) in present, (r, i, img[i])
