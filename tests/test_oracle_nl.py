"""The C neighbour-list oracle against the reference's own code: the
committed fixtures (made by the reference sources) and, where the reference
tree was compiled here, a live comparison on fresh seeded structures.
Semantics follow tests/test_neighbor_list.cpp of the reference."""
import glob
import os

import numpy as np
import pytest

from conftest import GOLDEN, nl_equal
from mlipcpp_b200 import workloads as wl
from oracle import nl

FIXTURES = sorted(glob.glob(os.path.join(GOLDEN, "nl_*.npz")))


def _args(f):
    cell = f["cell"] if f["cell"].size else None
    pbc = tuple(bool(x) for x in f["pbc"]) if cell is not None else None
    return f["positions"], cell, pbc, float(f["cutoff"])


@pytest.mark.parametrize("path", FIXTURES, ids=lambda p: os.path.basename(p)[3:-4])
def test_oracle_matches_reference_fixture(path):
    f = np.load(path)
    got = nl.build_oracle(*_args(f))
    assert nl_equal(got, f) is None


@pytest.mark.skipif(not nl.reference_available(), reason="reference sources not compiled here")
@pytest.mark.parametrize("seed", [11, 12, 13])
def test_oracle_matches_reference_live(seed):
    for s, rc in [(wl.si_diamond(2, seed=seed), 4.5), (wl.fcc_alloy(5, seed=seed), 4.5),
                  (wl.water_box(150, seed=seed), 4.0), (wl.molecules(1, seed=seed)[0], 4.5)]:
        assert nl_equal(nl.build_oracle(s.positions, s.cell, s.pbc, rc),
                        nl.build_reference(s.positions, s.cell, s.pbc, rc)) is None


@pytest.mark.skipif(not nl.reference_available(), reason="reference sources not compiled here")
def test_cell_inverse_bitexact():
    for s in [wl.fcc_alloy(3, seed=1), wl.si_diamond(2), wl.water_box(60)]:
        a = nl.cell_inverse(s.cell, "oracle")
        b = nl.cell_inverse(s.cell, "ref")
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_reference_semantics():
    # tests/test_neighbor_list.cpp:58-87: exclusive cutoff
    two = lambda d: np.array([[0, 0, 0], [d, 0, 0]], np.float32)
    assert len(nl.build_oracle(two(2.0), cutoff=3.0)["centers"]) == 2
    assert len(nl.build_oracle(two(5.0), cutoff=3.0)["centers"]) == 0
    assert len(nl.build_oracle(two(3.0), cutoff=3.0)["centers"]) == 0
    # :216-245 vectors point from centre to neighbour
    r = nl.build_oracle(two(2.0), cutoff=5.0)
    for c, n, v in zip(r["centers"], r["neighbors"], r["edge_vectors"]):
        assert v[0] == (2.0 if c == 0 else -2.0)
    # :129-140 isolated atom, full-list symmetry, periodic shifts
    assert len(nl.build_oracle(np.zeros((1, 3), np.float32), cutoff=5.0)["centers"]) == 0
    s = wl.si_diamond(1)
    r = nl.build_oracle(s.positions, s.cell, s.pbc, 5.0)
    assert (r["distances"] < 5.0).all() and (r["distances"] > 0).all()
    assert np.any(r["cell_shifts"] != 0)
    keys = {(a, b, *sh) for a, b, sh in zip(r["centers"], r["neighbors"], map(tuple, r["cell_shifts"]))}
    assert all((b, a, *(-np.asarray(sh))) in keys for (a, b, *sh) in keys)
