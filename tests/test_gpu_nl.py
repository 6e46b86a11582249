"""GPU neighbour list (through the C ABI) is bit-identical to the reference:
the committed fixtures made by the reference's own code, and the C oracle on
fresh seeded structures up to the 32k-atom benchmark cell."""
import glob
import os

import numpy as np
import pytest

from conftest import GOLDEN, nl_equal
import mlipcpp_b200 as mb
from mlipcpp_b200 import workloads as wl
from oracle import nl

pytestmark = pytest.mark.gpu
FIXTURES = sorted(glob.glob(os.path.join(GOLDEN, "nl_*.npz")))


@pytest.mark.parametrize("path", FIXTURES, ids=lambda p: os.path.basename(p)[3:-4])
def test_gpu_nl_matches_reference_fixture(path):
    f = np.load(path)
    cell = f["cell"] if f["cell"].size else None
    pbc = tuple(bool(x) for x in f["pbc"]) if cell is not None else None
    got = mb.neighbor_list(f["positions"], cell, pbc, float(f["cutoff"]))
    assert nl_equal(got, f) is None


@pytest.mark.parametrize("case", ["si_2k", "fcc_4k_triclinic", "water_1k", "molecule", "fcc32k",
                                  "si_partial_pbc", "si_small_cell_wide_cutoff"])
def test_gpu_nl_matches_oracle(case):
    s, rc = {
        "si_2k": lambda: (wl.si_diamond(6, seed=21), 4.5),
        "fcc_4k_triclinic": lambda: (wl.fcc_alloy(16, seed=22), 4.5),
        "water_1k": lambda: (wl.water_box(1024, seed=23), 4.5),
        "molecule": lambda: (wl.molecules(1, seed=24, n_min=60, n_max=60)[0], 4.5),
        "fcc32k": lambda: (wl.fcc_alloy(32, seed=0), 4.5),
        "si_partial_pbc": lambda: (wl.Structure(*(lambda t: (t.positions, t.numbers, t.cell))(
            wl.si_diamond(3, seed=25)), (True, False, True)), 4.5),
        "si_small_cell_wide_cutoff": lambda: (wl.si_diamond(1, seed=26), 7.0),
    }[case]()
    got = mb.neighbor_list(s.positions, s.cell, s.pbc, rc)
    ref = nl.build_oracle(s.positions, s.cell, s.pbc, rc)
    assert nl_equal(got, ref) is None


def test_gpu_nl_edge_cases():
    assert len(mb.neighbor_list(np.zeros((1, 3), np.float32), cutoff=5.0)["centers"]) == 0
    assert len(mb.neighbor_list(np.zeros((0, 3), np.float32), cutoff=5.0)["centers"]) == 0
    two = np.array([[0, 0, 0], [3.0, 0, 0]], np.float32)
    assert len(mb.neighbor_list(two, cutoff=3.0)["centers"]) == 0
    r = mb.neighbor_list(two, cutoff=3.5)
    assert list(r["centers"]) == [0, 1] and list(r["neighbors"]) == [1, 0]
