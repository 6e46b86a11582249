"""The C++ interface (include/mlipcpp.hpp, the reference's
include/mlipcpp/mlipcpp.hpp:132-303): a caller written against the
reference's mlipcpp::Predictor compiles against it and links the library
(CPU), and its predictions equal the Python Predictor's through the same C
ABI (GPU)."""
import os
import shutil
import subprocess

import numpy as np
import pytest

from conftest import ROOT
import mlipcpp_b200 as mb
from mlipcpp_b200 import workloads as wl

CALLER = os.path.join(ROOT, "tests", "cxx", "predictor_caller.cpp")
LIBDIR = os.path.dirname(mb.LIB_PATH)


@pytest.fixture(scope="module")
def caller(tmp_path_factory):
    if not shutil.which("g++"):
        pytest.skip("no C++ compiler")
    exe = str(tmp_path_factory.mktemp("cxx") / "predictor_caller")
    subprocess.run(["g++", "-std=c++20", "-O1", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                    CALLER, "-L", LIBDIR, "-lmlipcpp_b200", f"-Wl,-rpath,{LIBDIR}", "-o", exe], check=True)
    return exe


def test_cxx_caller_compiles_and_runs_api_checks(caller):
    out = subprocess.run([caller], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "api OK" in out.stdout


def write_system(path, s):
    n = s.n_atoms
    periodic = s.cell is not None
    cell = np.zeros(9, np.float32) if not periodic else np.asarray(s.cell, np.float32).reshape(9)
    with open(path, "wb") as f:
        f.write(np.array([n, int(periodic)], np.int32).tobytes())
        f.write(cell.tobytes())
        f.write(np.ascontiguousarray(s.positions, np.float32).tobytes())
        f.write(np.ascontiguousarray(s.numbers, np.int32).tobytes())


def parse(stdout):
    out = {}
    for line in stdout.splitlines():
        p = line.split()
        if len(p) >= 3 and p[1] == "energy":
            out.setdefault(p[0], {})["energy"] = float(p[2])
        elif len(p) == 5 and p[1] == "F":
            out[p[0]].setdefault("forces", []).append([float(x) for x in p[2:]])
        elif len(p) == 8 and p[1] == "S":
            out[p[0]]["stress"] = [float(x) for x in p[2:]]
    return out


@pytest.mark.gpu
def test_cxx_predictions_match_python_predictor(caller, model_file, tmp_path):
    path = model_file("pet-mad-s", seed=4)
    py = mb.Predictor(path)
    s = wl.si_diamond(2, seed=5)
    sysf = str(tmp_path / "si64.bin")
    write_system(sysf, s)
    run = subprocess.run([caller, path, sysf], capture_output=True, text=True, timeout=600)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "size check OK" in run.stdout
    got = parse(run.stdout)
    ref = py.predict(s.positions, s.numbers, s.cell, compute_stress=True)
    for tag in ("span", "raw"):
        assert abs(got[tag]["energy"] - ref.energy) <= 1e-6 * max(1.0, abs(ref.energy))
        np.testing.assert_allclose(np.asarray(got[tag]["forces"]), ref.forces, rtol=0, atol=1e-6)
        np.testing.assert_allclose(np.asarray(got[tag]["stress"]), ref.stress, rtol=0, atol=1e-7)
    # compute_forces = false, compute_stress = true: stress only
    assert "forces" not in got["opts"]
    np.testing.assert_allclose(np.asarray(got["opts"]["stress"]), ref.stress, rtol=0, atol=1e-7)
    fd = py.predict(s.positions, s.numbers, s.cell, compute_stress=True, fd_stress=True)
    np.testing.assert_allclose(np.asarray(got["fd"]["stress"]), fd.stress, rtol=0, atol=1e-6)

    mol = wl.molecules(1, seed=6)[0]
    molf = str(tmp_path / "mol.bin")
    write_system(molf, mol)
    run = subprocess.run([caller, path, molf], capture_output=True, text=True, timeout=600)
    assert run.returncode == 0, run.stdout + run.stderr
    got = parse(run.stdout)
    ref = py.predict(mol.positions, mol.numbers)
    assert abs(got["raw"]["energy"] - ref.energy) <= 1e-6 * max(1.0, abs(ref.energy))
    np.testing.assert_allclose(np.asarray(got["span"]["forces"]), ref.forces, rtol=0, atol=1e-6)
