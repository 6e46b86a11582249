"""GPU PET energy / forces / stress through the C ABI against the oracle.

fp32 tolerances of the parity bar: |dE|/N <= 1e-5 eV, |dF| <= 1e-4 eV/A,
|dsigma| <= 1e-4 eV/A^3 (against the float64 restatement)."""
import glob
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
import mlipcpp_b200 as mb
from mlipcpp_b200 import workloads as wl
from oracle import pet_oracle as po

pytestmark = pytest.mark.gpu
TOL_E, TOL_F, TOL_S = 1e-5, 1e-4, 1e-4
FIXTURES = sorted(glob.glob(os.path.join(GOLDEN, "pet_*.npz")))


def assert_close(res, e_ref, f_ref, s_ref, n):
    assert abs(res.energy - e_ref) / n <= TOL_E, (res.energy, e_ref)
    if f_ref is not None:
        assert res.has_forces()
        assert np.abs(res.forces - f_ref).max() <= TOL_F, np.abs(res.forces - f_ref).max()
    if s_ref is not None and len(s_ref):
        assert res.has_stress()
        assert np.abs(res.stress - s_ref).max() <= TOL_S, np.abs(res.stress - s_ref).max()


@pytest.mark.parametrize("path", FIXTURES, ids=lambda p: os.path.basename(p)[4:-4])
def test_gpu_matches_golden(path, model_file):
    f = np.load(path)
    nc = bool(f["nc"]) if "nc" in f else False
    pred = mb.Predictor(model_file(str(f["hypers"]), int(f["seed"]), nc=nc))
    n_sys = int(f["n_systems"])
    systems = []
    for k in range(n_sys):
        cell = f[f"cell_{k}"]
        systems.append(wl.Structure(f[f"positions_{k}"], f[f"numbers_{k}"],
                                    cell if cell.size else None, (True,) * 3 if cell.size else None))
    if n_sys == 1:
        s = systems[0]
        res = [pred.predict_with_options(s.positions, s.numbers, s.cell, s.pbc,
                                         mb.PredictOptions(True, s.cell is not None, nc))]
    else:
        res = pred.predict_batch(systems, use_nc_forces=nc)
    for k, r in enumerate(res):
        assert_close(r, float(f[f"energy_{k}"]), f[f"forces_{k}"], f[f"stress_{k}"],
                     systems[k].n_atoms)


@pytest.mark.parametrize("case", ["si216_mads", "water384_mads", "fcc512_oaml", "si_partial_pbc"])
def test_gpu_matches_oracle(case, model_file):
    hname, s = {
        "si216_mads": lambda: ("pet-mad-s", wl.si_diamond(3, seed=31)),
        "water384_mads": lambda: ("pet-mad-s", wl.water_box(384, seed=32)),
        "fcc512_oaml": lambda: ("pet-oam-l", wl.fcc_alloy(8, seed=33)),
        "si_partial_pbc": lambda: ("tiny", wl.Structure(*(lambda t: (t.positions, t.numbers, t.cell))(
            wl.si_diamond(2, seed=34)), (True, True, False))),
    }[case]()
    path = model_file(hname, 3)
    orc = po.load_oracle(path, torch.float64)
    ref = orc.predict([s])[0]
    res = mb.Predictor(path).predict(s.positions, s.numbers, s.cell, s.pbc, compute_stress=True)
    assert_close(res, ref["energy_f64"], ref["forces"], ref.get("stress"), s.n_atoms)


def test_gpu_many_species_matches_oracle(tmp_path):
    """A model with 130 species: the featurised rows' one-hot block spans two
    128-column blocks (x, y, z, r, 1 and 131 table rows), and the fused
    compress.0 weight has as many species columns; atoms use species on
    both sides of the block boundary."""
    path = str(tmp_path / "species130.gguf")
    wl.write_pet_gguf(path, wl.HYPERS["pet-mad-s"], atomic_numbers=np.arange(1, 131, dtype=np.int32), seed=41)
    s = wl.si_diamond(2, seed=41)
    rng = np.random.default_rng(41)
    numbers = rng.choice(np.array([1, 6, 8, 60, 118, 119, 122, 123, 124, 125, 129, 130], np.int32), s.n_atoms)
    s = wl.Structure(s.positions, numbers, s.cell, s.pbc)
    orc = po.load_oracle(path, torch.float64)
    ref = orc.predict([s])[0]
    res = mb.Predictor(path).predict(s.positions, s.numbers, s.cell, s.pbc, compute_stress=True)
    assert_close(res, ref["energy_f64"], ref["forces"], ref.get("stress"), s.n_atoms)


def test_gpu_molecule_batch_matches_single(model_file):
    """Batch == individual within 1e-5 (tests/test_pet.cpp:147-184)."""
    pred = mb.Predictor(model_file("tiny", 4))
    mols = wl.molecules(6, seed=41, n_min=3, n_max=40)
    batch = pred.predict_batch(mols)
    orc = po.load_oracle(model_file("tiny", 4), torch.float64)
    ref = orc.predict(mols)
    for k, m in enumerate(mols):
        single = pred.predict(m.positions, m.numbers)
        assert abs(batch[k].energy - single.energy) <= 1e-5 * max(1.0, abs(single.energy))
        np.testing.assert_allclose(batch[k].forces, single.forces, atol=1e-5)
        assert_close(batch[k], ref[k]["energy_f64"], ref[k]["forces"], None, m.n_atoms)


def test_gpu_edge_cases(model_file):
    path = model_file("tiny", 5)
    pred = mb.Predictor(path)
    orc = po.load_oracle(path, torch.float64)
    # isolated atom (test_pet.cpp:226-273)
    one = wl.Structure(np.zeros((1, 3), np.float32), np.array([6], np.int32))
    r = pred.predict(one.positions, one.numbers)
    assert_close(r, orc.predict([one])[0]["energy_f64"], np.zeros((1, 3)), None, 1)
    # a dimer and an isolated atom mixed in one batch
    dim = wl.Structure(np.array([[0, 0, 0], [1.1, 0.2, -0.1]], np.float32), np.array([1, 8], np.int32))
    out = pred.predict_batch([dim, one])
    ref = orc.predict([dim, one])
    assert_close(out[0], ref[0]["energy_f64"], ref[0]["forces"], None, 2)
    assert_close(out[1], ref[1]["energy_f64"], ref[1]["forces"], None, 1)
    # momentum conservation (test_pet_gradients.cpp:203-234)
    s = wl.water_box(96, seed=6)
    F = pred.predict(s.positions, s.numbers, s.cell).forces
    assert np.abs(F.sum(0)).max() < 1e-3
    # unknown species -> MLIPCPP_ERROR_COMPUTATION (pet_batch.cpp:156-163)
    with pytest.raises(mb.MLIPError) as ei:
        pred.predict(one.positions, np.array([150], np.int32))
    assert ei.value.code == mb.COMPUTATION


def test_gpu_options_semantics(model_file):
    """predict_with_options: gradient only when forces or stress are asked
    for; unrequested outputs are cleared (mlipcpp_api.cpp:569-593)."""
    pred = mb.Predictor(model_file("tiny", 6))
    s = wl.si_diamond(1, seed=7)
    full = pred.predict_with_options(s.positions, s.numbers, s.cell, None,
                                     mb.PredictOptions(True, True))
    assert full.has_forces() and full.has_stress()
    e_only = pred.predict_with_options(s.positions, s.numbers, s.cell, None,
                                       mb.PredictOptions(False, False))
    assert not e_only.has_forces() and not e_only.has_stress()
    assert abs(e_only.energy - full.energy) < 1e-4
    f_only = pred.predict_with_options(s.positions, s.numbers, s.cell, None, mb.PredictOptions(True, False))
    assert f_only.has_forces() and not f_only.has_stress()
    s_only = pred.predict_with_options(s.positions, s.numbers, s.cell, None, mb.PredictOptions(False, True))
    assert s_only.has_stress() and not s_only.has_forces()
    np.testing.assert_allclose(s_only.stress, full.stress, atol=1e-6)
    m = wl.molecules(1, seed=3)[0]
    r = pred.predict(m.positions, m.numbers, compute_stress=True)
    assert r.has_forces() and not r.has_stress()   # stress only for periodic cells
    assert pred.cutoff == pytest.approx(4.5)


def test_gpu_fd_stress_option(model_file):
    """fd_stress (mlipcpp_cpp.cpp:221-259) agrees with the virial within the
    reference's own FD tolerance (scripts/test_stress_fd.py:176).  The
    reference's virial treats the attention mask as constant, so the
    geometry keeps every edge out of the cutoff's transition region (first
    Si shell at 2.35 A, next at 3.84 A, cutoff 3.0 A, width 0.2 A) where the
    mask would otherwise move under strain."""
    pred = mb.Predictor(model_file("tiny", 2, cutoff=3.0, cutoff_width=0.2))
    s = wl.si_diamond(1, seed=3, jitter=0.03)
    an = pred.predict(s.positions, s.numbers, s.cell, compute_stress=True).stress
    fd = pred.predict(s.positions, s.numbers, s.cell, compute_stress=True, fd_stress=True).stress
    diff = np.abs(an - fd).max()
    assert diff < 5e-3 or diff / np.abs(fd).max() < 5e-2


def test_gpu_kernel_launches_counted(model_file):
    pred = mb.Predictor(model_file("tiny", 0))
    before = mb.kernel_launches()
    s = wl.si_diamond(1)
    pred.predict(s.positions, s.numbers, s.cell)
    assert mb.kernel_launches() > before


@pytest.mark.parametrize("mode", ["tf32", "f16"])
def test_gpu_tensor_core_matches_simt(mode, model_file, monkeypatch):
    """The 3xTF32 and 3xFP16 tcgen05 GEMM paths and the exact-fp32 SIMT path
    agree within the fp32 parity tolerances on the same inputs."""
    path = model_file("pet-mad-s", 8)
    s = wl.si_diamond(2, seed=8)
    monkeypatch.setenv("MLIPCPP_B200_GEMM", "simt")
    simt = mb.Predictor(path).predict(s.positions, s.numbers, s.cell, compute_stress=True)
    if mode == "tf32":
        monkeypatch.setenv("MLIPCPP_B200_GEMM", "tf32")
    else:
        monkeypatch.delenv("MLIPCPP_B200_GEMM")
    pred = mb.Predictor(path)
    pred.set_kernel_profiling(True)
    tc = pred.predict(s.positions, s.numbers, s.cell, compute_stress=True)
    st = pred.kernel_stats()
    assert st["gemm_f16" if mode == "f16" else "gemm_tc"]["launches"] > 0
    if mode == "tf32":
        assert st["gemm_f16"]["launches"] == 0
    assert_close(tc, simt.energy, simt.forces, simt.stress, s.n_atoms)


@pytest.mark.parametrize("hname,make,env", [
    ("pet-oam-l", lambda: [wl.fcc_alloy(6, seed=14)], {}),                       # split outputs, clusters of 4
    ("pet-mad-s", lambda: [wl.water_box(192, seed=14)], {}),                     # split outputs
    ("pet-mad-s", lambda: [wl.si_diamond(2, seed=14)], {"MLIPCPP_B200_CHAIN": "0"}),  # fp32 outputs
    ("pet-mad-s", lambda: wl.molecules(4, seed=14, n_min=2, n_max=60), {}),      # ragged, up to 60 tokens
    ("pet-mad-s", lambda: wl.molecules(6, seed=16, n_min=2, n_max=40), {}),      # ragged, 48-token kernels
    ("pet-mad-s", lambda: [wl.water_box(192, seed=15)], {"_cutoff": 6.5}),       # > 64 tokens: SIMT kernels
], ids=["oaml_fcc216", "mads_water192", "mads_si64_fp32", "mads_molecules", "mads_molecules48", "mads_wide"])
def test_gpu_mma_attention_matches_simt(hname, make, env, model_file, monkeypatch):
    """The tensor-core attention (register-resident split-fp16 mma.sync,
    forward and backward) and the SIMT thread-per-row kernels agree within
    the fp32 parity tolerances: energy, forces and stress, with split and
    fp32 outputs, ragged atoms and the fallback beyond 64 tokens."""
    env = dict(env)
    over = {"cutoff": env.pop("_cutoff")} if "_cutoff" in env else {}
    path = model_file(hname, 14, **over)
    systems = make()
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    monkeypatch.setenv("MLIPCPP_B200_ATTN", "rows")
    ref = mb.Predictor(path).predict_batch(systems, compute_stress=True)
    monkeypatch.delenv("MLIPCPP_B200_ATTN")  # default: tensor-core forward and backward
    pred = mb.Predictor(path)
    res = pred.predict_batch(systems, compute_stress=True)
    for s, r, q in zip(systems, res, ref):
        assert_close(r, q.energy, q.forces, q.stress if q.has_stress() else None, s.n_atoms)
    e_only = pred.predict_batch(systems, compute_forces=False)
    for s, r, q in zip(systems, e_only, ref):
        assert abs(r.energy - q.energy) / s.n_atoms <= TOL_E


# Stated tolerances of the reduced-precision mode (MLIPCPP_PRECISION_F16: dense
# layers multiply fp16 hi parts only, 11 significant bits per operand) against
# the fp32 path (about 4x the largest differences measured on these cases:
# 5.3e-4 eV/atom, 2.5e-3 eV/A, 1.8e-4 eV/A^3 for pet-oam-l).
TOL_E16, TOL_F16, TOL_S16 = 2e-3, 1e-2, 1e-3


@pytest.mark.parametrize("hname,make", [("pet-mad-s", lambda: wl.si_diamond(3, seed=13)),
                                        ("pet-oam-l", lambda: wl.fcc_alloy(6, seed=13))])
def test_gpu_reduced_precision_mode(hname, make, model_file):
    path = model_file(hname, 13)
    s = make()
    ref = mb.Predictor(path).predict(s.positions, s.numbers, s.cell, compute_stress=True)
    pred = mb.Predictor(path, mb.ModelOptions(precision=1))
    pred.set_kernel_profiling(True)
    res = pred.predict(s.positions, s.numbers, s.cell, compute_stress=True)
    assert pred.kernel_stats()["gemm_f16"]["launches"] > 0
    de = abs(res.energy - ref.energy) / s.n_atoms
    df = np.abs(res.forces - ref.forces).max()
    ds = np.abs(res.stress - ref.stress).max()
    print(f"{hname}: |dE|/N {de:.2e}  |dF| {df:.2e}  |dS| {ds:.2e}")
    assert de <= TOL_E16 and df <= TOL_F16 and ds <= TOL_S16


# ---- non-conservative heads (use_nc_forces) --------------------------------
@pytest.mark.parametrize("hname,make", [
    ("pet-oam-l", lambda: [wl.fcc_alloy(8, seed=61)]),
    ("pet-mad-s", lambda: [wl.water_box(192, seed=62)]),
    ("tiny", lambda: wl.molecules(5, seed=63, n_min=3, n_max=30)),
], ids=["fcc512_oaml", "water192_mads", "molecules5_tiny"])
def test_gpu_nc_heads_match_oracle(hname, make, model_file):
    """use_nc_forces: forces and stress from the non-conservative heads of
    both GNN layers (pet.cpp:742-784, 576-686), no gradients."""
    path = model_file(hname, 8, nc=True)
    systems = make()
    ref = po.load_oracle(path, torch.float64).predict(systems, compute_forces=False, compute_nc=True)
    pred = mb.Predictor(path)
    if len(systems) == 1:
        s = systems[0]
        res = [pred.predict_with_options(s.positions, s.numbers, s.cell, s.pbc,
                                         mb.PredictOptions(True, True, True))]
    else:
        res = pred.predict_batch(systems, compute_stress=True, use_nc_forces=True)
    for s, r, q in zip(systems, res, ref):
        assert_close(r, q["energy_f64"], q["forces"], q.get("stress"), s.n_atoms)
        assert r.has_stress() == ("stress" in q)


def test_gpu_nc_partial_heads(model_file):
    """A layer without heads contributes nothing; without a layer-0 head the
    property is absent (PETWeights::has_property, pet_types.h:247-250)."""
    s = wl.si_diamond(1, seed=64)
    only0 = model_file("tiny", 9, nc={"layers": (0,)})
    ref = po.load_oracle(only0, torch.float64).predict([s], compute_forces=False, compute_nc=True)[0]
    r = mb.Predictor(only0).predict_with_options(s.positions, s.numbers, s.cell, None,
                                                 mb.PredictOptions(True, True, True))
    assert_close(r, ref["energy_f64"], ref["forces"], ref["stress"], s.n_atoms)
    # forces only, and only on layer 1: no property, so no forces and no stress
    only1 = model_file("tiny", 9, nc={"layers": (1,), "props": ("nc_forces",)})
    r = mb.Predictor(only1).predict_with_options(s.positions, s.numbers, s.cell, None,
                                                 mb.PredictOptions(True, True, True))
    assert not r.has_forces() and not r.has_stress()


def test_gpu_nc_option_on_model_without_heads(model_file):
    """use_nc_forces on a model without the heads: energy only
    (pet.cpp:281-282 skips the heads, mlipcpp_api.cpp:572-577 no gradient)."""
    s = wl.si_diamond(1, seed=65)
    pred = mb.Predictor(model_file("tiny", 10))
    r = pred.predict_with_options(s.positions, s.numbers, s.cell, None, mb.PredictOptions(True, True, True))
    full = pred.predict(s.positions, s.numbers, s.cell, compute_stress=True)
    assert not r.has_forces() and not r.has_stress()
    assert abs(r.energy - full.energy) <= 1e-4


def test_gpu_nc_forces_without_stress_request(model_file):
    """compute_stress off clears the nc stress; compute_forces off clears the
    nc forces (mlipcpp_api.cpp:586-593)."""
    s = wl.si_diamond(1, seed=66)
    pred = mb.Predictor(model_file("tiny", 11, nc=True))
    r = pred.predict_with_options(s.positions, s.numbers, s.cell, None, mb.PredictOptions(True, False, True))
    assert r.has_forces() and not r.has_stress()
    r = pred.predict_with_options(s.positions, s.numbers, s.cell, None, mb.PredictOptions(False, True, True))
    assert r.has_stress() and not r.has_forces()
