"""Spatial domain decomposition with the GPU evaluator (C ABI
mlipcpp_b200_predict_local): 2 and 8 domains run one after another on one
GPU and summed must equal the whole-cell evaluation.  Tolerances are the
fp32 parity bar (|dE|/N <= 1e-5 eV, |dF| <= 1e-4 eV/A, |dsigma| <= 1e-4 eV/A^3)."""
import numpy as np
import pytest
import torch

import mlipcpp_b200 as mb
from mlipcpp_b200 import domain as dd
from mlipcpp_b200 import workloads as wl
from oracle import pet_oracle as po

pytestmark = pytest.mark.gpu
TOL_E, TOL_F, TOL_S = 1e-5, 1e-4, 1e-4


def run_domains(pred, s, cutoff, n_dom):
    run = dd.DomainRunner(dd.predictor_eval(pred), s.numbers, s.cell, cutoff, emulate=n_dom)
    e, F, vir = run.step(torch.from_numpy(s.positions).cuda())
    return e, F.cpu().numpy(), run.stress(vir)


@pytest.mark.parametrize("n_dom", [2, 8])
def test_domains_match_whole_cell(n_dom, model_file):
    s = wl.si_diamond(6, seed=41)
    pred = mb.Predictor(model_file("pet-mad-s", 5))
    full = pred.predict(s.positions, s.numbers, s.cell, s.pbc, compute_stress=True)
    e, F, S = run_domains(pred, s, 4.5, n_dom)
    assert abs(e - full.energy) / s.n_atoms <= TOL_E
    assert np.abs(F - full.forces).max() <= TOL_F
    assert np.abs(S - full.stress).max() <= TOL_S


def test_domains_match_oracle(model_file):
    path = model_file("tiny", 6, cutoff=3.0, cutoff_width=0.5)
    s = wl.si_diamond(4, seed=42)
    ref = po.load_oracle(path, torch.float64).predict([s])[0]
    e, F, S = run_domains(mb.Predictor(path), s, 3.0, 8)
    assert abs(e - ref["energy_f64"]) / s.n_atoms <= TOL_E
    assert np.abs(F - ref["forces"]).max() <= TOL_F
    assert np.abs(S - ref["stress"]).max() <= TOL_S
