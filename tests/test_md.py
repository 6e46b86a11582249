"""Velocity-Verlet driver (mlip.cpp_b200/md.py) on CPU with an analytic
force field, and the ASE adapter's behaviour without ASE."""
import numpy as np
import pytest
import torch

from mlipcpp_b200 import md


def _springs(k=2.0):
    """Pair springs between consecutive atoms of a chain (float32 in/out, like the library)."""
    def run(x):
        x64 = x.to(torch.float64)
        d = x64[1:] - x64[:-1]
        e = 0.5 * k * (d * d).sum()
        f = torch.zeros_like(x64)
        f[1:] -= k * d
        f[:-1] += k * d
        return float(e), f.to(torch.float32)
    return run


def _chain(n=16, seed=0):
    rng = np.random.default_rng(seed)
    x = np.stack([np.arange(n) * 1.5, np.zeros(n), np.zeros(n)], 1) + 0.1 * rng.standard_normal((n, 3))
    return x, np.full(n, 12.011)


def test_energy_conserved_and_reversible():
    x0, m = _chain()
    v0 = md.maxwell_boltzmann(m, 300.0, seed=1)
    vv = md.VelocityVerlet(_springs(), x0, m, 0.5, velocities=v0, device="cpu")
    e0 = vv.energy + vv.kinetic_energy()
    traj = vv.step(400)
    tot = np.array([p + k for p, k in traj])
    assert np.max(np.abs(tot - e0)) < 2e-3 * max(1.0, abs(e0))
    # time reversal: flip velocities and run back to the start (float32 forces)
    vv.v = -vv.v
    vv.step(400)
    assert np.abs(vv.x.numpy() - x0).max() < 1e-3


def test_maxwell_boltzmann_momentum_and_temperature():
    m = np.full(20000, 28.085)
    v = md.maxwell_boltzmann(m, 500.0, seed=2)
    assert np.abs((m[:, None] * v).sum(0)).max() < 1e-9
    ke = 0.5 * md.EV_PER_AMU_A2_FS2 * (m[:, None] * v * v).sum()
    t = 2 * ke / (3 * len(m) * md.KB_EV)
    assert t == pytest.approx(500.0, rel=0.03)


def test_wrapping_into_periodic_cell():
    x0 = np.array([[-0.5, 1.0, 11.0], [3.0, -2.0, 4.0]])
    cell = np.diag([10.0, 10.0, 10.0])
    seen = {}

    def zero(x):
        seen["x"] = x.clone()
        return 0.0, torch.zeros_like(x)
    md.VelocityVerlet(zero, x0, [1.0, 1.0], 1.0, cell=cell, pbc=(True, True, False), device="cpu")
    np.testing.assert_allclose(seen["x"].numpy(), [[9.5, 1.0, 11.0], [3.0, 8.0, 4.0]], atol=1e-5)


def test_ase_adapter_without_ase():
    from mlipcpp_b200 import ase as mase
    if mase.ASE_AVAILABLE:
        pytest.skip("ASE installed")
    with pytest.raises(ImportError):
        mase.MLIPCalculator("model.gguf")
