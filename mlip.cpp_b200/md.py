"""Molecular dynamics with the state on the GPU.

The reference drives MD through ASE (python/mlipcpp/ase.py:123-183): every
step copies positions to the host, calls predict, and copies forces back.
Here positions, velocities and forces stay in device memory between steps
(torch tensors); a step is two half kicks and a drift around one
`Predictor.predict_device_forces` call, and only the potential energy (a
scalar) comes back to the host.  By default the neighbour list is rebuilt
every step on the GPU, as the reference does (well under 1% of a step on
large cells).  `Predictor.set_neighbor_skin(s)` keeps a cutoff + s list
across steps until an atom has moved s / 2 (wrapping into the cell does not
count); the steps then keep their shapes and replay the model from a CUDA
graph, which pays on small, launch-bound cells.  The extra pairs raise the
tokens per atom, so on dense systems whose atoms have more than 47 pairs
within cutoff + s the model leaves its fastest attention kernels, and a
kept list costs more than it saves.

Units: Angstrom, eV, amu, fs.  1 amu A^2 / fs^2 = 103.6427 eV.
"""
from __future__ import annotations

import numpy as np

EV_PER_AMU_A2_FS2 = 103.642696  # (1.66053907e-27 kg)(1e-10 m / 1e-15 s)^2 / 1.602176634e-19 J
KB_EV = 8.617333262e-5          # Boltzmann constant, eV/K

#: standard atomic masses (amu) by atomic number, enough for tests and
#: examples; others default to 2 Z
_MASSES = {1: 1.008, 6: 12.011, 7: 14.007, 8: 15.999, 14: 28.085, 26: 55.845, 28: 58.693, 29: 63.546}


def masses_of(numbers) -> np.ndarray:
    z = np.asarray(numbers, np.int64)
    return np.array([_MASSES.get(int(k), 2.0 * float(k)) for k in z], np.float64)


class VelocityVerlet:
    """NVE velocity-Verlet integrator.

    `force_fn(positions) -> (energy, forces)` takes and returns torch tensors
    on the integrator's device: positions [n, 3] float32, forces [n, 3]
    float32 (for the GPU library: ``predictor_forces(...)``).  The state is
    kept in float64; positions are wrapped into the cell along periodic
    axes before each force call."""

    def __init__(self, force_fn, positions, masses, dt_fs: float, cell=None, pbc=None, velocities=None,
                 device=None):
        import torch
        self.torch = torch
        self.force_fn = force_fn
        dev = device or ("cuda" if torch.cuda.is_available() else "cpu")
        self.x = torch.as_tensor(np.asarray(positions, np.float64), device=dev).clone()
        n = self.x.shape[0]
        self.m = torch.as_tensor(np.asarray(masses, np.float64), device=dev).reshape(n, 1)
        self.v = (torch.zeros_like(self.x) if velocities is None
                  else torch.as_tensor(np.asarray(velocities, np.float64), device=dev).clone())
        self.dt = float(dt_fs)
        self.cell = None if cell is None else torch.as_tensor(np.asarray(cell, np.float64).reshape(3, 3), device=dev)
        self.pbc = tuple(bool(p) for p in (pbc if pbc is not None else (True,) * 3)) if cell is not None else None
        self.inv_cell = None if self.cell is None else torch.linalg.inv(self.cell)
        self.energy, self.f = self._forces()

    def _wrap(self):
        if self.cell is None or not any(self.pbc):
            return
        frac = self.x @ self.inv_cell
        for k, p in enumerate(self.pbc):
            if p:
                frac[:, k] -= self.torch.floor(frac[:, k])
        self.x = frac @ self.cell

    def _forces(self):
        self._wrap()
        e, f = self.force_fn(self.x.to(self.torch.float32).contiguous())
        return float(e), f.to(self.torch.float64)

    def kinetic_energy(self) -> float:
        return float(0.5 * EV_PER_AMU_A2_FS2 * (self.m * self.v * self.v).sum())

    def temperature(self) -> float:
        return 2.0 * self.kinetic_energy() / (3.0 * self.x.shape[0] * KB_EV)

    def step(self, n: int = 1):
        """Advance n steps; returns the list of (potential, kinetic) energies."""
        out = []
        a = 1.0 / (EV_PER_AMU_A2_FS2 * self.m)
        for _ in range(n):
            self.v += (0.5 * self.dt) * self.f * a
            self.x += self.dt * self.v
            self.energy, self.f = self._forces()
            self.v += (0.5 * self.dt) * self.f * a
            out.append((self.energy, self.kinetic_energy()))
        return out


def maxwell_boltzmann(masses, temperature_k: float, seed: int = 0) -> np.ndarray:
    """Velocities (A/fs) at the given temperature with zero total momentum."""
    rng = np.random.default_rng(seed)
    m = np.asarray(masses, np.float64).reshape(-1, 1)
    v = rng.standard_normal((m.shape[0], 3)) * np.sqrt(KB_EV * temperature_k / (EV_PER_AMU_A2_FS2 * m))
    v -= (m * v).sum(0) / m.sum()
    return v


def predictor_forces(predictor, numbers, cell=None, pbc=None):
    """force_fn backed by the GPU library: positions and forces stay on the
    device (mlipcpp_b200_predict_device_forces)."""
    import torch
    z = np.asarray(numbers, np.int32)
    buf = {}

    def run(x):
        n = x.shape[0]
        f = buf.get(n)
        if f is None:
            f = buf[n] = torch.empty((n, 3), dtype=torch.float32, device=x.device)
        e, _ = predictor.predict_device_forces(x.data_ptr(), n, z, cell, pbc, d_forces=f.data_ptr())
        return e, f
    return run
