"""ASE calculator over the GPU library, mirroring the reference's
MLIPCalculator (python/mlipcpp/ase.py:32-183): same constructor arguments,
properties and result conventions (stress in Voigt order, eV/A^3).  ASE is
optional; without it the class exists but constructing it raises
ImportError, as in the reference."""
from __future__ import annotations

from typing import Optional

import numpy as np

try:
    from ase.calculators.calculator import Calculator, all_changes
    ASE_AVAILABLE = True
except ImportError:
    ASE_AVAILABLE = False
    Calculator = object
    all_changes = []

from . import Backend, ModelOptions, Predictor

_BACKENDS = {"auto": Backend.Auto, "cpu": Backend.CPU, "cuda": Backend.CUDA, "hip": Backend.HIP,
             "metal": Backend.Metal, "vulkan": Backend.Vulkan, "sycl": Backend.SYCL, "cann": Backend.CANN}


class MLIPCalculator(Calculator):
    implemented_properties = ["energy", "forces", "stress"]
    default_parameters = {"backend": "auto", "cutoff_override": 0.0}

    def __init__(self, model_path: str, backend: str = "auto", cutoff_override: float = 0.0, **kwargs):
        if not ASE_AVAILABLE:
            raise ImportError("ASE is not installed")
        super().__init__(**kwargs)
        if backend.lower() not in _BACKENDS:
            raise ValueError(f"Unknown backend '{backend}'. Valid options: {', '.join(sorted(_BACKENDS))}")
        self.model_path = model_path
        self._predictor = Predictor(model_path, ModelOptions(backend=_BACKENDS[backend.lower()],
                                                             cutoff_override=cutoff_override))

    @property
    def cutoff(self) -> float:
        return self._predictor.cutoff

    @property
    def model_type(self) -> str:
        return self._predictor.model_type

    def calculate(self, atoms: Optional[object] = None, properties: list = ["energy"],
                  system_changes: list = all_changes):
        super().calculate(atoms, properties, system_changes)
        if atoms is None:
            atoms = self.atoms
        pbc = atoms.pbc
        cell = atoms.cell.array.astype(np.float32) if any(pbc) else None
        want_f, want_s = "forces" in properties, "stress" in properties
        r = self._predictor.predict(atoms.positions.astype(np.float32), atoms.numbers.astype(np.int32), cell=cell,
                                    pbc=tuple(bool(p) for p in pbc) if cell is not None else None,
                                    compute_forces=want_f or want_s, compute_stress=want_s)
        self.results["energy"] = float(r.energy)
        if want_f and r.has_forces():
            self.results["forces"] = np.array(r.forces)
        if want_s and r.has_stress():
            self.results["stress"] = np.array(r.stress)


def load_model(model_path: str, **kwargs) -> MLIPCalculator:
    return MLIPCalculator(model_path, **kwargs)
