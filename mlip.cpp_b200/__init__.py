"""B200 backend for mlip.cpp's PET energy / force / stress path.

Python mirror of mlip.cpp's ``mlipcpp`` module (src/api/python/
mlipcpp_bindings.cpp) over the C ABI of ``libmlipcpp_b200.so`` (declared in
include/mlipcpp.h and include/mlipcpp_b200.h).  The same names, argument
meanings and error behaviour: ``Predictor(path).predict(positions,
atomic_numbers, cell=None, pbc=None, compute_forces=True,
compute_stress=False, fd_stress=False)`` returns a ``Result`` with
``energy`` (eV), ``forces`` [n, 3] (eV/A) and ``stress`` [6] (Voigt, eV/A^3).

All arithmetic runs in the CUDA library; there is no CPU fallback.  Loading
fails loudly when the library has not been built (``make -C mlip.cpp_b200``).
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
# MLIPCPP_B200_LIB selects another build of the library (e.g. a variant).
LIB_PATH = os.environ.get("MLIPCPP_B200_LIB") or os.path.join(HERE, "libmlipcpp_b200.so")

# mlipcpp_error_t (include/mlipcpp.h)
OK, INVALID_HANDLE, NULL_POINTER, MODEL_NOT_LOADED, OUT_OF_MEMORY, IO_ERROR, COMPUTATION, \
    INVALID_PARAMETER, BACKEND, UNSUPPORTED = range(10)
INTERNAL = 255


class Backend:
    """mlipcpp_backend_t."""
    Auto, CPU, CUDA, HIP, Metal, Vulkan, SYCL, CANN, WebGPU = range(9)


class MLIPError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


class _System(ctypes.Structure):
    _fields_ = [("n_atoms", ctypes.c_int32), ("positions", ctypes.c_void_p),
                ("atomic_numbers", ctypes.c_void_p), ("cell", ctypes.c_void_p),
                ("pbc", ctypes.c_void_p)]


class _ModelOptions(ctypes.Structure):
    _fields_ = [("backend", ctypes.c_int), ("precision", ctypes.c_int),
                ("cutoff_override", ctypes.c_float)]


class _PredictOptions(ctypes.Structure):
    _fields_ = [("compute_forces", ctypes.c_bool), ("compute_stress", ctypes.c_bool),
                ("use_nc_forces", ctypes.c_bool)]


_lib = None


def lib() -> ctypes.CDLL:
    """The loaded C library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} not built; run `make -C {HERE}` (no CPU fallback exists)")
    L = ctypes.CDLL(LIB_PATH)
    vp, i32, i64, f32, b = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_bool
    sig = {
        "mlipcpp_version": (ctypes.c_char_p, []),
        "mlipcpp_error_string": (ctypes.c_char_p, [ctypes.c_int]),
        "mlipcpp_get_last_error": (ctypes.c_char_p, []),
        "mlipcpp_set_backend": (None, [ctypes.c_int]),
        "mlipcpp_get_backend_name": (ctypes.c_char_p, []),
        "mlipcpp_backend_is_gpu": (b, []),
        "mlipcpp_is_backend_available": (b, [ctypes.c_int]),
        "mlipcpp_suppress_logging": (None, []),
        "mlipcpp_model_options_default": (ctypes.c_int, [vp]),
        "mlipcpp_model_create": (vp, [vp]),
        "mlipcpp_model_load": (ctypes.c_int, [vp, ctypes.c_char_p]),
        "mlipcpp_model_free": (None, [vp]),
        "mlipcpp_model_get_cutoff": (ctypes.c_int, [vp, vp]),
        "mlipcpp_predict_options_default": (ctypes.c_int, [vp]),
        "mlipcpp_predict": (ctypes.c_int, [vp, vp, b, vp]),
        "mlipcpp_predict_ptr": (ctypes.c_int, [vp, i32, vp, vp, vp, vp, b, vp]),
        "mlipcpp_predict_with_options": (ctypes.c_int, [vp, vp, vp, vp]),
        "mlipcpp_predict_ptr_with_options": (ctypes.c_int, [vp, i32, vp, vp, vp, vp, vp, vp]),
        "mlipcpp_result_get_energy": (ctypes.c_int, [vp, vp]),
        "mlipcpp_result_get_forces": (ctypes.c_int, [vp, vp, i32]),
        "mlipcpp_result_get_stress": (ctypes.c_int, [vp, vp]),
        "mlipcpp_result_n_atoms": (ctypes.c_int, [vp, vp]),
        "mlipcpp_result_has_forces": (ctypes.c_int, [vp, vp]),
        "mlipcpp_result_has_stress": (ctypes.c_int, [vp, vp]),
        "mlipcpp_result_free": (None, [vp]),
        "mlipcpp_predict_batch": (ctypes.c_int, [vp, i32, vp, vp, vp]),
        "mlipcpp_b200_predict_packed": (ctypes.c_int, [vp, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp]),
        "mlipcpp_b200_predict_device": (ctypes.c_int, [vp, i32, vp, vp, vp, vp, vp, b, vp]),
        "mlipcpp_b200_predict_device_forces": (ctypes.c_int, [vp, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp]),
        "mlipcpp_b200_set_neighbor_skin": (ctypes.c_int, [vp, f32]),
        "mlipcpp_b200_neighbor_builds": (i64, [vp]),
        "mlipcpp_b200_set_timing": (ctypes.c_int, [vp, b]),
        "mlipcpp_b200_last_timings": (ctypes.c_int, [vp, vp]),
        "mlipcpp_b200_last_shape": (ctypes.c_int, [vp, vp]),
        "mlipcpp_b200_neighbor_list": (i64, [i32, vp, vp, vp, f32, i64, vp, vp, vp, vp, vp]),
        "mlipcpp_b200_kernel_launches": (i64, []),
        "mlipcpp_b200_device_allocations": (i64, []),
        "mlipcpp_b200_set_wait_bound_ns": (ctypes.c_int, [ctypes.c_uint64]),
        "mlipcpp_b200_inject_gemm_stall": (ctypes.c_int, []),
        "mlipcpp_b200_set_device": (ctypes.c_int, [i32]),
        "mlipcpp_b200_domain_create": (vp, [vp, vp, vp, i32, f32, vp]),
        "mlipcpp_b200_domain_free": (None, [vp]),
        "mlipcpp_b200_domain_set_atoms": (ctypes.c_int, [vp, i32, vp]),
        "mlipcpp_b200_domain_step": (ctypes.c_int, [vp, vp, vp, b, vp, vp]),
        "mlipcpp_b200_domain_stats": (ctypes.c_int, [vp, vp]),
        "mlipcpp_b200_set_kernel_profiling": (ctypes.c_int, [vp, b]),
        "mlipcpp_b200_kernel_stats": (ctypes.c_int, [vp, vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _check(code: int):
    if code != OK:
        msg = lib().mlipcpp_get_last_error() or lib().mlipcpp_error_string(code)
        raise MLIPError(code, msg.decode())


class LogLevel:
    """mlipcpp.LogLevel (logging is a no-op in this backend)."""
    Trace, Debug, Info, Warn, Error, Off = range(6)


def set_log_level(level) -> None:
    """Accepted for compatibility; the library does not log."""
    lib().mlipcpp_suppress_logging()


def enable_logging() -> None:
    """Accepted for compatibility; the library does not log."""


def set_backend(backend: int) -> None:
    """Global backend for Predictors created afterwards (CUDA / Auto only)."""
    lib().mlipcpp_set_backend(int(backend))


def get_backend_name() -> str:
    return lib().mlipcpp_get_backend_name().decode()


def backend_is_gpu() -> bool:
    return bool(lib().mlipcpp_backend_is_gpu())


def is_backend_available(backend: int) -> bool:
    return bool(lib().mlipcpp_is_backend_available(int(backend)))


def load_model(path: str, **kwargs) -> "Predictor":
    """mlipcpp.load_model: a Predictor with ModelOptions(**kwargs)."""
    return Predictor(path, ModelOptions(**kwargs))


def set_device(device: int):
    """CUDA device for Predictors created afterwards."""
    _check(lib().mlipcpp_b200_set_device(int(device)))


def version() -> str:
    return lib().mlipcpp_version().decode()


def kernel_launches() -> int:
    """Kernels this library has launched in this process."""
    return int(lib().mlipcpp_b200_kernel_launches())


@dataclass
class ModelOptions:
    backend: int = Backend.Auto
    cutoff_override: float = 0.0
    precision: int = 0


@dataclass
class PredictOptions:
    compute_forces: bool = True
    compute_stress: bool = False
    use_nc_forces: bool = False
    fd_stress: bool = False


@dataclass
class Result:
    energy: float = 0.0
    forces: np.ndarray = field(default_factory=lambda: np.zeros((0, 3), np.float32))
    stress: np.ndarray = field(default_factory=lambda: np.zeros(0, np.float32))
    _has_forces: bool = False
    _has_stress: bool = False

    def has_forces(self) -> bool:
        return self._has_forces

    def has_stress(self) -> bool:
        return self._has_stress


@dataclass
class PackedResult:
    """Results of Predictor.predict_packed: energies [n_systems], forces
    [sum n, 3] in the input's packed order, stress [n_systems, 6] (Voigt)."""
    energies: np.ndarray
    forces: np.ndarray | None = None
    stress: np.ndarray | None = None


def _read_result(handle, n_atoms: int, free: bool = True) -> Result:
    L = lib()
    try:
        e = ctypes.c_float()
        _check(L.mlipcpp_result_get_energy(handle, ctypes.byref(e)))
        hf, hs = ctypes.c_bool(), ctypes.c_bool()
        _check(L.mlipcpp_result_has_forces(handle, ctypes.byref(hf)))
        _check(L.mlipcpp_result_has_stress(handle, ctypes.byref(hs)))
        r = Result(energy=float(e.value), _has_forces=hf.value, _has_stress=hs.value)
        if hf.value:
            f = np.zeros((n_atoms, 3), np.float32)
            _check(L.mlipcpp_result_get_forces(handle, f.ctypes.data, n_atoms))
            r.forces = f
        if hs.value:
            s = np.zeros(6, np.float32)
            _check(L.mlipcpp_result_get_stress(handle, s.ctypes.data))
            r.stress = s
        return r
    finally:
        if free:
            L.mlipcpp_result_free(handle)


def _as_system(positions, atomic_numbers, cell=None, pbc=None):
    pos = np.ascontiguousarray(positions, dtype=np.float32).reshape(-1, 3)
    z = np.ascontiguousarray(atomic_numbers, dtype=np.int32).reshape(-1)
    if z.shape[0] != pos.shape[0]:
        raise RuntimeError("positions and atomic_numbers must have same length")
    c = None if cell is None else np.ascontiguousarray(cell, dtype=np.float32).reshape(9)
    p = None
    if c is not None:
        p = np.asarray([True, True, True] if pbc is None else [bool(x) for x in pbc], dtype=np.bool_)
    keep = (pos, z, c, p)
    s = _System(pos.shape[0], pos.ctypes.data, z.ctypes.data,
                None if c is None else c.ctypes.data, None if p is None else p.ctypes.data)
    return s, keep


def _strain(pos, cell, eta):
    """Symmetric Voigt strain of cell rows and positions
    (src/api/cpp/mlipcpp_cpp.cpp:174-210)."""
    e = np.array([[1.0 + eta[0], 0.5 * eta[5], 0.5 * eta[4]],
                  [0.5 * eta[5], 1.0 + eta[1], 0.5 * eta[3]],
                  [0.5 * eta[4], 0.5 * eta[3], 1.0 + eta[2]]])
    c = (np.asarray(cell, np.float64).reshape(3, 3) @ e.T).astype(np.float32)
    p = (np.asarray(pos, np.float64).reshape(-1, 3) @ e.T).astype(np.float32)
    return p, c


class Predictor:
    """mlipcpp.Predictor (src/api/python/mlipcpp_bindings.cpp:97-180)."""

    def __init__(self, path: str, options: ModelOptions | None = None):
        L = lib()
        options = options or ModelOptions()
        o = _ModelOptions()
        L.mlipcpp_model_options_default(ctypes.byref(o))
        o.backend = int(options.backend)
        o.precision = int(options.precision)
        o.cutoff_override = float(options.cutoff_override)
        self._h = L.mlipcpp_model_create(ctypes.byref(o))
        if not self._h:
            _check(INTERNAL)
        code = L.mlipcpp_model_load(self._h, os.fsencode(path))
        if code != OK:
            msg = L.mlipcpp_get_last_error()
            L.mlipcpp_model_free(self._h)
            self._h = None
            raise MLIPError(code, (msg or b"load failed").decode())

    def __del__(self):
        h = getattr(self, "_h", None)
        if h and lib is not None:
            try:
                lib().mlipcpp_model_free(h)
            except Exception:
                pass
            self._h = None

    @property
    def cutoff(self) -> float:
        c = ctypes.c_float()
        _check(lib().mlipcpp_model_get_cutoff(self._h, ctypes.byref(c)))
        return float(c.value)

    @property
    def model_type(self) -> str:
        return "PET"

    def predict(self, positions, atomic_numbers, cell=None, pbc=None, compute_forces=True,
                compute_stress=False, fd_stress=False) -> Result:
        opts = PredictOptions(compute_forces=compute_forces or compute_stress,
                              compute_stress=compute_stress, fd_stress=fd_stress)
        return self.predict_with_options(positions, atomic_numbers, cell, pbc, opts)

    def predict_with_options(self, positions, atomic_numbers, cell=None, pbc=None,
                             options: PredictOptions | None = None) -> Result:
        options = options or PredictOptions()
        s, keep = _as_system(positions, atomic_numbers, cell, pbc)
        po = _PredictOptions(options.compute_forces, options.compute_stress, options.use_nc_forces)
        h = ctypes.c_void_p()
        _check(lib().mlipcpp_predict_with_options(self._h, ctypes.byref(s), ctypes.byref(po),
                                                  ctypes.byref(h)))
        r = _read_result(h, s.n_atoms)
        if options.compute_stress and options.fd_stress and cell is not None:
            r.stress = self._fd_stress(keep[0], keep[1], cell, keep[3])
            r._has_stress = True
        return r

    def _fd_stress(self, pos, z, cell, pbc, delta=5e-3):
        """4th-order central difference of the energy under Voigt strain
        (src/api/cpp/mlipcpp_cpp.cpp:221-259)."""
        m = np.asarray(cell, np.float64).reshape(3, 3)
        vol = abs(np.linalg.det(m))
        if vol < 1e-10:
            return np.zeros(0, np.float32)
        out = np.zeros(6, np.float32)
        for k in range(6):
            e = {}
            for sc in (1, -1, 2, -2):
                eta = np.zeros(6, np.float32)
                eta[k] = np.float32(delta * sc)
                p, c = _strain(pos, m, eta.astype(np.float64))
                e[sc] = float(self.predict_with_options(
                    p, z, c, pbc, PredictOptions(compute_forces=False)).energy)
            out[k] = (8.0 * (e[1] - e[-1]) - (e[2] - e[-2])) / (12.0 * vol * delta)
        return out

    def predict_batch(self, systems, compute_forces=True, compute_stress=False,
                      use_nc_forces=False) -> list[Result]:
        """Batched prediction (extension; PETModel::predict_batch in the
        reference).  `systems`: iterable of objects with positions, numbers,
        cell and pbc attributes, or (positions, numbers[, cell[, pbc]]).
        use_nc_forces: forces and stress from the model's non-conservative
        heads instead of gradients, as in PredictOptions."""
        structs, keeps, ns = [], [], []
        for sy in systems:
            if hasattr(sy, "positions"):
                args = (sy.positions, sy.numbers, getattr(sy, "cell", None), getattr(sy, "pbc", None))
            else:
                args = tuple(sy) + (None,) * (4 - len(sy))
            s, keep = _as_system(*args)
            structs.append(s)
            keeps.append(keep)
            ns.append(s.n_atoms)
        n = len(structs)
        arr = (_System * max(n, 1))(*structs)
        handles = (ctypes.c_void_p * max(n, 1))()
        po = _PredictOptions(compute_forces or compute_stress, compute_stress, use_nc_forces)
        _check(lib().mlipcpp_predict_batch(self._h, n, arr, ctypes.byref(po), handles))
        return [_read_result(handles[k], ns[k]) for k in range(n)]

    def predict_packed(self, positions, numbers, n_atoms, cells=None, pbc=None, compute_forces=True,
                       compute_stress=False, use_nc_forces=False) -> "PackedResult":
        """Batched prediction from packed arrays (mlipcpp_b200_predict_packed):
        structure k is the next n_atoms[k] rows of `positions` [sum n, 3] and
        entries of `numbers`; `cells` [n_systems, 3, 3] (None: all
        non-periodic) and `pbc` [n_systems, 3].  Returns energies
        [n_systems], forces [sum n, 3] (None unless compute_forces) and
        stress [n_systems, 6] (None unless compute_stress) in one call,
        without a result object per structure."""
        counts = np.ascontiguousarray(n_atoms, np.int32).reshape(-1)
        pos = np.ascontiguousarray(positions, np.float32).reshape(-1, 3)
        z = np.ascontiguousarray(numbers, np.int32).reshape(-1)
        ns = counts.shape[0]
        if z.shape[0] != pos.shape[0] or int(counts.sum(dtype=np.int64)) != pos.shape[0]:
            raise RuntimeError("positions, numbers and n_atoms do not describe the same atoms")
        c = None if cells is None else np.ascontiguousarray(cells, np.float32).reshape(ns, 9)
        p = None if pbc is None else np.ascontiguousarray(pbc, np.bool_).reshape(ns, 3)
        e = np.empty(ns, np.float32)
        f = np.empty((pos.shape[0], 3), np.float32) if compute_forces else None
        st = np.empty((ns, 6), np.float32) if compute_stress else None
        po = _PredictOptions(compute_forces, compute_stress, use_nc_forces)
        ptr = lambda a: None if a is None else a.ctypes.data  # noqa: E731
        _check(lib().mlipcpp_b200_predict_packed(self._h, ns, counts.ctypes.data, pos.ctypes.data, z.ctypes.data,
                                                 ptr(c), ptr(p), ctypes.byref(po), e.ctypes.data, ptr(f), ptr(st)))
        return PackedResult(e, f, st)

    def predict_device(self, d_positions: int, n_atoms: int, atomic_numbers, cell=None, pbc=None,
                       compute_forces=True, compute_stress=False, copy_forces=True,
                       use_nc_forces=False) -> Result:
        """Positions already in device memory (`d_positions`: device pointer
        to [3n] float32)."""
        z = np.ascontiguousarray(atomic_numbers, dtype=np.int32)
        c = None if cell is None else np.ascontiguousarray(cell, dtype=np.float32).reshape(9)
        p = None if c is None else np.asarray([True] * 3 if pbc is None else list(pbc), np.bool_)
        po = _PredictOptions(compute_forces or compute_stress, compute_stress, use_nc_forces)
        h = ctypes.c_void_p()
        _check(lib().mlipcpp_b200_predict_device(
            self._h, n_atoms, ctypes.c_void_p(d_positions), z.ctypes.data,
            None if c is None else c.ctypes.data, None if p is None else p.ctypes.data,
            ctypes.byref(po), bool(copy_forces), ctypes.byref(h)))
        return _read_result(h, n_atoms if copy_forces else 0) if copy_forces else \
            _read_result_no_forces(h)

    def predict_device_forces(self, d_positions: int, n_atoms: int, atomic_numbers, cell=None, pbc=None,
                              d_forces: int = 0, compute_stress=False, use_nc_forces=False):
        """Positions and forces in device memory (`d_positions`, `d_forces`:
        device pointers to [3n] float32; d_forces may be 0).  Returns
        (energy, stress [6] or None)."""
        z = np.ascontiguousarray(atomic_numbers, dtype=np.int32)
        c = None if cell is None else np.ascontiguousarray(cell, dtype=np.float32).reshape(9)
        p = None if c is None else np.asarray([True] * 3 if pbc is None else list(pbc), np.bool_)
        po = _PredictOptions(True, bool(compute_stress), bool(use_nc_forces))
        e = ctypes.c_double()
        st = np.zeros(6, np.float32)
        hs = ctypes.c_bool(False)
        _check(lib().mlipcpp_b200_predict_device_forces(
            self._h, int(n_atoms), ctypes.c_void_p(d_positions), z.ctypes.data,
            None if c is None else c.ctypes.data, None if p is None else p.ctypes.data, ctypes.byref(po),
            ctypes.c_void_p(d_forces) if d_forces else None, ctypes.byref(e), st.ctypes.data, ctypes.byref(hs)))
        return float(e.value), (st if hs.value else None)

    def set_neighbor_skin(self, skin: float):
        """Keep a Verlet list of cutoff + skin across single-structure calls
        (mlipcpp_b200_set_neighbor_skin); 0 rebuilds every call."""
        _check(lib().mlipcpp_b200_set_neighbor_skin(self._h, float(skin)))

    def neighbor_builds(self) -> int:
        """Neighbour lists built by this model so far."""
        return int(lib().mlipcpp_b200_neighbor_builds(self._h))

    def set_timing(self, on: bool = True):
        _check(lib().mlipcpp_b200_set_timing(self._h, bool(on)))

    def last_timings(self) -> dict:
        t = np.zeros(8, np.float32)
        _check(lib().mlipcpp_b200_last_timings(self._h, t.ctypes.data))
        keys = ["h2d", "neighbor_list", "prep", "forward", "backward", "reduce", "d2h", "total"]
        return {k: float(v) for k, v in zip(keys, t)}

    def set_kernel_profiling(self, on: bool = True):
        _check(lib().mlipcpp_b200_set_kernel_profiling(self._h, bool(on)))

    def kernel_stats(self) -> dict:
        """Per kernel class: launches, ms, algorithmic flops and bytes."""
        a = np.zeros(24, np.float64)
        _check(lib().mlipcpp_b200_kernel_stats(self._h, a.ctypes.data))
        names = ["gemm_tc", "gemm_simt", "attention", "neighbor_list", "other", "gemm_f16"]
        return {n: {"launches": int(a[4 * k]), "ms": float(a[4 * k + 1]),
                    "flops": float(a[4 * k + 2]), "bytes": float(a[4 * k + 3])}
                for k, n in enumerate(names)}

    def last_shape(self) -> dict:
        s = np.zeros(4, np.int64)
        _check(lib().mlipcpp_b200_last_shape(self._h, s.ctypes.data))
        return {"atoms": int(s[0]), "edges": int(s[1]), "max_neighbors": int(s[2]),
                "device_mib": int(s[3])}


def _read_result_no_forces(handle) -> Result:
    L = lib()
    try:
        e = ctypes.c_float()
        _check(L.mlipcpp_result_get_energy(handle, ctypes.byref(e)))
        hs = ctypes.c_bool()
        _check(L.mlipcpp_result_has_stress(handle, ctypes.byref(hs)))
        r = Result(energy=float(e.value), _has_stress=hs.value)
        if hs.value:
            s = np.zeros(6, np.float32)
            _check(L.mlipcpp_result_get_stress(handle, s.ctypes.data))
            r.stress = s
        return r
    finally:
        L.mlipcpp_result_free(handle)


def neighbor_list(positions, cell=None, pbc=None, cutoff: float = 4.5) -> dict:
    """GPU neighbour list with the reference NeighborList fields
    (include/mlipcpp/neighbor_list.h:9-19), bit-identical to it."""
    L = lib()
    pos = np.ascontiguousarray(positions, dtype=np.float32).reshape(-1, 3)
    c = None if cell is None else np.ascontiguousarray(cell, dtype=np.float32).reshape(9)
    p = None if (c is None or pbc is None) else np.asarray([bool(x) for x in pbc], np.bool_)
    args = (pos.shape[0], pos.ctypes.data, None if c is None else c.ctypes.data,
            None if p is None else p.ctypes.data, float(cutoff))
    m = L.mlipcpp_b200_neighbor_list(*args, 0, None, None, None, None, None)
    if m < 0:
        _check(int(-m))
    out = dict(centers=np.zeros(m, np.int32), neighbors=np.zeros(m, np.int32),
               cell_shifts=np.zeros((m, 3), np.int32), edge_vectors=np.zeros((m, 3), np.float32),
               distances=np.zeros(m, np.float32))
    m2 = L.mlipcpp_b200_neighbor_list(*args, m, out["centers"].ctypes.data,
                                      out["neighbors"].ctypes.data, out["cell_shifts"].ctypes.data,
                                      out["edge_vectors"].ctypes.data, out["distances"].ctypes.data)
    if m2 < 0:
        _check(int(-m2))
    out["n_atoms"] = pos.shape[0]
    return out


def __getattr__(name):
    if name == "__version__":
        return version()
    raise AttributeError(name)
