"""TEST INFRASTRUCTURE -- ctypes front end for the neighbour-list checkers.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this.

* ``build_oracle``    -> oracle/_build/libnl_oracle.so (C restatement, nl_oracle.c)
* ``build_reference`` -> oracle/_ref/libnl_ref.so (the reference's own
  src/core/neighbor_list.cpp + system.cpp, compiled by oracle/Makefile)

Both return the reference's ``NeighborList`` fields
(include/mlipcpp/neighbor_list.h:9-19) as numpy arrays in the reference's
enumeration order.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIBS: dict[str, ctypes.CDLL] = {}


def _load(kind: str) -> ctypes.CDLL:
    if kind in _LIBS:
        return _LIBS[kind]
    path = os.path.join(HERE, "_build", "libnl_oracle.so") if kind == "oracle" else \
        os.path.join(HERE, "_ref", "libnl_ref.so")
    if not os.path.exists(path):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    if not os.path.exists(path):
        raise FileNotFoundError(path)
    lib = ctypes.CDLL(path)
    fn = getattr(lib, "nlo_build" if kind == "oracle" else "nlref_build")
    fn.restype = ctypes.c_int64
    fn.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_int64] + \
        [ctypes.c_void_p] * 5
    inv = getattr(lib, "nlo_cell_inverse" if kind == "oracle" else "nlref_cell_inverse")
    inv.restype = None
    inv.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    _LIBS[kind] = lib
    return lib


def reference_available() -> bool:
    try:
        _load("ref")
        return True
    except (OSError, subprocess.CalledProcessError):
        return False


def _ptr(a):
    return None if a is None else a.ctypes.data


def _build(kind, positions, cell=None, pbc=None, cutoff=4.5, full_list=True,
           self_interaction=False):
    lib = _load(kind)
    fn = lib.nlo_build if kind == "oracle" else lib.nlref_build
    pos = np.ascontiguousarray(positions, dtype=np.float32).reshape(-1, 3)
    n = pos.shape[0]
    c = None if cell is None else np.ascontiguousarray(cell, dtype=np.float32).reshape(9)
    p = None if (cell is None or pbc is None) else np.asarray([int(bool(x)) for x in pbc], np.int32)
    m = fn(n, _ptr(pos), _ptr(c), _ptr(p), float(cutoff), int(full_list), int(self_interaction),
           0, None, None, None, None, None)
    out = dict(centers=np.zeros(m, np.int32), neighbors=np.zeros(m, np.int32),
               cell_shifts=np.zeros((m, 3), np.int32), edge_vectors=np.zeros((m, 3), np.float32),
               distances=np.zeros(m, np.float32))
    m2 = fn(n, _ptr(pos), _ptr(c), _ptr(p), float(cutoff), int(full_list), int(self_interaction),
            m, _ptr(out["centers"]), _ptr(out["neighbors"]), _ptr(out["cell_shifts"]),
            _ptr(out["edge_vectors"]), _ptr(out["distances"]))
    assert m2 == m
    out["n_atoms"] = n
    return out


def build_oracle(positions, cell=None, pbc=None, cutoff=4.5, full_list=True, self_interaction=False):
    return _build("oracle", positions, cell, pbc, cutoff, full_list, self_interaction)


def build_reference(positions, cell=None, pbc=None, cutoff=4.5, full_list=True,
                    self_interaction=False):
    return _build("ref", positions, cell, pbc, cutoff, full_list, self_interaction)


def cell_inverse(cell, kind="oracle"):
    lib = _load(kind)
    fn = lib.nlo_cell_inverse if kind == "oracle" else lib.nlref_cell_inverse
    c = np.ascontiguousarray(cell, dtype=np.float32).reshape(9)
    out = np.zeros(9, np.float32)
    fn(_ptr(c), _ptr(out))
    return out.reshape(3, 3)
