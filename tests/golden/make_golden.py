"""Regenerate the committed golden fixtures in tests/golden/.

* nl_*.npz: neighbour lists produced by the reference's OWN neighbour-list
  code (src/core/neighbor_list.cpp + system.cpp compiled from the reference
  tree by oracle/Makefile into oracle/_ref/libnl_ref.so).  These pin both the
  C restatement (oracle/nl_oracle.c) and the GPU kernels bit-exactly.
* pet_*.npz: energies, forces and stress of the PyTorch restatement
  (oracle/pet_oracle.py, float64) on seeded random-init weights; the weights
  are regenerated from the seed (a digest is stored to detect drift).
  pet_nc_*.npz: the same for a model with non-conservative force and stress
  heads, predicted as use_nc_forces does (no gradients; forces and stress
  from the heads).

Run from the repository root:  python tests/golden/make_golden.py
Needs the reference tree (for oracle/_ref) only for the nl_* fixtures.
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "tests"))
sys.path.insert(0, ROOT)
import conftest  # noqa: E402  (loads the package as mlipcpp_b200)

from mlipcpp_b200 import workloads as wl  # noqa: E402


def nl_cases():
    """name -> (Structure, cutoff)."""
    si8 = wl.si_diamond(1, seed=4)
    out = {
        "si216": (wl.si_diamond(3, seed=0), 4.5),
        "fcc512_triclinic": (wl.fcc_alloy(8, seed=1), 4.5),
        "water192": (wl.water_box(192, seed=2), 4.5),
        "si8_one_bin": (si8, 5.0),
        "si8_wide_search": (si8, 6.0),
        "si64_partial_pbc": (wl.Structure(*_si64(5)[:3], (True, True, False)), 4.5),
        "si64_outside_cell": (_outside(), 4.5),
        "molecule": (wl.molecules(1, seed=6)[0], 4.5),
        "water3_open": (wl.Structure(np.array([[0, 0, 0], [0.757, 0.586, 0], [-0.757, 0.586, 0]],
                                              np.float32), np.array([8, 1, 1], np.int32)), 5.0),
        "dimer_at_cutoff": (wl.Structure(np.array([[0, 0, 0], [3.0, 0, 0]], np.float32),
                                         np.array([14, 14], np.int32)), 3.0),
    }
    return out


def _si64(seed):
    s = wl.si_diamond(2, seed=seed)
    return s.positions, s.numbers, s.cell, s.pbc


def _outside():
    s = wl.si_diamond(2, seed=8)
    rng = np.random.default_rng(8)
    shift = rng.integers(-1, 2, size=(s.n_atoms, 3)) @ s.cell.astype(np.float64)
    return wl.Structure((s.positions + shift).astype(np.float32), s.numbers, s.cell, s.pbc)


def pet_cases():
    """name -> (hypers name, seed, [Structure, ...], non-conservative heads)."""
    return {
        "tiny_si8": ("tiny", 0, [wl.si_diamond(1, seed=3)], False),
        "tiny_water96": ("tiny", 0, [wl.water_box(96, seed=5)], False),
        "tiny_molecules3": ("tiny", 0, wl.molecules(3, seed=7, n_min=5, n_max=20), False),
        "mads_si216": ("pet-mad-s", 1, [wl.si_diamond(3, seed=0)], False),
        "oaml_fcc64": ("pet-oam-l", 2, [wl.fcc_alloy(4, seed=9)], False),
        "nc_tiny_si8": ("tiny", 0, [wl.si_diamond(1, seed=3)], True),
        "nc_tiny_molecules3": ("tiny", 0, wl.molecules(3, seed=7, n_min=5, n_max=20), True),
        "nc_mads_si64": ("pet-mad-s", 1, [wl.si_diamond(2, seed=11)], True),
        # the benchmark configurations at their stated sizes (the fcc alloy
        # at the largest cell the float64 oracle holds here, 12^3 primitive)
        "mads_water4096": ("pet-mad-s", 1, [wl.water_box(4096, seed=0)], False),
        "mads_molecules512": ("pet-mad-s", 1, wl.molecules(512, seed=0), False),
        "oaml_fcc1728": ("pet-oam-l", 2, [wl.fcc_alloy(12, seed=0)], False),
    }


# Structures per oracle call: the oracle pads every atom to the batch's
# largest neighbour count, so large batches of independent molecules are
# evaluated in chunks (batch == single, test_oracle_pet.py)
CHUNK = 16


def weights_digest(h, seed, nc=False):
    w = wl.random_pet_weights(h, np.arange(1, 90, dtype=np.int32), seed, nc_heads=nc)
    m = hashlib.sha256()
    for k in sorted(w):
        m.update(k.encode())
        m.update(np.ascontiguousarray(w[k]).tobytes())
    return m.hexdigest()


def main(only=None):
    from oracle import nl
    import torch

    from oracle import pet_oracle

    torch.set_num_threads(os.cpu_count() or 1)
    if only is None and nl.reference_available():
        for name, (s, rc) in nl_cases().items():
            ref = nl.build_reference(s.positions, s.cell, s.pbc, rc)
            np.savez_compressed(
                os.path.join(HERE, f"nl_{name}.npz"), positions=s.positions,
                cell=np.zeros((0,), np.float32) if s.cell is None else s.cell,
                pbc=np.asarray(s.pbc if s.pbc is not None else (False,) * 3),
                cutoff=np.float32(rc), **{k: v for k, v in ref.items() if k != "n_atoms"})
            print("nl", name, len(ref["centers"]))
    elif only is None:
        print("reference tree absent: nl_* fixtures left unchanged")

    tmp = os.path.join(HERE, "_tmp.gguf")
    for name, (hname, seed, systems, nc) in pet_cases().items():
        if only is not None and name not in only:
            continue
        h = wl.HYPERS[hname]
        wl.write_pet_gguf(tmp, h, seed=seed, nc_heads=nc)
        orc = pet_oracle.load_oracle(tmp, torch.float64)
        periodic = systems[0].cell is not None
        step = 1 if periodic else CHUNK
        res = []
        for k in range(0, len(systems), step):
            res += orc.predict(systems[k:k + step], compute_forces=not nc, compute_nc=nc)
        payload = dict(hypers=hname, seed=seed, digest=weights_digest(h, seed, nc),
                       n_systems=len(systems), nc=nc)
        for k, (s, r) in enumerate(zip(systems, res)):
            payload[f"positions_{k}"] = s.positions
            payload[f"numbers_{k}"] = s.numbers
            payload[f"cell_{k}"] = np.zeros((0,), np.float32) if s.cell is None else s.cell
            payload[f"energy_{k}"] = np.float64(r["energy_f64"])
            payload[f"forces_{k}"] = r["forces"]
            payload[f"stress_{k}"] = r.get("stress", np.zeros((0,), np.float32))
        np.savez_compressed(os.path.join(HERE, f"pet_{name}.npz"), **payload)
        print("pet", name, [r["energy"] for r in res])
    os.remove(tmp)


if __name__ == "__main__":
    # optional arguments: names of the pet_* fixtures to regenerate (default: all)
    main(set(sys.argv[1:]) or None)
