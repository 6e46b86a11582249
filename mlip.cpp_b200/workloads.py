"""Seeded synthetic workloads and random-init ``"pet"`` GGUF weights.

No PET checkpoint or public structure set is available offline, so every
workload here is generated from a seed with the shapes, sizes and value
distributions of the benchmark configurations:

* ``si_diamond``   diamond Si supercell (a = 5.431 A, jitter N(0, 0.05 A))
* ``water_box``    liquid water at 1.0 g/cm^3 (O-H 0.96 A, H-O-H 104.5 deg)
* ``molecules``    non-periodic organic-like molecules of 10-60 atoms
* ``fcc_alloy``    32^3 primitive fcc cells, 20 random elements, jitter 0.08 A

``write_pet_gguf`` emits the legacy ``"pet"`` GGUF layout that mlip.cpp's
``PETModel::load_from_gguf`` reads (src/models/pet/pet.cpp:1177-1301): the
same metadata keys and tensor names as scripts/convert_pet_mad.py:184-275
writes, with linear weights and biases ~ U(+-1/sqrt(fan_in)), embeddings
~ N(0, 1), layer-norm scales 1 + 0.1 N(0, 1) and shifts 0.1 N(0, 1), and
composition energies ~ N(-3, 1).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, asdict

import numpy as np


# --------------------------------------------------------------------------
# Hyperparameters
# --------------------------------------------------------------------------
@dataclass(frozen=True)
class PETHypers:
    """PET hyperparameters as stored in GGUF metadata (pet_types.h:54-63)."""
    d_pet: int = 256
    num_heads: int = 8
    d_feedforward: int = 512
    d_head: int = 128
    cutoff: float = 4.5
    cutoff_width: float = 0.2
    num_gnn_layers: int = 2
    num_attention_layers: int = 2


#: Stand-in for pet-mad-s (its GGUF is not available): PET-MAD's published
#: legacy hypers (scripts/convert_pet_mad.py:65-73).
PET_MAD_S = PETHypers()
#: Stand-in for pet-oam-l (its GGUF is not available): twice the width of
#: PET_MAD_S inside the fixed 2 GNN x 2 attention-block layout of "pet".
PET_OAM_L = PETHypers(d_pet=512, num_heads=16, d_feedforward=1024, d_head=256)
#: Small hypers for fast tests.
PET_TINY = PETHypers(d_pet=64, num_heads=4, d_feedforward=128, d_head=32)

HYPERS = {"pet-mad-s": PET_MAD_S, "pet-oam-l": PET_OAM_L, "tiny": PET_TINY}


# --------------------------------------------------------------------------
# GGUF writer (legacy "pet" layout)
# --------------------------------------------------------------------------
def pet_tensor_shapes(h: PETHypers, n_species: int) -> dict[str, tuple[int, ...]]:
    """numpy shapes ([out, in] for linears) of every tensor of a "pet" GGUF."""
    d, f, r = h.d_pet, h.d_feedforward, h.d_head
    s = {"model.embedding.weight": (n_species + 1, d)}
    for l in range(2):
        p = f"model.gnn.{l}."
        s[p + "edge_embedder.weight"] = (d, 4)
        s[p + "edge_embedder.bias"] = (d,)
        s[p + "node_embedder.weight"] = (n_species + 1, d)
        if l > 0:
            s[p + "neighbor_embedder.weight"] = (n_species + 1, d)
        k = 2 if l == 0 else 3
        s[p + "compress.0.weight"] = (d, k * d)
        s[p + "compress.0.bias"] = (d,)
        s[p + "compress.2.weight"] = (d, d)
        s[p + "compress.2.bias"] = (d,)
        for t in range(2):
            q = p + f"tl.{t}."
            s[q + "attn.in.weight"] = (3 * d, d)
            s[q + "attn.in.bias"] = (3 * d,)
            s[q + "attn.out.weight"] = (d, d)
            s[q + "attn.out.bias"] = (d,)
            for nrm in ("norm_a", "norm_m"):
                s[q + nrm + ".weight"] = (d,)
                s[q + nrm + ".bias"] = (d,)
            s[q + "mlp.0.weight"] = (f, d)
            s[q + "mlp.0.bias"] = (f,)
            s[q + "mlp.3.weight"] = (d, f)
            s[q + "mlp.3.bias"] = (d,)
        for kind in ("node", "edge"):
            hp = f"model.{kind}_heads.energy.{l}."
            s[hp + "0.weight"] = (r, d)
            s[hp + "0.bias"] = (r,)
            s[hp + "2.weight"] = (r, r)
            s[hp + "2.bias"] = (r,)
            lp = f"model.{kind}_last_layers.energy.{l}.energy___0."
            s[lp + "weight"] = (1, r)
            s[lp + "bias"] = (1,)
    return s


#: Non-conservative property heads of PET-MAD v1.1+ (pet_types.h:130-138):
#: property -> (last-layer tensor suffix, outputs per atom).
NC_HEADS = {"nc_forces": ("nc_f", 3), "nc_stress": ("nc_s", 9)}


def nc_head_shapes(h: PETHypers, props=("nc_forces", "nc_stress"), layers=(0, 1)) -> dict[str, tuple[int, ...]]:
    """numpy shapes of the non-conservative head tensors (node and edge MLPs
    d -> d_head -> d_head -> od per GNN layer, pet.cpp:48-79)."""
    d, r = h.d_pet, h.d_head
    s = {}
    for prop in props:
        last, od = NC_HEADS[prop]
        for l in layers:
            for kind in ("node", "edge"):
                hp = f"model.{kind}_heads.{prop}.{l}."
                s[hp + "0.weight"] = (r, d)
                s[hp + "0.bias"] = (r,)
                s[hp + "2.weight"] = (r, r)
                s[hp + "2.bias"] = (r,)
                lp = f"model.{kind}_last_layers.{prop}.{l}.{last}."
                s[lp + "weight"] = (od, r)
                s[lp + "bias"] = (od,)
    return s


def random_pet_weights(h: PETHypers, atomic_numbers, seed: int = 0, nc_heads=False) -> dict[str, np.ndarray]:
    """Seeded random-init weights (float32) keyed by GGUF tensor name.

    nc_heads: False, True (both non-conservative properties on both layers)
    or a dict of nc_head_shapes keyword arguments.  Their weights come from a
    second generator, so the other tensors do not depend on this choice."""
    rng = np.random.default_rng(seed)
    z = np.asarray(atomic_numbers, dtype=np.int32)
    out: dict[str, np.ndarray] = {}
    for name, shape in pet_tensor_shapes(h, len(z)).items():
        if "embedding" in name or "embedder.weight" in name and "edge" not in name:
            w = rng.standard_normal(shape)
        elif ".norm_" in name:
            base = 1.0 if name.endswith("weight") else 0.0
            w = base + 0.1 * rng.standard_normal(shape)
        else:
            # linear weight [out, in] and its bias share fan_in = in
            wshape = shape if len(shape) == 2 else None
            fan_in = wshape[1] if wshape else _fan_in_of_bias(name, h)
            bound = 1.0 / math.sqrt(fan_in)
            w = rng.uniform(-bound, bound, size=shape)
        out[name] = np.ascontiguousarray(w, dtype=np.float32)
    out["composition.atomic_numbers"] = z
    out["composition.energies"] = (-3.0 + rng.standard_normal(len(z))).astype(np.float32)
    if nc_heads:
        nrng = np.random.default_rng(seed + 7919)
        kw = nc_heads if isinstance(nc_heads, dict) else {}
        for name, shape in nc_head_shapes(h, **kw).items():
            fan_in = shape[1] if len(shape) == 2 else _fan_in_of_bias(name, h)
            bound = 1.0 / math.sqrt(fan_in)
            out[name] = np.ascontiguousarray(nrng.uniform(-bound, bound, size=shape), dtype=np.float32)
    return out


def _fan_in_of_bias(name: str, h: PETHypers) -> int:
    d, f, r = h.d_pet, h.d_feedforward, h.d_head
    if "edge_embedder" in name:
        return 4
    if "compress.0" in name:
        return (2 if ".gnn.0." in name else 3) * d
    if "mlp.3" in name:
        return f
    if "_heads." in name and name.endswith("2.bias"):
        return r
    if "_last_layers." in name:
        return r
    return d


def write_pet_gguf(path: str, h: PETHypers, atomic_numbers=None, seed: int = 0,
                   weights: dict[str, np.ndarray] | None = None, nc_heads=False) -> dict[str, np.ndarray]:
    """Write a random-init ``"pet"`` GGUF and return the weights written
    (nc_heads: see random_pet_weights)."""
    import gguf

    if atomic_numbers is None:
        atomic_numbers = np.arange(1, 90, dtype=np.int32)
    if weights is None:
        weights = random_pet_weights(h, atomic_numbers, seed, nc_heads=nc_heads)
    w = gguf.GGUFWriter(path, arch="pet")
    w.add_name(f"random-init PET seed={seed}")
    w.add_float32("pet.cutoff", float(h.cutoff))
    w.add_float32("pet.cutoff_width", float(h.cutoff_width))
    w.add_int32("pet.d_pet", int(h.d_pet))
    w.add_int32("pet.d_head", int(h.d_head))
    w.add_int32("pet.num_heads", int(h.num_heads))
    w.add_int32("pet.num_gnn_layers", int(h.num_gnn_layers))
    w.add_int32("pet.d_feedforward", int(h.d_feedforward))
    w.add_int32("pet.num_attention_layers", int(h.num_attention_layers))
    for name, arr in weights.items():
        w.add_tensor(name, arr)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return weights


def read_pet_gguf(path: str) -> tuple[PETHypers, dict[str, np.ndarray]]:
    """Read hypers and tensors (numpy shapes) with the ``gguf`` package."""
    import gguf

    r = gguf.GGUFReader(path)
    meta = {}
    for f in r.fields.values():
        if f.name.startswith("pet.") and f.types and len(f.data) == 1:
            meta[f.name] = f.parts[f.data[0]][0]
    tensors = {}
    for t in r.tensors:
        shape = tuple(int(x) for x in reversed(t.shape.tolist()))
        tensors[t.name] = np.array(t.data).reshape(shape).copy()
    h = PETHypers(
        d_pet=int(tensors["model.embedding.weight"].shape[1]),
        num_heads=int(meta.get("pet.num_heads", 8)),
        d_feedforward=int(meta.get("pet.d_feedforward", 512)),
        d_head=int(meta.get("pet.d_head", 128)),
        cutoff=float(meta.get("pet.cutoff", 4.5)),
        cutoff_width=float(meta.get("pet.cutoff_width", 0.5)),
    )
    return h, tensors


# --------------------------------------------------------------------------
# Structures
# --------------------------------------------------------------------------
@dataclass
class Structure:
    positions: np.ndarray          # (N, 3) float32
    numbers: np.ndarray            # (N,) int32
    cell: np.ndarray | None = None  # (3, 3) float32, rows are lattice vectors
    pbc: tuple[bool, bool, bool] | None = None

    @property
    def n_atoms(self) -> int:
        return int(self.positions.shape[0])


def si_diamond(reps: int = 3, a: float = 5.431, jitter: float = 0.05, seed: int = 0) -> Structure:
    """Diamond Si supercell of reps^3 conventional cells (8 atoms each)."""
    basis = np.array([[0, 0, 0], [0, .5, .5], [.5, 0, .5], [.5, .5, 0],
                      [.25, .25, .25], [.25, .75, .75], [.75, .25, .75], [.75, .75, .25]])
    g = np.stack(np.meshgrid(*(np.arange(reps),) * 3, indexing="ij"), -1).reshape(-1, 1, 3)
    frac = (g + basis[None]).reshape(-1, 3)
    pos = frac * a
    rng = np.random.default_rng(seed)
    pos = pos + rng.normal(0.0, jitter, pos.shape)
    cell = np.eye(3) * a * reps
    return Structure(pos.astype(np.float32), np.full(len(pos), 14, np.int32),
                     cell.astype(np.float32), (True, True, True))


def fcc_alloy(reps=32, a: float = 3.6, n_elements: int = 20, jitter: float = 0.08,
              seed: int = 0) -> Structure:
    """reps^3 (or reps = (nx, ny, nz)) primitive fcc cells (one atom each; a
    triclinic supercell), species drawn uniformly from `n_elements` random
    elements among Z=1..89."""
    r = (reps,) * 3 if np.isscalar(reps) else tuple(int(x) for x in reps)
    prim = 0.5 * a * np.array([[0, 1, 1], [1, 0, 1], [1, 1, 0]], dtype=np.float64)
    g = np.stack(np.meshgrid(*(np.arange(k) for k in r), indexing="ij"), -1).reshape(-1, 3)
    pos = g @ prim
    rng = np.random.default_rng(seed)
    pos = pos + rng.normal(0.0, jitter, pos.shape)
    elements = rng.choice(np.arange(1, 90), size=n_elements, replace=False)
    z = rng.choice(elements, size=len(pos)).astype(np.int32)
    return Structure(pos.astype(np.float32), z, (prim * np.array(r)[:, None]).astype(np.float32),
                     (True, True, True))


def water_box(n_atoms: int = 4096, density: float = 1.0, seed: int = 0,
              min_oo: float = 2.0) -> Structure:
    """Liquid-water cube: floor(n/3) H2O molecules (1365 for n = 4096) padded
    to n atoms with lone H atoms, density in g/cm^3, O-H 0.96 A, H-O-H
    104.5 deg, seeded centres with a minimum O-O distance and seeded
    rotations."""
    n_mol = n_atoms // 3
    mass = 18.015 / 0.60221408  # g/mol -> 1e-24 g (so A^3 at 1 g/cm^3)
    L = (n_atoms / 3.0 * mass / density) ** (1.0 / 3.0)
    rng = np.random.default_rng(seed)
    centres = []
    tries = 0
    while len(centres) < n_mol:
        c = rng.uniform(0, L, 3)
        if centres:
            d = np.asarray(centres) - c
            d -= L * np.round(d / L)
            if np.min(np.einsum("ij,ij->i", d, d)) < min_oo ** 2:
                tries += 1
                if tries > 200000:
                    raise RuntimeError("water_box: packing failed")
                continue
        centres.append(c)
    th = math.radians(104.5) / 2
    local = np.array([[0, 0, 0], [0.96 * math.sin(th), 0.96 * math.cos(th), 0],
                      [-0.96 * math.sin(th), 0.96 * math.cos(th), 0]])
    pos, z = [], []
    for c in centres:
        q = rng.standard_normal(4)
        q /= np.linalg.norm(q)
        R = _quat_to_rot(q)
        pos.append(c + local @ R.T)
        z += [8, 1, 1]
    pos = np.concatenate(pos)
    z = np.asarray(z, np.int32)
    # 1365 H2O = 4095 atoms: pad with lone H atoms (>= 1.5 A from every atom)
    while len(pos) < n_atoms:
        c = rng.uniform(0, L, 3)
        d = pos - c
        d -= L * np.round(d / L)
        if np.min(np.einsum("ij,ij->i", d, d)) < 1.5 ** 2:
            continue
        pos = np.concatenate([pos, c[None]])
        z = np.concatenate([z, [1]]).astype(np.int32)
    pos = np.mod(pos, L)
    return Structure(pos.astype(np.float32), z.astype(np.int32),
                     (np.eye(3) * L).astype(np.float32), (True, True, True))


def _quat_to_rot(q):
    w, x, y, z = q
    return np.array([
        [1 - 2 * (y * y + z * z), 2 * (x * y - z * w), 2 * (x * z + y * w)],
        [2 * (x * y + z * w), 1 - 2 * (x * x + z * z), 2 * (y * z - x * w)],
        [2 * (x * z - y * w), 2 * (y * z + x * w), 1 - 2 * (x * x + y * y)],
    ])


def molecules(n_mol: int = 512, n_min: int = 10, n_max: int = 60, seed: int = 0,
              min_dist: float = 0.9) -> list[Structure]:
    """Non-periodic molecules: n ~ U{n_min..n_max}, Z from {H:.5, C:.3, N:.1,
    O:.1}, positions sampled one by one in a sphere of radius
    0.6 n^(1/3) 1.5 A with a minimum pair distance."""
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n_mol):
        n = int(rng.integers(n_min, n_max + 1))
        z = rng.choice([1, 6, 7, 8], size=n, p=[0.5, 0.3, 0.1, 0.1]).astype(np.int32)
        R = 0.6 * n ** (1 / 3) * 1.5
        pts = []
        while len(pts) < n:
            p = rng.uniform(-R, R, 3)
            if p @ p > R * R:
                continue
            if pts and np.min(np.sum((np.asarray(pts) - p) ** 2, 1)) < min_dist ** 2:
                continue
            pts.append(p)
        out.append(Structure(np.asarray(pts, np.float32), z))
    return out


CONFIGS = {
    "si216": lambda seed=0: si_diamond(3, seed=seed),
    "water4096": lambda seed=0: water_box(4096, seed=seed),
    "fcc32k": lambda seed=0: fcc_alloy(32, seed=seed),
    "si262k": lambda seed=0: si_diamond(32, seed=seed),
}


def hypers_dict(h: PETHypers) -> dict:
    return asdict(h)
