"""Spatial domain decomposition of one large periodic cell over several GPUs.

The reference evaluates one structure on one device (PETModel::predict_batch,
src/models/pet/pet.cpp:125-694). For cells too large or too slow for one
GPU, the cell is split into px x py x pz fractional-coordinate slabs, one per
rank (one process per GPU).

Atom i's energy depends on every atom within num_gnn_layers x cutoff of i:
* layer-1 tokens of i use messages from i's neighbours' layer-0 outputs;
* those outputs depend on the neighbours' own neighbours;
* attention is per atom.

So each rank builds a local system of three groups (ghosts only across the
faces the grid splits; along an unsplit axis the local system stays
periodic):

    owned atoms                           layer 0, layer 1 and the readout
    ghosts within 1 cutoff of the slab    layer 0 only (their outputs feed
                                          the owned atoms' messages)
    ghosts within 2 cutoffs of the slab   neighbour candidates only

The local energy is the owned atoms' energy. The local forces are its gradient
on every local atom, owned and ghost, and the local virial is over the local
edges. Summing the three over ranks gives the whole cell's energy, forces and
virial. That sum is the only exchange step: one NCCL all-reduce of the force
array and one of (energy, virial). Every rank holds the whole position array;
each step it partitions on the device (fractional coordinates, 27 image
shifts, two host synchronisations for the counts) and gathers its local
system with exact f64 image shifts.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass
class LocalDomain:
    index: np.ndarray       # [n_local] global atom of each local atom
    shift: np.ndarray       # [n_local, 3] integer image shift (in cell vectors)
    n_layer0: int           # owned + first ghost shell
    n_owned: int
    cell: np.ndarray        # (3, 3) float32 search-grid cell (the global cell)
    pbc: tuple              # periodic along the axes the grid does not split
    grid: tuple
    rank: int

    @property
    def n_local(self) -> int:
        return int(self.index.shape[0])


def face_distances(cell) -> np.ndarray:
    c = np.asarray(cell, np.float64).reshape(3, 3)
    vol = abs(np.linalg.det(c))
    n = [np.cross(c[1], c[2]), np.cross(c[2], c[0]), np.cross(c[0], c[1])]
    return np.array([vol / np.linalg.norm(v) for v in n])


def grid_for(world: int) -> tuple:
    """px, py, pz with px * py * pz == world, splitting the last axes first
    (1 -> 1x1x1, 2 -> 1x1x2, 4 -> 1x2x2, 8 -> 2x2x2)."""
    g = [1, 1, 1]
    k = 2
    w = world
    while w > 1:
        if w % 2:
            g[k] *= w
            break
        g[k] *= 2
        w //= 2
        k = (k - 1) % 3
    return tuple(g)


def partition(positions, cell, cutoff: float, grid: tuple, rank: int, layers: int = 2) -> LocalDomain:
    """Local system of `rank` on the fractional grid `grid` (px, py, pz),
    computed on the host in float64.  Atom order: owned atoms (ascending
    global index), then the first ghost shell, then the second, each shell
    ordered by image shift (x slowest, -1..1) and then global index."""
    import torch
    d = partition_device(torch.from_numpy(np.asarray(positions, np.float64).reshape(-1, 3)),
                         torch.from_numpy(np.asarray(cell, np.float64).reshape(3, 3)), cutoff, grid, rank, layers)
    return LocalDomain(d["index"].numpy(), d["shift"].numpy(), d["n_layer0"], d["n_owned"], d["cell"],
                       d["pbc"], tuple(int(x) for x in grid), rank)


_SHIFTS = np.array(np.meshgrid(*([(-1, 0, 1)] * 3), indexing="ij")).reshape(3, -1).T  # [27, 3]


def partition_device(positions, cell, cutoff: float, grid: tuple, rank: int, layers: int = 2) -> dict:
    """partition() with torch tensors on any device (positions [N, 3],
    cell [3, 3]).  An axis the grid does not split stays periodic and gets
    no ghosts.  Returns index and shift tensors on that device, the local
    positions (f64; translated along split axes so that their fractional
    coordinates start at 0), the counts, the search cell and its pbc flags.
    Two host synchronisations (the counts)."""
    import torch

    dev = positions.device
    pos = positions.to(torch.float64)
    c = cell.to(device=dev, dtype=torch.float64)
    p = torch.tensor(grid, dtype=torch.float64, device=dev)
    pi = torch.tensor(grid, dtype=torch.int64, device=dev)
    face = torch.from_numpy(face_distances(c.cpu().numpy())).to(dev)
    split = p > 1
    d1 = torch.where(split, cutoff / face, torch.zeros_like(face))
    dn = torch.where(split, layers * cutoff / face, torch.zeros_like(face))
    if bool(torch.any(dn >= 1.0 / p)):
        # one image (+-1) per axis suffices only if a ghost shell is thinner than a slab
        raise ValueError("cell too small for this many domains (ghost shell thicker than a slab)")
    frac = pos @ torch.linalg.inv(c)
    base = -torch.floor(frac)                 # shift into the primary cell
    fw = frac + base                          # in [0, 1)
    coord = torch.minimum((fw * p).to(torch.int64), pi - 1)
    rc = torch.tensor(np.unravel_index(rank, tuple(grid), order="F"), dtype=torch.int64, device=dev)
    lo, hi = rc / p, (rc + 1) / p
    own_mask = torch.all(coord == rc, dim=1)
    S = torch.from_numpy(_SHIFTS).to(dev)
    f = fw.unsqueeze(0) + S.unsqueeze(1).to(torch.float64)       # [27, N, 3]
    in2 = torch.all((f >= lo - dn) & (f < hi + dn), dim=2)
    in1 = torch.all((f >= lo - d1) & (f < hi + d1), dim=2)
    centre = 13                                                  # shift (0, 0, 0)
    in1[centre] &= ~own_mask
    in2[centre] &= ~own_mask
    in2 &= ~in1
    owned = torch.nonzero(own_mask).squeeze(1)
    k1, i1 = torch.nonzero(in1, as_tuple=True)
    k2, i2 = torch.nonzero(in2, as_tuple=True)
    index = torch.cat([owned, i1, i2])
    shift = torch.cat([torch.zeros((owned.shape[0], 3), dtype=torch.int64, device=dev), S[k1], S[k2]])
    shift = shift + base[index].to(torch.int64)
    n_owned = int(owned.shape[0])
    n_layer0 = n_owned + int(i1.shape[0])
    origin = torch.where(split, lo - dn, torch.zeros_like(lo))
    local = pos[index] + (shift.to(torch.float64) - origin) @ c
    pbc = tuple(bool(x) for x in (np.asarray(grid) == 1))
    return {"index": index, "shift": shift, "local": local, "n_owned": n_owned, "n_layer0": n_layer0,
            "cell": c.cpu().numpy().astype(np.float32), "pbc": pbc}


def predictor_eval(predictor):
    """Per-domain evaluator backed by the GPU library (C ABI
    mlipcpp_b200_predict_local).  Returns (owned energy, local virial)."""
    import torch

    def run(d: LocalDomain, local_pos, numbers, forces_out):
        torch.cuda.synchronize()  # the library runs on its own stream
        return predictor.predict_local(local_pos.data_ptr(), numbers, d.n_layer0, d.n_owned, d.cell, d.pbc,
                                       True, forces_out.data_ptr())
    return run


class DomainRunner:
    """Evaluates one cell split over the ranks of a torch.distributed group,
    or over `emulate` domains one after another in a single process.

    `local_eval(domain, local_pos f64 [n,3], numbers, forces_out f32 [n,3])`
    evaluates one local system and returns (owned energy, virial[6])."""

    def __init__(self, local_eval, numbers, cell, cutoff: float, world: int = 1, rank: int = 0,
                 group=None, emulate: int | None = None, device: str = "cuda"):
        import torch

        self.torch = torch
        self.local_eval = local_eval
        self.device = device
        self.numbers = np.asarray(numbers, np.int32)
        self.cell = np.asarray(cell, np.float64).reshape(3, 3)
        self.cutoff = float(cutoff)
        self.world, self.rank, self.group = world, rank, group
        self.n_domains = emulate if emulate else world
        self.my_domains = list(range(self.n_domains)) if emulate else [rank]
        self.grid = grid_for(self.n_domains)
        self.cell_t = torch.from_numpy(self.cell).to(device)

    def step(self, positions):
        """One E + F + virial evaluation from positions [N, 3] (f32 or f64)
        on the runner's device: partition, gather of the local systems,
        per-domain evaluation, scatter of the local forces and the sums over
        ranks.  Returns (energy, forces [N, 3] f32, virial [6] f64)."""
        torch = self.torch
        n = positions.shape[0]
        F = torch.zeros((n, 3), dtype=torch.float32, device=self.device)
        acc = torch.zeros(7, dtype=torch.float64)
        for r in self.my_domains:
            d = partition_device(positions, self.cell_t, self.cutoff, self.grid, r)
            idx = d["index"]
            dom = LocalDomain(idx, d["shift"], d["n_layer0"], d["n_owned"], d["cell"], d["pbc"], self.grid, r)
            z = self.numbers[idx.cpu().numpy()]
            local = d["local"].contiguous()
            forces = torch.empty((idx.shape[0], 3), dtype=torch.float32, device=self.device)
            e, vir = self.local_eval(dom, local, z, forces)
            F.index_add_(0, idx, forces)
            acc[0] += e
            acc[1:] += torch.from_numpy(np.asarray(vir, np.float64))
        if self.world > 1:
            import torch.distributed as dist
            dist.all_reduce(F, group=self.group)
            accd = acc.to(self.device)
            dist.all_reduce(accd, group=self.group)
            acc = accd.cpu()
        return float(acc[0]), F, acc[1:].numpy()

    def stress(self, virial) -> np.ndarray:
        """Voigt stress = virial / |det cell| (pet.cpp:1079-1097)."""
        vol = abs(float(np.linalg.det(self.cell)))
        return (np.asarray(virial) / vol).astype(np.float32)
