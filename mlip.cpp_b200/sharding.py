"""Batches of independent structures over several GPUs.

The reference evaluates a batch on one device (PETModel::predict_batch,
src/models/pet/pet.h:140-143, pet.cpp:125-694).  Here the structures of a
batch are split across the ranks of a torch.distributed group (one process
per GPU): each rank predicts its own share with one batched call, and the
only communication is the final gather of the per-structure results.

The split balances the attention-dominated cost: a structure of n atoms with
s_i tokens per atom (its neighbours + 1) costs about sum_i s_i^2 per layer,
which for small molecules inside one cutoff is close to n^3.  Structures
are assigned greedily, largest cost first, to the least-loaded rank (LPT).
"""
from __future__ import annotations

import numpy as np


def structure_cost(n_atoms: int, tokens_per_atom: float | None = None) -> float:
    """Relative cost of one structure: n * s^2 with s the tokens per atom
    (default: n, every atom within the cutoff of every other)."""
    s = float(n_atoms if tokens_per_atom is None else tokens_per_atom)
    return float(n_atoms) * s * s


def shard(costs, world: int) -> list[list[int]]:
    """Indices of the structures for each of `world` ranks (LPT: largest
    cost first onto the least-loaded rank).  Each rank's list is in
    ascending order; the union is every index exactly once."""
    order = np.argsort(-np.asarray(costs, np.float64), kind="stable")
    load = np.zeros(world)
    parts: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = int(np.argmin(load))
        parts[r].append(int(i))
        load[r] += costs[i]
    return [sorted(p) for p in parts]


class BatchRunner:
    """Predicts a batch of structures sharded over the ranks of a
    torch.distributed group.

    `evaluate(list_of_structures) -> list of (energy, forces [n,3],
    stress [6] or None)` runs one rank's share (for the GPU library:
    ``predictor_batch_eval(predictor)``).  `run` returns, on every rank, the
    results of the whole batch in input order."""

    def __init__(self, evaluate, world: int = 1, rank: int = 0, group=None):
        self.evaluate = evaluate
        self.world, self.rank, self.group = world, rank, group

    def run(self, systems, costs=None):
        costs = [structure_cost(s.n_atoms) for s in systems] if costs is None else costs
        parts = shard(costs, self.world)
        mine = parts[self.rank]
        local = self.evaluate([systems[i] for i in mine]) if mine else []
        payload = [(i, float(e), np.asarray(f, np.float32), None if st is None else np.asarray(st, np.float32))
                   for i, (e, f, st) in zip(mine, local)]
        if self.world > 1:
            import torch.distributed as dist
            gathered = [None] * self.world
            dist.all_gather_object(gathered, payload, group=self.group)
            payload = [x for part in gathered for x in part]
        out = [None] * len(systems)
        for i, e, f, st in payload:
            out[i] = (e, f, st)
        return out


def predictor_batch_eval(predictor, compute_forces: bool = True, compute_stress: bool = False):
    """Rank-local evaluator backed by the GPU library's batched predict."""

    def run(structs):
        res = predictor.predict_batch(structs, compute_forces=compute_forces, compute_stress=compute_stress)
        return [(r.energy, r.forces if r.has_forces() else np.zeros((0, 3), np.float32),
                 r.stress if r.has_stress() else None) for r in res]
    return run


class PackedBatch:
    """A batch of structures held as one block: the positions [sum n, 3] and
    atomic numbers [sum n] of structure k follow those of structure k - 1;
    n_atoms [n_systems]; cells [n_systems, 9] and pbc [n_systems, 3], or
    None for non-periodic structures.  The layout of
    Predictor.predict_packed."""

    def __init__(self, positions, numbers, n_atoms, cells=None, pbc=None):
        self.positions = np.ascontiguousarray(positions, np.float32).reshape(-1, 3)
        self.numbers = np.ascontiguousarray(numbers, np.int32).reshape(-1)
        self.n_atoms = np.ascontiguousarray(n_atoms, np.int32).reshape(-1)
        ns = self.n_atoms.shape[0]
        self.cells = None if cells is None else np.ascontiguousarray(cells, np.float32).reshape(ns, 9)
        self.pbc = None if pbc is None else np.ascontiguousarray(pbc, np.bool_).reshape(ns, 3)
        self.first = np.zeros(ns + 1, np.int64)
        np.cumsum(self.n_atoms, out=self.first[1:])
        if self.first[-1] != self.positions.shape[0] or self.numbers.shape[0] != self.positions.shape[0]:
            raise ValueError("positions, numbers and n_atoms do not describe the same atoms")

    @classmethod
    def pack(cls, structs) -> "PackedBatch":
        """From objects with positions, numbers and (optional) cell / pbc."""
        structs = list(structs)
        cells = [getattr(s, "cell", None) for s in structs]
        periodic = any(c is not None for c in cells)
        if periodic and any(c is None for c in cells):
            raise ValueError("a packed batch is either all periodic or all non-periodic")
        pbc = None
        if periodic:
            pbc = [getattr(s, "pbc", None) for s in structs]
            pbc = [[True] * 3 if p is None else list(p) for p in pbc]
        return cls(np.concatenate([np.asarray(s.positions, np.float32).reshape(-1, 3) for s in structs]),
                   np.concatenate([np.asarray(s.numbers, np.int32).reshape(-1) for s in structs]),
                   [len(s.numbers) for s in structs],
                   None if not periodic else np.stack([np.asarray(c, np.float32).reshape(9) for c in cells]),
                   pbc)

    def __len__(self) -> int:
        return int(self.n_atoms.shape[0])

    def structures(self) -> list:
        """The structures one by one (views with positions, numbers, n_atoms,
        cell and pbc)."""
        from types import SimpleNamespace
        out = []
        for k in range(len(self)):
            a, b = int(self.first[k]), int(self.first[k + 1])
            out.append(SimpleNamespace(positions=self.positions[a:b], numbers=self.numbers[a:b], n_atoms=b - a,
                                       cell=None if self.cells is None else self.cells[k].reshape(3, 3),
                                       pbc=None if self.pbc is None else self.pbc[k]))
        return out

    def atom_index(self, idx) -> np.ndarray:
        """Rows of the atoms of structures `idx`, in that order."""
        idx = np.asarray(idx, np.int64)
        n = self.n_atoms[idx].astype(np.int64)
        starts = np.repeat(self.first[idx] - np.concatenate([[0], np.cumsum(n)[:-1]]), n)
        return starts + np.arange(int(n.sum()), dtype=np.int64)

    def take(self, idx, rows=None) -> "PackedBatch":
        """The structures `idx`, in that order, as a batch of their own
        (`rows`: their atom_index, when the caller has it already)."""
        idx = np.asarray(idx, np.int64)
        if idx.shape[0] == len(self) and np.array_equal(idx, np.arange(len(self))):
            return self
        rows = self.atom_index(idx) if rows is None else rows
        return PackedBatch(self.positions[rows], self.numbers[rows], self.n_atoms[idx],
                           None if self.cells is None else self.cells[idx],
                           None if self.pbc is None else self.pbc[idx])


class PackedBatchRunner:
    """BatchRunner for packed batches: each rank evaluates its share with
    one call and the ranks exchange one set of arrays each, so nothing in the
    step is done per structure in Python.

    `evaluate(PackedBatch) -> (energies [n], forces [sum n, 3] or None,
    stress [n, 6] or None)` (for the GPU library:
    ``predictor_packed_eval(predictor)``).  `run` returns the same triple for
    the whole batch, in input order, on every rank; over several ranks the
    energies come back as float64 and forces and stress in the evaluator's
    dtype.  The results cross the process group in one all-gather (device
    tensors over NCCL, host tensors over gloo)."""

    def __init__(self, evaluate, world: int = 1, rank: int = 0, group=None):
        self.evaluate = evaluate
        self.world, self.rank, self.group = world, rank, group
        self._plan_cache = None

    def _plan(self, batch: PackedBatch, costs):
        """The split and every index array the exchange needs.  They depend
        only on the sizes of the structures, so they are kept while the
        sizes repeat (costs given: made anew)."""
        key = batch.n_atoms.tobytes() if costs is None else None
        if key is not None and self._plan_cache is not None and self._plan_cache[0] == key:
            return self._plan_cache[1]
        if costs is None:
            costs = [structure_cost(int(n)) for n in batch.n_atoms]
        parts = shard(costs, self.world)
        n_s = [len(p) for p in parts]
        n_a = [int(batch.n_atoms[p].sum()) if p else 0 for p in parts]
        rows = [batch.atom_index(p) if p else np.zeros(0, np.int64) for p in parts]
        # the gathered shares hold structures (atoms) in rank order; the
        # inverse permutations put them back in input order with one gather
        s_order = np.concatenate([np.asarray(p, np.int64) for p in parts])
        a_order = np.concatenate(rows)
        s_inv = np.empty_like(s_order)
        s_inv[s_order] = np.arange(s_order.shape[0])
        a_inv = np.empty_like(a_order)
        a_inv[a_order] = np.arange(a_order.shape[0])
        plan = {"parts": parts, "n_s": n_s, "n_a": n_a, "rows": rows, "s_inv": s_inv, "a_inv": a_inv,
                "width": max(2 + 7 * ns + 3 * na for ns, na in zip(n_s, n_a))}
        if key is not None:
            self._plan_cache = (key, plan)
        return plan

    def run(self, batch: PackedBatch, costs=None):
        if self.world == 1:
            return self.evaluate(batch)
        P = self._plan(batch, costs)
        parts, n_s, n_a = P["parts"], P["n_s"], P["n_a"]
        mine = parts[self.rank]
        e, f, st = self.evaluate(batch.take(mine, P["rows"][self.rank])) if mine else (None, None, None)
        # Every rank knows every share, so each sends one float64 row of a
        # fixed width: [forces itemsize, stress itemsize | energies | stress
        # | forces], padded to the largest share; one all-gather moves them.
        row = np.zeros(P["width"], np.float64)
        k, na = len(mine), n_a[self.rank]
        if mine:
            row[0] = 0 if f is None else np.asarray(f).dtype.itemsize
            row[1] = 0 if st is None else np.asarray(st).dtype.itemsize
            row[2:2 + k] = e
            if st is not None:
                row[2 + k:2 + 7 * k] = np.asarray(st).reshape(-1)
            if f is not None:
                row[2 + 7 * k:2 + 7 * k + 3 * na] = np.asarray(f).reshape(-1)
        import torch
        import torch.distributed as dist
        dev = (torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(self.group) == "nccl"
               else torch.device("cpu"))
        send = torch.from_numpy(row).to(dev)
        recv = [torch.empty_like(send) for _ in range(self.world)]
        dist.all_gather(recv, send, group=self.group)
        rows = torch.stack(recv).cpu().numpy()
        live = [r for r in range(self.world) if n_s[r]]
        if not live:
            return np.zeros(0, np.float64), None, None
        fsize, ssize = rows[live[0], 0], rows[live[0], 1]
        e_all = np.concatenate([rows[r, 2:2 + n_s[r]] for r in live])[P["s_inv"]]
        st_all = f_all = None
        if ssize:
            st_cat = np.concatenate([rows[r, 2 + n_s[r]:2 + 7 * n_s[r]] for r in live]).reshape(-1, 6)
            st_all = st_cat[P["s_inv"]].astype(np.float32 if ssize == 4 else np.float64)
        if fsize:
            f_cat = np.concatenate([rows[r, 2 + 7 * n_s[r]:2 + 7 * n_s[r] + 3 * n_a[r]] for r in live]).reshape(-1, 3)
            f_all = f_cat[P["a_inv"]].astype(np.float32 if fsize == 4 else np.float64)
        return e_all, f_all, st_all


def predictor_packed_eval(predictor, compute_forces: bool = True, compute_stress: bool = False):
    """Rank-local packed evaluator backed by the GPU library's
    Predictor.predict_packed."""

    def run(batch: PackedBatch):
        r = predictor.predict_packed(batch.positions, batch.numbers, batch.n_atoms, batch.cells, batch.pbc,
                                     compute_forces=compute_forces, compute_stress=compute_stress)
        return r.energies, r.forces, r.stress
    return run
