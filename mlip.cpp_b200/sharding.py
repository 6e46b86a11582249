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
