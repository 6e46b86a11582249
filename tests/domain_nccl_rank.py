"""One rank of the NCCL domain-decomposition check (launched by
tests/test_gpu_domain_nccl.py through torch.distributed.run): every rank
evaluates its spatial domain of one cell with NCCL exchanges; rank 0
gathers the forces and compares energy, forces and stress with the
whole-cell prediction."""
import datetime
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import conftest  # noqa: E402,F401  (registers mlipcpp_b200)
import mlipcpp_b200 as mb  # noqa: E402
from mlipcpp_b200 import domain as dd  # noqa: E402
from mlipcpp_b200 import workloads as wl  # noqa: E402


def main():
    path, out = sys.argv[1], sys.argv[2]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    mb.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    s = wl.fcc_alloy(16, seed=71)
    grid = dd.grid_for(world)
    pred = mb.Predictor(path)
    mine = np.nonzero(dd.owners(s.positions, s.cell, grid) == rank)[0]
    comm = dd.NcclComm()
    dom = dd.Domain(pred, s.cell, grid, rank, comm.c)
    dom.set_atoms(s.numbers[mine])
    pos = torch.from_numpy(np.ascontiguousarray(s.positions[mine])).cuda()
    F = torch.zeros_like(pos)
    for _ in range(2):
        e, vir = dom.step(pos, F)
    # gather the owned forces on rank 0
    n = torch.tensor([len(mine)], device="cuda")
    sizes = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(sizes, n)
    m = int(max(x.item() for x in sizes))
    pad = torch.zeros((m, 3), device="cuda")
    pad[:len(mine)] = F
    idx = torch.full((m,), -1, dtype=torch.int64, device="cuda")
    idx[:len(mine)] = torch.from_numpy(mine).cuda()
    allF = [torch.zeros_like(pad) for _ in range(world)]
    allI = [torch.zeros_like(idx) for _ in range(world)]
    dist.all_gather(allF, pad)
    dist.all_gather(allI, idx)
    if rank == 0:
        forces = np.zeros((s.n_atoms, 3), np.float32)
        for f, i in zip(allF, allI):
            i = i.cpu().numpy()
            forces[i[i >= 0]] = f.cpu().numpy()[i >= 0]
        full = pred.predict(s.positions, s.numbers, s.cell, s.pbc, compute_stress=True)
        stress = vir / abs(np.linalg.det(s.cell.astype(np.float64)))
        json.dump({"de_per_atom": abs(e - full.energy) / s.n_atoms,
                   "df": float(np.abs(forces - full.forces).max()),
                   "ds": float(np.abs(stress - full.stress).max()),
                   "stats": dom.stats()}, open(out, "w"))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
