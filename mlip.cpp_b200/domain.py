"""Spatial domain decomposition of one large periodic cell over several GPUs.

The reference evaluates one structure on one device (PETModel::predict_batch,
src/models/pet/pet.cpp:125-694).  Here the cell is split into px x py x pz
fractional-coordinate slabs, one per rank (one process per GPU); rank r owns
slab (r % px, r // px % py, r // (px py)) and the atoms whose wrapped
fractional coordinates fall in it.  The library's domain engine
(csrc/domain.cu, C ABI mlipcpp_b200_domain_*) does the work of a step on the
GPU:

* halo: owned atoms within cutoff (+ skin) of another slab go there as
  ghosts (periodic images included);
* both GNN layers and the readout run on the owned atoms only.  A layer-1
  message of edge i -> j reads the layer-0 token of the reverse edge j -> i
  (pet_layers.cpp:608-679); for a ghost j that token comes from j's owner,
  and its gradient goes back after the layer-1 backward;
* forces on ghosts go back to their owners; energy and virial are summed.

The exchanges are collectives this module supplies to the engine: over NCCL
with torch.distributed (``NcclComm``), or between threads of one process for
tests that emulate several ranks on one GPU (``LocalComm``).  Each exchange is
issued on the library's CUDA stream, so it is ordered with the kernels around
it without host synchronisation.
"""
from __future__ import annotations

import ctypes
import sys
import threading
import traceback

import numpy as np

ALLTOALLV = ctypes.CFUNCTYPE(ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64),
                             ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64), ctypes.c_int64, ctypes.c_void_p)
ALLREDUCE = ctypes.CFUNCTYPE(ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p)


class _CComm(ctypes.Structure):
    """mlipcpp_b200_comm_t (include/mlipcpp_b200.h)."""
    _fields_ = [("user", ctypes.c_void_p), ("alltoallv", ALLTOALLV), ("allreduce_sum_f64", ALLREDUCE)]


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


def slab_of_rank(rank: int, grid) -> tuple:
    px, py, _ = grid
    return rank % px, (rank // px) % py, rank // (px * py)


def owners(positions, cell, grid) -> np.ndarray:
    """Owning rank of every atom: the slab of its wrapped fractional
    coordinates (float64)."""
    pos = np.asarray(positions, np.float64).reshape(-1, 3)
    frac = pos @ np.linalg.inv(np.asarray(cell, np.float64).reshape(3, 3))
    fw = frac - np.floor(frac)
    p = np.asarray(grid, np.int64)
    c = np.minimum((fw * p).astype(np.int64), p - 1)
    return (c[:, 0] + p[0] * (c[:, 1] + p[1] * c[:, 2])).astype(np.int32)


def halo_copies(positions, cell, grid, rank: int, dest: int, width: float) -> list:
    """(atom, image shift) pairs that rank `rank`'s owned atoms send to rank
    `dest`: the images (shifted only along split axes) inside dest's slab
    widened by `width` (A) along each split axis; no unshifted copy to
    itself.  A float64 restatement of the engine's halo test, for the
    geometry checks."""
    pos = np.asarray(positions, np.float64).reshape(-1, 3)
    c = np.asarray(cell, np.float64).reshape(3, 3)
    frac = pos @ np.linalg.inv(c)
    fw = frac - np.floor(frac)
    face = face_distances(c)
    own = owners(pos, c, grid) == rank
    cd = slab_of_rank(dest, grid)
    out = []
    rng = [(-1, 0, 1) if grid[a] > 1 else (0,) for a in range(3)]
    for i in np.nonzero(own)[0]:
        for sx in rng[0]:
            for sy in rng[1]:
                for sz in rng[2]:
                    s = (sx, sy, sz)
                    if dest == rank and s == (0, 0, 0):
                        continue
                    ok = True
                    for a in range(3):
                        if grid[a] == 1:
                            continue
                        d1 = width / face[a]
                        v = fw[i, a] + s[a]
                        ok &= (cd[a] / grid[a] - d1) <= v < ((cd[a] + 1) / grid[a] + d1)
                    if ok:
                        out.append((int(i), s))
    return out


# ---------------------------------------------------------------------------
# Collectives
# ---------------------------------------------------------------------------
class _DevBytes:
    """A device byte range as a zero-copy torch tensor (CUDA array interface)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (int(nbytes),), "typestr": "|u1", "data": (int(ptr), False),
                                         "version": 2, "strides": None}


def _bytes(torch, ptr: int, nbytes: int):
    if nbytes == 0:
        return torch.empty(0, dtype=torch.uint8, device="cuda")
    return torch.as_tensor(_DevBytes(ptr, nbytes), device="cuda")


class NcclComm:
    """The engine's collectives over a torch.distributed process group (NCCL):
    all_to_all_single and all_reduce, issued on the library's stream."""

    def __init__(self, group=None):
        import torch
        import torch.distributed as dist
        self.torch, self.dist, self.group = torch, dist, group
        self.world = dist.get_world_size(group)
        self._a2a = ALLTOALLV(self._alltoallv)
        self._ar = ALLREDUCE(self._allreduce)
        self.c = _CComm(None, self._a2a, self._ar)

    def _alltoallv(self, user, send, sc, recv, rc, eb, stream):
        try:
            torch = self.torch
            s = [int(sc[r]) * eb for r in range(self.world)]
            r_ = [int(rc[r]) * eb for r in range(self.world)]
            st = torch.cuda.ExternalStream(int(stream))
            with torch.cuda.stream(st):
                self.dist.all_to_all_single(_bytes(torch, recv, sum(r_)), _bytes(torch, send, sum(s)), r_, s,
                                            group=self.group)
            return 0
        except Exception:  # noqa: BLE001 - the engine raises the error
            traceback.print_exc(file=sys.stderr)
            return 1

    def _allreduce(self, user, buf, n, stream):
        try:
            torch = self.torch
            st = torch.cuda.ExternalStream(int(stream))
            with torch.cuda.stream(st):
                t = _bytes(torch, buf, 8 * n).view(torch.float64)
                self.dist.all_reduce(t, group=self.group)
            return 0
        except Exception:  # noqa: BLE001
            traceback.print_exc(file=sys.stderr)
            return 1


class LocalComm:
    """The engine's collectives between `world` threads of one process, each
    driving one rank's engine on the same GPU (tests that emulate several
    ranks).  Each exchange synchronises the caller's stream, meets the other
    threads at a barrier (with a timeout, so a failing rank cannot hang the
    others) and copies its incoming segments from the senders' buffers."""

    def __init__(self, world: int, timeout: float = 300.0):
        import torch
        self.torch = torch
        self.world = world
        self.barrier = threading.Barrier(world, timeout=timeout)
        self.posts = [None] * world
        self._keep = []

    def for_rank(self, rank: int) -> _CComm:
        a2a = ALLTOALLV(lambda u, s, sc, r, rc, eb, st: self._alltoallv(rank, s, sc, r, rc, eb, st))
        ar = ALLREDUCE(lambda u, b, n, st: self._allreduce(rank, b, n, st))
        self._keep += [a2a, ar]
        return _CComm(None, a2a, ar)

    def _alltoallv(self, rank, send, sc, recv, rc, eb, stream):
        torch = self.torch
        try:
            torch.cuda.ExternalStream(int(stream)).synchronize()
            self.posts[rank] = (int(send or 0), [int(sc[r]) for r in range(self.world)])
            self.barrier.wait()
            off = 0
            for r in range(self.world):
                sp, scr = self.posts[r]
                n = scr[rank] * eb
                if n != int(rc[r]) * eb:
                    raise RuntimeError("alltoallv counts disagree")
                if n:
                    src_off = sum(scr[:rank]) * eb
                    _bytes(torch, recv + off, n).copy_(_bytes(torch, sp + src_off, n))
                off += n
            torch.cuda.synchronize()
            self.barrier.wait()
            return 0
        except Exception:  # noqa: BLE001
            traceback.print_exc(file=sys.stderr)
            self.barrier.abort()
            return 1

    def _allreduce(self, rank, buf, n, stream):
        torch = self.torch
        try:
            torch.cuda.ExternalStream(int(stream)).synchronize()
            self.posts[rank] = _bytes(torch, buf, 8 * n).view(torch.float64).clone()
            self.barrier.wait()
            total = sum(p.to(torch.float64) for p in self.posts)
            self.barrier.wait()
            _bytes(torch, buf, 8 * n).view(torch.float64).copy_(total)
            torch.cuda.synchronize()
            self.barrier.wait()
            return 0
        except Exception:  # noqa: BLE001
            traceback.print_exc(file=sys.stderr)
            self.barrier.abort()
            return 1


# ---------------------------------------------------------------------------
# One rank's domain
# ---------------------------------------------------------------------------
class Domain:
    """This rank's part of one periodic cell (mlipcpp_b200_domain_*).

    `numbers` are the owned atoms' atomic numbers; each step takes their
    positions as a device float32 tensor [n_owned, 3] and returns the energy
    and virial of the whole cell (and writes the owned atoms' forces into
    `forces`, a device float32 tensor of the same shape, when given)."""

    def __init__(self, predictor, cell, grid, rank: int, comm: _CComm, skin: float = 0.0):
        from . import lib, _check
        self._lib, self._check = lib(), _check
        self._comm = comm
        c = np.ascontiguousarray(cell, np.float32).reshape(9)
        g = np.ascontiguousarray(grid, np.int32).reshape(3)
        self._h = self._lib.mlipcpp_b200_domain_create(predictor._h, c.ctypes.data, g.ctypes.data, int(rank),
                                                       float(skin), ctypes.byref(comm))
        if not self._h:
            from . import MLIPError, INVALID_PARAMETER
            msg = self._lib.mlipcpp_get_last_error()
            raise MLIPError(INVALID_PARAMETER, (msg or b"domain set-up failed").decode())
        self.predictor = predictor  # keeps the model alive
        self.grid, self.rank = tuple(int(x) for x in grid), int(rank)
        self.cell = np.asarray(cell, np.float64).reshape(3, 3)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            try:
                self._lib.mlipcpp_b200_domain_free(h)
            except Exception:  # noqa: BLE001
                pass
            self._h = None

    def set_atoms(self, numbers):
        z = np.ascontiguousarray(numbers, np.int32)
        self._check(self._lib.mlipcpp_b200_domain_set_atoms(self._h, int(z.shape[0]), z.ctypes.data))
        self.n_owned = int(z.shape[0])

    def step(self, positions, forces=None, compute_forces: bool = True):
        e = ctypes.c_double()
        v = np.zeros(6, np.float64)
        self._check(self._lib.mlipcpp_b200_domain_step(
            self._h, ctypes.c_void_p(positions.data_ptr() if self.n_owned else 0),
            ctypes.c_void_p(forces.data_ptr()) if forces is not None else None, bool(compute_forces),
            ctypes.byref(e), v.ctypes.data))
        return float(e.value), v

    def stats(self) -> dict:
        a = np.zeros(13, np.float64)
        self._check(self._lib.mlipcpp_b200_domain_stats(self._h, a.ctypes.data))
        keys = ["halo_ms", "neighbors_requests_ms", "model_ms", "force_halo_ms", "sum_ms", "step_ms",
                "host_ms", "owned", "ghosts", "edges", "token_rows_in", "token_rows_out", "halo_copies_out"]
        return {k: (float(x) if k.endswith("ms") else int(x)) for k, x in zip(keys, a)}

    def stress(self, virial) -> np.ndarray:
        """Voigt stress = virial / |det cell| (pet.cpp:1079-1097)."""
        vol = abs(float(np.linalg.det(self.cell)))
        return (np.asarray(virial) / vol).astype(np.float32)


def run_emulated(make_predictor, structure, grid, skin: float = 0.0, steps: int = 1, compute_forces=True,
                 comm=None):
    """Evaluates `structure` (periodic) split over prod(grid) emulated ranks on
    the current GPU: one thread, one model (make_predictor()) and one engine
    per rank, exchanging through `comm` (default: a new LocalComm).  Returns
    (energy, forces [N, 3], virial, per-rank stats) of the last step; raises
    the first rank's error if any rank's step fails."""
    import torch
    world = int(np.prod(grid))
    own = owners(structure.positions, structure.cell, grid)
    comm = comm or LocalComm(world)
    doms, idx = [], []
    for r in range(world):
        d = Domain(make_predictor(), structure.cell, grid, r, comm.for_rank(r), skin)
        ix = np.nonzero(own == r)[0]
        d.set_atoms(structure.numbers[ix])
        doms.append(d)
        idx.append(ix)
    out = [None] * world
    errors = []

    def run(r):
        try:
            pos = torch.from_numpy(np.ascontiguousarray(structure.positions[idx[r]], np.float32)).cuda()
            F = torch.zeros_like(pos)
            for _ in range(steps):
                e, v = doms[r].step(pos, F, compute_forces)
            out[r] = (e, F.cpu().numpy(), v, doms[r].stats())
        except Exception as ex:  # noqa: BLE001
            errors.append(ex)
            comm.barrier.abort()

    th = [threading.Thread(target=run, args=(r,)) for r in range(world)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    if errors:
        raise errors[0]
    forces = np.zeros((structure.n_atoms, 3), np.float32)
    for r in range(world):
        forces[idx[r]] = out[r][1]
    return out[0][0], forces, out[0][2], [o[3] for o in out]
