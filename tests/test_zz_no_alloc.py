"""mlipcpp_b200_neighbor_list_noalloc: the neighbour list into caller-owned
device buffers with the library's fixed static working memory.  Its pairs
must equal mlipcpp_b200_neighbor_list's (bit-exact: same kernels, same
order) on consecutive calls, which share the static array.  This file is
collected last so the GPU test also runs after every other test in one
process; it passes alone as well."""
import ctypes

import numpy as np
import pytest

import mlipcpp_b200 as mb
from mlipcpp_b200 import workloads as wl

MAX_ATOMS = 65536
ERR_INVALID = 7


def noalloc_fn():
    fn = mb.lib().mlipcpp_b200_neighbor_list_noalloc
    vp = ctypes.c_void_p
    fn.restype = ctypes.c_int64
    fn.argtypes = [ctypes.c_int32, vp, vp, vp, ctypes.c_float, ctypes.c_int64, vp, vp, vp, vp, vp, vp]
    return fn


def test_noalloc_rejects_oversized_request_before_device_work():
    n = MAX_ATOMS + 1
    cell = np.eye(3, dtype=np.float32).reshape(9) * 200.0
    pbc = np.ones(3, np.bool_)
    # the size check comes first, before pointer checks and any device access
    rc = noalloc_fn()(n, None, cell.ctypes.data, pbc.ctypes.data, 4.5, 0,
                      None, None, None, None, None, None)
    assert rc == -ERR_INVALID
    assert "65536" in mb.lib().mlipcpp_get_last_error().decode()
    # too many bins for the static array: a 400 A cube at 1 A cutoff
    cell = np.eye(3, dtype=np.float32).reshape(9) * 400.0
    rc = noalloc_fn()(8, None, cell.ctypes.data, pbc.ctypes.data, 1.0, 0,
                      None, None, None, None, None, None)
    assert rc == -ERR_INVALID
    assert "bins" in mb.lib().mlipcpp_get_last_error().decode()
    # a cutoff that is not finite and positive
    cell = np.eye(3, dtype=np.float32).reshape(9) * 20.0
    for bad in (0.0, -1.0, float("nan"), float("inf")):
        rc = noalloc_fn()(8, None, cell.ctypes.data, pbc.ctypes.data, bad, 0,
                          None, None, None, None, None, None)
        assert rc == -ERR_INVALID, bad
        assert "cutoff" in mb.lib().mlipcpp_get_last_error().decode()
    # a cutoff spanning more than 511 cell widths (bin offsets are 10-bit)
    cell = np.eye(3, dtype=np.float32).reshape(9) * 0.5
    rc = noalloc_fn()(1, None, cell.ctypes.data, pbc.ctypes.data, 300.0, 0,
                      None, None, None, None, None, None)
    assert rc == -ERR_INVALID
    assert "511" in mb.lib().mlipcpp_get_last_error().decode()


@pytest.mark.gpu
def test_noalloc_matches_neighbor_list_on_consecutive_calls():
    import torch
    fn = noalloc_fn()
    cases = [
        (wl.si_diamond(3, seed=51), (True, True, True), 4.5),
        (wl.fcc_alloy(8, seed=52), (True, True, True), 4.5),
        (wl.si_diamond(2, seed=53), (True, True, False), 3.0),
    ]
    cap = 200_000
    dev = torch.device("cuda", torch.cuda.current_device())
    d_pos = torch.empty(3 * 4096, dtype=torch.float32, device=dev)
    out = {"c": torch.empty(cap, dtype=torch.int32, device=dev),
           "n": torch.empty(cap, dtype=torch.int32, device=dev),
           "s": torch.empty(3 * cap, dtype=torch.int32, device=dev),
           "v": torch.empty(3 * cap, dtype=torch.float32, device=dev),
           "d": torch.empty(cap, dtype=torch.float32, device=dev)}
    stream = torch.cuda.current_stream()
    free_after_setup = None
    for k, (s, pbc, rc_) in enumerate(cases):
        ref = mb.neighbor_list(s.positions, s.cell, pbc, rc_)
        d_pos[:3 * s.n_atoms].copy_(torch.from_numpy(s.positions.reshape(-1)))
        torch.cuda.synchronize()
        for o in out.values():
            o.fill_(-7)
        torch.cuda.synchronize()
        if k > 0:
            free_before = torch.cuda.mem_get_info()[0]
        allocs_before = int(mb.lib().mlipcpp_b200_device_allocations())
        cell = np.ascontiguousarray(s.cell, np.float32).reshape(9)
        p = np.asarray(pbc, np.bool_)
        m = fn(s.n_atoms, d_pos.data_ptr(), cell.ctypes.data, p.ctypes.data, rc_, cap,
               out["c"].data_ptr(), out["n"].data_ptr(), out["s"].data_ptr(), out["v"].data_ptr(),
               out["d"].data_ptr(), stream.cuda_stream)
        assert m >= 0, mb.lib().mlipcpp_get_last_error()
        # the library's own count of its cudaMalloc calls does not move
        assert int(mb.lib().mlipcpp_b200_device_allocations()) == allocs_before
        if k > 0:
            # a loose second check on the device's free memory (other
            # processes on the same GPU can move it by a little)
            assert torch.cuda.mem_get_info()[0] >= free_before - (64 << 20)
        n_ref = len(ref["centers"])
        assert m == n_ref
        np.testing.assert_array_equal(out["c"][:m].cpu().numpy(), ref["centers"])
        np.testing.assert_array_equal(out["n"][:m].cpu().numpy(), ref["neighbors"])
        np.testing.assert_array_equal(out["s"][:3 * m].cpu().numpy().reshape(-1, 3), ref["cell_shifts"])
        np.testing.assert_array_equal(out["v"][:3 * m].cpu().numpy().reshape(-1, 3), ref["edge_vectors"])
        np.testing.assert_array_equal(out["d"][:m].cpu().numpy(), ref["distances"])
        assert int(out["c"][m].item()) == -7  # nothing written past the pairs

    # capacity below the pair count: the count comes back, nothing is written
    s, pbc, rc_ = cases[0]
    d_pos[:3 * s.n_atoms].copy_(torch.from_numpy(s.positions.reshape(-1)))
    out["c"].fill_(-7)
    torch.cuda.synchronize()
    cell = np.ascontiguousarray(s.cell, np.float32).reshape(9)
    p = np.asarray(pbc, np.bool_)
    m = fn(s.n_atoms, d_pos.data_ptr(), cell.ctypes.data, p.ctypes.data, rc_, 10,
           out["c"].data_ptr(), out["n"].data_ptr(), out["s"].data_ptr(), out["v"].data_ptr(),
           out["d"].data_ptr(), stream.cuda_stream)
    assert m == len(mb.neighbor_list(s.positions, s.cell, pbc, rc_)["centers"])
    assert bool((out["c"][:10] == -7).all())
