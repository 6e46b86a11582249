"""Failure detection on the GPU without a GPU fault (the reference checks
its graph's compute status, src/models/pet/pet.cpp:471-474, and no
exception crosses its C ABI, src/api/c/mlipcpp_api.cpp:475-481).

Every wait of the tensor-core GEMM pipeline is bounded.  A test hook
withholds the operand loads of one CTA of one GEMM launch, with the bound
lowered to 1 ms: that CTA's waits run out, it drains its own copies and
MMAs, frees its tensor memory and records a device error.  The prediction
must fail with MLIPCPP_ERROR_COMPUTATION and the same model's next
prediction must equal the one before, bit for bit (a leaked tensor-memory
allocation would stall the next launch instead)."""
import numpy as np
import pytest

import mlipcpp_b200 as mb
from mlipcpp_b200 import workloads as wl

pytestmark = pytest.mark.gpu


def test_gpu_gemm_wait_timeout_is_reported_and_the_model_recovers(model_file):
    L = mb.lib()
    pred = mb.Predictor(model_file("pet-mad-s", 3))
    s = wl.si_diamond(3, seed=41)
    before = pred.predict(s.positions, s.numbers, s.cell, compute_stress=True)
    try:
        assert L.mlipcpp_b200_set_wait_bound_ns(1_000_000) == mb.OK
        assert L.mlipcpp_b200_inject_gemm_stall() == mb.OK
        with pytest.raises(mb.MLIPError) as ei:
            pred.predict(s.positions, s.numbers, s.cell, compute_stress=True)
        assert ei.value.code == mb.COMPUTATION
        assert "timed out" in str(ei.value)
    finally:
        assert L.mlipcpp_b200_set_wait_bound_ns(0) == mb.OK
    after = pred.predict(s.positions, s.numbers, s.cell, compute_stress=True)
    assert np.float32(after.energy).tobytes() == np.float32(before.energy).tobytes()
    np.testing.assert_array_equal(after.forces.view(np.uint32), before.forces.view(np.uint32))
    np.testing.assert_array_equal(after.stress.view(np.uint32), before.stress.view(np.uint32))
    # a second model on the same device is unaffected as well
    other = mb.Predictor(model_file("pet-mad-s", 3)).predict(s.positions, s.numbers, s.cell,
                                                           compute_stress=True)
    np.testing.assert_array_equal(other.forces.view(np.uint32), before.forces.view(np.uint32))
