"""Replay of a captured CUDA graph for repeated same-shape predictions.

The second prediction with the same shapes in the same buffers captures the
model's launches into a graph and later ones replay it.  Results must equal
those of a model that always launches eagerly (MLIPCPP_B200_GRAPH=0), also
after the positions changed in place (a graph reads its buffers' contents
at replay) and after a change of shape (a new capture).  The launch counter
counts the graph's kernels on every replay."""
import numpy as np
import pytest

import mlipcpp_b200 as mb
from mlipcpp_b200 import workloads as wl

pytestmark = pytest.mark.gpu


def same(a, b, atol):
    assert abs(a.energy - b.energy) <= 1e-6 * max(1.0, abs(b.energy))
    np.testing.assert_allclose(a.forces, b.forces, rtol=0, atol=atol)
    np.testing.assert_allclose(a.stress, b.stress, rtol=0, atol=atol)


@pytest.fixture(scope="module")
def models(model_file):
    path = model_file("pet-mad-s", 7)
    mp = pytest.MonkeyPatch()
    mp.setenv("MLIPCPP_B200_GRAPH", "0")
    eager = mb.Predictor(path)
    mp.undo()
    return mb.Predictor(path), eager


def test_gpu_graph_replay_matches_eager(models):
    graph, eager = models
    s = wl.si_diamond(3, seed=11)
    ref = eager.predict(s.positions, s.numbers, s.cell, compute_stress=True)
    counts = []
    for _ in range(4):  # eager, capture, replay, replay
        k0 = mb.kernel_launches()
        got = graph.predict(s.positions, s.numbers, s.cell, compute_stress=True)
        counts.append(mb.kernel_launches() - k0)
        same(got, ref, 2e-6)
    assert counts[0] > 50
    assert len(set(counts)) == 1, counts

    # positions moved in place: same shapes, new contents
    rng = np.random.default_rng(3)
    for _ in range(3):
        pos = s.positions + rng.normal(0, 0.02, s.positions.shape).astype(np.float32)
        same(graph.predict(pos, s.numbers, s.cell, compute_stress=True),
             eager.predict(pos, s.numbers, s.cell, compute_stress=True), 2e-6)

    # another shape, then back: each is captured under its own key
    t = wl.si_diamond(2, seed=12)
    for _ in range(3):
        same(graph.predict(t.positions, t.numbers, t.cell, compute_stress=True),
             eager.predict(t.positions, t.numbers, t.cell, compute_stress=True), 2e-6)
    for _ in range(2):
        same(graph.predict(s.positions, s.numbers, s.cell, compute_stress=True), ref, 2e-6)


def test_gpu_graph_energy_only_and_batches(models):
    graph, eager = models
    mols = wl.molecules(6, seed=21)
    ref = eager.predict_batch([(m.positions, m.numbers) for m in mols])
    for _ in range(3):
        got = graph.predict_batch([(m.positions, m.numbers) for m in mols])
        for g, r in zip(got, ref):
            assert abs(g.energy - r.energy) <= 1e-6 * max(1.0, abs(r.energy))
            np.testing.assert_allclose(g.forces, r.forces, rtol=0, atol=2e-6)
    s = wl.si_diamond(2, seed=13)
    e_ref = eager.predict(s.positions, s.numbers, s.cell, compute_forces=False).energy
    for _ in range(3):
        e = graph.predict(s.positions, s.numbers, s.cell, compute_forces=False).energy
        assert abs(e - e_ref) <= 1e-6 * max(1.0, abs(e_ref))
