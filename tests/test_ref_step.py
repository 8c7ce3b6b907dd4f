"""The reference's own data-parallel training step on the host cores (oracle/ref_step.py),
which bench.py times as the CPU baseline and as the `--impl reference` arm.  Checked on
a small batch: the shard gradients it sums are the whole-batch gradients of the CPU
restatement (GEMM tolerance), the loss is the whole-batch loss, and the update is the
reference SGD's float32 p - lr * g.  Skipped where the reference library was not built."""

import numpy as np
import pytest

from parity import GEMM_FROB_RTOL, assert_norm

import tinytensor_b200 as tt
from oracle import oracle as O
from oracle import ref_step

pytestmark = pytest.mark.skipif(not ref_step.available(), reason="oracle/_ref/libttref.so not built")


def _xavier(rng, fi, fo):
    lim = np.sqrt(6.0 / (fi + fo))
    return rng.uniform(-lim, lim, (fi, fo)).astype(np.float32)


def test_reference_step_is_the_whole_batch_sgd_step():
    rows, P = 32, 4
    rng = np.random.default_rng(4)
    x = rng.standard_normal((rows, 1024)).astype(np.float32)
    t = rng.standard_normal((rows, 10)).astype(np.float32)
    w0 = [_xavier(rng, 1024, 4096), _xavier(rng, 4096, 4096), _xavier(rng, 4096, 10)]
    rs = ref_step.ReferenceStep(x, t, w0, lr=0.01, processes=P)
    try:
        assert rs.P == P
        rs.step()
        grads = rs.mean_gradients()
        gsums = [s.copy() for s in rs.gradient_sums()]
        w1 = rs.weights()
        loss = rs.last["loss"]
    finally:
        rs.close()

    g = tt.Graph()
    X, T = g.input([rows, 1024], name="X"), g.input([rows, 10], name="T")
    W1, W2, W3 = g.input([1024, 4096], name="W1"), g.input([4096, 4096], name="W2"), g.input([4096, 10], name="W3")
    d = tt.tanh(tt.relu(X @ W1) @ W2) @ W3 - T
    lossn = tt.mean(d * d)
    feed = {X: x, T: t, W1: w0[0], W2: w0[1], W3: w0[2]}
    ref_g = O.gradients(g, lossn, feed, [W1, W2, W3])
    ref_loss = O.evaluate(g, feed, [lossn])[0]
    np.testing.assert_allclose(loss, ref_loss, rtol=1e-5)
    for got, r in zip(grads, ref_g):
        assert_norm(got, r, GEMM_FROB_RTOL)
    # the update the parent applies: p - (lr / P) * (sum of shard gradients), float32
    for a, b, gs in zip(w1, w0, gsums):
        np.testing.assert_array_equal(a, b - np.float32(0.01 / P) * gs)


def test_reference_step_needs_equal_shards():
    """The process count drops to a divisor of the batch so shards stay equal (the mean
    of shard means is then the batch mean)."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal((6, 1024)).astype(np.float32)
    t = rng.standard_normal((6, 10)).astype(np.float32)
    w = [np.zeros((1024, 4096), np.float32), np.zeros((4096, 4096), np.float32), np.zeros((4096, 10), np.float32)]
    rs = ref_step.ReferenceStep(x, t, w, processes=4)
    try:
        assert rs.P == 3 and rs.rows == 6
    finally:
        rs.close()
