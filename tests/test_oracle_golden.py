"""Pins the CPU oracle (oracle/tt_oracle.c + oracle/oracle.py) to the reference:
golden vectors made by the reference itself (tests/golden/make_golden.py) and the
known-answer values of the reference's own tests.  No GPU needed."""

import os

import numpy as np
import pytest

from cases import CASES, build
from parity import IDENTITY_ATOL, IDENTITY_RTOL, assert_bitexact

import tinytensor_b200 as tt
from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _golden(name):
    return np.load(os.path.join(GOLDEN, f"{name}.npz"))


def _feed_from_golden(c, gold):
    feed = {}
    for i, n in enumerate(c["graph"].inputs):
        feed[n] = gold[f"in{i}"]
        np.testing.assert_array_equal(gold[f"in{i}"], np.asarray(c["feed"][n], np.float32))
    return feed


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_reference_golden(name):
    c = build(name)
    gold = _golden(name)
    feed = _feed_from_golden(c, gold)
    if c["kind"] == "forward":
        got = O.evaluate(c["graph"], feed, c["outputs"])
    else:
        got = O.gradients(c["graph"], c["loss"], feed, c["wrt"])
    for i, g in enumerate(got):
        ref = gold[f"out{i}"]
        if c["ref_ok"] or name == "reduce_max":
            # same operation order and rounding as the reference interpreter: bit-exact
            assert_bitexact(g, ref)
        else:
            np.testing.assert_allclose(g, ref, rtol=IDENTITY_RTOL, atol=IDENTITY_ATOL)


@pytest.mark.parametrize("name", sorted(n for n in CASES if CASES[n]["ref_ok"] and CASES[n]["kind"] == "forward"))
def test_ir_text_matches_reference_printer(name):
    c = build(name)
    for o in c["outputs"]:
        c["graph"].mark_output(o)
    assert c["graph"].to_ir() == str(_golden(name)["ir"])


# ---- known answers from the reference test suite --------------------------------------

def test_known_relu_alternating():
    # tests/cpp/codegen/test_codegen.cpp:22-43
    x = np.array([-5.0 if i % 2 == 0 else 5.0 for i in range(8)], np.float32)
    np.testing.assert_array_equal(O.unary(O.RELU, x), [0, 5, 0, 5, 0, 5, 0, 5])


def test_known_matmul_values():
    # test_codegen.cpp:80-100 (= 16) and :135-156 batched (= 12)
    assert np.all(O.matmul(np.ones((4, 8), np.float32), np.full((8, 6), 2.0, np.float32)) == 16.0)
    out = O.matmul(np.ones((2, 3, 4), np.float32), np.full((2, 4, 2), 3.0, np.float32))
    assert out.shape == (2, 3, 2) and np.all(out == 12.0)


def test_known_comprehensive_ops():
    # test_codegen.cpp:180-217: (10 - 2 + 2) / 2 = 5; sum over 4 -> 20; mean -> 5
    g = tt.Graph()
    a, b, c = g.input([2, 4]), g.input([2, 4]), g.input([4])
    q = tt.div(tt.add(tt.sub(a, b), c), c)
    tr = tt.transpose(q, 0, 1)
    outs = [tr, tt.sum(tr, [0]), tt.mean(tr, [0, 1])]
    feed = {a: np.full((2, 4), 10, np.float32), b: np.full((2, 4), 2, np.float32), c: np.full((4,), 2, np.float32)}
    r = O.evaluate(g, feed, outs)
    assert r[0].shape == (4, 2) and np.all(r[0] == 5.0)
    assert r[1].shape == (2,) and np.all(r[1] == 20.0)
    assert r[2].shape == () and r[2] == 5.0


def test_known_relu_ieee_contract():
    # tests/python/test_ieee754_edge_cases.py:72-127: NaN -> +0, -0 -> +0, +inf kept
    sub = np.nextafter(np.float32(0), np.float32(1))
    v = np.array([np.nan, np.inf, -np.inf, 0.0, -0.0, sub, -sub, 1e38, -1e38, 42.5, -42.5], np.float32)
    r = O.unary(O.RELU, v)
    assert r[0] == 0 and not np.signbit(r[0])
    assert np.isposinf(r[1]) and r[2] == 0
    assert r[4] == 0 and not np.signbit(r[4])
    assert r[5] == sub and r[6] == 0 and r[7] == np.float32(1e38) and r[9] == 42.5


def test_known_sigmoid_extremes():
    # test_ieee754_edge_cases.py:130-154
    r = O.unary(O.SIGMOID, np.array([100, -100, np.inf, -np.inf, 0, -0.0], np.float32))
    assert r[0] == 1.0 and 0 <= r[1] < 1e-12 and r[2] == 1.0 and r[3] == 0.0 and r[4] == 0.5 and r[5] == 0.5


def test_known_autodiff_values():
    # tests/python/test_autodiff.py:6-60
    g = tt.Graph()
    a, b = g.input([2]), g.input([2])
    loss = tt.sum(a * b)
    ga, gb = O.gradients(g, loss, {a: [3.0, 4.0], b: [5.0, 6.0]}, [a, b])
    np.testing.assert_array_equal(ga, [5, 6])
    np.testing.assert_array_equal(gb, [3, 4])
    g = tt.Graph()
    x = g.input([3])
    (gx,) = O.gradients(g, tt.sum(tt.relu(x)), {x: [-2.0, 0.0, 3.0]}, [x])
    np.testing.assert_array_equal(gx, [0, 0, 1])


def test_reduce_max_nan_propagates():
    x = np.array([[1, np.nan, 3], [4, 5, 6]], np.float32)
    r = O.reduce(O.REDUCE_MAX, x, [1])
    assert np.isnan(r[0]) and r[1] == 6


def test_reduce_max_signed_zeros_give_plus_zero_in_any_order():
    """IEEE 754-2019 maximum(): -0 < +0, so a cell holding both zeros is +0 whichever
    comes first in the walk; a cell of -0 alone stays -0."""
    x = np.array([[-0.0, 0.0, -0.0], [0.0, -0.0, -0.0], [-0.0, -0.0, -0.0], [-0.0, -0.0, 0.0]], np.float32)
    r = O.reduce(O.REDUCE_MAX, x, [1])
    assert r.tolist() == [0.0, 0.0, 0.0, 0.0]
    assert np.signbit(r).tolist() == [False, False, True, False]
    c = O.reduce(O.REDUCE_MAX, x, [0])
    assert np.signbit(c).tolist() == [False, False, False]


def test_sgd_matches_numpy_float32():
    rng = np.random.default_rng(0)
    p, g = rng.standard_normal(100).astype(np.float32), rng.standard_normal(100).astype(np.float32)
    new, _ = O.sgd(p, g, 0.01)
    np.testing.assert_array_equal(new, p - np.float32(0.01) * g)
    v = rng.standard_normal(100).astype(np.float32)
    new, nv = O.sgd(p, g, 0.01, 0.9, v)
    v2 = np.float32(0.9) * v + g
    np.testing.assert_array_equal(nv, v2)
    np.testing.assert_array_equal(new, p - np.float32(0.01) * v2)


@pytest.mark.skipif(not O.reference_available(), reason="oracle/_ref not built")
def test_oracle_matches_reference_larger_random():
    """Restatement vs the reference on a larger seeded graph (both CPU)."""
    rng = np.random.default_rng(42)
    g = tt.Graph()
    a, b, c = g.input([200, 130]), g.input([130, 70]), g.input([70])
    y = tt.relu(a @ b + c)
    outs = [y, tt.sum(y, [0]), tt.mean(tt.transpose(y, 0, 1), [1])]
    for o in outs:
        g.mark_output(o)
    feed = {a: rng.standard_normal((200, 130)).astype(np.float32), b: rng.standard_normal((130, 70)).astype(np.float32),
            c: rng.standard_normal(70).astype(np.float32)}
    ref = O.Reference().run(g, feed, mode="interpreted")
    for got, r in zip(O.evaluate(g, feed), ref):
        assert_bitexact(got, r)
