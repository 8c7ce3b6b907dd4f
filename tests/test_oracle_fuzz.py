"""Pins the CPU oracle to the reference beyond the golden cases: seeded random graphs
(broadcasting elementwise chains with scalar constants, IEEE special values, reductions
over random axes with and without keepdims, transposes, 2-D and batched matmuls) run
through the oracle restatement (oracle/tt_oracle.c) and through the reference's own
interpreter (oracle/_ref, built from the reference sources), compared bit for bit;
and random differentiable graphs whose gradients are compared with the reference's
Autodiff::compute_gradients (src/autodiff/gradient.cpp:52-332) bit for bit.
No GPU needed."""

import numpy as np
import pytest

from parity import assert_bitexact

import tinytensor_b200 as tt
from oracle import oracle as O

pytestmark = pytest.mark.skipif(not O.reference_available(), reason="oracle/_ref not built")

SPECIALS = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-38, -3e38, 1.0, -1.0], np.float32)


# without values near the float maximum: sums of products then never overflow, so their
# non-finite classes do not depend on the summation order
SPECIALS_NO_OVERFLOW = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-38, 1.0, -1.0], np.float32)


def _values(rng, shape, special, specials=SPECIALS):
    x = rng.standard_normal(shape).astype(np.float32) * np.float32(rng.choice([0.1, 1.0, 30.0]))
    if special and x.size:
        mask = rng.random(shape) < 0.15
        x[mask] = rng.choice(specials, size=int(mask.sum()))
    return x


def _derived(rng, base):
    """A shape that broadcasts against `base`: some dims set to 1, leading dims dropped."""
    s = [d if rng.random() < 0.6 else 1 for d in base]
    return s[int(rng.integers(0, len(s))):] if len(s) > 1 and rng.random() < 0.3 else s


def _elementwise_case(seed):
    rng = np.random.default_rng(seed)
    rank = int(rng.integers(1, 4))
    base = [int(rng.integers(1, 7)) for _ in range(rank)]
    g = tt.Graph()
    shapes = [base] + [_derived(rng, base) for _ in range(int(rng.integers(1, 3)))]
    ins = [g.input(s) for s in shapes]
    pool = list(ins)
    for _ in range(int(rng.integers(3, 8))):
        k = int(rng.integers(0, 8))
        a = pool[int(rng.integers(0, len(pool)))]
        b = pool[int(rng.integers(0, len(pool)))]
        if k == 0:
            y = a + b
        elif k == 1:
            y = a - b
        elif k == 2:
            y = a * b
        elif k == 3:
            y = a / b
        elif k == 4:
            y = tt.relu(a)
        elif k == 5:
            y = tt.sigmoid(a)
        elif k == 6:
            y = a * float(rng.choice([0.5, -2.0, 3.0]))
        else:
            y = a + float(rng.choice([1.0, -0.25]))
        pool.append(y)
    y = pool[-1]
    outs = [y]
    if len(y.shape) >= 2 and rng.random() < 0.4:
        d0, d1 = (int(v) for v in rng.choice(len(y.shape), size=2, replace=False))
        outs.append(tt.transpose(y, d0, d1))
    if len(y.shape) >= 1 and rng.random() < 0.7:
        nax = int(rng.integers(1, len(y.shape) + 1))
        axes = sorted(int(v) for v in rng.choice(len(y.shape), size=nax, replace=False))
        red = tt.sum if rng.random() < 0.5 else tt.mean
        outs.append(red(y, axes, keepdims=bool(rng.random() < 0.5)))
    for o in outs:
        g.mark_output(o)
    special = rng.random() < 0.5
    feed = {n: _values(rng, n.shape, special) for n in ins}
    return g, feed


def _matmul_case(seed, specials=SPECIALS):
    rng = np.random.default_rng(seed)
    m, k, n = (int(v) for v in rng.integers(1, 40, size=3))
    g = tt.Graph()
    if rng.random() < 0.3:
        bsz = int(rng.integers(1, 4))
        a, b = g.input([bsz, m, k]), g.input([bsz, k, n])
    else:
        a, b = g.input([m, k]), g.input([k, n])
    y = a @ b
    g.mark_output(y)
    if rng.random() < 0.5:
        g.mark_output(tt.relu(y + 0.5))
    if len(y.shape) == 2 and rng.random() < 0.5:
        g.mark_output(tt.sum(tt.transpose(y, 0, 1), [1]))
    special = rng.random() < 0.3
    feed = {x: _values(rng, x.shape, special, specials) for x in (a, b)}
    return g, feed


@pytest.mark.parametrize("seed", range(200))
def test_elementwise_and_reduction_graphs_match_reference_interpreter(seed):
    g, feed = _elementwise_case(1000 + seed)
    ref = O.Reference().run(g, feed, mode="interpreted")
    for got, r in zip(O.evaluate(g, feed), ref):
        assert_bitexact(got, r)


@pytest.mark.parametrize("seed", range(60))
def test_matmul_graphs_match_reference_interpreter(seed):
    g, feed = _matmul_case(5000 + seed)
    ref = O.Reference().run(g, feed, mode="interpreted")
    for got, r in zip(O.evaluate(g, feed), ref):
        assert_bitexact(got, r)


def _gradient_case(seed, specials=SPECIALS):
    """A random differentiable graph with a scalar loss: an elementwise chain over
    broadcasting inputs, or a two-layer perceptron with random activations, reduced by
    sum or mean over every axis."""
    rng = np.random.default_rng(seed)
    g = tt.Graph()
    if rng.random() < 0.5:
        rank = int(rng.integers(1, 4))
        base = [int(rng.integers(1, 6)) for _ in range(rank)]
        ins = [g.input(base)] + [g.input(_derived(rng, base)) for _ in range(int(rng.integers(1, 3)))]
        pool = list(ins)
        for _ in range(int(rng.integers(2, 6))):
            k = int(rng.integers(0, 7))
            a = pool[int(rng.integers(0, len(pool)))]
            b = pool[int(rng.integers(0, len(pool)))]
            y = (a + b, a - b, a * b, a / b, tt.relu(a), tt.sigmoid(a), a * 0.5)[k]
            pool.append(y)
        y = pool[-1]
        if len(y.shape) >= 2 and rng.random() < 0.3:
            y = tt.transpose(y, 0, len(y.shape) - 1) * 2.0
    else:
        m, k, h, n = (int(v) for v in rng.integers(1, 12, size=4))
        x, w1, b1, w2 = g.input([m, k]), g.input([k, h]), g.input([h]), g.input([h, n])
        ins = [x, w1, b1, w2]
        act = tt.relu if rng.random() < 0.5 else tt.sigmoid
        y = act(x @ w1 + b1) @ w2
        if rng.random() < 0.5:
            t = g.input([m, n])
            ins.append(t)
            y = (y - t) * (y - t)
    loss = tt.sum(y) if rng.random() < 0.5 else tt.mean(y)
    feed = {n: _values(rng, n.shape, rng.random() < 0.3, specials) for n in ins}
    reach, stack = set(), [loss]
    while stack:  # the inputs the loss depends on: the ones a gradient reaches
        n = stack.pop()
        if n.index not in reach:
            reach.add(n.index)
            stack.extend(n.inputs)
    return g, loss, [n for n in ins if n.index in reach], feed


@pytest.mark.parametrize("seed", range(80))
def test_gradients_match_reference_autodiff(seed):
    g, loss, wrt, feed = _gradient_case(9000 + seed)
    ref = O.Reference().gradients(g, loss, feed, wrt)
    for got, r in zip(O.gradients(g, loss, feed, wrt), ref):
        assert_bitexact(got, r)


@pytest.mark.parametrize("shape", [[], [0], [0, 3], [2, 0], [1], [3, 1, 2]])
def test_rank0_and_empty_shapes_match_reference_interpreter(shape):
    """Rank-0 values stay rank 0 and empty extents give the reference's shapes and values
    (sums of nothing are 0) through elementwise ops, scalar constants and reductions."""
    g = tt.Graph()
    a, b = g.input(shape), g.input(shape)
    y = tt.relu(a * b + 1.0)
    outs = [y, tt.sigmoid(y) - 0.5 * a]
    if shape:
        outs += [tt.sum(y, [0]), tt.mean(y, [0], keepdims=True)]
    outs += [tt.sum(y), tt.mean(y * b)]
    for o in outs:
        g.mark_output(o)
    feed = {a: np.full(shape, 2.0, np.float32), b: np.full(shape, -3.0, np.float32)}
    ref = O.Reference().run(g, feed, mode="interpreted")
    got = O.evaluate(g, feed)
    for x, r in zip(got, ref):
        assert_bitexact(x, r)


def _edge_graphs():
    """Shape edge cases of the reference's builders and kernels."""
    cases = {
        "negative transpose dims": lambda g: (lambda a: ([a], [tt.transpose(a, -1, 0), tt.transpose(a, 1, -1)]))(
            g.input([2, 3, 4])),
        "negative reduce axes": lambda g: (lambda a: ([a], [tt.sum(a, [-1]), tt.mean(a, [-3, -1], keepdims=True),
                                                             tt.sum(a, [0, 2])]))(g.input([2, 3, 4])),
        "zero extent broadcast": lambda g: (lambda a, b: ([a, b], [a + b]))(g.input([0, 1]), g.input([1, 5])),
        "matmul with K = 0": lambda g: (lambda a, b: ([a, b], [a @ b]))(g.input([4, 0]), g.input([0, 3])),
        "batched matmul, broadcast batch": lambda g: (lambda a, b: ([a, b], [a @ b]))(g.input([1, 3, 4]),
                                                                                      g.input([5, 4, 2])),
        "batched matmul, unequal batch ranks": lambda g: (lambda a, b: ([a, b], [a @ b]))(g.input([2, 1, 3, 4]),
                                                                                          g.input([5, 4, 2])),
        "x / 0": lambda g: (lambda a: ([a], [a / (a - a)]))(g.input([3])),
        "reduction of a transpose": lambda g: (lambda a: ([a], [tt.sum(tt.transpose(a, 0, 1), [0], keepdims=True)
                                                                 / 3.0]))(g.input([2, 3])),
    }
    return cases


@pytest.mark.parametrize("name", sorted(_edge_graphs()))
def test_shape_edge_cases_match_reference_interpreter(name):
    g = tt.Graph()
    ins, outs = _edge_graphs()[name](g)
    for o in outs:
        g.mark_output(o)
    rng = np.random.default_rng(7)
    feed = {n: rng.standard_normal(n.shape).astype(np.float32) for n in ins}
    ref = O.Reference().run(g, feed, mode="interpreted")
    for x, r in zip(O.evaluate(g, feed), ref):
        assert_bitexact(x, r)


def test_matmul_rank_rules_match_reference():
    g = tt.Graph()
    with pytest.raises(tt.DimensionError, match="Unsupported ranks for matmul"):
        g.input([3, 4]) @ g.input([4])
