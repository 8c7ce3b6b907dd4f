"""Seeded parity cases shared by the golden-vector generator (make_golden.py), the
oracle pin tests and the GPU parity tests.

Each case builds a tinytensor_b200 Graph and its feed.  Shapes follow the
reference's own tests (tests/python/test_differential.py, test_compiler.py,
tests/cpp/codegen/test_codegen.cpp): prime lengths, broadcasting, transposed
operands, batched matmul, reductions with and without keepdims, small MLPs.
Cases marked `ref_ok=False` use ops the reference has no OpType for (exp, tanh,
neg, reduce_max); their golden outputs come from the reference through op
identities and are compared with the looser `ident_tol`.
"""

import numpy as np

import tinytensor_b200 as tt


def _n(rng, *shape):
    return rng.standard_normal(shape).astype(np.float32)


def _u(rng, *shape):
    return rng.uniform(-1, 1, shape).astype(np.float32)


CASES = {}


def case(name, kind="forward", ref_ok=True, exact=False):
    def deco(fn):
        CASES[name] = dict(fn=fn, kind=kind, ref_ok=ref_ok, exact=exact)
        return fn
    return deco


# ---- elementwise (reference test_differential.py:7-60, 155-196) ----
@case("add_shapes", exact=True)
def _c(seed=1):
    rng = np.random.default_rng(seed)
    g = tt.Graph()
    a1, b1 = g.input([10]), g.input([10])
    a2, b2 = g.input([4, 5]), g.input([4, 5])
    a3, b3 = g.input([2, 3, 4]), g.input([2, 3, 4])
    outs = [a1 + b1, a2 + b2, a3 + b3, a1 * b1, a2 - b2, a3 / (b3 * b3 + 0.5)]
    feed = {n: _n(rng, *n.shape) for n in g.inputs}
    return g, feed, outs


@case("broadcast_ops", exact=True)
def _c(seed=2):
    rng = np.random.default_rng(seed)
    g = tt.Graph()
    a = g.input([3, 1, 4])
    b = g.input([1, 5, 4])
    c = g.input([4])
    d = g.input([])
    outs = [a + b, a * c, (a - b) / (c * c + 1.0), a * d + c, d - b]
    feed = {n: _n(rng, *n.shape) for n in g.inputs}
    return g, feed, outs


@case("prime_tail", exact=True)
def _c(seed=3):
    # test_codegen.cpp:45-78: prime length 37 exercises vector tails
    rng = np.random.default_rng(seed)
    g = tt.Graph()
    a, b = g.input([37]), g.input([37])
    c = g.input([37, 37])
    outs = [tt.relu(a + b), tt.relu(c * a - b)]
    feed = {n: _n(rng, *n.shape) for n in g.inputs}
    return g, feed, outs


@case("fused_chain_small", ref_ok=False)
def _c(seed=0):
    # the fused chain relu(a*b + c)*0.5 - exp(-a) at a small shape
    rng = np.random.default_rng(seed)
    g = tt.Graph()
    a, b, c = g.input([64, 96]), g.input([64, 96]), g.input([1, 96])
    y = tt.relu(a * b + c) * 0.5 - tt.exp(-a)
    feed = {a: _n(rng, 64, 96), b: _n(rng, 64, 96), c: _n(rng, 1, 96)}
    return g, feed, [y]


@case("sigmoid_chain")
def _c(seed=4):
    rng = np.random.default_rng(seed)
    g = tt.Graph()
    x = g.input([33, 17])
    w = g.input([17])
    y = tt.sigmoid(x * w) - tt.sigmoid(x / (w * w + 1.0))
    feed = {x: 8 * _n(rng, 33, 17), w: _n(rng, 17)}
    return g, feed, [y]


@case("transposed_elementwise", exact=True)
def _c(seed=5):
    rng = np.random.default_rng(seed)
    g = tt.Graph()
    a = g.input([24, 40])
    b = g.input([40, 24])
    outs = [tt.transpose(a, 0, 1) + b, tt.relu(tt.transpose(b, 1, 0) * a), tt.transpose(a, 0, 1)]
    feed = {n: _n(rng, *n.shape) for n in g.inputs}
    return g, feed, outs


# ---- reductions (test_differential.py:78-94, test_codegen.cpp:180-217) ----
@case("reductions")
def _c(seed=6):
    rng = np.random.default_rng(seed)
    g = tt.Graph()
    x = g.input([48, 80])
    z = g.input([6, 10, 12])
    outs = [tt.sum(x, [1]), tt.mean(x, [1]), tt.sum(x, [0]), tt.mean(x, [0], keepdims=True),
            tt.sum(tt.transpose(x, 0, 1), [0]), tt.sum(x), tt.mean(x),
            tt.sum(z, [1]), tt.mean(z, [0, 2], keepdims=True), tt.sum(z, [-1]), tt.sum(tt.transpose(z, 0, 2), [1, 2])]
    feed = {x: _u(rng, 48, 80), z: _u(rng, 6, 10, 12)}
    return g, feed, outs


@case("reduce_max", ref_ok=False)
def _c(seed=7):
    rng = np.random.default_rng(seed)
    g = tt.Graph()
    x = g.input([40, 72])
    z = g.input([5, 9, 7])
    outs = [tt.max(x, [1]), tt.max(x, [0]), tt.max(tt.transpose(x, 0, 1), [0]), tt.max(z, [1], keepdims=True),
            tt.max(x)]
    feed = {x: _u(rng, 40, 72), z: _u(rng, 5, 9, 7)}
    return g, feed, outs


# ---- matmul (test_differential.py:62-76, 198-215; test_codegen.cpp:80-156) ----
@case("matmul_shapes")
def _c(seed=8):
    rng = np.random.default_rng(seed)
    g = tt.Graph()
    outs = []
    for (m, k, n) in [(8, 16, 12), (32, 32, 32), (3, 7, 5), (37, 33, 29), (130, 70, 150)]:
        a, b = g.input([m, k]), g.input([k, n])
        outs.append(a @ b)
    feed = {n: _n(rng, *n.shape) for n in g.inputs}
    return g, feed, outs


@case("matmul_transposed")
def _c(seed=9):
    rng = np.random.default_rng(seed)
    g = tt.Graph()
    a = g.input([4, 6])
    b = g.input([4, 5])
    c = g.input([40, 24])
    d = g.input([56, 24])
    outs = [tt.transpose(a, 0, 1) @ b, c @ tt.transpose(d, 0, 1), tt.transpose(c, 0, 1) @ tt.transpose(tt.transpose(c, 0, 1), 0, 1)]
    feed = {n: _n(rng, *n.shape) for n in g.inputs}
    return g, feed, outs


@case("matmul_batched")
def _c(seed=10):
    rng = np.random.default_rng(seed)
    g = tt.Graph()
    a, b = g.input([2, 3, 4]), g.input([2, 4, 2])
    c, d = g.input([3, 5, 8]), g.input([8, 6])
    outs = [a @ b, c @ d]
    feed = {n: _n(rng, *n.shape) for n in g.inputs}
    return g, feed, outs


# ---- gradients (test_autodiff.py, test_differential.py:96-152) ----
@case("grad_mlp_bias", kind="grad")
def _c(seed=11):
    rng = np.random.default_rng(seed)
    g = tt.Graph()
    x = g.input([16, 12])
    w1, b1 = g.input([12, 20]), g.input([20])
    w2, b2 = g.input([20, 3]), g.input([3])
    h = tt.relu(x @ w1 + b1)
    y = h @ w2 + b2
    loss = tt.mean(y)
    feed = {n: _n(rng, *n.shape) for n in g.inputs}
    return g, feed, loss, [x, w1, b1, w2, b2]


@case("grad_elementwise", kind="grad")
def _c(seed=12):
    rng = np.random.default_rng(seed)
    g = tt.Graph()
    a, b = g.input([7, 9]), g.input([9])
    c = g.input([7, 1])
    loss = tt.sum(tt.sigmoid(a * b) / (c * c + 1.0) - a)
    feed = {n: _n(rng, *n.shape) for n in g.inputs}
    return g, feed, loss, [a, b, c]


@case("grad_mse_tanh", kind="grad", ref_ok=False)
def _c(seed=13):
    # the benchmark MLP's structure at a small size: relu, tanh, linear, MSE
    rng = np.random.default_rng(seed)
    g = tt.Graph()
    x, t = g.input([32, 24]), g.input([32, 5])
    w1, w2, w3 = g.input([24, 40]), g.input([40, 40]), g.input([40, 5])
    h1 = tt.relu(x @ w1)
    h2 = tt.tanh(h1 @ w2)
    d = h2 @ w3 - t
    loss = tt.mean(d * d)
    feed = {x: _n(rng, 32, 24), t: _n(rng, 32, 5), w1: 0.2 * _n(rng, 24, 40), w2: 0.2 * _n(rng, 40, 40),
            w3: 0.2 * _n(rng, 40, 5)}
    return g, feed, loss, [w1, w2, w3]


def build(name):
    c = CASES[name]
    res = c["fn"]()
    if c["kind"] == "forward":
        g, feed, outs = res
        return dict(graph=g, feed=feed, outputs=outs, **{k: c[k] for k in ("kind", "ref_ok", "exact")})
    g, feed, loss, wrt = res
    return dict(graph=g, feed=feed, loss=loss, wrt=wrt, **{k: c[k] for k in ("kind", "ref_ok", "exact")})
