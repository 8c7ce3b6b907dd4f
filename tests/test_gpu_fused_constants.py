"""GPU parity for graph forms the reference produces or gets wrong:

* the reference optimizer's FusedElementwise node "relu(<op>(@0, @1))"
  (src/optimizer/fusion.cpp:31-58), which the reference codegen computes as relu(a + b)
  whatever <op> is (src/codegen/cpp_backend.cpp:345-387) and its interpreter as add for
  div (src/runtime/interpreter.cpp:99-121).  Here the node must compute what it
  records: compared bit-exact with the oracle's evaluation of the unfused graph;
* constants: array constants (uploaded into the program's arena) and scalars that are
  not dyadic (1/3, 0.1), which the reference's compiled mode prints with 6 significant
  digits (cpp_backend.cpp:94-110).  Here they must be used bit-exactly;
* reduce_max over rows holding only signed zeros, in every layout, where the result
  must not depend on the order of the scan (-0 < +0).
"""

import numpy as np
import pytest

from parity import GEMM_FROB_RTOL, assert_bitexact, assert_elementwise_scaled, assert_norm

import tinytensor_b200 as tt
from oracle import oracle as O
from tinytensor_b200 import _lib

pytestmark = pytest.mark.gpu


def _fused_node(g, expr, inputs, shape):
    f = tt.graph.Node(g, _lib.OP_FUSED, list(shape), "float32", list(inputs))
    f.expr = expr
    return g._add(f)


def _operands(shape, seed):
    rng = np.random.default_rng(seed)
    a = rng.standard_normal(shape).astype(np.float32)
    b = rng.standard_normal(shape).astype(np.float32)
    # specials the reference's IEEE tests use: signed zeros, x/0, infinities, NaN
    flat_a, flat_b = a.reshape(-1), b.reshape(-1)
    flat_a[:6] = [0.0, -0.0, 1.0, -1.0, np.inf, np.nan]
    flat_b[:6] = [-0.0, 0.0, 0.0, 0.0, 2.0, 1.0]
    return a, b


@pytest.mark.parametrize("inner", ["add", "sub", "mul", "div"])
@pytest.mark.parametrize("shape", [(257, 129), (3, 5, 7), (4096, 1024)])
def test_reference_fused_node_binary_matches_unfused_oracle(inner, shape, cache_dir):
    a, b = _operands(shape, seed=31)
    g = tt.Graph()
    na, nb = g.input(list(shape)), g.input(list(shape))
    y = _fused_node(g, f"relu({inner}(@0, @1))", [na, nb], shape)
    got = tt.compile(g, outputs=[y], cache_dir=cache_dir).run({na: a, nb: b}).numpy()
    # the same computation as primitive nodes, on the oracle
    g2 = tt.Graph()
    ma, mb = g2.input(list(shape)), g2.input(list(shape))
    y2 = tt.relu(getattr(g2, inner)(ma, mb))
    ref = O.evaluate(g2, {ma: a, mb: b}, [y2])[0]
    assert_bitexact(got, ref)
    if inner != "add":
        # what the reference's fused codegen computes instead (relu(a + b)) differs
        assert not np.array_equal(got, np.maximum(a + b, 0).astype(np.float32))


def test_reference_fused_node_unary_inner(cache_dir):
    """relu(relu(@0, @1)) and relu(sigmoid(@0, @1)) carry one input (the reference's
    interpreter throws on the first: it reads inputs()[1])."""
    shape = (300, 70)
    a, _ = _operands(shape, seed=5)
    g = tt.Graph()
    na = g.input(list(shape))
    y1 = _fused_node(g, "relu(relu(@0, @1))", [na], shape)
    y2 = _fused_node(g, "relu(sigmoid(@0, @1))", [na], shape)
    got = [t.numpy() for t in tt.compile(g, outputs=[y1, y2], cache_dir=cache_dir).run({na: a})]
    g2 = tt.Graph()
    ma = g2.input(list(shape))
    r1, r2 = tt.relu(tt.relu(ma)), tt.relu(tt.sigmoid(ma))
    ref = O.evaluate(g2, {ma: a}, [r1, r2])
    assert_bitexact(got[0], ref[0])
    mag = O.magnitude(g2, {ma: a}, [r2])[0]
    assert_elementwise_scaled(got[1], ref[1], mag)


def test_fused_node_feeding_further_ops(cache_dir):
    """A fused node inside a larger region and feeding a reduction and a matmul."""
    rng = np.random.default_rng(8)
    a = rng.standard_normal((512, 256)).astype(np.float32)
    b = rng.standard_normal((512, 256)).astype(np.float32)
    w = (rng.standard_normal((256, 128)) / 16).astype(np.float32)
    g = tt.Graph()
    na, nb, nw = g.input([512, 256]), g.input([512, 256]), g.input([256, 128])
    f = _fused_node(g, "relu(mul(@0, @1))", [na, nb], (512, 256))
    e = f * 2.0 - na
    s = tt.sum(e, [1])
    p = e @ nw
    got = [t.numpy() for t in tt.compile(g, outputs=[e, s, p], cache_dir=cache_dir).run({na: a, nb: b, nw: w})]
    g2 = tt.Graph()
    ma, mb, mw = g2.input([512, 256]), g2.input([512, 256]), g2.input([256, 128])
    e2 = tt.relu(ma * mb) * 2.0 - ma
    ref = O.evaluate(g2, {ma: a, mb: b, mw: w}, [e2, tt.sum(e2, [1]), e2 @ mw])
    assert_bitexact(got[0], ref[0])
    assert_norm(got[1], ref[1], 1e-6)
    assert_norm(got[2], ref[2], GEMM_FROB_RTOL)


def test_non_dyadic_scalar_constants_bitexact(cache_dir):
    rng = np.random.default_rng(11)
    x = rng.standard_normal((1000, 333)).astype(np.float32)
    g = tt.Graph()
    nx = g.input([1000, 333])
    y = nx * (1.0 / 3.0) + 0.1
    z = (nx - 0.7) / 0.3
    got = [t.numpy() for t in tt.compile(g, outputs=[y, z], cache_dir=cache_dir).run({nx: x})]
    ref = O.evaluate(g, {nx: x}, [y, z])
    assert_bitexact(got[0], ref[0])
    assert_bitexact(got[1], ref[1])
    # float32(1/3) itself, not the 6-digit literal 0.333333
    third = np.float32(1.0 / 3.0)
    assert_bitexact(got[0], (x * third + np.float32(0.1)).astype(np.float32))
    assert not np.array_equal(got[0], (x * np.float32(0.333333) + np.float32(0.1)).astype(np.float32))
    if O.reference_available():
        # the reference interpreter keeps exact constants: same bits
        r = O.Reference().run(g, {nx: x}, mode="interpreted", outputs=[y, z])
        assert_bitexact(got[0], r[0])
        assert_bitexact(got[1], r[1])


def test_array_constants_in_regions_reductions_and_gemm(cache_dir):
    """[1,1024] and [64,64] constants (arena upload), non-dyadic entries, used by an
    elementwise region (broadcast), a reduction and a GEMM operand."""
    rng = np.random.default_rng(12)
    crow = (rng.standard_normal((1, 1024)) / 3.0).astype(np.float32)
    csq = (np.arange(64 * 64, dtype=np.float64).reshape(64, 64) / 7.0 + 0.1).astype(np.float32)
    x = rng.standard_normal((256, 1024)).astype(np.float32)
    m = rng.standard_normal((64, 64)).astype(np.float32)
    g = tt.Graph()
    nx, nm = g.input([256, 1024]), g.input([64, 64])
    kr, ks = g.constant(crow), g.constant(csq)
    y = nx * kr + kr                 # broadcast rows of a constant
    s = tt.sum(ks * nm, [0])         # constant inside a reduced region
    p = nm @ ks                      # constant as a GEMM operand
    q = tt.sum(kr, [1])              # reduction of a constant alone
    prog = tt.compile(g, outputs=[y, s, p, q], cache_dir=cache_dir)
    got = [t.numpy() for t in prog.run({nx: x, nm: m})]
    ref = O.evaluate(g, {nx: x, nm: m}, [y, s, p, q])
    assert_bitexact(got[0], ref[0])
    assert_norm(got[1], ref[1], 1e-6)
    assert_norm(got[2], ref[2], GEMM_FROB_RTOL)
    assert_norm(got[3], ref[3], 1e-6)
    # run twice: constants stay in place across runs
    got2 = [t.numpy() for t in prog.run({nx: x, nm: m})]
    for a, b in zip(got, got2):
        assert_bitexact(a, b)
    if O.reference_available():
        r = O.Reference().run(g, {nx: x, nm: m}, mode="interpreted", outputs=[y])
        assert_bitexact(got[0], r[0])


def test_reduce_max_signed_zeros_order_independent(cache_dir):
    """Rows of only +-0 in shuffled orders: +0 wherever a +0 occurs, -0 only for rows of
    -0 alone, in the row, column and generic (3-D) layouts and with split partials."""
    rng = np.random.default_rng(13)
    R, C = 640, 4096
    x = np.where(rng.random((R, C)) < 0.999, -0.0, 0.0).astype(np.float32)
    x[:64] = -0.0            # rows of -0 only
    x[64:96] = 0.0           # rows of +0 only
    x[96:128, :] = -0.0
    x[96:128, -1] = 0.0      # a single +0 at the end of the scan
    x[128:160, :] = -0.0
    x[128:160, 0] = 0.0      # ... and at the start
    g = tt.Graph()
    nx = g.input([R, C])
    outs = [tt.max(nx, [1]), tt.max(nx, [0]), tt.max(tt.transpose(nx, 0, 1), [0]), tt.max(nx)]
    got = [t.numpy() for t in tt.compile(g, outputs=outs, cache_dir=cache_dir).run({nx: x})]
    ref = O.evaluate(g, {nx: x}, outs)
    for a, b in zip(got, ref):
        assert_bitexact(a, b)
    assert np.signbit(got[0][:64]).all() and not np.signbit(got[0][64:160]).any()
    # 3-D generic layout
    x3 = x[:, :1024].reshape(40, 16, 1024)
    g3 = tt.Graph()
    n3 = g3.input([40, 16, 1024])
    outs3 = [tt.max(n3, [0, 2]), tt.max(n3, [1])]
    got3 = [t.numpy() for t in tt.compile(g3, outputs=outs3, cache_dir=cache_dir).run({n3: x3})]
    for a, b in zip(got3, O.evaluate(g3, {n3: x3}, outs3)):
        assert_bitexact(a, b)
