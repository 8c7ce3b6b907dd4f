"""Skinny products formed in the epilogue of the GEMM that produced their operand.

P = act(X.W) . V with V [N][Q] (Q <= 16) a graph input: the CTA-pair tensor-core GEMM
forming act(X.W) also sums each half tile's 128 columns against the matching rows of V
and writes partial slices; P's launch only adds the slices in order.  Each case checks
the plan and compares P (and the intermediate, where it is an output) with the oracle's
fp32 matmuls at the GEMM tolerance.  Shapes include partial tiles in both dimensions."""

import numpy as np
import pytest

from parity import GEMM_FROB_RTOL, assert_norm

import tinytensor_b200 as tt
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,k,n,q,act,inter_out", [
    (512, 300, 520, 10, "tanh", False),     # the output layer's shape class, partial last N tile
    (300, 256, 768, 1, "relu", False),      # partial last M tile, one output column
    (640, 128, 256, 16, "none", True),      # widest side product; the intermediate is an output
    (4096, 1024, 4096, 10, "tanh", False),  # MLP widths at 4096 rows
])
def test_side_product_matches_oracle(m, k, n, q, act, inter_out, cache_dir):
    rng = np.random.default_rng(m + k + n + q)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = (rng.standard_normal((k, n)) / np.sqrt(k)).astype(np.float32)
    v = (rng.standard_normal((n, q)) / np.sqrt(n)).astype(np.float32)
    g = tt.Graph()
    nx, nw, nv = g.input([m, k]), g.input([k, n]), g.input([n, q])
    h = nx @ nw
    h = {"tanh": tt.tanh, "relu": tt.relu, "none": lambda t: t}[act](h)
    p = h @ nv
    prog = tt.compile(g, outputs=[p, h] if inter_out else [p], cache_dir=cache_dir)
    plan = prog.execution_plan()
    assert "(+ side product [" in plan and "gemm/side_product[" in plan, plan
    res = prog.run({nx: x, nw: w, nv: v})
    got = [t.numpy() for t in res] if inter_out else [res.numpy()]
    href = O.matmul(x, w)
    if act == "tanh":
        href = O.unary(O.TANH, href)
    elif act == "relu":
        href = O.unary(O.RELU, href)
    assert_norm(got[0], O.matmul(href, v), GEMM_FROB_RTOL)
    if inter_out:
        assert_norm(got[1], href, GEMM_FROB_RTOL)


def test_side_product_repeated_runs_are_identical(cache_dir):
    """The slices are rewritten in full on every run and added in a fixed order: two runs
    give the same bits."""
    rng = np.random.default_rng(3)
    x = rng.standard_normal((1024, 512)).astype(np.float32)
    w = (rng.standard_normal((512, 1024)) / np.sqrt(512)).astype(np.float32)
    v = (rng.standard_normal((1024, 10)) / 32).astype(np.float32)
    g = tt.Graph()
    nx, nw, nv = g.input([1024, 512]), g.input([512, 1024]), g.input([1024, 10])
    prog = tt.compile(g, outputs=[tt.tanh(nx @ nw) @ nv], cache_dir=cache_dir)
    a = prog.run({nx: x, nw: w, nv: v}).numpy()
    b = prog.run({nx: x, nw: w, nv: v}).numpy()
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
