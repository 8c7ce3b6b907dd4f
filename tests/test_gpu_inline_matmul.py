"""GPU parity of small-K matmuls evaluated inside the fused region of their readers.

A 2-D matmul with K <= 16 whose readers are all elementwise nodes of its shape is not a
GEMM launch: the region computes each element as a K-term fmaf chain over a row of A and
a column of B (the small-K GEMM kernel's own sum), so the product is never stored.  The
cases run the plain (flat) region kernel and the tiled one that also writes GEMM operand
copies, with transposed operands and an operand that is itself a region's output;
results are compared against the oracle's fp32 matmul and elementwise ops at the GEMM
tolerance."""

import numpy as np
import pytest

from parity import GEMM_FROB_RTOL, assert_norm

import tinytensor_b200 as tt
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _data(rng, shape, scale=1.0):
    return (rng.standard_normal(shape) * scale).astype(np.float32)


@pytest.mark.parametrize("k", [1, 4, 10, 16])
def test_small_k_product_inside_a_flat_region(k, cache_dir):
    rng = np.random.default_rng(60 + k)
    a, b, c = _data(rng, (300, k)), _data(rng, (k, 520)), _data(rng, (300, 520))
    g = tt.Graph()
    na, nb, nc = g.input([300, k]), g.input([k, 520]), g.input([300, 520])
    prog = tt.compile(g, outputs=[(na @ nb) * nc - nc], cache_dir=cache_dir)
    plan = prog.execution_plan()
    assert "gemm/" not in plan and "fused[matmul," in plan, plan
    got = prog.run({na: a, nb: b, nc: c}).numpy()
    ref = O.binary(O.SUB, O.binary(O.MUL, O.matmul(a, b), c), c)
    assert_norm(got, ref, GEMM_FROB_RTOL)


def test_small_k_product_with_transposed_operands(cache_dir):
    rng = np.random.default_rng(71)
    at, bt, c = _data(rng, (10, 258)), _data(rng, (646, 10)), _data(rng, (258, 646))
    g = tt.Graph()
    na, nb, nc = g.input([10, 258]), g.input([646, 10]), g.input([258, 646])
    y = tt.relu(tt.transpose(na, 0, 1) @ tt.transpose(nb, 0, 1) + nc)
    prog = tt.compile(g, outputs=[y], cache_dir=cache_dir)
    assert "gemm/" not in prog.execution_plan()
    got = prog.run({na: at, nb: bt, nc: c}).numpy()
    ref = O.unary(O.RELU, O.binary(O.ADD, O.matmul(np.ascontiguousarray(at.T), np.ascontiguousarray(bt.T)), c))
    assert_norm(got, ref, GEMM_FROB_RTOL)


def test_small_k_product_feeding_gemm_copies(cache_dir):
    """dZ = (dY @ W^T) * (1 - y^2) read by two tensor-core GEMMs, as in the MLP backward
    pass: the region forms the K=10 product inline and writes the GEMMs' operand copies;
    dY is itself a region output."""
    rng = np.random.default_rng(73)
    t, w, y = _data(rng, (1024, 10)), _data(rng, (512, 10), 0.1), np.tanh(_data(rng, (1024, 512))).astype(np.float32)
    h, v = _data(rng, (1024, 384)), _data(rng, (512, 256), 1 / np.sqrt(512))
    g = tt.Graph()
    nt, nw, ny, nh, nv = (g.input(list(a.shape)) for a in (t, w, y, h, v))
    dy = tt.relu(nt) * 2.0
    dz = (dy @ tt.transpose(nw, 0, 1)) * (1.0 - ny * ny)
    outs = [tt.transpose(nh, 0, 1) @ dz, dz @ nv]
    prog = tt.compile(g, outputs=outs, cache_dir=cache_dir)
    plan = prog.execution_plan()
    assert "simt_smallk" not in plan and "fused[matmul," in plan and "(writes hi/lo of X and X^T, not X)" in plan, plan
    g1, g2 = (r.numpy() for r in prog.run({nt: t, nw: w, ny: y, nh: h, nv: v}))
    dyr = O.binary(O.MUL, O.unary(O.RELU, t), np.float32(2.0))
    one_m = O.binary(O.SUB, np.float32(1.0), O.binary(O.MUL, y, y))
    dzr = O.binary(O.MUL, O.matmul(dyr, np.ascontiguousarray(w.T)), one_m)
    assert_norm(g1, O.matmul(np.ascontiguousarray(h.T), dzr), GEMM_FROB_RTOL)
    assert_norm(g2, O.matmul(dzr, v), GEMM_FROB_RTOL)


def test_small_k_product_that_is_an_output_stays_a_gemm(cache_dir):
    rng = np.random.default_rng(79)
    a, b = _data(rng, (300, 8)), _data(rng, (8, 256))
    g = tt.Graph()
    na, nb = g.input([300, 8]), g.input([8, 256])
    m = na @ nb
    prog = tt.compile(g, outputs=[m, m * 3.0], cache_dir=cache_dir)
    assert "simt_smallk" in prog.execution_plan()
    gm, g3 = (r.numpy() for r in prog.run({na: a, nb: b}))
    mr = O.matmul(a, b)
    assert_norm(gm, mr, GEMM_FROB_RTOL)
    assert_norm(g3, mr * np.float32(3.0), GEMM_FROB_RTOL)
