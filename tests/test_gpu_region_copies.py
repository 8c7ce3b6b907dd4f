"""GPU parity of tensor-core GEMMs that read hi/lo operand copies written by the
elementwise region that produced the operand (no pre-pass of their own).

When a region's stored [R][C] matrix X is a whole operand of later tensor-core GEMMs,
the region writes X's hi/lo copies itself: in X's layout for a GEMM that reads X along
its rows (A = X, or B = X^T), transposed for one that reads it across (A = X^T, or
B = X), and no fp32 X when nothing else reads it.  Each case checks the plan and
compares the GEMM's result against the oracle's fp32 elementwise op and matmul at the
GEMM tolerance; sizes include rows and columns that are not multiples of 4 or of the
region's 32 x 128 tiles."""

import numpy as np
import pytest

from parity import GEMM_FROB_RTOL, assert_norm, assert_bitexact

import tinytensor_b200 as tt
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _data(rng, shape, scale):
    return (rng.standard_normal(shape) * scale).astype(np.float32)


# X = a * b : [r, c]; `use` is how the GEMM reads X
CASES = [
    (1024, 512, "A=X"),
    (1024, 512, "A=Xt"),
    (1024, 512, "B=X"),
    (1024, 512, "B=Xt"),
    (646, 258, "A=X"),     # not multiples of 4 / 32 / 128
    (646, 258, "A=Xt"),
    (646, 258, "B=X"),
    (646, 258, "B=Xt"),
    (100, 1030, "A=Xt"),   # single-CTA reader (M <= 128) and a partial last row tile
]


@pytest.mark.parametrize("r,c,use", CASES)
def test_gemm_reads_region_copies(r, c, use, cache_dir):
    rng = np.random.default_rng(r + 5 * c + len(use))
    a, b = _data(rng, (r, c), 1.0), _data(rng, (r, c), 1.0)
    kdim = c if use in ("A=X", "B=Xt") else r
    y = _data(rng, (kdim, 320) if use.startswith("A") else (300, kdim), 1.0 / np.sqrt(kdim))
    g = tt.Graph()
    na, nb, ny = g.input([r, c]), g.input([r, c]), g.input(list(y.shape))
    x = na * nb
    out = {"A=X": lambda: x @ ny, "A=Xt": lambda: tt.transpose(x, 0, 1) @ ny,
           "B=X": lambda: ny @ x, "B=Xt": lambda: ny @ tt.transpose(x, 0, 1)}[use]()
    prog = tt.compile(g, outputs=[out], cache_dir=cache_dir)
    plan = prog.execution_plan()
    assert "(writes hi/lo of X" in plan and ", not X)" in plan, plan
    assert ("(A hi/lo from [0])" if use.startswith("A") else "(B hi/lo from [0])") in plan, plan
    got = prog.run({na: a, nb: b, ny: y}).numpy()
    xr = O.binary(O.MUL, a, b)
    ref = {"A=X": lambda: O.matmul(xr, y), "A=Xt": lambda: O.matmul(np.ascontiguousarray(xr.T), y),
           "B=X": lambda: O.matmul(y, xr), "B=Xt": lambda: O.matmul(y, np.ascontiguousarray(xr.T))}[use]()
    assert_norm(got, ref, GEMM_FROB_RTOL)


def test_region_output_also_read_elsewhere_keeps_fp32(cache_dir):
    """X feeds two GEMMs through its copies (both layouts) and is also a graph output
    and a reduction input: the region writes X in fp32 as well, bit-exact."""
    rng = np.random.default_rng(41)
    a, b = _data(rng, (768, 512), 1.0), _data(rng, (768, 512), 1.0)
    y1, y2 = _data(rng, (512, 192), 1 / np.sqrt(512)), _data(rng, (768, 160), 1 / np.sqrt(768))
    g = tt.Graph()
    na, nb, n1, n2 = g.input([768, 512]), g.input([768, 512]), g.input([512, 192]), g.input([768, 160])
    x = tt.relu(na - nb)
    outs = [x, x @ n1, tt.transpose(x, 0, 1) @ n2, tt.sum(x, [1])]
    prog = tt.compile(g, outputs=outs, cache_dir=cache_dir)
    plan = prog.execution_plan()
    assert "(writes hi/lo of X and X^T)" in plan, plan
    gx, g1, g2, gs = (t.numpy() for t in prog.run({na: a, nb: b, n1: y1, n2: y2}))
    xr = O.unary(O.RELU, O.binary(O.SUB, a, b))
    assert_bitexact(gx, xr)
    assert_norm(g1, O.matmul(xr, y1), GEMM_FROB_RTOL)
    assert_norm(g2, O.matmul(np.ascontiguousarray(xr.T), y2), GEMM_FROB_RTOL)
    assert_norm(gs, xr.astype(np.float64).sum(1), 1e-6)


def test_special_values_survive_the_copies(cache_dir):
    """NaN and inf in X reach the GEMM through the copies as the pre-pass would pass
    them: a row holding NaN gives NaN, a row holding inf gives the reference's signed
    infinities; the finite rows stay within tolerance."""
    rng = np.random.default_rng(43)
    a, b = _data(rng, (256, 256), 1.0), np.ones((256, 256), np.float32)
    a[3, 7] = np.nan
    a[9, 1] = np.inf
    y = _data(rng, (256, 128), 1 / 16)
    g = tt.Graph()
    na, nb, ny = g.input([256, 256]), g.input([256, 256]), g.input([256, 128])
    prog = tt.compile(g, outputs=[(na * nb) @ ny], cache_dir=cache_dir)
    assert "(A hi/lo from [0])" in prog.execution_plan()
    got = prog.run({na: a, nb: b, ny: y}).numpy()
    assert np.all(np.isnan(got[3])) and not np.any(np.isfinite(got[9]))
    ref9 = O.matmul(a[9:10], y)[0]
    assert np.array_equal(np.isnan(got[9]), np.isnan(ref9)) and np.array_equal(got[9][np.isinf(ref9)],
                                                                                   ref9[np.isinf(ref9)])
    keep = np.ones(256, bool)
    keep[[3, 9]] = False
    assert_norm(got[keep], O.matmul(a[keep], y), GEMM_FROB_RTOL)


@pytest.mark.parametrize("bshape", [(1, 520), (300, 1), ()])
def test_tiled_region_with_broadcast_operands(bshape, cache_dir):
    """The tiled region reads broadcast operands (a row vector, a column vector, a
    scalar constant) with their own strides; X = relu(a + b) * 0.5 feeds A = X^T."""
    rng = np.random.default_rng(47 + len(bshape))
    a = _data(rng, (300, 520), 1.0)
    y = _data(rng, (300, 96), 1 / np.sqrt(300))
    g = tt.Graph()
    na, ny = g.input([300, 520]), g.input([300, 96])
    feed = {na: a, ny: y}
    if bshape:
        b = _data(rng, bshape, 1.0)
        nb = g.input(list(bshape))
        feed[nb] = b
        x = tt.relu(na + nb) * 0.5
        xr = O.binary(O.MUL, O.unary(O.RELU, O.binary(O.ADD, a, b)), np.float32(0.5))
    else:
        x = tt.relu(na + 0.25) * 0.5
        xr = O.binary(O.MUL, O.unary(O.RELU, O.binary(O.ADD, a, np.float32(0.25))), np.float32(0.5))
    prog = tt.compile(g, outputs=[tt.transpose(x, 0, 1) @ ny], cache_dir=cache_dir)
    assert "(writes hi/lo of X^T, not X)" in prog.execution_plan()
    got = prog.run(feed).numpy()
    assert_norm(got, O.matmul(np.ascontiguousarray(xr.T), y), GEMM_FROB_RTOL)


def test_region_with_two_stores_copies_one(cache_dir):
    """A region storing two matrices (u = a * b, an output, and v = u + a, read by a
    GEMM): v's copies are written, u's fp32 store stays bit-exact."""
    rng = np.random.default_rng(53)
    a, b = _data(rng, (512, 384), 1.0), _data(rng, (512, 384), 1.0)
    y = _data(rng, (384, 200), 1 / np.sqrt(384))
    g = tt.Graph()
    na, nb, ny = g.input([512, 384]), g.input([512, 384]), g.input([384, 200])
    u = na * nb
    v = u + na
    prog = tt.compile(g, outputs=[u, v @ ny], cache_dir=cache_dir)
    assert "(writes hi/lo of X, not X)" in prog.execution_plan()
    gu, gv = (t.numpy() for t in prog.run({na: a, nb: b, ny: y}))
    ur = O.binary(O.MUL, a, b)
    assert_bitexact(gu, ur)
    assert_norm(gv, O.matmul(O.binary(O.ADD, ur, a), y), GEMM_FROB_RTOL)


@pytest.mark.parametrize("form", ["X Xt", "Xt X"])
def test_gram_matrix_reads_both_operands_from_one_set_of_copies(form, cache_dir):
    """X X^T (both operands along X's rows) and X^T X (both across): the GEMM takes A and
    B from the same region-written copies and runs no pre-pass at all."""
    rng = np.random.default_rng(59 + len(form))
    a, b = _data(rng, (512, 384), 1.0), _data(rng, (512, 384), 1.0)
    g = tt.Graph()
    na, nb = g.input([512, 384]), g.input([512, 384])
    x = na * nb
    out = x @ tt.transpose(x, 0, 1) if form == "X Xt" else tt.transpose(x, 0, 1) @ x
    prog = tt.compile(g, outputs=[out], cache_dir=cache_dir)
    plan = prog.execution_plan()
    assert "(A hi/lo from [0]) (B hi/lo from [0])" in plan, plan
    got = prog.run({na: a, nb: b}).numpy()
    xr = O.binary(O.MUL, a, b)
    xt = np.ascontiguousarray(xr.T)
    ref = O.matmul(xr, xt) if form == "X Xt" else O.matmul(xt, xr)
    assert_norm(got, ref, GEMM_FROB_RTOL)
