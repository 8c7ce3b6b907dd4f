"""Non-finite operands of the tensor-core GEMM against the reference's fp32 loop.

The reference's matmul (src/core/operators.cpp:235-319) sums fp32 products in order, so
an inf in A[i, k] makes every C[i, j] infinite (inf * b, signed) or NaN (inf * 0, or
+inf + -inf), and a NaN anywhere in row i / column j makes C[i, j] NaN.  The 3xTF32
split keeps these classes (a nonzero lo part for every nonzero operand value, lo = x
for +-inf), so each case asserts the oracle's NaN positions and its signed infinities
exactly, and the finite part at the GEMM tolerance.  The cases cover both pre-pass
kernels (K-major rows and the transposing split), the CTA-pair and single-CTA tensor-core
kernels, split-K, the fused ReLU epilogue and operand copies written by a region."""

import numpy as np
import pytest

from parity import GEMM_FROB_RTOL, assert_norm

import tinytensor_b200 as tt
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _operands(rng, m, k, n):
    a = (rng.standard_normal((m, k)) / np.sqrt(k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    a[3, 5] = np.inf            # row 3: inf * b[5, :]
    b[5, 50] = 0.0              #   ... NaN at column 50 (inf * 0)
    b[:, 40] = 2.0              #   ... column of tf32-exact values: lo is the sign marker
    a[7, 9] = -np.inf           # row 7: -inf * b[9, :]
    a[11, 2] = np.nan           # row 11: NaN
    a[20, :] = 0.5              # row 20: tf32-exact values and one inf
    a[20, 30] = np.inf
    a[30, 1] = np.inf           # row 30: +inf + -inf at column 60 -> NaN
    a[30, 2] = np.inf
    b[1, 60], b[2, 60] = 1.0, -1.0
    b[4, 10] = np.inf           # column 10: inf in B
    b[8, 20] = -np.inf          # column 20: -inf in B (meets a zero in row 40 below)
    a[40, 8] = 0.0
    return a, b


def _check(got, ref):
    assert got.shape == ref.shape
    assert np.array_equal(np.isnan(got), np.isnan(ref)), (
        f"NaN pattern differs at {np.argwhere(np.isnan(got) != np.isnan(ref))[:5].tolist()}")
    inf = np.isinf(ref)
    assert np.array_equal(got[inf], ref[inf]), "signed infinities differ"
    fin = np.isfinite(ref)
    assert np.all(np.isfinite(got[fin]))
    assert_norm(np.where(fin, got, 0.0), np.where(fin, ref, 0.0), GEMM_FROB_RTOL)


@pytest.mark.parametrize("m,k,n,layout", [
    (256, 300, 160, "NN"),     # CTA pair, A rows split, B through the transposing split
    (256, 300, 160, "TT"),     # A^T and B^T views: the other pre-pass kernel for each
    (96, 300, 256, "NN"),      # single-CTA kernel (M <= 128)
    (1024, 1024, 1024, "NN"),  # split-K (the wave model splits 1024^3)
])
def test_nonfinite_products_match_reference(m, k, n, layout, cache_dir):
    rng = np.random.default_rng(m + k + n)
    a, b = _operands(rng, m, k, n)
    g = tt.Graph()
    if layout == "NN":
        na, nb = g.input([m, k]), g.input([k, n])
        out = na @ nb
        feed_vals = (a, b)
    else:
        na, nb = g.input([k, m]), g.input([n, k])
        out = tt.transpose(na, 0, 1) @ tt.transpose(nb, 0, 1)
        feed_vals = (np.ascontiguousarray(a.T), np.ascontiguousarray(b.T))
    prog = tt.compile(g, outputs=[out, tt.relu(out)], cache_dir=cache_dir)
    assert "tcgen05" in prog.execution_plan()
    got, got_relu = (t.numpy() for t in prog.run({na: feed_vals[0], nb: feed_vals[1]}))
    ref = O.matmul(a, b)
    _check(got, ref)
    _check(got_relu, O.unary(O.RELU, ref))
    # the cases built into the operands
    assert np.isnan(got[3, 50]) and np.isnan(got[11]).all() and np.isnan(got[30, 60])
    assert got[20, 40] == np.inf and np.isinf(got[3, 40])


def test_nonfinite_through_relu_epilogue(cache_dir):
    """relu(A @ B) with the ReLU in the GEMM epilogue (the product is not an output):
    -inf becomes 0, NaN becomes +0, +inf stays, as relu of the reference's product."""
    rng = np.random.default_rng(5)
    a, b = _operands(rng, 512, 256, 256)
    g = tt.Graph()
    na, nb = g.input([512, 256]), g.input([256, 256])
    prog = tt.compile(g, outputs=[tt.relu(na @ nb)], cache_dir=cache_dir)
    assert "+relu" in prog.execution_plan()
    got = prog.run({na: a, nb: b}).numpy()
    _check(got, O.unary(O.RELU, O.matmul(a, b)))


def test_nonfinite_through_region_copies(cache_dir):
    """The operand's hi/lo copies come from the region that produced it (a * 1): the
    region's split keeps the classes exactly as the pre-pass does."""
    rng = np.random.default_rng(6)
    a, y = _operands(rng, 256, 256, 128)
    ones = np.ones_like(a)
    g = tt.Graph()
    na, nb, ny = g.input([256, 256]), g.input([256, 256]), g.input([256, 128])
    prog = tt.compile(g, outputs=[(na * nb) @ ny], cache_dir=cache_dir)
    assert "(A hi/lo from [0])" in prog.execution_plan()
    got = prog.run({na: a, nb: ones, ny: y}).numpy()
    _check(got, O.matmul(O.binary(O.MUL, a, ones), y))
