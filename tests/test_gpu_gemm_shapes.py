"""GPU parity of the CUDA-core GEMM kernels for the shapes the tensor-core kernel does
not take well: skinny products (N <= 16, or M <= 16 with the operand roles exchanged),
products with K <= 16, and operands with odd strides.  Each case checks the kernel the
planner chose (execution plan) and compares against the oracle's fp32 matmul and an
fp64 product, at the GEMM tolerance (relative Frobenius)."""

import numpy as np
import pytest

from parity import GEMM_FROB_RTOL, assert_norm

import tinytensor_b200 as tt
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _data(rng, shape, k):
    return (rng.standard_normal(shape) / np.sqrt(k)).astype(np.float32)


def _check(c, a, b, rows=None):
    """c = a @ b (2-D), on all rows or on sampled ones."""
    if rows is None:
        assert_norm(c, O.matmul(a, b), GEMM_FROB_RTOL)
        assert_norm(c, a.astype(np.float64) @ b.astype(np.float64), GEMM_FROB_RTOL)
    else:
        idx = np.unique(np.random.default_rng(5).integers(0, a.shape[0], rows)).astype(np.int64)
        assert_norm(c[idx], O.matmul_rows(a, b, idx), GEMM_FROB_RTOL)
        assert_norm(c[idx], a[idx].astype(np.float64) @ b.astype(np.float64), GEMM_FROB_RTOL)


@pytest.mark.parametrize("m,n,k", [(32768, 10, 4096), (3000, 16, 700), (129, 9, 1000), (200, 8, 5000), (77, 1, 300)])
def test_skinny_n(m, n, k, cache_dir):
    rng = np.random.default_rng(m + n + k)
    a, b = _data(rng, (m, k), k), _data(rng, (k, n), k)
    g = tt.Graph()
    na, nb = g.input([m, k]), g.input([k, n])
    prog = tt.compile(g, outputs=[na @ nb], cache_dir=cache_dir)
    assert "simt_skinny[" in prog.execution_plan()
    c = prog.run({na: a, nb: b}).numpy()
    _check(c, a, b, rows=64 if m > 4096 else None)


def test_skinny_n_transposed_a_long_k(cache_dir):
    """The output layer's weight gradient: A = H^T (an M-major view), K = 32768, split-K."""
    rng = np.random.default_rng(21)
    m, n, k = 4096, 10, 32768
    h = _data(rng, (k, m), k)
    t = _data(rng, (k, n), k)
    g = tt.Graph()
    nh, nt = g.input([k, m]), g.input([k, n])
    prog = tt.compile(g, outputs=[tt.transpose(nh, 0, 1) @ nt], cache_dir=cache_dir)
    plan = prog.execution_plan()
    assert "simt_skinny[" in plan and "splitk" in plan and "A:M" in plan
    c = prog.run({nh: h, nt: t}).numpy()
    _check(c, np.ascontiguousarray(h.T), t, rows=96)


@pytest.mark.parametrize("m,n,k", [(10, 4096, 4096), (1, 300, 1000), (16, 515, 64)])
def test_skinny_m(m, n, k, cache_dir):
    rng = np.random.default_rng(m * 7 + n + k)
    a, b = _data(rng, (m, k), k), _data(rng, (k, n), k)
    g = tt.Graph()
    na, nb = g.input([m, k]), g.input([k, n])
    prog = tt.compile(g, outputs=[na @ nb], cache_dir=cache_dir)
    assert "simt_skinny_t[" in prog.execution_plan()
    _check(prog.run({na: a, nb: b}).numpy(), a, b)


@pytest.mark.parametrize("m,n,k", [(32768, 4096, 10), (100, 130, 3), (64, 127, 16), (1000, 10, 1)])
def test_small_k(m, n, k, cache_dir):
    rng = np.random.default_rng(m + 3 * n + k)
    a, b = _data(rng, (m, k), k), _data(rng, (k, n), k)
    g = tt.Graph()
    na, nb = g.input([m, k]), g.input([k, n])
    prog = tt.compile(g, outputs=[na @ nb], cache_dir=cache_dir)
    assert "simt_smallk[" in prog.execution_plan()
    _check(prog.run({na: a, nb: b}).numpy(), a, b, rows=64 if m > 4096 else None)


def test_small_k_transposed_b_relu_epilogue(cache_dir):
    """relu(dY . W^T) with K = 10: B is a K-major view and ReLU is fused into the store."""
    rng = np.random.default_rng(33)
    m, n, k = 5000, 4096, 10
    dy, w = _data(rng, (m, k), k), _data(rng, (n, k), k)
    g = tt.Graph()
    ndy, nw = g.input([m, k]), g.input([n, k])
    prog = tt.compile(g, outputs=[tt.relu(ndy @ tt.transpose(nw, 0, 1))], cache_dir=cache_dir)
    assert "simt_smallk[" in prog.execution_plan()
    c = prog.run({ndy: dy, nw: w}).numpy()
    idx = np.arange(0, m, 37, dtype=np.int64)
    ref = np.maximum(dy[idx].astype(np.float64) @ w.T.astype(np.float64), 0.0)
    assert_norm(c[idx], ref, GEMM_FROB_RTOL)


def test_skinny_generic_strides_and_batch(cache_dir):
    """Rows of 37 floats (not 16-B aligned: scalar loads) and a broadcast batch of 3."""
    rng = np.random.default_rng(44)
    bsz, m, n, k = 3, 1000, 10, 37
    a = _data(rng, (bsz, m, k), k)
    b = _data(rng, (k, n), k)
    g = tt.Graph()
    na, nb = g.input([bsz, m, k]), g.input([k, n])
    prog = tt.compile(g, outputs=[na @ nb], cache_dir=cache_dir)
    assert "simt_skinny[" in prog.execution_plan()
    c = prog.run({na: a, nb: b}).numpy()
    assert c.shape == (bsz, m, n)
    for i in range(bsz):
        _check(c[i], a[i], b)


@pytest.mark.parametrize("sa,sb,kernel", [
    ((6, 300, 512), (6, 512, 700), "tcgen05"),        # batched, M > 128: CTA-pair tiles, ragged M and N
    ((3, 520, 1024), (1024, 384), "tcgen05"),         # B broadcast over the batch (stride 0)
    ((4, 100, 2048), (4, 2048, 300), "tcgen05"),      # M <= 128: single-CTA tiles
    ((2, 1, 64, 256), (5, 256, 96), "tcgen05"),       # broadcast batch dims [2,1] x [5] -> [2,5]
])
def test_batched_tensor_core(sa, sb, kernel, cache_dir):
    rng = np.random.default_rng(sum(sa) + sum(sb))
    k = sa[-1]
    a, b = _data(rng, sa, k), _data(rng, sb, k)
    g = tt.Graph()
    na, nb = g.input(list(sa)), g.input(list(sb))
    prog = tt.compile(g, outputs=[na @ nb], cache_dir=cache_dir)
    assert kernel in prog.execution_plan()
    c = prog.run({na: a, nb: b}).numpy()
    ref64 = np.matmul(a.astype(np.float64), b.astype(np.float64))
    assert c.shape == ref64.shape
    assert_norm(c, O.matmul(a, b), GEMM_FROB_RTOL)
    assert_norm(c, ref64, GEMM_FROB_RTOL)


def test_batched_transposed_operands(cache_dir):
    """Per-batch transposes of both operands (M- and K-major views inside a batch)."""
    rng = np.random.default_rng(71)
    bsz, m, n, k = 3, 384, 272, 640
    at = _data(rng, (bsz, k, m), k)   # A = at^T per batch
    bt = _data(rng, (bsz, n, k), k)   # B = bt^T per batch
    g = tt.Graph()
    nat, nbt = g.input([bsz, k, m]), g.input([bsz, n, k])
    prog = tt.compile(g, outputs=[tt.transpose(nat, 1, 2) @ tt.transpose(nbt, 1, 2)], cache_dir=cache_dir)
    assert "tcgen05" in prog.execution_plan()
    c = prog.run({nat: at, nbt: bt}).numpy()
    a = np.ascontiguousarray(np.transpose(at, (0, 2, 1)))
    b = np.ascontiguousarray(np.transpose(bt, (0, 2, 1)))
    assert_norm(c, O.matmul(a, b), GEMM_FROB_RTOL)
    assert_norm(c, np.matmul(a.astype(np.float64), b.astype(np.float64)), GEMM_FROB_RTOL)


@pytest.mark.parametrize("m,n,k", [(20000, 12, 8224), (4099, 3, 256), (64, 16, 128)])
def test_skinny_n_k_split_at_odd_boundaries(m, n, k, cache_dir):
    """Row-major X and a contiguous [K][Q] right operand: splits of K whose starts are
    not multiples of the 128-wide tile, a last tile cut short, rows past the 64-row
    block, one tile only."""
    rng = np.random.default_rng(m + 5 * n + k)
    a, b = _data(rng, (m, k), k), _data(rng, (k, n), k)
    g = tt.Graph()
    na, nb = g.input([m, k]), g.input([k, n])
    prog = tt.compile(g, outputs=[na @ nb], cache_dir=cache_dir)
    assert "simt_skinny[" in prog.execution_plan()
    _check(prog.run({na: a, nb: b}).numpy(), a, b, rows=80 if m > 4096 else None)


@pytest.mark.parametrize("ep", ["tanh", "relu"])
def test_skinny_n_epilogue(ep, cache_dir):
    """An activation of a 10-wide product runs in the skinny kernel's store."""
    rng = np.random.default_rng(7)
    m, n, k = 32768, 10, 512
    a, b = _data(rng, (m, k), 1.0), _data(rng, (k, n), k)
    g = tt.Graph()
    na, nb = g.input([m, k]), g.input([k, n])
    y = tt.tanh(na @ nb) if ep == "tanh" else tt.relu(na @ nb)
    prog = tt.compile(g, outputs=[y], cache_dir=cache_dir)
    assert f"+{ep}]" in prog.execution_plan()
    c = prog.run({na: a, nb: b}).numpy()
    idx = np.arange(0, m, 97, dtype=np.int64)
    z = a[idx].astype(np.float64) @ b.astype(np.float64)
    ref = np.tanh(z) if ep == "tanh" else np.maximum(z, 0.0)
    assert_norm(c[idx], ref, GEMM_FROB_RTOL)


@pytest.mark.parametrize("m,n,k", [(1000, 7, 5000), (4096, 16, 32768), (257, 1, 100)])
def test_skinny_n_transposed_a_shapes(m, n, k, cache_dir):
    """A = H^T (rows of H contiguous along M): M past the 256-row block, K not a multiple
    of the 32-row tile, one and sixteen output columns."""
    rng = np.random.default_rng(m + n + 3 * k)
    h, t = _data(rng, (k, m), k), _data(rng, (k, n), k)
    g = tt.Graph()
    nh, nt = g.input([k, m]), g.input([k, n])
    prog = tt.compile(g, outputs=[tt.transpose(nh, 0, 1) @ nt], cache_dir=cache_dir)
    assert "simt_skinny[" in prog.execution_plan()
    c = prog.run({nh: h, nt: t}).numpy()
    _check(c, np.ascontiguousarray(h.T), t, rows=96 if m * k > 1 << 24 else None)


def test_skinny_batched_both_layouts(cache_dir):
    """Batched skinny products (batch 3, each operand with its own batch): row-major A,
    and A^T as an M-major view."""
    rng = np.random.default_rng(55)
    bsz, m, n, k = 3, 2000, 10, 1024
    a = _data(rng, (bsz, m, k), k)
    h = _data(rng, (bsz, k, m), k)
    b = _data(rng, (bsz, k, n), k)
    g = tt.Graph()
    na, nh, nb = g.input([bsz, m, k]), g.input([bsz, k, m]), g.input([bsz, k, n])
    prog = tt.compile(g, outputs=[na @ nb, tt.transpose(nh, 1, 2) @ nb], cache_dir=cache_dir)
    c1, c2 = [t.numpy() for t in prog.run({na: a, nh: h, nb: b})]
    for i in range(bsz):
        _check(c1[i], a[i], b[i])
        _check(c2[i], np.ascontiguousarray(h[i].T), b[i])


@pytest.mark.parametrize("m,n,k,batch,act", [
    (4096, 4096, 4096, 1, None),     # 256 tiles on 74 clusters: 34 tail tiles in 2 K pieces
    (16384, 1024, 4096, 1, "relu"),  # the rectangular config shape, ReLU applied by the tail reduce
    (3000, 2000, 1024, 1, "tanh"),   # partial edge tiles among the tail tiles
    (1024, 1024, 512, 5, None),      # batched: tail tiles in the last batch
    (256, 256, 8192, 1, "relu"),     # a single tile in 32 K pieces
    (4096, 4096, 2050, 1, None),     # K not a multiple of 4 or of the pieces: uneven last piece
])
def test_tail_split_tiles(m, n, k, batch, act, cache_dir):
    """The persistent pair kernel splits the tiles of its last, part-filled round of
    clusters along K; their pieces go through partial tiles that a reduce adds in piece
    order.  Checked against the oracle on sampled rows (all rows of the tail tiles
    included) and against fp64."""
    rng = np.random.default_rng(m + n + k + batch)
    shape_a = [batch, m, k] if batch > 1 else [m, k]
    a, b = _data(rng, shape_a, k), _data(rng, (k, n), k)
    g = tt.Graph()
    na, nb = g.input(shape_a), g.input([k, n])
    y = na @ nb
    y = {"relu": tt.relu, "tanh": tt.tanh, None: lambda t: t}[act](y)
    prog = tt.compile(g, outputs=[y], cache_dir=cache_dir)
    assert " tail" in prog.execution_plan(), prog.execution_plan()
    c = prog.run({na: a, nb: b}).numpy()
    act_np = {"relu": lambda v: O.unary(O.RELU, v), "tanh": lambda v: O.unary(O.TANH, v), None: lambda v: v}[act]
    if batch > 1:
        for z in range(batch):
            assert_norm(c[z], act_np(O.matmul(a[z], b)), GEMM_FROB_RTOL)
        return
    # the last rows of C hold the tail tiles (row-major tile order): check every third of them
    rows = np.unique(np.concatenate([np.random.default_rng(9).integers(0, m, 64), np.arange(max(0, m - 600), m, 3)]))
    ref = act_np(O.matmul_rows(a, b, rows.astype(np.int64)))
    assert_norm(c[rows], ref, GEMM_FROB_RTOL)
    assert_norm(c[rows], act_np((a[rows].astype(np.float64) @ b.astype(np.float64)).astype(np.float32)),
                GEMM_FROB_RTOL)
