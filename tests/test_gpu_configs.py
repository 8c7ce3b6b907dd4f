"""GPU parity at the benchmark configurations' full sizes (seeded inputs of the
documented shapes and distributions; rng = np.random.default_rng(seed), drawn in
float64 and cast to float32).  Large products are checked on sampled rows, which the
reference's blocked loop computes independently of the other rows."""

import numpy as np
import pytest

from parity import GEMM_FROB_RTOL, REDUCTION_NORM_RTOL, assert_bitexact, assert_elementwise_scaled, assert_norm, norm_rel

import tinytensor_b200 as tt
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_fused_chain_1024x1024(cache_dir):
    rng = np.random.default_rng(0)
    a = rng.standard_normal((1024, 1024)).astype(np.float32)
    b = rng.standard_normal((1024, 1024)).astype(np.float32)
    c = rng.standard_normal((1, 1024)).astype(np.float32)
    g = tt.Graph()
    na, nb, nc = g.input([1024, 1024]), g.input([1024, 1024]), g.input([1, 1024])
    y = tt.relu(na * nb + nc) * 0.5 - tt.exp(-na)
    prog = tt.compile(g, outputs=[y], cache_dir=cache_dir)
    assert "Kernel Launches (1)" in prog.execution_plan()  # one fused kernel: 3 loads + 1 store
    got = prog.run({na: a, nb: b, nc: c}).numpy()
    ref = O.evaluate(g, {na: a, nb: b, nc: c}, [y])[0]
    mag = O.magnitude(g, {na: a, nb: b, nc: c}, [y])[0]
    assert_elementwise_scaled(got, ref, mag)
    assert_norm(got, ref, 1e-6)
    # the part without exp rounds identically to the reference
    g2 = tt.Graph()
    ma, mb, mc = g2.input([1024, 1024]), g2.input([1024, 1024]), g2.input([1, 1024])
    y2 = tt.relu(ma * mb + mc) * 0.5
    got2 = tt.compile(g2, outputs=[y2], cache_dir=cache_dir).run({ma: a, mb: b, mc: c}).numpy()
    assert_bitexact(got2, O.evaluate(g2, {ma: a, mb: b, mc: c}, [y2])[0])


def test_row_reductions_8192x4096(cache_dir):
    rng = np.random.default_rng(1)
    x = rng.uniform(-1, 1, (8192, 4096)).astype(np.float32)
    g = tt.Graph()
    nx = g.input([8192, 4096])
    outs = [tt.sum(nx, [1]), tt.mean(nx, [1]), tt.max(nx, [1]), tt.sum(tt.transpose(nx, 0, 1), [0])]
    prog = tt.compile(g, outputs=outs, cache_dir=cache_dir)
    got = [t.numpy() for t in prog.run({nx: x})]
    ref = O.evaluate(g, {nx: x}, outs)
    assert_norm(got[0], ref[0], REDUCTION_NORM_RTOL)
    assert_norm(got[1], ref[1], REDUCTION_NORM_RTOL)
    assert_bitexact(got[2], ref[2])
    assert_norm(got[3], ref[3], REDUCTION_NORM_RTOL)
    # the transposed view is folded: no copy kernel in the plan
    assert "copy" not in prog.execution_plan()


@pytest.mark.parametrize("rows,cols", [(5000, 2048), (4800, 2052), (4737, 4100), (6000, 12288)])
def test_long_row_reductions_one_block_per_row(rows, cols, cache_dir):
    """Rows of >= 2048 floats with many rows take the one-CTA-per-row kernel: row lengths
    that leave a partial 4 KB step, NaN and +-inf in some rows, rows of signed zeros."""
    rng = np.random.default_rng(rows + cols)
    x = rng.uniform(-1, 1, (rows, cols)).astype(np.float32)
    x[3, 17] = np.nan
    x[5, cols - 1] = np.inf
    x[6, 0] = -np.inf
    x[7, :] = -0.0
    x[8, :] = -0.0
    x[8, cols - 3] = 0.0
    g = tt.Graph()
    nx = g.input([rows, cols])
    outs = [tt.sum(nx, [1]), tt.mean(nx, [1], keepdims=True), tt.max(nx, [1]), tt.sum(tt.transpose(nx, 0, 1), [0])]
    got = [t.numpy() for t in tt.compile(g, outputs=outs, cache_dir=cache_dir).run({nx: x})]
    ref = O.evaluate(g, {nx: x}, outs)
    assert_bitexact(got[2], ref[2])
    assert np.signbit(got[2][7]) and not np.signbit(got[2][8])
    for a, b in ((got[0], ref[0]), (got[1], ref[1]), (got[3], ref[3])):
        a, b = a.reshape(-1), b.reshape(-1)
        fin = np.isfinite(b)
        assert_bitexact(a[~fin], b[~fin])      # NaN / inf rows
        assert_norm(a[fin], b[fin], REDUCTION_NORM_RTOL)


def _gemm(m, n, k, cache_dir, rows=None):
    rng = np.random.default_rng(2)
    a = (rng.standard_normal((m, k)) / np.sqrt(k)).astype(np.float32)
    b = (rng.standard_normal((k, n)) / np.sqrt(k)).astype(np.float32)
    g = tt.Graph()
    na, nb = g.input([m, k]), g.input([k, n])
    c = tt.compile(g, outputs=[na @ nb], cache_dir=cache_dir).run({na: a, nb: b}).numpy()
    if rows is None:
        ref = O.matmul(a, b)
        assert_norm(c, ref, GEMM_FROB_RTOL)
    else:
        idx = np.unique(np.random.default_rng(9).integers(0, m, rows)).astype(np.int64)
        ref = O.matmul_rows(a, b, idx)
        assert_norm(c[idx], ref, GEMM_FROB_RTOL)
        # fp64 check of the same rows
        exact = a[idx].astype(np.float64) @ b.astype(np.float64)
        assert_norm(c[idx], exact, GEMM_FROB_RTOL)


def test_gemm_1024_cubed(cache_dir):
    _gemm(1024, 1024, 1024, cache_dir)


def test_gemm_4096_cubed_sampled(cache_dir):
    _gemm(4096, 4096, 4096, cache_dir, rows=48)


def test_gemm_16384x1024x4096_sampled(cache_dir):
    _gemm(16384, 1024, 4096, cache_dir, rows=64)


def test_gemm_8192_cubed_sampled(cache_dir):
    _gemm(8192, 8192, 8192, cache_dir, rows=24)


def test_gemm_long_k_split_and_tails(cache_dir):
    """K = 32768 (TMEM chunking + split-K), N not a multiple of the tile, transposed A."""
    rng = np.random.default_rng(12)
    m, n, k = 520, 300, 32768
    at = (rng.standard_normal((k, m)) / np.sqrt(k)).astype(np.float32)  # A = at^T, an M-major view
    b = (rng.standard_normal((k, n)) / np.sqrt(k)).astype(np.float32)
    g = tt.Graph()
    nat, nb = g.input([k, m]), g.input([k, n])
    prog = tt.compile(g, outputs=[tt.transpose(nat, 0, 1) @ nb], cache_dir=cache_dir)
    assert "tcgen05" in prog.execution_plan() and "splitk" in prog.execution_plan()
    c = prog.run({nat: at, nb: b}).numpy()
    idx = np.arange(0, m, 13, dtype=np.int64)
    assert_norm(c[idx], O.matmul_rows(at.T, b, idx), GEMM_FROB_RTOL)
    assert_norm(c[idx], at.T[idx].astype(np.float64) @ b.astype(np.float64), GEMM_FROB_RTOL)


def _mlp_graph(B):
    g = tt.Graph()
    X, T = g.input([B, 1024], name="X"), g.input([B, 10], name="T")
    W1, W2, W3 = g.input([1024, 4096], name="W1"), g.input([4096, 4096], name="W2"), g.input([4096, 10], name="W3")
    h1 = tt.relu(X @ W1)
    h2 = tt.tanh(h1 @ W2)
    d = h2 @ W3 - T
    loss = tt.mean(d * d)
    return g, (X, T, W1, W2, W3), loss


def _xavier(rng, fi, fo):
    lim = np.sqrt(6.0 / (fi + fo))
    return rng.uniform(-lim, lim, (fi, fo)).astype(np.float32)


def test_mlp_gradients_small_batch(cache_dir):
    """Full layer widths (1024 -> 4096 -> 4096 -> 10) at batch 64 against the oracle."""
    B = 64
    rng = np.random.default_rng(3)
    g, (X, T, W1, W2, W3), loss = _mlp_graph(B)
    feed = {X: rng.standard_normal((B, 1024)).astype(np.float32), T: rng.standard_normal((B, 10)).astype(np.float32),
            W1: _xavier(rng, 1024, 4096), W2: _xavier(rng, 4096, 4096), W3: _xavier(rng, 4096, 10)}
    prog = tt.compile_gradients(g, loss, [W1, W2, W3], cache_dir=cache_dir)
    out = [t.numpy() for t in prog.run(feed)]
    ref = O.gradients(g, loss, feed, [W1, W2, W3])
    lref = O.evaluate(g, feed, [loss])[0]
    np.testing.assert_allclose(out[0], lref, rtol=1e-5)
    for got, r in zip(out[1:], ref):
        assert_norm(got, r, GEMM_FROB_RTOL)


def _fp64_mlp(x, t, w, cols):
    """fp64 forward and backward of the MLP (the VJPs of src/autodiff/gradient.cpp:
    relu mask g * (z > 0), tanh' = 1 - y^2, matmul g.B^T and A^T.g, mean = sum / n).
    Returns the loss, dW3 in full, and columns `cols` of dW2 and dW1.  Runs in torch
    float64 on the GPU (cuBLAS DGEMM), an independent fp64 computation."""
    import torch

    dev = torch.device("cuda")
    X = torch.from_numpy(x).to(dev, torch.float64)
    T = torch.from_numpy(t).to(dev, torch.float64)
    W1, W2, W3 = (torch.from_numpy(a).to(dev, torch.float64) for a in w)
    c = torch.from_numpy(np.asarray(cols, np.int64)).to(dev)
    z1 = X @ W1
    h1 = torch.clamp_min(z1, 0.0)
    h2 = torch.tanh(h1 @ W2)
    d = h2 @ W3 - T
    loss = torch.mean(d * d)
    dy = 2.0 * d / d.numel()
    dz2 = (dy @ W3.T) * (1.0 - h2 * h2)
    gw3 = h2.T @ dy
    gw2 = h1.T @ dz2[:, c]
    dz1c = (dz2 @ W2[c, :].T) * (z1[:, c] > 0).to(torch.float64)
    gw1 = X.T @ dz1c
    out = (float(loss), gw3.cpu().numpy(), gw2.cpu().numpy(), gw1.cpu().numpy())
    del X, T, W1, W2, W3, z1, h1, h2, d, dy, dz2
    torch.cuda.empty_cache()
    return out


def test_mlp_gradients_batch_4096(cache_dir):
    """Batch 4096 (the single-GPU MLP benchmark's size): loss, dW3 in full and sampled columns of dW2 and
    dW1 against an fp64 recomputation, relative Frobenius <= 1e-5."""
    B = 4096
    rng = np.random.default_rng(3)
    g, (X, T, W1, W2, W3), loss = _mlp_graph(B)
    feed = {X: rng.standard_normal((B, 1024)).astype(np.float32), T: rng.standard_normal((B, 10)).astype(np.float32),
            W1: _xavier(rng, 1024, 4096), W2: _xavier(rng, 4096, 4096), W3: _xavier(rng, 4096, 10)}
    prog = tt.compile_gradients(g, loss, [W1, W2, W3], cache_dir=cache_dir)
    out = [t.numpy() for t in prog.run(feed)]
    assert all(np.all(np.isfinite(o)) for o in out)
    cols = np.unique(np.random.default_rng(21).integers(0, 4096, 96))
    l64, gw3, gw2, gw1 = _fp64_mlp(feed[X], feed[T], [feed[W1], feed[W2], feed[W3]], cols)
    np.testing.assert_allclose(out[0], l64, rtol=1e-5)
    assert_norm(out[3], gw3, GEMM_FROB_RTOL)
    assert_norm(out[2][:, cols], gw2, GEMM_FROB_RTOL)
    assert_norm(out[1][:, cols], gw1, GEMM_FROB_RTOL)


def test_dp_step_global_batch_32768_one_gpu(cache_dir):
    """One DataParallelSGD step at the benchmark's global batch 32768 on one GPU (the
    program, the single all-reduce-free update with lr 0.01): the gradients it used
    against fp64 (dW3 in full, sampled columns of dW2 and dW1, relative Frobenius
    <= 1e-5), the loss, and the updated weights bit-exact against numpy's float32
    p - lr * g on those gradients (python/tinytensor/optim.py:18-35)."""
    B = 32768
    rng = np.random.default_rng(4)
    x = rng.standard_normal((B, 1024)).astype(np.float32)
    t = rng.standard_normal((B, 10)).astype(np.float32)
    ws = [_xavier(rng, 1024, 4096), _xavier(rng, 4096, 4096), _xavier(rng, 4096, 10)]
    g, (X, T, W1, W2, W3), loss = _mlp_graph(B)
    prog = tt.compile_gradients(g, loss, [W1, W2, W3], cache_dir=cache_dir)
    dx, dt = tt.DeviceBuffer.from_numpy(x), tt.DeviceBuffer.from_numpy(t)
    dw = [tt.DeviceBuffer.from_numpy(w) for w in ws]
    trainer = tt.DataParallelSGD(prog, dw, lr=0.01)
    st = tt.Stream()
    trainer.step([dx, dt], st)
    st.synchronize()
    assert prog.status() == 0
    grads = trainer.grads.numpy()
    offs = np.cumsum([0] + trainer.sizes)
    gpu_g = [grads[offs[i]:offs[i + 1]].reshape(ws[i].shape) for i in range(3)]
    cols = np.unique(np.random.default_rng(22).integers(0, 4096, 64))
    l64, gw3, gw2, gw1 = _fp64_mlp(x, t, ws, cols)
    np.testing.assert_allclose(trainer.loss.numpy(), l64, rtol=1e-5)
    assert_norm(gpu_g[2], gw3, GEMM_FROB_RTOL)
    assert_norm(gpu_g[1][:, cols], gw2, GEMM_FROB_RTOL)
    assert_norm(gpu_g[0][:, cols], gw1, GEMM_FROB_RTOL)
    for w0, gg, d in zip(ws, gpu_g, dw):
        assert_bitexact(d.numpy(), (w0 - np.float32(0.01) * gg).astype(np.float32))


def test_mlp_sgd_steps_match_oracle(cache_dir):
    """Three SGD steps (lr 0.01) of the MLP on device vs the oracle's full-batch steps."""
    B = 32
    rng = np.random.default_rng(4)
    g, (X, T, W1, W2, W3), loss = _mlp_graph(B)
    x = rng.standard_normal((B, 1024)).astype(np.float32)
    t = rng.standard_normal((B, 10)).astype(np.float32)
    ws = [_xavier(rng, 1024, 4096), _xavier(rng, 4096, 4096), _xavier(rng, 4096, 10)]
    prog = tt.compile_gradients(g, loss, [W1, W2, W3], cache_dir=cache_dir)
    dx, dt = tt.DeviceBuffer.from_numpy(x), tt.DeviceBuffer.from_numpy(t)
    dw = [tt.DeviceBuffer.from_numpy(w) for w in ws]
    outs = [tt.DeviceBuffer(s) for s in prog.output_shapes]
    opt = tt.SGD(dw, lr=0.01)
    st = tt.Stream()
    for _ in range(3):
        prog.run_device([dx, dt] + dw, outs, st)
        opt.step(outs[1:], st)
    st.synchronize()
    ref = [w.copy() for w in ws]
    for _ in range(3):
        grads = O.gradients(g, loss, {X: x, T: t, W1: ref[0], W2: ref[1], W3: ref[2]}, [W1, W2, W3])
        ref = [O.sgd(w, gw, 0.01)[0] for w, gw in zip(ref, grads)]
    for d, r in zip(dw, ref):
        assert_norm(d.numpy(), r, GEMM_FROB_RTOL)


def test_reductions_against_both_reference_paths(cache_dir):
    """The reference has two CPU paths for reductions: the interpreter accumulates in
    double (src/core/operators.cpp:394-516), its compiled AVX2 code in float, one
    sequential += per element (src/codegen/cpp_backend.cpp:389-478).  The GPU result
    (double accumulation) is held to the interpreter at the reduction tolerance, and its
    distance to the compiled path is reported and bounded by that path's own distance to
    the interpreter plus the tolerance.  The reference itself (oracle/_ref) runs both."""
    if not O.reference_available():
        pytest.skip("oracle/_ref not built")
    R = O.Reference()
    rng = np.random.default_rng(1)
    x = rng.uniform(-1, 1, (2048, 4096)).astype(np.float32)
    g = tt.Graph()
    nx = g.input([2048, 4096])
    outs = [tt.sum(nx, [1]), tt.mean(nx, [1]), tt.sum(tt.transpose(nx, 0, 1), [0])]
    got = [t.numpy() for t in tt.compile(g, outputs=outs, cache_dir=cache_dir).run({nx: x})]
    interp = R.run(g, {nx: x}, mode="interpreted", optimize=False, outputs=outs)
    avx2 = R.run(g, {nx: x}, mode="avx2", optimize=False, outputs=outs)
    for name, gv, ri, ra in zip(["sum", "mean", "sum of the transpose"], got, interp, avx2):
        assert_norm(gv, ri, REDUCTION_NORM_RTOL)
        e_ref = norm_rel(ra, ri)     # the compiled path's own fp32 accumulation error
        e_gpu = norm_rel(gv, ra)
        print(f"{name}: |gpu - interpreter| {norm_rel(gv, ri):.2e}, |gpu - avx2| {e_gpu:.2e}, "
              f"|avx2 - interpreter| {e_ref:.2e}")
        assert e_gpu <= e_ref + REDUCTION_NORM_RTOL


def test_gemm_against_both_reference_paths(cache_dir):
    """The reference's eager matmul (src/core/operators.cpp:235-319, fp32 multiply then add)
    and its compiled AVX2+FMA code (src/codegen/cpp_backend.cpp:294-329, 32x32x32 blocks of
    fused multiply-adds) round differently.  The 3xTF32 result is held to the eager path and
    to fp64 at the GEMM tolerance; its distance to the compiled path is reported and bounded
    by that path's own distance to the eager one plus the tolerance."""
    if not O.reference_available():
        pytest.skip("oracle/_ref not built")
    R = O.Reference()
    rng = np.random.default_rng(2)
    m, k, n = 768, 1024, 512
    a = (rng.standard_normal((m, k)) / np.sqrt(k)).astype(np.float32)
    b = (rng.standard_normal((k, n)) / np.sqrt(k)).astype(np.float32)
    g = tt.Graph()
    na, nb = g.input([m, k]), g.input([k, n])
    y = na @ nb
    got = tt.compile(g, outputs=[y], cache_dir=cache_dir).run({na: a, nb: b}).numpy()
    eager = O.matmul(a, b)
    fma = R.run(g, {na: a, nb: b}, mode="avx2_fma", optimize=False, outputs=[y])[0]
    exact = a.astype(np.float64) @ b.astype(np.float64)
    assert_norm(got, eager, GEMM_FROB_RTOL)
    assert_norm(got, exact, GEMM_FROB_RTOL)
    e_ref, e_gpu = norm_rel(fma, eager), norm_rel(got, fma)
    print(f"|gpu - eager| {norm_rel(got, eager):.2e}, |gpu - fp64| {norm_rel(got, exact):.2e}, "
          f"|gpu - avx2_fma| {e_gpu:.2e}, |avx2_fma - eager| {e_ref:.2e}")
    assert e_gpu <= e_ref + GEMM_FROB_RTOL
