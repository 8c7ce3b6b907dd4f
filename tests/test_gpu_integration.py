"""The reference's own Executor driving the B200 backend (ExecutionMode::CompiledCUDA):
integration/_build/libttref_cuda.so is the reference built from its sources with
integration/executor.patch and integration/{include,src} added, linked against
libtt_cuda.so.  Each graph runs through that Executor in CUDA mode and in the
Interpreted mode of the same library, with the reference Optimizer on and off, and the
results are compared (bit-exact for + - * / relu, the GEMM tolerance for products,
norm-wise for reductions).  Device-resident tensors (a reference Tensor over device
memory) run without host staging and chain from one Executor to the next on the device.
The patched reference Python package is exercised with mode="cuda" in a subprocess."""

import ctypes
import os
import subprocess
import sys

import numpy as np
import pytest

from parity import GEMM_FROB_RTOL, REDUCTION_NORM_RTOL, assert_bitexact, assert_elementwise_scaled, assert_norm

import tinytensor_b200 as tt
from oracle import oracle as O

pytestmark = pytest.mark.gpu

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
LIB = os.path.join(ROOT, "integration", "_build", "libttref_cuda.so")
PKG = os.path.join(ROOT, "integration", "_build", "pkg")


@pytest.fixture(scope="module")
def R():
    if not os.path.exists(LIB):
        pytest.fail(f"{LIB} missing: build it with `make -C integration` where the reference sources are")
    r = O.Reference(LIB)
    L = r.lib
    L.ttref_exec_text.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t]
    L.ttref_exec_text.restype = ctypes.c_size_t
    L.ttref_run_device.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p),
                                   ctypes.POINTER(ctypes.c_void_p)]
    return r


def _elementwise_graph():
    g = tt.Graph()
    a, b, c = g.input([300, 257], name="a"), g.input([300, 257], name="b"), g.input([1, 257], name="c")
    y1 = tt.relu(a * b)          # the reference optimizer fuses this into FusedElementwise
    y2 = (a - c) / (b + 2.5) + tt.relu(a - b)
    return g, (a, b, c), [y1, y2]


def _feed(nodes, seed):
    rng = np.random.default_rng(seed)
    return {n: rng.standard_normal(n.shape).astype(np.float32) for n in nodes}


@pytest.mark.parametrize("optimize", [False, True])
def test_executor_cuda_mode_elementwise_bitexact(R, optimize):
    g, ins, outs = _elementwise_graph()
    feed = _feed(ins, 1)
    got = R.run(g, feed, mode="cuda", optimize=optimize, outputs=outs)
    ref = R.run(g, feed, mode="interpreted", optimize=False, outputs=outs)
    for a, b in zip(got, ref):
        assert_bitexact(a, b)
    if optimize:
        # the reference's own compiled mode computes the fused node as relu(a + b)
        avx = R.run(g, feed, mode="avx2", optimize=True, outputs=outs)
        assert not np.array_equal(avx[0], ref[0])


@pytest.mark.parametrize("optimize", [False, True])
def test_executor_cuda_mode_mlp_forward_and_reductions(R, optimize):
    g = tt.Graph()
    x, w1, w2 = g.input([512, 256]), g.input([256, 384]), g.input([384, 10])
    h = tt.sigmoid(tt.relu(x @ w1) @ w2)
    s = tt.sum(h, [1])
    m = tt.mean(tt.transpose(x @ w1, 0, 1), [1], keepdims=True)
    rng = np.random.default_rng(2)
    feed = {x: rng.standard_normal((512, 256)).astype(np.float32),
            w1: (rng.standard_normal((256, 384)) / 16).astype(np.float32),
            w2: (rng.standard_normal((384, 10)) / 20).astype(np.float32)}
    got = R.run(g, feed, mode="cuda", optimize=optimize, outputs=[h, s, m])
    ref = R.run(g, feed, mode="interpreted", optimize=False, outputs=[h, s, m])
    assert_norm(got[0], ref[0], GEMM_FROB_RTOL)
    assert_norm(got[1], ref[1], GEMM_FROB_RTOL)
    assert_norm(got[2], ref[2], GEMM_FROB_RTOL)
    # the reduction of a plain input is exact to the reduction tolerance
    g2 = tt.Graph()
    z = g2.input([640, 4096])
    outs = [tt.sum(z, [1]), tt.mean(z, [0]), tt.sum(z)]
    zf = {z: np.random.default_rng(3).uniform(-1, 1, (640, 4096)).astype(np.float32)}
    got2 = R.run(g2, zf, mode="cuda", optimize=optimize, outputs=outs)
    ref2 = R.run(g2, zf, mode="interpreted", optimize=False, outputs=outs)
    for a, b in zip(got2, ref2):
        assert_norm(a, b, REDUCTION_NORM_RTOL)


def test_executor_cuda_mode_exp_identity_and_sigmoid(R):
    """sigmoid in the CUDA mode against the reference interpreter's sigmoid, at the
    elementwise bound (glibc's expf and CUDA's round some exponentials differently)."""
    g = tt.Graph()
    a = g.input([1000, 97])
    y = tt.sigmoid(a * 3.0) - tt.sigmoid(-a)
    feed = {a: np.random.default_rng(4).standard_normal((1000, 97)).astype(np.float32)}
    got = R.run(g, feed, mode="cuda", outputs=[y])[0]
    ref = R.run(g, feed, mode="interpreted", outputs=[y])[0]
    assert_elementwise_scaled(got, ref, O.magnitude(g, feed, [y])[0])


def test_executor_plan_and_source(R):
    g, ins, outs = _elementwise_graph()
    h, _ = R.build(g, outs)
    try:
        ex = R.lib.ttref_compile(h, R.MODES["cuda"], 1)
        assert ex, R.lib.ttref_last_error().decode()
        texts = []
        for what in (0, 1):
            n = R.lib.ttref_exec_text(ex, what, None, 0)
            buf = ctypes.create_string_buffer(n)
            R.lib.ttref_exec_text(ex, what, buf, n)
            texts.append(buf.value.decode())
        R.lib.ttref_exec_free(ex)
    finally:
        R.lib.ttref_graph_free(h)
    plan, src = texts
    assert "Execution Mode: Compiled CUDA" in plan and "Memory Planning:" in plan
    assert "__global__" in src


def _device_run(R, g, feed, outs, g2=None, outs2=None):
    h, _ = R.build(g, outs)
    h2 = R.build(g2, outs2)[0] if g2 is not None else None
    try:
        ex = R.lib.ttref_compile(h, R.MODES["cuda"], 1)
        assert ex, R.lib.ttref_last_error().decode()
        ex2 = None
        if h2 is not None:
            ex2 = R.lib.ttref_compile(h2, R.MODES["cuda"], 1)
            assert ex2, R.lib.ttref_last_error().decode()
        ins = [np.ascontiguousarray(feed[n], np.float32) for n in g.inputs]
        final = outs2 if g2 is not None else outs
        res = [np.empty(o.shape, np.float32) for o in final]
        ip = (ctypes.c_void_p * len(ins))(*[a.ctypes.data for a in ins])
        op = (ctypes.c_void_p * len(res))(*[r.ctypes.data for r in res])
        rc = R.lib.ttref_run_device(ex, ex2, ip, op)
        assert rc == 0, R.lib.ttref_last_error().decode()
        R.lib.ttref_exec_free(ex)
        if ex2:
            R.lib.ttref_exec_free(ex2)
        return res
    finally:
        R.lib.ttref_graph_free(h)
        if h2 is not None:
            R.lib.ttref_graph_free(h2)


def test_device_tensors_through_the_executor(R):
    """Inputs as device tensors: Executor::run takes them without host staging and
    returns device tensors (the harness checks they are), equal to the host run."""
    g, ins, outs = _elementwise_graph()
    feed = _feed(ins, 5)
    got = _device_run(R, g, feed, outs)
    ref = R.run(g, feed, mode="interpreted", outputs=outs)
    for a, b in zip(got, ref):
        assert_bitexact(a, b)


def test_device_tensors_chain_two_executors(R):
    """The outputs of one CUDA-mode Executor feed the next one on the device: a linear
    layer then relu/sum, against the interpreted composition."""
    g1 = tt.Graph()
    x, w = g1.input([1024, 512]), g1.input([512, 256])
    y = x @ w
    g2 = tt.Graph()
    yi = g2.input([1024, 256])
    z = [tt.relu(yi), tt.sum(yi, [1])]
    rng = np.random.default_rng(6)
    feed = {x: rng.standard_normal((1024, 512)).astype(np.float32),
            w: (rng.standard_normal((512, 256)) / 22).astype(np.float32)}
    got = _device_run(R, g1, feed, [y], g2, z)
    mid = R.run(g1, feed, mode="interpreted", outputs=[y])[0]
    ref = R.run(g2, {yi: mid}, mode="interpreted", outputs=z)
    assert_norm(got[0], ref[0], GEMM_FROB_RTOL)
    assert_norm(got[1], ref[1], GEMM_FROB_RTOL)


def test_patched_python_package_mode_cuda():
    """tt.compile(..., mode="cuda") in the reference's own Python package (patched), host
    numpy feeds and device-tensor feeds, against mode="interpreted"."""
    if not os.path.isdir(os.path.join(PKG, "tinytensor")):
        pytest.fail(f"{PKG}/tinytensor missing: build it with `make -C integration py`")
    code = r'''
import sys
sys.path.insert(0, %r)
import numpy as np
import tinytensor as tt
from tinytensor import _tinytensor as N
g = tt.Graph()
a = g.input([256, 300], name="a")
b = g.input([256, 300], name="b")
w = g.input([300, 64], name="w")
y = g.relu(g.matmul(g.mul(a, b), w))
s = g.reduce_sum(y, [1])
rng = np.random.default_rng(0)
fa = rng.standard_normal((256, 300)).astype(np.float32)
fb = rng.standard_normal((256, 300)).astype(np.float32)
fw = (rng.standard_normal((300, 64)) / 17).astype(np.float32)
feed = {a: fa, b: fb, w: fw}
cu = tt.compile(g, outputs=[y, s], mode="cuda")
ip = tt.compile(g, mode="interpreted", optimize=False)  # outputs already marked
got = [o.numpy() for o in cu.run(feed)]
ref = [o.numpy() for o in ip.run(feed)]
def rel(x, r):
    return float(np.linalg.norm((x.astype(np.float64) - r)) / np.linalg.norm(r))
assert "Compiled CUDA" in cu.execution_plan(), cu.execution_plan()
assert "__global__" in cu.generated_source()
e = [rel(x, r) for x, r in zip(got, ref)]
assert max(e) <= 1e-5, e
# device tensors in, device tensors out; numpy() copies them back
dfeed = {n: N.cuda_to_device(N.Tensor.from_numpy(v)) for n, v in feed.items()}
assert all(N.cuda_is_device(t) for t in dfeed.values())
dout = cu.run(dfeed)
assert all(N.cuda_is_device(o) for o in dout)
e2 = [rel(o.numpy(), r) for o, r in zip(dout, ref)]
assert max(e2) <= 1e-5, e2
print("ok", e, e2)
''' % PKG
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.strip().startswith("ok"), r.stdout
