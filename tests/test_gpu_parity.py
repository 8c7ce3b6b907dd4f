"""GPU parity: every case of tests/golden/cases.py compiled and run through the C ABI
(tt_compile / tt_program_run), compared with the reference's golden outputs and with
the CPU oracle; known answers and IEEE edge cases of the reference's tests."""

import os

import numpy as np
import pytest

from cases import CASES, build
from parity import (
    GEMM_FROB_RTOL,
    REDUCTION_NORM_RTOL,
    assert_bitexact,
    assert_elementwise,
    assert_elementwise_scaled,
    assert_norm,
)

import tinytensor_b200 as tt
from oracle import oracle as O

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _has_op(graph, ops):
    return any(n.op in ops for n in graph.nodes)


def _check(name, got, gold, oracle_vals, graph, feed=None, outputs=None):
    c = CASES[name]
    mags = None
    if c["kind"] == "forward" and _has_op(graph, (O.EXP, O.TANH, O.SIGMOID)):
        mags = O.magnitude(graph, feed, outputs)
    for i, g in enumerate(got):
        ref = gold[f"out{i}"] if gold is not None else None
        orc = oracle_vals[i]
        if c["exact"]:
            assert_bitexact(g, ref)
        elif name in ("reductions",):
            assert_norm(g, ref, REDUCTION_NORM_RTOL)
        elif name == "reduce_max":
            assert_bitexact(g, ref)
        elif _has_op(graph, (O.MATMUL,)) or c["kind"] == "grad":
            assert_norm(g, orc, GEMM_FROB_RTOL)
            if c["ref_ok"]:
                assert_norm(g, ref, GEMM_FROB_RTOL)
        elif mags is not None:
            assert_elementwise_scaled(g, orc, mags[i])
            if c["ref_ok"]:
                assert_elementwise_scaled(g, ref, mags[i])
        else:
            assert_elementwise(g, orc)
            if c["ref_ok"]:
                assert_elementwise(g, ref)


@pytest.mark.parametrize("name", sorted(CASES))
def test_case_matches_reference_and_oracle(name, cache_dir):
    c = build(name)
    gold = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    g, feed = c["graph"], c["feed"]
    if c["kind"] == "forward":
        prog = tt.compile(g, outputs=c["outputs"], cache_dir=cache_dir)
        res = prog.run(feed)
        res = res if isinstance(res, list) else [res]
        got = [r.numpy() for r in res]
        orc = O.evaluate(g, feed, c["outputs"])
        _check(name, got, gold, orc, g, feed, c["outputs"])
        return
    else:
        grads = tt.gradients(g, c["loss"], feed, cache_dir=cache_dir)
        got = [grads[w].numpy() for w in c["wrt"]]
        orc = O.gradients(g, c["loss"], feed, c["wrt"])
    _check(name, got, gold, orc, g)


@pytest.mark.parametrize("name", ["add_shapes", "reductions", "matmul_shapes", "fused_chain_small"])
def test_device_mode_equals_host_mode(name, cache_dir):
    c = build(name)
    g, feed, outs = c["graph"], c["feed"], c["outputs"]
    prog = tt.compile(g, outputs=outs, cache_dir=cache_dir)
    host = prog.run(feed)
    host = host if isinstance(host, list) else [host]
    ins = [tt.DeviceBuffer.from_numpy(feed[n]) for n in g.inputs]
    dev_out = [tt.DeviceBuffer(s) for s in prog.output_shapes]
    st = tt.Stream()
    prog.run_device(ins, dev_out, st)
    st.synchronize()
    assert prog.status() == 0
    for h, d in zip(host, dev_out):
        assert_bitexact(d.numpy(), h.numpy())


def test_known_answers(cache_dir):
    # tests/cpp/codegen/test_codegen.cpp:22-43, 80-156, 180-217
    g = tt.Graph()
    x = g.input([8])
    y = tt.relu(x)
    r = tt.compile(g, outputs=[y], cache_dir=cache_dir).run({x: [(-5.0 if i % 2 == 0 else 5.0) for i in range(8)]})
    np.testing.assert_array_equal(r.numpy(), [0, 5, 0, 5, 0, 5, 0, 5])

    g = tt.Graph()
    a, b = g.input([4, 8]), g.input([8, 6])
    r = tt.compile(g, outputs=[a @ b], cache_dir=cache_dir).run({a: np.ones((4, 8)), b: np.full((8, 6), 2.0)})
    assert r.shape == [4, 6] and np.all(r.numpy() == 16.0)

    g = tt.Graph()
    a, b = g.input([2, 3, 4]), g.input([2, 4, 2])
    r = tt.compile(g, outputs=[a @ b], cache_dir=cache_dir).run({a: np.ones((2, 3, 4)), b: np.full((2, 4, 2), 3.0)})
    assert r.shape == [2, 3, 2] and np.all(r.numpy() == 12.0)

    g = tt.Graph()
    a, b, c = g.input([2, 4]), g.input([2, 4]), g.input([4])
    q = tt.div(tt.add(tt.sub(a, b), c), c)
    tr = tt.transpose(q, 0, 1)
    prog = tt.compile(g, outputs=[tr, tt.sum(tr, [0]), tt.mean(tr, [0, 1])], cache_dir=cache_dir)
    r = prog.run({a: np.full((2, 4), 10.0), b: np.full((2, 4), 2.0), c: np.full((4,), 2.0)})
    assert r[0].shape == [4, 2] and np.all(r[0].numpy() == 5.0)
    assert r[1].shape == [2] and np.all(r[1].numpy() == 20.0)
    assert r[2].shape == [] and r[2].item() == 5.0

    g = tt.Graph()
    a = g.input([4])
    r = tt.compile(g, outputs=[tt.sigmoid(a)], cache_dir=cache_dir).run({a: np.zeros(4)})
    np.testing.assert_allclose(r.numpy(), 0.5, atol=1e-6)


def test_ieee_edge_cases(cache_dir):
    # tests/python/test_ieee754_edge_cases.py:37-154
    sub = float(np.nextafter(np.float32(0), np.float32(1)))
    v = np.array([np.nan, np.inf, -np.inf, 0.0, -0.0, sub, -sub, 1e38, -1e38, 42.5, -42.5, 1, -1, 2, -2, 3],
                 np.float32)
    g = tt.Graph()
    x = g.input([16])
    z = g.input([16])
    prog = tt.compile(g, outputs=[tt.relu(x), tt.sigmoid(x), x / z], cache_dir=cache_dir)
    relu, sig, div = (t.numpy() for t in prog.run({x: v, z: np.zeros(16, np.float32)}))
    for val, r in zip(v, relu):
        if np.isnan(val):
            assert r == 0.0
        elif np.isposinf(val):
            assert np.isposinf(r)
        elif val <= 0:
            assert r == 0.0 and not np.signbit(r)
        else:
            assert r == val
    assert_bitexact(relu, O.unary(O.RELU, v))
    assert_elementwise_scaled(sig, O.unary(O.SIGMOID, v), 1.0)
    with np.errstate(divide="ignore", invalid="ignore"):
        assert_bitexact(div, v / np.zeros(16, np.float32))
    g2 = tt.Graph()
    x2 = g2.input([6])
    s = tt.compile(g2, outputs=[tt.sigmoid(x2)], cache_dir=cache_dir).run(
        {x2: np.array([100, -100, np.inf, -np.inf, 0, -0.0], np.float32)}).numpy()
    assert s[0] == 1.0 and 0 <= s[1] < 1e-12 and s[2] == 1.0 and s[3] == 0.0 and s[4] == 0.5 and s[5] == 0.5


def test_error_paths(cache_dir):
    # tests/cpp/codegen/test_codegen.cpp:158-178
    g = tt.Graph()
    a = g.input([4])
    prog = tt.compile(g, outputs=[tt.relu(a)], cache_dir=cache_dir)
    with pytest.raises(tt.RuntimeExecutionError):
        prog.run({})
    with pytest.raises(tt.ShapeError):
        prog.run({a: np.ones(8, np.float32)})
    with pytest.raises(tt.RuntimeExecutionError):
        prog.run_device([], [])


def test_empty_and_ragged(cache_dir):
    rng = np.random.default_rng(3)
    g = tt.Graph()
    e = g.input([0, 5])
    r = g.input([3, 7, 1])
    q = g.input([1])
    outs = [tt.relu(e), tt.sum(e, [0]), tt.mean(e, [1]), r * q + 1.0, tt.sum(r, [1], keepdims=True), tt.max(e, [0])]
    prog = tt.compile(g, outputs=outs, cache_dir=cache_dir)
    feed = {e: np.zeros((0, 5), np.float32), r: rng.standard_normal((3, 7, 1)).astype(np.float32),
            q: np.array([2.0], np.float32)}
    got = [t.numpy() for t in prog.run(feed)]
    ref = O.evaluate(g, feed, outs)
    for a_, b_ in zip(got, ref):
        assert a_.shape == b_.shape
        assert_bitexact(a_, b_) if a_.size else None
    assert np.all(got[1] == 0) and got[5].shape == (5,) and np.all(np.isneginf(got[5]))


def test_sgd_step_matches_oracle():
    rng = np.random.default_rng(5)
    ps = [rng.standard_normal(s).astype(np.float32) for s in [(1000,), (33, 7), (4096,)]]
    gs = [rng.standard_normal(p.shape).astype(np.float32) for p in ps]
    bufs = [tt.DeviceBuffer.from_numpy(p) for p in ps]
    gbufs = [tt.DeviceBuffer.from_numpy(g) for g in gs]
    opt = tt.SGD(bufs, lr=0.01, momentum=0.9)
    opt.step(gbufs)
    opt.step(gbufs)
    for b, p, g in zip(bufs, ps, gs):
        p1, v1 = O.sgd(p, g, 0.01, 0.9, np.zeros_like(p))
        p2, _ = O.sgd(p1, g, 0.01, 0.9, v1)
        assert_bitexact(b.numpy(), p2)


def test_profile_and_launch_count(cache_dir):
    g = tt.Graph()
    a, b = g.input([256, 128]), g.input([128, 64])
    y = tt.relu(a @ b)
    prog = tt.compile(g, outputs=[y, tt.sum(y, [1])], cache_dir=cache_dir)
    prog.set_profiling(True)
    n0 = tt.launch_count()
    prog.run({a: np.ones((256, 128)), b: np.ones((128, 64))})
    assert tt.launch_count() > n0
    prof = prog.profile()
    assert len(prof) >= 2 and all(ms >= 0 for _, ms in prof)
    assert any(lbl.startswith("gemm") for lbl, _ in prof)


def test_cache_reuse_and_diagnostics(cache_dir):
    g = tt.Graph()
    x = g.input([10, 20], name="X")
    y = tt.relu(x + 1.0)
    p1 = tt.compile(g, outputs=[y], cache_dir=cache_dir)
    p2 = tt.compile(g, outputs=[y], cache_dir=cache_dir)
    assert p1.cubin_path() == p2.cubin_path() and os.path.exists(p1.cubin_path())
    assert "input<float32>[10, 20]" in p1.original_ir() and "relu" in p1.optimized_ir()
    src = p1.generated_source()
    assert "__global__" in src and "ttk_region" in src
    plan = p1.execution_plan()
    assert "Execution Mode: Compiled CUDA" in plan and "Memory Planning:" in plan
    np.testing.assert_array_equal(p2.run({x: np.zeros((10, 20))}).numpy(), np.ones((10, 20)))
