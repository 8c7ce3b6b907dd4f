"""GPU parity on seeded random graphs: the graphs of the oracle's reference cross-check
(broadcasting elementwise chains with scalar constants and IEEE special values,
reductions over random axes with and without keepdims, transposes, 2-D and batched
matmuls, and random differentiable graphs through their compiled backward pass)
compiled for the B200 and run through the C ABI, held to the oracle with the parity
contract's tolerances: bit-exact for chains of + - * / relu and for transposes of them,
the transcendental bound where sigmoid appears, norm-wise for reductions, products and
gradients, with NaN / inf patterns equal everywhere."""

import numpy as np
import pytest

from parity import (
    GEMM_FROB_RTOL,
    REDUCTION_NORM_RTOL,
    assert_bitexact,
    assert_elementwise_scaled,
    assert_norm,
)
from test_oracle_fuzz import SPECIALS_NO_OVERFLOW, _elementwise_case, _gradient_case, _matmul_case

import tinytensor_b200 as tt
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _assert_classes_then_norm(got, ref, rtol):
    got, ref = np.asarray(got, np.float32), np.asarray(ref, np.float32)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert np.array_equal(np.isnan(got), np.isnan(ref)), "NaN pattern differs"
    inf = np.isinf(ref)
    assert np.array_equal(got[inf], ref[inf]), "inf values differ"
    assert not np.isinf(got[~inf]).any(), "inf where the oracle is finite"
    fin = np.isfinite(ref)
    assert_norm(got[fin], ref[fin], rtol)


def _run(g, cache_dir):
    outs = list(g.outputs)
    prog = tt.compile(g, outputs=outs, cache_dir=cache_dir)
    return prog, outs


@pytest.mark.parametrize("seed", range(60))
def test_elementwise_and_reduction_graphs(seed, cache_dir):
    g, feed = _elementwise_case(1000 + seed)
    prog, outs = _run(g, cache_dir)
    res = prog.run(feed)
    got = [r.numpy() for r in (res if isinstance(res, list) else [res])]
    orc = O.evaluate(g, feed, outs)
    transcendental = any(n.op == O.SIGMOID for n in g.nodes)
    mags = O.magnitude(g, feed, outs) if transcendental else None
    for i, (o, gv, ov) in enumerate(zip(outs, got, orc)):
        if o.op in (O.REDUCE_SUM, O.REDUCE_MEAN):
            _assert_classes_then_norm(gv, ov, REDUCTION_NORM_RTOL)
        elif transcendental:
            assert_elementwise_scaled(gv, ov, mags[i])
        else:
            assert_bitexact(gv, ov)


@pytest.mark.parametrize("seed", range(30))
def test_matmul_graphs(seed, cache_dir):
    g, feed = _matmul_case(5000 + seed, SPECIALS_NO_OVERFLOW)
    prog, outs = _run(g, cache_dir)
    res = prog.run(feed)
    got = [r.numpy() for r in (res if isinstance(res, list) else [res])]
    for gv, ov in zip(got, O.evaluate(g, feed, outs)):
        _assert_classes_then_norm(gv, ov, GEMM_FROB_RTOL)


@pytest.mark.parametrize("seed", range(40))
def test_gradient_graphs(seed, cache_dir):
    g, loss, wrt, feed = _gradient_case(9000 + seed, SPECIALS_NO_OVERFLOW)
    prog = tt.compile_gradients(g, loss, wrt, cache_dir=cache_dir)
    got = [r.numpy() for r in prog.run(feed)[1:]]
    assert len(got) == len(wrt)
    for gv, ov in zip(got, O.gradients(g, loss, feed, wrt)):
        _assert_classes_then_norm(gv, ov, GEMM_FROB_RTOL)
