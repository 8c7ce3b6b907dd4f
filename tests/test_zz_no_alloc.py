"""tt_gemm_f32_noalloc: the GEMM entry point for callers that cannot allocate device
memory (code that must not touch the device allocator, or a host that hands the
library only one call's buffers); its scratch is a static device array inside the
library.  Checked through the C ABI against the CPU oracle's matmul (the reference's
blocked fp32 loop) and an fp64 product, on two calls in a row so that the second call
runs over the scratch the first one left behind, and against the regular compiled
matmul.  Shapes cover the tensor-core path (CTA pairs and single CTAs) and a 10-wide
product whose plan splits K, so its partial sums live in the static array too.
This file is collected last on purpose."""

import ctypes

import numpy as np
import pytest

from parity import GEMM_FROB_RTOL, assert_norm

import tinytensor_b200 as tt
from oracle import oracle as O
from tinytensor_b200 import _lib

pytestmark = pytest.mark.gpu


def _noalloc(a_dev, b_dev, c_dev, m, n, k, stream, status=None):
    _lib.check(_lib.lib.tt_gemm_f32_noalloc(a_dev.ptr if a_dev is not None else None,
                                            b_dev.ptr if b_dev is not None else None, c_dev.ptr, m, n, k,
                                            status, stream.handle))


@pytest.mark.parametrize("m,n,k", [(640, 384, 1536), (200, 96, 2048), (4096, 10, 4096)])
def test_noalloc_gemm_matches_oracle_and_fp64_twice(m, n, k, tmp_path):
    tt.device_init(0)
    st = tt.Stream()
    for call in range(2):
        rng = np.random.default_rng(100 + call)
        a = (rng.standard_normal((m, k)) / np.sqrt(k)).astype(np.float32)
        b = (rng.standard_normal((k, n)) / np.sqrt(k)).astype(np.float32)
        da, db, dc = tt.DeviceBuffer.from_numpy(a), tt.DeviceBuffer.from_numpy(b), tt.DeviceBuffer([m, n])
        _noalloc(da, db, dc, m, n, k, st)
        st.synchronize()
        got = dc.numpy()
        assert_norm(got, O.matmul(a, b), GEMM_FROB_RTOL)
        assert_norm(got, a.astype(np.float64) @ b.astype(np.float64), GEMM_FROB_RTOL)
        g = tt.Graph()
        na, nb = g.input([m, k]), g.input([k, n])
        compiled = tt.compile(g, outputs=[na @ nb], cache_dir=str(tmp_path)).run({na: a, nb: b}).numpy()
        assert_norm(got, compiled, GEMM_FROB_RTOL)


def test_noalloc_skinny_plan_uses_split_k():
    """The (4096, 10, 4096) case above runs the skinny kernel with K split across CTAs,
    whose partials live in the static array."""
    tt.device_init(0)
    g = tt.Graph()
    na, nb = g.input([4096, 4096]), g.input([4096, 10])
    plan = tt.compile(g, outputs=[na @ nb]).execution_plan()
    assert "simt_skinny" in plan and "splitk" in plan, plan


def test_noalloc_gemm_reports_through_caller_status_word():
    """A caller-supplied status word stays 0 after correct runs (a bounded-wait timeout
    would set it); the product is right on both calls."""
    tt.device_init(0)
    st = tt.Stream()
    m, n, k = 512, 256, 1024
    status = tt.DeviceBuffer([1])
    _lib.check(_lib.lib.tt_memcpy(status.ptr, bytes(4), 4, _lib.H2D, None))
    for call in range(2):
        rng = np.random.default_rng(7 + call)
        a = (rng.standard_normal((m, k)) / np.sqrt(k)).astype(np.float32)
        b = (rng.standard_normal((k, n)) / np.sqrt(k)).astype(np.float32)
        da, db, dc = tt.DeviceBuffer.from_numpy(a), tt.DeviceBuffer.from_numpy(b), tt.DeviceBuffer([m, n])
        _noalloc(da, db, dc, m, n, k, st, status=ctypes.c_void_p(status.ptr))
        st.synchronize()
        assert_norm(dc.numpy(), a.astype(np.float64) @ b.astype(np.float64), GEMM_FROB_RTOL)
        word = np.frombuffer(status.numpy().tobytes(), dtype=np.int32)[0]
        assert word == 0, f"status word {word:#x} after a correct run"


def test_noalloc_gemm_k0_gives_zeros():
    """K = 0: C = 0, as the reference's matmul returns (operators.cpp:256-259); the empty
    operands may be NULL.  C is filled with garbage first so the zeros are written."""
    tt.device_init(0)
    st = tt.Stream()
    m, n = 64, 48
    dc = tt.DeviceBuffer.from_numpy(np.full((m, n), 7.0, np.float32))
    for _ in range(2):
        _noalloc(None, None, dc, m, n, 0, st)
        st.synchronize()
        assert np.array_equal(dc.numpy(), np.zeros((m, n), np.float32))


def test_noalloc_gemm_rejects_products_beyond_its_scratch():
    tt.device_init(0)
    # M <= 128 runs on single-CTA tiles, whose operands are split into hi/lo copies in
    # scratch: 2 * (m + n) * k floats = 264 MB, far above the 32 MiB capacity
    m, n, k = 128, 4096, 8192
    da, db, dc = tt.DeviceBuffer([m, k]), tt.DeviceBuffer([k, n]), tt.DeviceBuffer([m, n])
    with pytest.raises(tt.MemoryError, match="scratch"):
        _lib.check(_lib.lib.tt_gemm_f32_noalloc(da.ptr, db.ptr, dc.ptr, m, n, k, None, None))
