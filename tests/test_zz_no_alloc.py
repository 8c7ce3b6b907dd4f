"""tt_gemm_f32_noalloc: the GEMM entry point for callers that cannot allocate device
memory (its scratch is a static device array inside the library).  Checked through the
C ABI against the regular compiled matmul (tt_compile / tt_program_run), on two calls
in a row so that the second call runs over the scratch the first one left behind.
This file is collected last on purpose."""

import ctypes

import numpy as np
import pytest

from parity import GEMM_FROB_RTOL, assert_norm

import tinytensor_b200 as tt
from tinytensor_b200 import _lib

pytestmark = pytest.mark.gpu


def _noalloc(a_dev, b_dev, c_dev, m, n, k, stream):
    _lib.check(_lib.lib.tt_gemm_f32_noalloc(a_dev.ptr, b_dev.ptr, c_dev.ptr, m, n, k, None, stream.handle))


@pytest.mark.parametrize("m,n,k", [(640, 384, 1536), (200, 96, 2048)])
def test_noalloc_gemm_matches_compiled_matmul_twice(m, n, k, tmp_path):
    tt.device_init(0)
    st = tt.Stream()
    for call in range(2):
        rng = np.random.default_rng(100 + call)
        a = (rng.standard_normal((m, k)) / np.sqrt(k)).astype(np.float32)
        b = (rng.standard_normal((k, n)) / np.sqrt(k)).astype(np.float32)
        g = tt.Graph()
        na, nb = g.input([m, k]), g.input([k, n])
        ref = tt.compile(g, outputs=[na @ nb], cache_dir=str(tmp_path)).run({na: a, nb: b}).numpy()
        da, db, dc = tt.DeviceBuffer.from_numpy(a), tt.DeviceBuffer.from_numpy(b), tt.DeviceBuffer([m, n])
        _noalloc(da, db, dc, m, n, k, st)
        st.synchronize()
        assert_norm(dc.numpy(), ref, GEMM_FROB_RTOL)


def test_noalloc_gemm_rejects_products_beyond_its_scratch():
    tt.device_init(0)
    # M <= 128 runs on single-CTA tiles, whose operands are split into hi/lo copies in
    # scratch: 2 * (m + n) * k floats = 264 MB, far above the 32 MiB capacity
    m, n, k = 128, 4096, 8192
    da, db, dc = tt.DeviceBuffer([m, k]), tt.DeviceBuffer([k, n]), tt.DeviceBuffer([m, n])
    with pytest.raises(tt.MemoryError, match="scratch"):
        _lib.check(_lib.lib.tt_gemm_f32_noalloc(da.ptr, db.ptr, dc.ptr, m, n, k, None, None))
