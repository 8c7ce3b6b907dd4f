"""Failure detection on the GPU without a fault: a wait whose arrival never comes (an
mbarrier nothing arrives at) gives up after its clock budget through the same bounded
wait the tensor-core GEMM kernels use, records its code in a status word the host
reads, and leaves the context usable for the next work."""

import ctypes
import time

import numpy as np
import pytest

from parity import GEMM_FROB_RTOL, assert_norm

import tinytensor_b200 as tt
from tinytensor_b200 import _lib

pytestmark = pytest.mark.gpu

ST_TIMEOUT_FULL = 0x200


def test_missing_arrival_ends_in_a_status_not_a_hang(cache_dir):
    tt.device_init(0)
    status = ctypes.c_int32(-1)
    t0 = time.time()
    _lib.check(_lib.lib.tt_selftest_bounded_wait(20_000_000, ctypes.byref(status)))  # ~10 ms of SM clock
    assert status.value == ST_TIMEOUT_FULL
    assert time.time() - t0 < 30.0
    # the context is still usable: a tensor-core GEMM runs and is correct
    rng = np.random.default_rng(3)
    a = (rng.standard_normal((512, 512)) / np.sqrt(512)).astype(np.float32)
    b = (rng.standard_normal((512, 512)) / np.sqrt(512)).astype(np.float32)
    g = tt.Graph()
    na, nb = g.input([512, 512]), g.input([512, 512])
    prog = tt.compile(g, outputs=[na @ nb], cache_dir=cache_dir)
    assert "tcgen05" in prog.execution_plan()
    c = prog.run({na: a, nb: b}).numpy()
    assert_norm(c, a.astype(np.float64) @ b.astype(np.float64), GEMM_FROB_RTOL)

