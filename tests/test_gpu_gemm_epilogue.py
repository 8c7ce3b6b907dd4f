"""GPU parity of GEMMs that apply a ReLU or tanh in their epilogue.

The scheduler folds an activation whose only input is a matmul into that GEMM (the
matmul's pre-activation value is then never stored).  Every GEMM kernel variant carries
the epilogue: the tcgen05 CTA-pair and single-CTA kernels (and their split-K reduce),
the CUDA-core skinny kernels (N <= 16 and M <= 16), the small-K kernel and the FFMA
tile kernel.  Each case checks that the planner chose that kernel with the folded
activation, and compares act(A @ B) against the oracle's fp32 matmul followed by its
activation at the GEMM tolerance (relative Frobenius; tanh and ReLU are 1-Lipschitz,
so they do not amplify the product's error)."""

import numpy as np
import pytest

from parity import GEMM_FROB_RTOL, assert_norm

import tinytensor_b200 as tt
from oracle import oracle as O

pytestmark = pytest.mark.gpu

CASES = [
    # m, n, k, kernel label in the plan
    (512, 384, 256, "tcgen05_3xtf32["),          # CTA pairs (M > 128)
    (128, 512, 640, "tcgen05_3xtf32["),          # one CTA per 128-row tile
    (1024, 1024, 1024, "splitk"),                # tensor cores, K split, epilogue in the reduce
    (3000, 10, 700, "simt_skinny["),             # N <= 16
    (10, 515, 640, "simt_skinny_t["),            # M <= 16
    (2048, 512, 10, "simt_smallk["),             # K <= 16
    (40, 300, 200, "simt["),                     # FFMA tiles
]


@pytest.mark.parametrize("act", ["relu", "tanh"])
@pytest.mark.parametrize("m,n,k,kernel", CASES)
def test_activation_in_gemm_epilogue(m, n, k, kernel, act, cache_dir):
    rng = np.random.default_rng(m * 7 + n * 3 + k)
    # entries of A @ B are O(1): both signs and tanh's curved range are exercised
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = (rng.standard_normal((k, n)) / np.sqrt(k)).astype(np.float32)
    g = tt.Graph()
    na, nb = g.input([m, k]), g.input([k, n])
    y = tt.relu(na @ nb) if act == "relu" else tt.tanh(na @ nb)
    prog = tt.compile(g, outputs=[y], cache_dir=cache_dir)
    plan = prog.execution_plan()
    assert kernel in plan and f"+{act}]" in plan, plan
    assert "fused[" not in plan  # no separate activation pass
    got = prog.run({na: a, nb: b}).numpy()
    op = O.RELU if act == "relu" else O.TANH
    ref = O.unary(op, O.matmul(a, b))
    assert_norm(got, ref, GEMM_FROB_RTOL)
    if act == "relu":
        assert np.all(got >= 0) and not np.any(np.signbit(got))  # ReLU contract: -0 and NaN become +0


def test_relu_mask_reads_the_relu_output(cache_dir):
    """relu(X W1) W2 with gradients: the ReLU folds into the forward GEMM and the
    backward mask step() reads the ReLU's output, which gives the same mask bit for
    bit; the gradients match the oracle's."""
    rng = np.random.default_rng(8)
    x = rng.standard_normal((256, 192)).astype(np.float32)
    w1 = (rng.standard_normal((192, 320)) / np.sqrt(192)).astype(np.float32)
    w2 = (rng.standard_normal((320, 64)) / np.sqrt(320)).astype(np.float32)
    g = tt.Graph()
    nx, n1, n2 = g.input([256, 192]), g.input([192, 320]), g.input([320, 64])
    loss = tt.mean(tt.tanh(tt.relu(nx @ n1) @ n2))
    prog = tt.compile_gradients(g, loss, [n1, n2], cache_dir=cache_dir)
    plan = prog.execution_plan()
    assert "+relu]" in plan and "+tanh]" in plan, plan
    got = prog.run({nx: x, n1: w1, n2: w2})
    ref = O.gradients(g, loss, {nx: x, n1: w1, n2: w2}, [n1, n2])
    assert_norm(got[1].numpy(), ref[0], GEMM_FROB_RTOL)
    assert_norm(got[2].numpy(), ref[1], GEMM_FROB_RTOL)
