"""Host-side logic of the backend, no GPU: the C ABI exports, graph building and
its errors, IR text, scheduling/fusion, the memory plan, CUDA generation (NVRTC
compiles every case to an sm_100a cubin here) and the kernel cache protocol."""

import os
import re

import numpy as np
import pytest

from cases import CASES, build

import tinytensor_b200 as tt
from tinytensor_b200 import _lib

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
HOST = tt.FLAG_HOST_ONLY


def _host_compile(g, outs, cache_dir, **kw):
    return tt.compile(g, outputs=outs, cache_dir=cache_dir, flags=HOST | kw.pop("flags", 0), **kw)


def test_library_exports_every_declared_symbol():
    with open(os.path.join(ROOT, "include", "tt_cuda.h")) as f:
        hdr = f.read()
    declared = set(re.findall(r"^\s*(?:int|const char\*|uint64_t)\s+(tt_\w+)\s*\(", hdr, re.M))
    assert len(declared) >= 25
    for name in declared:
        assert hasattr(_lib.lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert set(_lib.SIGNATURES) == declared


def test_no_device_is_reported_not_faked():
    # Without a GPU the library still loads; device calls fail loudly (no CPU fallback).
    if os.environ.get("CUDA_VISIBLE_DEVICES") is None and os.path.exists("/dev/nvidia0"):
        pytest.skip("a GPU is present")
    with pytest.raises(tt.NoDeviceError):
        tt.device_init(0)


def test_builder_errors_match_reference():
    g = tt.Graph()
    a, b = g.input([2, 3]), g.input([4, 5])
    with pytest.raises(tt.ShapeError):
        a @ b
    with pytest.raises(tt.BroadcastError):
        a + b
    with pytest.raises(tt.DimensionError):
        tt.transpose(a, 0, 2)
    with pytest.raises(tt.DimensionError):
        tt.sum(a, [3])
    with pytest.raises(tt.TypeError):
        tt.relu(1.0)


@pytest.mark.parametrize("name", sorted(CASES))
def test_every_case_generates_and_compiles(name, cache_dir):
    c = build(name)
    if c["kind"] == "forward":
        p = _host_compile(c["graph"], c["outputs"], cache_dir)
    else:
        p = tt.compile_gradients(c["graph"], c["loss"], c["wrt"], cache_dir=cache_dir, flags=HOST)
    src = p.generated_source()
    plan = p.execution_plan()
    assert "Execution Mode: Compiled CUDA" in plan and "Memory Planning:" in plan
    if "ttk_region" in src:
        assert os.path.exists(p.cubin_path())
        with open(p.cubin_path(), "rb") as f:
            assert f.read(4) == b"\x7fELF"


def test_fused_chain_is_one_kernel(cache_dir):
    g = tt.Graph()
    a, b, c = g.input([1024, 1024]), g.input([1024, 1024]), g.input([1, 1024])
    y = tt.relu(a * b + c) * 0.5 - tt.exp(-a)
    p = _host_compile(g, [y], cache_dir)
    plan = p.execution_plan()
    assert "Kernel Launches (1)" in plan
    src = p.generated_source()
    assert src.count("__global__") == 1
    assert src.count("float4") >= 3  # vectorised loads of a, b and the broadcast row of c
    assert "0x3f000000u" in src      # the 0.5 constant, bit-exact
    # no intermediate buffers: peak planned memory 0
    assert "Memory Planning: Peak 0 bytes" in plan


def test_transposes_fold_into_consumers(cache_dir):
    g = tt.Graph()
    x = g.input([64, 32])
    w = g.input([48, 32])
    y = x @ tt.transpose(w, 0, 1)
    s = tt.sum(tt.transpose(x, 0, 1), [0])
    p = _host_compile(g, [y, s], cache_dir)
    plan = p.execution_plan()
    assert "copy" not in plan
    assert "B:K" in plan            # GEMM reads W as a K-major operand directly
    assert "reduce_sum/row" in plan  # the transposed column sum is a row reduction of x


def test_batched_matmul_broadcasts(cache_dir):
    """Whole-batch broadcast is a zero batch stride; a partial broadcast
    ([2,1,..] x [5,..] -> [2,5,..]) is copied to the output's batch shape first."""
    g = tt.Graph()
    a, b = g.input([3, 64, 32]), g.input([32, 48])
    plan = _host_compile(g, [a @ b], cache_dir).execution_plan()
    assert "copy" not in plan and " b3 " in plan
    g = tt.Graph()
    a, b = g.input([2, 1, 64, 32]), g.input([5, 32, 48])
    y = a @ b
    assert y.shape == [2, 5, 64, 48]
    plan = _host_compile(g, [y], cache_dir).execution_plan()
    assert "copy[2, 5, 64, 32]" in plan and "copy[2, 5, 32, 48]" in plan and " b10 " in plan


def test_fusion_respects_launch_dependencies(cache_dir):
    # sum(x) feeds back into an elementwise chain of x: the two regions must not merge
    g = tt.Graph()
    x = g.input([128, 64])
    s = tt.sum(tt.relu(x), [1], keepdims=True)
    y = tt.relu(x) * s + x
    p = _host_compile(g, [y], cache_dir)
    plan = p.execution_plan()
    assert re.search(r"Kernel Launches \((\d+)\)", plan).group(1) == "3"


def test_memory_planner_reuses_slots_on_a_chain(cache_dir):
    # test_adversarial_memory_planner.cpp: a linear chain needs at most 2 buffers
    # 48x48 products take the CUDA-core kernel, which needs no scratch buffer
    g = tt.Graph()
    x = g.input([48, 48])
    ws = [g.input([48, 48]) for _ in range(6)]
    h = x
    for w in ws:
        h = h @ w
    p = _host_compile(g, [h], cache_dir)
    plan = p.execution_plan()
    nslots = int(re.search(r"slots \d+ in (\d+) slots", plan).group(1))
    assert nslots <= 2
    # slots never overlap in the arena
    slots = [(int(o), int(c)) for o, c in re.findall(r"slot \d+ @ (\d+) capacity (\d+)", plan)]
    for (o1, c1), (o2, _) in zip(slots, slots[1:]):
        assert o1 + c1 <= o2


def test_memory_planner_keeps_live_values_apart(cache_dir):
    # diamond: both branches are live at the join, so they cannot share a slot
    g = tt.Graph()
    x, w1, w2 = g.input([32, 32]), g.input([32, 32]), g.input([32, 32])
    a = x @ w1
    b = x @ w2
    y = a @ b
    p = _host_compile(g, [y], cache_dir)
    plan = p.execution_plan()
    outs = re.findall(r"gemm/[^\]]*\] -> arena:(\d+)", plan)
    assert len(outs) == 2 and outs[0] != outs[1]


def test_ir_of_fused_reference_node_is_expanded(cache_dir):
    # A reference FusedElementwise node "relu(sub(@0, @1))" is computed as written
    # (the reference codegen would emit relu(a + b): src/codegen/cpp_backend.cpp:345-387).
    g = tt.Graph()
    a, b = g.input([16]), g.input([16])
    f = tt.graph.Node(g, _lib.OP_FUSED, [16], "float32", [a, b])
    f.expr = "relu(sub(@0, @1))"
    g._add(f)
    p = _host_compile(g, [f], cache_dir)
    assert "relu" in p.optimized_ir() and "sub" in p.optimized_ir()
    assert "v - " in p.generated_source() or " - a" in p.generated_source()


def test_cache_hit_and_truncated_entry_heals(cache_dir, tmp_path):
    d = str(tmp_path / "cache")
    g = tt.Graph()
    x = g.input([40])
    y = tt.sigmoid(x) * 3.0
    p1 = _host_compile(g, [y], d)
    path = p1.cubin_path()
    assert os.path.exists(path)
    mtime = os.path.getmtime(path)
    p2 = _host_compile(g, [y], d)
    assert p2.cubin_path() == path and os.path.getmtime(path) == mtime  # hit: not rewritten
    with open(path, "wb") as f:
        f.write(b"\x7fELF")  # truncated (< 64 bytes)
    p3 = _host_compile(g, [y], d)
    assert os.path.getsize(p3.cubin_path()) > 64
    assert not [f for f in os.listdir(d) if ".tmp." in f]


def test_cache_concurrent_processes(tmp_path):
    """Several processes compile the same graph into one cache dir: one cubin, no temp
    leftovers (tests/python/test_multiprocess_cache.py:30-92)."""
    import multiprocessing as mp
    d = str(tmp_path / "mp")
    ctx = mp.get_context("spawn")
    with ctx.Pool(4) as pool:
        paths = pool.map(_mp_compile, [d] * 4)
    assert len(set(paths)) == 1
    files = os.listdir(d)
    assert sum(f.endswith(".cubin") for f in files) == 1
    assert not [f for f in files if ".tmp." in f]


def _mp_compile(d):
    import sys
    sys.path.insert(0, ROOT)
    import tinytensor_b200 as tt2
    g = tt2.Graph()
    x = g.input([33, 9])
    y = tt2.relu(x * x - 1.0)
    return tt2.compile(g, outputs=[y], cache_dir=d, flags=tt2.FLAG_HOST_ONLY).cubin_path()


def test_gradient_graph_structure(cache_dir):
    g = tt.Graph()
    x, w = g.input([8, 4]), g.input([4, 3])
    loss = tt.mean(tt.relu(x @ w))
    p = tt.compile_gradients(g, loss, [w], cache_dir=cache_dir, flags=HOST)
    ir = p.optimized_ir()
    assert "step" in ir and "transpose" in ir and ir.count("matmul") == 2  # dx is dead and eliminated
    assert p.num_outputs == 2 and p.output_shapes == [[], [4, 3]]


def test_run_validates_inputs_before_device(cache_dir):
    g = tt.Graph()
    a = g.input([4])
    p = _host_compile(g, [tt.relu(a)], cache_dir)
    with pytest.raises(tt.RuntimeExecutionError):
        p.run({})
    with pytest.raises(tt.ShapeError):
        p.run({a: np.ones(8, np.float32)})
    with pytest.raises(tt.NoDeviceError):
        p.run({a: np.ones(4, np.float32)})


def test_unsupported_dtype_is_a_compile_error(cache_dir):
    g = tt.Graph()
    a = g.input([4], dtype=tt.float64)
    with pytest.raises(tt.CompileError):
        _host_compile(g, [tt.relu(a)], cache_dir)


def test_gradients_are_scheduled_early_with_output_steps(cache_dir):
    """Launches that finish graph outputs run as soon as their inputs allow: in the MLP
    gradient program dW2's GEMM precedes the dH1 GEMM, so its all-reduce can overlap it;
    output_steps() gives the launch after which each output is complete."""
    rows = 64
    g = tt.Graph()
    X, T = g.input([rows, 96]), g.input([rows, 10])
    W1, W2, W3 = g.input([96, 256]), g.input([256, 256]), g.input([256, 10])
    d = tt.tanh(tt.relu(X @ W1) @ W2) @ W3 - T
    loss = tt.mean(d * d)
    p = tt.compile_gradients(g, loss, [W1, W2, W3], cache_dir=cache_dir, flags=HOST)
    launches = [line.strip() for line in p.execution_plan().splitlines() if line.strip().startswith("[")]
    steps = p.output_steps()
    assert len(steps) == 4 and len(set(steps)) == 4
    for k, s in enumerate(steps):
        assert 0 <= s < len(launches) and f"output:{k}" in launches[s]
    loss_s, dw1_s, dw2_s, dw3_s = steps
    assert dw3_s < dw2_s < dw1_s
    dh1 = [i for i, l in enumerate(launches) if "[64x256x256" in l and "B:K" in l]
    assert dh1 and dw2_s < dh1[0]
    # input_steps(): the launch after which each input is no longer read — W1 only by the
    # first GEMM, W2 last by dH1 = dZ2 W2^T (after dW2 is out), X last by dW1 = X^T dZ1
    x_s, t_s, w1_s, w2_s, w3_s = p.input_steps()
    assert w1_s == 0 and x_s == dw1_s == len(launches) - 1
    assert w2_s == dh1[0] and dw2_s < w2_s
    assert 0 <= t_s < dw3_s and 0 <= w3_s < len(launches)


def test_independent_gemms_run_side_by_side_without_sharing_memory(cache_dir):
    """dW2 and dH1 of the MLP backward are adjacent, independent GEMMs: they are marked to
    run on two streams, and none of their buffers overlap in the arena.  TT_FLAG_SERIAL
    keeps every launch on one stream."""
    rows = 512
    g = tt.Graph()
    X, T = g.input([rows, 256]), g.input([rows, 10])
    W1, W2, W3 = g.input([256, 512]), g.input([512, 512]), g.input([512, 10])
    d = tt.tanh(tt.relu(X @ W1) @ W2) @ W3 - T
    loss = tt.mean(d * d)
    p = tt.compile_gradients(g, loss, [W1, W2, W3], cache_dir=cache_dir, flags=HOST)
    lines = [line.strip() for line in p.execution_plan().splitlines() if line.strip().startswith("[")]
    pairs = [i for i, line in enumerate(lines) if "runs beside" in line]
    assert pairs
    sizes = {}
    for i in pairs:
        a, b = lines[i], lines[i + 1]
        assert "gemm/" in a and "gemm/" in b

        def spans(line):
            out = []
            m = re.search(r"-> arena:(\d+)", line)
            shape = re.search(r"\[(\d+)x(\d+)x(\d+)", line)
            if m and shape:
                out.append((int(m.group(1)), int(shape.group(1)) * int(shape.group(2)) * 4))
            s = re.search(r"scratch=(\d+)@(\d+)", line)
            if s:
                out.append((int(s.group(2)), int(s.group(1))))
            return out

        for (o1, n1) in spans(a):
            for (o2, n2) in spans(b):
                assert o1 + n1 <= o2 or o2 + n2 <= o1, (a, b)
        sizes[i] = (a, b)
    serial = tt.compile_gradients(g, loss, [W1, W2, W3], cache_dir=cache_dir, flags=HOST | tt.FLAG_SERIAL)
    assert "runs beside" not in serial.execution_plan()


def test_bounded_wait_selftest_rejects_unbounded_budgets():
    import ctypes
    status = ctypes.c_int32(0)
    with pytest.raises(ValueError):
        _lib.check(_lib.lib.tt_selftest_bounded_wait(10**12, ctypes.byref(status)))


def test_activations_fold_into_gemm_epilogues(cache_dir):
    """A ReLU or tanh whose only input is a matmul runs in that GEMM's epilogue; the
    ReLU's backward mask reads the ReLU output (the same mask), so the forward matmul
    keeps a single reader and no separate activation pass remains."""
    g = tt.Graph()
    x, w1, w2 = g.input([256, 192]), g.input([192, 320]), g.input([320, 64])
    loss = tt.mean(tt.tanh(tt.relu(x @ w1) @ w2))
    plan = tt.compile_gradients(g, loss, [w1, w2], cache_dir=cache_dir, flags=HOST).execution_plan()
    gemms = [line for line in plan.splitlines() if "] gemm/" in line]
    assert sum("+relu]" in line for line in gemms) == 1 and sum("+tanh]" in line for line in gemms) == 1, plan
    regions = [line for line in plan.splitlines() if "fused[" in line]
    assert not any("relu" in line or "tanh" in line for line in regions), plan
    # TT_FLAG_NO_GEMM_FUSION keeps the epilogues plain
    plain = tt.compile_gradients(g, loss, [w1, w2], cache_dir=cache_dir,
                                 flags=HOST | tt.FLAG_NO_GEMM_FUSION).execution_plan()
    assert "+relu]" not in plain and "+tanh]" not in plain


def test_matmul_with_another_reader_keeps_its_activation_apart(cache_dir):
    g = tt.Graph()
    a, b = g.input([256, 128]), g.input([128, 256])
    m = a @ b
    plan = _host_compile(g, [tt.relu(m), m * 2.0], cache_dir).execution_plan()
    assert "+relu]" not in plan and "relu" in plan
    # the activation as a graph output: the GEMM writes that output directly
    g2 = tt.Graph()
    a2, b2 = g2.input([256, 128]), g2.input([128, 256])
    plan2 = _host_compile(g2, [tt.tanh(a2 @ b2)], cache_dir).execution_plan()
    assert "+tanh] -> output:0" in plan2 and "Kernel Launches (1)" in plan2, plan2


def test_dz_regions_write_the_gemm_operand_copies(cache_dir):
    """In the MLP backward pass the dZ regions write the hi/lo copies their tensor-core
    GEMMs read (dZ2 in both layouts for dW2 = H1^T dZ2 and dH1 = dZ2 W2^T, dZ1
    transposed for dW1 = X^T dZ1) and no fp32 dZ; those GEMMs run no pre-pass for that
    operand, and the copies' buffer stays apart from every buffer of the launches it
    outlives."""
    g = tt.Graph()
    x, t = g.input([4096, 1024]), g.input([4096, 10])
    w1, w2, w3 = g.input([1024, 4096]), g.input([4096, 4096]), g.input([4096, 10])
    d = tt.tanh(tt.relu(x @ w1) @ w2) @ w3 - t
    loss = tt.mean(d * d)
    plan = tt.compile_gradients(g, loss, [w1, w2, w3], cache_dir=cache_dir, flags=HOST).execution_plan()
    lines = [line.strip() for line in plan.splitlines() if line.strip().startswith("[")]
    producers = [i for i, line in enumerate(lines) if "(writes hi/lo of" in line]
    assert len(producers) == 2, plan
    both, tr = lines[producers[0]], lines[producers[1]]
    assert "(writes hi/lo of X and X^T, not X)" in both and "(writes hi/lo of X^T, not X)" in tr, plan
    readers = [line for line in lines if "hi/lo from [" in line]
    assert len(readers) == 3 and all("tcgen05" in line for line in readers), plan
    for p in producers:
        m = re.search(r"copies=(\d+)@(\d+)", lines[p])
        size, off = int(m.group(1)), int(m.group(2))
        last = max(i for i, line in enumerate(lines) if f"hi/lo from [{p}])" in line)
        for line in lines[p + 1: last + 1]:
            for sz, o in re.findall(r"scratch=(\d+)@(\d+)", line):
                assert int(o) + int(sz) <= off or off + size <= int(o), line
            for o in re.findall(r"(?:-> |copies=\d+@)arena:(\d+)", line):
                assert not (off <= int(o) < off + size), line
    # TT_FLAG_NO_GEMM_FUSION: plain regions, every GEMM splits its own operands
    plain = tt.compile_gradients(g, loss, [w1, w2, w3], cache_dir=cache_dir,
                                 flags=HOST | tt.FLAG_NO_GEMM_FUSION).execution_plan()
    assert "hi/lo" not in plain


def test_small_k_product_is_formed_inside_its_region(cache_dir):
    """The MLP's dH2 = dY W3^T (K = 10, read only by the dZ2 region) is no GEMM launch:
    the dZ2 region forms it; a small-K product that is also a graph output stays a GEMM."""
    g = tt.Graph()
    x, t = g.input([4096, 1024]), g.input([4096, 10])
    w1, w2, w3 = g.input([1024, 4096]), g.input([4096, 4096]), g.input([4096, 10])
    d = tt.tanh(tt.relu(x @ w1) @ w2) @ w3 - t
    loss = tt.mean(d * d)
    plan = tt.compile_gradients(g, loss, [w1, w2, w3], cache_dir=cache_dir, flags=HOST).execution_plan()
    assert "simt_smallk" not in plan and "fused[matmul,mul,sub,mul]" in plan, plan
    g2 = tt.Graph()
    a, b = g2.input([300, 8]), g2.input([8, 256])
    m = a @ b
    assert "simt_smallk" in _host_compile(g2, [m, m * 3.0], cache_dir).execution_plan()


def test_tiled_small_k_region_forms_the_product_k_outermost(cache_dir):
    """The tiled dZ2 region forms its K = 10 product with k outermost (one float4 of B per
    k for the tile's four rows) and asks for 5 resident CTAs per SM; the 10-wide output
    and weight-gradient GEMMs take the skinny kernels."""
    g = tt.Graph()
    x, t = g.input([4096, 1024]), g.input([4096, 10])
    w1, w2, w3 = g.input([1024, 4096]), g.input([4096, 4096]), g.input([4096, 10])
    d = tt.tanh(tt.relu(x @ w1) @ w2) @ w3 - t
    p = tt.compile_gradients(g, tt.mean(d * d), [w1, w2, w3], cache_dir=cache_dir, flags=HOST)
    src, plan = p.generated_source(), p.execution_plan()
    tiled = [k for k in src.split("extern \"C\" __global__")[1:] if "sb" in k and "tile[32][132]" in k]
    assert len(tiled) == 1, plan
    body = tiled[0]
    assert body.startswith(" void __launch_bounds__(256, 5)"), body[:80]
    # the k loop sits between the row loads and the per-row loop that uses the products
    rows = "const I rr = r0 + w + 8 * i;"
    assert body.index(rows) < body.index("for (int k = 0; k < 10; ++k)") < body.rindex(rows)
    assert plan.count("simt_skinny[") == 2, plan


def _region_variant_graphs():
    """Graphs whose regions use every generated-kernel variant of the GEMM-adjacent
    fusion: tiled regions writing one or both copy layouts (with and without the fp32
    store, odd sizes, broadcast operands) and small-K products in flat and tiled regions."""
    out = []
    for r, c, use in [(1024, 512, "A=Xt"), (646, 258, "B=X"), (646, 258, "A=X"), (100, 1030, "A=Xt")]:
        g = tt.Graph()
        a, b = g.input([r, c]), g.input([r, c])
        x = a * b
        k = c if use == "A=X" else r
        y = g.input([k, 64] if use.startswith("A") else [64, k])
        o = {"A=X": lambda: x @ y, "A=Xt": lambda: tt.transpose(x, 0, 1) @ y, "B=X": lambda: y @ x}[use]()
        out.append((g, [o]))
    for bshape in [(1, 520), (300, 1)]:
        g = tt.Graph()
        a, b, y = g.input([300, 520]), g.input(list(bshape)), g.input([300, 96])
        out.append((g, [tt.transpose(tt.relu(a + b) * 0.5, 0, 1) @ y]))
    g = tt.Graph()
    a, b, y1, y2 = g.input([768, 512]), g.input([768, 512]), g.input([512, 192]), g.input([768, 160])
    x = tt.relu(a - b)
    out.append((g, [x, x @ y1, tt.transpose(x, 0, 1) @ y2]))
    g = tt.Graph()
    a, b, c = g.input([300, 10]), g.input([10, 522]), g.input([300, 522])
    out.append((g, [(a @ b) * c]))  # flat region, scalar lanes (522 % 4 != 0)
    g = tt.Graph()
    t, w, yy, h, v = g.input([1024, 10]), g.input([512, 10]), g.input([1024, 512]), g.input([1024, 384]), g.input([512, 256])
    dz = (tt.relu(t) @ tt.transpose(w, 0, 1)) * (1.0 - yy * yy)
    out.append((g, [tt.transpose(h, 0, 1) @ dz, dz @ v]))
    return out


def test_gemm_adjacent_region_variants_compile(cache_dir):
    """NVRTC compiles every variant (host-only: plan + generate + compile to sm_100a)."""
    seen = set()
    for g, outs in _region_variant_graphs():
        p = _host_compile(g, outs, cache_dir)
        plan, src = p.execution_plan(), p.generated_source()
        assert "Binary Object:" in plan
        seen.update(k for k in ("tiled", "(writes hi/lo of X^T", "(writes hi/lo of X,", "hi/lo of X and X^T)",
                                "fused[matmul,") if k in src or k in plan)
    assert len(seen) == 5, seen
