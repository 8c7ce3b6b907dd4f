"""Output-ready events on the GPU: a second stream that waits on a gradient's event
and copies it sees the finished gradient while the program may still be running
the launches after it (the data-parallel exchange relies on this)."""

import numpy as np
import pytest

from parity import GEMM_FROB_RTOL, assert_norm

import tinytensor_b200 as tt
from tinytensor_b200 import _lib
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_output_events_order_gradient_copies(cache_dir):
    rows, dims = 512, (256, 512, 512, 10)
    rng = np.random.default_rng(8)
    g = tt.Graph()
    X, T = g.input([rows, dims[0]]), g.input([rows, dims[3]])
    W = [g.input([a, b]) for a, b in zip(dims[:-1], dims[1:])]
    d = tt.tanh(tt.relu(X @ W[0]) @ W[1]) @ W[2] - T
    loss = tt.mean(d * d)
    prog = tt.compile_gradients(g, loss, W, cache_dir=cache_dir)
    x = rng.standard_normal((rows, dims[0])).astype(np.float32)
    t = rng.standard_normal((rows, dims[3])).astype(np.float32)
    ws = [(rng.standard_normal((a, b)) / np.sqrt(a)).astype(np.float32) for a, b in zip(dims[:-1], dims[1:])]
    ins = [tt.DeviceBuffer.from_numpy(a) for a in [x, t] + ws]
    outs = [tt.DeviceBuffer([])] + [tt.DeviceBuffer(w.shape) for w in ws]
    copies = [tt.DeviceBuffer(w.shape) for w in ws]
    events = [tt.Event() for _ in ws]
    prog.set_output_events([None] + events)
    steps = prog.output_steps()
    assert steps[3] < steps[2] < steps[1]          # dW3, then dW2, then dW1
    main, side = tt.Stream(), tt.Stream()
    for _ in range(2):
        prog.run_device(ins, outs, main)
        for k in (2, 1, 0):                          # production order
            events[k].wait(side)
            _lib.check(_lib.lib.tt_memcpy(copies[k].ptr, outs[k + 1].ptr, copies[k].nbytes, _lib.D2D, side.handle))
        side.synchronize()
        main.synchronize()
    assert prog.status() == 0
    ref = O.gradients(g, loss, {X: x, T: t, W[0]: ws[0], W[1]: ws[1], W[2]: ws[2]}, W)
    for k in range(3):
        got = outs[k + 1].numpy()
        assert np.array_equal(copies[k].numpy(), got)
        assert_norm(got, ref[k], GEMM_FROB_RTOL)
    prog.set_output_events([])


def test_step_host_matches_device_steps(cache_dir):
    """DataParallelSGD.step_host (overlapped H2D into alternating slots) gives the same
    weights, bit for bit, as step() on device-resident batches, batch by batch."""
    rows, dims = 256, (128, 256, 256, 10)
    rng = np.random.default_rng(13)
    g = tt.Graph()
    X, T = g.input([rows, dims[0]]), g.input([rows, dims[3]])
    W = [g.input([a, b]) for a, b in zip(dims[:-1], dims[1:])]
    d = tt.tanh(tt.relu(X @ W[0]) @ W[1]) @ W[2] - T
    loss = tt.mean(d * d)
    ws = [(rng.standard_normal((a, b)) / np.sqrt(a)).astype(np.float32) for a, b in zip(dims[:-1], dims[1:])]
    batches = [(rng.standard_normal((rows, dims[0])).astype(np.float32),
                rng.standard_normal((rows, dims[3])).astype(np.float32)) for _ in range(4)]
    results = []
    for host in (False, True):
        prog = tt.compile_gradients(g, loss, W, cache_dir=cache_dir)
        params = [tt.DeviceBuffer.from_numpy(w) for w in ws]
        trainer = tt.DataParallelSGD(prog, params, lr=0.05)
        stream = tt.Stream()
        hosts = [[tt.PinnedBuffer([rows, dims[0]]), tt.PinnedBuffer([rows, dims[3]])] for _ in range(2)]
        for i, (x, t) in enumerate(batches):
            if host:
                hosts[i % 2][0].array[...] = x
                hosts[i % 2][1].array[...] = t
                trainer.step_host(hosts[i % 2], stream)
                if i % 2 == 1:
                    stream.synchronize()   # both host buffers are reused by the next two steps
            else:
                dev = [tt.DeviceBuffer.from_numpy(x), tt.DeviceBuffer.from_numpy(t)]
                trainer.step(dev, stream)
                stream.synchronize()
                del dev
        stream.synchronize()
        assert prog.status() == 0
        results.append([p.numpy() for p in params])
    for a, b in zip(*results):
        assert np.array_equal(a, b)


def test_concurrent_gemm_pairs_match_serial_program(cache_dir):
    """The same gradient program with its independent GEMM pairs on two streams and with
    TT_FLAG_SERIAL gives bit-identical outputs (same kernels, same data)."""
    rows, dims = 1024, (256, 512, 512, 10)
    rng = np.random.default_rng(17)
    g = tt.Graph()
    X, T = g.input([rows, dims[0]]), g.input([rows, dims[3]])
    W = [g.input([a, b]) for a, b in zip(dims[:-1], dims[1:])]
    d = tt.tanh(tt.relu(X @ W[0]) @ W[1]) @ W[2] - T
    loss = tt.mean(d * d)
    feeds = [rng.standard_normal((rows, dims[0])).astype(np.float32),
             rng.standard_normal((rows, dims[3])).astype(np.float32)]
    feeds += [(rng.standard_normal((a, b)) / np.sqrt(a)).astype(np.float32) for a, b in zip(dims[:-1], dims[1:])]
    results = []
    for flags in (0, tt.FLAG_SERIAL):
        prog = tt.compile_gradients(g, loss, W, cache_dir=cache_dir, flags=flags)
        assert ("runs beside" in prog.execution_plan()) == (flags == 0)
        ins = [tt.DeviceBuffer.from_numpy(a) for a in feeds]
        outs = [tt.DeviceBuffer([])] + [tt.DeviceBuffer(w.shape) for w in feeds[2:]]
        stream = tt.Stream()
        for _ in range(3):
            prog.run_device(ins, outs, stream)
        stream.synchronize()
        assert prog.status() == 0
        results.append([o.numpy() for o in outs])
    for a, b in zip(*results):
        assert np.array_equal(a, b)
