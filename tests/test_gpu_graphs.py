"""CUDA-graph capture and replay of queued work: replays give the same results as the
same work run eagerly (bit for bit), for a fused elementwise program called many times
and for whole SGD steps."""

import numpy as np
import pytest

import tinytensor_b200 as tt

pytestmark = pytest.mark.gpu


def test_replayed_program_matches_eager(cache_dir):
    rng = np.random.default_rng(0)
    g = tt.Graph()
    a, b, c = g.input([1024, 1024]), g.input([1024, 1024]), g.input([1, 1024])
    y = tt.relu(a * b + c) * 0.5 - tt.exp(-a)
    prog = tt.compile(g, outputs=[y], cache_dir=cache_dir)
    feeds = [rng.standard_normal(s).astype(np.float32) for s in ([1024, 1024], [1024, 1024], [1, 1024])]
    ins = [tt.DeviceBuffer.from_numpy(f) for f in feeds]
    eager, replayed = tt.DeviceBuffer([1024, 1024]), tt.DeviceBuffer([1024, 1024])
    stream = tt.Stream()
    prog.run_device(ins, [eager], stream)
    stream.synchronize()
    graph = tt.CudaGraph()
    n0 = tt.launch_count()
    with graph.capture(stream):
        for _ in range(8):
            prog.run_device(ins, [replayed], stream)
    assert tt.launch_count() - n0 == 8          # counted when queued into the graph
    for _ in range(3):
        graph.replay(stream)
    stream.synchronize()
    assert np.array_equal(eager.numpy(), replayed.numpy())


def test_replayed_sgd_steps_match_eager_steps(cache_dir):
    rows, dims = 256, (128, 256, 256, 10)
    rng = np.random.default_rng(5)
    g = tt.Graph()
    X, T = g.input([rows, dims[0]]), g.input([rows, dims[3]])
    W = [g.input([i, o]) for i, o in zip(dims[:-1], dims[1:])]
    d = tt.tanh(tt.relu(X @ W[0]) @ W[1]) @ W[2] - T
    loss = tt.mean(d * d)
    ws = [(rng.standard_normal((i, o)) / np.sqrt(i)).astype(np.float32) for i, o in zip(dims[:-1], dims[1:])]
    x = tt.DeviceBuffer.from_numpy(rng.standard_normal((rows, dims[0])).astype(np.float32))
    t = tt.DeviceBuffer.from_numpy(rng.standard_normal((rows, dims[3])).astype(np.float32))
    results = []
    for use_graph in (False, True):
        prog = tt.compile_gradients(g, loss, W, cache_dir=cache_dir)
        params = [tt.DeviceBuffer.from_numpy(w) for w in ws]
        trainer = tt.DataParallelSGD(prog, params, lr=0.05)
        stream = tt.Stream()
        trainer.step([x, t], stream)                # eager first step (sets up kernels)
        if use_graph:
            graph = tt.CudaGraph()
            with graph.capture(stream):
                trainer.step([x, t], stream)
            for _ in range(4):
                graph.replay(stream)
        else:
            for _ in range(4):
                trainer.step([x, t], stream)
        stream.synchronize()
        assert prog.status() == 0
        results.append([p.numpy() for p in params] + [trainer.loss.numpy()])
    for e, r in zip(*results):
        assert np.array_equal(e, r)
