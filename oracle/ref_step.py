"""ORACLE — test infrastructure only (the CPU-baseline leg and the `--impl reference`
arm of bench.py run it; the tinytensor_b200 package never imports it, and this module
imports nothing of tinytensor_b200).

The reference's own training step of the benchmark MLP, 1024 -> 4096 (ReLU) -> 4096
(tanh) -> 10 with MSE loss, on the host cores, as its example trains a network
(examples/neural_network_example.py:86-117):

    prog.run(feed)                 compiled forward, mode "avx2", optimize=True
                                   (Executor + CppBackend, src/runtime/executor.cpp)
    tt.gradients(g, loss, feed)    eager Autodiff::compute_gradients
                                   (src/autodiff/gradient.cpp:52-332)
    SGD.step(grads)                numpy float32 p -= lr * g (python/tinytensor/optim.py)

The reference is single-threaded; to use every host core the global batch is split by
rows over P worker processes, each running the step above on its shard through
oracle/_ref/libttref.so (the reference compiled from its sources).  Shard gradients
land in shared memory, the parent sums them and applies the update with lr / P (the
mean of equal shards' mean losses is the global mean), so one call of `step()` is one
data-parallel SGD step of the whole batch.  tanh, which the reference has no op for,
is its identity 2*sigmoid(2x) - 1 over reference ops (oracle/ref_harness.cpp).

The graph is built directly through the harness's C functions (ttref_*), not through
tinytensor_b200, so a process running this loads only the oracle's libraries.
"""

import ctypes
import multiprocessing as mp
import os
import time
from multiprocessing import shared_memory

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_SO = os.path.join(HERE, "_ref", "libttref.so")

# op codes of oracle/ref_harness.cpp (reference OpType order)
_MATMUL, _RELU, _SUB, _MUL, _TANH, _REDUCE_MEAN = 8, 6, 3, 4, 16, 11
_MODE_AVX2 = 2
LAYERS = (1024, 4096, 4096, 10)


def available():
    return os.path.exists(REF_SO)


def _lib():
    lib = ctypes.CDLL(REF_SO)
    vp, i32, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
    I64P = ctypes.POINTER(i64)
    lib.ttref_last_error.restype = ctypes.c_char_p
    lib.ttref_graph_new.restype = vp
    lib.ttref_graph_free.argtypes = [vp]
    lib.ttref_input.argtypes = [vp, I64P, i32, ctypes.c_char_p]
    lib.ttref_op.argtypes = [vp, i32, i32, i32]
    lib.ttref_reduce.argtypes = [vp, i32, i32, I64P, i32, i32]
    lib.ttref_mark_output.argtypes = [vp, i32]
    lib.ttref_compile.argtypes = [vp, i32, i32]
    lib.ttref_compile.restype = vp
    lib.ttref_exec_free.argtypes = [vp]
    lib.ttref_run.argtypes = [vp, ctypes.POINTER(vp), ctypes.POINTER(vp)]
    lib.ttref_gradients.argtypes = [vp, i32, ctypes.POINTER(vp), ctypes.POINTER(i32), i32, ctypes.POINTER(vp)]
    return lib


def _chk(lib, v):
    if v is None or (isinstance(v, int) and v < 0):
        raise RuntimeError(lib.ttref_last_error().decode())
    return v


class _Shard:
    """One worker's reference graph, compiled forward program and buffer pointers."""

    def __init__(self, rows):
        L = self.L = _lib()
        h = self.h = L.ttref_graph_new()

        def inp(shape, name):
            s = (ctypes.c_int64 * len(shape))(*shape)
            return _chk(L, L.ttref_input(h, s, len(shape), name.encode()))

        X, T = inp([rows, 1024], "X"), inp([rows, 10], "T")
        W1, W2, W3 = inp([1024, 4096], "W1"), inp([4096, 4096], "W2"), inp([4096, 10], "W3")
        op = lambda code, a, b=-1: _chk(L, L.ttref_op(h, code, a, b))  # noqa: E731
        h1 = op(_RELU, op(_MATMUL, X, W1))
        h2 = op(_TANH, op(_MATMUL, h1, W2))
        d = op(_SUB, op(_MATMUL, h2, W3), T)
        sq = op(_MUL, d, d)
        axes = (ctypes.c_int64 * 1)(0)
        self.loss = _chk(L, L.ttref_reduce(h, _REDUCE_MEAN, sq, axes, 0, 0))
        _chk(L, L.ttref_mark_output(h, self.loss))
        self.wrt = (ctypes.c_int * 3)(W1, W2, W3)
        self.ex = L.ttref_compile(h, _MODE_AVX2, 1)  # tt.compile(..., mode="avx2", optimize=True)
        if not self.ex:
            raise RuntimeError(L.ttref_last_error().decode())

    def run(self, x, t, w, grads, loss_out):
        """Compiled forward (the loss) then eager gradients of W1..W3 into `grads`."""
        L = self.L
        ins = (ctypes.c_void_p * 5)(*[a.ctypes.data for a in (x, t, w[0], w[1], w[2])])
        outs = (ctypes.c_void_p * 1)(loss_out.ctypes.data)
        _chk(L, L.ttref_run(self.ex, ins, outs))
        gp = (ctypes.c_void_p * 3)(*[gg.ctypes.data for gg in grads])
        _chk(L, L.ttref_gradients(self.h, self.loss, ins, self.wrt, 3, gp))


# ---- worker processes ------------------------------------------------------------------

_W = {}


def _views(shm, shapes, offset=0):
    out, off = [], offset
    for s in shapes:
        n = int(np.prod(s))
        out.append(np.ndarray(s, dtype=np.float32, buffer=shm.buf, offset=off * 4))
        off += n
    return out, off


def _weight_shapes():
    return [(LAYERS[i], LAYERS[i + 1]) for i in range(3)]


def _init(names, rows_total, P, barrier):
    """Worker set-up (not timed): attach the shared memory the parent owns.  Spawned
    workers share the parent's resource tracker, so attaching registers nothing new
    and the parent's unlink is the only clean-up."""
    _W["shm"] = [shared_memory.SharedMemory(name=n) for n in names]
    data, w, grads = _W["shm"]
    (X, T), _ = _views(data, [(rows_total, 1024), (rows_total, 10)])
    _W["w"], _ = _views(w, _weight_shapes())
    _W["grads"] = grads
    _W["X"], _W["T"] = X, T
    _W["rows"] = rows_total // P
    _W["shard"] = None
    _W["P"] = P
    _W["barrier"] = barrier


def _work(rank):
    """One shard's forward + gradients; returns (rank, seconds, shard loss)."""
    rows = _W["rows"]
    if _W["shard"] is None:
        _W["shard"] = _Shard(rows)
    x = np.ascontiguousarray(_W["X"][rank * rows:(rank + 1) * rows])
    t = np.ascontiguousarray(_W["T"][rank * rows:(rank + 1) * rows])
    per = sum(int(np.prod(s)) for s in _weight_shapes())
    g, _ = _views(_W["grads"], _weight_shapes(), offset=rank * per)
    loss = np.zeros(1, np.float32)
    t0 = time.perf_counter()
    _W["shard"].run(x, t, _W["w"], g, loss)
    return rank, time.perf_counter() - t0, float(loss[0])


def _prepare(_rank):
    """Builds and compiles the shard graph (g++ JIT of the forward) outside the timing.
    The barrier holds each task until all P have started, so every worker process
    takes exactly one and is prepared."""
    if _W["shard"] is None:
        _W["shard"] = _Shard(_W["rows"])
    _W["barrier"].wait(timeout=600)
    return os.getpid()


class ReferenceStep:
    """The reference's data-parallel SGD step over P host processes (see module doc).

    x [rows, 1024], t [rows, 10], weights [W1, W2, W3] float32; rows % P == 0."""

    def __init__(self, x, t, weights, lr=0.01, processes=None):
        if not available():
            raise FileNotFoundError(f"{REF_SO} missing: build it with `make -C oracle ref` where the reference sources are")
        rows = x.shape[0]
        P = processes or max(1, min(os.cpu_count() or 1, 64))
        while rows % P:
            P -= 1
        self.P, self.rows, self.lr = P, rows, lr
        per = sum(int(np.prod(s)) for s in _weight_shapes())
        self._shm = [shared_memory.SharedMemory(create=True, size=4 * rows * (1024 + 10)),
                     shared_memory.SharedMemory(create=True, size=4 * per),
                     shared_memory.SharedMemory(create=True, size=4 * per * P)]
        (X, T), _ = _views(self._shm[0], [(rows, 1024), (rows, 10)])
        X[...] = x
        T[...] = t
        self.w, _ = _views(self._shm[1], _weight_shapes())
        for dst, src in zip(self.w, weights):
            dst[...] = src
        self._g = np.ndarray((P, per), dtype=np.float32, buffer=self._shm[2].buf)
        ctx = mp.get_context("spawn")
        barrier = ctx.Barrier(P)
        self.pool = ctx.Pool(P, initializer=_init, initargs=([s.name for s in self._shm], rows, P, barrier))
        pids = self.pool.map(_prepare, range(P), chunksize=1)
        assert len(set(pids)) == P, "every worker process prepares its graph once"
        self.last = {}

    def step(self):
        """One global step; returns its wall-clock seconds (shard work in parallel, then
        the gradient sum and the update in this process)."""
        t0 = time.perf_counter()
        res = self.pool.map(_work, range(self.P), chunksize=1)
        t1 = time.perf_counter()
        gsum = self._g.sum(axis=0, dtype=np.float32)
        off = 0
        scale = np.float32(self.lr / self.P)
        for w in self.w:
            n = w.size
            w -= scale * gsum[off:off + n].reshape(w.shape)
            off += n
        t2 = time.perf_counter()
        self._gsum = gsum
        self.last = {"shard_s_max": max(r[1] for r in res), "shard_s_median": float(np.median([r[1] for r in res])),
                     "parallel_s": t1 - t0, "reduce_update_s": t2 - t1,
                     "loss": float(np.mean([r[2] for r in res]))}
        return t2 - t0

    def gradient_sums(self):
        """The last step's sums over shards of the shard-mean-loss gradients (W1..W3)."""
        out, off = [], 0
        for s in _weight_shapes():
            n = int(np.prod(s))
            out.append(self._gsum[off:off + n].reshape(s))
            off += n
        return out

    def mean_gradients(self):
        """The last step's gradients of the whole-batch mean loss (shard sum / P)."""
        return [g / np.float32(self.P) for g in self.gradient_sums()]

    def weights(self):
        return [w.copy() for w in self.w]

    def close(self):
        if self.pool is not None:
            self.pool.close()
            self.pool.join()
            self.pool = None
        for s in self._shm:
            try:
                s.close()
                s.unlink()
            except FileNotFoundError:
                pass
        self._shm = []

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
