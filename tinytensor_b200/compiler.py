"""tt.compile / CompiledProgram / tt.gradients with the reference's API
(python/tinytensor/compiler.py:24-137), running on the B200 backend.

A CompiledProgram owns one tt_program: the generated CUDA module, the launch
schedule and its device arena.  `run(feed)` has Executable::run semantics (host
arrays in, host tensors out, synchronous).  `run_device(...)` takes device buffers
and queues the work on a stream without synchronising (for chained programs, the
training step and the benchmarks).
"""

import contextlib
import ctypes
import os
from collections.abc import Mapping, Sequence

import numpy as np

from . import _lib
from ._lib import RuntimeExecutionError, ShapeError, TypeError
from .graph import Graph, Node

__all__ = ["compile", "compile_gradients", "CompiledProgram", "gradients", "Tensor", "tensor",
           "DeviceBuffer", "Stream", "Event", "CudaGraph", "launch_count"]


def _release(fn_name, handle):
    """Frees a native handle from a destructor.  At interpreter exit the module globals
    may already be gone (then the process teardown frees everything anyway)."""
    lib = getattr(_lib, "lib", None)
    if lib is None or not handle:
        return
    try:
        getattr(lib, fn_name)(handle)
    except Exception:
        pass


def _default_cache_dir():
    return os.environ.get("TT_CUDA_CACHE", os.path.join(os.path.expanduser("~"), ".cache", "tinytensor_b200"))


class Tensor:
    """Host result tensor (the reference returns tinytensor.Tensor with .numpy())."""

    __slots__ = ("_a",)

    def __init__(self, array):
        self._a = array

    def numpy(self):
        return self._a

    @property
    def shape(self):
        return list(self._a.shape)

    @property
    def dtype(self):
        return "float32"

    def item(self):
        if self._a.size != 1:
            raise ShapeError(f"item() requires a single element, got {self._a.size}")
        return float(self._a.reshape(-1)[0])

    def __array__(self, dtype=None, copy=None):
        return self._a if dtype is None else self._a.astype(dtype)

    def __repr__(self):
        return f"Tensor(shape={self.shape}, dtype=float32)"


def tensor(data, dtype=None) -> Tensor:
    return Tensor(np.array(data, dtype=np.float32, order="C"))


class Stream:
    """A CUDA stream owned by the backend (non-blocking)."""

    def __init__(self, handle=None):
        if handle is None:
            h = ctypes.c_void_p()
            _lib.check(_lib.lib.tt_stream_create(ctypes.byref(h)))
            self.handle = h.value
            self._own = True
        else:
            self.handle = int(handle)
            self._own = False

    def synchronize(self):
        _lib.check(_lib.lib.tt_stream_sync(self.handle))

    def __del__(self):
        if getattr(self, "_own", False) and self.handle:
            _release("tt_stream_destroy", self.handle)
            self.handle = None


class Event:
    """A CUDA event for ordering work across streams (no timing)."""

    def __init__(self):
        h = ctypes.c_void_p()
        _lib.check(_lib.lib.tt_event_create(ctypes.byref(h)))
        self.handle = h.value

    def record(self, stream) -> None:
        _lib.check(_lib.lib.tt_event_record(self.handle, getattr(stream, "handle", stream)))

    def wait(self, stream) -> None:
        """Makes `stream` wait (on the device) until this event has completed."""
        _lib.check(_lib.lib.tt_stream_wait_event(getattr(stream, "handle", stream), self.handle))

    def __del__(self):
        if getattr(self, "handle", None):
            _release("tt_event_destroy", self.handle)
            self.handle = None


class CudaGraph:
    """Work queued on a stream, captured once and replayed (cudaGraph).

        g = CudaGraph()
        with g.capture(stream):
            prog.run_device(ins, outs, stream)   # queued, not run
        g.replay(stream)                        # runs it; repeat as often as needed

    The captured work reads and writes the same buffers on every replay.  Run the
    work once outside capture first (kernel attributes and modules are set up then).
    """

    def __init__(self):
        self.handle = None

    @contextlib.contextmanager
    def capture(self, stream):
        h = getattr(stream, "handle", stream)
        _lib.check(_lib.lib.tt_stream_begin_capture(h))
        ok = False
        try:
            yield self
            ok = True
        finally:
            g = ctypes.c_void_p()
            rc = _lib.lib.tt_stream_end_capture(h, ctypes.byref(g))
            if ok:
                _lib.check(rc)
            if self.handle:
                _lib.lib.tt_graph_destroy(self.handle)
            self.handle = g.value

    def replay(self, stream) -> None:
        _lib.check(_lib.lib.tt_graph_launch(self.handle, getattr(stream, "handle", stream)))

    def __del__(self):
        if getattr(self, "handle", None):
            _release("tt_graph_destroy", self.handle)
            self.handle = None


class DeviceBuffer:
    """A float32 device allocation (cudaMalloc) with a shape."""

    def __init__(self, shape, pinned_host=False):
        self.shape = [int(d) for d in shape]
        self.nbytes = int(np.prod(self.shape, dtype=np.int64)) * 4
        p = ctypes.c_void_p()
        _lib.check(_lib.lib.tt_device_alloc(self.nbytes, ctypes.byref(p)))
        self.ptr = p.value

    @classmethod
    def from_numpy(cls, arr, stream=None):
        arr = np.ascontiguousarray(arr, dtype=np.float32)
        b = cls(arr.shape)
        b.copy_from(arr, stream)
        return b

    def copy_from(self, arr, stream=None):
        arr = np.ascontiguousarray(arr, dtype=np.float32)
        if arr.nbytes != self.nbytes:
            raise ShapeError(f"copy of {arr.nbytes} bytes into a {self.nbytes}-byte buffer")
        h = stream.handle if stream is not None else None
        _lib.check(_lib.lib.tt_memcpy(self.ptr, arr.ctypes.data, self.nbytes, _lib.H2D, h))
        _lib.check(_lib.lib.tt_stream_sync(h))

    def numpy(self, stream=None):
        out = np.empty(self.shape, dtype=np.float32)
        h = stream.handle if stream is not None else None
        _lib.check(_lib.lib.tt_memcpy(out.ctypes.data, self.ptr, self.nbytes, _lib.D2H, h))
        _lib.check(_lib.lib.tt_stream_sync(h))
        return out

    def free(self):
        if self.ptr:
            _lib.lib.tt_device_free(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class PinnedBuffer:
    """Page-locked host float32 array (cudaMallocHost), usable as a numpy array."""

    def __init__(self, shape):
        self.shape = [int(d) for d in shape]
        n = int(np.prod(self.shape, dtype=np.int64))
        p = ctypes.c_void_p()
        _lib.check(_lib.lib.tt_host_alloc(max(4, n * 4), ctypes.byref(p)))
        self.ptr = p.value
        self.array = np.ctypeslib.as_array(ctypes.cast(p, ctypes.POINTER(ctypes.c_float)), shape=(max(1, n),))[:n]
        self.array = self.array.reshape(self.shape)

    def __del__(self):
        if getattr(self, "ptr", None):
            _release("tt_host_free", self.ptr)
            self.ptr = None


def launch_count() -> int:
    """Kernels launched by this library so far (all programs and helpers)."""
    return int(_lib.lib.tt_launch_count())


class CompiledProgram:
    """Executable compiled TinyTensor program on the B200 backend."""

    def __init__(self, graph: Graph, outputs, handle, grad_nodes=()):
        self._graph = graph
        self._outputs = list(outputs)
        self._grad_nodes = list(grad_nodes)
        self._h = handle
        self._inputs = graph.inputs
        self._dev_args = None  # (input pointers, output pointers, their ctypes arrays) of the last run_device
        ni, no = ctypes.c_int32(), ctypes.c_int32()
        _lib.check(_lib.lib.tt_program_num_io(self._h, ctypes.byref(ni), ctypes.byref(no)))
        self.num_inputs, self.num_outputs = ni.value, no.value
        self.output_shapes = []
        for i in range(no.value):
            r = ctypes.c_int32()
            s = (ctypes.c_int64 * _lib.TT_MAX_RANK)()
            _lib.check(_lib.lib.tt_program_output_shape(self._h, i, ctypes.byref(r), s))
            self.output_shapes.append([int(s[k]) for k in range(r.value)])

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            _release("tt_program_destroy", h)
            self._h = None

    # -- diagnostics (Executor::original_ir etc.) -----------------------------------------
    def original_ir(self) -> str:
        return _lib.cstr(_lib.lib.tt_program_info, self._h, _lib.INFO_ORIGINAL_IR)

    def optimized_ir(self) -> str:
        return _lib.cstr(_lib.lib.tt_program_info, self._h, _lib.INFO_OPTIMIZED_IR)

    def generated_source(self) -> str:
        return _lib.cstr(_lib.lib.tt_program_info, self._h, _lib.INFO_SOURCE)

    def execution_plan(self) -> str:
        return _lib.cstr(_lib.lib.tt_program_info, self._h, _lib.INFO_PLAN)

    def cubin_path(self) -> str:
        return _lib.cstr(_lib.lib.tt_program_info, self._h, _lib.INFO_CUBIN_PATH)

    @property
    def ir(self) -> str:
        return self._graph.to_ir()

    # -- execution -----------------------------------------------------------------------------
    def _host_inputs(self, inputs: Mapping):
        arrays = []
        for n in self._inputs:
            if n not in inputs:
                raise RuntimeExecutionError(f"Missing input binding for node %{n.id}")
            v = inputs[n]
            if isinstance(v, Tensor):
                v = v.numpy()
            # converted to the node dtype like tensor(v, dtype=expected_dtype) (compiler.py:31-45);
            # the device computes in float32
            a = np.array(v, dtype=np.float32, order="C", copy=None)  # 0-d stays 0-d
            if list(a.shape) != n.shape:
                raise ShapeError(f"Input %{n.id} shape mismatch: expected {n.shape} but got {list(a.shape)}")
            arrays.append(a)
        return arrays

    def run(self, inputs: Mapping, profiler=None):
        """Runs on host arrays; returns one Tensor, or a list for several outputs."""
        arrays = self._host_inputs(inputs)
        outs = [np.empty(s, dtype=np.float32) for s in self.output_shapes]
        ip = (ctypes.c_void_p * max(1, len(arrays)))(*[a.ctypes.data for a in arrays])
        op = (ctypes.c_void_p * max(1, len(outs)))(*[o.ctypes.data for o in outs])
        _lib.check(_lib.lib.tt_program_run(self._h, ip, op, _lib.HOST, None))
        res = [Tensor(o) for o in outs]
        return res[0] if len(res) == 1 else res

    def run_device(self, inputs: Sequence, outputs: Sequence, stream=None):
        """Queues one run on `stream` with device buffers (DeviceBuffer or raw pointers)."""
        if len(inputs) != self.num_inputs:
            raise RuntimeExecutionError(f"Expected {self.num_inputs} inputs, but got {len(inputs)}")
        if len(outputs) != self.num_outputs:
            raise RuntimeExecutionError(f"Expected {self.num_outputs} outputs, but got {len(outputs)}")
        # the pointer arrays of the last call are reused when the buffers repeat (a loop over
        # the same buffers pays for building them once: ~2 us of a launch-bound call); the
        # pointer lists are list comprehensions, ~0.5 us cheaper per call than tuples of
        # generators
        ki = [getattr(x, "ptr", x) for x in inputs]
        ko = [getattr(x, "ptr", x) for x in outputs]
        cached = self._dev_args
        if cached is None or cached[0] != ki or cached[1] != ko:
            ip = (ctypes.c_void_p * max(1, len(ki)))(*ki)
            op = (ctypes.c_void_p * max(1, len(ko)))(*ko)
            cached = self._dev_args = (ki, ko, ip, op)
        h = stream.handle if isinstance(stream, Stream) else stream
        _lib.check(_lib.lib.tt_program_run(self._h, cached[2], cached[3], _lib.DEVICE, h))

    def status(self) -> int:
        """Synchronises and returns the device status word (raises if a kernel gave up)."""
        s = ctypes.c_int32()
        _lib.check(_lib.lib.tt_program_status(self._h, ctypes.byref(s)))
        return s.value

    def set_output_events(self, events) -> None:
        """events[k] (an Event or None) is recorded on the run's stream as soon as output k
        is complete, while the rest of the program may still be running."""
        self._out_events = list(events)
        n = len(self._out_events)
        arr = (ctypes.c_void_p * max(1, n))(*[e.handle if e is not None else None for e in self._out_events])
        _lib.check(_lib.lib.tt_program_set_output_events(self._h, arr, n))

    def set_input_events(self, events) -> None:
        """events[k] (an Event or None) is recorded on the run's stream as soon as the
        last launch reading input k is done: the input's buffer may then be overwritten
        (e.g. a parameter update) while the rest of the program still runs."""
        self._in_events = list(events)
        n = len(self._in_events)
        arr = (ctypes.c_void_p * max(1, n))(*[e.handle if e is not None else None for e in self._in_events])
        _lib.check(_lib.lib.tt_program_set_input_events(self._h, arr, n))

    def input_steps(self):
        """Per input, the launch after which it is no longer read (-1: never read)."""
        out = []
        for k in range(self.num_inputs):
            s = ctypes.c_int32()
            _lib.check(_lib.lib.tt_program_input_step(self._h, k, ctypes.byref(s)))
            out.append(s.value)
        return out

    def output_steps(self):
        """Per output, the launch after which it is complete (the order its event fires)."""
        out = []
        for k in range(self.num_outputs):
            s = ctypes.c_int32()
            _lib.check(_lib.lib.tt_program_output_step(self._h, k, ctypes.byref(s)))
            out.append(s.value)
        return out

    def set_profiling(self, enable: bool = True) -> None:
        _lib.check(_lib.lib.tt_program_set_profiling(self._h, int(enable)))

    def profile(self):
        """[(launch label, ms)] of the last profiled run."""
        cap, ncap = 4096, 160
        names = ctypes.create_string_buffer(cap * ncap)
        ms = (ctypes.c_float * cap)()
        cnt = ctypes.c_int32()
        _lib.check(_lib.lib.tt_program_profile(self._h, cap, names, ncap, ms, ctypes.byref(cnt)))
        out = []
        for i in range(min(cnt.value, cap)):
            raw = names.raw[i * ncap:(i + 1) * ncap]
            out.append((raw.split(b"\0", 1)[0].decode(), float(ms[i])))
        return out


def _compile(graph, outputs, optimize, cache_dir, grad_loss=None, wrt=(), device=0, flags=0):
    if outputs is not None:
        for o in outputs:
            graph.mark_output(o)
    outs = graph.outputs
    g, keep = graph._to_c(outs)
    opt = _lib.TTCompileOptions()
    opt.optimize = int(bool(optimize))
    opt.device = int(device)
    cdir = _default_cache_dir() if cache_dir is None else cache_dir
    cdir_b = cdir.encode() if cdir else None
    opt.cache_dir = cdir_b
    opt.grad_loss = -1 if grad_loss is None else grad_loss.index
    wrt_arr = (ctypes.c_int32 * max(1, len(wrt)))(*[n.index for n in wrt])
    opt.num_grad_wrt = len(wrt)
    opt.grad_wrt = wrt_arr
    opt.flags = int(flags)
    h = ctypes.c_void_p()
    _lib.check(_lib.lib.tt_compile(ctypes.byref(g), ctypes.byref(opt), ctypes.byref(h)))
    return CompiledProgram(graph, outs, h.value, wrt)


def compile(graph: Graph, outputs: Sequence[Node] | None = None, mode: str = "cuda", optimize: bool = True,
            cache_dir: str | None = None, device: int = 0, flags: int = 0) -> CompiledProgram:
    """tt.compile: marks `outputs` and compiles the graph for the B200 backend.

    mode accepts "cuda" (also "gpu", "compiled_cuda").  The reference's CPU modes
    ("avx2", "scalar", "interpreted") are not provided by this backend.
    """
    m = mode.lower()
    if m not in ("cuda", "gpu", "compiled_cuda", "b200"):
        raise ValueError(f"Unknown compilation mode: {mode}. This backend provides 'cuda'.")
    return _compile(graph, outputs, optimize, cache_dir, device=device, flags=flags)


def compile_gradients(graph: Graph, loss: Node, wrt: Sequence[Node], outputs: Sequence[Node] | None = None,
                      optimize: bool = True, cache_dir: str | None = None, device: int = 0,
                      flags: int = 0) -> CompiledProgram:
    """Compiles forward + symbolic backward: program outputs are `outputs` (default
    [loss]) followed by d loss / d w for every w in `wrt`, in order."""
    outs = [loss] if outputs is None else list(outputs)
    g2 = graph  # outputs are marked on the graph, as tt.compile does
    for o in outs:
        g2.mark_output(o)
    return _compile(g2, None, optimize, cache_dir, grad_loss=loss, wrt=list(wrt), device=device, flags=flags)


def gradients(graph: Graph, loss: Node, inputs: Mapping, mode: str = "cuda", cache_dir: str | None = None):
    """tt.gradients: d loss / d node for every node in `inputs`, as {node: Tensor}.

    The reference evaluates this eagerly on the host (src/autodiff/gradient.cpp); here
    the backward pass is emitted as graph nodes and run as one compiled GPU program."""
    wrt = [n for n in inputs.keys() if isinstance(n, Node)]
    key = (loss.index, tuple(n.index for n in wrt), graph._version)
    cache = graph.__dict__.setdefault("_grad_programs", {}) if hasattr(graph, "__dict__") else {}
    prog = cache.get(key)
    if prog is None:
        saved = list(graph._outputs)
        graph._outputs = []
        try:
            prog = _compile(graph, [loss], True, cache_dir, grad_loss=loss, wrt=wrt)
        finally:
            graph._outputs = saved
        cache[(loss.index, tuple(n.index for n in wrt), graph._version)] = prog
    res = prog.run(inputs)
    res = res if isinstance(res, list) else [res]
    return {n: res[1 + i] for i, n in enumerate(wrt)}
