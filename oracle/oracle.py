"""ORACLE — test infrastructure only (tests/, __graft_entry__.smoke and the CPU-baseline
leg of bench.py may use it; the tinytensor_b200 package never imports it).

Two checkers for tinytensor_b200 graphs:

* `evaluate` / `gradients`: a CPU restatement of the reference's eager execution —
  Interpreter::run (src/runtime/interpreter.cpp:17-150) and
  Autodiff::compute_gradients (src/autodiff/gradient.cpp:52-332) — over the C kernels
  of oracle/tt_oracle.c (restating src/core/operators.cpp).  Pinned against the
  reference itself by tests/test_oracle_golden.py.

* `Reference`: the reference library itself (oracle/_ref/libttref.so, compiled from the
  reference sources by oracle/Makefile), driven through oracle/ref_harness.cpp.  Used
  to generate golden vectors and as the CPU baseline.  Ops the reference lacks are
  expressed with reference-op identities (see ref_harness.cpp).
"""

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libtt_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libttref.so")

# op codes (same numbering as include/tt_cuda.h)
INPUT, CONSTANT, ADD, SUB, MUL, DIV, RELU, SIGMOID, MATMUL, TRANSPOSE = range(10)
REDUCE_SUM, REDUCE_MEAN = 10, 11
EXP, NEG, TANH, REDUCE_MAX, STEP, RESHAPE, EXPAND = range(14, 21)

_P = np.ctypeslib.ndpointer
_F32 = _P(dtype=np.float32, flags="C_CONTIGUOUS")
_I64 = _P(dtype=np.int64, flags="C_CONTIGUOUS")


def build():
    """Compiles the C restatement (cheap); oracle/_ref needs the reference sources."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)


def _load_oracle():
    if not os.path.exists(ORACLE_SO):
        build()
    lib = ctypes.CDLL(ORACLE_SO)
    i64, i32, vp = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
    lib.tto_binary.argtypes = [i32, _F32, _I64, i32, _F32, _I64, i32, _F32]
    lib.tto_binary.restype = i32
    lib.tto_unary.argtypes = [i32, _F32, i64, _F32]
    lib.tto_matmul.argtypes = [_F32, _F32, i64, i64, i64, _F32]
    lib.tto_matmul_rows.argtypes = [vp, i64, i64, vp, i64, i64, i64, i64, _I64, i64, _F32]
    lib.tto_transpose.argtypes = [_F32, _I64, i32, i32, i32, _F32]
    lib.tto_transpose.restype = i32
    lib.tto_reduce.argtypes = [i32, vp, _I64, _I64, i32, ctypes.c_uint, _F32]
    lib.tto_reduce.restype = i32
    lib.tto_sgd.argtypes = [_F32, _F32, vp, i64, ctypes.c_float, ctypes.c_float]
    lib.tto_broadcast_shapes.argtypes = [_I64, i32, _I64, i32, _I64, ctypes.POINTER(i32)]
    lib.tto_broadcast_shapes.restype = i32
    return lib


_o = _load_oracle()


def _f32(a):
    # not np.ascontiguousarray alone: it returns at least 1-d, and a rank-0 value must
    # stay rank 0 (shape ()), as the reference's scalar tensors do
    a = np.asarray(a, dtype=np.float32)
    return a if a.flags.c_contiguous else np.ascontiguousarray(a)


def _shape(a):
    return np.asarray(a.shape, dtype=np.int64) if a.ndim else np.zeros(1, dtype=np.int64)


def broadcast_shapes(sa, sb):
    out = np.zeros(8, dtype=np.int64)
    r = ctypes.c_int(0)
    a = np.asarray(sa, dtype=np.int64) if len(sa) else np.zeros(1, np.int64)
    b = np.asarray(sb, dtype=np.int64) if len(sb) else np.zeros(1, np.int64)
    if _o.tto_broadcast_shapes(a, len(sa), b, len(sb), out, ctypes.byref(r)) != 0:
        raise ValueError(f"shapes {sa} and {sb} do not broadcast")
    return tuple(int(x) for x in out[: r.value])


def binary(op, a, b):
    a, b = _f32(a), _f32(b)
    out = np.empty(broadcast_shapes(a.shape, b.shape), dtype=np.float32)
    rc = _o.tto_binary(op, a, _shape(a), a.ndim, b, _shape(b), b.ndim, out.reshape(-1) if out.size else np.zeros(1, np.float32))
    if rc:
        raise ValueError("tto_binary failed")
    return out


def unary(op, a):
    a = _f32(a)
    out = np.empty_like(a)
    if a.size:
        _o.tto_unary(op, a.reshape(-1), a.size, out.reshape(-1))
    return out


def matmul(a, b):
    """operators.cpp:235-392: 2-D blocked IKJ, batched with broadcast batch dims."""
    a, b = _f32(a), _f32(b)
    if a.ndim == 2 and b.ndim == 2:
        M, K = a.shape
        N = b.shape[1]
        out = np.empty((M, N), dtype=np.float32)
        if out.size:
            _o.tto_matmul(a if a.size else np.zeros(1, np.float32), b if b.size else np.zeros(1, np.float32),
                          M, K, N, out)
        return out
    batch = broadcast_shapes(a.shape[:-2], b.shape[:-2])
    ab = np.ascontiguousarray(np.broadcast_to(a, batch + a.shape[-2:]))
    bb = np.ascontiguousarray(np.broadcast_to(b, batch + b.shape[-2:]))
    out = np.empty(batch + (a.shape[-2], b.shape[-1]), dtype=np.float32)
    for idx in np.ndindex(*batch):
        out[idx] = matmul(ab[idx], bb[idx])
    return out


def matmul_rows(a, b, rows):
    """Rows `rows` of a@b exactly as the reference's blocked loop computes them.
    a and b may be transposed (non-contiguous) 2-D views."""
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    rows = np.ascontiguousarray(rows, dtype=np.int64)
    K, N = b.shape
    out = np.empty((len(rows), N), dtype=np.float32)
    sa0, sa1 = (s // 4 for s in a.strides)
    sb0, sb1 = (s // 4 for s in b.strides)
    _o.tto_matmul_rows(a.ctypes.data, sa0, sa1, b.ctypes.data, sb0, sb1, K, N, rows, len(rows), out)
    return out


def transpose(a, d0, d1):
    a = _f32(a)
    r = a.ndim
    s = list(a.shape)
    d0n, d1n = d0 % r, d1 % r
    s[d0n], s[d1n] = s[d1n], s[d0n]
    out = np.empty(s, dtype=np.float32)
    if a.size:
        _o.tto_transpose(a.reshape(-1), _shape(a), r, d0, d1, out.reshape(-1))
    return out


def reduce(op, a, axes=None, keepdims=False):
    """operators.cpp:394-516 semantics; `a` may be a strided (e.g. transposed) view."""
    a = np.asarray(a, dtype=np.float32)
    r = a.ndim
    norm = set(range(r)) if not axes else {x % r for x in axes}
    mask = 0
    for x in norm:
        mask |= 1 << x
    oshape = [a.shape[i] if i not in norm else 1 for i in range(r)]
    out = np.empty([d for d in oshape], dtype=np.float32)
    st = np.asarray([s // 4 for s in a.strides], dtype=np.int64) if r else np.zeros(1, np.int64)
    if a.size == 0:
        out[...] = -np.inf if op == REDUCE_MAX else 0.0
    else:
        base = a
        _o.tto_reduce(op, base.ctypes.data, _shape(a), st, r, mask, out.reshape(-1))
    if not keepdims:
        out = out.reshape([a.shape[i] for i in range(r) if i not in norm])
    return out


def sgd(p, g, lr, momentum=0.0, v=None):
    p = _f32(p).copy()
    g = _f32(g)
    vv = None if v is None else _f32(v).copy()
    _o.tto_sgd(p.reshape(-1), g.reshape(-1), None if vv is None else vv.ctypes.data, p.size, lr, momentum)
    return p, vv


# ---- graph evaluation over tinytensor_b200.Graph nodes ------------------------------------

def _normalize_axes(n, rank):
    return sorted(set(range(rank))) if not n.axes else sorted({a % rank for a in n.axes})


def _eval_node(n, vals):
    ins = [vals[q.index] for q in n.inputs]
    op = n.op
    if op in (ADD, SUB, MUL, DIV):
        return binary(op, ins[0], ins[1])
    if op in (RELU, SIGMOID, EXP, NEG, TANH, STEP):
        return unary(op, ins[0])
    if op == MATMUL:
        return matmul(ins[0], ins[1])
    if op == TRANSPOSE:
        return transpose(ins[0], n.dim0, n.dim1)
    if op in (REDUCE_SUM, REDUCE_MEAN, REDUCE_MAX):
        return reduce(op, ins[0], n.axes, n.keepdims)
    if op == RESHAPE:
        return _f32(ins[0]).reshape(n.shape)
    if op == EXPAND:
        return np.ascontiguousarray(np.broadcast_to(ins[0], n.shape))
    raise ValueError(f"oracle: unsupported op {op}")


def evaluate(graph, feed, outputs=None):
    """Interpreter::run restated: every node in order; returns the output arrays."""
    vals = {}
    for n in graph.nodes:
        if n.op == INPUT:
            vals[n.index] = _f32(feed[n]).reshape(n.shape)
        elif n.op == CONSTANT:
            vals[n.index] = _f32(n.data)
        else:
            vals[n.index] = _eval_node(n, vals)
    outs = graph.outputs if outputs is None else outputs
    return [vals[o.index] for o in outs]


def magnitude(graph, feed, outputs=None):
    """Per-element magnitude bound m(x) of each output, in float64: the expression
    evaluated with |.| on every operand and + for every + or -, so that the rounding
    error of any float32 evaluation order is O(u * m).  Used as the scale of the
    elementwise tolerance for expressions with transcendental functions, whose float
    libm results (glibc vs CUDA) may differ by an ulp before a cancelling subtraction."""
    vals, mags = {}, {}
    for n in graph.nodes:
        if n.op == INPUT:
            v = np.asarray(feed[n], dtype=np.float64).reshape(n.shape)
            vals[n.index], mags[n.index] = v, np.abs(v)
            continue
        if n.op == CONSTANT:
            v = np.asarray(n.data, dtype=np.float64)
            vals[n.index], mags[n.index] = v, np.abs(v)
            continue
        x = [vals[q.index] for q in n.inputs]
        m = [mags[q.index] for q in n.inputs]
        op = n.op
        with np.errstate(all="ignore"):
            if op in (ADD, SUB):
                v, mg = (x[0] + x[1]) if op == ADD else (x[0] - x[1]), m[0] + m[1]
            elif op == MUL:
                v, mg = x[0] * x[1], m[0] * m[1]
            elif op == DIV:
                v, mg = x[0] / x[1], m[0] / np.abs(x[1])
            elif op == RELU:
                v = np.where(x[0] > 0, x[0], 0.0)
                mg = np.where(x[0] > 0, m[0], 0.0)
            elif op == STEP:
                v = np.where(x[0] > 0, 1.0, 0.0)
                mg = v
            elif op == NEG:
                v, mg = -x[0], m[0]
            elif op == EXP:
                v = np.exp(x[0])
                mg = v * (1.0 + m[0])
            elif op == TANH:
                v = np.tanh(x[0])
                mg = np.abs(v) + m[0] * (1.0 - v * v)
            elif op == SIGMOID:
                v = 1.0 / (1.0 + np.exp(-x[0]))
                mg = v + m[0] * v * (1.0 - v)
            elif op == TRANSPOSE:
                v, mg = np.swapaxes(x[0], n.dim0, n.dim1), np.swapaxes(m[0], n.dim0, n.dim1)
            elif op == RESHAPE:
                v, mg = x[0].reshape(n.shape), m[0].reshape(n.shape)
            elif op == EXPAND:
                v, mg = np.broadcast_to(x[0], n.shape), np.broadcast_to(m[0], n.shape)
            elif op in (REDUCE_SUM, REDUCE_MEAN, REDUCE_MAX):
                rank = x[0].ndim
                ax = tuple(sorted(set(range(rank)) if not n.axes else {a % rank for a in n.axes}))
                f = {REDUCE_SUM: np.sum, REDUCE_MEAN: np.mean, REDUCE_MAX: np.max}[op]
                v, mg = f(x[0], axis=ax, keepdims=n.keepdims), f(m[0], axis=ax, keepdims=n.keepdims)
            elif op == MATMUL:
                v, mg = np.matmul(x[0], x[1]), np.matmul(m[0], m[1])
            else:
                raise ValueError(f"magnitude: unsupported op {op}")
        vals[n.index], mags[n.index] = v, mg
    outs = graph.outputs if outputs is None else outputs
    return [mags[o.index] for o in outs]


def unbroadcast(g, target):
    """Autodiff::unbroadcast (gradient.cpp:10-50)."""
    target = tuple(target)
    if tuple(g.shape) == target:
        return g
    if len(target) == 0:
        return reduce(REDUCE_SUM, g)
    cur = g
    if cur.ndim > len(target):
        cur = reduce(REDUCE_SUM, cur, list(range(cur.ndim - len(target))), False)
    single = [i for i in range(len(target)) if target[i] == 1 and cur.shape[i] > 1]
    if single:
        cur = reduce(REDUCE_SUM, cur, single, True)
    return cur.reshape(target)


def gradients(graph, loss, feed, wrt):
    """Autodiff::compute_gradients restated (gradient.cpp:52-332) with the VJPs of the
    added ops (exp, neg, tanh); returns [d loss / d w for w in wrt]."""
    vals = {}
    for n in graph.nodes:
        if n.op == INPUT:
            vals[n.index] = _f32(feed[n]).reshape(n.shape)
        elif n.op == CONSTANT:
            vals[n.index] = _f32(n.data)
        else:
            vals[n.index] = _eval_node(n, vals)
    grads = {loss.index: np.ones(loss.shape, dtype=np.float32)}

    def acc(node, c):
        c = _f32(c)
        grads[node.index] = c if node.index not in grads else binary(ADD, grads[node.index], c)

    for n in reversed(graph.nodes[: loss.index + 1]):
        if n.index not in grads:
            continue
        g = grads[n.index]
        op = n.op
        if op in (INPUT, CONSTANT, STEP):
            continue
        a = n.inputs[0]
        b = n.inputs[1] if len(n.inputs) > 1 else None
        if op == ADD:
            acc(a, unbroadcast(g, a.shape))
            acc(b, unbroadcast(g, b.shape))
        elif op == SUB:
            acc(a, unbroadcast(g, a.shape))
            acc(b, unbroadcast(binary(MUL, g, np.float32(-1.0)), b.shape))
        elif op == MUL:
            ga, gb = binary(MUL, g, vals[b.index]), binary(MUL, g, vals[a.index])
            acc(a, unbroadcast(ga, a.shape))
            acc(b, unbroadcast(gb, b.shape))
        elif op == DIV:
            acc(a, unbroadcast(binary(DIV, g, vals[b.index]), a.shape))
            bsq = binary(MUL, vals[b.index], vals[b.index])
            negg = binary(MUL, g, np.float32(-1.0))
            acc(b, unbroadcast(binary(DIV, binary(MUL, negg, vals[a.index]), bsq), b.shape))
        elif op == RELU:
            acc(a, binary(MUL, g, unary(STEP, vals[a.index])))
        elif op == SIGMOID:
            s = vals[n.index]
            acc(a, binary(MUL, g, binary(MUL, s, binary(SUB, np.ones_like(s), s))))
        elif op == EXP:
            acc(a, binary(MUL, g, vals[n.index]))
        elif op == NEG:
            acc(a, unary(NEG, g))
        elif op == TANH:
            t = vals[n.index]
            acc(a, binary(MUL, g, binary(SUB, np.ones_like(t), binary(MUL, t, t))))
        elif op == MATMUL:
            A, B = vals[a.index], vals[b.index]
            acc(a, unbroadcast(matmul(g, np.swapaxes(B, -1, -2)), a.shape))
            acc(b, unbroadcast(matmul(np.swapaxes(A, -1, -2), g), b.shape))
        elif op == TRANSPOSE:
            acc(a, transpose(g, n.dim0, n.dim1))
        elif op in (REDUCE_SUM, REDUCE_MEAN):
            ash = a.shape
            gg = g
            if op == REDUCE_MEAN:
                nred = max(1, int(np.prod(ash)) // max(1, g.size))
                gg = binary(MUL, g, np.float32(1.0 / nred))
            if not n.keepdims:
                ax = _normalize_axes(n, len(ash))
                gg = gg.reshape([1 if i in ax else ash[i] for i in range(len(ash))])
            acc(a, np.broadcast_to(gg, ash))
        elif op == RESHAPE:
            acc(a, g.reshape(a.shape))
        elif op == EXPAND:
            acc(a, unbroadcast(g, a.shape))
        else:
            raise ValueError(f"oracle: no gradient for op {op}")
    return [grads.get(w.index, np.zeros(w.shape, dtype=np.float32)) for w in wrt]


# ---- the reference itself ------------------------------------------------------------------

class Reference:
    """The reference TinyTensor library (oracle/_ref/libttref.so)."""

    # "cuda" exists only in the integration build (integration/_build/libttref_cuda.so)
    MODES = {"interpreted": 0, "scalar": 1, "avx2": 2, "avx2_fma": 3, "avx2_nofma": 4, "cuda": 5}

    def __init__(self, path=REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle ref` where the reference sources exist")
        lib = ctypes.CDLL(path)
        vp, i32, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
        lib.ttref_last_error.restype = ctypes.c_char_p
        lib.ttref_graph_new.restype = vp
        lib.ttref_graph_free.argtypes = [vp]
        lib.ttref_input.argtypes = [vp, _I64, i32, ctypes.c_char_p]
        lib.ttref_constant.argtypes = [vp, _F32, _I64, i32]
        lib.ttref_op.argtypes = [vp, i32, i32, i32]
        lib.ttref_transpose.argtypes = [vp, i32, i64, i64]
        lib.ttref_reduce.argtypes = [vp, i32, i32, _I64, i32, i32]
        lib.ttref_mark_output.argtypes = [vp, i32]
        lib.ttref_ir.argtypes = [vp, ctypes.c_char_p, ctypes.c_size_t]
        lib.ttref_ir.restype = ctypes.c_size_t
        lib.ttref_compile.argtypes = [vp, i32, i32]
        lib.ttref_compile.restype = vp
        lib.ttref_exec_free.argtypes = [vp]
        lib.ttref_run.argtypes = [vp, ctypes.POINTER(vp), ctypes.POINTER(vp)]
        lib.ttref_time_runs.argtypes = [vp, ctypes.POINTER(vp), i32]
        lib.ttref_time_runs.restype = ctypes.c_double
        lib.ttref_gradients.argtypes = [vp, i32, ctypes.POINTER(vp), ctypes.POINTER(i32), i32, ctypes.POINTER(vp)]
        lib.ttref_time_gradients.argtypes = [vp, i32, ctypes.POINTER(vp), i32]
        lib.ttref_time_gradients.restype = ctypes.c_double
        self.lib = lib

    def _chk(self, v):
        if (isinstance(v, int) and v < 0) or v is None:
            raise RuntimeError(self.lib.ttref_last_error().decode())
        return v

    def build(self, graph, outputs=None):
        """Re-creates a tinytensor_b200.Graph in the reference; returns (handle, node map)."""
        L = self.lib
        h = L.ttref_graph_new()
        m = {}
        for n in graph.nodes:
            if n.op == INPUT:
                m[n.index] = self._chk(L.ttref_input(h, np.asarray(n.shape or [0], np.int64), len(n.shape),
                                                     n.name.encode()))
            elif n.op == CONSTANT:
                m[n.index] = self._chk(L.ttref_constant(h, _f32(n.data).reshape(-1) if n.data.size else
                                                        np.zeros(1, np.float32),
                                                        np.asarray(n.shape or [0], np.int64), len(n.shape)))
            elif n.op == TRANSPOSE:
                m[n.index] = self._chk(L.ttref_transpose(h, m[n.inputs[0].index], n.dim0, n.dim1))
            elif n.op in (REDUCE_SUM, REDUCE_MEAN, REDUCE_MAX):
                ax = np.asarray(n.axes or [0], np.int64)
                m[n.index] = self._chk(L.ttref_reduce(h, n.op, m[n.inputs[0].index], ax, len(n.axes),
                                                      int(n.keepdims)))
            else:
                a = m[n.inputs[0].index]
                b = m[n.inputs[1].index] if len(n.inputs) > 1 else -1
                m[n.index] = self._chk(L.ttref_op(h, n.op, a, b))
        for o in (graph.outputs if outputs is None else outputs):
            self._chk(L.ttref_mark_output(h, m[o.index]))
        return h, m

    def ir(self, graph):
        h, _ = self.build(graph)
        try:
            n = self.lib.ttref_ir(h, None, 0)
            buf = ctypes.create_string_buffer(n)
            self.lib.ttref_ir(h, buf, n)
            return buf.value.decode()
        finally:
            self.lib.ttref_graph_free(h)

    def run(self, graph, feed, mode="interpreted", optimize=False, outputs=None):
        outs = graph.outputs if outputs is None else outputs
        h, _ = self.build(graph, outs)
        try:
            ex = self.lib.ttref_compile(h, self.MODES[mode], int(optimize))
            if not ex:
                raise RuntimeError(self.lib.ttref_last_error().decode())
            ins = [_f32(feed[n]) for n in graph.inputs]
            res = [np.empty(o.shape, dtype=np.float32) for o in outs]
            ip = (ctypes.c_void_p * max(1, len(ins)))(*[a.ctypes.data for a in ins])
            op = (ctypes.c_void_p * max(1, len(res)))(*[r.ctypes.data for r in res])
            self._chk(self.lib.ttref_run(ex, ip, op))
            self.lib.ttref_exec_free(ex)
            return res
        finally:
            self.lib.ttref_graph_free(h)

    def time_runs(self, graph, feed, mode="avx2", reps=3, optimize=False):
        """Seconds per Executor::run (compile excluded, input copies excluded)."""
        h, _ = self.build(graph)
        try:
            ex = self.lib.ttref_compile(h, self.MODES[mode], int(optimize))
            if not ex:
                raise RuntimeError(self.lib.ttref_last_error().decode())
            ins = [_f32(feed[n]) for n in graph.inputs]
            ip = (ctypes.c_void_p * max(1, len(ins)))(*[a.ctypes.data for a in ins])
            t = self.lib.ttref_time_runs(ex, ip, reps)
            self.lib.ttref_exec_free(ex)
            if t < 0:
                raise RuntimeError(self.lib.ttref_last_error().decode())
            return t / reps
        finally:
            self.lib.ttref_graph_free(h)

    def gradients(self, graph, loss, feed, wrt):
        h, m = self.build(graph, [])
        try:
            ins = [_f32(feed[n]) for n in graph.inputs]
            res = [np.empty(w.shape, dtype=np.float32) for w in wrt]
            ip = (ctypes.c_void_p * max(1, len(ins)))(*[a.ctypes.data for a in ins])
            rp = (ctypes.c_void_p * max(1, len(res)))(*[r.ctypes.data for r in res])
            wi = (ctypes.c_int * max(1, len(wrt)))(*[m[w.index] for w in wrt])
            self._chk(self.lib.ttref_gradients(h, m[loss.index], ip, wi, len(wrt), rp))
            return res
        finally:
            self.lib.ttref_graph_free(h)

    def time_gradients(self, graph, loss, feed, reps=1):
        h, m = self.build(graph, [])
        try:
            ins = [_f32(feed[n]) for n in graph.inputs]
            ip = (ctypes.c_void_p * max(1, len(ins)))(*[a.ctypes.data for a in ins])
            t = self.lib.ttref_time_gradients(h, m[loss.index], ip, reps)
            if t < 0:
                raise RuntimeError(self.lib.ttref_last_error().decode())
            return t / reps
        finally:
            self.lib.ttref_graph_free(h)


def reference_available():
    return os.path.exists(REF_SO)
