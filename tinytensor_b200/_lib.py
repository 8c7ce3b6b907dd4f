"""ctypes binding of libtt_cuda.so (include/tt_cuda.h) and the error mapping onto the
reference exception names (include/tinytensor/utils/errors.hpp:8-66).

The library is built in-tree (tinytensor_b200/lib/libtt_cuda.so).  There is no CPU
fallback: if the library is missing, importing this module raises ImportError.
"""

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libtt_cuda.so")

TT_MAX_RANK = 8
TT_MAX_NODE_INPUTS = 2
TT_DP_ID_BYTES = 128

# op codes (reference OpType order, then additions)
OP_INPUT, OP_CONSTANT, OP_ADD, OP_SUB, OP_MUL, OP_DIV, OP_RELU, OP_SIGMOID = range(8)
OP_MATMUL, OP_TRANSPOSE, OP_REDUCE_SUM, OP_REDUCE_MEAN, OP_OUTPUT, OP_FUSED = range(8, 14)
OP_EXP, OP_NEG, OP_TANH, OP_REDUCE_MAX, OP_STEP, OP_RESHAPE, OP_EXPAND = range(14, 21)

HOST, DEVICE = 0, 1
H2D, D2H, D2D = 1, 2, 3
INFO_ORIGINAL_IR, INFO_OPTIMIZED_IR, INFO_SOURCE, INFO_PLAN, INFO_CUBIN_PATH = range(5)
FLAG_NO_FUSION, FLAG_NO_GEMM_FUSION, FLAG_HOST_ONLY, FLAG_SERIAL = 1, 2, 4, 8


class TinyTensorError(Exception):
    """Base of all backend errors (reference TinyTensorException)."""


class ShapeError(TinyTensorError):
    pass


class DimensionError(TinyTensorError):
    pass


class BroadcastError(TinyTensorError):
    pass


class TypeError(TinyTensorError):  # noqa: A001 - mirrors the reference name
    pass


class MemoryError(TinyTensorError):  # noqa: A001 - mirrors the reference name
    pass


class ResourceLimitError(TinyTensorError):
    pass


class IRError(TinyTensorError):
    pass


class CompileError(TinyTensorError):
    pass


class RuntimeExecutionError(TinyTensorError):
    pass


class DeviceStatusError(RuntimeExecutionError):
    """A kernel gave up a bounded wait and reported it through the status word."""


class NoDeviceError(RuntimeExecutionError):
    pass


class CommError(RuntimeExecutionError):
    pass


_STATUS = {
    1: ShapeError,
    2: DimensionError,
    3: BroadcastError,
    4: TypeError,
    5: MemoryError,
    6: IRError,
    7: CompileError,
    8: RuntimeExecutionError,
    9: DeviceStatusError,
    10: NoDeviceError,
    11: ValueError,
    12: CommError,
}


class TTNode(ctypes.Structure):
    _fields_ = [
        ("op", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("num_inputs", ctypes.c_int32),
        ("inputs", ctypes.c_int32 * TT_MAX_NODE_INPUTS),
        ("rank", ctypes.c_int32),
        ("shape", ctypes.c_int64 * TT_MAX_RANK),
        ("id", ctypes.c_int64),
        ("dim0", ctypes.c_int64),
        ("dim1", ctypes.c_int64),
        ("num_axes", ctypes.c_int32),
        ("keepdims", ctypes.c_int32),
        ("axes", ctypes.c_int64 * TT_MAX_RANK),
        ("data", ctypes.c_void_p),
        ("name", ctypes.c_char_p),
        ("expr", ctypes.c_char_p),
    ]


class TTGraph(ctypes.Structure):
    _fields_ = [
        ("num_nodes", ctypes.c_int32),
        ("nodes", ctypes.POINTER(TTNode)),
        ("num_inputs", ctypes.c_int32),
        ("inputs", ctypes.POINTER(ctypes.c_int32)),
        ("num_outputs", ctypes.c_int32),
        ("outputs", ctypes.POINTER(ctypes.c_int32)),
    ]


class TTCompileOptions(ctypes.Structure):
    _fields_ = [
        ("optimize", ctypes.c_int32),
        ("device", ctypes.c_int32),
        ("cache_dir", ctypes.c_char_p),
        ("grad_loss", ctypes.c_int32),
        ("num_grad_wrt", ctypes.c_int32),
        ("grad_wrt", ctypes.POINTER(ctypes.c_int32)),
        ("flags", ctypes.c_int32),
    ]


# Every entry point of include/tt_cuda.h with its ctypes signature.
_VP, _I32, _I64, _SZ, _F = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t, ctypes.c_float
SIGNATURES = {
    "tt_last_error": (ctypes.c_char_p, []),
    "tt_version": (ctypes.c_int, []),
    "tt_device_init": (ctypes.c_int, [_I32]),
    "tt_launch_count": (ctypes.c_uint64, []),
    "tt_graph_ir": (ctypes.c_int, [ctypes.POINTER(TTGraph), ctypes.c_char_p, _SZ, ctypes.POINTER(_SZ)]),
    "tt_graph_verify": (ctypes.c_int, [ctypes.POINTER(TTGraph)]),
    "tt_compile": (ctypes.c_int, [ctypes.POINTER(TTGraph), ctypes.POINTER(TTCompileOptions), ctypes.POINTER(_VP)]),
    "tt_program_info": (ctypes.c_int, [_VP, _I32, ctypes.c_char_p, _SZ, ctypes.POINTER(_SZ)]),
    "tt_program_num_io": (ctypes.c_int, [_VP, ctypes.POINTER(_I32), ctypes.POINTER(_I32)]),
    "tt_program_output_shape": (ctypes.c_int, [_VP, _I32, ctypes.POINTER(_I32), ctypes.POINTER(_I64)]),
    "tt_program_run": (ctypes.c_int, [_VP, ctypes.POINTER(_VP), ctypes.POINTER(_VP), _I32, _VP]),
    "tt_program_status": (ctypes.c_int, [_VP, ctypes.POINTER(_I32)]),
    "tt_program_set_profiling": (ctypes.c_int, [_VP, _I32]),
    "tt_program_profile": (
        ctypes.c_int,
        [_VP, _I32, ctypes.c_char_p, _I32, ctypes.POINTER(_F), ctypes.POINTER(_I32)],
    ),
    "tt_program_destroy": (ctypes.c_int, [_VP]),
    "tt_program_set_output_events": (ctypes.c_int, [_VP, ctypes.POINTER(_VP), _I32]),
    "tt_program_output_step": (ctypes.c_int, [_VP, _I32, ctypes.POINTER(_I32)]),
    "tt_program_set_input_events": (ctypes.c_int, [_VP, ctypes.POINTER(_VP), _I32]),
    "tt_program_input_step": (ctypes.c_int, [_VP, _I32, ctypes.POINTER(_I32)]),
    "tt_device_alloc": (ctypes.c_int, [_SZ, ctypes.POINTER(_VP)]),
    "tt_device_free": (ctypes.c_int, [_VP]),
    "tt_host_alloc": (ctypes.c_int, [_SZ, ctypes.POINTER(_VP)]),
    "tt_host_free": (ctypes.c_int, [_VP]),
    "tt_memcpy": (ctypes.c_int, [_VP, _VP, _SZ, _I32, _VP]),
    "tt_stream_create": (ctypes.c_int, [ctypes.POINTER(_VP)]),
    "tt_stream_destroy": (ctypes.c_int, [_VP]),
    "tt_stream_sync": (ctypes.c_int, [_VP]),
    "tt_event_create": (ctypes.c_int, [ctypes.POINTER(_VP)]),
    "tt_event_destroy": (ctypes.c_int, [_VP]),
    "tt_event_record": (ctypes.c_int, [_VP, _VP]),
    "tt_stream_wait_event": (ctypes.c_int, [_VP, _VP]),
    "tt_selftest_bounded_wait": (ctypes.c_int, [_I64, ctypes.POINTER(_I32)]),
    "tt_stream_begin_capture": (ctypes.c_int, [_VP]),
    "tt_stream_end_capture": (ctypes.c_int, [_VP, ctypes.POINTER(_VP)]),
    "tt_graph_launch": (ctypes.c_int, [_VP, _VP]),
    "tt_graph_destroy": (ctypes.c_int, [_VP]),
    "tt_sgd_step": (
        ctypes.c_int,
        [_I32, ctypes.POINTER(_VP), ctypes.POINTER(_VP), ctypes.POINTER(_VP), ctypes.POINTER(_I64), _F, _F, _VP],
    ),
    "tt_gemm_f32_noalloc": (ctypes.c_int, [_VP, _VP, _VP, _I64, _I64, _I64, _VP, _VP]),
    "tt_dp_unique_id": (ctypes.c_int, [ctypes.c_char_p]),
    "tt_dp_init": (ctypes.c_int, [_I32, _I32, ctypes.c_char_p, _I32, ctypes.POINTER(_VP)]),
    "tt_dp_allreduce_sum": (ctypes.c_int, [_VP, _VP, _SZ, _VP]),
    "tt_dp_destroy": (ctypes.c_int, [_VP]),
}


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `make -C tinytensor_b200/csrc` "
            "(or __graft_entry__.build()); the CUDA backend has no CPU fallback"
        )
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def check(status: int) -> None:
    """Raises the exception class that mirrors the reference for a nonzero status."""
    if status == 0:
        return
    msg = lib.tt_last_error().decode(errors="replace")
    raise _STATUS.get(status, RuntimeExecutionError)(msg)


def cstr(fn, *args) -> str:
    """Calls a (…, char* buf, size_t cap, size_t* needed) entry point and returns the text."""
    needed = ctypes.c_size_t(0)
    check(fn(*args, None, 0, ctypes.byref(needed)))
    buf = ctypes.create_string_buffer(needed.value)
    check(fn(*args, buf, needed.value, ctypes.byref(needed)))
    return buf.value.decode()
