"""tinytensor_b200: a B200 (sm_100a) execution backend for TinyTensor graphs.

The Python API mirrors the reference package (python/tinytensor): Graph builders,
tt.compile(...) -> CompiledProgram with run / original_ir / optimized_ir /
generated_source / execution_plan, tt.gradients, SGD.  Compilation and execution go
through the C ABI of libtt_cuda.so (include/tt_cuda.h); there is no CPU fallback.
"""

__version__ = "0.1.0"

from ._lib import (  # noqa: F401
    BroadcastError,
    CommError,
    CompileError,
    DeviceStatusError,
    DimensionError,
    IRError,
    MemoryError,
    NoDeviceError,
    ResourceLimitError,
    RuntimeExecutionError,
    ShapeError,
    TinyTensorError,
    TypeError,
)
from ._lib import FLAG_HOST_ONLY, FLAG_NO_FUSION, FLAG_NO_GEMM_FUSION, FLAG_SERIAL  # noqa: F401
from .compiler import (  # noqa: F401
    CompiledProgram,
    CudaGraph,
    DeviceBuffer,
    Event,
    PinnedBuffer,
    Stream,
    Tensor,
    compile,
    compile_gradients,
    gradients,
    launch_count,
    tensor,
)
from .dp import Communicator, DataParallelSGD, broadcast_unique_id, shard_rows  # noqa: F401
from .graph import (  # noqa: F401
    Graph,
    Node,
    add,
    div,
    exp,
    float32,
    float64,
    matmul,
    max,
    mean,
    mul,
    neg,
    relu,
    sigmoid,
    sub,
    sum,
    tanh,
    transpose,
)
from .optim import SGD  # noqa: F401
from . import _lib as native  # noqa: F401


def device_init(device: int = 0) -> None:
    """Checks that `device` is an sm_100 GPU and creates its context."""
    native.check(native.lib.tt_device_init(device))
