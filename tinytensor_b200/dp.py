"""Data parallelism for batch-sharded graphs (no reference counterpart).

One process per GPU.  Rank r runs the full forward/backward program on rows
[r*B/N, (r+1)*B/N) of the global batch; the weight gradients are summed across ranks
with an NCCL all-reduce over NVLink (tt_dp_allreduce_sum) and the SGD step applies
lr/N, so every replica stays bit-identical.  Because the shards are equal, the mean of
the shard losses is the global-batch mean and the summed shard gradients / N are its
gradients.  torch.distributed (any backend) is used only to hand the NCCL unique id
from rank 0 to the others.
"""

import ctypes

import numpy as np

from . import _lib

__all__ = ["Communicator", "DataParallelSGD", "shard_rows", "broadcast_unique_id"]


def shard_rows(global_rows: int, rank: int, world: int):
    """Contiguous row range of `rank` (equal shards; global_rows % world == 0)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    if global_rows % world:
        raise ValueError(f"global batch {global_rows} is not divisible by world size {world}")
    per = global_rows // world
    return rank * per, (rank + 1) * per


def _load_process_nccl() -> None:
    """The library binds to the libnccl.so.2 already in the process; importing torch
    first makes that torch's NCCL, so torch.distributed and this module share one."""
    try:
        import torch  # noqa: F401
    except ImportError:
        pass


def broadcast_unique_id() -> bytes:
    """Rank 0 creates an NCCL unique id and the initialised torch.distributed group
    (gloo or nccl) broadcasts it; every rank returns the same 128 bytes."""
    import torch.distributed as dist

    obj = [Communicator.new_unique_id() if dist.get_rank() == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    uid = obj[0]
    if not isinstance(uid, bytes) or len(uid) != _lib.TT_DP_ID_BYTES:
        raise _lib.RuntimeExecutionError("NCCL unique id broadcast returned a malformed id")
    return uid


class Communicator:
    def __init__(self, rank: int, world: int, device: int, unique_id: bytes):
        if len(unique_id) != _lib.TT_DP_ID_BYTES:
            raise ValueError("NCCL unique id must be 128 bytes")
        self.handle = None
        _load_process_nccl()
        h = ctypes.c_void_p()
        _lib.check(_lib.lib.tt_dp_init(rank, world, unique_id, device, ctypes.byref(h)))
        self.handle = h.value
        self.rank, self.world = rank, world

    @staticmethod
    def new_unique_id() -> bytes:
        _load_process_nccl()
        buf = ctypes.create_string_buffer(_lib.TT_DP_ID_BYTES)
        _lib.check(_lib.lib.tt_dp_unique_id(buf))
        return buf.raw

    @classmethod
    def from_torch_distributed(cls, device: int):
        """Bootstraps from an initialised torch.distributed group (rank 0 makes the id)."""
        import torch.distributed as dist

        uid = broadcast_unique_id()
        return cls(dist.get_rank(), dist.get_world_size(), device, uid)

    def allreduce_sum(self, buf, count: int | None = None, stream=None) -> None:
        ptr = getattr(buf, "ptr", buf)
        n = count if count is not None else buf.nbytes // 4
        h = getattr(stream, "handle", stream)
        _lib.check(_lib.lib.tt_dp_allreduce_sum(self.handle, ptr, n, h))

    def close(self):
        if self.handle:
            _lib.check(_lib.lib.tt_dp_destroy(self.handle))
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DataParallelSGD:
    """One data-parallel SGD step per call.

    `program` is a compiled gradient program (tt.compile_gradients) whose inputs are
    `batch_inputs + params` and whose outputs are `[loss] + [d loss / d p]`.  The
    gradients land in one contiguous buffer.  With a communicator, each gradient is
    all-reduced on a second stream as soon as the program has produced it (the
    program's output events; the scheduler runs output-producing launches as early as
    their inputs allow), in the order the program produces them — the same on every
    rank — so the exchange of one layer's gradient overlaps the backward pass of the
    layers before it.  With early_update, each parameter is then updated on the same
    side stream as soon as its gradient is exchanged and the program's last launch that
    reads the parameter is done (the program's input-released events), so only the last
    layer's exchange and update remain after the backward pass; the next step waits for
    all updates.  Updates apply lr / world.  With comm=None (one process) there is no
    exchange (early updates still overlap the backward pass); overlap=False all-reduces
    the whole buffer once after the program and updates after that.
    """

    def __init__(self, program, params, lr: float = 0.01, momentum: float = 0.0, comm=None, overlap: bool = True,
                 early_update: bool = True):
        from .compiler import DeviceBuffer, Event, Stream
        from .optim import SGD

        self.program = program
        self.params = list(params)
        self.comm = comm
        self.world = comm.world if comm is not None else 1
        self.sizes = [int(np.prod(p.shape, dtype=np.int64)) for p in self.params]
        self.grads = DeviceBuffer([max(1, sum(self.sizes))])
        offs = np.cumsum([0] + self.sizes)[:-1]
        self.grad_ptrs = [self.grads.ptr + int(o) * 4 for o in offs]
        self.loss = DeviceBuffer([])
        self.opt = SGD(self.params, lr=lr, momentum=momentum)
        self.overlap = bool(overlap and comm is not None and comm.world > 1)
        self.early_update = bool(early_update and (self.overlap or comm is None or comm.world == 1))
        if self.overlap or self.early_update:
            self.comm_stream = Stream()
            self.ready = [Event() for _ in self.params]
            self.exchanged = Event()
            program.set_output_events([None] + self.ready)
            steps = program.output_steps()[1:1 + len(self.params)]
            # exchange order = production order (ties: parameter order), identical on all ranks
            self.order = sorted(range(len(self.params)), key=lambda i: (steps[i], i))
        if self.early_update:
            # parameters are the program's last inputs: released once no launch reads them
            self.released = [Event() for _ in self.params]
            nin = program.num_inputs
            program.set_input_events([None] * (nin - len(self.params)) + self.released)

    def step_host(self, host_inputs, stream) -> None:
        """step() with the batch in page-locked host memory (PinnedBuffer per input).
        This call's host-to-device copies run on a copy stream into one of two device
        slots, so they overlap the previous step still running on the GPU; the step
        waits for its own copies, and a slot is refilled only after the step that read
        it has finished.  The copies read the host buffers asynchronously: keep a
        buffer unchanged until the next step_host call (or a synchronize) — e.g.
        alternate two host buffers."""
        from .compiler import DeviceBuffer, Event, Stream

        if getattr(self, "_slots", None) is None:
            self._slots = [[DeviceBuffer(h.shape) for h in host_inputs] for _ in range(2)]
            self._copy_stream = Stream()
            self._copied = [Event(), Event()]
            self._consumed = [Event(), Event()]
            self._consumed_pending = [False, False]
            self._slot = 0
        j = self._slot
        bufs = self._slots[j]
        if self._consumed_pending[j]:
            self._consumed[j].wait(self._copy_stream)
        for h, b in zip(host_inputs, bufs):
            if h.array.nbytes != b.nbytes:
                raise ValueError("host batch shapes changed between steps")
            _lib.check(_lib.lib.tt_memcpy(b.ptr, h.ptr, b.nbytes, _lib.H2D, self._copy_stream.handle))
        self._copied[j].record(self._copy_stream)
        self._copied[j].wait(stream)
        self.step(bufs, stream)
        self._consumed[j].record(stream)
        self._consumed_pending[j] = True
        self._slot ^= 1

    def step(self, batch_inputs, stream) -> None:
        """Queues forward+backward on the local shard, the gradient all-reduce and the
        update; the local shard's loss is left in `self.loss` (device)."""
        self.program.run_device(list(batch_inputs) + self.params, [self.loss] + self.grad_ptrs, stream)
        if self.overlap or self.early_update:
            for i in self.order:
                self.ready[i].wait(self.comm_stream)
                if self.overlap:
                    self.comm.allreduce_sum(self.grad_ptrs[i], self.sizes[i], self.comm_stream)
                if self.early_update:
                    self.released[i].wait(self.comm_stream)
                    self.opt.step_one(i, self.grad_ptrs[i], self.comm_stream, lr_scale=1.0 / self.world)
            self.exchanged.record(self.comm_stream)
            self.exchanged.wait(stream)
            if not self.early_update:
                self.opt.step(self.grad_ptrs, stream, lr_scale=1.0 / self.world)
            return
        if self.comm is not None:
            self.comm.allreduce_sum(self.grads.ptr, sum(self.sizes), stream)
        self.opt.step(self.grad_ptrs, stream, lr_scale=1.0 / self.world)
