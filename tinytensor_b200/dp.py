"""Data parallelism for batch-sharded graphs (no reference counterpart).

One process per GPU.  Rank r runs the full forward/backward program on rows
[r*B/N, (r+1)*B/N) of the global batch; the weight gradients are summed across ranks
with an NCCL all-reduce over NVLink (tt_dp_allreduce_sum) and the SGD step applies
lr/N, so every replica stays bit-identical.  torch.distributed (any backend) is used
only to hand the NCCL unique id from rank 0 to the others.
"""

import ctypes

from . import _lib

__all__ = ["Communicator", "shard_rows"]


def shard_rows(global_rows: int, rank: int, world: int):
    """Contiguous row range of `rank` (equal shards; global_rows % world == 0)."""
    if global_rows % world:
        raise ValueError(f"global batch {global_rows} is not divisible by world size {world}")
    per = global_rows // world
    return rank * per, (rank + 1) * per


class Communicator:
    def __init__(self, rank: int, world: int, device: int, unique_id: bytes):
        if len(unique_id) != _lib.TT_DP_ID_BYTES:
            raise ValueError("NCCL unique id must be 128 bytes")
        h = ctypes.c_void_p()
        _lib.check(_lib.lib.tt_dp_init(rank, world, unique_id, device, ctypes.byref(h)))
        self.handle = h.value
        self.rank, self.world = rank, world

    @staticmethod
    def new_unique_id() -> bytes:
        buf = ctypes.create_string_buffer(_lib.TT_DP_ID_BYTES)
        _lib.check(_lib.lib.tt_dp_unique_id(buf))
        return buf.raw

    @classmethod
    def from_torch_distributed(cls, device: int):
        """Bootstraps from an initialised torch.distributed group (rank 0 makes the id)."""
        import torch.distributed as dist

        rank, world = dist.get_rank(), dist.get_world_size()
        obj = [cls.new_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        return cls(rank, world, device, obj[0])

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
