"""Worker processes of the data-parallel tests (spawned, one per rank).

CPU workers use torch.distributed with the gloo backend on 127.0.0.1; the GPU worker
(`gpu_dp_worker`, run under torchrun on >= 2 GPUs) drives the real NCCL path through
tinytensor_b200.DataParallelSGD.  Every worker reports through files or a queue and
never waits without a timeout.
"""

import datetime
import os
import sys
import traceback

import numpy as np

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

DIMS = (24, 32, 32, 10)   # small MLP: in -> hidden -> hidden -> out
GLOBAL_ROWS = 32
LR = 0.05
STEPS = 3


def mlp(tt, rows, dims=DIMS):
    g = tt.Graph()
    X, T = g.input([rows, dims[0]], name="X"), g.input([rows, dims[3]], name="T")
    W1 = g.input([dims[0], dims[1]], name="W1")
    W2 = g.input([dims[1], dims[2]], name="W2")
    W3 = g.input([dims[2], dims[3]], name="W3")
    d = tt.tanh(tt.relu(X @ W1) @ W2) @ W3 - T
    return g, (X, T, W1, W2, W3), tt.mean(d * d)


def mlp_data(seed, rows=GLOBAL_ROWS, dims=DIMS):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, dims[0])).astype(np.float32)
    t = rng.standard_normal((rows, dims[3])).astype(np.float32)
    ws = []
    for fi, fo in zip(dims[:-1], dims[1:]):
        lim = np.sqrt(6.0 / (fi + fo))
        ws.append(rng.uniform(-lim, lim, (fi, fo)).astype(np.float32))
    return x, t, ws


def full_batch_oracle_steps(seed, steps=STEPS):
    """Single-process reference: SGD on the mean loss of the whole batch."""
    import tinytensor_b200 as tt
    from oracle import oracle as O

    x, t, ws = mlp_data(seed)
    g, (X, T, W1, W2, W3), loss = mlp(tt, GLOBAL_ROWS)
    for _ in range(steps):
        grads = O.gradients(g, loss, {X: x, T: t, W1: ws[0], W2: ws[1], W3: ws[2]}, [W1, W2, W3])
        ws = [O.sgd(w, gw, LR)[0] for w, gw in zip(ws, grads)]
    return ws


def _init_gloo(rank, world, port, timeout_s):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def dp_protocol_worker(rank, world, port, seed, q):
    """Shard the batch with shard_rows, take oracle gradients of the local shard's mean
    loss, sum them over ranks (gloo all-reduce) and apply SGD with lr / world: the
    protocol DataParallelSGD runs on the GPU.  Reports the final weights."""
    try:
        import torch

        import tinytensor_b200 as tt
        from oracle import oracle as O

        dist = _init_gloo(rank, world, port, 60)
        x, t, ws = mlp_data(seed)
        r0, r1 = tt.shard_rows(GLOBAL_ROWS, rank, world)
        g, (X, T, W1, W2, W3), loss = mlp(tt, r1 - r0)
        for _ in range(STEPS):
            grads = O.gradients(g, loss, {X: x[r0:r1], T: t[r0:r1], W1: ws[0], W2: ws[1], W3: ws[2]}, [W1, W2, W3])
            flat = torch.from_numpy(np.concatenate([gw.reshape(-1) for gw in grads]).copy())
            dist.all_reduce(flat, op=dist.ReduceOp.SUM)
            parts = np.split(flat.numpy(), np.cumsum([w.size for w in ws])[:-1])
            ws = [O.sgd(w, p.reshape(w.shape), LR / world)[0] for w, p in zip(ws, parts)]
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok", [w.copy() for w in ws]))
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


def bootstrap_worker(rank, world, port, q):
    """Every rank receives rank 0's NCCL unique id through the gloo group; without a GPU
    the communicator then fails with NoDeviceError (never a hang)."""
    try:
        import torch

        import tinytensor_b200 as tt

        dist = _init_gloo(rank, world, port, 60)
        uid = tt.broadcast_unique_id()
        ids = [None] * world
        dist.all_gather_object(ids, uid)
        outcome = "skipped"
        if not torch.cuda.is_available():
            try:
                tt.Communicator(rank, world, 0, uid)
                outcome = "no error"
            except tt.native.NoDeviceError:
                outcome = "NoDeviceError"
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok", (len(uid), all(i == ids[0] for i in ids), outcome)))
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


def failing_rank_worker(rank, world, port, q):
    """Rank 1 fails on the host before the step's collective and leaves the group;
    rank 0's collective must end with an error within the group's short timeout."""
    import time

    try:
        import torch

        dist = _init_gloo(rank, world, port, 5)
        if rank == 1:
            q.put((rank, "ok", "raised"))
            raise SystemExit(3)
        t0 = time.time()
        try:
            dist.all_reduce(torch.ones(4), op=dist.ReduceOp.SUM)
            q.put((rank, "ok", ("completed", time.time() - t0)))
        except Exception as e:  # gloo reports the lost peer / timeout as RuntimeError
            q.put((rank, "ok", ("detected", time.time() - t0, type(e).__name__)))
    except SystemExit:
        raise
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


def gpu_dp_worker():
    """torchrun worker (>= 2 GPUs): STEPS DataParallelSGD steps over NCCL on a larger
    MLP; every rank writes its final weights to $TT_DP_OUT/rank<r>.npz."""
    import torch
    import torch.distributed as dist

    import tinytensor_b200 as tt

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    out_dir = os.environ["TT_DP_OUT"]
    dims = (256, 512, 512, 10)
    rows = 1024
    torch.cuda.set_device(local)
    tt.device_init(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    comm = tt.Communicator.from_torch_distributed(local)
    x, t, ws = mlp_data(7, rows, dims)
    r0, r1 = tt.shard_rows(rows, rank, world)
    g, (X, T, W1, W2, W3), loss = mlp(tt, r1 - r0, dims)
    prog = tt.compile_gradients(g, loss, [W1, W2, W3], device=local)
    params = [tt.DeviceBuffer.from_numpy(w) for w in ws]
    trainer = tt.DataParallelSGD(prog, params, lr=LR, comm=comm)
    dx, dt = tt.DeviceBuffer.from_numpy(x[r0:r1]), tt.DeviceBuffer.from_numpy(t[r0:r1])
    stream = tt.Stream()
    for _ in range(STEPS):
        trainer.step([dx, dt], stream)
    stream.synchronize()
    if prog.status() != 0:
        raise RuntimeError(f"device status {prog.status()}")
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), *[p.numpy() for p in params])
    dist.barrier()
    comm.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    gpu_dp_worker()
