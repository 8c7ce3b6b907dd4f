"""Data-parallel host logic at world_size 2 on CPU (gloo), and the NCCL path on >= 2
GPUs.  The CPU tests cover: batch sharding, the NCCL-id bootstrap through a
torch.distributed group, the step protocol DataParallelSGD runs (sum of shard
gradients of the shard means, lr / world) against full-batch SGD, and a rank that
fails on the host between steps (the survivor's collective errors out within the
group's timeout instead of hanging)."""

import multiprocessing as mp
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

import dp_workers as W
from parity import GEMM_FROB_RTOL, assert_norm

import tinytensor_b200 as tt

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run_ranks(target, world, *args, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port) + args + (q,)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, status, payload = q.get(timeout=timeout)
            assert status == "ok", f"rank {rank} failed:\n{payload}"
            results[rank] = payload
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
                p.join()
    return results, [p.exitcode for p in procs]


def test_shard_rows_cover_the_batch_in_order():
    for world in (1, 2, 4, 8):
        spans = [tt.shard_rows(32768, r, world) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == 32768
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        assert len({e - s for s, e in spans}) == 1
    with pytest.raises(ValueError):
        tt.shard_rows(10, 0, 3)
    with pytest.raises(ValueError):
        tt.shard_rows(8, 2, 2)


def test_unique_id_bootstrap_over_gloo():
    res, codes = _run_ranks(W.bootstrap_worker, 2)
    assert codes == [0, 0]
    for rank in (0, 1):
        nbytes, same, outcome = res[rank]
        assert nbytes == 128 and same
        assert outcome in ("NoDeviceError", "skipped")


def test_dp_protocol_matches_full_batch_sgd():
    seed = 11
    res, codes = _run_ranks(W.dp_protocol_worker, 2, seed)
    assert codes == [0, 0]
    w0, w1 = res[0], res[1]
    for a, b in zip(w0, w1):
        assert np.array_equal(a, b), "replicas diverged"
    ref = W.full_batch_oracle_steps(seed)
    for a, r in zip(w0, ref):
        assert_norm(a, r, GEMM_FROB_RTOL)
    # the step really moved the weights (the comparison is not vacuous)
    _, _, w_init = W.mlp_data(seed)
    assert all(np.abs(a - i).max() > 1e-4 for a, i in zip(w0, w_init))


def test_failed_rank_is_detected_not_waited_for():
    res, codes = _run_ranks(W.failing_rank_worker, 2, timeout=90)
    assert res[1] == "raised" and codes[1] == 3
    outcome = res[0]
    assert outcome[0] == "detected", outcome
    assert outcome[1] < 60.0


def _gpu_count():
    import torch

    return torch.cuda.device_count()


@pytest.mark.gpu
def test_gpu_dp_two_ranks_match_single_gpu_full_batch(tmp_path, cache_dir):
    """DataParallelSGD over NCCL on 2 GPUs == the same steps on one GPU with the whole
    batch (GEMM tolerance), and the two replicas are bit-identical."""
    if _gpu_count() < 2:
        pytest.skip(f"needs 2 GPUs, {_gpu_count()} visible")
    env = dict(os.environ, TT_DP_OUT=str(tmp_path), NCCL_NVLS_ENABLE="0", TT_CUDA_CACHE=cache_dir)
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           os.path.join(HERE, "dp_workers.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    w = [np.load(tmp_path / f"rank{i}.npz") for i in range(2)]
    for k in w[0].files:
        assert np.array_equal(w[0][k], w[1][k]), "replicas diverged"

    dims, rows = (256, 512, 512, 10), 1024
    x, t, ws = W.mlp_data(7, rows, dims)
    g, (X, T, W1, W2, W3), loss = W.mlp(tt, rows, dims)
    prog = tt.compile_gradients(g, loss, [W1, W2, W3], cache_dir=cache_dir)
    params = [tt.DeviceBuffer.from_numpy(a) for a in ws]
    trainer = tt.DataParallelSGD(prog, params, lr=W.LR)
    dx, dt = tt.DeviceBuffer.from_numpy(x), tt.DeviceBuffer.from_numpy(t)
    stream = tt.Stream()
    for _ in range(W.STEPS):
        trainer.step([dx, dt], stream)
    stream.synchronize()
    for i, p in enumerate(params):
        assert_norm(w[0][f"arr_{i}"], p.numpy(), GEMM_FROB_RTOL)
