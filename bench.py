"""Benchmark of the TinyTensor B200 backend.

Headline workload (the one that runs at 1/2/4/8 GPUs): the data-parallel SGD step of
the 3-layer MLP 1024 -> 4096 (ReLU) -> 4096 (tanh) -> 10 with MSE loss, global batch
32768 split by rows over the ranks (32768/N each), lr 0.01.  One step = forward +
symbolic backward (one compiled program) + NCCL sum all-reduce of the weight
gradients + fused SGD (lr/N).  Total work is fixed as N grows ("strong").
Synthetic data: X, T ~ N(0,1) seed 4, Xavier-uniform weights seed 4.

At N=1 the line also carries the single-GPU components of the metric (fused
elementwise GB/s, reductions GB/s, fp32-accurate GEMM TFLOP/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
    python bench.py --batch 8192 ...          # a smaller MLP step (profiling case)
    python bench.py --workload gemm --size M,N,K ...   # one compiled program (profiling case)
"""

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

GLOBAL_BATCH = 32768
LR = 0.01
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


def load_traffic(label):
    """DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum, one ncu capture,
    scaled to the benchmarked batch) for the launch whose label, up to its first ']', is
    listed in profiles/traffic_per_launch.txt (tab-separated lines 'label, bytes, how');
    None when that launch was not captured."""
    p = os.path.join(ROOT, "profiles", "traffic_per_launch.txt")
    if not os.path.exists(p) or "]" not in label:
        return None
    key = label[:label.index("]") + 1]
    with open(p) as f:
        for line in f:
            parts = line.rstrip("\n").split("\t")
            if len(parts) >= 2 and not line.startswith("#") and parts[0] == key:
                return int(float(parts[1]))
    return None


def headline_config(batch, world):
    """The workload's config, identical in both arms."""
    return {"workload": "mlp_dp_sgd_step", "model": "MLP 1024-4096-4096-10 MSE", "global_batch": batch,
            "per_gpu_batch": batch // world, "lr": LR, "parallelism": f"dp{world}",
            "l2": "inputs larger than L2 (activations 512 MiB per 32768 rows, weights 84 MB)",
            "tflops_per_step": round(mlp_flops(batch) / 1e12, 4)}


HEADLINE_METRIC = "MLP DP SGD step/s (1024-4096-4096-10, global batch {})"


def mlp_flops(rows, with_dx=False):
    fwd = 2 * rows * (1024 * 4096 + 4096 * 4096 + 4096 * 10)
    bwd = 2 * fwd if with_dx else 2 * fwd - 2 * rows * 1024 * 4096
    return fwd + bwd


def xavier(rng, fi, fo):
    lim = np.sqrt(6.0 / (fi + fo))
    return rng.uniform(-lim, lim, (fi, fo)).astype(np.float32)


def mlp_data(seed=4, rows=GLOBAL_BATCH):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, 1024)).astype(np.float32)
    t = rng.standard_normal((rows, 10)).astype(np.float32)
    w = [xavier(rng, 1024, 4096), xavier(rng, 4096, 4096), xavier(rng, 4096, 10)]
    return x, t, w


def mlp_graph(tt, rows):
    g = tt.Graph()
    X, T = g.input([rows, 1024], name="X"), g.input([rows, 10], name="T")
    W1, W2, W3 = g.input([1024, 4096], name="W1"), g.input([4096, 4096], name="W2"), g.input([4096, 10], name="W3")
    h1 = tt.relu(X @ W1)
    h2 = tt.tanh(h1 @ W2)
    d = h2 @ W3 - T
    loss = tt.mean(d * d)
    return g, (X, T, W1, W2, W3), loss


def bind_to_gpu_numa_node(torch, device):
    """Restricts this process to the CPUs of the NUMA node that GPU `device` hangs off
    (sysfs), before any page-locked host buffer is allocated, so that the per-step
    host-to-device copies of the end-to-end loop read node-local memory when several
    ranks copy at once.  Returns the node, or None where the topology is not exposed."""
    try:
        p = torch.cuda.get_device_properties(device)
        bus = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        with open(f"/sys/bus/pci/devices/{bus}/numa_node") as f:
            node = int(f.read().strip())
        if node < 0:
            return None
        with open(f"/sys/devices/system/node/node{node}/cpulist") as f:
            cpus = set()
            for part in f.read().strip().split(","):
                lo, _, hi = part.partition("-")
                cpus.update(range(int(lo), int(hi or lo) + 1))
        if cpus:
            os.sched_setaffinity(0, cpus)
        return node
    except (OSError, ValueError, AttributeError, RuntimeError):
        return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        # raw samples: TT_BENCH_CLOCKS_DIR if set, else the system temp directory
        out_dir = os.environ.get("TT_BENCH_CLOCKS_DIR") or tempfile.gettempdir()
        self.path = os.path.join(out_dir, f"clocks_bench_{os.getpid()}.csv")

    def start(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        self.proc.wait()
        self.f.close()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    smax = float(parts[2])
                except ValueError:
                    continue
                for nm, v in zip(names, parts[5:9]):
                    if v.lower() == "active":
                        reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax, "samples": len(sm),
                "reasons": sorted(reasons)}


# --------------------------------------------------------------------------------------------
# B200 arm
# --------------------------------------------------------------------------------------------

def run_b200(args):
    import torch

    import tinytensor_b200 as tt

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 with torch.distributed.run")
    torch.cuda.set_device(local)
    numa_node = bind_to_gpu_numa_node(torch, local)
    tt.device_init(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    peaks, peak_src = load_peaks()

    batch = args.batch
    rows = batch // world
    r0 = rank * rows
    x, t, w = mlp_data(rows=batch)
    xs, ts = x[r0:r0 + rows], t[r0:r0 + rows]
    g, (X, T, W1, W2, W3), loss = mlp_graph(tt, rows)
    prog = tt.compile_gradients(g, loss, [W1, W2, W3], device=local)
    stream = tt.Stream()
    tstream = torch.cuda.ExternalStream(stream.handle)
    dx, dt = tt.DeviceBuffer.from_numpy(xs), tt.DeviceBuffer.from_numpy(ts)
    dw = [tt.DeviceBuffer.from_numpy(a) for a in w]
    comm = tt.Communicator.from_torch_distributed(local) if world > 1 else None
    trainer = tt.DataParallelSGD(prog, dw, lr=LR, comm=comm, early_update=not args.no_early_update)
    dloss = trainer.loss

    def step():
        trainer.step([dx, dt], stream)

    def barrier():
        torch.cuda.synchronize()
        stream.synchronize()
        if dist is not None:
            dist.barrier()

    def max_over_ranks(v):
        if dist is None:
            return v
        tv = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(tv, op=dist.ReduceOp.MAX)
        return float(tv.item())

    for _ in range(args.warmup):
        step()
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n0 = tt.launch_count()
    barrier()
    ev0.record(tstream)
    for _ in range(args.steps):
        step()
    ev1.record(tstream)
    barrier()
    launches = tt.launch_count() - n0
    ms = ev0.elapsed_time(ev1) / args.steps
    clk = clocks.stop()
    ms = max_over_ranks(ms)
    assert prog.status() == 0

    # per-launch device times: a second pass of the same steps with an event pair around
    # every launch (kept out of the headline pass above, whose timing it would disturb)
    prog.set_profiling(True)
    barrier()
    for _ in range(args.steps):
        step()
    barrier()
    prof = prog.profile()
    prog.set_profiling(False)
    assert prog.status() == 0

    # end to end through the public API: per step H2D of this rank's (X, T) shard from
    # pinned host memory (DataParallelSGD.step_host: copies on a copy stream into
    # alternating device slots, overlapping the previous step), the step, D2H of the loss.
    # Two host batches alternate, as step_host asks.
    hosts = []
    for _ in range(2):
        px, pt = tt.PinnedBuffer(xs.shape), tt.PinnedBuffer(ts.shape)
        px.array[...] = xs
        pt.array[...] = ts
        hosts.append([px, pt])
    hloss = tt.PinnedBuffer([1])
    from tinytensor_b200 import _lib
    trainer.step_host(hosts[1], stream)  # allocates the device slots outside the timed region
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(tstream)
    for i in range(args.steps):
        trainer.step_host(hosts[i % 2], stream)
        _lib.check(_lib.lib.tt_memcpy(hloss.ptr, dloss.ptr, 4, _lib.D2H, stream.handle))
    e1.record(tstream)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)

    # dominant kernel of the step and its roofline
    labels = {}
    for lbl, t_ms in prof:
        labels.setdefault(lbl, []).append(t_ms)
    top_lbl, top_ms = max(prof, key=lambda p: p[1])
    gemm_flops = None
    if top_lbl.startswith("gemm"):
        dims = top_lbl.split("[")[1].split()[0].split("x")
        m, n, k = (int(v) for v in dims)
        gemm_flops = 2.0 * m * n * k
    # The dominant launch is timed inside a long step, so its denominator is the
    # sustained (power-capped) bf16 figure; the burst-based fraction is reported beside it.
    sustained = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
    eff_peak = sustained / 2.0 / 3.0        # TF32 = bf16/2; 3xTF32: three TF32 products per fp32 product
    burst_peak = peaks["bf16_tflops"] / 2.0 / 3.0
    achieved = gemm_flops / (top_ms * 1e-3) / 1e12 if gemm_flops else None
    roofline = {
        "kernel": top_lbl,
        "bound": "tensor",
        "achieved": round(achieved, 2) if achieved else None,
        "peak": round(eff_peak, 1),
        "unit": "TFLOP/s",
        "frac": round(achieved / eff_peak, 4) if achieved else None,
        "traffic": load_traffic(top_lbl),
        "peak_source": f"{peak_src} sustained bf16 (bf16_tflops_sustained) /2 (TF32) /3 (3xTF32 products), "
                       "fp32-equivalent",
        "frac_of_burst_peak": round(achieved / burst_peak, 4) if achieved else None,
        "burst_peak": round(burst_peak, 1),
        "avg_ms": round(top_ms, 4),
        "timed": "CUDA events on the launch stream around the GEMM launch (its hi/lo split pre-pass and "
                 "split-K reduce included), averaged over a second pass of the same steps run right after the "
                 "headline pass (the headline pass itself records no per-launch events)",
    }
    total_prof = sum(t for _, t in prof)
    step_profile = [{"launch": lbl, "ms": round(t, 4), "share": round(t / total_prof, 4)}
                    for lbl, t in sorted(prof, key=lambda p: -p[1])[:10]]
    step_flops = mlp_flops(batch)
    out = {
        "metric": HEADLINE_METRIC.format(batch),
        "value": round(1000.0 / ms, 4),
        "unit": "step/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32 (3xTF32 tensor-core GEMM, fp32 accumulate)",
        "data": "synthetic: X,T ~ N(0,1) seed 4; Xavier-uniform weights seed 4",
        "config": headline_config(batch, world),
        "tflops": round(step_flops / (ms * 1e-3) / 1e12, 2),
        "e2e": {"value": round(1000.0 / e2e_ms, 4), "unit": "step/s",
                "h2d_bytes_per_step": int(dx.nbytes + dt.nbytes) * world, "d2h_bytes_per_step": 4 * world},
        "gpu_launches": int(launches),
        "roofline": roofline,
        "step_profile": step_profile,
        "clocks": clk,
        "host_numa_node": numa_node,
    }
    if world == 1 and not args.no_components:
        out["components"] = components(tt, torch, args, peaks, peak_src)
    if rank == 0 and not args.no_cpu_baseline and world == 1 and batch == GLOBAL_BATCH:
        out["cpu_baseline"] = cpu_baseline(batch)
        if not args.no_components:
            try:
                out["cpu_baseline"]["components"] = cpu_components(tt)
            except (RuntimeError, OSError, ValueError) as e:  # reported, not fatal: the headline baseline stands
                out["cpu_baseline"]["components"] = {"unavailable": str(e)[:200]}
    if dist is not None:
        dist.barrier()
        comm.close()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out))


def _time_program(torch, tt, prog, ins, outs, reps, warm=3, rounds=1):
    """ms per run_device call: `rounds` back-to-back batches of `reps` calls between CUDA
    events on the program's stream, after `warm` untimed calls; the median batch."""
    st = tt.Stream()
    ts = torch.cuda.ExternalStream(st.handle)
    for _ in range(warm):
        prog.run_device(ins, outs, st)
    st.synchronize()
    per_call = []
    for _ in range(rounds):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(ts)
        for _ in range(reps):
            prog.run_device(ins, outs, st)
        e1.record(ts)
        st.synchronize()
        per_call.append(e0.elapsed_time(e1) / reps)
    return float(np.median(per_call))


def components(tt, torch, args, peaks, peak_src):
    """Single-GPU parts of the metric: fused elementwise, reductions, GEMM."""
    res = {}
    hbm = peaks["hbm_gbs"]
    # fused elementwise chain relu(a*b + c)*0.5 - exp(-a); c broadcast along rows
    ew = {}
    for n in (1024, 8192, 16384):
        rng = np.random.default_rng(0)
        g = tt.Graph()
        a, b, c = g.input([n, n]), g.input([n, n]), g.input([1, n])
        y = tt.relu(a * b + c) * 0.5 - tt.exp(-a)
        prog = tt.compile(g, outputs=[y])
        ins = [tt.DeviceBuffer.from_numpy(rng.standard_normal(s).astype(np.float32)) for s in ([n, n], [n, n], [1, n])]
        out = [tt.DeviceBuffer([n, n])]
        # the launch-bound size: 50 untimed calls, then the median of 5 batches of 200
        ms = (_time_program(torch, tt, prog, ins, out, 200, warm=50, rounds=5) if n == 1024
              else _time_program(torch, tt, prog, ins, out, 20))
        nbytes = 3 * n * n * 4 + n * 4
        ew[f"{n}x{n}"] = {"ms": round(ms, 5), "GB/s": round(nbytes / ms / 1e6, 1),
                          "frac_of_measured_hbm": round(nbytes / ms / 1e6 / hbm, 3),
                          "note": ("fits in L2 (126 MB): repeated calls hit L2; median of 5 batches of 200 "
                                   "back-to-back eager calls after 50 untimed") if n == 1024 else "> L2"}
        if n == 1024:
            # launch-bound at this size: 100 calls captured in one CUDA graph, replayed
            st = tt.Stream()
            ts = torch.cuda.ExternalStream(st.handle)
            graph = tt.CudaGraph()
            with graph.capture(st):
                for _ in range(100):
                    prog.run_device(ins, out, st)
            graph.replay(st)
            st.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(ts)
            for _ in range(5):
                graph.replay(st)
            e1.record(ts)
            st.synchronize()
            gms = e0.elapsed_time(e1) / 500
            ew["1024x1024_cuda_graph"] = {"ms": round(gms, 5), "GB/s": round(nbytes / gms / 1e6, 1),
                                          "note": "100 calls per graph, L2-resident"}
            # one call after writing 512 MB elsewhere (L2 flushed): HBM-cold latency
            flush = torch.empty(128 * 1024 * 1024, dtype=torch.float32, device="cuda")
            times = []
            for _ in range(20):
                with torch.cuda.stream(ts):
                    flush.fill_(1.0)
                a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a0.record(ts)
                prog.run_device(ins, out, st)
                a1.record(ts)
                st.synchronize()
                times.append(a0.elapsed_time(a1))
            cms = float(np.median(times))
            ew["1024x1024_l2_flushed"] = {"ms": round(cms, 5), "GB/s": round(nbytes / cms / 1e6, 1),
                                          "note": "median of 20 single calls after a 512 MB write"}
            del flush, graph
        del ins, out, prog
    res["fused_elementwise"] = ew
    # reductions over X [8192, 4096] U(-1,1): sum/mean/max over axis 1, sum over axis 0 of X^T
    rng = np.random.default_rng(1)
    xr = rng.uniform(-1, 1, (8192, 4096)).astype(np.float32)
    red = {}
    for name, fn in (("sum_ax1", lambda x: tt.sum(x, [1])), ("mean_ax1", lambda x: tt.mean(x, [1])),
                     ("max_ax1", lambda x: tt.max(x, [1])), ("sum_ax0_of_T", lambda x: tt.sum(tt.transpose(x, 0, 1), [0]))):
        g = tt.Graph()
        nx = g.input([8192, 4096])
        prog = tt.compile(g, outputs=[fn(nx)])
        ins = [tt.DeviceBuffer.from_numpy(xr)]
        out = [tt.DeviceBuffer([8192])]
        ms = _time_program(torch, tt, prog, ins, out, 50)
        nbytes = 8192 * 4096 * 4 + 8192 * 4
        red[name] = {"ms": round(ms, 5), "GB/s": round(nbytes / ms / 1e6, 1),
                     "frac_of_measured_hbm": round(nbytes / ms / 1e6 / hbm, 3)}
        del ins, out, prog
    res["reductions_8192x4096"] = red
    # GEMM C = A.B, A,B ~ N(0, 1/K)
    gm = {}
    eff = peaks["bf16_tflops"] / 2.0 / 3.0
    for (m, n, k) in ((1024, 1024, 1024), (4096, 4096, 4096), (8192, 8192, 8192), (16384, 1024, 4096)):
        rng = np.random.default_rng(2)
        g = tt.Graph()
        a, b = g.input([m, k]), g.input([k, n])
        prog = tt.compile(g, outputs=[a @ b])
        ins = [tt.DeviceBuffer.from_numpy((rng.standard_normal((m, k)) / np.sqrt(k)).astype(np.float32)),
               tt.DeviceBuffer.from_numpy((rng.standard_normal((k, n)) / np.sqrt(k)).astype(np.float32))]
        out = [tt.DeviceBuffer([m, n])]
        reps = 5 if m * n * k >= 8192 ** 3 else 20
        ms = _time_program(torch, tt, prog, ins, out, reps)
        tf = 2.0 * m * n * k / (ms * 1e-3) / 1e12
        gm[f"{m}x{n}x{k}"] = {"ms": round(ms, 4), "TFLOP/s": round(tf, 2), "frac_of_3xtf32_peak": round(tf / eff, 4)}
        del ins, out, prog
    res["gemm_fp32"] = gm
    res["peaks"] = {"source": peak_src, "hbm_gbs": hbm, "3xtf32_tflops": round(eff, 1)}
    return res


# --------------------------------------------------------------------------------------------
# CPU baseline: the reference itself (oracle/_ref) on the host cores
# --------------------------------------------------------------------------------------------

def _reference_runner(batch):
    """The reference's own data-parallel step (oracle/ref_step.py) over all host cores
    on the headline batch, prepared (graphs built, forward JIT-compiled) outside any
    timing; (runner, None) or (None, why not)."""
    from oracle import ref_step
    if not ref_step.available():
        return None, "oracle/_ref/libttref.so not built (the reference sources were absent at build time)"
    x, t, w = mlp_data(rows=batch)
    return ref_step.ReferenceStep(x, t, w, lr=LR), None


def _reference_sample(runner, steps, wall_s):
    return (f"{steps} full {runner.rows}-row step(s) of the reference itself (oracle/_ref: compiled from its "
            f"sources), each = {runner.P} processes x {runner.rows // runner.P} rows running the compiled AVX2 "
            f"forward (tt.compile mode avx2, optimize=True) + eager tt.gradients, shard gradients summed and "
            f"SGD (lr/{runner.P} on the sum) applied in the parent; graph build and g++ JIT excluded; "
            f"{wall_s:.1f} s timed")


def cpu_baseline(batch):
    """One real step of the reference at the headline batch on the host cores (rank 0,
    N=1): no extrapolation from smaller shards."""
    runner, why = _reference_runner(batch)
    if runner is None:
        return {"value": None, "unit": "step/s", "cores": 0, "kind": "reference", "sample": why}
    try:
        s = runner.step()
        info = {"value": round(1.0 / s, 6), "unit": "step/s", "cores": runner.P, "kind": "reference",
                "sample": _reference_sample(runner, 1, s), "shard_s_max": round(runner.last["shard_s_max"], 2),
                "reduce_update_s": round(runner.last["reduce_update_s"], 2)}
    finally:
        runner.close()
    return info


def cpu_components(tt):
    """The reference's compiled AVX2 code (oracle/_ref, the reference built from its
    sources; single-threaded as shipped, one host core) on the single-GPU component
    workloads, seconds per Executor::run with the JIT compile excluded: the CPU numbers
    beside `components`."""
    from oracle import oracle as O
    if not O.reference_available():
        return {"unavailable": "oracle/_ref/libttref.so not built"}
    R = O.Reference()
    rng = np.random.default_rng(0)
    res = {"kind": "reference", "cores": 1, "mode": "compiled avx2 (avx2_fma for the GEMM), optimize=False"}
    g = tt.Graph()  # the fused chain at [1024, 1024] with sigmoid(a) for exp(-a): the reference has no exp
    a, b, c = g.input([1024, 1024]), g.input([1024, 1024]), g.input([1, 1024])
    g.mark_output(tt.relu(a * b + c) * 0.5 - tt.sigmoid(a))
    feed = {a: rng.standard_normal((1024, 1024)).astype(np.float32),
            b: rng.standard_normal((1024, 1024)).astype(np.float32), c: rng.standard_normal((1, 1024)).astype(np.float32)}
    t = R.time_runs(g, feed, mode="avx2", reps=5)
    res["fused_elementwise_1024x1024_sigmoid"] = {"ms": round(t * 1e3, 3), "GB/s": round((3 * 1024 * 1024 * 4 + 4096) / t / 1e9, 2)}
    g = tt.Graph()  # sum over axis 1 of [8192, 4096]
    x = g.input([8192, 4096])
    g.mark_output(tt.sum(x, [1]))
    t = R.time_runs(g, {x: rng.uniform(-1, 1, (8192, 4096)).astype(np.float32)}, mode="avx2", reps=3)
    res["reduce_sum_ax1_8192x4096"] = {"ms": round(t * 1e3, 2), "GB/s": round((8192 * 4096 * 4 + 8192 * 4) / t / 1e9, 2)}
    g = tt.Graph()  # GEMM 1024^3
    a, b = g.input([1024, 1024]), g.input([1024, 1024])
    g.mark_output(a @ b)
    feed = {a: rng.standard_normal((1024, 1024)).astype(np.float32),
            b: rng.standard_normal((1024, 1024)).astype(np.float32)}
    t = R.time_runs(g, feed, mode="avx2_fma", reps=3)
    res["gemm_1024x1024x1024"] = {"ms": round(t * 1e3, 1), "TFLOP/s": round(2 * 1024 ** 3 / t / 1e12, 4)}
    return res


# Timed full reference steps stop once this much wall time is spent (at least one step),
# so `--impl reference` ends within a few minutes whatever --steps asks for; the line
# reports the steps actually timed.
REFERENCE_TIME_BUDGET_S = 120.0


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    runner, why = _reference_runner(args.batch)
    if runner is None:
        print(json.dumps({"impl": "reference", "unavailable": why}))
        return
    try:
        # No untimed full steps: preparing the runner already built the graphs and compiled
        # the forward, and the reference allocates afresh in every call, so its first step
        # costs what later ones do (measured: 90 and 95 s for 2048-row shards on 8 cores).
        warm = 0
        times = []
        while len(times) < args.steps and (not times or sum(times) < REFERENCE_TIME_BUDGET_S):
            times.append(runner.step())
        last = dict(runner.last)
        P = runner.P
        sample = _reference_sample(runner, len(times), sum(times))
    finally:
        runner.close()
    s = float(np.mean(times))
    v = 1.0 / s
    out = {
        "impl": "reference",
        "metric": HEADLINE_METRIC.format(args.batch),
        "value": round(v, 6),
        "unit": "step/s",
        "n_gpus": args.gpus,
        "steps": len(times),
        "warmup": warm,
        "ms_per_step": round(1000.0 * s, 1),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic: X,T ~ N(0,1) seed 4; Xavier-uniform weights seed 4",
        "config": headline_config(args.batch, world),
        "note": (f"the reference is CPU-only: {P} host processes run it; steps/warmup are the full steps actually "
                 f"run ({REFERENCE_TIME_BUDGET_S:.0f} s budget for timed steps)"),
        "cpu_baseline": {"value": round(v, 6), "unit": "step/s", "cores": P, "kind": "reference", "sample": sample,
                         "step_s": [round(t, 2) for t in times], "shard_s_max_last": round(last["shard_s_max"], 2)},
        "e2e": {"value": round(v, 6), "unit": "step/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-components", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-early-update", action="store_true",
                    help="update the parameters after the whole exchange instead of as each one is ready")
    ap.add_argument("--workload", default="mlp", choices=["mlp", "gemm", "elementwise", "reduce"],
                    help="mlp: the headline step; the others time one compiled program (profiling cases)")
    ap.add_argument("--size", default=None, help="gemm: M,N,K; elementwise: n (an n x n chain); reduce: R,C")
    ap.add_argument("--batch", type=int, default=GLOBAL_BATCH,
                    help="mlp: global batch (the headline is 32768; smaller values are profiling cases)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload != "mlp":
        run_single(args)
    else:
        run_b200(args)


def run_single(args):
    """One compiled program of a single-GPU component, timed with CUDA events over
    `steps` runs on device-resident inputs (inputs > L2 for the default sizes)."""
    import torch

    import tinytensor_b200 as tt

    tt.device_init(0)
    rng = np.random.default_rng(0)
    g = tt.Graph()
    if args.workload == "gemm":
        m, n, k = (int(v) for v in (args.size or "4096,4096,4096").split(","))
        a, b = g.input([m, k]), g.input([k, n])
        outs = [a @ b]
        feeds = [(rng.standard_normal((m, k)) / np.sqrt(k)).astype(np.float32),
                 (rng.standard_normal((k, n)) / np.sqrt(k)).astype(np.float32)]
        work, unit, metric = 2.0 * m * n * k / 1e12, "TFLOP/s", f"fp32 GEMM TFLOP/s ({m}x{n}x{k}, 3xTF32)"
    elif args.workload == "elementwise":
        n = int(args.size or 8192)
        a, b, c = g.input([n, n]), g.input([n, n]), g.input([1, n])
        outs = [tt.relu(a * b + c) * 0.5 - tt.exp(-a)]
        feeds = [rng.standard_normal(s).astype(np.float32) for s in ([n, n], [n, n], [1, n])]
        work, unit, metric = (3 * n * n * 4 + n * 4) / 1e9, "GB/s", f"fused elementwise GB/s ({n}x{n})"
    else:
        r, c_ = (int(v) for v in (args.size or "8192,4096").split(","))
        x = g.input([r, c_])
        outs = [tt.sum(x, [1]), tt.mean(x, [1]), tt.max(x, [1]), tt.sum(tt.transpose(x, 0, 1), [0])]
        feeds = [rng.uniform(-1, 1, (r, c_)).astype(np.float32)]
        work, unit, metric = 4 * (r * c_ * 4 + r * 4) / 1e9, "GB/s", f"reductions GB/s ({r}x{c_}, 4 reductions)"
    prog = tt.compile(g, outputs=outs)
    ins = [tt.DeviceBuffer.from_numpy(f) for f in feeds]
    res = [tt.DeviceBuffer(s) for s in prog.output_shapes]
    ms = _time_program(torch, tt, prog, ins, res, args.steps, warm=args.warmup)
    print(json.dumps({"metric": metric, "value": round(work / (ms * 1e-3), 2), "unit": unit, "n_gpus": 1,
                      "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
                      "higher_is_better": True, "config": {"workload": args.workload, "size": args.size}}))


if __name__ == "__main__":
    main()
