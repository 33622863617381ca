#!/usr/bin/env python
"""FWLoss forward+backward throughput on B200 (rows/s, HBM roofline).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config cfgX] [--weak]

Default workload: cfg2 of the reference's benchmark set -- B=4096 rows x
C=32000 classes, fp32 Student-t(3)*2 logits, int64 labels (seeded synthetic
data, fwloss_b200.workloads).  A step is one fused forward+backward of the
whole batch (threshold search, per-row loss, dense gradient) plus the
deterministic loss reduction.  With N > 1 ranks (torchrun, one per GPU) the
batch's B rows are split into contiguous row blocks (strong scaling, the
metric's fixed B; --weak gives every rank B rows of its own), every rank runs
the same step on its block with the gradient scaled by 1/B, and the global
mean is combined per step by the cross-GPU loss sum: one kernel that reduces
the rank's losses and exchanges the partials over NVLink peer memory
(fw_loss_allreduce; the loss reduction + a scalar NCCL all-reduce where the
GPUs lack peer access).  Each step's loss path runs on a side stream after
that step's kernel, under the next step's kernel: nothing of the next step
reads the loss.  The K timed steps are captured once in a CUDA graph, and
every step's loss path is complete before the timed region closes.

Printed JSON line (rank 0):
  value     rows/s of the whole job, inputs resident in HBM, device-timed with
            CUDA events over exactly K steps (barrier + synchronize on both
            sides, max over ranks).
  e2e       same metric through the public API -- familywise_loss on one GPU,
            fwloss_b200.distributed.sharded_familywise_loss on N -- with the
            logits and labels copied from pinned host memory every step and
            the loss read back (host<->device copies inside the timed region).
  roofline  the fused kernel alone: algorithmic bytes per launch
            (B * (8C + 12): read logits, write gradient, label, loss) over its
            CUDA-event average duration, against the measured HBM copy peak.
  forward_only  the same for the forward-only kernel (B * (4C + 12) bytes).
  weak      (N > 1) the weak-scaling figure: every rank B rows.
  cpu_baseline  the reference's own CPU implementation (src/cpu/fw_cpu.cpp,
            compiled by oracle/build.py) on this host's cores, on a bounded
            sample of the same workload (rank 0, N = 1 only).
--impl reference runs only that CPU implementation (the reference arm).
"""
import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.join(REPO, "fast-familywise-loss_b200")
for _p in (REPO, PKG_ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "FWLoss fwd+bwd rows/s & HBM GB/s vs peak, B=4096 C=32000, 1/2/4/8 B200"
UNIT = "rows/s"
FALLBACK_HBM_GBS = 6650.0
L2_BYTES = 126 * 1000 * 1000


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-cuda"],
                   help="reference: the reference's CPU implementation (the reference arm); reference-cuda: "
                        "the reference's own CUDA extension built for sm_100a, timed on the GPU beside ours")
    p.add_argument("--config", default="cfg2",
                   help="cfg0..cfg4, or gaussBxC (N(0,1) logits, the reference CUDA benchmark's workload)")
    p.add_argument("--e2e-steps", type=int, default=0, help="0: min(steps, 10)")
    p.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU-baseline sample budget")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-graph", action="store_true", help="launch steps eagerly")
    p.add_argument("--weak", action="store_true",
                   help="rows mode: give every rank B rows of its own (weak scaling) instead of splitting the "
                        "configuration's B rows across the ranks (strong scaling, the default; the weak figure "
                        "is also reported under 'weak' at N > 1)")
    p.add_argument("--mode", default="rows", choices=["rows", "class-sharded", "lm-head"],
                   help="rows: rows sharded across GPUs (default); class-sharded: every GPU holds a "
                        "column shard of every row (vocabulary-parallel), cfg4 shape; lm-head: "
                        "logits = hidden @ weight^T (B=8192, D=4096, C=128256, bf16) with the chunked "
                        "forward and sparse backward, next to the dense path")
    p.add_argument("--shard-k", type=int, default=32, help="class-sharded: support entries per shard summary")
    p.add_argument("--lm-forms", default="staged,fused,dense",
                   help="lm-head mode: comma list of the forms to time (staged, fused, dense)")
    p.add_argument("--lm-shape", default="8192,4096,128256",
                   help="lm-head mode: B,D,C (rows, hidden size, classes)")
    p.add_argument("--dtype", default="f32", choices=["f32", "bf16", "f16", "f64"],
                   help="logits/gradient element type (the metric is defined on f32)")
    return p.parse_args()


def bench_config(name, world, strong=True, esize=4):
    """The `config` object of the bench line, identical in both arms for the
    same (configuration, N, scaling): strong scaling splits the
    configuration's B rows across the N ranks, weak scaling gives every rank
    B rows."""
    from fwloss_b200 import workloads

    B_cfg, C = workloads.shape_of(name)
    Bg = B_cfg if (strong or world == 1) else B_cfg * world
    rows = -(-B_cfg // world) if (strong and world > 1) else B_cfg  # largest rank block
    kinds = {"cfg0": "N(0,1)", "cfg1": "N(0,1) +4 at label", "cfg2": "Student-t(3) x2",
             "cfg3": "8 levels + 1% signed zeros", "cfg4": "N(0,1) +8 at a non-label class"}
    per = rows * C * esize
    return {
        "workload": f"{name}: FWLoss fwd+bwd, B={B_cfg} x C={C}, "
                    f"{dict([(8, 'fp64'), (4, 'fp32'), (2, '16-bit')])[esize]} logits "
                    f"{kinds.get(name, 'N(0,1)' if name.startswith('gauss') else '')}, int64 labels",
        "rows_per_gpu": rows, "classes": C, "global_batch": Bg,
        "parallelism": f"row-sharded dp{world}" + (" + cross-GPU scalar loss sum" if world > 1 else ""),
        "l2": f"inputs {per / 1e6:.1f} MB logits + {per / 1e6:.1f} MB gradient per step and GPU"
              + (" (> 3x the 126 MB L2, no flush needed)" if per > 3 * L2_BYTES else
                 f" (rotating over {min(64, -(-3 * L2_BYTES // per))} input copies)"),
    }


def measured_peak():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def profile_traffic(name):
    """DRAM bytes per launch of the fused kernel from the committed ncu summary."""
    try:
        with open(os.path.join(REPO, "profiles", "traffic.json")) as f:
            return json.load(f).get(name)
    except (OSError, ValueError):
        return None


def rows_traffic(t, rows, profiled_rows):
    """The profiled launch's DRAM bytes scaled to a launch of `rows` rows (a
    strong-scaling rank's share): the fused kernel's traffic is proportional
    to the rows it processes."""
    if t is None or rows == profiled_rows:
        return t
    f = rows / profiled_rows
    return dict(t, bytes=int(t["bytes"] * f), dram_read=int(t["dram_read"] * f), dram_write=int(t["dram_write"] * f),
                note=f"scaled from the profiled {profiled_rows}-row launch to this rank's {rows} rows")


class Clocks:
    """nvidia-smi sampler (200 ms) around the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, phys_index):
        self.idx = phys_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.idx), "-lms", "200", "-f", self.path],
                                         stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        sm, mx, reasons = [], [], set()
        try:
            lines = open(self.path).read().strip().splitlines()
        except OSError:
            lines = []
        for ln in lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        try:
            os.unlink(self.path)
        except OSError:
            pass
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_baseline(name, B, C, seconds, f64=False):
    """The reference CPU implementation (or the C restatement) on a bounded
    sample of the workload; returns the cpu_baseline object.  f64: float64
    logits (the reference's float64 branch; there is no float64 port)."""
    import torch
    from fwloss_b200 import workloads

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    rows = min(B, 1024)
    z, y = workloads.make(name, rows=rows)
    if f64:
        z = z.double()
    try:
        from oracle import ref_cpu

        mod = ref_cpu.ref_module()
        kind = "reference"

        def step():
            Z = z.clone().requires_grad_(True)
            mod.familywise_loss(Z, y, 1).backward()
    except ImportError:
        from oracle import ref_cpu

        kind = "port"
        zn, yn = z.numpy(), y.numpy()

        def step():
            ref_cpu.c_solve(zn, yn, threads)
    step()
    n, t0 = 0, time.perf_counter()
    while True:
        step()
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return {"value": rows * n / el, "unit": UNIT, "cores": threads, "kind": kind,
            "sample": f"{rows} rows of {name} (C={C}) per call, {n} calls in {el:.1f} s, "
                      f"familywise_loss(..., mean).backward()" if kind == "reference" else
                      f"{rows} rows of {name} per call, {n} calls in {el:.1f} s (C restatement)"}


def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(a.gpus)))
    if rank != 0:
        return 0
    import torch
    from fwloss_b200 import workloads

    B, C = workloads.shape_of(a.config)
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    from oracle import ref_cpu

    mod = ref_cpu.ref_module()
    z, y = workloads.make(a.config)

    def step(zz, yy):
        Z = zz.clone().requires_grad_(True)
        mod.familywise_loss(Z, yy, 1).backward()

    # bounded sample: shrink the rows per step if one full step is slow
    t = time.perf_counter()
    step(z, y)
    one = time.perf_counter() - t
    rows = B if one * (a.steps + a.warmup) < 120 else max(64, int(B * 120 / (one * (a.steps + a.warmup))))
    zs, ys = z[:rows].contiguous(), y[:rows].contiguous()
    for _ in range(a.warmup):
        step(zs, ys)
    t = time.perf_counter()
    for _ in range(a.steps):
        step(zs, ys)
    el = time.perf_counter() - t
    value = rows * a.steps / el
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": 1e3 * el / a.steps,
        "higher_is_better": True, "scaling": "strong" if not a.weak else "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic", "config": bench_config(a.config, world, not a.weak),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "reference",
                         "sample": f"{rows} of the {B} rows of {a.config} per step (reference "
                                   f"src/cpu/fw_cpu.cpp, familywise_loss mean + backward, simd={mod.simd()}; "
                                   f"host cores only, the same whatever the GPU count)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_reference_cuda(a):
    """The reference's own CUDA path (src/cuda/fw_radix_argmax.cu, built for
    sm_100a by oracle/build.py) on the same workload, one GPU, inputs
    resident in HBM, dispatched as its benchmark does
    (CE_FW_perf.py:76-88); CUDA events over exactly K steps.  Prints a line
    with impl "reference-cuda" (rank 0 only)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    import torch

    from fwloss_b200 import workloads
    from oracle import ref_cuda

    if not ref_cuda.available():
        print(json.dumps({"impl": "reference-cuda", "unavailable": "reference CUDA extension not built "
                                                                    "(oracle/build.py needs the reference checkout)"}))
        return 0
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, C = workloads.shape_of(a.config)
    z_cpu, y_cpu = workloads.make(a.config)
    copies = 1 if B * C * 4 > 3 * L2_BYTES else min(64, -(-3 * L2_BYTES // (B * C * 4)))
    zs = [z_cpu.to(dev) for _ in range(copies)]
    y = y_cpu.to(dev)
    for i in range(max(3, a.warmup)):
        ref_cuda.forward_backward(zs[i % copies], y)
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(a.steps):
        ref_cuda.forward_backward(zs[i % copies], y)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / a.steps
    alg = B * (8 * C + 12)
    peak, peak_kind = measured_peak()
    print(json.dumps({
        "impl": "reference-cuda", "metric": METRIC, "value": B / (ms / 1e3), "unit": UNIT, "n_gpus": 1,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": bench_config(a.config, 1),
        "path": "fw_forward_small + fw_backward_small" if C < 10000 else "fw_forward + fw_backward",
        "hbm": {"alg_bytes_per_step": alg, "achieved_gbs": alg / (ms / 1e3) / 1e9,
                "frac": alg / (ms / 1e3) / 1e9 / peak, "peak": peak, "peak_kind": peak_kind},
    }), flush=True)
    return 0


def _rank_inputs(a, world, rank, dev, strong):
    """(z_local, y_local) on the device and (global rows, rows of the
    configuration).  Strong scaling: rank 0 draws the configuration's whole
    batch on the host and broadcasts it over NCCL; every rank keeps its
    contiguous row block (fwloss_b200.distributed.shard_rows).  Weak scaling:
    every rank draws a batch of its own (workloads.make_rank)."""
    import torch
    import torch.distributed as dist

    from fwloss_b200 import workloads
    from fwloss_b200.distributed import shard_rows

    B_cfg, C = workloads.shape_of(a.config)
    if world == 1 or not strong:
        z, y = workloads.make_rank(a.config, rank)
        return z.to(dev), y.to(dev), B_cfg * world, B_cfg
    if rank == 0:
        z, y = workloads.make(a.config)
        z, y = z.to(dev), y.to(dev)
    else:
        z = torch.empty((B_cfg, C), dtype=torch.float32, device=dev)
        y = torch.empty((B_cfg,), dtype=torch.int64, device=dev)
    dist.broadcast(z, 0)
    dist.broadcast(y, 0)
    lo, hi = shard_rows(B_cfg, rank, world)
    zl, yl = z[lo:hi].clone(), y[lo:hi].clone()
    del z, y
    torch.cuda.empty_cache()
    return zl, yl, B_cfg, B_cfg


def _graph_of(fn, dev, warm_fn=None):
    """fn() captured once in a CUDA graph, after warm_fn() (or fn()) ran
    eagerly on the capture stream; returns the graph.  Raises RuntimeError
    when capture is not possible."""
    import torch

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        (warm_fn or fn)()
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize(dev)
    return g


def run_ours(a):
    import torch
    import torch.distributed as dist

    from fwloss_b200 import familywise_loss, workloads
    from fwloss_b200._native import ext
    from fwloss_b200.distributed import sharded_familywise_loss

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if a.gpus != world and world > 1:
        print(f"warning: --gpus {a.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    strong = not a.weak
    B_cfg, C = workloads.shape_of(a.config)
    fw = ext()
    z_dev, y, Bg, _ = _rank_inputs(a, world, rank, dev, strong)
    B = z_dev.shape[0]
    tdt = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16, "f64": torch.float64}[a.dtype]
    esize = torch.tensor([], dtype=tdt).element_size()
    z_dev = z_dev.to(tdt)
    # inputs larger than L2 (126 MB): small batches rotate over enough copies
    # that 3x the L2 size is touched between two uses of one copy
    copies = 1 if B * C * esize > 3 * L2_BYTES else min(64, -(-3 * L2_BYTES // (B * C * esize)))
    zs = [z_dev] + [z_dev.clone() for _ in range(copies - 1)]
    scale = 1.0 / Bg
    stream = torch.cuda.current_stream(dev)

    side = torch.cuda.Stream(dev)  # the scalar loss path of every step
    # N > 1: the cross-GPU loss sum as one kernel over peer memory (built
    # collectively here, before any capture); None without peer access
    from fwloss_b200.distributed import loss_exchange
    exchange = loss_exchange(None, dev) if world > 1 else None

    def steps(n, inputs=zs, rows_y=y, sc=scale, forward_only=False):
        """n steps: the fused forward+backward (or the forward-only kernel) on
        the launching stream; each step's loss path -- the deterministic loss
        reduction, with N > 1 ranks fused with the cross-GPU sum -- on a side
        stream after that step's kernel, so that it runs under the next
        step's kernel (nothing of the next step reads the loss).  The side
        stream is joined before returning: all n steps are complete."""
        main = torch.cuda.current_stream(dev)
        losses = []  # kept alive until the side stream has read them
        for i in range(n):
            zi = inputs[i % len(inputs)]
            if forward_only:
                _, loss, _ = fw.forward_rows(zi, rows_y, None)
            else:
                _, _, loss, _ = fw.fused_fwd_bwd(zi, rows_y, sc)
            losses.append(loss)
            side.wait_stream(main)
            with torch.cuda.stream(side):
                if exchange is not None:
                    exchange.reduce(loss, sc)
                else:
                    s = fw.loss_reduce(loss, sc)
                    if world > 1:
                        dist.all_reduce(s)
        main.wait_stream(side)
        del losses

    def kernels(n, inputs=zs, rows_y=y, forward_only=False):
        for i in range(n):
            if forward_only:
                fw.forward_rows(inputs[i % len(inputs)], rows_y, None)
            else:
                fw.fused_fwd_bwd(inputs[i % len(inputs)], rows_y, scale)

    # The K timed steps are captured once in a CUDA graph (the same kernels and
    # NCCL call, without Python launch overhead); --no-graph runs them eagerly.
    warm = max(3, a.warmup)
    launch_mode = "eager"
    run_steps = lambda: steps(a.steps)  # noqa: E731
    g_steps = None
    if not a.no_graph:
        try:
            g_steps = _graph_of(lambda: steps(a.steps), dev, warm_fn=lambda: steps(warm))
            run_steps, launch_mode = g_steps.replay, "one CUDA graph of the K timed steps"
        except RuntimeError as ex:  # capture not possible here: time eagerly, say so
            launch_mode = f"eager (graph capture failed: {str(ex)[:120]})"
            torch.cuda.synchronize(dev)
    else:
        steps(warm)
    run_steps()  # untimed warm replay
    torch.cuda.synchronize(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(ms):
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(fn):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize(dev)
        e0.record(stream)
        fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        return max_over_ranks(e0.elapsed_time(e1))

    phys = local
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        try:
            phys = int(vis.split(",")[local])
        except (ValueError, IndexError):
            phys = local
    with Clocks(phys) as clk:
        ms = timed(run_steps)
    clocks = clk.summary()
    value = Bg * a.steps / (ms / 1e3)

    # roofline: the fused kernel alone, K launches back to back (one graph)
    def kernel_ms(forward_only):
        fn = lambda: kernels(a.steps, forward_only=forward_only)  # noqa: E731
        if not a.no_graph:
            try:
                fn = _graph_of(fn, dev, warm_fn=lambda: kernels(3, forward_only=forward_only)).replay
            except RuntimeError:
                pass
        fn()
        torch.cuda.synchronize(dev)
        kd0, kd1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        kd0.record(stream)
        fn()
        kd1.record(stream)
        torch.cuda.synchronize(dev)
        return kd0.elapsed_time(kd1) / a.steps

    k_ms = kernel_ms(False)
    tail = 16 if esize == 8 else 12  # label + loss (fp64 loss for fp64 logits)
    alg_bytes = B * (2 * esize * C + tail)
    achieved = alg_bytes / (k_ms / 1e3) / 1e9
    peak, peak_kind = measured_peak()

    # forward only (no gradient): the kernel a no_grad / evaluation call runs
    f_ms = kernel_ms(True)
    f_bytes = B * (esize * C + tail)
    fwd = {"kernel_ms": f_ms, "alg_bytes_per_launch": f_bytes, "achieved": f_bytes / (f_ms / 1e3) / 1e9,
           "frac": f_bytes / (f_ms / 1e3) / 1e9 / peak, "unit": "GB/s",
           "rows_per_s": Bg / (f_ms / 1e3) if world == 1 else None,
           "what": "fw_forward_rows: H, loss and kappa, logits read once, no gradient written"}

    # weak scaling (N > 1): every rank a full batch of the configuration's
    # B rows (its own row block tiled up to B rows), same step
    weak = None
    if world > 1 and strong:
        reps = -(-B_cfg // B)
        zw = zs[0].repeat(reps, 1)[:B_cfg].contiguous()
        yw = y.repeat(reps)[:B_cfg].contiguous()
        fnw = lambda: steps(a.steps, inputs=[zw], rows_y=yw, sc=1.0 / (B_cfg * world))  # noqa: E731
        if launch_mode.startswith("one CUDA graph"):
            fnw = _graph_of(fnw, dev, warm_fn=lambda: steps(3, inputs=[zw], rows_y=yw)).replay
        fnw()
        torch.cuda.synchronize(dev)
        w_ms = timed(fnw)
        weak = {"value": B_cfg * world * a.steps / (w_ms / 1e3), "unit": UNIT, "ms_per_step": w_ms / a.steps,
                "rows_per_gpu": B_cfg, "global_batch": B_cfg * world,
                "what": "weak scaling: every rank runs the configuration's full batch size"}
        del fnw, zw, yw  # the graph (it holds NCCL calls) and its inputs
        torch.cuda.synchronize(dev)

    # e2e: the public API with host buffers; every step copies this rank's
    # logits and labels from pinned host memory and reads the loss back.
    # One rank: familywise_loss(mean).backward(); N > 1:
    # sharded_familywise_loss(rows, labels, global batch).backward().
    ne = a.e2e_steps or min(a.steps, 10)
    zh = zs[0].cpu().pin_memory()
    yh = y.cpu().pin_memory()
    zd = torch.empty_like(zs[0]).requires_grad_(True)
    yd = torch.empty_like(y)
    lh = torch.empty(ne + a.warmup, dtype=torch.float32).pin_memory()

    def e2e_step(i):
        with torch.no_grad():
            zd.copy_(zh, non_blocking=True)
            yd.copy_(yh, non_blocking=True)
        zd.grad = None
        if world > 1:
            loss = sharded_familywise_loss(zd, yd, Bg)
        else:
            loss = familywise_loss(zd, yd, reduction="mean")
        loss.backward()
        lh[i:i + 1].copy_(loss.detach().reshape(1).float(), non_blocking=True)

    for i in range(min(2, a.warmup)):
        e2e_step(i)
    torch.cuda.synchronize(dev)

    def e2e_loop():
        for i in range(ne):
            e2e_step(a.warmup + i)

    e_ms = timed(e2e_loop)
    e2e = {"value": Bg * ne / (e_ms / 1e3), "unit": UNIT,
           "h2d_bytes_per_step": int(Bg * C * esize + Bg * 8), "d2h_bytes_per_step": 4 * world,
           "ms_per_step": e_ms / ne,
           "api": ("fwloss_b200.distributed.sharded_familywise_loss(rows, labels, global_batch).backward()"
                   if world > 1 else "fwloss_b200.familywise_loss(mean).backward()"),
           "bytes": "summed over the ranks"}

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        try:
            cpu = cpu_baseline(a.config, B, C, a.cpu_seconds, f64=a.dtype == "f64")
        except Exception as ex:  # report, do not fail the GPU measurement
            cpu = {"value": None, "unit": UNIT, "cores": os.cpu_count(), "kind": "unavailable",
                   "sample": f"failed: {ex!r}"[:200]}

    if rank == 0:
        launches_per_step = 2  # fused kernel + loss reduction (with N > 1: + the cross-GPU sum, same kernel)
        traffic = rows_traffic(profile_traffic(a.config if a.dtype == "f32" else f"{a.config}_{a.dtype}"), B,
                               B_cfg)
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": ms / a.steps, "higher_is_better": True,
            "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": a.dtype,
            "data": "synthetic",
            "config": bench_config(a.config, world, strong, esize),
            "launch": launch_mode,
            "hbm_gbs": alg_bytes * a.steps / (ms / 1e3) / 1e9,
            "roofline": {"bound": "hbm", "kernel": ("fw_f64_rows_kernel" if esize == 8 else
                                                    "fw_stream_rows_kernel" if C > 2048 else "fw_warp_rows_kernel"),
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": peak_kind, "traffic": traffic,
                         "alg_bytes_per_launch": alg_bytes, "kernel_ms": k_ms, "rows_per_launch": B},
            "forward_only": fwd,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches_per_step * a.steps,
            "clocks": clocks,
        }
        if weak is not None:
            line["weak"] = weak
        if world > 1:
            line["loss_sum"] = ("fw_loss_allreduce (loss reduction + NVLink peer-memory exchange, one kernel)"
                                if exchange is not None else "fw_loss_reduce + NCCL all-reduce")
        print(json.dumps(line), flush=True)
    run_steps = g_steps = None  # graphs holding NCCL calls go before the process group
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_class_sharded(a):
    """cfg4-shaped rows (B=8192, C=128256) whose classes are split evenly across
    the ranks; strong scaling (the whole job is one batch).  The logits are
    drawn on the GPU from one seeded generator (identical on every rank, each
    rank keeps its columns) with the cfg4 recipe."""
    import torch
    import torch.distributed as dist

    from fwloss_b200._native import ext
    from fwloss_b200.sharded import even_col_start, scan_phase, sharded_loss_step

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    B, C = 8192, 128256
    g = torch.Generator(device=dev).manual_seed(4)
    z = torch.randn(B, C, generator=g, device=dev)
    y = torch.randint(0, C, (B,), generator=g, device=dev)
    b = (y + torch.randint(1, C, (B,), generator=g, device=dev)) % C
    z[torch.arange(B, device=dev), b] += 8.0
    cs = even_col_start(C, world)
    zl = z[:, cs[rank]:cs[rank + 1]].contiguous()
    del z
    torch.cuda.empty_cache()
    scale = 1.0 / B
    fw = ext()

    def all_gather(x):
        if world == 1:
            return x.unsqueeze(0)
        out = torch.empty((world,) + tuple(x.shape), dtype=x.dtype, device=dev)
        dist.all_gather_into_tensor(out, x.contiguous())
        return out

    def all_reduce(t):
        if world > 1:
            dist.all_reduce(t)
        return t

    def step():
        return sharded_loss_step(zl, y, cs, rank, scale, all_gather, all_reduce, a.shard_k)[1]

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(a.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    # the local scan kernel alone
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    k0.record(stream)
    for _ in range(a.steps):
        scan_phase(zl, a.shard_k)
    k1.record(stream)
    torch.cuda.synchronize(dev)
    k_ms = k0.elapsed_time(k1) / a.steps
    Cl = cs[rank + 1] - cs[rank]
    alg = B * (8 * Cl + 4 * (4 + a.shard_k) + 4 * a.shard_k)
    peak, peak_kind = measured_peak()
    if rank == 0:
        print(json.dumps({
            "metric": "FWLoss fwd+bwd rows/s, class-sharded rows (vocabulary-parallel)", "value": B * a.steps / (ms / 1e3),
            "unit": UNIT, "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms / a.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (cfg4 recipe, drawn on the GPU)",
            "config": {"workload": f"B={B} x C={C}, classes split over {world} GPUs ({Cl} per GPU), K={a.shard_k}",
                       "l2": "logits shard > L2 per GPU" if B * Cl * 4 > 3 * L2_BYTES else "logits shard < 3x L2"},
            "roofline": {"bound": "hbm", "kernel": "shard scan (fused kernel, kOutShard)", "kernel_ms": k_ms,
                         "achieved": alg / (k_ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": alg / (k_ms / 1e3) / 1e9 / peak, "peak_kind": peak_kind},
            "gpu_launches": 4 * a.steps,
        }), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_lm_head(a):
    """LM head + FW loss, fwd+bwd, one GPU: B=8192 rows, D=4096, C=128256
    classes (cfg4's shape), bf16 hidden/weight.  Ours: logits chunk by chunk
    (cuBLAS GEMM, fp32 out) reduced to summaries by the fused kernel, sparse
    backward.  Dense: the bf16 GEMM's logits materialised, the fused FW kernel,
    and autograd through the GEMM (two dense bf16 backward GEMMs)."""
    import torch

    from fwloss_b200 import familywise_loss
    from fwloss_b200.lm_head import fw_lm_head_loss

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, D, C = (int(v) for v in a.lm_shape.split(","))
    g = torch.Generator(device=dev).manual_seed(4)
    hidden = (torch.randn(B, D, generator=g, device=dev) / D ** 0.5 * 4).to(torch.bfloat16).requires_grad_(True)
    weight = torch.randn(C, D, generator=g, device=dev).to(torch.bfloat16).requires_grad_(True)
    target = torch.randint(0, C, (B,), generator=g, device=dev)

    def ours(impl):
        def step():
            hidden.grad = weight.grad = None
            fw_lm_head_loss(hidden, weight, target, impl=impl).backward()
        return step

    def ours_fwd(impl):
        def step():
            with torch.no_grad():
                fw_lm_head_loss(hidden, weight, target, impl=impl)
        return step

    def dense():
        hidden.grad = weight.grad = None
        z = (hidden @ weight.t()).float()  # bf16 GEMM, logits materialised
        familywise_loss(z, target).backward()

    def timed(fn, steps):
        for _ in range(a.warmup):
            fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / steps

    want = [f.strip() for f in a.lm_forms.split(",") if f.strip()]
    impls = [i for i in ("fused", "staged") if i in want]
    # The GEMMs run under the 1 kW power cap, so the clock drifts over a run:
    # the forms are timed alternately, twice each, and the two runs averaged.
    runs = {i: {"ms_per_step": [], "forward_ms": []} for i in impls}
    for _ in range(2):
        for impl in impls:
            runs[impl]["ms_per_step"].append(timed(ours(impl), a.steps))
            runs[impl]["forward_ms"].append(timed(ours_fwd(impl), a.steps))
    forms = {i: {k: statistics.mean(v) for k, v in r.items()} for i, r in runs.items()}
    best = min(forms, key=lambda k: forms[k]["ms_per_step"])
    ms = forms[best]["ms_per_step"]
    ms_dense = timed(dense, max(1, a.steps // 2)) if "dense" in want else float("nan")
    gemm_tflop = 2.0 * B * D * C / 1e12
    for f in forms.values():
        f["forward_gemm_tflops"] = gemm_tflop / (f["forward_ms"] / 1e3)
    print(json.dumps({
        "metric": f"LM head + FWLoss fwd+bwd rows/s (B={B}, D={D}, C={C}, bf16)",
        "value": B / (ms / 1e3), "unit": UNIT, "n_gpus": 1, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": {"workload": f"hidden [{B}, {D}] x weight [{C}, {D}]^T -> FW loss",
                                        "forward_gemm_tflop": gemm_tflop},
        "dense_path": {"ms_per_step": ms_dense, "value": B / (ms_dense / 1e3),
                       "what": "bf16 GEMM, logits materialised (fp32), fused FW kernel, dense bf16 GEMM backward"},
        "speedup_vs_dense": ms_dense / ms,
        "forms": forms, "best_form": best,
        "forms_what": {"staged": "cuBLAS GEMM per column chunk (fp32 logits) + summary scans",
                       "fused": "tcgen05 GEMM with the chunk summaries in its epilogue (no logits stored)"},
    }), flush=True)
    return 0


def run_lm_head_vocab_parallel(a):
    """LM head + FW loss, fwd+bwd, vocabulary-parallel over N GPUs (torchrun):
    every rank holds the same hidden [B, D] and labels and C/N weight rows
    (bf16), and runs vocab_parallel_lm_head_loss (the fused tcgen05 kernel on
    its rows, an all-gather of the chunk summaries, the combined solve, the
    sparse backward with an fp32 all-reduce of dhidden).  Strong scaling: the
    job is one B x C head per step whatever N is."""
    import torch
    import torch.distributed as dist

    from fwloss_b200.sharded import even_col_start
    from fwloss_b200.vocab_parallel import vocab_parallel_lm_head_loss

    world = int(os.environ["WORLD_SIZE"])
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    B, D, C = (int(v) for v in a.lm_shape.split(","))
    cs = even_col_start(C, world)
    g = torch.Generator(device=dev).manual_seed(4)  # same hidden and labels on every rank
    hidden = (torch.randn(B, D, generator=g, device=dev) / D ** 0.5 * 4).to(torch.bfloat16).requires_grad_(True)
    target = torch.randint(0, C, (B,), generator=g, device=dev)
    gw = torch.Generator(device=dev).manual_seed(1000 + rank)  # this rank's weight rows
    weight = torch.randn(cs[rank + 1] - cs[rank], D, generator=gw, device=dev).to(torch.bfloat16).requires_grad_(True)
    forms = [f.strip() for f in a.lm_forms.split(",") if f.strip() in ("fused", "staged")] or ["fused"]
    impl = forms[0]

    def step():
        hidden.grad = weight.grad = None
        vocab_parallel_lm_head_loss(hidden, weight, target, cs, impl=impl).backward()

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize(dev)
    dist.barrier()
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(a.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item()) / a.steps
    if rank == 0:
        print(json.dumps({
            "metric": f"LM head + FWLoss fwd+bwd rows/s (B={B}, D={D}, C={C}, bf16), vocabulary-parallel",
            "value": B / (ms / 1e3), "unit": UNIT, "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic", "config": {"workload": f"hidden [{B}, {D}] x weight [{C}, {D}]^T -> FW loss, "
                                                        f"{C // world} classes per GPU", "form": impl,
                                            "forward_gemm_tflop": 2.0 * B * D * C / 1e12},
        }), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    return 0


def main():
    a = parse()
    if a.impl == "reference":
        return run_reference(a)
    if a.impl == "reference-cuda":
        return run_reference_cuda(a)
    if a.mode == "class-sharded":
        return run_class_sharded(a)
    if a.mode == "lm-head":
        if int(os.environ.get("WORLD_SIZE", "1")) > 1:
            return run_lm_head_vocab_parallel(a)
        return run_lm_head(a)
    return run_ours(a)


if __name__ == "__main__":
    sys.exit(main())
