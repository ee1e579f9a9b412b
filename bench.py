#!/usr/bin/env python
"""Throughput of the README ``build_model()`` training step on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--widened]
                    [--model build_model|uwb_loc_v3]

One step = forward + MSE loss + backward (the 19 custom ops) + gradient
averaging across ranks + Adam, on a fixed synthetic batch of 256 images per
GPU (input ~U(0,1) [256,64,64,3], targets ~U(0,1) [256,8,8,8], fixed seed,
random-init weights).  For N > 1 run under torchrun: one process per GPU,
NCCL, weak scaling (256 images per GPU).

Reported (one JSON line from rank 0):
  value     images/s over all ranks, inputs already in HBM, the step replayed
            from one CUDA graph; per-step CUDA events, L2 flushed (256 MiB
            write) between steps outside the timed events, max over ranks;
            the K steps form a window, repeated until ~1 s of timed work has
            passed (5 to 100 windows), and the median window is reported
            (`timing` gives the count and the spread);
  e2e       the same metric through the public API with the batch copied from
            pinned host memory every step and the loss copied back; the next
            step's copy runs on a copy stream during the current step (an
            input pipeline) and is enclosed by that step's events; the median
            of 5 windows of K steps;
  roofline  the op with the largest share of the step, timed alone with CUDA
            events (L2 flushed before each repetition) against its algorithmic
            bytes / FLOPs; per_op has every op type;
  cpu_baseline  the reference's own kernels (kernels/*.cl compiled for the host,
            oracle/_ref) running the same step on all host cores, on a bounded
            sample of the batch.
``--impl reference`` times only that CPU implementation (rank 0).
``--model uwb_loc_v3`` measures the second network instead (the reference's
examples/train_full_model.py model; 1024 samples of stacked IQ per GPU).
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "opencl-tensorflow_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "build_model train images/s at 1/2/4/8 B200; per-op % of HBM/TC roofline"
METRIC_UWB = "uwb_loc_v3 train samples/s; per-op % of HBM/TC roofline"
PER_GPU_BATCH = 256


def workload(widened: bool, model: str = "build_model") -> dict:
    """The measured workload.  cpu_sample: images of the batch in one step of
    the reference arm (the whole batch unless a step would take minutes)."""
    if model == "uwb_loc_v3":
        return {"workload": "uwb_loc_v3 training step (examples/train_full_model.py): stacked IQ [8,6,3,16,2] -> "
                            "[8,16,36], conv 48 (3,7)/(1,2), dsconv 96/144/192 stride 2, neck 64, Dense 432, head "
                            "9x6x8 -> up, conv 16 -> up, conv 16 -> 36x24x1; fwd+bwd+Adam(1e-3), MSE",
                "batch_per_gpu": 1024, "model": model, "metric": METRIC_UWB, "cpu_sample": 1024,
                "unit": "samples/s"}
    if widened:
        return {"workload": "README build_model training step, widened: input 256x256x3, filters 96/192/288, "
                            "Dense 512, head 8x8x8 -> 16x16x8; fwd+bwd+Adam(1e-3), MSE",
                "batch_per_gpu": 128, "in_hw": 256, "out_hw": 16, "model": model, "metric": METRIC, "cpu_sample": 4,
                "unit": "images/s"}
    return {"workload": "README build_model training step: input 64x64x3, conv 48 (3,7)/(1,2), dsconv 96 and 144 "
                        "stride 2, Dense 128, head 4x4x8 -> 8x8x8; fwd+bwd+Adam(1e-3), MSE",
            "batch_per_gpu": PER_GPU_BATCH, "in_hw": 64, "out_hw": 8, "model": model, "metric": METRIC,
            "cpu_sample": PER_GPU_BATCH, "unit": "images/s"}


def config_of(w: dict, world: int) -> dict:
    """The JSON line's config: the same dict for both arms."""
    return {"workload": w["workload"], "global_batch": w["batch_per_gpu"] * world,
            "per_gpu_batch": w["batch_per_gpu"], "parallelism": f"dp{world}",
            "l2": "flushed between timed steps (256 MiB write outside the step's events)",
            "math": "fp32 activations; contractions on tcgen05 tensor cores in 3xTF32 (the reference arm: fp32 "
                    "FMA on the host cores)"}


def host_cores() -> int:
    """Host cores this process may run on (affinity-aware)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def make_batch(w, n, seed):
    rng = np.random.default_rng(seed)
    if w["model"] == "uwb_loc_v3":  # the example's make_batch: IQ ~ N(0, 1), heatmap ~ U(0, 1)
        x = rng.standard_normal((n, 8, 6, 3, 16, 2)).astype(np.float32)
        t = rng.uniform(0, 1, (n, 36, 24, 1)).astype(np.float32)
        return x, t
    in_hw, out_hw = w["in_hw"], w["out_hw"]
    x = rng.uniform(0, 1, (n, in_hw, in_hw, 3)).astype(np.float32)
    t = rng.uniform(0, 1, (n, out_hw, out_hw, 8)).astype(np.float32)
    return x, t


def build_net(w, widened, device=None):
    from opencl_tf.model import build_model, build_uwb_loc_v3
    if w["model"] == "uwb_loc_v3":
        return build_uwb_loc_v3(device=device)
    return build_model(widened=widened, device=device)


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi sampling (200 ms) of the GPUs in use during the timed region."""

    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, uuids):
        self.uuids = set(uuids)
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix="b2_clocks_", suffix=".csv")
            os.close(fd)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:  # noqa: BLE001
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:  # noqa: BLE001
            self.proc.kill()
        self.fh.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in Path(self.path).read_text().splitlines():
            f = [s.strip() for s in line.split(",")]
            if len(f) < 8:
                continue
            uuid = f[0]
            if self.uuids and not any(u in uuid or uuid in u for u in self.uuids):
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------- reference (CPU)

def adam_np(params, grads, state, lr=1e-3, b1=0.9, b2=0.999, eps=1e-7):
    state["t"] = state.get("t", 0) + 1
    t = state["t"]
    for k, p in params.items():
        g = grads[k]
        m = state.setdefault(("m", k), np.zeros_like(p))
        v = state.setdefault(("v", k), np.zeros_like(p))
        m *= b1
        m += (1 - b1) * g
        v *= b2
        v += (1 - b2) * g * g
        p -= lr * (m / (1 - b1 ** t)) / (np.sqrt(v / (1 - b2 ** t)) + eps)


def _flat(p, prefix=""):
    out = {}
    for k, v in p.items():
        if isinstance(v, list):
            for i, d in enumerate(v):
                out.update(_flat(d, f"{prefix}{k}{i}."))
        else:
            out[prefix + k] = v
    return out


def cpu_reference_steps(widened, sample_images, steps, warmup, min_seconds=0.0, model_name="build_model"):
    """Runs the training step with the reference's host-compiled kernels on
    every host core (OpenMP thread count set explicitly, whatever a launcher
    exported); the weights are initialised in numpy, so none of this
    repository's GPU code is loaded.  Returns (images/s, cores, kind, seconds,
    steps_done)."""
    from oracle.netstep import readme_params, seq_train_grads, train_grads, uwb_input, uwb_seq
    from oracle.oracle import Oracle, available
    kind = "reference" if available("ref") else "port"
    o = Oracle("ref" if kind == "reference" else "port", threads=host_cores())
    w = workload(widened, model_name)
    x, t = make_batch(w, sample_images, 1234)
    state = {}
    if model_name == "uwb_loc_v3":
        seq = uwb_seq(seed=0)
        xi = uwb_input(x)
        flat = {f"{i}.{k}": v for i, (_, p, _) in enumerate(seq) for k, v in p.items() if k in ("w", "b", "g")}

        def step():
            _, _, g = seq_train_grads(o, seq, xi, t)
            adam_np(flat, {f"{i}.{k}": v for i, d in enumerate(g) for k, v in d.items()}, state)
    else:
        p = readme_params(widened=widened, seed=0)
        head = (8, 8, 8) if widened else (4, 4, 8)
        flat = _flat(p)

        def step():
            _, _, g = train_grads(o, p, x, t, head=head)
            adam_np(flat, _flat(g), state)

    for _ in range(warmup):
        step()
    done, t0 = 0, time.perf_counter()
    while done < steps or (time.perf_counter() - t0) < min_seconds:
        step()
        done += 1
    dt = time.perf_counter() - t0
    return sample_images * done / dt, o.threads(), kind, dt, done


# DRAM bytes (read + write) of one launch of the dominant op's kernel, from
# one ncu capture of that workload; keyed by op and its algorithmic bytes so a
# different workload reports null.  Source: the named summary under profiles/.
NCU_TRAFFIC = {
    ("conv2d_backprop_filter", 113258304): (118956288, "profiles/tma_gemm_conv_wgrad_readme_stem.md"),
    ("depthwise_conv2d_backprop_filter", 125830848): (132687360, "profiles/dw_wgrad_staged_readme_dsconv1.md"),
    ("batch_norm_relu_grad", 301991040): (469819136, "profiles/bn_relu_grad_op_readme_stem.md"),
}


def ncu_traffic(op, algorithmic_bytes):
    """(DRAM bytes per launch, summary file) or (None, None)."""
    return NCU_TRAFFIC.get((op, int(algorithmic_bytes)), (None, None))


# ------------------------------------------------------------------ ours

def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import opencl_tf
    from opencl_tf import profile
    from opencl_tf.train import TrainStep

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    w = workload(args.widened, args.model)
    B = w["batch_per_gpu"]
    torch.manual_seed(0)
    model = build_net(w, args.widened, device=dev)
    x_np, t_np = make_batch(w, B, 1000 + rank)
    x_dev = torch.from_numpy(x_np).to(dev)
    t_dev = torch.from_numpy(t_np).to(dev)
    step = TrainStep(model, lr=1e-3, graphed=True, warmup=3)
    flush = profile._Flusher(dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    # ---- warm-up (the first call also captures the graph)
    launches0 = opencl_tf._library.kernel_launch_count()
    step(x_dev, t_dev)
    launches_capture = opencl_tf._library.kernel_launch_count() - launches0
    for _ in range(max(args.warmup - 1, 0)):
        step(x_dev, t_dev)
    # kernels per step: the captured step enqueued launches_capture / 4 of ours (3 eager warm-ups + capture)
    per_step_launches = launches_capture // 4

    uuids = []
    try:
        uuids = [str(torch.cuda.get_device_properties(dev).uuid)]
    except Exception:  # noqa: BLE001
        pass
    clocks = ClockSampler(uuids)

    def timed(fn, K):
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
        barrier()
        for i in range(K):
            flush()
            starts[i].record()
            fn()
            ends[i].record()
        barrier()
        ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
        if world > 1:
            tt = torch.tensor([ms], device=dev, dtype=torch.float64)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            ms = float(tt.item())
        return ms

    clocks.start()
    time.sleep(0.3)
    torch.cuda.nvtx.range_push("timed_steps")
    # the batch is already in HBM: in the graph's own input buffers (the
    # capture copied x_dev / t_dev there), so a step is the graph replay alone.
    # The K steps are timed as a window, and the window is repeated until about
    # a second of timed work has passed (so the clock sampler sees it under
    # load); every window is exactly K steps, max over ranks, and the value is
    # the median window.  The window count follows from the first window's
    # time, which every rank has after the max-reduction, so all agree.
    replay = lambda: step(step.static_x, step.static_y)  # noqa: E731
    windows = [timed(replay, args.steps)]
    n_windows = max(5, min(100, int(math.ceil(1000.0 / max(windows[0], 1e-3)))))
    while len(windows) < n_windows:
        windows.append(timed(replay, args.steps))
    ms_dev = statistics.median(windows)
    torch.cuda.nvtx.range_pop()

    # ---- end to end: pinned host batch in, loss out, every step.  Like an
    # input pipeline, the next step's batch is copied host->device on a copy
    # stream while this step computes -- straight into the input buffers of
    # the captured graph that will run it (two graphs of the step alternate);
    # each step's timed interval contains the complete copy of the next
    # step's batch (step 0 also its own) and the device->host copy of its
    # loss, so every byte crosses inside the timing.
    x_host = torch.from_numpy(x_np).pin_memory()
    t_host = torch.from_numpy(t_np).pin_memory()
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()
    copy_stream = torch.cuda.Stream(dev)
    slots = [step.graph_inputs(0), step.graph_inputs(1)]
    torch.cuda.synchronize(dev)

    def e2e_timed(K):
        cs = torch.cuda.current_stream(dev)
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
        ready = [torch.cuda.Event() for _ in range(K)]
        done = [torch.cuda.Event() for _ in range(K)]

        def h2d(j, after):
            with torch.cuda.stream(copy_stream):
                copy_stream.wait_event(after)
                if j >= 2:
                    copy_stream.wait_event(done[j - 2])  # graph j % 2 finished step j - 2
                slots[j % 2][0].copy_(x_host, non_blocking=True)
                slots[j % 2][1].copy_(t_host, non_blocking=True)
                ready[j].record(copy_stream)

        barrier()
        for i in range(K):
            flush()
            starts[i].record(cs)
            if i == 0:
                h2d(0, starts[0])
            if i + 1 < K:
                h2d(i + 1, starts[i])
            cs.wait_event(ready[i])
            loss = step.replay(i % 2)
            done[i].record(cs)
            loss_host.copy_(loss, non_blocking=True)
            if i + 1 < K:
                cs.wait_event(ready[i + 1])
            ends[i].record(cs)
        barrier()
        ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
        if world > 1:
            tt = torch.tensor([ms], device=dev, dtype=torch.float64)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            ms = float(tt.item())
        return ms

    e2e_windows = [e2e_timed(args.steps) for _ in range(5)]
    ms_e2e = statistics.median(e2e_windows)
    clk = clocks.stop()
    loss_value = float(loss_host)

    # the batch's host->device copy alone (copy stream, events), for reading e2e
    h_s, h_e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(copy_stream):
        h_s.record(copy_stream)
        for _ in range(5):
            slots[0][0].copy_(x_host, non_blocking=True)
            slots[0][1].copy_(t_host, non_blocking=True)
        h_e.record(copy_stream)
    torch.cuda.synchronize(dev)
    h2d_ms = h_s.elapsed_time(h_e) / 5

    # ---- per-op table and the dominant op's roofline (rank 0, outside the timed regions)
    per_op, roof = None, None
    if rank == 0:
        from opencl_tf.train import mse
        _, log = profile.record_step(lambda: mse(model(x_dev, training=True), t_dev).backward())
        rows = profile.time_ops(log, reps=5, device=dev)
        per_op = profile.summarize(rows)
        top = max(rows, key=lambda r: r["ms"])
        roof = {"kernel": top["op"], "bound": top["bound"], "achieved": round(top["achieved"], 1),
                "peak": round(top["peak"], 1), "unit": top["unit"], "frac": round(top["frac"], 4),
                "peak_source": profile.peaks()["source"], "traffic": ncu_traffic(top["op"], top["bytes"])[0],
                "traffic_source": ncu_traffic(top["op"], top["bytes"])[1],
                "algorithmic_bytes": top["bytes"], "algorithmic_flops": top["flops"], "ms": round(top["ms"], 4),
                "step_ms_sum_of_ops": round(sum(r["ms"] for r in rows), 4)}
        model.zero_grad(set_to_none=True)

    # ---- CPU baseline (rank 0 at N=1 only; bounded sample)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        ns = w["cpu_sample"]
        ips, cores, kind, secs, nsteps = cpu_reference_steps(args.widened, ns, 1, 1, min_seconds=10.0,
                                                             model_name=args.model)
        cpu = {"value": round(ips, 3), "unit": w["unit"], "cores": cores, "kind": kind,
               "sample": f"{nsteps} training steps of {ns} images (of the {B}-image "
                         f"batch) through the host-compiled reference kernels on all host cores, {secs:.1f} s"}

    images = B * world * args.steps
    line = {
        "metric": w["metric"], "value": round(images / (ms_dev * 1e-3), 2), "unit": w["unit"], "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_dev / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_of(w, world),
        "e2e": {"value": round(images / (ms_e2e * 1e-3), 2), "unit": w["unit"],
                "h2d_bytes_per_step": int(x_host.numel() * 4 + t_host.numel() * 4), "d2h_bytes_per_step": 4,
                "ms_per_step": round(ms_e2e / args.steps, 4),
                "h2d_ms_alone": round(h2d_ms, 4),
                "pipeline": "next batch copied host->device on a copy stream during the step, into the input "
                            "buffers of the second captured graph of the step (two alternate); each step's events "
                            "enclose that copy and the loss read-back"},
        "gpu_launches": int(per_step_launches * args.steps),
        "timing": {"windows": len(windows), "steps_per_window": args.steps,
                   "ms_per_step_min": round(min(windows) / args.steps, 4),
                   "ms_per_step_median": round(ms_dev / args.steps, 4),
                   "ms_per_step_max": round(max(windows) / args.steps, 4),
                   "e2e_windows": len(e2e_windows),
                   "note": "value and e2e are the median window of K steps (max over ranks per window); "
                           "gpu_launches counts one window"},
        "roofline": roof, "per_op": per_op, "cpu_baseline": cpu, "clocks": clk,
        "final_loss": round(loss_value, 6),
        "when": datetime.datetime.now(datetime.timezone.utc).isoformat(timespec="seconds"),
    }
    step.release()
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--widened", action="store_true")
    ap.add_argument("--model", choices=["build_model", "uwb_loc_v3"], default="build_model")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--stress-gemm", action="store_true",
                    help="time the 8192x4096x4096 stress GEMM's three passes (one JSON line) and exit")
    args = ap.parse_args()
    if args.stress_gemm:
        import torch
        import opencl_tf  # noqa: F401
        from opencl_tf import profile
        torch.cuda.set_device(0)
        print(json.dumps({"workload": "stress GEMM M=8192 K=4096 N=4096 fp32 ~N(0,1) (Dense fwd / dgrad / wgrad)",
                          **profile.stress_gemm(torch.device("cuda", 0), reps=max(args.steps, 3))}), flush=True)
        return 0
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(1)))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    w = workload(args.widened, args.model)

    if args.impl == "reference":
        if rank != 0:
            return 0
        sample = w["cpu_sample"]
        ips, cores, kind, secs, nsteps = cpu_reference_steps(args.widened, sample, args.steps, args.warmup,
                                                             model_name=args.model)
        whole = sample == w["batch_per_gpu"]
        line = {"metric": w["metric"], "value": round(ips, 3), "unit": w["unit"], "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(secs / nsteps * 1e3, 3),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic", "impl": "reference",
                "config": config_of(w, world),
                "cpu_baseline": {"value": round(ips, 3), "unit": w["unit"], "cores": cores, "kind": kind,
                                 "sample": (f"each step is the whole {sample}-image batch" if whole else
                                            f"each step is {sample} images of the {w['batch_per_gpu']}-image batch")
                                           + " through the reference's kernels compiled for the host (OpenMP over "
                                             "work-items, all host cores), weights initialised in numpy"},
                "e2e": {"value": round(ips, 3), "unit": w["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        line = run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
