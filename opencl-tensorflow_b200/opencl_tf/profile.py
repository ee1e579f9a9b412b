"""Per-op timing and roofline accounting for a training step.

``record_step(fn)`` runs ``fn()`` once (eagerly) while logging every op this
library executes -- its name, the tensors and attrs it received -- and
``time_ops(log)`` re-runs each logged call on its own: L2 is flushed (a
256 MiB write) before every repetition and CUDA events on the current stream
bracket the op only.  ``roofline(entry)`` gives each op's algorithmic work:

* FLOPs = 2*M*N*K for the contractions (conv: 2*N*Ho*Wo*Co*kH*kW*Ci; dense
  2*B*in*out), 2*taps per output for depthwise, 0 for the rest;
* bytes = every input tensor read once + every output written once (fp32);

and the binding ceiling: tensor cores when FLOPs/bytes exceeds the ridge
(3xTF32 peak / HBM bandwidth), HBM otherwise.
"""
from __future__ import annotations

import json
import os
from collections import defaultdict
from pathlib import Path

import torch

from . import _library as L

_KERNELS = ["_k_conv2d", "_k_conv2d_backprop_input", "_k_conv2d_backprop_filter", "_k_depthwise_conv2d",
            "_k_depthwise_conv2d_backprop_input", "_k_depthwise_conv2d_backprop_filter", "_k_relu", "_k_relu_grad",
            "_k_sigmoid", "_k_sigmoid_grad", "_k_batch_norm_training", "_k_batch_norm_inference",
            "_k_batch_norm_grad", "_k_dense", "_k_dense_relu", "_k_dense_backprop_input", "_k_dense_backprop_weight",
            "_k_dense_backprop_bias", "_k_upsampling_bilinear2d", "_k_upsampling_bilinear2d_grad",
            "_k_batch_norm_relu_training", "_k_batch_norm_relu_grad", "_k_mse_loss", "_k_mse_loss_grad"]


def peaks(path=None) -> dict:
    """Roofline denominators: the measured copy bandwidth and bf16 GEMM rate of
    this pool's B200s when MEASURED_PEAKS.json is present, else fallbacks."""
    p = Path(path) if path else Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    except Exception:  # noqa: BLE001
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def tf32x3_peak_tflops(pk: dict) -> float:
    """Algorithmic FLOP/s ceiling of 3xTF32: TF32 runs at half the bf16 rate
    and every product costs three MMAs."""
    return pk["bf16_tflops"] / 2.0 / 3.0


def record_step(fn):
    """Run ``fn()`` with every library op logged; returns (result, log)."""
    log = []
    saved = {}
    for name in _KERNELS:
        orig = getattr(L, name)
        saved[name] = orig

        def wrap(*args, _orig=orig, _name=name, **kw):
            out = _orig(*args, **kw)
            log.append((_name[3:], _orig, args, kw, out))
            return out

        setattr(L, name, wrap)
    try:
        res = fn()
    finally:
        for name, orig in saved.items():
            setattr(L, name, orig)
    return res, log


def _numel(t):
    return t.numel() if isinstance(t, torch.Tensor) else 0


def work(name, args, kw, out) -> tuple[float, float]:
    """(algorithmic FLOPs, algorithmic bytes) of one logged op call."""
    outs = out if isinstance(out, tuple) else (out,)
    tin = [a for a in list(args) + list(kw.values()) if isinstance(a, torch.Tensor)]
    byts = 4.0 * (sum(_numel(t) for t in tin) + sum(_numel(t) for t in outs))
    flops = 0.0
    if name in ("conv2d", "conv2d_backprop_input", "conv2d_backprop_filter"):
        if name == "conv2d":
            y, w = outs[0], args[1]
            flops = 2.0 * y.numel() * w.shape[0] * w.shape[1] * w.shape[2]
        elif name == "conv2d_backprop_input":
            w, dy = args[1], args[2]
            flops = 2.0 * dy.numel() * w.shape[0] * w.shape[1] * w.shape[2]
        else:
            dy, dw = args[2], outs[0]
            flops = 2.0 * dy.numel() * dw.shape[0] * dw.shape[1] * dw.shape[2]
    elif name.startswith("depthwise"):
        w = args[1] if name != "depthwise_conv2d_backprop_filter" else outs[0]
        taps = w.shape[0] * w.shape[1]
        big = outs[0] if name == "depthwise_conv2d" else args[2]
        flops = 2.0 * big.numel() * taps
    elif name in ("dense", "dense_relu"):
        x, w = args[0], args[1]
        flops = 2.0 * x.shape[0] * x.shape[1] * w.shape[1]
    elif name == "dense_backprop_input":
        dy, w = args[0], args[1]
        flops = 2.0 * dy.shape[0] * dy.shape[1] * w.shape[0]
    elif name == "dense_backprop_weight":
        x, dy = args[0], args[1]
        flops = 2.0 * x.shape[0] * x.shape[1] * dy.shape[1]
    return flops, byts


class _Flusher:
    def __init__(self, device, mib=256):
        self.buf = torch.empty(mib * (1 << 20) // 4, dtype=torch.float32, device=device)

    def __call__(self):
        self.buf.fill_(1.0)


def time_call(fn, reps=5, flush=None) -> float:
    """Mean device milliseconds of ``fn()`` over ``reps`` runs (events on the
    current stream around the call only; ``flush()`` runs between)."""
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
    fn()  # warm
    for i in range(reps):
        if flush:
            flush()
        starts[i].record()
        fn()
        ends[i].record()
    torch.cuda.synchronize()
    return sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / reps


def time_ops(log, reps=5, device=None) -> list[dict]:
    """Times every logged op call; returns one dict per call."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    flush = _Flusher(dev)
    pk = peaks()
    tc_peak = tf32x3_peak_tflops(pk) * 1e12
    ridge = tc_peak / (pk["hbm_gbs"] * 1e9)
    rows = []
    for name, orig, args, kw, out in log:
        ms = time_call(lambda: orig(*args, **kw), reps=reps, flush=flush)
        flops, byts = work(name, args, kw, out)
        bound = "tensor" if byts > 0 and flops / byts > ridge else "hbm"
        if bound == "tensor":
            ach, peak, unit = flops / (ms * 1e-3) / 1e12, tc_peak / 1e12, "TFLOP/s"
        else:
            ach, peak, unit = byts / (ms * 1e-3) / 1e9, pk["hbm_gbs"], "GB/s"
        rows.append({"op": name, "ms": ms, "flops": flops, "bytes": byts, "bound": bound, "achieved": ach,
                     "peak": peak, "unit": unit, "frac": ach / peak if peak else 0.0})
    return rows


def summarize(rows) -> dict:
    """Aggregate per op type: total ms, call count, time-weighted roofline fraction."""
    agg = defaultdict(lambda: {"ms": 0.0, "calls": 0, "wfrac": 0.0})
    for r in rows:
        a = agg[r["op"]]
        a["ms"] += r["ms"]
        a["calls"] += 1
        a["wfrac"] += r["frac"] * r["ms"]
    out = {}
    for k, a in sorted(agg.items(), key=lambda kv: -kv[1]["ms"]):
        out[k] = {"ms": round(a["ms"], 4), "calls": a["calls"], "frac": round(a["wfrac"] / a["ms"], 3) if a["ms"] else 0}
    return out



def stress_gemm_inputs(device, m=8192, k=4096, n=4096, seed=0):
    """The tensor-core stress case of the Dense + head workload: x [m, k], W
    [k, n], dy [m, n], all ~N(0, 1), b = 0."""
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(m, k, device=device, generator=g)
    w = torch.randn(k, n, device=device, generator=g)
    dy = torch.randn(m, n, device=device, generator=g)
    return x, w, torch.zeros(n, device=device), dy


def stress_gemm(device=None, reps=10) -> dict:
    """Times the stress GEMM's three passes (Dense forward M=8192, N=4096,
    K=4096; input gradient; weight gradient, K=8192), each 2*8192*4096*4096 =
    274.9 GFLOP: ms per pass (L2 flushed between repetitions), TFLOP/s and the
    fraction of the 3xTF32 ceiling (the bf16 tensor peak / 6)."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    x, w, b, dy = stress_gemm_inputs(dev)
    flush = _Flusher(dev)
    pk = peaks()
    ceiling = tf32x3_peak_tflops(pk)
    flops = 2.0 * x.shape[0] * x.shape[1] * w.shape[1]
    passes = {"forward": lambda: L._k_dense(x, w, b), "backprop_input": lambda: L._k_dense_backprop_input(dy, w),
              "backprop_weight": lambda: L._k_dense_backprop_weight(x, dy)}
    out = {}
    for name, fn in passes.items():
        ms = time_call(fn, reps=reps, flush=flush)
        tf = flops / (ms * 1e-3) / 1e12
        out[name] = {"ms": round(ms, 4), "tflops": round(tf, 1), "frac_3xtf32": round(tf / ceiling, 4)}
    out["ceiling_tflops"] = round(ceiling, 1)
    out["peak_source"] = pk["source"]
    out["gflop_per_pass"] = round(flops / 1e9, 1)
    return out


def _warm_step(batch: int, reps: int) -> int:
    """Prints each kernel's device time per step of the README training step
    replayed from its CUDA graph, L2 warm (as inside a training loop), from
    CUPTI records of ``reps`` replays."""
    import collections

    from torch.profiler import ProfilerActivity, profile

    from .model import build_model
    from .train import TrainStep
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    model = build_model(device=dev)
    g = torch.Generator(device=dev).manual_seed(1)
    x = torch.rand(batch, 64, 64, 3, device=dev, generator=g)
    t = torch.rand(batch, 8, 8, 8, device=dev, generator=g)
    step = TrainStep(model, graphed=True, warmup=3)
    for _ in range(6):
        step(x, t)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(reps):
            step(x, t)
        torch.cuda.synchronize()
    agg = collections.defaultdict(lambda: [0.0, 0])
    for e in prof.events():
        if e.device_type == torch.autograd.DeviceType.CUDA:
            agg[e.name][0] += getattr(e, "device_time_total", 0.0) or e.cuda_time_total
            agg[e.name][1] += 1
    total = sum(v[0] for v in agg.values())
    print(f"kernel time per step: {total / reps:.1f} us over {reps} replays of the batch-{batch} step")
    for name, (us, n) in sorted(agg.items(), key=lambda kv: -kv[1][0]):
        print(f"{us / reps:8.1f} us  {n // reps:3d}x  {name[:100]}")
    step.release()
    return 0


def _cli() -> int:
    """Replay one op of a network's training step, e.g. for ncu:

        PYTHONPATH=opencl-tensorflow_b200 python -m opencl_tf.profile --op conv2d --call 0 --reps 3

    records one step of --model (build_model, the default, or uwb_loc_v3) at
    --batch (default 256), then runs the --call-th call of --op (in step
    order) --reps times after one warm-up run; --list prints the step's op
    calls with their per-op times.
    """
    import argparse
    import sys

    ap = argparse.ArgumentParser()
    ap.add_argument("--op", default="conv2d_backprop_filter")
    ap.add_argument("--call", type=int, default=0)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--list", action="store_true")
    ap.add_argument("--model", choices=["build_model", "uwb_loc_v3"], default="build_model")
    ap.add_argument("--stress", choices=["forward", "backprop_input", "backprop_weight"],
                    help="run one pass of the 8192x4096x4096 stress GEMM instead")
    ap.add_argument("--warm-step", action="store_true",
                    help="per-kernel device time of the captured training step, warm (CUPTI through "
                         "torch.profiler over --reps replays)")
    a = ap.parse_args()
    if a.warm_step:
        return _warm_step(a.batch, max(a.reps, 1))
    if a.stress:
        dev = torch.device("cuda", 0)
        x, w, b, dy = stress_gemm_inputs(dev)
        fn = {"forward": lambda: L._k_dense(x, w, b), "backprop_input": lambda: L._k_dense_backprop_input(dy, w),
              "backprop_weight": lambda: L._k_dense_backprop_weight(x, dy)}[a.stress]
        for _ in range(1 + a.reps):
            fn()
        torch.cuda.synchronize()
        return 0
    from .model import build_model, build_uwb_loc_v3
    from .train import mse
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    g = torch.Generator(device=dev).manual_seed(1)
    if a.model == "uwb_loc_v3":
        model = build_uwb_loc_v3(device=dev)
        x = torch.randn(a.batch, 8, 6, 3, 16, 2, device=dev, generator=g)
        t = torch.rand(a.batch, 36, 24, 1, device=dev, generator=g)
    else:
        model = build_model(device=dev)
        x = torch.rand(a.batch, 64, 64, 3, device=dev, generator=g)
        t = torch.rand(a.batch, 8, 8, 8, device=dev, generator=g)
    _, log = record_step(lambda: mse(model(x, training=True), t).backward())
    if a.list:
        for r, (name, *_rest) in zip(time_ops(log), log):
            print(f"{name:36s} {r['ms']:8.4f} ms  {r['achieved']:9.1f} {r['unit']:8s} frac {r['frac']:.3f}")
        return 0
    calls = [e for e in log if e[0] == a.op]
    if a.call >= len(calls):
        print(f"op {a.op} has {len(calls)} calls in the step", file=sys.stderr)
        return 2
    _, orig, args, kw, _ = calls[a.call]
    for _ in range(1 + a.reps):
        orig(*args, **kw)
    torch.cuda.synchronize()
    return 0


if __name__ == "__main__":
    raise SystemExit(_cli())
