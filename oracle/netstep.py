"""TEST INFRASTRUCTURE (oracle). The README network's training step (forward, MSE loss, backward) composed
from the oracle's per-op functions, with the reference's gradient wiring --
the CPU arbiter for the end-to-end GPU tests."""
from __future__ import annotations

import numpy as np


def _np(t):
    return t.detach().cpu().numpy()


def params_of(model):
    """Weights of an opencl_tf.model.BuildModel as numpy arrays."""
    p = {"stem_w": _np(model.stem_conv.kernel), "stem_g": _np(model.stem_bn.gamma), "stem_b": _np(model.stem_bn.beta),
         "blocks": [], "dense_w": _np(model.dense.kernel), "dense_b": _np(model.dense.bias)}
    for dw, bn1, _, pw, bn2, _ in model.blocks:
        p["blocks"].append({"dw": _np(dw.kernel), "g1": _np(bn1.gamma), "b1": _np(bn1.beta), "pw": _np(pw.kernel),
                            "g2": _np(bn2.gamma), "b2": _np(bn2.beta)})
    return p


def train_grads(o, p, x, target, head=(4, 4, 8), up=(2, 2), eps=1e-3):
    """Returns (loss, out, grads) with grads keyed like params_of()."""
    S1 = (1, 1, 2, 1)
    S2 = (1, 2, 2, 1)
    S0 = (1, 1, 1, 1)
    t = {}
    t["c0"] = o.conv2d(x, p["stem_w"], S1, "SAME")
    t["bn0"], t["m0"], t["v0"] = o.batch_norm_training(t["c0"], p["stem_g"], p["stem_b"], eps)
    a = o.relu(t["bn0"])
    t["r0"] = a
    blk = []
    for b in p["blocks"]:
        s = {"in": a}
        s["dw"] = o.depthwise_conv2d(a, b["dw"], S2, "SAME")
        s["bn1"], s["m1"], s["v1"] = o.batch_norm_training(s["dw"], b["g1"], b["b1"], eps)
        s["r1"] = o.relu(s["bn1"])
        s["pw"] = o.conv2d(s["r1"], b["pw"], S0, "SAME")
        s["bn2"], s["m2"], s["v2"] = o.batch_norm_training(s["pw"], b["g2"], b["b2"], eps)
        a = o.relu(s["bn2"])
        blk.append(s)
    N = x.shape[0]
    flat = a.reshape(N, -1)
    dn = o.dense(flat, p["dense_w"], p["dense_b"])
    r = o.relu(dn)
    hd = r.reshape(N, *head)
    u = o.upsampling_bilinear_2d(hd, up)
    out = o.sigmoid(u)
    diff = out.astype(np.float64) - target.astype(np.float64)
    loss = float(np.mean(diff * diff))

    g = {"blocks": [dict() for _ in p["blocks"]]}
    dout = (2.0 * diff / diff.size).astype(np.float32)
    du = o.sigmoid_grad(out, dout)
    dhd = o.upsampling_bilinear_2d_grad(du, hd.shape, up)
    ddn = o.relu_grad(dhd.reshape(N, -1), dn)
    g["dense_w"] = o.dense_backprop_weight(flat, ddn)
    g["dense_b"] = o.dense_backprop_bias(ddn)
    da = o.dense_backprop_input(ddn, p["dense_w"]).reshape(a.shape)
    for b, s, gb in reversed(list(zip(p["blocks"], blk, g["blocks"]))):
        d = o.relu_grad(da, s["bn2"])
        d, gb["g2"], gb["b2"] = o.batch_norm_grad(d, s["pw"], b["g2"], s["m2"], s["v2"], eps)
        gb["pw"] = o.conv2d_backprop_filter(s["r1"], b["pw"].shape, d, S0, "SAME")
        d = o.conv2d_backprop_input(s["r1"].shape, b["pw"], d, S0, "SAME")
        d = o.relu_grad(d, s["bn1"])
        d, gb["g1"], gb["b1"] = o.batch_norm_grad(d, s["dw"], b["g1"], s["m1"], s["v1"], eps)
        gb["dw"] = o.depthwise_conv2d_backprop_filter(s["in"], b["dw"].shape, d, S2, "SAME")
        da = o.depthwise_conv2d_backprop_input(s["in"].shape, b["dw"], d, S2, "SAME")
    d = o.relu_grad(da, t["bn0"])
    d, g["stem_g"], g["stem_b"] = o.batch_norm_grad(d, t["c0"], p["stem_g"], t["m0"], t["v0"], eps)
    g["stem_w"] = o.conv2d_backprop_filter(x, p["stem_w"].shape, d, S1, "SAME")
    return loss, out, g
