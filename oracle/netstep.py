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


def _glorot_uniform(rng, shape):
    """Keras's default kernel initializer: U(-l, l), l = sqrt(6 / (fan_in +
    fan_out)), fans of a [..., in, out] kernel scaled by its receptive field."""
    rf = int(np.prod(shape[:-2])) if len(shape) > 2 else 1
    fi, fo = shape[-2] * rf, shape[-1] * rf
    lim = np.sqrt(6.0 / max(1, fi + fo))
    return rng.uniform(-lim, lim, shape).astype(np.float32)


def readme_params(widened=False, seed=0):
    """Random-init weights of the README network (README.md:162-183) without
    the GPU package: glorot-uniform kernels, zero Dense bias, BatchNorm gamma 1
    and beta 0, keyed like params_of().  ``widened``: input 256x256x3, filters
    96/192/288, Dense 512."""
    rng = np.random.default_rng(seed)
    in_hw, filters, units = ((256, (96, 192, 288), 512) if widened else (64, (48, 96, 144), 128))
    ones = lambda c: np.ones(c, np.float32)  # noqa: E731
    zeros = lambda c: np.zeros(c, np.float32)  # noqa: E731
    f0 = filters[0]
    p = {"stem_w": _glorot_uniform(rng, (3, 7, 3, f0)), "stem_g": ones(f0), "stem_b": zeros(f0), "blocks": []}
    H, W, C = in_hw, -(-in_hw // 2), f0
    for f in filters[1:]:
        p["blocks"].append({"dw": _glorot_uniform(rng, (3, 3, C, 1)), "g1": ones(C), "b1": zeros(C),
                            "pw": _glorot_uniform(rng, (1, 1, C, f)), "g2": ones(f), "b2": zeros(f)})
        H, W, C = -(-H // 2), -(-W // 2), f
    p["dense_w"] = _glorot_uniform(rng, (H * W * C, units))
    p["dense_b"] = zeros(units)
    return p


def uwb_seq(seed=0, t_ctx=8, n_bins=16, head=(9, 6, 8), eps=1e-3):
    """Random-init stage list of the uwb_loc_v3 network
    (examples/train_full_model.py:70-100) without the GPU package, in
    seq_of()'s format: glorot-uniform kernels, zero Dense bias, BatchNorm
    gamma 1, beta 0, moving mean 0, moving variance 1."""
    rng = np.random.default_rng(seed)
    st = []
    H, W, C = t_ctx, n_bins, 36

    def conv_bn_relu(f, k, s=(1, 1)):
        nonlocal H, W, C
        st.append(("conv", {"w": _glorot_uniform(rng, (k[0], k[1], C, f))}, ((1, s[0], s[1], 1), "SAME")))
        H, W, C = -(-H // s[0]), -(-W // s[1]), f
        st.append(("bn", {"g": np.ones(f, np.float32), "b": np.zeros(f, np.float32),
                          "mean": np.zeros(f, np.float32), "var": np.ones(f, np.float32)}, eps))
        st.append(("relu", {}, None))

    conv_bn_relu(48, (3, 7), (1, 2))
    for f in (96, 144, 192):
        st.append(("dw", {"w": _glorot_uniform(rng, (3, 3, C, 1))}, ((1, 2, 2, 1), "SAME")))
        H, W = -(-H // 2), -(-W // 2)
        st.append(("bn", {"g": np.ones(C, np.float32), "b": np.zeros(C, np.float32),
                          "mean": np.zeros(C, np.float32), "var": np.ones(C, np.float32)}, eps))
        st.append(("relu", {}, None))
        conv_bn_relu(f, (1, 1))
    conv_bn_relu(64, (1, 1))
    units = head[0] * head[1] * head[2]
    st += [("flatten", {}, None),
           ("dense", {"w": _glorot_uniform(rng, (H * W * C, units)), "b": np.zeros(units, np.float32)}, None),
           ("relu", {}, None), ("reshape", {}, tuple(head))]
    H, W, C = head
    for _ in range(2):
        st.append(("up", {}, (2, 2)))
        H, W = 2 * H, 2 * W
        conv_bn_relu(16, (3, 3))
    st += [("conv", {"w": _glorot_uniform(rng, (1, 1, C, 1))}, ((1, 1, 1, 1), "SAME")), ("sigmoid", {}, None)]
    return st


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


def train_grads_f64(p, x, target, head=(4, 4, 8), up=(2, 2), eps=1e-3, device="cpu"):
    """The same training step in float64 torch autograd (NCHW convolutions with
    TF SAME padding, biased-variance BN, half-pixel bilinear) -- the exact
    arbiter.  Returns (loss, out, grads) keyed like train_grads()."""
    import torch
    import torch.nn.functional as F

    dev = torch.device(device)
    tt = lambda a: torch.tensor(np.asarray(a), dtype=torch.float64, device=dev, requires_grad=True)  # noqa: E731
    P = {k: tt(p[k]) for k in ("stem_w", "stem_g", "stem_b", "dense_w", "dense_b")}
    Bl = [{k: tt(v) for k, v in b.items()} for b in p["blocks"]]

    def conv(z, w, stride, groups=1):
        kh, kw = w.shape[0], w.shape[1]
        H, W = z.shape[2], z.shape[3]
        oh, ow = -(-H // stride[0]), -(-W // stride[1])
        ph = max((oh - 1) * stride[0] + kh - H, 0)
        pw = max((ow - 1) * stride[1] + kw - W, 0)
        z = F.pad(z, (pw // 2, pw - pw // 2, ph // 2, ph - ph // 2))
        wt = w.permute(3, 2, 0, 1) if groups == 1 else w.permute(2, 3, 0, 1)
        return F.conv2d(z, wt, stride=stride, groups=groups)

    def bn(z, gm, bt):
        m = z.mean(dim=(0, 2, 3), keepdim=True)
        v = (z * z).mean(dim=(0, 2, 3), keepdim=True) - m * m
        return gm.view(1, -1, 1, 1) * (z - m) / torch.sqrt(v + eps) + bt.view(1, -1, 1, 1)

    N = x.shape[0]
    z = torch.tensor(x, dtype=torch.float64, device=dev).permute(0, 3, 1, 2)
    z = torch.relu(bn(conv(z, P["stem_w"], (1, 2)), P["stem_g"], P["stem_b"]))
    for b in Bl:
        z = torch.relu(bn(conv(z, b["dw"], (2, 2), groups=z.shape[1]), b["g1"], b["b1"]))
        z = torch.relu(bn(conv(z, b["pw"], (1, 1)), b["g2"], b["b2"]))
    z = z.permute(0, 2, 3, 1).reshape(N, -1)
    z = torch.relu(z @ P["dense_w"] + P["dense_b"]).reshape(N, *head).permute(0, 3, 1, 2)
    z = F.interpolate(z, scale_factor=up, mode="bilinear", align_corners=False)
    out = torch.sigmoid(z).permute(0, 2, 3, 1)
    loss = torch.mean((out - torch.tensor(target, dtype=torch.float64, device=dev)) ** 2)
    loss.backward()
    g = {k: P[k].grad.cpu().numpy() for k in P}
    g["blocks"] = [{k: v.grad.cpu().numpy() for k, v in b.items()} for b in Bl]
    return float(loss), out.detach().cpu().numpy(), g


# ---------------------------------------------------------------------------
# Any network given as a stage list (opencl_tf.model: BuildModel.stages(),
# UwbLocV3.stages()): the forward pass, MSE loss and backward pass with the
# reference's gradient wiring (opencl_tf/gradients.py:18-119), and the
# inference forward with BatchNormalization on its moving statistics.

def seq_of(model):
    """The model's stages as plain data: (kind, params, arg) with numpy weights
    (conv/dw/dense: w [, b]; bn: g, b, mean, var, eps) and the strides,
    upsampling size or reshape target as arg."""
    out = []
    for kind, layer, arg in model.stages():
        if kind in ("conv", "dw"):
            s = layer.strides
            out.append((kind, {"w": _np(layer.kernel)}, ((1, s[0], s[1], 1), layer.padding)))
        elif kind == "bn":
            out.append((kind, {"g": _np(layer.gamma), "b": _np(layer.beta), "mean": _np(layer.moving_mean),
                               "var": _np(layer.moving_var)}, float(layer.epsilon)))
        elif kind == "dense":
            b = _np(layer.bias) if layer.use_bias else np.zeros(layer.units, np.float32)
            out.append((kind, {"w": _np(layer.kernel), "b": b}, None))
        elif kind == "up":
            out.append((kind, {}, tuple(layer.size)))
        else:
            out.append((kind, {}, arg))
    return out


def uwb_input(x):
    """Permute((1, 4, 2, 3, 5)) + Reshape((T, bins, 36)) of the uwb_loc_v3 input."""
    n, t, _, _, bins, _ = x.shape
    return np.ascontiguousarray(np.transpose(x, (0, 1, 4, 2, 3, 5))).reshape(n, t, bins, 36)


def seq_forward_inference(o, seq, x):
    """Inference forward: BatchNormalization -> OpenclBatchNormInference with
    the moving statistics."""
    a = x
    for kind, p, arg in seq:
        if kind == "conv":
            a = o.conv2d(a, p["w"], arg[0], arg[1])
        elif kind == "dw":
            a = o.depthwise_conv2d(a, p["w"], arg[0], arg[1])
        elif kind == "bn":
            a = o.batch_norm_inference(a, p["g"], p["b"], p["mean"], p["var"], arg)
        elif kind == "relu":
            a = o.relu(a)
        elif kind == "dense":
            a = o.dense(a, p["w"], p["b"])
        elif kind == "flatten":
            a = a.reshape(a.shape[0], -1)
        elif kind == "reshape":
            a = a.reshape(a.shape[0], *arg)
        elif kind == "up":
            a = o.upsampling_bilinear_2d(a, arg)
        elif kind == "sigmoid":
            a = o.sigmoid(a)
        else:
            raise ValueError(kind)
    return a


def seq_train_grads(o, seq, x, target):
    """Training step: returns (loss, out, grads) with grads[i] a dict of the
    i-th stage's weight gradients (conv/dw: w; bn: g, b; dense: w, b)."""
    acts, saved = [], []
    a = x
    for kind, p, arg in seq:
        acts.append(a)
        if kind == "conv":
            a = o.conv2d(a, p["w"], arg[0], arg[1])
        elif kind == "dw":
            a = o.depthwise_conv2d(a, p["w"], arg[0], arg[1])
        elif kind == "bn":
            a, m, v = o.batch_norm_training(a, p["g"], p["b"], arg)
            saved.append((m, v))
        elif kind == "relu":
            a = o.relu(a)
        elif kind == "dense":
            a = o.dense(a, p["w"], p["b"])
        elif kind in ("flatten", "reshape"):
            a = a.reshape(a.shape[0], -1) if kind == "flatten" else a.reshape(a.shape[0], *arg)
        elif kind == "up":
            a = o.upsampling_bilinear_2d(a, arg)
        elif kind == "sigmoid":
            a = o.sigmoid(a)
        else:
            raise ValueError(kind)
    out = a
    diff = out.astype(np.float64) - target.astype(np.float64)
    loss = float(np.mean(diff * diff))
    d = (2.0 * diff / diff.size).astype(np.float32)
    grads = [dict() for _ in seq]
    bn_i = len(saved)
    for i in range(len(seq) - 1, -1, -1):
        kind, p, arg = seq[i]
        xin = acts[i]
        if kind == "conv":
            grads[i]["w"] = o.conv2d_backprop_filter(xin, p["w"].shape, d, arg[0], arg[1])
            d = o.conv2d_backprop_input(xin.shape, p["w"], d, arg[0], arg[1]) if i else None
        elif kind == "dw":
            grads[i]["w"] = o.depthwise_conv2d_backprop_filter(xin, p["w"].shape, d, arg[0], arg[1])
            d = o.depthwise_conv2d_backprop_input(xin.shape, p["w"], d, arg[0], arg[1]) if i else None
        elif kind == "bn":
            bn_i -= 1
            m, v = saved[bn_i]
            d, grads[i]["g"], grads[i]["b"] = o.batch_norm_grad(d, xin, p["g"], m, v, arg)
        elif kind == "relu":
            d = o.relu_grad(d, xin)
        elif kind == "dense":
            grads[i]["w"] = o.dense_backprop_weight(xin, d)
            grads[i]["b"] = o.dense_backprop_bias(d)
            d = o.dense_backprop_input(d, p["w"])
        elif kind in ("flatten", "reshape"):
            d = d.reshape(xin.shape)
        elif kind == "up":
            d = o.upsampling_bilinear_2d_grad(d, xin.shape, arg)
        elif kind == "sigmoid":
            d = o.sigmoid_grad(acts[i + 1] if i + 1 < len(acts) else out, d)
    return loss, out, grads


def seq_train_grads_f64(seq, x, target, device="cpu"):
    """The same training step in float64 torch autograd (TF SAME padding,
    biased-variance BN, half-pixel bilinear) -- the exact arbiter."""
    import torch
    import torch.nn.functional as F

    dev = torch.device(device)
    tt = lambda a: torch.tensor(np.asarray(a), dtype=torch.float64, device=dev, requires_grad=True)  # noqa: E731
    P = [{k: tt(v) for k, v in p.items() if k in ("w", "b", "g")} for _, p, _ in seq]

    def conv(z, w, strides, padding, groups=1):
        kh, kw = w.shape[0], w.shape[1]
        sh, sw = strides[1], strides[2]
        H, W = z.shape[2], z.shape[3]
        if padding == "SAME":
            oh, ow = -(-H // sh), -(-W // sw)
            ph = max((oh - 1) * sh + kh - H, 0)
            pw = max((ow - 1) * sw + kw - W, 0)
            z = F.pad(z, (pw // 2, pw - pw // 2, ph // 2, ph - ph // 2))
        wt = w.permute(3, 2, 0, 1) if groups == 1 else w.permute(2, 3, 0, 1).reshape(-1, 1, kh, kw)
        return F.conv2d(z, wt, stride=(sh, sw), groups=groups)

    z = torch.tensor(x, dtype=torch.float64, device=dev).permute(0, 3, 1, 2)  # NCHW while spatial
    for (kind, p, arg), q in zip(seq, P):
        if kind == "conv":
            z = conv(z, q["w"], arg[0], arg[1])
        elif kind == "dw":
            z = conv(z, q["w"], arg[0], arg[1], groups=z.shape[1])
        elif kind == "bn":
            m = z.mean(dim=(0, 2, 3), keepdim=True)
            v = (z * z).mean(dim=(0, 2, 3), keepdim=True) - m * m
            z = q["g"].view(1, -1, 1, 1) * (z - m) / torch.sqrt(v + arg) + q["b"].view(1, -1, 1, 1)
        elif kind == "relu":
            z = torch.relu(z)
        elif kind == "flatten":
            z = z.permute(0, 2, 3, 1).reshape(z.shape[0], -1)
        elif kind == "dense":
            z = z @ q["w"] + q["b"]
        elif kind == "reshape":
            z = z.reshape(z.shape[0], *arg).permute(0, 3, 1, 2)
        elif kind == "up":
            z = F.interpolate(z, scale_factor=arg, mode="bilinear", align_corners=False)
        elif kind == "sigmoid":
            z = torch.sigmoid(z)
    out = z.permute(0, 2, 3, 1)
    loss = torch.mean((out - torch.tensor(target, dtype=torch.float64, device=dev)) ** 2)
    loss.backward()
    return float(loss.detach()), out.detach().cpu().numpy(), [{k: v.grad.cpu().numpy() for k, v in q.items()} for q in P]
