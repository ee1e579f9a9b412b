"""The TensorFlow DEVICE_GPU kernel shim (opencl-tensorflow_b200/tf_shim).

TensorFlow is not installed here, so the shim cannot be built against it.
These tests check what can be checked without it:

* it registers a GPU kernel for every one of the reference's 19 ops, with the
  reference's HostMemory shape inputs (src/ops/*.cc REGISTER_KERNEL_BUILDER
  blocks: conv2d_ops.cc:196,320,446; depthwise_conv2d_ops.cc:191,309,430;
  relu_ops.cc:93,165; sigmoid_ops.cc:103,174; batchnorm_ops.cc:185,281,421;
  dense_ops.cc:146,229,313,381; upsampling_ops.cc:159,270);
* every library entry it calls is declared in include/b2_opencl_tf.h;
* it type-checks (g++ -fsyntax-only) against tests/tf_stub, a stand-in for
  the few TensorFlow declarations it uses, and the real C ABI header — so the
  argument lists of all 19 ABI calls are checked by the compiler.
"""
from __future__ import annotations

import re
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
SHIM = ROOT / "opencl-tensorflow_b200" / "tf_shim" / "b2_tf_gpu_kernels.cc"
HEADER = ROOT / "include" / "b2_opencl_tf.h"

# op name -> HostMemory inputs, as the reference registers them
REFERENCE_OPS = {
    "OpenclConv2d": (),
    "OpenclConv2dBackpropInput": ("input_sizes",),
    "OpenclConv2dBackpropFilter": ("filter_sizes",),
    "OpenclDepthwiseConv2d": (),
    "OpenclDepthwiseConv2dBackpropInput": ("input_sizes",),
    "OpenclDepthwiseConv2dBackpropFilter": ("filter_sizes",),
    "OpenclRelu": (),
    "OpenclReluGrad": (),
    "OpenclSigmoid": (),
    "OpenclSigmoidGrad": (),
    "OpenclBatchNormTraining": (),
    "OpenclBatchNormInference": (),
    "OpenclBatchNormGrad": (),
    "OpenclDense": (),
    "OpenclDenseBackpropInput": (),
    "OpenclDenseBackpropWeight": (),
    "OpenclDenseBackpropBias": (),
    "OpenclUpsamplingBilinear2d": (),
    "OpenclUpsamplingBilinear2dGrad": ("input_sizes",),
}


def _registrations():
    src = re.sub(r"\s+", " ", SHIM.read_text())
    regs = {}
    for m in re.finditer(r'REGISTER_KERNEL_BUILDER\( ?Name\("(\w+)"\)((?:\.\w+\([^)]*\))*), ?([\w<>:]+)\)', src):
        name, chain, cls = m.group(1), m.group(2), m.group(3)
        assert ".Device(DEVICE_GPU)" in chain, name
        host = tuple(re.findall(r'\.HostMemory\("(\w+)"\)', chain))
        regs[name] = (host, cls)
    return regs


def test_every_reference_op_has_a_gpu_kernel():
    regs = _registrations()
    assert set(regs) == set(REFERENCE_OPS)
    for name, host in REFERENCE_OPS.items():
        assert regs[name][0] == host, name


def test_every_called_entry_is_declared():
    declared = set(re.findall(r"\b(b2_\w+)\s*\(", HEADER.read_text()))
    called = set(re.findall(r"\b(b2_\w+)\s*[(<>]", SHIM.read_text())) | set(
        re.findall(r"<(b2_\w+)>", SHIM.read_text()))
    called -= {"b2_stream_t", "b2_status_t"}
    assert called, "no library calls found"
    assert called <= declared, sorted(called - declared)


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_shim_type_checks_against_the_abi_header():
    cmd = ["g++", "-std=c++17", "-fsyntax-only", "-Wall", "-Wextra", "-Werror",
           "-I", str(ROOT / "tests" / "tf_stub"), "-I", str(ROOT / "include"), str(SHIM)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
