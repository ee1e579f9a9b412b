"""B200 backend for the seven custom ops of OpenCL-Tensorflow 0.3.0.

Importing this package (as importing the reference's ``opencl_tf`` does,
opencl_tf/__init__.py:19-42):

* loads the compiled op library (``libb2ocl.so``: hand-written sm_100a CUDA
  behind the C ABI of ``include/b2_opencl_tf.h``) -- ImportError if missing;
* registers the gradient of every differentiable op;
* exposes one function per op and the layers.

Ops: conv2d (+ backprop_input / backprop_filter), depthwise_conv2d (+ both
backprops), relu (+ grad), batch_norm_training / batch_norm_inference /
batch_norm_grad, sigmoid (+ grad), dense (+ backprop_input / _weight /
_bias), upsampling_bilinear_2d (+ grad).

Layers (``opencl_tf.layers``): OpenCLConv2D, OpenCLDepthwiseConv2D,
OpenCLBatchNormalization, OpenCLReLU, OpenCLSigmoid, OpenCLDense,
OpenCLUpSampling2D.

Beyond the reference's op set: ``fused_ops`` (BatchNorm -> ReLU in one op),
``step_ops`` (the MSE loss of the training recipe) and ``optimizers.Adam``
(Keras Adam as one multi-tensor kernel); ``train.TrainStep`` runs the whole
training step from one CUDA graph.
"""

from ._library import (raw_ops, fused_ops, step_ops, init, pool_stats, pool_trim, device_timeouts, stream_status,
                       set_wait_limit_ns, set_reserved_sms, library_path)
from .ops import (
    conv2d,
    conv2d_backprop_input,
    conv2d_backprop_filter,
    depthwise_conv2d,
    depthwise_conv2d_backprop_input,
    depthwise_conv2d_backprop_filter,
    relu,
    relu_grad,
    batch_norm_training,
    batch_norm_inference,
    batch_norm_grad,
    sigmoid,
    sigmoid_grad,
    dense,
    dense_backprop_input,
    dense_backprop_weight,
    dense_backprop_bias,
    upsampling_bilinear_2d,
    upsampling_bilinear_2d_grad,
)
from . import errors  # noqa: F401
from . import gradients  # noqa: F401  -- registers the gradient functions
from . import layers  # noqa: F401
from . import optimizers  # noqa: F401

__all__ = [
    "raw_ops",
    "conv2d", "conv2d_backprop_input", "conv2d_backprop_filter",
    "depthwise_conv2d", "depthwise_conv2d_backprop_input", "depthwise_conv2d_backprop_filter",
    "relu", "relu_grad",
    "batch_norm_training", "batch_norm_inference", "batch_norm_grad",
    "sigmoid", "sigmoid_grad",
    "dense", "dense_backprop_input", "dense_backprop_weight", "dense_backprop_bias",
    "upsampling_bilinear_2d", "upsampling_bilinear_2d_grad",
    "fused_ops", "step_ops", "optimizers",
    "layers", "errors", "init", "pool_stats", "pool_trim", "device_timeouts", "stream_status",
    "set_wait_limit_ns", "set_reserved_sms", "library_path",
]

__version__ = "0.3.0+b200"
