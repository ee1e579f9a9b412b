/* b2_opencl_tf.h -- C ABI of the B200 backend for the seven custom ops of
 * amanzargari/OpenCL-Tensorflow 0.3.0 (Conv2D, DepthwiseConv2D,
 * BatchNormalization, ReLU, Dense, bilinear UpSampling2D, Sigmoid; forward
 * and backward).
 *
 * One entry point per reference op (the 19 REGISTER_OPs in src/ops).
 * Each entry replaces the body of that op's OpKernel::Compute: the caller
 * (a TF DEVICE_GPU OpKernel, the torch frontend in opencl_tf/, or any C
 * program) owns every input and output buffer and passes device pointers;
 * this library validates shapes and attrs exactly where the reference does,
 * then enqueues the work on the caller's stream and returns without
 * synchronising.  The CLBackend singleton, its per-call clCreateBuffer
 * copies and its global queue mutex (src/cl_backend.h:32-98) are gone:
 *
 *   - pointers are device (HBM) pointers owned by the caller; shape tensors
 *     that the reference marks HostMemory (input_sizes, filter_sizes) are
 *     host arrays here;
 *   - calls are asynchronous on `stream` (a cudaStream_t; NULL means the
 *     legacy default stream) and safe to make from several host threads at
 *     once -- no global lock, state is per device;
 *   - scratch memory (reduction partials) comes from a per-device,
 *     stream-ordered caching pool (cudaMallocAsync on a dedicated memory
 *     pool), which is also legal inside CUDA-graph capture;
 *   - the return value is B2_OK or a b2_status_t code; b2_last_error()
 *     returns this thread's message for the last failed call.  A TF shim maps
 *     B2_ERR_INVALID_ARGUMENT to errors::InvalidArgument and every other code
 *     to errors::Internal, as the reference's OP_REQUIRES / OP_REQUIRES_CL do
 *     (src/ops/conv2d_ops.cc:43-45, 101-122).
 *
 * Layouts are the reference's: activations NHWC, conv filters HWIO
 * [kH,kW,Cin,Cout], depthwise filters [kH,kW,C,dm], dense W [in_f,out_f],
 * all float32, dense row-major with no padding between rows.
 * `strides` is the NHWC stride attr (length >= 4) and `padding` the attr
 * string "SAME" or "VALID".
 */
#ifndef B2_OPENCL_TF_H_
#define B2_OPENCL_TF_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B2_ABI_VERSION 1

typedef void* b2_stream_t; /* cudaStream_t */

typedef enum b2_status {
  B2_OK = 0,
  B2_ERR_INVALID_ARGUMENT = 1, /* shape / attr problem (InvalidArgument)   */
  B2_ERR_INTERNAL = 2,         /* CUDA runtime / launch failure (Internal) */
  B2_ERR_OUT_OF_MEMORY = 3,    /* scratch pool could not grow              */
  B2_ERR_NO_DEVICE = 4,        /* no usable sm_100 device                  */
  B2_ERR_TIMEOUT = 5           /* a bounded device-side wait gave up       */
} b2_status_t;

/* ---------------------------------------------------------------- runtime */

/* Replaces CLBackend::Instance() device probing (src/cl_backend.cc:21-95):
 * selects `device` for the calling thread, checks it is compute capability
 * 10.x and warms the per-device state.  Optional: every op initialises its
 * device lazily (the device current on the calling thread). */
int b2_init(int device);

/* Message for the last non-OK return on this thread ("" if none). */
const char* b2_last_error(void);

int b2_abi_version(void);

/* Replaces opencl_tf::ResolvePadding (src/padding_utils.h:22-33). */
int b2_resolve_padding(int64_t in_size, int64_t k, int64_t stride,
                       const char* padding, int64_t* out_size,
                       int64_t* pad_before);

/* Output shape of OpenclConv2d / OpenclDepthwiseConv2d, as their shape
 * functions compute it (src/ops/conv2d_ops.cc:58-94,
 * src/ops/depthwise_conv2d_ops.cc:55-92). */
int b2_conv2d_output_shape(const int64_t input_shape[4],
                           const int64_t filter_shape[4],
                           const int32_t* strides, int num_strides,
                           const char* padding, int64_t out_shape[4]);
int b2_depthwise_conv2d_output_shape(const int64_t input_shape[4],
                                     const int64_t filter_shape[4],
                                     const int32_t* strides, int num_strides,
                                     const char* padding,
                                     int64_t out_shape[4]);

/* Caching pool for scratch (the buffer pool the reference lacks,
 * docs/ARCHITECTURE.md:141-149).  Stats are for the calling thread's current
 * device. */
typedef struct b2_pool_stats {
  uint64_t bytes_in_use;   /* scratch currently handed out             */
  uint64_t bytes_reserved; /* held by the pool, including cached bytes */
  uint64_t peak_in_use;
  uint64_t num_allocs;     /* scratch requests served                  */
} b2_pool_stats_t;

int b2_pool_stats(b2_pool_stats_t* out);
/* Return cached, unused pool memory to the driver (after synchronising). */
int b2_pool_trim(void);

/* Kernels this library has enqueued since it was loaded (all devices). */
int b2_kernel_launch_count(uint64_t* count);

/* Leave `count` SMs of every device free of this library's persistent
 * (one-CTA-per-SM) tensor-core kernels, for kernels that must run beside
 * them -- NCCL's all-reduce during data-parallel training, which otherwise
 * waits for SMs until the GEMM in flight ends.  0 (the default) uses every
 * SM.  Split-K GEMMs size their splits to the remaining SMs, so their sums
 * are added in a different (still fixed) order than with 0.  Applies to
 * launches after the call (a captured graph keeps its grids). */
int b2_set_reserved_sms(int count);

/* ------------------------------------------------------------- Conv2D */

/* OpenclConv2d(input, filter; strides, padding) -> output
 * src/ops/conv2d_ops.cc:53-197.  output: out_shape from
 * b2_conv2d_output_shape. */
int b2_conv2d(b2_stream_t stream, const float* input,
              const int64_t input_shape[4], const float* filter,
              const int64_t filter_shape[4], const int32_t* strides,
              int num_strides, const char* padding, float* output,
              const int64_t output_shape[4]);

/* OpenclConv2dBackpropInput(input_sizes[HostMemory], filter, out_backprop)
 * src/ops/conv2d_ops.cc:203-322.  output: [input_sizes]. */
int b2_conv2d_backprop_input(b2_stream_t stream, const int32_t input_sizes[4],
                             const float* filter,
                             const int64_t filter_shape[4],
                             const float* out_backprop,
                             const int64_t out_backprop_shape[4],
                             const int32_t* strides, int num_strides,
                             const char* padding, float* output);

/* OpenclConv2dBackpropFilter(input, filter_sizes[HostMemory], out_backprop)
 * src/ops/conv2d_ops.cc:328-448.  output: [filter_sizes]. */
int b2_conv2d_backprop_filter(b2_stream_t stream, const float* input,
                              const int64_t input_shape[4],
                              const int32_t filter_sizes[4],
                              const float* out_backprop,
                              const int64_t out_backprop_shape[4],
                              const int32_t* strides, int num_strides,
                              const char* padding, float* output);

/* ---------------------------------------------------- DepthwiseConv2D */

/* OpenclDepthwiseConv2d -- src/ops/depthwise_conv2d_ops.cc:49-192 */
int b2_depthwise_conv2d(b2_stream_t stream, const float* input,
                        const int64_t input_shape[4], const float* filter,
                        const int64_t filter_shape[4], const int32_t* strides,
                        int num_strides, const char* padding, float* output,
                        const int64_t output_shape[4]);

/* OpenclDepthwiseConv2dBackpropInput -- depthwise_conv2d_ops.cc:198-312 */
int b2_depthwise_conv2d_backprop_input(
    b2_stream_t stream, const int32_t input_sizes[4], const float* filter,
    const int64_t filter_shape[4], const float* out_backprop,
    const int64_t out_backprop_shape[4], const int32_t* strides,
    int num_strides, const char* padding, float* output);

/* OpenclDepthwiseConv2dBackpropFilter -- depthwise_conv2d_ops.cc:318-433 */
int b2_depthwise_conv2d_backprop_filter(
    b2_stream_t stream, const float* input, const int64_t input_shape[4],
    const int32_t filter_sizes[4], const float* out_backprop,
    const int64_t out_backprop_shape[4], const int32_t* strides,
    int num_strides, const char* padding, float* output);

/* ---------------------------------------------------------------- ReLU */

/* OpenclRelu -- src/ops/relu_ops.cc:40-93.  y = fmax(x, 0); bit-exact. */
int b2_relu(b2_stream_t stream, const float* input, float* output,
            int64_t num_elements);

/* OpenclReluGrad(gradients, features) -- src/ops/relu_ops.cc:101-165.
 * backprops = features > 0 ? gradients : 0; bit-exact. */
int b2_relu_grad(b2_stream_t stream, const float* gradients,
                 const float* features, float* backprops,
                 int64_t num_elements);

/* ------------------------------------------------------------- Sigmoid */

/* OpenclSigmoid -- src/ops/sigmoid_ops.cc:49-103 */
int b2_sigmoid(b2_stream_t stream, const float* input, float* output,
               int64_t num_elements);

/* OpenclSigmoidGrad(y, dy) -- src/ops/sigmoid_ops.cc:110-175.
 * grad_x = dy * y * (1 - y), y the forward OUTPUT. */
int b2_sigmoid_grad(b2_stream_t stream, const float* y, const float* dy,
                    float* grad_x, int64_t num_elements);

/* ---------------------------------------------------------- BatchNorm */

/* OpenclBatchNormTraining(x, gamma, beta; epsilon) -> (y, saved_mean,
 * saved_var) -- src/ops/batchnorm_ops.cc:64-186.  saved_var is the biased
 * batch variance E[x^2] - mean^2. */
int b2_batch_norm_training(b2_stream_t stream, const float* x,
                           const int64_t x_shape[4], const float* gamma,
                           int64_t gamma_len, const float* beta,
                           int64_t beta_len, float epsilon, float* y,
                           float* saved_mean, float* saved_var);

/* The computation of b2_batch_norm_training, for callers that must not
 * have device memory allocated during a call -- a runtime whose memory
 * manager owns all of HBM, or a warm serving loop that cannot accept an
 * allocation's synchronisation and latency.  It has no counterpart in the
 * reference.  Its outputs equal b2_batch_norm_training's within the fp32
 * tolerance; they are bit-identical only while C <= 55: for more channels
 * the statistics are summed over fewer row-block partials (so that they fit
 * the fixed array below), which changes the order of the additions.  Its
 * reduction scratch is a fixed 256 KiB array in the library's device image
 * (held on every GPU that loads the library until exit), so it accepts at
 * most 16384 channels and returns B2_ERR_INVALID_ARGUMENT beyond that.  The
 * first call on each device looks up that array's device address
 * (cudaGetSymbolAddress); make that first call before any stream capture (a
 * failed lookup is retried by the next call).
 * All calls on a device share the array: calls whose work overlaps on the GPU
 * (different streams, no ordering between them) race and corrupt each
 * other's statistics, so order them (e.g. issue them on one stream). */
int b2_batch_norm_training_no_alloc(b2_stream_t stream, const float* x,
                                    const int64_t x_shape[4],
                                    const float* gamma, int64_t gamma_len,
                                    const float* beta, int64_t beta_len,
                                    float epsilon, float* y, float* saved_mean,
                                    float* saved_var);

/* OpenclBatchNormTraining followed by OpenclRelu on its output, in one call:
 * z = relu(BN(x)) with the statistics of b2_batch_norm_training; z is bit-for-
 * bit the two ops in sequence (src/ops/batchnorm_ops.cc:87-180 then
 * src/ops/relu_ops.cc), with one pass over x and no intermediate tensor.  When
 * moving_mean / moving_var are not NULL it also applies the layer's
 * moving-average update exactly as b2_batch_norm_update_moving would (same
 * rounding), in the statistics pass.  Not an op of the reference: the fusion
 * of the pair its layers run back to back. */
int b2_batch_norm_relu_training(b2_stream_t stream, const float* x,
                                const int64_t x_shape[4], const float* gamma,
                                int64_t gamma_len, const float* beta,
                                int64_t beta_len, float epsilon, float* z,
                                float* saved_mean, float* saved_var,
                                float* moving_mean, float* moving_var,
                                float momentum, float one_minus_momentum);

/* The gradient of b2_batch_norm_relu_training: OpenclReluGrad followed by
 * OpenclBatchNormGrad (src/ops/relu_ops.cc, src/ops/batchnorm_ops.cc:313-416)
 * given grad_z; the ReLU mask (BN(x) > 0) is recomputed from x, the saved
 * statistics, gamma and beta exactly as the forward computed it, so the
 * results equal the two ops in sequence bit for bit. */
int b2_batch_norm_relu_grad(b2_stream_t stream, const float* grad_z,
                            const int64_t grad_z_shape[4], const float* x,
                            const int64_t x_shape[4], const float* gamma,
                            const float* beta, const float* saved_mean,
                            const float* saved_var, float epsilon,
                            float* grad_x, float* grad_gamma, float* grad_beta);

/* The Keras layer's moving-statistics update after a training step,
 * opencl_tf/layers.py:189-194: for c < channels,
 *   moving_mean[c] = momentum * moving_mean[c] + one_minus_momentum * batch_mean[c]
 *   moving_var[c]  = momentum * moving_var[c]  + one_minus_momentum * batch_var[c]
 * with both products and the sum rounded to fp32 (the reference's three
 * tensor ops).  one_minus_momentum is passed as the caller rounds 1 -
 * momentum (the reference: in double, then to fp32).  Not an op of the
 * reference's kernel library: it fuses the four elementwise ops the layer
 * runs into one launch. */
int b2_batch_norm_update_moving(b2_stream_t stream, float* moving_mean,
                                float* moving_var, const float* batch_mean,
                                const float* batch_var, int64_t channels,
                                float momentum, float one_minus_momentum);

/* OpenclBatchNormInference(x, gamma, beta, mean, var; epsilon) -> y
 * src/ops/batchnorm_ops.cc:192-282 */
int b2_batch_norm_inference(b2_stream_t stream, const float* x,
                            const int64_t x_shape[4], const float* gamma,
                            int64_t gamma_len, const float* beta,
                            int64_t beta_len, const float* mean,
                            int64_t mean_len, const float* var,
                            int64_t var_len, float epsilon, float* y);

/* OpenclBatchNormGrad(grad_y, x, gamma, saved_mean, saved_var; epsilon)
 * -> (grad_x, grad_gamma, grad_beta) -- src/ops/batchnorm_ops.cc:288-422 */
int b2_batch_norm_grad(b2_stream_t stream, const float* grad_y,
                       const int64_t grad_y_shape[4], const float* x,
                       const int64_t x_shape[4], const float* gamma,
                       const float* saved_mean, const float* saved_var,
                       float epsilon, float* grad_x, float* grad_gamma,
                       float* grad_beta);

/* --------------------------------------------------------------- Dense */

/* OpenclDense(x, w, b) -> y = b + x . W -- src/ops/dense_ops.cc:57-146 */
int b2_dense(b2_stream_t stream, const float* x, const int64_t x_shape[2],
             const float* w, const int64_t w_shape[2], const float* b,
             int64_t b_len, float* y);

/* OpenclDense then OpenclRelu fused: y = relu(b + x . W), the ReLU applied
 * where each sum is finished; the same bits as b2_dense then b2_relu.
 * Replaces the pair src/ops/dense_ops.cc:57-146 + src/ops/relu_ops.cc:40-93
 * (the README model's Dense(128, activation="relu") head). */
int b2_dense_relu(b2_stream_t stream, const float* x, const int64_t x_shape[2],
                  const float* w, const int64_t w_shape[2], const float* b,
                  int64_t b_len, float* y);

/* OpenclDenseBackpropInput(grad_y, w) -> grad_y . W^T
 * src/ops/dense_ops.cc:152-230 */
int b2_dense_backprop_input(b2_stream_t stream, const float* grad_y,
                            const int64_t grad_y_shape[2], const float* w,
                            const int64_t w_shape[2], float* grad_x);

/* OpenclDenseBackpropWeight(x, grad_y) -> x^T . grad_y
 * src/ops/dense_ops.cc:236-314 */
int b2_dense_backprop_weight(b2_stream_t stream, const float* x,
                             const int64_t x_shape[2], const float* grad_y,
                             const int64_t grad_y_shape[2], float* grad_w);

/* OpenclDenseBackpropBias(grad_y) -> sum over batch
 * src/ops/dense_ops.cc:320-382 */
int b2_dense_backprop_bias(b2_stream_t stream, const float* grad_y,
                           const int64_t grad_y_shape[2], float* grad_b);

/* --------------------------------------------------- UpSampling2D (bilinear) */

/* OpenclUpsamplingBilinear2d(input; size) -- src/ops/upsampling_ops.cc:59-159.
 * Half-pixel centres, clamped corners; output [N, H*size[0], W*size[1], C]. */
int b2_upsampling_bilinear2d(b2_stream_t stream, const float* input,
                             const int64_t input_shape[4],
                             const int32_t* size, int num_size,
                             float* output);

/* OpenclUpsamplingBilinear2dGrad(grad_out, input_sizes[HostMemory]; size)
 * src/ops/upsampling_ops.cc:166-272.  Deterministic gather form of the
 * reference's zero-fill + float-atomic scatter. */
int b2_upsampling_bilinear2d_grad(b2_stream_t stream, const float* grad_out,
                                  const int64_t grad_out_shape[4],
                                  const int32_t input_sizes[4],
                                  const int32_t* size, int num_size,
                                  float* grad_in);

/* Per-axis source coordinates the upsampling kernels use, written to device
 * arrays of length out_size: clamped lower / upper source index and the
 * fraction (kernels/upsampling_bilinear_kernels.cl:51-64).  Exposed so the
 * index and weight arithmetic can be checked bit for bit. */
int b2_upsampling_coords(b2_stream_t stream, int32_t in_size,
                         int32_t out_size, int32_t* lo, int32_t* hi,
                         float* frac);

/* ---- The training step around the ops ----------------------------------
 * The reference trains with model.compile(optimizer=tf.keras.optimizers.Adam(
 * 1e-3), loss="mse") (README.md:188-196); loss and optimizer are stock
 * TensorFlow (2.10-2.15) host ops.  These entries replace them on the device;
 * they are not ops of the reference's kernel library. */

/* Keras "mse" for one batch: *loss = sum((pred - target)^2) / num_elements
 * (the mean over the last axis, then over the batch, is the same mean).  One
 * cluster of 8 CTAs, deterministic; `loss` is a device float. */
int b2_mse_loss(b2_stream_t stream, const float* pred, const float* target,
                int64_t num_elements, float* loss);

/* Gradient of b2_mse_loss: grad_pred = (pred - target) * (2 * grad_loss /
 * num_elements), grad_loss a device float (the upstream gradient). */
int b2_mse_loss_grad(b2_stream_t stream, const float* pred,
                     const float* target, int64_t num_elements,
                     const float* grad_loss, float* grad_pred);

/* Keras Adam's update of num_tensors parameter tensors (params[i], grads[i],
 * m[i], v[i]: device fp32 arrays of sizes[i] elements; the pointer arrays are
 * host memory), keras/optimizers/adam.py (TF 2.11+) / ApplyAdam (TF 2.10):
 *   t = *iterations + 1,  alpha = lr * sqrt(1 - beta_2^t) / (1 - beta_1^t)
 *   m += (g - m) * one_minus_beta_1;  v += (g*g - v) * one_minus_beta_2
 *   p -= (m * alpha) / (sqrt(v) + epsilon)
 * then *iterations = t.  one_minus_beta_* are passed as the caller rounds
 * them (Keras: 1 - beta in double, then fp32).  `iterations` (int64) and
 * `ticket` (uint32, zero before the first call; the kernel leaves it zero)
 * are device memory owned by the optimizer, so the update replays correctly
 * from a captured CUDA graph.  Calls sharing one ticket must be ordered. */
int b2_adam_update(b2_stream_t stream, int num_tensors, float* const* params,
                   const float* const* grads, float* const* m,
                   float* const* v, const int64_t* sizes,
                   float learning_rate, float beta_1, float beta_2,
                   float one_minus_beta_1, float one_minus_beta_2,
                   float epsilon, int64_t* iterations, unsigned int* ticket);

/* Number of bounded device-side waits (tensor-core pipeline barriers) that
 * expired since the library was loaded; synchronise the stream first.  A
 * nonzero count means a kernel gave up waiting and its output is invalid. */
int b2_device_timeouts(unsigned int* count);

/* ---- Gradient exchange over NVLink peer memory (data parallelism) --------
 * No reference op: the reference trains on one device.  Averages a small
 * fp32 tensor across the `world` ranks (GPUs of one node, one process each)
 * in one kernel per rank: each rank stores its copy into every rank's
 * exchange block, raises a flag there, waits (bounded: an expired wait makes
 * later calls return B2_ERR_TIMEOUT) for every rank's flag and adds the copies
 * in rank order, so every rank gets the same bits.  Every rank must make the
 * same calls in the same order.
 *
 * Setup, once per rank: b2_peer_buffer_create(b2_peer_exchange_bytes(n,
 * world)) gives this rank's block and a 64-byte handle; the handles are
 * exchanged between the processes (any host channel), and each rank maps the
 * others' blocks with b2_peer_buffer_open.  peer_blocks[r] is rank r's block
 * as mapped in the calling process (its own block at [rank]); counters: two
 * zeroed uint32 of device memory per rank (call epoch and a ticket). */
size_t b2_peer_exchange_bytes(int64_t n, int world);
int b2_peer_buffer_create(size_t bytes, void** ptr, unsigned char handle[64]);
int b2_peer_buffer_open(const unsigned char handle[64], void** ptr);
int b2_peer_buffer_close(void* peer_ptr);
int b2_peer_buffer_free(void* ptr);
int b2_peer_allreduce_avg(b2_stream_t stream, float* data, int64_t n, int rank,
                          int world, void* const* peer_blocks,
                          unsigned int* counters);

/* ---- Device-side wait failures as op errors ------------------------------
 * The reference turns every device failure into a TF status
 * (OP_REQUIRES_CL -> errors::Internal, src/ops/conv2d_ops.cc:43-45).  Here
 * the ops are asynchronous, so a kernel whose bounded wait expired (its
 * pipeline then tears down cleanly and the context stays usable) records the
 * expiry in host-mapped memory, and:
 *   - every op call made once the expiry is visible returns B2_ERR_TIMEOUT
 *     (the work is still enqueued; its results are invalid), until
 *   - b2_stream_status(stream), which synchronises `stream`, returns
 *     B2_ERR_TIMEOUT once for the expiry and clears it (else B2_OK).
 * The state is process-wide (all devices and streams). */
int b2_stream_status(b2_stream_t stream);

/* Limit of each bounded device-side wait, in nanoseconds, for kernels
 * launched after the call; 0 restores the default (10 s).  A test hook: a
 * very short limit makes a real pipeline's waits run out. */
int b2_set_wait_limit_ns(uint64_t limit_ns);

#ifdef __cplusplus
}
#endif

#endif /* B2_OPENCL_TF_H_ */
