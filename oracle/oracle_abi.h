/* oracle_abi.h -- TEST INFRASTRUCTURE (oracle).  Only tests/, the smoke check
 * and bench.py's CPU-baseline leg load the libraries declared here.
 *
 * One C ABI, two implementations of the reference's path on host memory:
 *   ORC_PREFIX=ref_   oracle/_ref/libref_ocl.so : the reference's own
 *                     kernels/*.cl compiled through cl_shim.h, driven the
 *                     way src/ops/*.cc launch them (ref_driver.cc)
 *   ORC_PREFIX=port_  oracle/liboracle_port.so  : a plain-C restatement
 *                     of the same arithmetic (port.c)
 *
 * Arguments follow the reference ops (src/ops/*.cc): NHWC float tensors,
 * HWIO filters, int dims, `same` = 1 for padding "SAME", 0 for "VALID".
 * Every function returns 0, or -1 for an argument the reference op would
 * reject with InvalidArgument.  Work-items run as an OpenMP loop; set the
 * thread count with <prefix>set_threads (1 = a fixed, reproducible order
 * for the float atomics of the upsampling backward).
 */
#ifndef B2_ORACLE_ABI_H_
#define B2_ORACLE_ABI_H_

#ifndef ORC_PREFIX_CAT
#define ORC_PREFIX_CAT2(p, n) p##n
#define ORC_PREFIX_CAT(p, n) ORC_PREFIX_CAT2(p, n)
#endif
#define ORC(name) ORC_PREFIX_CAT(ORC_PREFIX, name)

#ifdef __cplusplus
extern "C" {
#endif

void ORC(set_threads)(int n);
int ORC(get_threads)(void);
int ORC(resolve_padding)(int in_size, int k, int stride, int same,
                         int* out_size, int* pad_before);

int ORC(conv2d)(const float* x, const float* w, float* y, int N, int H, int W,
                int Ci, int kH, int kW, int Co, int sH, int sW, int same);
int ORC(conv2d_backprop_input)(const float* dy, const float* w, float* dx,
                               int N, int H, int W, int Ci, int kH, int kW,
                               int Co, int sH, int sW, int same);
int ORC(conv2d_backprop_filter)(const float* x, const float* dy, float* dw,
                                int N, int H, int W, int Ci, int kH, int kW,
                                int Co, int sH, int sW, int same);

int ORC(depthwise_conv2d)(const float* x, const float* w, float* y, int N,
                          int H, int W, int C, int kH, int kW, int dm, int sH,
                          int sW, int same);
int ORC(depthwise_conv2d_backprop_input)(const float* dy, const float* w,
                                         float* dx, int N, int H, int W, int C,
                                         int kH, int kW, int dm, int sH, int sW,
                                         int same);
int ORC(depthwise_conv2d_backprop_filter)(const float* x, const float* dy,
                                          float* dw, int N, int H, int W,
                                          int C, int kH, int kW, int dm,
                                          int sH, int sW, int same);

int ORC(relu)(const float* x, float* y, long n);
int ORC(relu_grad)(const float* gradients, const float* features,
                   float* backprops, long n);
int ORC(sigmoid)(const float* x, float* y, long n);
int ORC(sigmoid_grad)(const float* y, const float* dy, float* grad_x, long n);

int ORC(batch_norm_training)(const float* x, const float* gamma,
                             const float* beta, float* y, float* saved_mean,
                             float* saved_var, int N, int H, int W, int C,
                             float epsilon);
int ORC(batch_norm_inference)(const float* x, const float* gamma,
                              const float* beta, const float* mean,
                              const float* var, float* y, int N, int H, int W,
                              int C, float epsilon);
int ORC(batch_norm_grad)(const float* grad_y, const float* x,
                         const float* gamma, const float* saved_mean,
                         const float* saved_var, float* grad_x,
                         float* grad_gamma, float* grad_beta, int N, int H,
                         int W, int C, float epsilon);

int ORC(dense)(const float* x, const float* w, const float* b, float* y,
               int batch, int in_f, int out_f);
int ORC(dense_backprop_input)(const float* grad_y, const float* w,
                              float* grad_x, int batch, int in_f, int out_f);
int ORC(dense_backprop_weight)(const float* x, const float* grad_y,
                               float* grad_w, int batch, int in_f, int out_f);
int ORC(dense_backprop_bias)(const float* grad_y, float* grad_b, int batch,
                             int out_f);

int ORC(upsampling_bilinear2d)(const float* x, float* y, int N, int H, int W,
                               int C, int sy, int sx);
int ORC(upsampling_bilinear2d_grad)(const float* grad_out, float* grad_in,
                                    int N, int H, int W, int C, int sy,
                                    int sx);

#ifdef __cplusplus
}
#endif

#endif  // B2_ORACLE_ABI_H_
