// Stand-in for TensorFlow's op_kernel.h (see tensor_shape.h here): the
// OpKernel / OpKernelConstruction / OpKernelContext members, status helpers
// and registration macros that the GPU kernel shim uses.
#pragma once
#include <string>
#include <vector>
#include "tensorflow/core/framework/tensor.h"
#include "tensorflow/core/framework/tensor_shape.h"

struct CUstream_st;
namespace Eigen {
using gpuStream_t = CUstream_st*;  // cudaStream_t
struct GpuDevice {
  const gpuStream_t& stream() const;
};
}  // namespace Eigen

namespace tensorflow {
class Status {
 public:
  Status() = default;
  Status(int code, std::string msg) : code_(code), msg_(std::move(msg)) {}
  bool ok() const { return code_ == 0; }

 private:
  int code_ = 0;
  std::string msg_;
};

namespace errors {
template <typename... Args> Status InvalidArgument(const Args&... args);
template <typename... Args> Status Internal(const Args&... args);
template <typename... Args> Status DeadlineExceeded(const Args&... args);
template <typename... Args> Status ResourceExhausted(const Args&... args);
}  // namespace errors

constexpr const char DEVICE_GPU[] = "GPU";

class OpKernelConstruction {
 public:
  Status GetAttr(const char* name, std::vector<int32_t>* value) const;
  Status GetAttr(const char* name, std::string* value) const;
  Status GetAttr(const char* name, float* value) const;
  void CtxFailure(const Status& s);
};

class OpKernelContext {
 public:
  const Tensor& input(int index) const;
  Status allocate_output(int index, const TensorShape& shape, Tensor** out);
  const Eigen::GpuDevice& eigen_gpu_device() const;
  const Status& status() const;
  void CtxFailure(const Status& s);
};

class OpKernel {
 public:
  explicit OpKernel(OpKernelConstruction* context);
  virtual ~OpKernel();
  virtual void Compute(OpKernelContext* context) = 0;
};

#define OP_REQUIRES(CTX, EXP, STATUS) \
  do {                                \
    if (!(EXP)) {                     \
      (CTX)->CtxFailure((STATUS));    \
      return;                         \
    }                                 \
  } while (0)

#define OP_REQUIRES_OK(CTX, ...)                \
  do {                                          \
    const ::tensorflow::Status _s(__VA_ARGS__); \
    if (!_s.ok()) {                             \
      (CTX)->CtxFailure(_s);                    \
      return;                                   \
    }                                           \
  } while (0)

namespace register_kernel {
class Name {
 public:
  explicit Name(const char* op);
  Name& Device(const char* device_type);
  Name& HostMemory(const char* arg_name);
  int Build();
};
}  // namespace register_kernel

template <typename Kernel>
int RegisterKernelFactory(int def) {
  OpKernel* (*factory)(OpKernelConstruction*) = [](OpKernelConstruction* c) -> OpKernel* {
    return new Kernel(c);
  };
  (void)factory;
  return def;
}

#define REGISTER_KERNEL_BUILDER(kernel_builder, ...) \
  REGISTER_KERNEL_BUILDER_UNIQ_HELPER(__COUNTER__, kernel_builder, __VA_ARGS__)
#define REGISTER_KERNEL_BUILDER_UNIQ_HELPER(ctr, kernel_builder, ...) \
  REGISTER_KERNEL_BUILDER_UNIQ(ctr, kernel_builder, __VA_ARGS__)
#define REGISTER_KERNEL_BUILDER_UNIQ(ctr, kernel_builder, ...)             \
  static const int registrar__body__##ctr##__object =                      \
      ::tensorflow::RegisterKernelFactory<__VA_ARGS__>(                    \
          ::tensorflow::register_kernel::kernel_builder.Build())
}  // namespace tensorflow
