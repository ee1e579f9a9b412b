// Stand-in for TensorFlow's tensor_shape.h: only the members the GPU kernel
// shim uses, declared with TensorFlow's names and signatures, so that
// tests/test_cpu_7_tf_shim.py can type-check the shim where TensorFlow is
// not installed.  Test infrastructure; never linked into anything.
#pragma once
#include <cstdint>
#include <vector>

namespace tensorflow {
class TensorShape {
 public:
  TensorShape() = default;
  void AddDim(int64_t size) { dims_.push_back(size); }
  int dims() const { return static_cast<int>(dims_.size()); }
  int64_t dim_size(int d) const { return dims_[d]; }
  bool operator==(const TensorShape& b) const { return dims_ == b.dims_; }
  bool operator!=(const TensorShape& b) const { return !(*this == b); }

 private:
  std::vector<int64_t> dims_;
};
}  // namespace tensorflow
