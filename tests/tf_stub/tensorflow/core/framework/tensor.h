// Stand-in for TensorFlow's tensor.h (see tensor_shape.h here).
#pragma once
#include <cstdint>
#include "tensorflow/core/framework/tensor_shape.h"

namespace tensorflow {
template <typename T>
struct FlatView {
  T* ptr;
  int64_t n;
  T* data() const { return ptr; }
  int64_t size() const { return n; }
  T& operator()(int64_t i) const { return ptr[i]; }
};

class Tensor {
 public:
  int dims() const { return shape_.dims(); }
  int64_t dim_size(int d) const { return shape_.dim_size(d); }
  int64_t NumElements() const;
  const TensorShape& shape() const { return shape_; }
  template <typename T>
  FlatView<T> flat();
  template <typename T>
  FlatView<const T> flat() const;

 private:
  TensorShape shape_;
};
}  // namespace tensorflow
