// conv_common.cuh -- attribute parsing and geometry shared by the Conv2D and
// DepthwiseConv2D entry points.
#pragma once

#include "b2_internal.cuh"

namespace b2 {

struct ConvGeom {
  int64_t N = 0, H = 0, W = 0, Ci = 0;  // input NHWC
  int64_t kH = 0, kW = 0;               // filter taps
  int64_t Co = 0;                       // output channels (Ci*dm for depthwise)
  int64_t dm = 1;                       // depth multiplier (depthwise only)
  int64_t sH = 1, sW = 1;               // strides[1], strides[2]
  int64_t Ho = 0, Wo = 0, pH = 0, pW = 0;
  bool same = true;

  int64_t in_elems() const { return N * H * W * Ci; }
  int64_t out_elems() const { return N * Ho * Wo * Co; }
  int64_t filter_elems() const { return kH * kW * Ci * (dm > 1 ? dm : (Co / (Ci ? Ci : 1))); }
};

// strides / padding attrs.  `forward` adds the checks the forward ops make in
// their constructors (src/ops/conv2d_ops.cc:101-104,
// src/ops/depthwise_conv2d_ops.cc:101-104); the backprop ops only read
// strides[1] and strides[2].  Non-positive strides are rejected (the
// reference would divide by zero).
inline int parse_conv_attrs(const int32_t* strides, int num_strides, const char* padding, bool forward,
                            ConvGeom* g) {
  B2_REQUIRE(strides != nullptr && num_strides >= 4, "strides must have at least 4 elements");
  if (forward) {
    B2_REQUIRE(num_strides == 4, "strides must be length 4 (NHWC)");
    B2_REQUIRE(strides[0] == 1 && strides[3] == 1, "strides on N and C must be 1");
  }
  B2_REQUIRE(strides[1] > 0 && strides[2] > 0, "strides must be positive");
  B2_RETURN_IF_ERROR(parse_padding(padding, &g->same));
  g->sH = strides[1];
  g->sW = strides[2];
  return B2_OK;
}

inline void finish_geom(ConvGeom* g) {
  resolve_padding(g->H, g->kH, g->sH, g->same, &g->Ho, &g->pH);
  resolve_padding(g->W, g->kW, g->sW, g->same, &g->Wo, &g->pW);
}

inline int check_dims_nonneg(const int64_t* s, int n, const char* what) {
  B2_REQUIRE(s != nullptr, "%s shape missing", what);
  for (int i = 0; i < n; ++i) B2_REQUIRE(s[i] >= 0, "%s has a negative dimension", what);
  return B2_OK;
}

inline int check_int32_sizes(const ConvGeom& g) {
  B2_REQUIRE(g.in_elems() <= kMaxInt32 && g.out_elems() <= kMaxInt32 && g.Ho >= 0 && g.Wo >= 0,
             "tensor too large for this op (more than 2^31 elements)");
  return B2_OK;
}

// Narrow-filter Conv2D on the CUDA cores (conv_direct.cu): eligible when
// Ci, Co <= 32 and kH*kW*Ci*Co <= 4608.  Callers have checked the shapes and
// the 2^31-element limits.
bool conv_direct_ok(const ConvGeom& g);
int conv_direct_forward(const ConvGeom& g, const float* x, const float* w, float* y, cudaStream_t s);
int conv_direct_backprop_input(const ConvGeom& g, const float* dy, const float* w, float* dx, cudaStream_t s);
int conv_direct_backprop_filter(const ConvGeom& g, const float* x, const float* dy, float* dw, cudaStream_t s);

}  // namespace b2
