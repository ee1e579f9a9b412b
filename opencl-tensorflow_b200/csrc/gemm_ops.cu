// gemm_ops.cu -- Conv2D (forward, input grad, filter grad) and Dense
// (forward, input grad, weight grad, bias grad) on the tcgen05 3xTF32 engine.
//
// Reference kernels: kernels/conv2d_kernels.cl:30-158 and
// kernels/dense_kernels.cl:18-102 (one work-item per output, serial fp32
// loops).  Each op is expressed as D[M,N] = A[M,K] . B[K,N] over views of the
// caller's tensors, without materialising im2col or transposes:
//
//   op                     M            N      K              A view             B view
//   conv2d forward         N*Ho*Wo      Co     kH*kW*Ci       im2col(x)          W[k,co]
//   conv2d input grad      N*H*W        Ci     kH*kW*Co       strided gather dy  W[tap,ci,co]
//   conv2d filter grad     kH*kW*Ci     Co     N*Ho*Wo        im2col(x)^T        dy[p,co]
//   dense forward (+b)     batch        out_f  in_f           x                  W
//   dense input grad       batch        in_f   out_f          dy                 W^T
//   dense weight grad      in_f         out_f  batch          x^T                dy
//
// 1x1 / stride-1 / unpadded convolutions take the plain-matrix views.  When
// the output tiles alone cannot fill the GPU (filter grads, the dense forward
// at small batch) K is split across CTAs; partials are summed in split order
// by a second kernel, so every result is deterministic.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <type_traits>

#include "conv_common.cuh"
#include "tc_gemm.cuh"
#include "tma_gemm.cuh"

namespace b2 {
unsigned int dw_timeouts();    // depthwise.cu
unsigned int peer_timeouts();  // peer_exchange.cu

namespace tc {

// D = sum_z P[z] (+ bias) in a fixed order: CTA (32 elements x kRedParts);
// part j adds splits j, j + kRedParts, ... in order, then the parts are added
// in part order -- deterministic, with all of a CTA's loads in flight at once.
constexpr int kRedParts = 16;
__global__ void __launch_bounds__(32 * kRedParts) splitk_reduce_kernel(const float* __restrict__ part, int splits,
                                                                       int64_t M, int64_t N,
                                                                       const float* __restrict__ bias,
                                                                       float* __restrict__ out, int64_t ldo,
                                                                       int relu) {
  __shared__ float s_part[kRedParts][32];
  const int64_t total = M * N;
  const int64_t i = (int64_t)blockIdx.x * 32 + threadIdx.x;
  float acc = 0.0f;
  if (i < total) {
#pragma unroll 4
    for (int z = threadIdx.y; z < splits; z += kRedParts) acc += __ldg(part + (int64_t)z * total + i);
  }
  s_part[threadIdx.y][threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.y == 0 && i < total) {
    float sum = s_part[0][threadIdx.x];
    for (int j = 1; j < kRedParts; ++j) sum += s_part[j][threadIdx.x];
    const int64_t m = i / N, n = i - m * N;
    if (bias) sum += bias[n];
    out[m * ldo + n] = relu && !(sum > 0.0f) ? 0.0f : sum;
  }
}

// N tile: the whole N when it fits in kMaxBN columns, else balanced tiles of
// at most 128 (multiples of 16, the UMMA N granularity at M = 128).
int choose_bn(int64_t N) {
  if (N <= kMaxBN) return (int)(ceil_div(N < 16 ? 16 : N, 16) * 16);
  const int64_t tiles = ceil_div(N, 128);
  return (int)(ceil_div(ceil_div(N, tiles), 16) * 16);
}

int choose_stages(int bn, int max_smem) {
  const KernelSmem one = smem_plan(bn, 1);
  int st = (int)((max_smem - (int)(one.total - one.stage_bytes)) / (int)one.stage_bytes);
  if (st > kMaxStages) st = kMaxStages;
  if (st < 2) st = 2;
  return st;
}

int splits_for(int64_t tiles, int64_t K, int sm_count, int min_kb_per_split) {
  if (tiles >= sm_count) return 1;
  int64_t s = sm_count / tiles;
  const int64_t cap = ceil_div(K, (int64_t)BK * min_kb_per_split);
  if (s > cap) s = cap;
  return s < 1 ? 1 : (int)s;
}

// ------------------------------------------------------- convolution views

// A of the forward conv: row m = output pixel (n, ho, wo); k = (kh, kw, ci).
struct ConvFpropA {
  const float* x;
  int64_t M;
  int H, W, Ci, kW, sH, sW, pH, pW, Ho, Wo;
  bool vec;  // Ci % 4 == 0 and x 16-byte aligned
  struct Ctx {
    const float* img;
    int hi0, wi0;
    bool valid;
  };
  __device__ Ctx row(int64_t m) const {
    Ctx c;
    c.valid = m < M;
    const uint32_t mm = c.valid ? (uint32_t)m : 0u;  // M < 2^31 (checked on the host)
    const uint32_t t = mm / (uint32_t)Wo;
    const int wo = (int)(mm - t * (uint32_t)Wo);
    const uint32_t n = t / (uint32_t)Ho;
    const int ho = (int)(t - n * (uint32_t)Ho);
    c.img = x + (int64_t)n * H * W * Ci;
    c.hi0 = ho * sH - pH;
    c.wi0 = wo * sW - pW;
    return c;
  }
  __device__ void load8(const Ctx& c, int64_t k0, int64_t k_end, float (&v)[kUnit]) const {
    if (!c.valid) {
      zero_unit(v);
      return;
    }
    if (vec) {
#pragma unroll
      for (int q = 0; q < kUnit / 4; ++q) {
        const int64_t k = k0 + 4 * q;
        float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
        if (k < k_end) {
          const int tap = (int)(k / Ci), ci = (int)(k - (int64_t)tap * Ci);
          const int kh = tap / kW, kw = tap - kh * kW;
          const int hi = c.hi0 + kh, wi = c.wi0 + kw;
          if ((unsigned)hi < (unsigned)H && (unsigned)wi < (unsigned)W)
            t = __ldg(reinterpret_cast<const float4*>(c.img + ((int64_t)hi * W + wi) * Ci + ci));
        }
        v[4 * q] = t.x;
        v[4 * q + 1] = t.y;
        v[4 * q + 2] = t.z;
        v[4 * q + 3] = t.w;
      }
    } else {
      // walk (kh, kw, ci) from k0 without dividing per element
      const uint32_t tap0 = (uint32_t)k0 / (uint32_t)Ci;
      int ci = (int)((uint32_t)k0 - tap0 * (uint32_t)Ci);
      int kh = (int)(tap0 / (uint32_t)kW), kw = (int)(tap0 - (uint32_t)kh * (uint32_t)kW);
#pragma unroll
      for (int i = 0; i < kUnit; ++i) {
        float val = 0.0f;
        if (k0 + i < k_end) {
          const int hi = c.hi0 + kh, wi = c.wi0 + kw;
          if ((unsigned)hi < (unsigned)H && (unsigned)wi < (unsigned)W)
            val = __ldg(c.img + (hi * W + wi) * Ci + ci);
        }
        v[i] = val;
        if (++ci == Ci) {
          ci = 0;
          if (++kw == kW) {
            kw = 0;
            ++kh;
          }
        }
      }
    }
  }
};

// A of the input-gradient conv: row m = input pixel (n, hi, wi);
// k = (kh, kw, co); value dy[n, ho, wo, co] when hi + pH - kh = ho*sH and
// wi + pW - kw = wo*sW land inside the output (conv2d_kernels.cl:97-117).
struct ConvDgradA {
  const float* dy;
  int64_t M;
  int H, W, Co, kW, sH, sW, pH, pW, Ho, Wo;
  bool vec;  // Co % 4 == 0 and dy 16-byte aligned
  struct Ctx {
    const float* img;
    int hn0, wn0;
    bool valid;
  };
  __device__ Ctx row(int64_t m) const {
    Ctx c;
    c.valid = m < M;
    if (!c.valid) m = 0;
    const int wi = (int)(m % W);
    const int64_t t = m / W;
    const int hi = (int)(t % H);
    const int64_t n = t / H;
    c.img = dy + n * Ho * Wo * Co;
    c.hn0 = hi + pH;
    c.wn0 = wi + pW;
    return c;
  }
  __device__ __forceinline__ bool tap_src(const Ctx& c, int tap, int64_t* off) const {
    const int kh = tap / kW, kw = tap - kh * kW;
    const int hn = c.hn0 - kh, wn = c.wn0 - kw;
    if (hn < 0 || wn < 0) return false;
    const int ho = hn / sH, wo = wn / sW;
    if (ho * sH != hn || wo * sW != wn || ho >= Ho || wo >= Wo) return false;
    *off = ((int64_t)ho * Wo + wo) * Co;
    return true;
  }
  __device__ void load8(const Ctx& c, int64_t k0, int64_t k_end, float (&v)[kUnit]) const {
    if (!c.valid) {
      zero_unit(v);
      return;
    }
    if (vec) {
#pragma unroll
      for (int q = 0; q < kUnit / 4; ++q) {
        const int64_t k = k0 + 4 * q;
        float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
        int64_t off;
        if (k < k_end) {
          const int tap = (int)(k / Co), co = (int)(k - (int64_t)tap * Co);
          if (tap_src(c, tap, &off)) t = __ldg(reinterpret_cast<const float4*>(c.img + off + co));
        }
        v[4 * q] = t.x;
        v[4 * q + 1] = t.y;
        v[4 * q + 2] = t.z;
        v[4 * q + 3] = t.w;
      }
    } else {
      int tap = (int)(k0 / Co), co = (int)(k0 - (int64_t)tap * Co);
      int64_t off = 0;
      bool ok = tap_src(c, tap, &off);
#pragma unroll
      for (int i = 0; i < kUnit; ++i) {
        v[i] = (k0 + i < k_end && ok) ? __ldg(c.img + off + co) : 0.0f;
        if (++co == Co) {
          co = 0;
          ++tap;
          ok = tap_src(c, tap, &off);
        }
      }
    }
  }
};

// B of the input-gradient conv: row n = ci; k = (tap, co); value
// W[tap, ci, co] (HWIO).
struct ConvDgradB {
  const float* w;
  int Ci, Co;
  bool vec;  // Co % 4 == 0 and w 16-byte aligned
  struct Ctx {
    int ci;
    bool valid;
  };
  __device__ Ctx row(int64_t n) const { return Ctx{(int)(n < Ci ? n : 0), n < Ci}; }
  __device__ void load8(const Ctx& c, int64_t k0, int64_t k_end, float (&v)[kUnit]) const {
    if (!c.valid) {
      zero_unit(v);
      return;
    }
    if (vec) {
#pragma unroll
      for (int q = 0; q < kUnit / 4; ++q) {
        const int64_t k = k0 + 4 * q;
        float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
        if (k < k_end) {
          const int64_t tap = k / Co, co = k - tap * Co;
          t = __ldg(reinterpret_cast<const float4*>(w + (tap * Ci + c.ci) * Co + co));
        }
        v[4 * q] = t.x;
        v[4 * q + 1] = t.y;
        v[4 * q + 2] = t.z;
        v[4 * q + 3] = t.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < kUnit; ++i) {
        const int64_t k = k0 + i;
        float val = 0.0f;
        if (k < k_end) {
          const int64_t tap = k / Co, co = k - tap * Co;
          val = __ldg(w + (tap * Ci + c.ci) * Co + co);
        }
        v[i] = val;
      }
    }
  }
};

// A of the filter-gradient conv: row m = (kh, kw, ci); k = output pixel p;
// value x[n, ho*sH - pH + kh, wo*sW - pW + kw, ci] (conv2d_kernels.cl:143-156).
struct ConvWgradA {
  const float* x;
  int64_t M;
  int H, W, Ci, kW, sH, sW, pH, pW, Ho, Wo;
  struct Ctx {
    int kh, kw, ci;
    bool valid;
  };
  __device__ Ctx row(int64_t m) const {
    Ctx c;
    c.valid = m < M;
    if (!c.valid) m = 0;
    const int tap = (int)(m / Ci);
    c.ci = (int)(m - (int64_t)tap * Ci);
    c.kh = tap / kW;
    c.kw = tap - c.kh * kW;
    return c;
  }
  __device__ void load8(const Ctx& c, int64_t k0, int64_t k_end, float (&v)[kUnit]) const {
    if (!c.valid) {
      zero_unit(v);
      return;
    }
    const uint32_t t = (uint32_t)k0 / (uint32_t)Wo;  // pixel count < 2^31 (checked on the host)
    int wo = (int)((uint32_t)k0 - t * (uint32_t)Wo);
    uint32_t n = t / (uint32_t)Ho;
    int ho = (int)(t - n * (uint32_t)Ho);
#pragma unroll
    for (int i = 0; i < kUnit; ++i) {
      float val = 0.0f;
      if (k0 + i < k_end) {
        const int hi = ho * sH - pH + c.kh, wi = wo * sW - pW + c.kw;
        if ((unsigned)hi < (unsigned)H && (unsigned)wi < (unsigned)W)
          val = __ldg(x + (((int64_t)n * H + hi) * W + wi) * Ci + c.ci);
      }
      v[i] = val;
      if (++wo == Wo) {
        wo = 0;
        if (++ho == Ho) {
          ho = 0;
          ++n;
        }
      }
    }
  }
};

// ------------------------------------------------- TMA engine (host side)

// A plain matrix operand: op(r, k) = p[r*ld + k] (K-major) or p[k*ld + r].
struct MatOperand {
  const float* p;
  int64_t rows, ld;
  bool k_major;
};

inline MatOperand mat_of(const KContig& v) { return MatOperand{v.p, v.rows, v.ld, true}; }
inline MatOperand mat_of(const MNMajor& v) { return MatOperand{v.p, v.rows, v.ld, false}; }
template <class V>
struct is_mat_view : std::false_type {};
template <>
struct is_mat_view<KContig> : std::true_type {};
template <>
struct is_mat_view<MNMajor> : std::true_type {};

// cuTensorMapEncodeTiled, fetched once through the runtime (no libcuda link).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }();
  return fn;
}

// The TMA engine is on unless B2_TMA_GEMM=0 (then every contraction runs on
// the register-fed engine).
bool tma_engine_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("B2_TMA_GEMM");
    return !(e && e[0] == '0');
  }();
  return on && tensor_map_encoder() != nullptr;
}

constexpr int64_t kI32 = 2147483647;

bool tma_operand_ok(const MatOperand& o, int64_t K) {
  return aligned16(o.p) && o.ld % 4 == 0 && o.rows <= kI32 && K <= kI32 && o.ld <= kI32;
}

int encode_map(CUtensorMap* m, const float* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides,
               const cuuint32_t* box, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  const cuuint32_t elem[3] = {1, 1, 1};
  const CUresult r = tensor_map_encoder()(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (cuuint32_t)rank,
                                          const_cast<float*>(base), dims, strides, box, elem,
                                          CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(B2_ERR_INTERNAL, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return B2_OK;
}

// Operand map: K-major -> dims {K, rows}, box {32, box_rows}, 128-byte
// swizzle; MN-major -> dims {rows, K}, box {32, 32}, with `mn_swizzle` (B:
// the 128-byte swizzle of 32-byte atoms that MN-major tf32 UMMA reads; A:
// none, the converters read it).
int encode_operand(CUtensorMap* m, const MatOperand& o, int64_t K, int box_rows, CUtensorMapSwizzle mn_swizzle) {
  const cuuint64_t strides[1] = {(cuuint64_t)o.ld * 4};
  if (o.k_major) {
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)o.rows};
    const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    return encode_map(m, o.p, 2, dims, strides, box);
  }
  const cuuint64_t dims[2] = {(cuuint64_t)o.rows, (cuuint64_t)K};
  const cuuint32_t box[2] = {32, (cuuint32_t)BK};
  return encode_map(m, o.p, 2, dims, strides, box, mn_swizzle);
}

// N tile of the TMA engine: a multiple of 32 (whole 32-column output blocks),
// at most 128, balanced over the N tiles.
int tma_bn(int64_t N) {
  if (N <= kTmaMaxBN) return (int)(ceil_div(N < 32 ? 32 : N, 32) * 32);
  const int64_t tiles = ceil_div(N, kTmaMaxBN);
  return (int)(ceil_div(ceil_div(N, tiles), 32) * 32);
}

// Operand stages: limited by the TMEM columns left for A slots; raw stages
// take the remaining shared memory.
void tma_stages(int bn, bool use_s, int table_entries, int max_smem, int* raw_stages, int* op_stages,
                int b_res_kb = 0) {
  int q = (int)((kTmemCols - tma_acc_cols(bn, use_s)) / kASlotCols);
  if (q > kTmaMaxOpStages) q = kTmaMaxOpStages;
  const TmaSmem fixed = tma_smem_plan(bn, 0, q, table_entries, b_res_kb);
  int r = (int)((max_smem - (int)fixed.total) / (int)fixed.raw_bytes);
  if (r > kTmaMaxStages) r = kTmaMaxStages;
  // An even ring: k-block i goes to converter group i % 2 and raw stage i % R,
  // so with R even every stage is always read by the same group, whose
  // successive parity waits on it are then one phase apart.  With R odd a group
  // would wait two phases after its previous use and could mistake the older
  // completed phase of the same parity for the load it waits for.
  r &= ~1;
  *raw_stages = r;
  *op_stages = q;
}

template <int AK, bool kBK>
int launch_tma(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& md, const TmaProblem& prob,
               int raw_stages, int op_stages, int grid, cudaStream_t s, const char* name) {
  const TmaSmem plan = tma_smem_plan(prob.bn, raw_stages, op_stages, AK == kAFpropRows ? im_table_entries(prob.K) : 0,
                                     prob.b_res_kb);
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  static SmemOptIn opt_in;  // per instantiation
  B2_RETURN_IF_ERROR(
      opt_in.ensure(reinterpret_cast<const void*>(tma_gemm_kernel<AK, kBK>), d->device, (int)plan.total));
  TmaProblem p = prob;
  p.wait = wait_params();
  tma_gemm_kernel<AK, kBK><<<grid, kTmaThreads, plan.total, s>>>(ma, mb, md, p, raw_stages, op_stages);
  return check_launch(s, name);
}

// The A operand of a TMA-engine contraction: a plain matrix, or an im2col
// view of an NHWC input whose rows the TMA stages (x, n_images, cr).
struct ASpec {
  AKind kind;
  MatOperand mat;
  const float* x;
  int64_t n_images;
  ConvRows cr;
};

inline ASpec a_matrix(const MatOperand& m) { return ASpec{m.k_major ? kAK : kAMN, m, nullptr, 0, ConvRows{}}; }

int run_tma_gemm(const ASpec& a, const MatOperand& b, int64_t M, int64_t N, int64_t K, float* out,
                 const float* bias, cudaStream_t s, const char* name, int min_kb_per_split, bool relu = false) {
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  const int bn = tma_bn(N);
  const int64_t tiles = ceil_div(N, bn) * ceil_div(M, BM);
  int splits = splits_for(tiles, K, persistent_ctas(d), min_kb_per_split);
  int64_t kps = ceil_div(ceil_div(K, splits), BK) * BK;
  if (kps < BK) kps = BK;
  splits = (int)ceil_div(K, kps);
  const bool use_s = kps > (int64_t)kChunkKB * BK;
  const int table = a.kind == kAFpropRows ? im_table_entries(K) : 0;
  int raw_stages = 0, op_stages = 0;
  // Resident B: with one split and a short K, every tile of a CTA multiplies
  // by the same B tile when the grid is a multiple of the N-tile count; it is
  // then loaded and split once per CTA instead of once per k-block.
  const int64_t nt = ceil_div(N, bn);
  int b_res_kb = 0;
  const int ctas = persistent_ctas(d);
  int grid = (int)(tiles * splits < ctas ? tiles * splits : ctas);
  if (splits == 1 && K <= (int64_t)kTmaMaxResKB * BK && grid / nt * nt > 0 &&
      ceil_div(K, BK) * 2 * (int64_t)bn * BK * 4 <= kTmaMaxResBytes) {
    tma_stages(bn, use_s, table, d->max_smem_optin, &raw_stages, &op_stages, (int)ceil_div(K, BK));
    if (raw_stages >= 4) {
      b_res_kb = (int)ceil_div(K, BK);
      grid = (int)(grid / nt * nt);
    }
  }
  if (b_res_kb == 0) tma_stages(bn, use_s, table, d->max_smem_optin, &raw_stages, &op_stages);
  if (raw_stages < 2 || op_stages < 2)
    return set_error(B2_ERR_INTERNAL, "%s: shared memory too small for the TMA engine", name);
  TmaProblem prob{a.cr, M, N, K, kps, splits, bn, bias, false, use_s, (uint32_t)BM * BK * 4, relu && splits == 1,
                  b_res_kb};
  B2_REQUIRE(tiles * splits <= kMaxInt32, "%s: too many output tiles", name);
  prob.nt_div = FastDiv((uint32_t)nt);
  prob.mt_div = FastDiv((uint32_t)ceil_div(M, BM));
  if (a.kind == kAFpropRows || a.kind == kAWgradRows) {
    prob.wo_div = FastDiv((uint32_t)a.cr.Wo);
    prob.ho_div = FastDiv((uint32_t)a.cr.Ho);
    prob.kwc_div = FastDiv((uint32_t)(a.cr.kW * a.cr.Ci));
  }
  CUtensorMap ma, mb, md;
  if (a.kind == kAK || a.kind == kAMN) {
    B2_RETURN_IF_ERROR(encode_operand(&ma, a.mat, K, BM, CU_TENSOR_MAP_SWIZZLE_NONE));
  } else {
    const ConvRows& cr = a.cr;
    const int64_t wc = (int64_t)cr.W * cr.Ci;
    const cuuint64_t dims[3] = {(cuuint64_t)wc, (cuuint64_t)cr.H, (cuuint64_t)a.n_images};
    const cuuint64_t strides[2] = {(cuuint64_t)wc * 4, (cuuint64_t)(wc * cr.H * 4)};
    const cuuint32_t box[3] = {(cuuint32_t)cr.wcp, (cuuint32_t)cr.span, 1};
    B2_RETURN_IF_ERROR(encode_map(&ma, a.x, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE));
    prob.a_tx = (uint32_t)(cr.wcp * cr.span * 4);
  }
  B2_RETURN_IF_ERROR(encode_operand(&mb, b, K, bn, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B));
  const cuuint32_t obox[3] = {32, 32, 1};
  Scratch part;
  if (splits == 1) {
    const cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)M};
    const cuuint64_t strides[1] = {(cuuint64_t)N * 4};
    B2_RETURN_IF_ERROR(encode_map(&md, out, 2, dims, strides, obox));
  } else {
    B2_RETURN_IF_ERROR(part.alloc(sizeof(float) * (size_t)splits * M * N, s));
    const cuuint64_t dims[3] = {(cuuint64_t)N, (cuuint64_t)M, (cuuint64_t)splits};
    const cuuint64_t strides[2] = {(cuuint64_t)N * 4, (cuuint64_t)(M * N * 4)};
    B2_RETURN_IF_ERROR(encode_map(&md, part.as<float>(), 3, dims, strides, obox));
    prob.partial = true;
    prob.bias = nullptr;
  }
  int rc;
  switch (a.kind) {
    case kAK:
      rc = b.k_major ? launch_tma<kAK, true>(ma, mb, md, prob, raw_stages, op_stages, grid, s, name)
                     : launch_tma<kAK, false>(ma, mb, md, prob, raw_stages, op_stages, grid, s, name);
      break;
    case kAMN:
      rc = b.k_major ? launch_tma<kAMN, true>(ma, mb, md, prob, raw_stages, op_stages, grid, s, name)
                     : launch_tma<kAMN, false>(ma, mb, md, prob, raw_stages, op_stages, grid, s, name);
      break;
    case kAFpropRows:
      rc = launch_tma<kAFpropRows, false>(ma, mb, md, prob, raw_stages, op_stages, grid, s, name);
      break;
    default:
      rc = launch_tma<kAWgradRows, false>(ma, mb, md, prob, raw_stages, op_stages, grid, s, name);
      break;
  }
  B2_RETURN_IF_ERROR(rc);
  if (splits == 1) return B2_OK;
  splitk_reduce_kernel<<<(unsigned)ceil_div(M * N, 32), dim3(32, kRedParts), 0, s>>>(part.as<float>(), splits, M, N,
                                                                                   bias, out, N, relu ? 1 : 0);
  return check_launch(s, "splitk_reduce");
}

// Staged-row im2col A for a Conv2D forward (rows = output pixels,
// rows_per_unit = BM) or filter gradient (k = output pixels, rows_per_unit =
// BK): eligible when whole input rows fit one TMA box (W*Ci <= 256 floats,
// 16-byte pitch), a tile / k-block never spans two images, and the staged
// rows fit the 16 KB raw A area.
bool conv_rows_spec(const ConvGeom& g, const float* x, int64_t pixels_per_unit, ASpec* a) {
  const int64_t wc = g.W * g.Ci;
  if (!tma_engine_enabled() || !aligned16(x) || wc <= 0 || wc % 4 != 0 || g.Wo <= 0 ||
      (g.Ho * g.Wo) % pixels_per_unit != 0 || g.H > kI32 || g.N > kI32)
    return false;
  const int64_t jmax = (g.Wo - 1 + pixels_per_unit - 1) / g.Wo + 1;
  const int64_t span = (jmax - 1) * g.sH + g.kH;
  // staged row: xpad zeros, the W*Ci values, zeros up to the last tap's column
  const int64_t xpad = ceil_div(g.pW * g.Ci, 4) * 4;
  const int64_t last_col = ((g.Wo - 1) * g.sW - g.pW + g.kW) * g.Ci;  // one past the last tap read
  const int64_t wcp = ceil_div(xpad + (last_col > wc ? last_col : wc), 4) * 4;
  if (wcp > 256 || span > 256 || span * wcp * 4 > (int64_t)BM * BK * 4) return false;
  if (pixels_per_unit == BM && g.kH * g.kW * g.Ci > kMaxImTable) return false;
  a->kind = pixels_per_unit == BM ? kAFpropRows : kAWgradRows;
  a->mat = MatOperand{nullptr, 0, 0, false};
  a->x = x;
  a->n_images = g.N;
  a->cr = ConvRows{(int)g.H, (int)g.W, (int)g.Ci, (int)g.kW, (int)g.sH, (int)g.sW, (int)g.pH, (int)g.pW,
                   (int)g.Ho, (int)g.Wo, (int)span, (int)xpad, (int)wcp};
  return true;
}

bool tma_output_ok(const float* out, int64_t M, int64_t N) {
  return aligned16(out) && N % 4 == 0 && M <= kI32 && N <= kI32;
}

template <class AV, class BV>
int run_gemm(const AV& a, const BV& b, int64_t M, int64_t N, int64_t K, float* out, const float* bias,
             cudaStream_t s, const char* name, int min_kb_per_split = 4, bool relu = false) {
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  if (M == 0 || N == 0) return B2_OK;
  if constexpr (is_mat_view<AV>::value && is_mat_view<BV>::value) {
    const MatOperand ma = mat_of(a), mb = mat_of(b);
    if (K > 0 && tma_engine_enabled() && tma_operand_ok(ma, K) && tma_operand_ok(mb, K) && aligned16(out) &&
        N % 4 == 0 && M <= kI32 && N <= kI32)
      return run_tma_gemm(a_matrix(ma), mb, M, N, K, out, bias, s, name, min_kb_per_split, relu);
  }
  const int bn = choose_bn(N);
  const int64_t tiles = ceil_div(N, bn) * ceil_div(M, BM);
  int splits = splits_for(tiles, K, persistent_ctas(d), min_kb_per_split);
  int64_t kps = ceil_div(ceil_div(K, splits), BK) * BK;
  if (kps < BK) kps = BK;
  splits = (int)(K > 0 ? ceil_div(K, kps) : 1);
  GemmProblem<AV, BV> prob{a, b, M, N, K, kps, splits, Epilogue{out, N, bias, false}};
  if (splits == 1) {
    B2_RETURN_IF_ERROR(launch_gemm(prob, bn, s, name));
    // this engine's epilogue has no ReLU: apply it in place
    return relu ? b2_relu(s, out, out, M * N) : B2_OK;
  }
  Scratch part;
  B2_RETURN_IF_ERROR(part.alloc(sizeof(float) * (size_t)splits * M * N, s));
  prob.ep = Epilogue{part.as<float>(), N, nullptr, true};
  B2_RETURN_IF_ERROR(launch_gemm(prob, bn, s, name));
  splitk_reduce_kernel<<<(unsigned)ceil_div(M * N, 32), dim3(32, kRedParts), 0, s>>>(part.as<float>(), splits, M, N, bias,
                                                                                   out, N, relu ? 1 : 0);
  return check_launch(s, "splitk_reduce");
}

// dense_kernels.cl:88-102: db[o] = sum_n dy[n, o], added in the reference's
// order (n ascending, one serial sum per column: bit-identical result).  A CTA
// owns kBiasCols columns; its eight warps stage kBiasRows rows of them in
// shared memory with independent coalesced loads, then warp 0 adds each
// column's staged values in order.  The loads are off the serial chain, which
// is what bounds a one-thread-per-column loop over global memory.
constexpr int kBiasCols = 32;
constexpr int kBiasRows = 256;
constexpr int kBiasThreads = 256;

__global__ void __launch_bounds__(kBiasThreads) dense_bias_grad_kernel(const float* __restrict__ dy, int64_t batch,
                                                                        int64_t out_f, float* __restrict__ db) {
  __shared__ float tile[kBiasRows][kBiasCols];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t o = (int64_t)blockIdx.x * kBiasCols + lane;
  const bool col_ok = o < out_f;
  float acc = 0.0f;
  for (int64_t n0 = 0; n0 < batch; n0 += kBiasRows) {
    const int rows = (int)(batch - n0 < kBiasRows ? batch - n0 : kBiasRows);
#pragma unroll 8
    for (int r = warp; r < rows; r += kBiasThreads / 32)
      tile[r][lane] = col_ok ? __ldg(dy + (n0 + r) * out_f + o) : 0.0f;
    __syncthreads();
    if (warp == 0) {
#pragma unroll 16
      for (int r = 0; r < rows; ++r) acc = __fadd_rn(acc, tile[r][lane]);
    }
    __syncthreads();
  }
  if (warp == 0 && col_ok) db[o] = acc;
}

int conv_geom_fwd(const int64_t* input_shape, const int64_t* filter_shape, const int32_t* strides,
                  int num_strides, const char* padding, bool forward, ConvGeom* g) {
  B2_RETURN_IF_ERROR(check_dims_nonneg(input_shape, 4, "input"));
  B2_RETURN_IF_ERROR(check_dims_nonneg(filter_shape, 4, "filter"));
  B2_RETURN_IF_ERROR(parse_conv_attrs(strides, num_strides, padding, forward, g));
  g->N = input_shape[0]; g->H = input_shape[1]; g->W = input_shape[2]; g->Ci = input_shape[3];
  g->kH = filter_shape[0]; g->kW = filter_shape[1]; g->Co = filter_shape[3];
  finish_geom(g);
  return B2_OK;
}

bool is_pointwise(const ConvGeom& g) {
  return g.kH == 1 && g.kW == 1 && g.sH == 1 && g.sW == 1 && g.pH == 0 && g.pW == 0;
}

}  // namespace tc
}  // namespace b2

using namespace b2;
using namespace b2::tc;

extern "C" {

int b2_conv2d_output_shape(const int64_t input_shape[4], const int64_t filter_shape[4], const int32_t* strides,
                           int num_strides, const char* padding, int64_t out_shape[4]) {
  clear_error();
  ConvGeom g;
  B2_RETURN_IF_ERROR(conv_geom_fwd(input_shape, filter_shape, strides, num_strides, padding, true, &g));
  B2_REQUIRE(filter_shape[2] == input_shape[3], "filter[2] must equal input channels");
  out_shape[0] = g.N; out_shape[1] = g.Ho; out_shape[2] = g.Wo; out_shape[3] = g.Co;
  return B2_OK;
}

// src/ops/conv2d_ops.cc:107-190
int b2_conv2d(b2_stream_t stream, const float* input, const int64_t input_shape[4], const float* filter,
              const int64_t filter_shape[4], const int32_t* strides, int num_strides, const char* padding,
              float* output, const int64_t output_shape[4]) {
  clear_error();
  ConvGeom g;
  B2_RETURN_IF_ERROR(conv_geom_fwd(input_shape, filter_shape, strides, num_strides, padding, true, &g));
  B2_REQUIRE(filter_shape[2] == g.Ci, "filter[2] must equal input channels");
  B2_RETURN_IF_ERROR(check_dims_nonneg(output_shape, 4, "output"));
  B2_REQUIRE(output_shape[0] == g.N && output_shape[1] == g.Ho && output_shape[2] == g.Wo && output_shape[3] == g.Co,
             "output shape must be [%lld, %lld, %lld, %lld]", (long long)g.N, (long long)g.Ho, (long long)g.Wo,
             (long long)g.Co);
  B2_RETURN_IF_ERROR(check_int32_sizes(g));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t M = g.N * g.Ho * g.Wo, K = g.kH * g.kW * g.Ci;
  if (M == 0 || g.Co == 0) return B2_OK;
  if (conv_direct_ok(g)) return conv_direct_forward(g, input, filter, output, s);
  const MNMajor bv{filter, g.Co, g.Co};
  if (is_pointwise(g)) {
    const KContig av{input, M, g.Ci, aligned16(input) && g.Ci % 4 == 0};
    return run_gemm(av, bv, M, g.Co, K, output, nullptr, s, "conv2d_forward");
  }
  ASpec rows;
  const MatOperand fb = mat_of(bv);
  if (conv_rows_spec(g, input, BM, &rows) && tma_operand_ok(fb, K) && tma_output_ok(output, M, g.Co))
    return run_tma_gemm(rows, fb, M, g.Co, K, output, nullptr, s, "conv2d_forward", 4);
  const ConvFpropA av{input, M, (int)g.H, (int)g.W, (int)g.Ci, (int)g.kW, (int)g.sH, (int)g.sW,
                      (int)g.pH, (int)g.pW, (int)g.Ho, (int)g.Wo, aligned16(input) && g.Ci % 4 == 0};
  return run_gemm(av, bv, M, g.Co, K, output, nullptr, s, "conv2d_forward");
}

// src/ops/conv2d_ops.cc:225-314
int b2_conv2d_backprop_input(b2_stream_t stream, const int32_t input_sizes[4], const float* filter,
                             const int64_t filter_shape[4], const float* out_backprop,
                             const int64_t out_backprop_shape[4], const int32_t* strides, int num_strides,
                             const char* padding, float* output) {
  clear_error();
  B2_REQUIRE(input_sizes != nullptr, "input_sizes must have 4 elements");
  const int64_t in_shape[4] = {input_sizes[0], input_sizes[1], input_sizes[2], input_sizes[3]};
  ConvGeom g;
  B2_RETURN_IF_ERROR(conv_geom_fwd(in_shape, filter_shape, strides, num_strides, padding, false, &g));
  B2_REQUIRE(filter_shape[2] == g.Ci, "filter[2] != Cin");
  B2_RETURN_IF_ERROR(check_dims_nonneg(out_backprop_shape, 4, "out_backprop"));
  B2_REQUIRE(out_backprop_shape[0] == g.N && out_backprop_shape[1] == g.Ho && out_backprop_shape[2] == g.Wo &&
                 out_backprop_shape[3] == g.Co,
             "out_backprop shape mismatch");
  B2_RETURN_IF_ERROR(check_int32_sizes(g));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t M = g.N * g.H * g.W, K = g.kH * g.kW * g.Co;
  if (M == 0 || g.Ci == 0) return B2_OK;
  if (conv_direct_ok(g)) return conv_direct_backprop_input(g, out_backprop, filter, output, s);
  if (is_pointwise(g)) {
    const KContig av{out_backprop, M, g.Co, aligned16(out_backprop) && g.Co % 4 == 0};
    const KContig bv{filter, g.Ci, g.Co, aligned16(filter) && g.Co % 4 == 0};
    return run_gemm(av, bv, M, g.Ci, K, output, nullptr, s, "conv2d_backprop_input");
  }
  const ConvDgradA av{out_backprop, M, (int)g.H, (int)g.W, (int)g.Co, (int)g.kW, (int)g.sH, (int)g.sW,
                      (int)g.pH, (int)g.pW, (int)g.Ho, (int)g.Wo, aligned16(out_backprop) && g.Co % 4 == 0};
  const ConvDgradB bv{filter, (int)g.Ci, (int)g.Co, aligned16(filter) && g.Co % 4 == 0};
  return run_gemm(av, bv, M, g.Ci, K, output, nullptr, s, "conv2d_backprop_input");
}

// src/ops/conv2d_ops.cc:350-440
int b2_conv2d_backprop_filter(b2_stream_t stream, const float* input, const int64_t input_shape[4],
                              const int32_t filter_sizes[4], const float* out_backprop,
                              const int64_t out_backprop_shape[4], const int32_t* strides, int num_strides,
                              const char* padding, float* output) {
  clear_error();
  B2_REQUIRE(filter_sizes != nullptr, "filter_sizes must have 4 elements");
  const int64_t f_shape[4] = {filter_sizes[0], filter_sizes[1], filter_sizes[2], filter_sizes[3]};
  ConvGeom g;
  B2_RETURN_IF_ERROR(conv_geom_fwd(input_shape, f_shape, strides, num_strides, padding, false, &g));
  B2_REQUIRE(input_shape[3] == f_shape[2], "input channels != filter_sizes[2]");
  B2_RETURN_IF_ERROR(check_dims_nonneg(out_backprop_shape, 4, "out_backprop"));
  B2_REQUIRE(out_backprop_shape[0] == g.N && out_backprop_shape[1] == g.Ho && out_backprop_shape[2] == g.Wo &&
                 out_backprop_shape[3] == g.Co,
             "out_backprop shape mismatch");
  B2_RETURN_IF_ERROR(check_int32_sizes(g));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t M = g.kH * g.kW * g.Ci, K = g.N * g.Ho * g.Wo;
  if (M == 0 || g.Co == 0) return B2_OK;
  if (conv_direct_ok(g)) return conv_direct_backprop_filter(g, input, out_backprop, output, s);
  const MNMajor bv{out_backprop, g.Co, g.Co};
  if (is_pointwise(g)) {
    const MNMajor av{input, g.Ci, g.Ci};
    return run_gemm(av, bv, M, g.Co, K, output, nullptr, s, "conv2d_backprop_filter");
  }
  ASpec rows;
  const MatOperand gb = mat_of(bv);
  if (conv_rows_spec(g, input, BK, &rows) && tma_operand_ok(gb, K) && tma_output_ok(output, M, g.Co))
    return run_tma_gemm(rows, gb, M, g.Co, K, output, nullptr, s, "conv2d_backprop_filter", 4);
  const ConvWgradA av{input, M, (int)g.H, (int)g.W, (int)g.Ci, (int)g.kW, (int)g.sH, (int)g.sW,
                      (int)g.pH, (int)g.pW, (int)g.Ho, (int)g.Wo};
  return run_gemm(av, bv, M, g.Co, K, output, nullptr, s, "conv2d_backprop_filter");
}

// src/ops/dense_ops.cc:77-143
int b2_dense(b2_stream_t stream, const float* x, const int64_t x_shape[2], const float* w, const int64_t w_shape[2],
             const float* b, int64_t b_len, float* y) {
  clear_error();
  B2_REQUIRE(x_shape && w_shape, "x must be rank 2");
  const int64_t batch = x_shape[0], in_f = x_shape[1], out_f = w_shape[1];
  B2_REQUIRE(batch >= 0 && in_f >= 0 && out_f >= 0 && w_shape[0] >= 0, "dimensions must be non-negative");
  B2_REQUIRE(w_shape[0] == in_f, "W[0] must equal x[1] (in_features)");
  B2_REQUIRE(b_len == out_f, "b[0] must equal W[1] (out_features)");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const KContig av{x, batch, in_f, aligned16(x) && in_f % 4 == 0};
  const MNMajor bv{w, out_f, out_f};
  return run_gemm(av, bv, batch, out_f, in_f, y, b, s, "dense_forward");
}

// OpenclDense followed by OpenclRelu (src/ops/dense_ops.cc:57-140, src/ops/relu_ops.cc):
// relu(x W + b) with the ReLU applied where the sum is finished (the GEMM
// epilogue or the split-K reduction), the same bits as the two ops in sequence.
int b2_dense_relu(b2_stream_t stream, const float* x, const int64_t x_shape[2], const float* w,
                  const int64_t w_shape[2], const float* b, int64_t b_len, float* y) {
  clear_error();
  B2_REQUIRE(x_shape && w_shape, "x must be rank 2");
  const int64_t batch = x_shape[0], in_f = x_shape[1], out_f = w_shape[1];
  B2_REQUIRE(batch >= 0 && in_f >= 0 && out_f >= 0 && w_shape[0] >= 0, "dimensions must be non-negative");
  B2_REQUIRE(w_shape[0] == in_f, "W[0] must equal x[1] (in_features)");
  B2_REQUIRE(b_len == out_f, "b[0] must equal W[1] (out_features)");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const KContig av{x, batch, in_f, aligned16(x) && in_f % 4 == 0};
  const MNMajor bv{w, out_f, out_f};
  return run_gemm(av, bv, batch, out_f, in_f, y, b, s, "dense_relu_forward", 4, true);
}

// src/ops/dense_ops.cc:170-227
int b2_dense_backprop_input(b2_stream_t stream, const float* grad_y, const int64_t grad_y_shape[2], const float* w,
                            const int64_t w_shape[2], float* grad_x) {
  clear_error();
  B2_REQUIRE(grad_y_shape && w_shape, "grad_y must be rank 2");
  const int64_t batch = grad_y_shape[0], out_f = grad_y_shape[1], in_f = w_shape[0];
  B2_REQUIRE(batch >= 0 && out_f >= 0 && in_f >= 0, "dimensions must be non-negative");
  B2_REQUIRE(w_shape[1] == out_f, "W[1] must equal grad_y[1]");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const KContig av{grad_y, batch, out_f, aligned16(grad_y) && out_f % 4 == 0};
  const KContig bv{w, in_f, out_f, aligned16(w) && out_f % 4 == 0};
  return run_gemm(av, bv, batch, in_f, out_f, grad_x, nullptr, s, "dense_backprop_input");
}

// src/ops/dense_ops.cc:254-311
int b2_dense_backprop_weight(b2_stream_t stream, const float* x, const int64_t x_shape[2], const float* grad_y,
                             const int64_t grad_y_shape[2], float* grad_w) {
  clear_error();
  B2_REQUIRE(x_shape && grad_y_shape, "x must be rank 2");
  const int64_t batch = x_shape[0], in_f = x_shape[1], out_f = grad_y_shape[1];
  B2_REQUIRE(batch >= 0 && in_f >= 0 && out_f >= 0, "dimensions must be non-negative");
  B2_REQUIRE(grad_y_shape[0] == batch, "x and grad_y must have the same batch size");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const MNMajor av{x, in_f, in_f};
  const MNMajor bv{grad_y, out_f, out_f};
  return run_gemm(av, bv, in_f, out_f, batch, grad_w, nullptr, s, "dense_backprop_weight");
}

// src/ops/dense_ops.cc:334-379
int b2_dense_backprop_bias(b2_stream_t stream, const float* grad_y, const int64_t grad_y_shape[2], float* grad_b) {
  clear_error();
  B2_REQUIRE(grad_y_shape, "grad_y must be rank 2");
  const int64_t batch = grad_y_shape[0], out_f = grad_y_shape[1];
  B2_REQUIRE(batch >= 0 && out_f >= 0, "dimensions must be non-negative");
  if (out_f == 0) return B2_OK;
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  B2_REQUIRE(ceil_div(out_f, kBiasCols) <= kMaxInt32, "dense_backprop_bias: too many output features");
  dense_bias_grad_kernel<<<(unsigned)ceil_div(out_f, kBiasCols), kBiasThreads, 0, s>>>(grad_y, batch, out_f,
                                                                                        grad_b);
  return check_launch(s, "dense_backprop_bias");
}

// Number of bounded device-side waits that expired since load (tensor-core
// kernels); the caller synchronises first.  Nonzero means a kernel gave up.
int b2_device_timeouts(unsigned int* count) {
  clear_error();
  B2_CUDA_OR_RETURN(cudaMemcpyFromSymbol(count, g_tc_timeouts, sizeof(unsigned int)));
  *count += b2::dw_timeouts() + b2::peer_timeouts();
  return B2_OK;
}

}  // extern "C"
