/* cl_shim.h -- TEST INFRASTRUCTURE (oracle), never shipped or linked into the
 * product library.
 *
 * Lets the reference's OpenCL C 1.2 kernel sources (kernels/*.cl of
 * amanzargari/OpenCL-Tensorflow 0.3.0) compile unmodified as C++ for the host
 * CPU, so that the reference's own arithmetic can serve as the parity oracle
 * and as the timed CPU baseline.
 *
 * Mapping of the OpenCL C built-ins used by those files:
 *   __kernel            -> static inline function (called once per work-item
 *                          by the drivers in ref_driver.cc)
 *   __global, restrict  -> plain pointer / __restrict__
 *   get_global_id(0)    -> a thread-local work-item id set by the driver loop
 *   exp, floor, fmax    -> the host libm's single-precision expf/floorf/fmaxf
 *   rsqrt(x)            -> 1.0f / sqrtf(x)
 *   min, max (int)      -> integer min/max
 *   atomic_cmpxchg      -> GCC __atomic compare-exchange (returns old value)
 *
 * Exactness: +, -, *, / (correctly rounded on the host), comparisons, casts
 * and floor are exactly specified, so kernels built only from those are
 * reproduced bit for bit.  OpenCL lets exp/rsqrt differ by a few ulp per
 * device; here they take the host's single-precision libm values, so those
 * outputs are one valid OpenCL result, not the only one.
 *
 * The kernel sources must be included inside namespace clk (see
 * ref_driver.cc) so the float overloads below hide the double versions in
 * the global namespace.
 */
#ifndef B2_ORACLE_CL_SHIM_H_
#define B2_ORACLE_CL_SHIM_H_

#include <cmath>
#include <cstddef>
#include <cstdint>

namespace clk {

typedef unsigned int uint;

/* Work-item id of the calling host thread (one work-item at a time). */
extern thread_local size_t g_work_item_id;

static inline size_t get_global_id(int /*dim*/) { return g_work_item_id; }

static inline float exp(float x) { return expf(x); }
static inline float floor(float x) { return floorf(x); }
static inline float fmax(float a, float b) { return fmaxf(a, b); }
static inline float rsqrt(float x) { return 1.0f / sqrtf(x); }
static inline int min(int a, int b) { return a < b ? a : b; }
static inline int max(int a, int b) { return a > b ? a : b; }

static inline uint atomic_cmpxchg(volatile uint* p, uint cmp, uint val) {
  uint expected = cmp;
  __atomic_compare_exchange_n(const_cast<uint*>(p), &expected, val, false,
                              __ATOMIC_SEQ_CST, __ATOMIC_SEQ_CST);
  return expected; /* the value found at *p, equal to cmp on success */
}

}  // namespace clk

#define __kernel static inline
#define __global
#define restrict __restrict__

#endif  // B2_ORACLE_CL_SHIM_H_
