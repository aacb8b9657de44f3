// Shared numerics for the AVQ-attention kernels (sm_100a).
//
// Every kernel reproduces the reference's rounding points: a torch CPU op
// computes in fp32 and narrows its result to the tensor dtype once.  Here a
// value "in dtype DT" is carried as a float that holds a DT-representable
// number; rnd<DT>() performs the narrowing (round-to-nearest-even).
// Reductions that the reference performs in fp32 are accumulated in double
// and narrowed fp64 -> fp32 -> DT, i.e. the exactly rounded sum.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace avq {

enum DType : int { DT_F32 = 0, DT_BF16 = 1, DT_F16 = 2 };

template <int DT> struct Storage;
template <> struct Storage<DT_F32> { using T = float; };
template <> struct Storage<DT_BF16> { using T = __nv_bfloat16; };
template <> struct Storage<DT_F16> { using T = __half; };

__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f(__half x) { return __half2float(x); }

template <int DT> __device__ __forceinline__ typename Storage<DT>::T from_f(float x);
template <> __device__ __forceinline__ float from_f<DT_F32>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<DT_BF16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half from_f<DT_F16>(float x) { return __float2half_rn(x); }

// Narrow an fp32 value to DT and widen it back (RNE; NaN stays NaN, fp16
// overflow becomes inf).
template <int DT> __device__ __forceinline__ float rnd(float x) { return to_f(from_f<DT>(x)); }

// fp64 -> fp32 -> DT (the narrowing of an fp32-accumulated reduction).
template <int DT> __device__ __forceinline__ float rnd64(double x) { return rnd<DT>(__double2float_rn(x)); }

// A Python scalar bound (clamp_min(1e-12)) cast to DT: 1e-12 in bf16, 0 in fp16.
template <int DT> __device__ __forceinline__ float eps_dt() { return rnd<DT>(1e-12f); }

// Saturating count: index_add_ of ones in DT stops growing at 2^(mantissa+1).
template <int DT> __device__ __forceinline__ float count_dt(int n) {
  const int sat = DT == DT_BF16 ? 256 : (DT == DT_F16 ? 2048 : (1 << 24));
  return (float)(n < sat ? n : sat);
}

// True when every fp32 value within k ulps of the finite nonzero y narrows to
// the same DT value, which is then stored in *r.  Stepping the bit pattern by
// k moves |y| by k ulps in either direction (the sign bit is untouched for
// |y| above k ulps of zero, which the caller ensures).
template <int DT>
__device__ __forceinline__ bool narrow_certain(float y, uint32_t k, float* r) {
  const uint32_t u = __float_as_uint(y);
  const float a = rnd<DT>(__uint_as_float(u - k)), b = rnd<DT>(__uint_as_float(u + k));
  *r = a;
  return a == b;
}

// rnd<DT>(correctly rounded fp32 exp(x)).  CUDA's expf is within 2 ulp; when
// every fp32 value within 3 ulp of it narrows to the same DT value the answer
// is known, otherwise the exponential is recomputed in double.  A result
// below 2^-140 (far below half of the smallest fp16 / bf16 step) narrows to 0.
template <int DT> __device__ __forceinline__ float exp_rn(float x) {
  if (DT != DT_F32) {
    const float y = expf(x);
    float r;
    if (isfinite(y)) {
      if (y < 7.0e-43f) return 0.f;
      if (narrow_certain<DT>(y, 3u, &r)) return r;
    }
  }
  return rnd<DT>(__double2float_rn(exp((double)x)));
}

// Same for the natural logarithm (HVAQ entropy), x > 0 (log(1) = 0 exactly).
template <int DT> __device__ __forceinline__ float log_rn(float x) {
  if (DT != DT_F32) {
    const float y = logf(x);
    float r;
    if (y == 0.f && x == 1.f) return 0.f;
    if (isfinite(y) && fabsf(y) > 1e-30f && narrow_certain<DT>(y, 3u, &r)) return r;
  }
  return rnd<DT>(__double2float_rn(log((double)x)));
}

// True when an fp32 value y (within +-3 ulp of the correctly rounded result)
// is too close to a DT rounding midpoint for the narrowing to be certain
// (and, for fp16, when the result lies in the fp16 subnormal range).
template <int DT>
__device__ __forceinline__ bool near_midpoint(float y) {
  const uint32_t u = __float_as_uint(y);
  if (DT == DT_BF16) return ((u & 0xFFFFu) - 0x7FFDu) < 7u;
  if (DT == DT_F16) return ((u & 0x1FFFu) - 0x0FFDu) < 7u || fabsf(y) < 6.2e-5f;
  return true;
}

// DT(correctly rounded fp32 exp(x)): expf is within 2 ulp, so only results
// near a rounding midpoint need the double-precision recomputation.  fp16
// results in the subnormal range (steps of 2^-24, where the midpoint test on
// the fp32 mantissa does not apply) are certified by bracketing 3 fp32 ulps;
// below 2^-140 they narrow to 0.
template <int DT>
__device__ __forceinline__ float exp_dt_fast(float x) {
  if (DT != DT_F32) {
    const float y = expf(x);
    if (!near_midpoint<DT>(y)) return rnd<DT>(y);
    if (DT == DT_F16 && y < 6.2e-5f) {
      float r;
      if (y < 7.0e-43f) return 0.f;
      if (narrow_certain<DT>(y, 3u, &r)) return r;
    }
  }
  return rnd<DT>(__double2float_rn(exp((double)x)));
}

// DT(a / b) with the correctly rounded fp32 quotient; rb = 1/b (any rounding):
// a * rb is within 2 ulp of a / b.
template <int DT>
__device__ __forceinline__ float div_dt_fast(float a, float rb, float b) {
  if (DT != DT_F32) {
    const float y = a * rb;
    if (isfinite(y) && !near_midpoint<DT>(y)) return rnd<DT>(y);
  }
  return rnd<DT>(__fdiv_rn(a, b));
}

// DT(x / sqrt(D)) with the correctly rounded fp32 quotient (pipeline.py:81).
template <int DT>
__device__ __forceinline__ float scale_logit(float x, float sqrtD, float inv_sqrtD) {
  return div_dt_fast<DT>(x, inv_sqrtD, sqrtD);
}

// Order-preserving map of a float onto uint32 (ascending); NaN maps above +inf.
__device__ __forceinline__ uint32_t float_order_key(float f) {
  if (isnan(f)) return 0xFFFFFFFFu;
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Load a DT row element as float.
template <typename T> __device__ __forceinline__ float ld(const T* p, long i) { return to_f(p[i]); }

}  // namespace avq

// Status codes shared with the host wrapper.
#define AVQ_OK 0
#define AVQ_ERR_ARG 1
#define AVQ_ERR_CUDA 2
#define AVQ_ERR_UNSUPPORTED 3
#define AVQ_ERR_WORKSPACE 4
