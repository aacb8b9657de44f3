// Warp-level tensor-core helpers: cp.async staging, ldmatrix fragments and
// m16n8k16 MMAs with fp32 accumulation for bf16 / fp16 operands.
#pragma once

#include "avq_common.cuh"

namespace avq {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  const int sz = pred ? 16 : 0;  // zero-fill when out of range
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem), "r"(sz));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}

// D = A(16x16, row) * B(16x8, col) + D, fp32 accumulators.
template <int DT>
__device__ __forceinline__ void mma16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1);

template <>
__device__ __forceinline__ void mma16816<DT_BF16>(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<DT_F16>(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Pack two floats (exactly representable in DT) into a DT x2 register.
template <int DT>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  uint32_t r;
  if (DT == DT_BF16) {
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;\n" : "=r"(r) : "f"(hi), "f"(lo));
  } else {
    asm("cvt.rn.f16x2.f32 %0, %1, %2;\n" : "=r"(r) : "f"(hi), "f"(lo));
  }
  return r;
}


// NaN-propagating max and clamp (torch.max / clamp_min semantics).
__device__ __forceinline__ float nanmax(float a, float b) {
  if (isnan(a) || isnan(b)) return NAN;
  return a > b ? a : b;
}
__device__ __forceinline__ float clamp_min_nan(float x, float lo) { return isnan(x) ? x : (x < lo ? lo : x); }

// Packed fp32 pair arithmetic (sm_100): one instruction for both elements,
// IEEE rounding per element to nearest (rn), down (rm) or up (rp).
#define AVQ_F32X2_OP(name, op)                                                                   \
  __device__ __forceinline__ float2 name(float2 a, float2 b) {                                  \
    float2 d;                                                                                    \
    asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t" op \
        " rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"                                            \
        : "=f"(d.x), "=f"(d.y)                                                                   \
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));                                               \
    return d;                                                                                    \
  }
AVQ_F32X2_OP(add_f32x2, "add.rn.f32x2")
AVQ_F32X2_OP(mul_f32x2_rd, "mul.rm.f32x2")
AVQ_F32X2_OP(mul_f32x2_ru, "mul.rp.f32x2")
AVQ_F32X2_OP(mul_f32x2_rn, "mul.rn.f32x2")
#undef AVQ_F32X2_OP

// The neighbouring fp32 values of a positive finite nonzero x.
__device__ __forceinline__ float next_down(float x) { return __uint_as_float(__float_as_uint(x) - 1u); }
__device__ __forceinline__ float next_up(float x) { return __uint_as_float(__float_as_uint(x) + 1u); }

// Halves of a DT x2 register as floats.
template <int DT>
__device__ __forceinline__ float half_lo(uint32_t w) {
  return DT == DT_BF16 ? __uint_as_float(w << 16) : __half2float(__ushort_as_half((unsigned short)(w & 0xffffu)));
}
template <int DT>
__device__ __forceinline__ float half_hi(uint32_t w) {
  return DT == DT_BF16 ? __uint_as_float(w & 0xffff0000u) : __half2float(__ushort_as_half((unsigned short)(w >> 16)));
}

template <int DT>
__device__ __forceinline__ uint32_t hsub2_dt(uint32_t a, uint32_t b) {
  uint32_t r;
  if (DT == DT_BF16) asm("sub.rn.bf16x2 %0, %1, %2;\n" : "=r"(r) : "r"(a), "r"(b));
  else asm("sub.rn.f16x2 %0, %1, %2;\n" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

template <int DT>
__device__ __forceinline__ uint32_t hmax2_nan_dt(uint32_t a, uint32_t b) {
  uint32_t r;
  if (DT == DT_BF16) asm("max.NaN.bf16x2 %0, %1, %2;\n" : "=r"(r) : "r"(a), "r"(b));
  else asm("max.NaN.f16x2 %0, %1, %2;\n" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

template <int DT>
__device__ __forceinline__ uint32_t dup2(float x) {
  return pack2<DT>(x, x);
}

// DT(a * b) per half: the exact product rounded once (for DT operands whose
// product is exact in fp32, the same as narrowing the fp32 product).
template <int DT>
__device__ __forceinline__ uint32_t hmul2_dt(uint32_t a, uint32_t b) {
  uint32_t r;
  if (DT == DT_BF16) asm("mul.rn.bf16x2 %0, %1, %2;\n" : "=r"(r) : "r"(a), "r"(b));
  else asm("mul.rn.f16x2 %0, %1, %2;\n" : "=r"(r) : "r"(a), "r"(b));
  return r;
}


}  // namespace avq
