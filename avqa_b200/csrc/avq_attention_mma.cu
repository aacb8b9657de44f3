// Tensor-core parent attention for bf16 / fp16 and D in {64, 128}
// (reference pipeline.py:46-151 and :192-258, routing.py:61-63).
//
// One CTA = 64 queries of one (b,h) = 4 warps x 16 rows; every warp owns its
// rows across all M0 parents, so row statistics stay inside a lane quad.
//
//   phase 1  S = Q P^T (m16n8k16, fp32 accumulate), narrowed to the dtype,
//            / sqrt(D), -inf for empty parents; row max.  [HVAQ: beta per row
//            from the stored pre-HVAQ statistics, S rescaled in place.]
//   phase 2  e = dtype(exp(dtype(s - m))) written over S; l = sum dtype(e*n)
//            and z = sum e in fp64; A = e @ V with e as the MMA A operand
//            straight from registers and V (parent sums) via ldmatrix.trans.
//   phase 3  probs = dtype(e / max(z, eps)); per-parent fp64 column sums over
//            the CTA's queries -> importance partials.
//
// S lives in shared memory when 64 x M0 dtype values fit, else in a global
// scratch slice (generic addressing covers both).
#include "avq_kernels.cuh"
#include "avq_mma.cuh"

namespace avq {

constexpr int PM_ROWS = 64;
constexpr int PM_CH = 64;
constexpr int PM_MAX_SMEM_M0 = 1024;

template <int DT>
__device__ __forceinline__ float half_lo(uint32_t w) {
  return DT == DT_BF16 ? __uint_as_float(w << 16) : __half2float(__ushort_as_half((unsigned short)(w & 0xffffu)));
}
template <int DT>
__device__ __forceinline__ float half_hi(uint32_t w) {
  return DT == DT_BF16 ? __uint_as_float(w & 0xffff0000u) : __half2float(__ushort_as_half((unsigned short)(w >> 16)));
}

__device__ __forceinline__ float nanmax2(float a, float b) {
  if (isnan(a) || isnan(b)) return NAN;
  return a > b ? a : b;
}
__device__ __forceinline__ float clamp_min_nan2(float x, float lo) { return isnan(x) ? x : (x < lo ? lo : x); }

// dtype(correctly rounded fp32 exp(x)) for x <= 0 (x a dtype value):
// expf is within 2 ulp, so only results near a rounding midpoint (or in the
// fp16 subnormal range) need the double-precision recomputation.
template <int DT>
__device__ __forceinline__ float exp_dt_fast(float x) {
  const float y = expf(x);
  const uint32_t u = __float_as_uint(y);
  bool amb;
  if (DT == DT_BF16) {
    const int low = (int)(u & 0xFFFFu) - 0x8000;
    amb = low >= -3 && low <= 3;
  } else {
    const int low = (int)(u & 0x1FFFu) - 0x1000;
    amb = (low >= -3 && low <= 3) || y < 6.2e-5f;
  }
  if (!amb) return rnd<DT>(y);
  return rnd<DT>(__double2float_rn(exp((double)x)));
}

// dtype(a / b) for dtype values a, b > 0 with the correctly rounded fp32
// quotient: a * (1/b) is within 2 ulp; ambiguous cases use the exact division.
template <int DT>
__device__ __forceinline__ float div_dt_fast(float a, float rb, float b) {
  const float y = a * rb;
  const uint32_t u = __float_as_uint(y);
  bool amb;
  if (DT == DT_BF16) {
    const int low = (int)(u & 0xFFFFu) - 0x8000;
    amb = low >= -3 && low <= 3;
  } else {
    const int low = (int)(u & 0x1FFFu) - 0x1000;
    amb = (low >= -3 && low <= 3) || y < 6.2e-5f;
  }
  if (!amb) return rnd<DT>(y);
  return rnd<DT>(__fdiv_rn(a, b));
}

// dtype(x / sqrt(D)) with the correctly rounded fp32 quotient, x a dtype
// value (pipeline.py:81).  x * (1/sqrt(D)) is within 2 ulp of x / sqrt(D) and
// exact when sqrt(D) is a power of two; near a rounding midpoint the exact
// division decides.
template <int DT>
__device__ __forceinline__ float scale_logit(float x, float sqrtD, float inv_sqrtD) {
  const float y = x * inv_sqrtD;
  if (!isfinite(y)) return rnd<DT>(__fdiv_rn(x, sqrtD));
  const uint32_t u = __float_as_uint(y);
  bool amb;
  if (DT == DT_BF16) {
    const int low = (int)(u & 0xFFFFu) - 0x8000;
    amb = low >= -3 && low <= 3;
  } else {
    const int low = (int)(u & 0x1FFFu) - 0x1000;
    amb = (low >= -3 && low <= 3) || fabsf(y) < 6.2e-5f;
  }
  return amb ? rnd<DT>(__fdiv_rn(x, sqrtD)) : rnd<DT>(y);
}

template <int DT, int D>
__global__ void __launch_bounds__(128) parent_attn_mma_kernel(
    const typename Storage<DT>::T* __restrict__ q, Strides3 qs, int H, int Tq, int M0, float sqrtD,
    const typename Storage<DT>::T* __restrict__ parents, const typename Storage<DT>::T* __restrict__ pagg,
    const int* __restrict__ pcnt, int mode, typename Storage<DT>::T* __restrict__ sglobal, float* __restrict__ m_io,
    float* __restrict__ l_out, float* __restrict__ z_io, typename Storage<DT>::T* __restrict__ a_out,
    double* __restrict__ imp_part, const int* __restrict__ sel0, int sel_stride, const int* __restrict__ pass_cnt,
    int hvaq, float beta0, float alpha, float* __restrict__ beta_out, int s_in_smem, int keep_logits) {
  using T = typename Storage<DT>::T;
  constexpr int LDS = D + 8, KS = D / 16, CPR = D / 8, NT = D / 8;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* sq_ = (T*)smem_raw;                       // [PM_ROWS][LDS] queries
  T* sb = sq_ + PM_ROWS * LDS;                 // [2][PM_CH][LDS] parents / parent sums
  float* sn = (float*)(sb + 2 * PM_CH * LDS);  // [2][PM_CH] dtype counts
  double* scol = (double*)(sn + 2 * PM_CH);    // [PM_CH] importance column sums
  T* slog = (T*)(scol + PM_CH);                // [PM_ROWS][M0 + 8] logits / exps (smem mode)
  const int g = blockIdx.y, b = g / H, h = g % H, qt = blockIdx.x, t0 = qt * PM_ROWS;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int LDL = M0 + 8;
  const float inv_sqrtD = 1.f / sqrtD;
  T* S_ = s_in_smem ? slog : sglobal + ((long)g * gridDim.x + qt) * PM_ROWS * LDL;
  const int r0 = warp * 16 + (lane >> 2), r1 = r0 + 8;  // this thread's two rows (CTA-local)
  const bool live0 = t0 + r0 < Tq, live1 = t0 + r1 < Tq;
  const int cq = (lane & 3) * 2;                         // column pair offset inside an n8 tile

  const T* qb = q + (long)b * qs.b + (long)h * qs.h;
  for (int i = tid; i < PM_ROWS * CPR; i += blockDim.x) {
    const int r = i / CPR, c = i % CPR, t = t0 + r;
    cp_async16(sq_ + r * LDS + c * 8, qb + (long)(t < Tq ? t : 0) * qs.s + c * 8, t < Tq);
  }
  cp_async_commit();
  const int nch = (M0 + PM_CH - 1) / PM_CH;
  const T* pb = parents + (long)h * M0 * D;
  auto load_parents = [&](int buf, int p0) {
    for (int i = tid; i < PM_CH * CPR; i += blockDim.x) {
      const int r = i / CPR, c = i % CPR, p = p0 + r;
      cp_async16(sb + (buf * PM_CH + r) * LDS + c * 8, pb + (long)(p < M0 ? p : 0) * D + c * 8, p < M0);
    }
    if (tid < PM_CH) sn[buf * PM_CH + tid] = p0 + tid < M0 ? (float)pcnt[(long)g * M0 + p0 + tid] : 0.f;
  };
  const T* vb = pagg + (long)g * M0 * D;
  auto load_values = [&](int buf, int p0) {
    for (int i = tid; i < PM_CH * CPR; i += blockDim.x) {
      const int r = i / CPR, c = i % CPR, p = p0 + r;
      cp_async16(sb + (buf * PM_CH + r) * LDS + c * 8, vb + (long)(p < M0 ? p : 0) * D + c * 8, p < M0);
    }
    if (tid < PM_CH) sn[buf * PM_CH + tid] = p0 + tid < M0 ? count_dt<DT>(pcnt[(long)g * M0 + p0 + tid]) : 0.f;
  };

  float rmax0 = -INFINITY, rmax1 = -INFINITY;
  if (mode == 0) {
    load_parents(0, 0);
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    uint32_t af[KS][4];
#pragma unroll
    for (int k = 0; k < KS; ++k)
      ldsm_x4(af[k][0], af[k][1], af[k][2], af[k][3], sq_ + (warp * 16 + (lane & 15)) * LDS + k * 16 + (lane >> 4) * 8);
    for (int ci = 0; ci < nch; ++ci) {
      const int buf = ci & 1, p0 = ci * PM_CH;
      if (ci + 1 < nch) load_parents(buf ^ 1, p0 + PM_CH);
      cp_async_commit();
      float acc[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
      const T* spb = sb + buf * PM_CH * LDS;
#pragma unroll
      for (int k = 0; k < KS; ++k) {
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          uint32_t b0, b1, b2, b3;
          const int qd = lane >> 3;
          ldsm_x4(b0, b1, b2, b3, spb + (jj * 16 + (qd >> 1) * 8 + (lane & 7)) * LDS + k * 16 + (qd & 1) * 8);
          mma16816<DT>(acc[2 * jj], af[k], b0, b1);
          mma16816<DT>(acc[2 * jj + 1], af[k], b2, b3);
        }
      }
      const float* nb = sn + buf * PM_CH;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int cl = j * 8 + cq, p = p0 + cl;
        float s[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int cc = cl + (e & 1);
          // pipeline.py:81 and :107
          s[e] = (p0 + cc < M0 && nb[cc] > 0.f) ? scale_logit<DT>(rnd<DT>(acc[j][e]), sqrtD, inv_sqrtD) : -INFINITY;
        }
        rmax0 = nanmax2(rmax0, nanmax2(s[0], s[1]));
        rmax1 = nanmax2(rmax1, nanmax2(s[2], s[3]));
        if (p < M0) {
          *reinterpret_cast<uint32_t*>(S_ + (long)r0 * LDL + p) = pack2<DT>(s[0], s[1]);
          *reinterpret_cast<uint32_t*>(S_ + (long)r1 * LDL + p) = pack2<DT>(s[2], s[3]);
        }
      }
      cp_async_wait<0>();
      __syncthreads();
    }
  } else {
    // HVAQ on the stored pre-HVAQ logits (S_ in global memory from the first pass)
    cp_async_wait<0>();
    __syncthreads();
    const int nsel = pass_cnt[0];
    const int* sl = sel0 + (long)g * sel_stride;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int r = half ? r1 : r0;
      const bool live = half ? live1 : live0;
      const long row = (long)g * Tq + t0 + r;
      const float safe0 = live ? m_io[row] : 0.f;
      const float zc0 = clamp_min_nan2(live ? z_io[row] : 1.f, eps_dt<DT>());
      const T* Sr = S_ + (long)r * LDL;
      double gs = 0.0;
      for (int j = lane & 3; j < nsel; j += 4) {
        float e = exp_rn<DT>(rnd<DT>(__fsub_rn(to_f(Sr[sl[j]]), safe0)));
        if (isnan(e)) e = 0.f;
        gs += (double)rnd<DT>(__fdiv_rn(e, zc0));
      }
      gs += __shfl_xor_sync(0xffffffffu, gs, 1);
      gs += __shfl_xor_sync(0xffffffffu, gs, 2);
      const float gsc = clamp_min_nan2(rnd64<DT>(gs), eps_dt<DT>());
      double ent = 0.0;
      for (int j = lane & 3; j < nsel; j += 4) {
        float e = exp_rn<DT>(rnd<DT>(__fsub_rn(to_f(Sr[sl[j]]), safe0)));
        if (isnan(e)) e = 0.f;
        const float pi = rnd<DT>(__fdiv_rn(e, zc0));
        const float top = rnd<DT>(__fdiv_rn(pi, gsc));
        const float lp = top > 0.f ? log_rn<DT>(top) : 0.f;
        ent += (double)rnd<DT>(__fmul_rn(top, lp));
      }
      ent += __shfl_xor_sync(0xffffffffu, ent, 1);
      ent += __shfl_xor_sync(0xffffffffu, ent, 2);
      const float hq = -rnd64<DT>(ent);
      const float sched = hvaq == 1 ? rnd<DT>(__fadd_rn(1.f, rnd<DT>(__fdiv_rn(1.f, rnd<DT>(__fadd_rn(1.f, hq))))))
                                    : rnd<DT>(__fadd_rn(1.f, rnd<DT>(__fmul_rn(alpha, hq))));
      const float beta = rnd<DT>(__fmul_rn(beta0, sched));
      if (live && (lane & 3) == 0) beta_out[row] = beta;
      __syncwarp();
      float mx = -INFINITY;
      T* Sw = S_ + (long)r * LDL;
      for (int p = (lane & 3); p < M0; p += 4) {
        const float s = rnd<DT>(__fmul_rn(beta, rnd<DT>(__fmul_rn(to_f(Sw[p]), sqrtD))));
        Sw[p] = from_f<DT>(s);
        mx = nanmax2(mx, s);
      }
      if (half) rmax1 = mx; else rmax0 = mx;
    }
  }
  rmax0 = nanmax2(rmax0, __shfl_xor_sync(0xffffffffu, rmax0, 1));
  rmax0 = nanmax2(rmax0, __shfl_xor_sync(0xffffffffu, rmax0, 2));
  rmax1 = nanmax2(rmax1, __shfl_xor_sync(0xffffffffu, rmax1, 1));
  rmax1 = nanmax2(rmax1, __shfl_xor_sync(0xffffffffu, rmax1, 2));
  const float safe0 = rmax0 == -INFINITY ? 0.f : rmax0;  // pipeline.py:137-141
  const float safe1 = rmax1 == -INFINITY ? 0.f : rmax1;
  __syncthreads();

  // Phase 2
  double l0 = 0.0, l1 = 0.0, z0 = 0.0, z1 = 0.0;
  float oacc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) oacc[j][0] = oacc[j][1] = oacc[j][2] = oacc[j][3] = 0.f;
  load_values(0, 0);
  cp_async_commit();
  for (int ci = 0; ci < nch; ++ci) {
    const int buf = ci & 1, p0 = ci * PM_CH;
    cp_async_wait<0>();
    __syncthreads();
    if (ci + 1 < nch) load_values(buf ^ 1, p0 + PM_CH);
    cp_async_commit();
    const float* nb = sn + buf * PM_CH;
    const T* svb = sb + buf * PM_CH * LDS;
#pragma unroll
    for (int k = 0; k < PM_CH / 16; ++k) {
      // A fragment = e for rows r0/r1, parents p0 + 16k + {cq, cq+1, cq+8, cq+9}
      float ev[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int cl = k * 16 + cq + (e & 1) + ((e >> 2) << 3);
        const int r = (e & 2) ? r1 : r0;
        const int p = p0 + cl;
        float x = 0.f;
        if (p < M0) {
          const float s = to_f(S_[(long)r * LDL + p]);
          x = exp_dt_fast<DT>(rnd<DT>(__fsub_rn(s, (e & 2) ? safe1 : safe0)));
          if (isnan(x)) x = 0.f;  // pipeline.py:143-145
          const double w = (double)rnd<DT>(__fmul_rn(x, nb[cl]));
          if (e & 2) { l1 += w; z1 += (double)x; } else { l0 += w; z0 += (double)x; }
        }
        ev[e] = x;
      }
      uint32_t a[4];
      a[0] = pack2<DT>(ev[0], ev[1]);
      a[1] = pack2<DT>(ev[2], ev[3]);
      a[2] = pack2<DT>(ev[4], ev[5]);
      a[3] = pack2<DT>(ev[6], ev[7]);
      // keep e for phase 3 (unless the logits must survive for the HVAQ pass)
      if (!keep_logits && p0 + k * 16 + cq < M0) {
        *reinterpret_cast<uint32_t*>(S_ + (long)r0 * LDL + p0 + k * 16 + cq) = a[0];
        *reinterpret_cast<uint32_t*>(S_ + (long)r1 * LDL + p0 + k * 16 + cq) = a[1];
      }
      if (!keep_logits && p0 + k * 16 + cq + 8 < M0) {
        *reinterpret_cast<uint32_t*>(S_ + (long)r0 * LDL + p0 + k * 16 + cq + 8) = a[2];
        *reinterpret_cast<uint32_t*>(S_ + (long)r1 * LDL + p0 + k * 16 + cq + 8) = a[3];
      }
#pragma unroll
      for (int jj = 0; jj < NT / 2; ++jj) {
        uint32_t b0, b1, b2, b3;
        const int qd = lane >> 3;
        // V chunk is [parent k][d n]: trans ldmatrix gives the col-major B fragment
        ldsm_x4_t(b0, b1, b2, b3, svb + (k * 16 + (qd & 1) * 8 + (lane & 7)) * LDS + jj * 16 + (qd >> 1) * 8);
        mma16816<DT>(oacc[2 * jj], a, b0, b1);
        mma16816<DT>(oacc[2 * jj + 1], a, b2, b3);
      }
    }
  }
  cp_async_wait<0>();
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, o);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    z0 += __shfl_xor_sync(0xffffffffu, z0, o);
    z1 += __shfl_xor_sync(0xffffffffu, z1, o);
  }
  const float zd0 = rnd64<DT>(z0), zd1 = rnd64<DT>(z1);
  const long row0 = (long)g * Tq + t0 + r0, row1 = (long)g * Tq + t0 + r1;
  if ((lane & 3) == 0) {
    if (live0) { m_io[row0] = safe0; l_out[row0] = rnd64<DT>(l0); z_io[row0] = zd0; }
    if (live1) { m_io[row1] = safe1; l_out[row1] = rnd64<DT>(l1); z_io[row1] = zd1; }
  }
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int d = j * 8 + cq;
    if (live0) *reinterpret_cast<uint32_t*>(a_out + row0 * D + d) = pack2<DT>(rnd<DT>(oacc[j][0]), rnd<DT>(oacc[j][1]));
    if (live1) *reinterpret_cast<uint32_t*>(a_out + row1 * D + d) = pack2<DT>(rnd<DT>(oacc[j][2]), rnd<DT>(oacc[j][3]));
  }
  __syncthreads();

  // Phase 3: probs and importance partial sums (pipeline.py:150, routing.py:62)
  const float zc0 = clamp_min_nan2(zd0, eps_dt<DT>()), zc1 = clamp_min_nan2(zd1, eps_dt<DT>());
  const float rz0 = 1.f / zc0, rz1 = 1.f / zc1;
  const int nqt = gridDim.x;
  for (int p0 = 0; p0 < M0; p0 += PM_CH) {
    if (tid < PM_CH) scol[tid] = 0.0;
    __syncthreads();
#pragma unroll
    for (int j = 0; j < PM_CH / 8; ++j) {
      const int cl = j * 8 + cq;
      double c0 = 0.0, c1 = 0.0;
      if (p0 + cl < M0) {
        const uint32_t e0 = *reinterpret_cast<const uint32_t*>(S_ + (long)r0 * LDL + p0 + cl);
        const uint32_t e1 = *reinterpret_cast<const uint32_t*>(S_ + (long)r1 * LDL + p0 + cl);
        float ea[2] = {half_lo<DT>(e0), half_hi<DT>(e0)};
        float eb[2] = {half_lo<DT>(e1), half_hi<DT>(e1)};
        if (keep_logits) {  // S_ still holds logits: recompute e exactly as in phase 2
#pragma unroll
          for (int q2 = 0; q2 < 2; ++q2) {
            float x = exp_dt_fast<DT>(rnd<DT>(__fsub_rn(ea[q2], safe0)));
            ea[q2] = isnan(x) ? 0.f : x;
            x = exp_dt_fast<DT>(rnd<DT>(__fsub_rn(eb[q2], safe1)));
            eb[q2] = isnan(x) ? 0.f : x;
          }
        }
        if (live0) {
          c0 += (double)div_dt_fast<DT>(ea[0], rz0, zc0);
          c1 += (double)div_dt_fast<DT>(ea[1], rz0, zc0);
        }
        if (live1) {
          c0 += (double)div_dt_fast<DT>(eb[0], rz1, zc1);
          c1 += (double)div_dt_fast<DT>(eb[1], rz1, zc1);
        }
      }
#pragma unroll
      for (int o = 4; o <= 16; o <<= 1) {
        c0 += __shfl_xor_sync(0xffffffffu, c0, o);
        c1 += __shfl_xor_sync(0xffffffffu, c1, o);
      }
      if (lane < 4 && p0 + cl < M0) {
        atomicAdd(&scol[cl], c0);
        atomicAdd(&scol[cl + 1], c1);
      }
    }
    __syncthreads();
    if (tid < PM_CH && p0 + tid < M0) imp_part[((long)g * nqt + qt) * M0 + p0 + tid] = scol[tid];
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Tensor-core child correction (refinement.py:82-304, attention.py:100-163,
// multipass.py:207-262, attention_module.py:532-535).
//
// CTA = 64 queries; the selected parents of a pass are staged 16 at a time
// with their children.  Per query and slot: the parent's logit (MMA, narrowed
// exactly as in the parent pass, HVAQ-rescaled when active) gives the
// probability pi; the parent term exp(pi - m) * n and the child terms
// exp(u - m) * n_c are fp32.  Their sums l-terms accumulate in fp64; the value
// sums  sum_w w * V  run on the tensor cores with every fp32 weight split into
// three bf16 parts (24 significant bits), so they carry fp32 accuracy.
// fp16 value sums (whose weights may exceed the fp16 range) use fp32 FMAs.
// ---------------------------------------------------------------------------
constexpr int CM_ROWS = 64;
constexpr int CM_J = 16;

__device__ __forceinline__ void split3_bf16(float w, float& hi, float& mid, float& lo) {
  hi = __bfloat162float(__float2bfloat16_rn(w));
  const float r = w - hi;
  mid = __bfloat162float(__float2bfloat16_rn(r));
  lo = __bfloat162float(__float2bfloat16_rn(r - mid));
}

template <int DT, int D, int C>
__global__ void __launch_bounds__(128) correct_mma_kernel(
    const typename Storage<DT>::T* __restrict__ q, Strides3 qs, int H, int Tq, int M0, float sqrtD,
    const typename Storage<DT>::T* __restrict__ parents, const typename Storage<DT>::T* __restrict__ children,
    const typename Storage<DT>::T* __restrict__ pagg, const typename Storage<DT>::T* __restrict__ cagg,
    const int* __restrict__ pcnt, const int* __restrict__ ccnt, const float* __restrict__ m_in,
    const float* __restrict__ l_in, const float* __restrict__ z_in, const float* __restrict__ beta_in,
    const typename Storage<DT>::T* __restrict__ a_in, const int* __restrict__ sel, int sel_stride,
    const int* __restrict__ pass_cnt, int npass, PassOffsets po, int multipass, float* __restrict__ out,
    Strides3 os) {
  using T = typename Storage<DT>::T;
  constexpr bool TC = DT == DT_BF16;  // tensor-core value sums
  constexpr int LDS = D + 8, KS = D / 16, CPR = D / 8, NT = D / 8, NCH = CM_J * C;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* sQ = (T*)smem_raw;            // [64][LDS]
  T* sP = sQ + CM_ROWS * LDS;      // [CM_J][LDS] selected parents (logit rows)
  T* sCh = sP + CM_J * LDS;        // [NCH][LDS] children (logit rows)
  T* sPv = sCh + NCH * LDS;        // [CM_J][LDS] parent sums
  T* sCv = sPv + CM_J * LDS;       // [NCH][LDS] child sums
  float* snp = (float*)(sCv + NCH * LDS);  // [CM_J] parent counts (dtype); <0: empty slot
  float* snc = snp + CM_J;                 // [NCH] child counts (dtype)
  float* smk = snc + NCH;                  // [NCH] 1: logit child non-empty
  float* spe = smk + NCH;                  // [64][CM_J] parent weights  (fp32 value-sum path)
  float* sce = spe + (TC ? 0 : CM_ROWS * CM_J);  // [64][NCH] child weights
  const int g = blockIdx.y, b = g / H, h = g % H, t0 = blockIdx.x * CM_ROWS;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r0 = warp * 16 + (lane >> 2), r1 = r0 + 8, cq = (lane & 3) * 2;
  const bool live0 = t0 + r0 < Tq, live1 = t0 + r1 < Tq;
  const long row0 = (long)g * Tq + (live0 ? t0 + r0 : 0), row1 = (long)g * Tq + (live1 ? t0 + r1 : 0);
  const float inv_sqrtD = 1.f / sqrtD;

  const T* qb = q + (long)b * qs.b + (long)h * qs.h;
  for (int i = tid; i < CM_ROWS * CPR; i += blockDim.x) {
    const int r = i / CPR, c = i % CPR, t = t0 + r;
    cp_async16(sQ + r * LDS + c * 8, qb + (long)(t < Tq ? t : 0) * qs.s + c * 8, t < Tq);
  }
  cp_async_commit();
  const float m0 = m_in[row0], m1 = m_in[row1];
  const float zc0 = clamp_min_nan2(z_in[row0], eps_dt<DT>()), zc1 = clamp_min_nan2(z_in[row1], eps_dt<DT>());
  const float rz0 = 1.f / zc0, rz1 = 1.f / zc1;
  const float bt0 = beta_in ? beta_in[row0] : 0.f, bt1 = beta_in ? beta_in[row1] : 0.f;
  float l0 = l_in[row0], l1 = l_in[row1];
  float oa[NT][4];
  const T* ab = a_in;
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int d = j * 8 + cq;
    const uint32_t w0 = *reinterpret_cast<const uint32_t*>(ab + row0 * D + d);
    const uint32_t w1 = *reinterpret_cast<const uint32_t*>(ab + row1 * D + d);
    oa[j][0] = half_lo<DT>(w0); oa[j][1] = half_hi<DT>(w0);
    oa[j][2] = half_lo<DT>(w1); oa[j][3] = half_hi<DT>(w1);
  }
  cp_async_wait<0>();
  __syncthreads();
  uint32_t af[KS][4];
#pragma unroll
  for (int k = 0; k < KS; ++k)
    ldsm_x4(af[k][0], af[k][1], af[k][2], af[k][3], sQ + (warp * 16 + (lane & 15)) * LDS + k * 16 + (lane >> 4) * 8);
  const int* sg = sel + (long)g * sel_stride;
  const T* pbase = parents + (long)h * M0 * D;
  const T* cbase = children + (long)h * M0 * C * D;
  const T* pvb = pagg + (long)g * M0 * D;
  const T* cvb = cagg + (long)g * M0 * C * D;

  for (int pass = 0; pass < npass; ++pass) {
    const int cnt = pass_cnt[pass];
    if (cnt <= 0) break;
    const bool quirk = multipass && cnt == M0;  // refinement.py:256-260
    double rl0 = 0.0, rl1 = 0.0, al0 = 0.0, al1 = 0.0;
    float ra[NT][4], aa[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) ra[j][e] = aa[j][e] = 0.f;
    for (int j0 = 0; j0 < cnt; j0 += CM_J) {
      __syncthreads();
      for (int i = tid; i < CM_J * CPR; i += blockDim.x) {
        const int jj = i / CPR, c = i % CPR, j = j0 + jj;
        const bool ok = j < cnt;
        const int p = ok ? sg[po.off[pass] + j] : 0;
        cp_async16(sP + jj * LDS + c * 8, pbase + (long)p * D + c * 8, ok);
        cp_async16(sPv + jj * LDS + c * 8, pvb + (long)p * D + c * 8, ok);
      }
      for (int i = tid; i < NCH * CPR; i += blockDim.x) {
        const int jc = i / CPR, c = i % CPR, jj = jc / C, ch = jc % C, j = j0 + jj;
        const bool ok = j < cnt;
        const int p = ok ? sg[po.off[pass] + j] : 0;
        const int pl = quirk ? j : p;
        cp_async16(sCh + jc * LDS + c * 8, cbase + ((long)pl * C + ch) * D + c * 8, ok);
        cp_async16(sCv + jc * LDS + c * 8, cvb + ((long)p * C + ch) * D + c * 8, ok);
      }
      cp_async_commit();
      if (tid < CM_J) {
        const int j = j0 + tid;
        snp[tid] = j < cnt ? count_dt<DT>(pcnt[(long)g * M0 + sg[po.off[pass] + j]]) : -1.f;
      }
      for (int jc = tid; jc < NCH; jc += blockDim.x) {
        const int jj = jc / C, ch = jc % C, j = j0 + jj;
        float n = 0.f, mk = 0.f;
        if (j < cnt) {
          const int p = sg[po.off[pass] + j];
          const int pl = quirk ? j : p;
          n = count_dt<DT>(ccnt[((long)g * M0 + p) * C + ch]);
          mk = ccnt[((long)g * M0 + pl) * C + ch] > 0 ? 1.f : 0.f;
        }
        snc[jc] = n;
        smk[jc] = mk;
      }
      cp_async_wait<0>();
      __syncthreads();
      // --- parent terms: logits of the selected parents -> pi -> weights
      float px[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) px[nt][0] = px[nt][1] = px[nt][2] = px[nt][3] = 0.f;
#pragma unroll
      for (int k = 0; k < KS; ++k) {
        uint32_t b0, b1, b2, b3;
        const int qd = lane >> 3;
        ldsm_x4(b0, b1, b2, b3, sP + ((qd >> 1) * 8 + (lane & 7)) * LDS + k * 16 + (qd & 1) * 8);
        mma16816<DT>(px[0], af[k], b0, b1);
        mma16816<DT>(px[1], af[k], b2, b3);
      }
      float pw[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int jj = nt * 8 + cq + (e & 1);
          const bool hi = e >= 2;
          const float n = snp[jj];
          float w = 0.f;
          if (n >= 0.f) {
            float s = n > 0.f ? scale_logit<DT>(rnd<DT>(px[nt][e]), sqrtD, inv_sqrtD) : -INFINITY;
            if (beta_in) s = rnd<DT>(__fmul_rn(hi ? bt1 : bt0, rnd<DT>(__fmul_rn(s, sqrtD))));
            float ex = exp_dt_fast<DT>(rnd<DT>(__fsub_rn(s, hi ? m1 : m0)));
            if (isnan(ex)) ex = 0.f;
            const float pi = div_dt_fast<DT>(ex, hi ? rz1 : rz0, hi ? zc1 : zc0);
            w = __fmul_rn(expf(__fsub_rn(pi, hi ? m1 : m0)), n);  // refinement.py:335
            if (hi) rl1 += (double)w; else rl0 += (double)w;
          }
          pw[nt][e] = w;
        }
      }
      // --- child terms
      float cw[2 * C][4];
#pragma unroll
      for (int nt = 0; nt < 2 * C; ++nt) cw[nt][0] = cw[nt][1] = cw[nt][2] = cw[nt][3] = 0.f;
#pragma unroll
      for (int k = 0; k < KS; ++k) {
#pragma unroll
        for (int jj = 0; jj < C; ++jj) {
          uint32_t b0, b1, b2, b3;
          const int qd = lane >> 3;
          ldsm_x4(b0, b1, b2, b3, sCh + (jj * 16 + (qd >> 1) * 8 + (lane & 7)) * LDS + k * 16 + (qd & 1) * 8);
          mma16816<DT>(cw[2 * jj], af[k], b0, b1);
          mma16816<DT>(cw[2 * jj + 1], af[k], b2, b3);
        }
      }
#pragma unroll
      for (int nt = 0; nt < 2 * C; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int jc = nt * 8 + cq + (e & 1);
          const bool hi = e >= 2;
          float w = 0.f;
          if (snp[jc / C] >= 0.f) {
            const float u = smk[jc] > 0.f ? scale_logit<DT>(rnd<DT>(cw[nt][e]), sqrtD, inv_sqrtD) : -INFINITY;
            w = __fmul_rn(expf(__fsub_rn(u, hi ? m1 : m0)), snc[jc]);  // refinement.py:341-343
            if (hi) al1 += (double)w; else al0 += (double)w;
          }
          cw[nt][e] = w;
        }
      }
      // --- value sums
      if constexpr (TC) {
#pragma unroll
        for (int part = 0; part < 3; ++part) {
          uint32_t ap[4];
          {
            float v[8];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float hi_, mid_, lo_;
              split3_bf16(pw[0][e], hi_, mid_, lo_);
              v[e] = part == 0 ? hi_ : (part == 1 ? mid_ : lo_);
              split3_bf16(pw[1][e], hi_, mid_, lo_);
              v[4 + e] = part == 0 ? hi_ : (part == 1 ? mid_ : lo_);
            }
            ap[0] = pack2<DT_BF16>(v[0], v[1]);
            ap[1] = pack2<DT_BF16>(v[2], v[3]);
            ap[2] = pack2<DT_BF16>(v[4], v[5]);
            ap[3] = pack2<DT_BF16>(v[6], v[7]);
          }
#pragma unroll
          for (int jj = 0; jj < NT / 2; ++jj) {
            uint32_t b0, b1, b2, b3;
            const int qd = lane >> 3;
            ldsm_x4_t(b0, b1, b2, b3, sPv + ((qd & 1) * 8 + (lane & 7)) * LDS + jj * 16 + (qd >> 1) * 8);
            mma16816<DT_BF16>(ra[2 * jj], ap, b0, b1);
            mma16816<DT_BF16>(ra[2 * jj + 1], ap, b2, b3);
          }
#pragma unroll
          for (int kc = 0; kc < C; ++kc) {
            uint32_t ac[4];
            float v[8];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float hi_, mid_, lo_;
              split3_bf16(cw[2 * kc][e], hi_, mid_, lo_);
              v[e] = part == 0 ? hi_ : (part == 1 ? mid_ : lo_);
              split3_bf16(cw[2 * kc + 1][e], hi_, mid_, lo_);
              v[4 + e] = part == 0 ? hi_ : (part == 1 ? mid_ : lo_);
            }
            ac[0] = pack2<DT_BF16>(v[0], v[1]);
            ac[1] = pack2<DT_BF16>(v[2], v[3]);
            ac[2] = pack2<DT_BF16>(v[4], v[5]);
            ac[3] = pack2<DT_BF16>(v[6], v[7]);
#pragma unroll
            for (int jj = 0; jj < NT / 2; ++jj) {
              uint32_t b0, b1, b2, b3;
              const int qd = lane >> 3;
              ldsm_x4_t(b0, b1, b2, b3, sCv + (kc * 16 + (qd & 1) * 8 + (lane & 7)) * LDS + jj * 16 + (qd >> 1) * 8);
              mma16816<DT_BF16>(aa[2 * jj], ac, b0, b1);
              mma16816<DT_BF16>(aa[2 * jj + 1], ac, b2, b3);
            }
          }
        }
      } else {
        // fp32 FMAs through shared memory (weights are per thread fragments)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) spe[((e >= 2) ? r1 : r0) * CM_J + nt * 8 + cq + (e & 1)] = pw[nt][e];
#pragma unroll
        for (int nt = 0; nt < 2 * C; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) sce[((e >= 2) ? r1 : r0) * NCH + nt * 8 + cq + (e & 1)] = cw[nt][e];
        __syncwarp();
#pragma unroll
        for (int j = 0; j < NT; ++j) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int r = e >= 2 ? r1 : r0, d = j * 8 + cq + (e & 1);
            float s1 = 0.f, s2 = 0.f;
            for (int jj = 0; jj < CM_J; ++jj) s1 = fmaf(spe[r * CM_J + jj], to_f(sPv[jj * LDS + d]), s1);
            for (int jc = 0; jc < NCH; ++jc) s2 = fmaf(sce[r * NCH + jc], to_f(sCv[jc * LDS + d]), s2);
            ra[j][e] += s1;
            aa[j][e] += s2;
          }
        }
      }
    }
    // OnlineSoftmaxState.replace with unit scales (attention.py:149-158)
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      rl0 += __shfl_xor_sync(0xffffffffu, rl0, o);
      rl1 += __shfl_xor_sync(0xffffffffu, rl1, o);
      al0 += __shfl_xor_sync(0xffffffffu, al0, o);
      al1 += __shfl_xor_sync(0xffffffffu, al1, o);
    }
    l0 = __fadd_rn(__fsub_rn(l0, __double2float_rn(rl0)), __double2float_rn(al0));
    l1 = __fadd_rn(__fsub_rn(l1, __double2float_rn(rl1)), __double2float_rn(al1));
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) oa[j][e] = __fadd_rn(__fsub_rn(oa[j][e], ra[j][e]), aa[j][e]);
  }
  const float den0 = clamp_min_nan2(l0, 1e-12f), den1 = clamp_min_nan2(l1, 1e-12f);
  float* o0 = out + (long)b * os.b + (long)(t0 + r0) * os.s + (long)h * os.h;
  float* o1 = out + (long)b * os.b + (long)(t0 + r1) * os.s + (long)h * os.h;
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int d = j * 8 + cq;
    if (live0) { o0[d] = __fdiv_rn(oa[j][0], den0); o0[d + 1] = __fdiv_rn(oa[j][1], den0); }
    if (live1) { o1[d] = __fdiv_rn(oa[j][2], den1); o1[d + 1] = __fdiv_rn(oa[j][3], den1); }
  }
}

size_t correct_mma_smem(int D, int C, int dt) {
  const int LDS = D + 8, NCH = 16 * C;
  size_t s = (size_t)(64 + 16 + NCH + 16 + NCH) * LDS * 2 + (16 + 2 * NCH) * sizeof(float);
  if (dt != DT_BF16) s += (size_t)64 * (16 + NCH) * sizeof(float);
  return s;
}

template <int DT>
int launch_correct_mma(const CorrArgs& a, cudaStream_t st) {
  using T = typename Storage<DT>::T;
  const int G = a.B * a.H, nqt = (a.T + CM_ROWS - 1) / CM_ROWS;
  PassOffsets po;
  for (int k = 0; k < 8; ++k) po.off[k] = a.pass_off[k];
  const size_t smem = correct_mma_smem(a.D, a.C <= 4 ? 4 : 8, DT);
  auto go = [&](auto kfn) {
    AVQ_TIMED("correct", st);
    cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kfn<<<dim3(nqt, G), 128, smem, st>>>((const T*)a.q, a.qs, a.H, a.T, a.M0, a.sqrtD, (const T*)a.parents,
                                          (const T*)a.children, (const T*)a.pagg, (const T*)a.cagg, a.pcnt, a.ccnt,
                                          a.m, a.l, a.z, a.beta, (const T*)a.a, a.sel, a.sel_stride, a.pass_cnt,
                                          a.npass, po, a.multipass, a.out, a.os);
  };
  if (a.C == 4) {
    if (a.D == 64) go(correct_mma_kernel<DT, 64, 4>); else go(correct_mma_kernel<DT, 128, 4>);
  } else if (a.C == 8) {
    if (a.D == 64) go(correct_mma_kernel<DT, 64, 8>); else go(correct_mma_kernel<DT, 128, 8>);
  } else {
    return AVQ_ERR_UNSUPPORTED;
  }
  return cudaPeekAtLastError() == cudaSuccess ? AVQ_OK : AVQ_ERR_CUDA;
}

template int launch_correct_mma<DT_BF16>(const CorrArgs&, cudaStream_t);
template int launch_correct_mma<DT_F16>(const CorrArgs&, cudaStream_t);

// ---------------------------------------------------------------------------
size_t parent_attn_mma_smem(int D, int M0, bool s_in_smem, int dt_bytes) {
  size_t s = (size_t)(PM_ROWS + 2 * PM_CH) * (D + 8) * dt_bytes + 2 * PM_CH * sizeof(float) + PM_CH * sizeof(double);
  if (s_in_smem) s += (size_t)PM_ROWS * (M0 + 8) * dt_bytes;
  return s;
}

bool parent_attn_mma_ok(int dt, int D, int M0) { return dt != DT_F32 && (D == 64 || D == 128) && M0 % 8 == 0; }

// Shared-memory logits cost occupancy (64 x M0 dtype values per 4-warp CTA);
// the per-CTA global slice (64 x M0) stays L2-resident while the CTA runs.
bool parent_attn_mma_smem_mode(int D, int M0) { return M0 <= PM_MAX_SMEM_M0 && M0 <= 128; }

size_t parent_attn_mma_scratch(int G, int T, int M0, int dt_bytes) {
  const int nqt = (T + PM_ROWS - 1) / PM_ROWS;
  return (size_t)G * nqt * PM_ROWS * (M0 + 8) * dt_bytes;
}

template <int DT>
int launch_parent_attn_mma(const PAArgs& a, cudaStream_t st) {
  using T = typename Storage<DT>::T;
  const int G = a.B * a.H, nqt = (a.T + PM_ROWS - 1) / PM_ROWS;
  const bool sm = a.s_in_smem;
  const size_t smem = parent_attn_mma_smem(a.D, a.M0, sm, sizeof(T));
  auto go = [&](auto kfn) {
    AVQ_TIMED(a.mode ? "parent_attn_hvaq" : "parent_attn", st);
    cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kfn<<<dim3(nqt, G), 128, smem, st>>>((const T*)a.q, a.qs, a.H, a.T, a.M0, a.sqrtD, (const T*)a.parents,
                                          (const T*)a.pagg, a.pcnt, a.mode, (T*)a.sglobal, a.m, a.l, a.z, (T*)a.a,
                                          a.imp_part, a.sel0, a.sel_stride, a.pass_cnt, a.hvaq, a.beta0, a.alpha,
                                          a.beta, sm ? 1 : 0, a.keep_logits);
  };
  if (a.D == 64) go(parent_attn_mma_kernel<DT, 64>);
  else go(parent_attn_mma_kernel<DT, 128>);
  return cudaPeekAtLastError() == cudaSuccess ? AVQ_OK : AVQ_ERR_CUDA;
}

template int launch_parent_attn_mma<DT_BF16>(const PAArgs&, cudaStream_t);
template int launch_parent_attn_mma<DT_F16>(const PAArgs&, cudaStream_t);

}  // namespace avq
