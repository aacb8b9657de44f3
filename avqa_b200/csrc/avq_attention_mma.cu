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

// ---------------------------------------------------------------------------
// Parent attention kernel.  CTA = 64 queries = 4 warps x 16 rows; a lane quad
// owns two rows (r0, r0+8) and a quarter of their columns, so row statistics
// combine with two shuffles.  The logits / exponentials of the CTA's rows live
// in a per-CTA global slice (64 x exp_slice_pitch(M0) dtype values, L2-resident while the
// CTA runs) that the routing kernel can re-read for its exactness fallback.
// ---------------------------------------------------------------------------
template <int DT, int D>
__global__ void __launch_bounds__(128, 4) parent_attn_mma_kernel(
    const typename Storage<DT>::T* __restrict__ q, Strides3 qs, int H, int Tq, int M0, float sqrtD,
    const typename Storage<DT>::T* __restrict__ parents, const typename Storage<DT>::T* __restrict__ pagg,
    const int* __restrict__ pcnt, int mode, int keep_logits, typename Storage<DT>::T* __restrict__ scratch,
    float* __restrict__ m_io, float* __restrict__ l_out, float* __restrict__ z_io,
    typename Storage<DT>::T* __restrict__ a_out, float* __restrict__ colpart, const int* __restrict__ sel0,
    int sel_stride, const int* __restrict__ pass_cnt, int hvaq, float beta0, float alpha,
    float* __restrict__ beta_out, int sG, const unsigned int* __restrict__ present) {
  using T = typename Storage<DT>::T;
  constexpr int LDS = D + 8, KS = D / 16, CPR = D / 8, NT = D / 8;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* sq_ = (T*)smem_raw;                      // [64][LDS] queries
  T* sb = sq_ + PM_ROWS * LDS;                // [2][PM_CH][LDS] parents / parent sums
  float* sn = (float*)(sb + 2 * PM_CH * LDS);  // [2][PM_CH] counts
  float* srow = sn + 2 * PM_CH;                // [64][4] per-row zc, 1/zc, max, live
  float* scomb = srow + 4 * PM_ROWS;           // [4][64] column partials of the 4 warps
  const int g = blockIdx.y, b = g / H, h = g % H, qt = blockIdx.x, t0 = qt * PM_ROWS, nqt = gridDim.x, gs = g % sG;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int LDL = exp_slice_pitch(M0);
  const float inv_sqrtD = 1.f / sqrtD;
  T* S_ = scratch + ((long)g * nqt + qt) * PM_ROWS * LDL;
  const int r0 = warp * 16 + (lane >> 2), r1 = r0 + 8, cq = (lane & 3) * 2;
  const bool live0 = t0 + r0 < Tq, live1 = t0 + r1 < Tq;
  const int nch = (M0 + PM_CH - 1) / PM_CH;
  const T* qb = q + (long)b * qs.b + (long)h * qs.h;
  for (int i = tid; i < PM_ROWS * CPR; i += blockDim.x) {
    const int r = i / CPR, c = i % CPR, t = t0 + r;
    cp_async16(sq_ + r * LDS + c * 8, qb + (long)(t < Tq ? t : 0) * qs.s + c * 8, t < Tq);
  }
  cp_async_commit();
  const T* pb = parents + (long)h * M0 * D;
  const T* vb = pagg + (long)gs * M0 * D;
  auto load_rows = [&](const T* src, int buf, int p0, bool dtype_counts) {
    for (int i = tid; i < PM_CH * CPR; i += blockDim.x) {
      const int r = i / CPR, c = i % CPR, p = p0 + r;
      cp_async16(sb + (buf * PM_CH + r) * LDS + c * 8, src + (long)(p < M0 ? p : 0) * D + c * 8, p < M0);
    }
    if (tid < PM_CH) {
      const int p = p0 + tid;
      const int n = p < M0 ? pcnt[(long)gs * M0 + p] : 0;
      sn[buf * PM_CH + tid] = dtype_counts ? count_dt<DT>(n) : (float)n;
    }
  };

  uint32_t mx0 = dup2<DT>(-INFINITY), mx1 = mx0;  // packed running row maxima
  if (mode == 0) {
    // ---- phase 1: logits (pipeline.py:81,107) ----
    load_rows(pb, 0, 0, false);
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    uint32_t af[KS][4];
#pragma unroll
    for (int k = 0; k < KS; ++k)
      ldsm_x4(af[k][0], af[k][1], af[k][2], af[k][3], sq_ + (warp * 16 + (lane & 15)) * LDS + k * 16 + (lane >> 4) * 8);
    for (int ci = 0; ci < nch; ++ci) {
      const int buf = ci & 1, p0 = ci * PM_CH;
      if (ci + 1 < nch) load_rows(pb, buf ^ 1, p0 + PM_CH, false);
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
          const float x = rnd<DT>(acc[j][e]);
          // pipeline.py:106 (user / causal mask), :107 (empty); element e is column cl + (e & 1)
          const int tq = t0 + (e >= 2 ? r1 : r0), pe = p + (e & 1);
          const bool vis =
              !present || (tq < Tq && pe < M0 && present_bit(present, (M0 + 31) >> 5, (long)g * Tq + tq, pe));
          s[e] = nb[cl + (e & 1)] > 0.f && vis ? scale_logit<DT>(x, sqrtD, inv_sqrtD) : -INFINITY;
        }
        const uint32_t s01 = pack2<DT>(s[0], s[1]), s23 = pack2<DT>(s[2], s[3]);
        if (p < M0) {
          mx0 = hmax2_nan_dt<DT>(mx0, s01);
          mx1 = hmax2_nan_dt<DT>(mx1, s23);
          *reinterpret_cast<uint32_t*>(S_ + (long)r0 * LDL + p) = s01;
          *reinterpret_cast<uint32_t*>(S_ + (long)r1 * LDL + p) = s23;
        }
      }
      cp_async_wait<0>();
      __syncthreads();
    }
  } else {
    // ---- HVAQ (pipeline.py:192-258, hopfield.py:55-144) on the stored logits ----
    cp_async_wait<0>();
    __syncthreads();
    const int nsel = pass_cnt[0];
    const int* sl = sel0 + (long)g * sel_stride;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int r = half ? r1 : r0;
      const bool live = half ? live1 : live0;
      const long row = (long)g * Tq + (live ? t0 + r : 0);
      const float safe0 = live ? m_io[row] : 0.f;
      const float zc0 = clamp_min_nan(live ? z_io[row] : 1.f, eps_dt<DT>());
      T* Sr = S_ + (long)r * LDL;
      double gs = 0.0;
      for (int j = lane & 3; j < nsel; j += 4) {
        float e = exp_rn<DT>(rnd<DT>(__fsub_rn(to_f(Sr[sl[j]]), safe0)));
        if (isnan(e)) e = 0.f;
        gs += (double)rnd<DT>(__fdiv_rn(e, zc0));
      }
      gs += __shfl_xor_sync(0xffffffffu, gs, 1);
      gs += __shfl_xor_sync(0xffffffffu, gs, 2);
      const float gsc = clamp_min_nan(rnd64<DT>(gs), eps_dt<DT>());
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
      uint32_t mx = dup2<DT>(-INFINITY);
      for (int p = (lane & 3) * 2; p < M0; p += 8) {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(Sr + p);
        const float sA = rnd<DT>(__fmul_rn(beta, rnd<DT>(__fmul_rn(half_lo<DT>(w), sqrtD))));
        const float sB = rnd<DT>(__fmul_rn(beta, rnd<DT>(__fmul_rn(half_hi<DT>(w), sqrtD))));
        const uint32_t nw = pack2<DT>(sA, sB);
        *reinterpret_cast<uint32_t*>(Sr + p) = nw;
        mx = hmax2_nan_dt<DT>(mx, nw);
      }
      if (half) mx1 = mx; else mx0 = mx;
    }
  }
  float rm0 = nanmax(half_lo<DT>(mx0), half_hi<DT>(mx0)), rm1 = nanmax(half_lo<DT>(mx1), half_hi<DT>(mx1));
  rm0 = nanmax(rm0, __shfl_xor_sync(0xffffffffu, rm0, 1));
  rm0 = nanmax(rm0, __shfl_xor_sync(0xffffffffu, rm0, 2));
  rm1 = nanmax(rm1, __shfl_xor_sync(0xffffffffu, rm1, 1));
  rm1 = nanmax(rm1, __shfl_xor_sync(0xffffffffu, rm1, 2));
  const float safe0 = rm0 == -INFINITY ? 0.f : rm0;  // pipeline.py:137-141
  const float safe1 = rm1 == -INFINITY ? 0.f : rm1;
  const uint32_t sf0 = dup2<DT>(safe0), sf1 = dup2<DT>(safe1);
  __syncthreads();

  // ---- phase 2: e, l = sum dtype(e*n), z = sum e, a = e @ V (pipeline.py:142-147) ----
  float la0 = 0.f, la1 = 0.f, za0 = 0.f, za1 = 0.f;
  float oacc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) oacc[j][0] = oacc[j][1] = oacc[j][2] = oacc[j][3] = 0.f;
  load_rows(vb, 0, 0, true);
  cp_async_commit();
  // logits of the next 16-column step are loaded one step ahead
  auto load_s = [&](int pk, uint32_t (&s)[4]) {
#pragma unroll
    for (int hh = 0; hh < 4; ++hh) {
      const int p = pk + cq + ((hh >> 1) << 3);
      s[hh] = p < M0 ? *reinterpret_cast<const uint32_t*>(S_ + (long)((hh & 1) ? r1 : r0) * LDL + p) : 0u;
    }
  };
  uint32_t snext[4];
  load_s(0, snext);
  for (int ci = 0; ci < nch; ++ci) {
    const int buf = ci & 1, p0 = ci * PM_CH;
    cp_async_wait<0>();
    __syncthreads();
    if (ci + 1 < nch) load_rows(vb, buf ^ 1, p0 + PM_CH, true);
    cp_async_commit();
    const float* nb = sn + buf * PM_CH;
    const T* svb = sb + buf * PM_CH * LDS;
#pragma unroll
    for (int k = 0; k < PM_CH / 16; ++k) {
      uint32_t a[4], scur[4];
#pragma unroll
      for (int hh = 0; hh < 4; ++hh) scur[hh] = snext[hh];
      load_s(p0 + k * 16 + 16, snext);
#pragma unroll
      for (int hh = 0; hh < 4; ++hh) {  // a[hh]: rows (hh&1 ? r1 : r0), columns +8*(hh>>1)
        const int cl = k * 16 + cq + ((hh >> 1) << 3), p = p0 + cl;
        const int r = (hh & 1) ? r1 : r0;
        uint32_t e2 = 0u;
        if (p < M0) {
          const uint32_t s2 = scur[hh];
          const uint32_t d2 = hsub2_dt<DT>(s2, (hh & 1) ? sf1 : sf0);
          const float e0 = fmaxf(exp_dt_fast<DT>(half_lo<DT>(d2)), 0.f);  // NaN -> 0 (pipeline.py:143-145)
          const float e1 = fmaxf(exp_dt_fast<DT>(half_hi<DT>(d2)), 0.f);
          const float w0 = rnd<DT>(e0 * nb[cl]), w1 = rnd<DT>(e1 * nb[cl + 1]);  // exact products
          if (hh & 1) { la1 += w0 + w1; za1 += e0 + e1; } else { la0 += w0 + w1; za0 += e0 + e1; }
          e2 = pack2<DT>(e0, e1);
          if (!keep_logits) *reinterpret_cast<uint32_t*>(S_ + (long)r * LDL + p) = e2;
        }
        a[hh] = e2;
      }
      const uint32_t af2[4] = {a[0], a[1], a[2], a[3]};
#pragma unroll
      for (int jj = 0; jj < NT / 2; ++jj) {
        uint32_t b0, b1, b2, b3;
        const int qd = lane >> 3;
        ldsm_x4_t(b0, b1, b2, b3, svb + (k * 16 + (qd & 1) * 8 + (lane & 7)) * LDS + jj * 16 + (qd >> 1) * 8);
        mma16816<DT>(oacc[2 * jj], af2, b0, b1);
        mma16816<DT>(oacc[2 * jj + 1], af2, b2, b3);
      }
    }
  }
  cp_async_wait<0>();
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    la0 += __shfl_xor_sync(0xffffffffu, la0, o);
    la1 += __shfl_xor_sync(0xffffffffu, la1, o);
    za0 += __shfl_xor_sync(0xffffffffu, za0, o);
    za1 += __shfl_xor_sync(0xffffffffu, za1, o);
  }
  // z feeds the probabilities (an index-relevant quantity): the fp32 sum is
  // within M0 * 2^-23 relative of the exact one; when that interval straddles
  // a dtype rounding point the row is summed again exactly.
  float zd[2];
  __syncwarp();
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const float za = hh ? za1 : za0;
    const float eps = za * (float)M0 * 1.1920929e-7f;
    const float lo = rnd<DT>(za - eps), hi = rnd<DT>(za + eps);
    float z = rnd<DT>(za);
    const bool amb = lo != hi;
    if (__any_sync(0xffffffffu, amb)) {
      double ex = 0.0;
      if (amb) {
        const int r = hh ? r1 : r0;
        const float sf = hh ? safe1 : safe0;
        const T* Sr = S_ + (long)r * LDL;
        for (int p = lane & 3; p < M0; p += 4) {
          float e = to_f(Sr[p]);
          if (keep_logits) e = fmaxf(exp_dt_fast<DT>(rnd<DT>(e - sf)), 0.f);
          ex += (double)e;
        }
      }
      ex += __shfl_xor_sync(0xffffffffu, ex, 1);
      ex += __shfl_xor_sync(0xffffffffu, ex, 2);
      if (amb) z = rnd64<DT>(ex);
    }
    zd[hh] = z;
  }
  const long row0 = (long)g * Tq + t0 + r0, row1 = (long)g * Tq + t0 + r1;
  if ((lane & 3) == 0) {
    if (live0) { m_io[row0] = safe0; l_out[row0] = rnd<DT>(la0); z_io[row0] = zd[0]; }
    if (live1) { m_io[row1] = safe1; l_out[row1] = rnd<DT>(la1); z_io[row1] = zd[1]; }
    const float zc0 = clamp_min_nan(zd[0], eps_dt<DT>()), zc1 = clamp_min_nan(zd[1], eps_dt<DT>());
    srow[r0 * 4] = zc0;
    srow[r0 * 4 + 1] = 1.f / zc0;
    srow[r0 * 4 + 2] = safe0;
    srow[r0 * 4 + 3] = live0 ? 1.f : 0.f;
    srow[r1 * 4] = zc1;
    srow[r1 * 4 + 1] = 1.f / zc1;
    srow[r1 * 4 + 2] = safe1;
    srow[r1 * 4 + 3] = live1 ? 1.f : 0.f;
  }
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int d = j * 8 + cq;
    if (live0) *reinterpret_cast<uint32_t*>(a_out + row0 * D + d) = pack2<DT>(rnd<DT>(oacc[j][0]), rnd<DT>(oacc[j][1]));
    if (live1) *reinterpret_cast<uint32_t*>(a_out + row1 * D + d) = pack2<DT>(rnd<DT>(oacc[j][2]), rnd<DT>(oacc[j][3]));
  }
  __syncthreads();

  // ---- phase 3: probs (pipeline.py:150) summed over the CTA's queries ----
  // warp w sums its 16 rows for 64 columns (2 per lane, coalesced row reads),
  // the 4 warp partials are combined through shared memory.
  for (int p0 = 0; p0 < M0; p0 += 64) {
    const int p = p0 + 2 * lane;
    float c0 = 0.f, c1 = 0.f;
    if (p < M0) {
      uint32_t ws[16];
#pragma unroll
      for (int rr = 0; rr < 16; ++rr) ws[rr] = *reinterpret_cast<const uint32_t*>(S_ + (long)(warp * 16 + rr) * LDL + p);
#pragma unroll
      for (int rr = 0; rr < 16; ++rr) {
        const int r = warp * 16 + rr;
        if (srow[r * 4 + 3] == 0.f) continue;  // query beyond T
        const float zc = srow[r * 4], rz = srow[r * 4 + 1];
        const uint32_t w = ws[rr];
        float e0 = half_lo<DT>(w), e1 = half_hi<DT>(w);
        if (keep_logits) {  // the slice still holds logits (an HVAQ pass follows)
          const float sf = srow[r * 4 + 2];
          e0 = fmaxf(exp_dt_fast<DT>(rnd<DT>(e0 - sf)), 0.f);
          e1 = fmaxf(exp_dt_fast<DT>(rnd<DT>(e1 - sf)), 0.f);
        }
        c0 += div_dt_fast<DT>(e0, rz, zc);
        c1 += div_dt_fast<DT>(e1, rz, zc);
      }
    }
    scomb[warp * 64 + 2 * lane] = c0;
    scomb[warp * 64 + 2 * lane + 1] = c1;
    __syncthreads();
    if (tid < 64 && p0 + tid < M0) {
      const float s = (scomb[tid] + scomb[64 + tid]) + (scomb[128 + tid] + scomb[192 + tid]);
      colpart[((long)g * nqt + qt) * M0 + p0 + tid] = s;
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Tensor-core child correction (refinement.py:82-304, attention.py:100-163,
// multipass.py:207-262, attention_module.py:532-535).
//
// CTA = 64 queries (4 warps x 16 rows).  The selected parents of a pass are
// staged 16 at a time with their children.  Per query and slot: the parent's
// logit (MMA, narrowed exactly as in the parent pass, HVAQ-rescaled when
// active) gives the probability pi; the parent term exp(pi - m) * n and the
// child terms exp(u - m) * n_c are fp32.  The denominator terms accumulate in
// fp64.  The value terms  -sum w_p V_p + sum w_c V_c  are accumulated straight
// into the fp32 state a on the tensor cores, every fp32 weight split into
// three bf16 parts (24 significant bits); fp16 value sums, whose weights may
// exceed the fp16 range, use fp32 FMAs.  Children are processed 16 at a time
// so only one group of logits is live.
// ---------------------------------------------------------------------------
constexpr int CM_ROWS = 64;
constexpr int CM_J = 16;

__device__ __forceinline__ void split3(float w, float& hi, float& mid, float& lo) {
  hi = __bfloat162float(__float2bfloat16_rn(w));
  const float r = w - hi;
  mid = __bfloat162float(__float2bfloat16_rn(r));
  lo = __bfloat162float(__float2bfloat16_rn(r - mid));
}

// Three bf16 A fragments (hi, mid, lo parts) of a 16x16 weight block held as
// two m16n8 accumulator tiles t0 (k 0-7) and t1 (k 8-15).
__device__ __forceinline__ void weight_frags(const float* t0, const float* t1, uint32_t (&fr)[3][4]) {
  float h[8], m[8], l[8];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    split3(t0[e], h[e], m[e], l[e]);
    split3(t1[e], h[4 + e], m[4 + e], l[4 + e]);
  }
  const float* parts[3] = {h, m, l};
#pragma unroll
  for (int s = 0; s < 3; ++s) {
    fr[s][0] = pack2<DT_BF16>(parts[s][0], parts[s][1]);
    fr[s][1] = pack2<DT_BF16>(parts[s][2], parts[s][3]);
    fr[s][2] = pack2<DT_BF16>(parts[s][4], parts[s][5]);
    fr[s][3] = pack2<DT_BF16>(parts[s][6], parts[s][7]);
  }
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
    Strides3 os, int sG, const unsigned int* __restrict__ present) {
  using T = typename Storage<DT>::T;
  constexpr bool TC = DT == DT_BF16;  // tensor-core value sums
  constexpr int LDS = D + 8, KS = D / 16, CPR = D / 8, NT = D / 8, NCH = CM_J * C;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* sQ = (T*)smem_raw;            // [64][LDS]
  T* sP = sQ + CM_ROWS * LDS;      // [CM_J][LDS] selected parents (logit rows)
  T* sCh = sP + CM_J * LDS;        // [NCH][LDS] children (logit rows)
  T* sPv = sCh + NCH * LDS;        // [CM_J][LDS] parent sums
  T* sCv = sPv + CM_J * LDS;       // [NCH][LDS] child sums
  float* snp = (float*)(sCv + NCH * LDS);  // [CM_J] parent counts (dtype); < 0: empty slot
  float* snc = snp + CM_J;                 // [NCH] child counts (dtype)
  float* smk = snc + NCH;                  // [NCH] 1: logit child non-empty
  float* sw = smk + NCH;                   // fp16 path: [64][16] weights of one group
  int* spi = reinterpret_cast<int*>(sw + CM_ROWS * 16);  // [CM_J] the selected parents (-1: empty slot)
  const int g = blockIdx.y, b = g / H, h = g % H, t0 = blockIdx.x * CM_ROWS, gs = g % sG;
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
  const float zc0 = clamp_min_nan(z_in[row0], eps_dt<DT>()), zc1 = clamp_min_nan(z_in[row1], eps_dt<DT>());
  const float rz0 = 1.f / zc0, rz1 = 1.f / zc1;
  const float bt0 = beta_in ? beta_in[row0] : 0.f, bt1 = beta_in ? beta_in[row1] : 0.f;
  float l0 = l_in[row0], l1 = l_in[row1];
  // the fp32 state a (attention.py:154-158) doubles as the MMA accumulator
  float oa[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int d = j * 8 + cq;
    const uint32_t w0 = *reinterpret_cast<const uint32_t*>(a_in + row0 * D + d);
    const uint32_t w1 = *reinterpret_cast<const uint32_t*>(a_in + row1 * D + d);
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
  const T* pvb = pagg + (long)gs * M0 * D;
  const T* cvb = cagg + (long)gs * M0 * C * D;

  // 16 rows x 16 slots of logits -> weights w (two m16n8 tiles), then
  // oa += sign * w @ V[16 slots] (V rows staged in sv)
  auto value_sum = [&](const float (&wt)[2][4], const T* sv, float sign) {
    if constexpr (TC) {
      float t0f[4], t1f[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) { t0f[e] = sign * wt[0][e]; t1f[e] = sign * wt[1][e]; }
      uint32_t fr[3][4];
      weight_frags(t0f, t1f, fr);
#pragma unroll
      for (int s = 0; s < 3; ++s) {
#pragma unroll
        for (int jj = 0; jj < NT / 2; ++jj) {
          uint32_t b0, b1, b2, b3;
          const int qd = lane >> 3;
          ldsm_x4_t(b0, b1, b2, b3, sv + ((qd & 1) * 8 + (lane & 7)) * LDS + jj * 16 + (qd >> 1) * 8);
          mma16816<DT_BF16>(oa[2 * jj], fr[s], b0, b1);
          mma16816<DT_BF16>(oa[2 * jj + 1], fr[s], b2, b3);
        }
      }
    } else {
      // fp32 FMAs: weights of the warp's 16 rows through shared memory
      float* wr = sw + warp * 16 * 16;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        wr[(lane >> 2) * 16 + nt * 8 + cq] = sign * wt[nt][0];
        wr[(lane >> 2) * 16 + nt * 8 + cq + 1] = sign * wt[nt][1];
        wr[((lane >> 2) + 8) * 16 + nt * 8 + cq] = sign * wt[nt][2];
        wr[((lane >> 2) + 8) * 16 + nt * 8 + cq + 1] = sign * wt[nt][3];
      }
      __syncwarp();
#pragma unroll
      for (int j = 0; j < NT; ++j) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int rr = (lane >> 2) + ((e >> 1) << 3), d = j * 8 + cq + (e & 1);
          float s = 0.f;
#pragma unroll
          for (int k = 0; k < 16; ++k) s = fmaf(wr[rr * 16 + k], to_f(sv[k * LDS + d]), s);
          oa[j][e] += s;
        }
      }
      __syncwarp();
    }
  };

  for (int pass = 0; pass < npass; ++pass) {
    const int cnt = pass_cnt[pass];
    if (cnt <= 0) break;
    const bool quirk = multipass && cnt == M0;  // refinement.py:256-260
    double rl0 = 0.0, rl1 = 0.0, al0 = 0.0, al1 = 0.0;
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
        snp[tid] = j < cnt ? count_dt<DT>(pcnt[(long)gs * M0 + sg[po.off[pass] + j]]) : -1.f;
        spi[tid] = j < cnt ? sg[po.off[pass] + j] : -1;
      }
      for (int jc = tid; jc < NCH; jc += blockDim.x) {
        const int jj = jc / C, ch = jc % C, j = j0 + jj;
        float n = 0.f, mk = 0.f;
        if (j < cnt) {
          const int p = sg[po.off[pass] + j];
          const int pl = quirk ? j : p;
          n = count_dt<DT>(ccnt[((long)gs * M0 + p) * C + ch]);
          mk = ccnt[((long)gs * M0 + pl) * C + ch] > 0 ? 1.f : 0.f;
        }
        snc[jc] = n;
        smk[jc] = mk;
      }
      cp_async_wait<0>();
      __syncthreads();
      // ---- parent terms: probabilities of the selected parents ----
      {
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
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const bool hi = e >= 2;
            const float n = snp[nt * 8 + cq + (e & 1)];
            float w = 0.f;
            if (n >= 0.f) {
              // a parent masked for this query (pipeline.py:106) has probability 0
              const int tq = t0 + (hi ? r1 : r0), pp = spi[nt * 8 + cq + (e & 1)];
              const bool vis = !present || tq >= Tq || present_bit(present, (M0 + 31) >> 5, (long)g * Tq + tq, pp);
              float s = n > 0.f && vis ? scale_logit<DT>(rnd<DT>(px[nt][e]), sqrtD, inv_sqrtD) : -INFINITY;
              if (beta_in) s = rnd<DT>(__fmul_rn(hi ? bt1 : bt0, rnd<DT>(__fmul_rn(s, sqrtD))));
              const float ex = fmaxf(exp_dt_fast<DT>(rnd<DT>(s - (hi ? m1 : m0))), 0.f);
              const float pi = div_dt_fast<DT>(ex, hi ? rz1 : rz0, hi ? zc1 : zc0);
              w = __fmul_rn(expf(__fsub_rn(pi, hi ? m1 : m0)), n);  // refinement.py:335
              if (hi) rl1 += (double)w; else rl0 += (double)w;
            }
            px[nt][e] = w;
          }
        }
        value_sum(px, sPv, -1.f);
      }
      // ---- child terms, 16 children at a time ----
#pragma unroll 1
      for (int cg = 0; cg < C; ++cg) {
        float cw[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) cw[nt][0] = cw[nt][1] = cw[nt][2] = cw[nt][3] = 0.f;
#pragma unroll
        for (int k = 0; k < KS; ++k) {
          uint32_t b0, b1, b2, b3;
          const int qd = lane >> 3;
          ldsm_x4(b0, b1, b2, b3, sCh + (cg * 16 + (qd >> 1) * 8 + (lane & 7)) * LDS + k * 16 + (qd & 1) * 8);
          mma16816<DT>(cw[0], af[k], b0, b1);
          mma16816<DT>(cw[1], af[k], b2, b3);
        }
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int jc = cg * 16 + nt * 8 + cq + (e & 1);
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
        value_sum(cw, sCv + cg * 16 * LDS, 1.f);
      }
    }
    // OnlineSoftmaxState.replace with unit scales (attention.py:149-153)
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      rl0 += __shfl_xor_sync(0xffffffffu, rl0, o);
      rl1 += __shfl_xor_sync(0xffffffffu, rl1, o);
      al0 += __shfl_xor_sync(0xffffffffu, al0, o);
      al1 += __shfl_xor_sync(0xffffffffu, al1, o);
    }
    l0 = __fadd_rn(__fsub_rn(l0, __double2float_rn(rl0)), __double2float_rn(al0));
    l1 = __fadd_rn(__fsub_rn(l1, __double2float_rn(rl1)), __double2float_rn(al1));
  }
  const float den0 = clamp_min_nan(l0, 1e-12f), den1 = clamp_min_nan(l1, 1e-12f);
  float* o0 = out + (long)b * os.b + (long)(t0 + r0) * os.s + (long)h * os.h;
  float* o1 = out + (long)b * os.b + (long)(t0 + r1) * os.s + (long)h * os.h;
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int d = j * 8 + cq;
    if (live0) *reinterpret_cast<float2*>(o0 + d) = make_float2(__fdiv_rn(oa[j][0], den0), __fdiv_rn(oa[j][1], den0));
    if (live1) *reinterpret_cast<float2*>(o1 + d) = make_float2(__fdiv_rn(oa[j][2], den1), __fdiv_rn(oa[j][3], den1));
  }
}

size_t correct_mma_smem(int D, int C, int dt) {
  const int LDS = D + 8, NCH = 16 * C;
  return (size_t)(64 + 16 + NCH + 16 + NCH) * LDS * 2 + (16 + 2 * NCH) * sizeof(float) + 64 * 16 * sizeof(float) +
         16 * sizeof(int);
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
                                          a.npass, po, a.multipass, a.out, a.os, a.sG > 0 ? a.sG : G, a.present);
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
  (void)M0;
  (void)s_in_smem;
  return (size_t)(PM_ROWS + 2 * PM_CH) * (D + 8) * dt_bytes + (2 * PM_CH + 4 * PM_ROWS + 4 * 64) * sizeof(float);
}

bool parent_attn_mma_ok(int dt, int D, int M0) { return dt != DT_F32 && (D == 64 || D == 128) && M0 % 8 == 0; }

// The logits always live in the per-CTA global slice (64 x exp_slice_pitch(M0) dtype
// values): shared-memory logits would cost occupancy, and the routing
// kernel's exactness fallback re-reads the slices.
bool parent_attn_mma_smem_mode(int D, int M0) { return false; }

size_t parent_attn_mma_scratch(int G, int T, int M0, int dt_bytes) {
  const int nqt = (T + PM_ROWS - 1) / PM_ROWS;
  return (size_t)G * nqt * PM_ROWS * exp_slice_pitch(M0) * dt_bytes;
}

template <int DT>
int launch_parent_attn_mma(const PAArgs& a, cudaStream_t st) {
  using T = typename Storage<DT>::T;
  const int G = a.B * a.H, nqt = (a.T + PM_ROWS - 1) / PM_ROWS;
  const size_t smem = parent_attn_mma_smem(a.D, a.M0, false, sizeof(T));
  auto go = [&](auto kfn) {
    AVQ_TIMED(a.mode ? "parent_attn_hvaq" : "parent_attn", st);
    cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kfn<<<dim3(nqt, G), 128, smem, st>>>((const T*)a.q, a.qs, a.H, a.T, a.M0, a.sqrtD, (const T*)a.parents,
                                          (const T*)a.pagg, a.pcnt, a.mode, a.keep_logits, (T*)a.sglobal, a.m, a.l,
                                          a.z, (T*)a.a, a.colpart, a.sel0, a.sel_stride, a.pass_cnt, a.hvaq, a.beta0,
                                          a.alpha, a.beta, a.sG > 0 ? a.sG : G, a.present);
  };
  if (a.D == 64) go(parent_attn_mma_kernel<DT, 64>);
  else go(parent_attn_mma_kernel<DT, 128>);
  return cudaPeekAtLastError() == cudaSuccess ? AVQ_OK : AVQ_ERR_CUDA;
}

template int launch_parent_attn_mma<DT_BF16>(const PAArgs&, cudaStream_t);
template int launch_parent_attn_mma<DT_F16>(const PAArgs&, cudaStream_t);

}  // namespace avq
