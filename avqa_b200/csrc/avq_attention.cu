// Parent attention, routing and the child correction (reference
// pipeline.py:46-399, routing.py:24-170, hopfield.py:55-144,
// refinement.py:82-304, multipass.py:40-264, attention_module.py:471-544).
//
//   parent_attn (mode 0): logits over all parents, row max, the dtype-rounded
//       exponentials, l = sum e*n, z = sum e, a = e @ V (V = parent sums),
//       probs = e / max(z, eps) and per-query-tile importance partial sums.
//   parent_attn (mode 1): the HVAQ temperature: beta per query from the
//       entropy of the renormalised top-P probabilities, logits rescaled,
//       then the same softmax statistics.
//   route: importance = n * sum_t probs, global budget, stable descending
//       top-k with lowest-index ties; every refinement pass's disjoint set.
//   correct: per query, subtract each selected parent's term and add its
//       children's terms (fp32), pass after pass, then out = a / max(l, eps).
#include "avq_kernels.cuh"
#include "avq_select.cuh"

namespace avq {

constexpr int PA_ROWS = 32;
constexpr int PA_COLS = 32;
constexpr int MAX_PASSES = 8;

struct PassLayout {
  int n;
  int off[MAX_PASSES];
  int cap[MAX_PASSES];
};

__device__ __forceinline__ float nanmax(float a, float b) {
  if (isnan(a) || isnan(b)) return NAN;
  return a > b ? a : b;
}
// torch clamp_min: NaN stays NaN.
__device__ __forceinline__ float clamp_min_nan(float x, float lo) { return isnan(x) ? x : (x < lo ? lo : x); }

// ---------------------------------------------------------------------------
// Parent attention
// ---------------------------------------------------------------------------
template <int DT, int DMAX>
__global__ void __launch_bounds__(256) parent_attn_kernel(
    const typename Storage<DT>::T* __restrict__ q, Strides3 qs, int H, int T, int D, int M0, float sqrtD,
    const typename Storage<DT>::T* __restrict__ parents, const typename Storage<DT>::T* __restrict__ pagg,
    const int* __restrict__ pcnt, int mode, float* __restrict__ sbuf, float* __restrict__ m_io,
    float* __restrict__ l_out, float* __restrict__ z_io, float* __restrict__ a_out, double* __restrict__ imp_part,
    const int* __restrict__ sel0, int sel_stride, const int* __restrict__ pass_cnt, int hvaq, float beta0,
    float alpha, float* __restrict__ beta_out, int sG, const unsigned int* __restrict__ present) {
  constexpr int NK = DMAX / 8;
  extern __shared__ float smem[];
  const int ld = D + 1;
  float* qq = smem;                      // [PA_ROWS][ld]
  float* pp = qq + PA_ROWS * ld;         // [PA_COLS][ld]
  float* ee = pp + PA_COLS * ld;         // [PA_ROWS][PA_COLS + 1]
  float* nn = ee + PA_ROWS * (PA_COLS + 1);  // [PA_COLS]
  const int g = blockIdx.y, b = g / H, h = g % H, qt = blockIdx.x, gs = g % sG;
  const int tid = threadIdx.x, r = tid >> 3, l8 = tid & 7;
  const int t = qt * PA_ROWS + r;
  const bool live = t < T;
  const long srow = ((long)g * T + (live ? t : 0)) * M0;
  const long ph = (long)h * M0;
  float rowmax = -INFINITY;

  if (mode == 0) {
    const long qbase = (long)b * qs.b + (long)h * qs.h;
    for (int e = tid; e < PA_ROWS * D; e += blockDim.x) {
      const int rr = e / D, d = e % D, tt = qt * PA_ROWS + rr;
      qq[rr * ld + d] = tt < T ? to_f(q[qbase + (long)tt * qs.s + d]) : 0.f;
    }
    for (int p0 = 0; p0 < M0; p0 += PA_COLS) {
      for (int e = tid; e < PA_COLS * D; e += blockDim.x) {
        const int j = e / D, d = e % D;
        pp[j * ld + d] = p0 + j < M0 ? to_f(parents[(ph + p0 + j) * D + d]) : 0.f;
      }
      __syncthreads();
      double acc[PA_COLS / 8];
#pragma unroll
      for (int i = 0; i < PA_COLS / 8; ++i) acc[i] = 0.0;
      for (int d = 0; d < D; ++d) {
        const double qv = (double)qq[r * ld + d];
#pragma unroll
        for (int i = 0; i < PA_COLS / 8; ++i) acc[i] = fma(qv, (double)pp[(l8 + 8 * i) * ld + d], acc[i]);
      }
#pragma unroll
      for (int i = 0; i < PA_COLS / 8; ++i) {
        const int p = p0 + l8 + 8 * i;
        if (p < M0) {
          // pipeline.py:81 (matmul, / sqrt(D)) and :107 (invalid -> -inf)
          // pipeline.py:106 (user / causal mask) and :107 (empty parent)
          const bool vis = !live || present_bit(present, (M0 + 31) >> 5, (long)g * T + t, p);
          float s = pcnt[(long)gs * M0 + p] > 0 && vis ? rnd<DT>(__fdiv_rn(rnd64<DT>(acc[i]), sqrtD)) : -INFINITY;
          if (live) sbuf[srow + p] = s;
          rowmax = nanmax(rowmax, s);
        }
      }
      __syncthreads();
    }
  } else {
    // HVAQ (pipeline.py:192-258, hopfield.py:55-144) on the stored logits.
    const float safe0 = live ? m_io[(long)g * T + t] : 0.f;
    const float zc0 = clamp_min_nan(live ? z_io[(long)g * T + t] : 1.f, eps_dt<DT>());
    const int nsel = pass_cnt[0];
    const int* sl = sel0 + (long)g * sel_stride;
    double gs = 0.0;
    for (int j = l8; j < nsel; j += 8) {
      float e = exp_rn<DT>(rnd<DT>(__fsub_rn(live ? sbuf[srow + sl[j]] : 0.f, safe0)));
      if (isnan(e)) e = 0.f;
      gs += (double)rnd<DT>(__fdiv_rn(e, zc0));
    }
    for (int o = 1; o < 8; o <<= 1) gs += __shfl_xor_sync(0xffffffffu, gs, o);
    const float gsc = clamp_min_nan(rnd64<DT>(gs), eps_dt<DT>());
    double ent = 0.0;
    for (int j = l8; j < nsel; j += 8) {
      float e = exp_rn<DT>(rnd<DT>(__fsub_rn(live ? sbuf[srow + sl[j]] : 0.f, safe0)));
      if (isnan(e)) e = 0.f;
      const float pi = rnd<DT>(__fdiv_rn(e, zc0));
      const float top = rnd<DT>(__fdiv_rn(pi, gsc));
      const float lp = top > 0.f ? log_rn<DT>(top) : 0.f;
      ent += (double)rnd<DT>(__fmul_rn(top, lp));
    }
    for (int o = 1; o < 8; o <<= 1) ent += __shfl_xor_sync(0xffffffffu, ent, o);
    const float hq = -rnd64<DT>(ent);
    float sched;
    if (hvaq == 1) {
      sched = rnd<DT>(__fadd_rn(1.f, rnd<DT>(__fdiv_rn(1.f, rnd<DT>(__fadd_rn(1.f, hq))))));
    } else {
      sched = rnd<DT>(__fadd_rn(1.f, rnd<DT>(__fmul_rn(alpha, hq))));
    }
    const float beta = rnd<DT>(__fmul_rn(beta0, sched));
    if (live && l8 == 0) beta_out[(long)g * T + t] = beta;
    __syncwarp();
    for (int p = l8; p < M0; p += 8) {
      float s = live ? sbuf[srow + p] : -INFINITY;
      s = rnd<DT>(__fmul_rn(beta, rnd<DT>(__fmul_rn(s, sqrtD))));
      if (live) sbuf[srow + p] = s;
      rowmax = nanmax(rowmax, s);
    }
  }
  for (int o = 1; o < 8; o <<= 1) rowmax = nanmax(rowmax, __shfl_xor_sync(0xffffffffu, rowmax, o));
  const float safe = (rowmax == -INFINITY) ? 0.f : rowmax;  // pipeline.py:137-141
  __syncthreads();

  // Phase 2: e, l, z and a = e @ V.
  double lacc = 0.0, zacc = 0.0;
  double aacc[NK];
#pragma unroll
  for (int k = 0; k < NK; ++k) aacc[k] = 0.0;
  for (int p0 = 0; p0 < M0; p0 += PA_COLS) {
    for (int e = tid; e < PA_COLS * D; e += blockDim.x) {
      const int j = e / D, d = e % D;
      pp[j * ld + d] = p0 + j < M0 ? to_f(pagg[((long)gs * M0 + p0 + j) * D + d]) : 0.f;
    }
    if (tid < PA_COLS) nn[tid] = p0 + tid < M0 ? count_dt<DT>(pcnt[(long)gs * M0 + p0 + tid]) : 0.f;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < PA_COLS / 8; ++i) {
      const int j = l8 + 8 * i, p = p0 + j;
      float e = 0.f;
      if (p < M0 && live) {
        e = exp_rn<DT>(rnd<DT>(__fsub_rn(sbuf[srow + p], safe)));
        if (isnan(e)) e = 0.f;  // pipeline.py:143-145
        lacc += (double)rnd<DT>(__fmul_rn(e, nn[j]));
        zacc += (double)e;
      }
      ee[r * (PA_COLS + 1) + j] = e;
    }
    __syncthreads();
    for (int j = 0; j < PA_COLS; ++j) {
      const double e = (double)ee[r * (PA_COLS + 1) + j];
#pragma unroll
      for (int k = 0; k < NK; ++k) {
        const int d = l8 + 8 * k;
        if (d < D) aacc[k] = fma(e, (double)pp[j * ld + d], aacc[k]);
      }
    }
    __syncthreads();
  }
  for (int o = 1; o < 8; o <<= 1) {
    lacc += __shfl_xor_sync(0xffffffffu, lacc, o);
    zacc += __shfl_xor_sync(0xffffffffu, zacc, o);
  }
  const float zd = rnd64<DT>(zacc);
  if (live) {
    if (l8 == 0) {
      m_io[(long)g * T + t] = safe;
      l_out[(long)g * T + t] = rnd64<DT>(lacc);
      z_io[(long)g * T + t] = zd;
    }
#pragma unroll
    for (int k = 0; k < NK; ++k) {
      const int d = l8 + 8 * k;
      if (d < D) a_out[((long)g * T + t) * D + d] = rnd64<DT>(aacc[k]);
    }
  }

  // Phase 3: probs (pipeline.py:150) and the importance partial sums over
  // this CTA's queries (routing.py:62).
  const float zc = clamp_min_nan(zd, eps_dt<DT>());
  const int nqt = gridDim.x;
  for (int p0 = 0; p0 < M0; p0 += PA_COLS) {
#pragma unroll
    for (int i = 0; i < PA_COLS / 8; ++i) {
      const int j = l8 + 8 * i, p = p0 + j;
      float pr = 0.f;
      if (p < M0 && live) {
        float e = exp_rn<DT>(rnd<DT>(__fsub_rn(sbuf[srow + p], safe)));
        if (isnan(e)) e = 0.f;
        pr = rnd<DT>(__fdiv_rn(e, zc));
      }
      ee[r * (PA_COLS + 1) + j] = pr;
    }
    __syncthreads();
    if (tid < PA_COLS && p0 + tid < M0) {
      double s = 0.0;
      for (int rr = 0; rr < PA_ROWS; ++rr) s += (double)ee[rr * (PA_COLS + 1) + tid];
      imp_part[((long)g * nqt + qt) * M0 + p0 + tid] = s;
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Routing
// ---------------------------------------------------------------------------
__device__ void pass_counts(int budget0, int passes, float decay, int M0, int* cnt) {
  int used = 0;
  for (int k = 0; k < passes; ++k) {
    int cur;
    if (k == 0) {
      cur = budget0;
    } else {
      // multipass.py:67 max(1, round(base * decay**i)) with round-half-even
      const double pb = rint((double)budget0 * pow((double)decay, (double)k));
      cur = max(1, (int)pb);
      const int remaining = M0 - used;  // multipass.py:216 (uniform over (b,h))
      cur = min(cur, remaining);
      if (cur <= 0) cur = 0;
    }
    if (k > 0 && cnt[k - 1] == 0) cur = 0;  // a pass that broke ends the loop
    cnt[k] = cur;
    used += cur;
  }
}

// One CTA per (b,h).  phase 0: pre-HVAQ importance, pass 0 (and, without
// HVAQ, every later pass).  phase 1: post-HVAQ importance, passes >= 1.
// descending, NaN first (torch.sort), ties by ascending index
__device__ __forceinline__ unsigned long long route_key(float w, int p) {
  return ((unsigned long long)(~float_order_key(w)) << 32) | (unsigned)p;
}

// route_kernel's shared memory: keys [npow2] u64, ambiguous columns [M0]
// int32, refined flags [M0] bytes, then (16-byte aligned) the selection
// scratch and the selected keys [SEL_MAX] u64.
__host__ __device__ inline size_t route_sel_offset(int M0) {
  int npow2 = 1;
  while (npow2 < M0) npow2 <<= 1;
  return ((size_t)npow2 * 8 + (size_t)M0 * 4 + (size_t)M0 + 15) & ~(size_t)15;
}
__host__ __device__ inline size_t route_smem(int M0) {
  return route_sel_offset(M0) + (size_t)select_scratch_words(M0, SEL_MAX) * 4 + (size_t)SEL_MAX * 8;
}

template <int DT>
__global__ void __launch_bounds__(1024) route_kernel(const double* __restrict__ imp_part, int nqt,
                                                     const int* __restrict__ pcnt, int M0,
                                                     const int* __restrict__ min_valid, int P, int passes,
                                                     float decay, int phase, int all_passes, PassLayout lay,
                                                     int* __restrict__ sel, int sel_stride,
                                                     int* __restrict__ pass_cnt_out,
                                                     float* __restrict__ importance_out, RouteExact rx,
                                                     int sG) {
  extern __shared__ unsigned long long keys[];  // [npow2]
  __shared__ int cnt[MAX_PASSES];
  __shared__ int namb;
  constexpr int AMB_BATCH = 8;  // ambiguous columns recounted per sweep over the rows
  __shared__ double red[AMB_BATCH][32];
  const int g = blockIdx.x, gs = g % sG;
  int npow2 = 1;
  while (npow2 < M0) npow2 <<= 1;
  int* amb = (int*)(keys + npow2);                     // [M0] ambiguous columns
  unsigned char* refined = (unsigned char*)(amb + M0);  // [M0]
  if (threadIdx.x == 0) {
    const int budget0 = min(P, *min_valid);  // pipeline.py:340-343
    pass_counts(budget0, passes, decay, M0, cnt);
    if (g == 0 && pass_cnt_out)
      for (int k = 0; k < passes; ++k) pass_cnt_out[k] = cnt[k];
    namb = 0;
  }
  __syncthreads();
  // importance = n * dtype(sum_t probs) (routing.py:61-63)
  // fp32 tile partials: their sum is within 2^-18 relative of the exact one;
  // where that window straddles a rounding point the column is recomputed
  // exactly below, so the fp64 order of the partials does not matter
  auto tile_sum = [&](int p, int i0, int i1) -> double {  // 16 independent loads at a time
    const float* cp = rx.colpart + (long)g * nqt * M0 + p;
    double acc = 0.0;
    for (int b0 = i0; b0 < i1; b0 += 16) {
      float x[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) x[k] = b0 + k < i1 ? cp[(long)(b0 + k) * M0] : 0.f;
#pragma unroll
      for (int k = 0; k < 16; ++k) acc += (double)x[k];
    }
    return acc;
  };
  auto from_partials = [&](int p, double s) {
    const float n = count_dt<DT>(pcnt[(long)gs * M0 + p]);
    const double eps = fabs(s) * 3.814697265625e-06;
    const float w = rnd<DT>(__fmul_rn(n, rnd64<DT>(s)));
    const float w_lo = rnd<DT>(__fmul_rn(n, rnd64<DT>(s - eps)));
    const float w_hi = rnd<DT>(__fmul_rn(n, rnd64<DT>(s + eps)));
    if (w_lo != w_hi) amb[atomicAdd(&namb, 1)] = p;
    if (importance_out) importance_out[(long)g * M0 + p] = w;
    keys[p] = route_key(w, p);
    refined[p] = 0;
  };
  if (rx.colpart && 2 * M0 <= (int)blockDim.x) {
    // two threads per parent: thread p sums the first half of the tiles,
    // thread M0 + p the second, which passes through the parent's key slot
    const int half = threadIdx.x / M0, p = threadIdx.x % M0, hq = (nqt + 1) / 2;
    double part = 0.0;
    if (half < 2) part = tile_sum(p, half ? hq : 0, half ? nqt : hq);
    if (half == 1) keys[p] = (unsigned long long)__double_as_longlong(part);
    __syncthreads();
    if (half == 0) from_partials(p, part + __longlong_as_double((long long)keys[p]));
    for (int q = M0 + threadIdx.x; q < npow2; q += blockDim.x) keys[q] = ~0ull;
  } else {
  for (int p = threadIdx.x; p < npow2; p += blockDim.x) {
    if (p < M0) {
      const float n = count_dt<DT>(pcnt[(long)gs * M0 + p]);
      float w;
      if (rx.colpart) {
        from_partials(p, tile_sum(p, 0, nqt));
        continue;
      } else {
        double s = 0.0;
        for (int i = 0; i < nqt; ++i) s += imp_part[((long)g * nqt + i) * M0 + p];
        w = rnd<DT>(__fmul_rn(n, rnd64<DT>(s)));
      }
      if (importance_out) importance_out[(long)g * M0 + p] = w;
      keys[p] = route_key(w, p);
      refined[p] = 0;
    } else {
      keys[p] = ~0ull;
    }
  }
  }
  __syncthreads();
  // exact column sums for the ambiguous entries, from the stored tiles: up to
  // eight columns per sweep over the rows, so a row's row statistics are read
  // once per sweep and its columns come from the same cached lines
  const int LDL = exp_slice_pitch(M0);
  using T = typename Storage<DT>::T;
  const T* scr = (const T*)rx.scratch;
  const int nwarps = (int)(blockDim.x >> 5);
  for (int a0 = 0; a0 < namb; a0 += AMB_BATCH) {
    const int na = min(AMB_BATCH, namb - a0);
    int cols[AMB_BATCH];
    double s[AMB_BATCH];
#pragma unroll
    for (int k = 0; k < AMB_BATCH; ++k) {
      cols[k] = k < na ? amb[a0 + k] : 0;
      s[k] = 0.0;
    }
    for (int t = threadIdx.x; t < rx.T; t += blockDim.x) {
      const long row = (long)g * rx.T + t;
      const T* srow = scr + (((long)g * nqt + (t >> 6)) * 64 + (t & 63)) * LDL;
      const float m = rx.m[row];
      const float zc = rx.z[row] < eps_dt<DT>() ? eps_dt<DT>() : rx.z[row];
      const float rz = 1.f / zc;
#pragma unroll
      for (int k = 0; k < AMB_BATCH; ++k) {
        if (k < na) {
          const float x = to_f(srow[cols[k]]);
          const float e = rx.scr_logits ? fmaxf(exp_dt_fast<DT>(rnd<DT>(x - m)), 0.f) : x;
          s[k] += (double)div_dt_fast<DT>(e, rz, zc);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < AMB_BATCH; ++k) {
      for (int o = 16; o > 0; o >>= 1) s[k] += __shfl_xor_sync(0xffffffffu, s[k], o);
      if ((threadIdx.x & 31) == 0) red[k][threadIdx.x >> 5] = s[k];
    }
    __syncthreads();
    if ((int)threadIdx.x < na) {
      const int k = threadIdx.x, p = amb[a0 + k];
      double tot = 0.0;
      for (int i = 0; i < nwarps; ++i) tot += red[k][i];
      const float w = rnd<DT>(__fmul_rn(count_dt<DT>(pcnt[(long)gs * M0 + p]), rnd64<DT>(tot)));
      if (importance_out) importance_out[(long)g * M0 + p] = w;
      keys[p] = route_key(w, p);
    }
    __syncthreads();
  }
  // stable descending order (routing.py:152-170).  Pass k takes the next
  // cnt[k] parents of the order not refined before, so the order is needed
  // only as far as the passes' total: a radix select of that many keys when
  // it is small, else a bitonic sort of all of them.
  int need = 0;
  for (int k = 0; k < passes; ++k) need += cnt[k];
  need = min(need, M0);
  const unsigned long long* order = keys;
  int span = M0;
  if (need <= SEL_MAX) {
    uint32_t* scr = reinterpret_cast<uint32_t*>(reinterpret_cast<unsigned char*>(keys) + route_sel_offset(M0));
    unsigned long long* chosen = reinterpret_cast<unsigned long long*>(scr + select_scratch_words(M0, SEL_MAX));
    select_smallest<1024>(keys, M0, need, chosen, scr);
    order = chosen;
    span = need;
  } else {
  for (int k = 2; k <= npow2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < npow2; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned long long a = keys[i], c = keys[ixj];
          const bool up = (i & k) == 0;
          if ((a > c) == up) {
            keys[i] = c;
            keys[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  }
  int* sg = sel + (long)g * sel_stride;
  if (phase == 0) {
    for (int j = threadIdx.x; j < lay.cap[0]; j += blockDim.x) sg[lay.off[0] + j] = j < cnt[0] ? (int)(order[j] & 0xffffffffu) : -1;
  }
  if (phase == 1 || (phase == 0 && all_passes)) {
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int j = 0; j < cnt[0]; ++j) refined[phase == 0 ? (int)(order[j] & 0xffffffffu) : sg[lay.off[0] + j]] = 1;
      int pos = 0;
      for (int k = 1; k < passes; ++k) {
        int taken = 0;
        while (taken < cnt[k] && pos < span) {
          const int p = (int)(order[pos++] & 0xffffffffu);
          if (!refined[p]) sg[lay.off[k] + taken++] = p;
        }
        for (int j = 0; j < cnt[k]; ++j) refined[sg[lay.off[k] + j]] = 1;
        for (int j = cnt[k]; j < lay.cap[k]; ++j) sg[lay.off[k] + j] = -1;
        pos = 0;  // the next pass re-scans the order, skipping refined parents
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Child correction + output
// ---------------------------------------------------------------------------
constexpr int CJ = 4;  // selected parents staged per chunk

template <int DT, int DMAX, int CMAX>
__global__ void __launch_bounds__(256) correct_kernel(
    const typename Storage<DT>::T* __restrict__ q, Strides3 qs, int H, int T, int D, int M0, int C, float sqrtD,
    const typename Storage<DT>::T* __restrict__ children, const typename Storage<DT>::T* __restrict__ pagg,
    const typename Storage<DT>::T* __restrict__ cagg, const int* __restrict__ pcnt, const int* __restrict__ ccnt,
    const float* __restrict__ sbuf, const float* __restrict__ m_in, const float* __restrict__ z_in,
    const float* __restrict__ l_in, const float* __restrict__ a_in, const int* __restrict__ sel, int sel_stride,
    const int* __restrict__ pass_cnt, PassLayout lay, int multipass, float* __restrict__ out, Strides3 os, int sG) {
  constexpr int NK = DMAX / 8;
  constexpr int NCH = CJ * CMAX;
  extern __shared__ float smem[];
  const int ld = D + 1;
  float* qq = smem;                       // [PA_ROWS][ld]
  float* chv = qq + PA_ROWS * ld;         // [NCH][ld] child codewords
  float* cav = chv + NCH * ld;            // [NCH][D] child sums
  float* pav = cav + NCH * D;             // [CJ][D] parent sums
  float* wp = pav + CJ * D;               // [PA_ROWS][CJ]
  float* wc = wp + PA_ROWS * CJ;          // [PA_ROWS][NCH]
  float* ncc = wc + PA_ROWS * NCH;        // [NCH] child counts (dtype)
  float* cmask = ncc + NCH;               // [NCH] 1 if the logit's child is non-empty
  float* nsel = cmask + NCH;              // [CJ]
  int* psel = (int*)(nsel + CJ);          // [CJ]
  const int g = blockIdx.y, b = g / H, h = g % H, qt = blockIdx.x, gs = g % sG;
  const int tid = threadIdx.x, r = tid >> 3, l8 = tid & 7;
  const int t = qt * PA_ROWS + r;
  const bool live = t < T;
  const long qbase = (long)b * qs.b + (long)h * qs.h;
  for (int e = tid; e < PA_ROWS * D; e += blockDim.x) {
    const int rr = e / D, d = e % D, tt = qt * PA_ROWS + rr;
    qq[rr * ld + d] = tt < T ? to_f(q[qbase + (long)tt * qs.s + d]) : 0.f;
  }
  const long row = (long)g * T + (live ? t : 0);
  const float m = m_in[row];
  const float zc = clamp_min_nan(z_in[row], eps_dt<DT>());
  float l = l_in[row];
  float a[NK];
#pragma unroll
  for (int k = 0; k < NK; ++k) {
    const int d = l8 + 8 * k;
    a[k] = d < D ? a_in[row * D + d] : 0.f;
  }
  const int* sg = sel + (long)g * sel_stride;
  for (int pass = 0; pass < lay.n; ++pass) {
    const int cnt = pass_cnt[pass];
    if (cnt <= 0) break;
    const bool quirk = multipass && cnt == M0;  // refinement.py:256-260
    double rl = 0.0, al = 0.0;
    double ra[NK], aa[NK];
#pragma unroll
    for (int k = 0; k < NK; ++k) ra[k] = aa[k] = 0.0;
    for (int j0 = 0; j0 < cnt; j0 += CJ) {
      __syncthreads();
      for (int e = tid; e < NCH * D; e += blockDim.x) {
        const int jc = e / D, d = e % D, jj = jc / CMAX, c = jc % CMAX, j = j0 + jj;
        float cv = 0.f, ca = 0.f;
        if (j < cnt && c < C) {
          const int p = sg[lay.off[pass] + j];
          const int pl = quirk ? j : p;
          cv = to_f(children[(((long)h * M0 + pl) * C + c) * D + d]);
          ca = to_f(cagg[(((long)gs * M0 + p) * C + c) * D + d]);
        }
        chv[(jj * CMAX + c) * ld + d] = cv;
        cav[(jj * CMAX + c) * D + d] = ca;
      }
      for (int e = tid; e < CJ * D; e += blockDim.x) {
        const int jj = e / D, d = e % D, j = j0 + jj;
        pav[jj * D + d] = j < cnt ? to_f(pagg[((long)gs * M0 + sg[lay.off[pass] + j]) * D + d]) : 0.f;
      }
      if (tid < CJ * CMAX) {
        const int jj = tid / CMAX, c = tid % CMAX, j = j0 + jj;
        float n = 0.f, mk = 0.f;
        if (j < cnt && c < C) {
          const int p = sg[lay.off[pass] + j];
          const int pl = quirk ? j : p;
          n = count_dt<DT>(ccnt[((long)gs * M0 + p) * C + c]);
          mk = ccnt[((long)gs * M0 + pl) * C + c] > 0 ? 1.f : 0.f;
        }
        ncc[tid] = n;
        cmask[tid] = mk;
      }
      if (tid < CJ) {
        const int j = j0 + tid;
        const int p = j < cnt ? sg[lay.off[pass] + j] : -1;
        psel[tid] = p;
        nsel[tid] = p >= 0 ? count_dt<DT>(pcnt[(long)gs * M0 + p]) : 0.f;
      }
      __syncthreads();
      // weights: parent terms exp(pi - m) * n (refinement.py:335), child
      // terms exp(u - m) * n_c (refinement.py:341-343)
      for (int it = l8; it < CJ * (1 + CMAX); it += 8) {
        if (it < CJ) {
          const int jj = it, p = psel[jj];
          float w = 0.f;
          if (p >= 0 && live) {
            float e = exp_rn<DT>(rnd<DT>(__fsub_rn(sbuf[row * M0 + p], m)));
            if (isnan(e)) e = 0.f;
            const float pi = rnd<DT>(__fdiv_rn(e, zc));
            w = __fmul_rn(exp_rn<DT_F32>(__fsub_rn(pi, m)), nsel[jj]);
          }
          wp[r * CJ + jj] = w;
        } else {
          const int jc = it - CJ, jj = jc / CMAX, c = jc % CMAX;
          float w = 0.f;
          if (psel[jj] >= 0 && c < C && live) {
            float u = -INFINITY;
            if (cmask[jc] > 0.f) {
              double acc = 0.0;
              for (int d = 0; d < D; ++d) acc = fma((double)qq[r * ld + d], (double)chv[jc * ld + d], acc);
              u = rnd<DT>(__fdiv_rn(rnd64<DT>(acc), sqrtD));
            }
            w = __fmul_rn(exp_rn<DT_F32>(__fsub_rn(u, m)), ncc[jc]);
          }
          wc[r * NCH + jc] = w;
        }
      }
      __syncthreads();
      for (int jj = 0; jj < CJ; ++jj) {
        const float w = wp[r * CJ + jj];
        rl += (double)w;
#pragma unroll
        for (int k = 0; k < NK; ++k) {
          const int d = l8 + 8 * k;
          if (d < D) ra[k] += (double)__fmul_rn(w, pav[jj * D + d]);
        }
      }
      for (int jc = 0; jc < NCH; ++jc) {
        const float w = wc[r * NCH + jc];
        al += (double)w;
#pragma unroll
        for (int k = 0; k < NK; ++k) {
          const int d = l8 + 8 * k;
          if (d < D) aa[k] += (double)__fmul_rn(w, cav[jc * D + d]);
        }
      }
    }
    // OnlineSoftmaxState.replace with unit scales (attention.py:149-158)
    l = __fadd_rn(__fsub_rn(l, __double2float_rn(rl)), __double2float_rn(al));
#pragma unroll
    for (int k = 0; k < NK; ++k) a[k] = __fadd_rn(__fsub_rn(a[k], __double2float_rn(ra[k])), __double2float_rn(aa[k]));
  }
  if (live) {
    const float den = clamp_min_nan(l, 1e-12f);  // attention_module.py:532-535
    const long obase = (long)b * os.b + (long)t * os.s + (long)h * os.h;
#pragma unroll
    for (int k = 0; k < NK; ++k) {
      const int d = l8 + 8 * k;
      if (d < D) out[obase + d] = __fdiv_rn(a[k], den);
    }
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
void pass_budget_caps(int P, int passes, float decay, int* caps) {
  int used = 0;
  for (int k = 0; k < passes; ++k) {
    int cur = k == 0 ? P : std::max(1, (int)std::nearbyint((double)P * std::pow((double)decay, (double)k)));
    caps[k] = cur;
    used += cur;
  }
  (void)used;
}

int selection_stride(int P, int passes, float decay) {
  int caps[MAX_PASSES];
  pass_budget_caps(P, passes, decay, caps);
  int s = 0;
  for (int k = 0; k < passes; ++k) s += caps[k];
  return s;
}

struct FwdWorkspace {
  float *sbuf, *m, *l, *z, *a, *beta, *imp;
  double *part0, *part1;
  int *sel, *pass_cnt;
  void* slog;  // tensor-core path: logits scratch when not in shared memory (or kept for HVAQ)
  void* exptab;  // tcgen05 path: the bf16 exponential table
  void* cdesc;   // tcgen05 correction: slot descriptors
  void* dlog;    // decode path: the [G, M0] dtype logits of the step's queries
  size_t bytes;
};

bool forward_uses_mma(int dtype, int D, int M0, int C) {
  return parent_attn_mma_ok(dtype, D, M0) && (C == 4 || C == 8);
}

// Layout of the caller's workspace.  The exact path keeps fp32 logits
// [G,T,M0]; the tensor-core path keeps dtype logits only when they do not fit
// in shared memory or must survive for the HVAQ pass.
static FwdWorkspace carve(void* base, int dtype, int G, int T, int D, int M0, int C, int P, int passes,
                          int sel_stride, int hvaq) {
  if (decode_forward_ok(dtype, T, D, M0, C, P, passes, hvaq)) {
    // one query per (b,h): logits, the exponential table, the selection
    char* p = (char*)base;
    FwdWorkspace w{};
    auto take = [&](size_t n) {
      char* r = p;
      p += align_up(n);
      return (void*)r;
    };
    w.dlog = take(decode_work_bytes(G, M0, P));
    w.exptab = take(parent_attn_tc_table_bytes());
    w.sel = (int*)take(sizeof(int) * (long)G * sel_stride);
    w.pass_cnt = (int*)take(sizeof(int) * MAX_PASSES);
    w.bytes = (size_t)(p - (char*)base);
    return w;
  }
  const bool mma = forward_uses_mma(dtype, D, M0, C);
  const int rows = mma ? PM_ROWS_PUBLIC : PA_ROWS;
  const int nqt = (T + rows - 1) / rows;
  const long GT = (long)G * (T > 0 ? T : 1);
  const int dtb = dtype == DT_F32 ? 4 : 2;
  char* p = (char*)base;
  FwdWorkspace w;
  auto take = [&](size_t n) {
    char* r = p;
    p += align_up(n);
    return (void*)r;
  };
  w.sbuf = mma ? nullptr : (float*)take(sizeof(float) * GT * M0);
  w.slog = (mma && (hvaq || !parent_attn_mma_smem_mode(D, M0))) ? take(parent_attn_mma_scratch(G, T, M0, dtb)) : nullptr;
  w.m = (float*)take(sizeof(float) * GT);
  w.l = (float*)take(sizeof(float) * GT);
  w.z = (float*)take(sizeof(float) * GT);
  w.beta = (float*)take(sizeof(float) * GT);
  w.a = (float*)take((size_t)(mma ? dtb : 4) * GT * D);
  w.imp = (float*)take(sizeof(float) * (long)G * M0);
  w.part0 = (double*)take(sizeof(double) * (long)G * (nqt > 0 ? nqt : 1) * M0);
  w.part1 = hvaq ? (double*)take(sizeof(double) * (long)G * (nqt > 0 ? nqt : 1) * M0) : nullptr;
  w.sel = (int*)take(sizeof(int) * (long)G * sel_stride);
  w.pass_cnt = (int*)take(sizeof(int) * MAX_PASSES);
  w.exptab = mma ? take(parent_attn_tc_table_bytes()) : nullptr;
  w.cdesc = (mma && (C == 4 || C == 8)) ? take(correct_tc_desc_bytes(G, sel_stride, C)) : nullptr;
  w.dlog = nullptr;
  w.bytes = (size_t)(p - (char*)base);
  return w;
}

size_t forward_workspace_bytes(int dtype, int G, int T, int D, int M0, int C, int P, int passes, float decay,
                               int hvaq) {
  return carve(nullptr, dtype, G, T, D, M0, C, P, passes, selection_stride(P, passes, decay), hvaq).bytes;
}

// Groups of the quantized state (see ForwardArgs::state_groups).
static int state_groups(const ForwardArgs& a) { return a.state_groups > 0 ? a.state_groups : a.B * a.H; }

template <int DT, int DMAX, int CMAX>
static void launch_correct(const ForwardArgs& a, const FwdWorkspace& w, float sqrtD, int sel_stride,
                           const PassLayout& lay, cudaStream_t st) {
  using T = typename Storage<DT>::T;
  const int G = a.B * a.H;
  const int nqt = (a.T + PA_ROWS - 1) / PA_ROWS;
  constexpr int NCH = CJ * CMAX;
  const size_t smem = sizeof(float) * ((size_t)PA_ROWS * (a.D + 1) + (size_t)NCH * (a.D + 1) + (size_t)NCH * a.D +
                                       (size_t)CJ * a.D + PA_ROWS * CJ + PA_ROWS * NCH + 2 * NCH + CJ) +
                      sizeof(int) * CJ;
  AVQ_TIMED("correct_exact", st);
  auto k = correct_kernel<DT, DMAX, CMAX>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  k<<<dim3(nqt, G), 256, smem, st>>>((const T*)a.q, a.qs, a.H, a.T, a.D, a.M0, a.C, sqrtD, (const T*)a.children_dt,
                                     (const T*)a.pagg, (const T*)a.cagg, a.pcnt, a.ccnt, w.sbuf, w.m, w.z, w.l, w.a,
                                     a.selected_out ? a.selected_out : w.sel, sel_stride,
                                     a.pass_counts_out ? a.pass_counts_out : w.pass_cnt, lay, a.passes > 1 ? 1 : 0,
                                     a.out, a.os, state_groups(a));
}

template <int DT>
int launch_forward(const ForwardArgs& a, cudaStream_t st) {
  using T = typename Storage<DT>::T;
  if (a.D > 256 || a.C > 8 || a.M0 > 8192 || a.passes < 1 || a.passes > MAX_PASSES) return AVQ_ERR_UNSUPPORTED;
  const int G = a.B * a.H;
  if (G == 0 || a.T == 0) return AVQ_OK;
  const int sel_stride = selection_stride(a.P, a.passes, a.pass_decay);
  const bool qaligned = ((uintptr_t)a.q % 16 == 0) && a.qs.s % 8 == 0 && a.qs.h % 8 == 0 && a.qs.b % 8 == 0;
  const bool mma = forward_uses_mma(DT, a.D, a.M0, a.C);
  if (mma && !qaligned) return AVQ_ERR_UNSUPPORTED;
  FwdWorkspace w = carve(a.workspace, DT, G, a.T, a.D, a.M0, a.C, a.P, a.passes, sel_stride, a.hvaq);
  if (a.workspace_bytes < w.bytes) return AVQ_ERR_WORKSPACE;
  if constexpr (DT != DT_F32) {
    if (w.dlog) {  // a decode step: one query per (b,h)
      if (DT == DT_BF16) launch_exp_table(w.exptab, st);
      return launch_decode_forward<DT>(a, w.dlog, w.exptab, a.selected_out, sel_stride, a.pass_counts_out,
                                       a.importance_out, st);
    }
  }
  PassLayout lay;
  lay.n = a.passes;
  pass_budget_caps(a.P, a.passes, a.pass_decay, lay.cap);
  for (int k = 0, off = 0; k < a.passes; ++k) {
    lay.off[k] = off;
    off += lay.cap[k];
  }
  int* sel = a.selected_out ? a.selected_out : w.sel;
  int* pcnt_out = a.pass_counts_out ? a.pass_counts_out : w.pass_cnt;
  const float sqrtD = (float)std::sqrt((double)a.D);
  const size_t rt_smem = route_smem(a.M0);
  auto rk = route_kernel<DT>;
  cudaFuncSetAttribute(rk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rt_smem);
  const int sG = state_groups(a);
  bool waited = false;
  auto route = [&](auto... args) {
    if (!waited && a.min_valid_ready) {  // *min_valid comes from another stream (a cross-rank reduction)
      cudaStreamWaitEvent(st, static_cast<cudaEvent_t>(a.min_valid_ready), 0);
      waited = true;
    }
    AVQ_TIMED("route", st);
    rk<<<G, 1024, rt_smem, st>>>(args..., sG);
  };
  const bool hv = a.hvaq != 0;
  float* imp_out = a.importance_out ? a.importance_out : w.imp;

  if constexpr (DT != DT_F32) {
    if (mma) {
      const int nqt = (a.T + PM_ROWS_PUBLIC - 1) / PM_ROWS_PUBLIC;
      // both parent passes on tcgen05 when they fit (the HVAQ rescaling pass
      // gathers the first budget's parents into one 64-row tile); otherwise
      // both on the mma.sync kernels, whose plain pass then keeps its logits
      // in the scratch slices for the rescaling pass
      const bool tc_ok = parent_attn_tc_ok(DT, a.D, a.M0);
      bool pa_tc = tc_ok && (!hv || parent_attn_tc_hvaq_ok(DT, a.D, a.M0, a.P));
      const bool corr_tc = correct_tc_ok(DT, a.D, a.C);
      PAArgs pa{a.q, a.qs, a.B, a.H, a.T, a.D, a.M0, sqrtD, a.parents_dt, a.pagg, a.pcnt, 0, (hv && !pa_tc) ? 1 : 0,
                w.slog, false, w.m, w.l, w.z, w.a, (float*)w.part0, sel, sel_stride, pcnt_out, a.hvaq, a.beta0,
                a.alpha, w.beta, sG, a.present};
      if (DT == DT_BF16 && (pa_tc || corr_tc)) launch_exp_table(w.exptab, st);
      int rc = AVQ_ERR_UNSUPPORTED;
      if (pa_tc && (rc = launch_parent_attn_tc<DT>(pa, w.exptab, st)) == AVQ_ERR_UNSUPPORTED) {
        pa_tc = false;  // an operand the tensor maps cannot describe: the mma.sync kernels
        pa.keep_logits = hv ? 1 : 0;
      }
      if (!pa_tc) rc = launch_parent_attn_mma<DT>(pa, st);
      if (rc != AVQ_OK) return rc;
      // the routing fallback reads exponentials, or the mma.sync HVAQ path's kept logits
      RouteExact rx0{(const float*)w.part0, w.slog, pa.keep_logits, w.m, w.z, a.T};
      route(w.part0, nqt, a.pcnt, a.M0, a.min_valid, a.P, a.passes, a.pass_decay, 0, (!hv && a.passes > 1) ? 1 : 0,
            lay, sel, sel_stride, pcnt_out, imp_out, rx0);
      if (hv) {
        pa.mode = 1;
        pa.keep_logits = 0;
        pa.colpart = (float*)w.part1;
        rc = pa_tc ? launch_parent_attn_tc<DT>(pa, w.exptab, st) : launch_parent_attn_mma<DT>(pa, st);
        if (rc != AVQ_OK) return rc;
        RouteExact rx1{(const float*)w.part1, w.slog, 0, w.m, w.z, a.T};
        if (a.passes > 1)
          route(w.part1, nqt, a.pcnt, a.M0, a.min_valid, a.P, a.passes, a.pass_decay, 1, 1, lay, sel, sel_stride,
                pcnt_out, w.imp, rx1);
      }
      CorrArgs ca{a.q, a.qs, a.B, a.H, a.T, a.D, a.M0, a.C, sqrtD, a.parents_dt, a.children_dt, a.pagg, a.cagg,
                  a.pcnt, a.ccnt, w.m, w.l, w.z, hv ? w.beta : nullptr, w.a, sel, sel_stride, pcnt_out, a.passes,
                  {0, 0, 0, 0, 0, 0, 0, 0}, a.passes > 1 ? 1 : 0, a.out, a.os, sG, a.present};
      for (int k = 0; k < a.passes; ++k) ca.pass_off[k] = lay.off[k];
      rc = (corr_tc && w.cdesc) ? launch_correct_tc<DT>(ca, w.exptab, w.cdesc, st) : AVQ_ERR_UNSUPPORTED;
      if (rc == AVQ_ERR_UNSUPPORTED) rc = launch_correct_mma<DT>(ca, st);
      if (rc != AVQ_OK) return rc;
      return cudaPeekAtLastError() == cudaSuccess ? AVQ_OK : AVQ_ERR_CUDA;
    }
  }

  const int nqt = (a.T + PA_ROWS - 1) / PA_ROWS;
  const size_t pa_smem = sizeof(float) * ((size_t)(PA_ROWS + PA_COLS) * (a.D + 1) + PA_ROWS * (PA_COLS + 1) + PA_COLS);
#define AVQ_PA(DM, MODE, PART)                                                                                       \
  do {                                                                                                               \
    AVQ_TIMED(MODE ? "parent_attn_hvaq_exact" : "parent_attn_exact", st);                                            \
    auto k = parent_attn_kernel<DT, DM>;                                                                             \
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pa_smem);                              \
    k<<<dim3(nqt, G), 256, pa_smem, st>>>((const T*)a.q, a.qs, a.H, a.T, a.D, a.M0, sqrtD, (const T*)a.parents_dt,   \
                                          (const T*)a.pagg, a.pcnt, MODE, w.sbuf, w.m, w.l, w.z, w.a, PART, sel,     \
                                          sel_stride, pcnt_out, a.hvaq, a.beta0, a.alpha, w.beta, sG, a.present);    \
  } while (0)
#define AVQ_PA_D(MODE, PART)                                   \
  do {                                                         \
    if (a.D <= 64) AVQ_PA(64, MODE, PART);                     \
    else if (a.D <= 128) AVQ_PA(128, MODE, PART);              \
    else AVQ_PA(256, MODE, PART);                              \
  } while (0)
  AVQ_PA_D(0, w.part0);
  const RouteExact rxn{nullptr, nullptr, 0, nullptr, nullptr, a.T};
  route(w.part0, nqt, a.pcnt, a.M0, a.min_valid, a.P, a.passes, a.pass_decay, 0,
                               (!hv && a.passes > 1) ? 1 : 0, lay, sel, sel_stride, pcnt_out, imp_out, rxn);
  if (hv) {
    AVQ_PA_D(1, w.part1);
    if (a.passes > 1)
      route(w.part1, nqt, a.pcnt, a.M0, a.min_valid, a.P, a.passes, a.pass_decay, 1, 1, lay,
                                   sel, sel_stride, pcnt_out, w.imp, rxn);
  }
#undef AVQ_PA_D
#undef AVQ_PA
  if (a.C <= 4) {
    if (a.D <= 64) launch_correct<DT, 64, 4>(a, w, sqrtD, sel_stride, lay, st);
    else if (a.D <= 128) launch_correct<DT, 128, 4>(a, w, sqrtD, sel_stride, lay, st);
    else launch_correct<DT, 256, 4>(a, w, sqrtD, sel_stride, lay, st);
  } else {
    if (a.D <= 64) launch_correct<DT, 64, 8>(a, w, sqrtD, sel_stride, lay, st);
    else if (a.D <= 128) launch_correct<DT, 128, 8>(a, w, sqrtD, sel_stride, lay, st);
    else launch_correct<DT, 256, 8>(a, w, sqrtD, sel_stride, lay, st);
  }
  return cudaPeekAtLastError() == cudaSuccess ? AVQ_OK : AVQ_ERR_CUDA;
}

template int launch_forward<DT_F32>(const ForwardArgs&, cudaStream_t);
template int launch_forward<DT_BF16>(const ForwardArgs&, cudaStream_t);
template int launch_forward<DT_F16>(const ForwardArgs&, cudaStream_t);

}  // namespace avq
