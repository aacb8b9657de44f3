// Decode-step attention: one query per (b,h) (T = 1), bf16 / fp16, D in
// {64, 128}, one routing pass without the HVAQ temperature (reference
// pipeline.py:46-189, routing.py:24-170, refinement.py:82-304,
// attention.py:100-163, attention_module.py:532-535).
//
// A decode step's work is dominated by reading every (b,h)'s parent sums
// V = pagg[g] once ([M0, D] in the dtype), plus the selected parents'
// children sums; the arithmetic is small.  Three kernels:
//
//   decode_logits_kernel  per head, the logits of all B queries against a
//       128-parent chunk: S = Q_h P_h^T on mma.sync tensor cores (fp32
//       accumulators, the same K-order as the prefill kernels), narrowed,
//       scaled by 1/sqrt(D) (pipeline.py:81) and masked where the parent is
//       empty (:107).  The codebook tile is read once per head, not once per
//       (b,h).
//   decode_route_kernel   per (b,h): row max, exponentials, l and z, the
//       probabilities and the importance n * p (with one query, its sum over
//       queries is p itself), the stable top-P over M0 (bitonic sort of
//       packed keys: descending value, NaN first, ascending index).
//   decode_value_kernel   per (b,h): a = e @ V streamed from HBM, then the
//       child correction of the selected parents and out = a' / max(l', 1e-12).
//
// Rounding points are those of the prefill path: DT(exp(DT(s - m))), z and l
// as exactly rounded sums, p = DT(e / max(z, eps)), w = DT(n p); the
// correction weights are fp32 quantities (exp(p - m) n for a parent -- the
// probability used as a logit, refinement.py:233 -- and exp(u - m) n_c for a
// child, u = DT(DT(q.c) / sqrt(D)), -inf for an empty child).
#include <cmath>
#include <cstdlib>
#include <type_traits>

#include "avq_kernels.cuh"
#include "avq_mma.cuh"
#include "avq_select.cuh"

namespace avq {

namespace {

constexpr int DL_ROWS = 64;    // queries (the batch entries of one head) per logits CTA
constexpr int DL_COLS = 128;   // parents per logits CTA
constexpr int DA_THREADS = 256;
constexpr int DA_WARPS = DA_THREADS / 32;
constexpr uint32_t DA_EXP_BASE = 0x3AFF;  // the bf16 exponential table (launch_exp_table)
constexpr int DA_EXP_N = 2051;

// DT(exp(d)) for a bf16 value d <= 0 or NaN (NaN -> 0) from the table of
// DT(correctly rounded fp32 exp(-x)) over the bf16 x in [2^-9, 128].
__device__ __forceinline__ float exp_bf16_lookup(float d, const uint16_t* __restrict__ tab) {
  uint32_t a = (__float_as_uint(d) >> 16) & 0x7FFFu;
  a = a < DA_EXP_BASE ? DA_EXP_BASE : (a > DA_EXP_BASE + DA_EXP_N - 1 ? DA_EXP_BASE + DA_EXP_N - 1 : a);
  return __uint_as_float((uint32_t)__ldg(tab + (a - DA_EXP_BASE)) << 16);
}

template <int DT>
__device__ __forceinline__ float exp_of_diff(float d, const uint16_t* __restrict__ tab) {
  if constexpr (DT == DT_BF16) return exp_bf16_lookup(d, tab);
  else return fmaxf(exp_dt_fast<DT>(d), 0.f);  // NaN -> 0 (pipeline.py:143-145)
}

__device__ __forceinline__ float fmax_nan_f(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Packed routing key: descending value (NaN first, as torch.sort), then
// ascending index.
__device__ __forceinline__ unsigned long long decode_route_key(float w, int p) {
  return ((unsigned long long)(~float_order_key(w)) << 32) | (unsigned)p;
}

template <int DT, int D>
__global__ void __launch_bounds__(256) decode_logits_kernel(const typename Storage<DT>::T* __restrict__ q,
                                                            Strides3 qs, int B, int H, int M0, float sqrtD,
                                                            const typename Storage<DT>::T* __restrict__ parents,
                                                            const int* __restrict__ pcnt, int sG,
                                                            const unsigned int* __restrict__ present,
                                                            typename Storage<DT>::T* __restrict__ logits) {
  using T = typename Storage<DT>::T;
  constexpr int LDS = D + 8, KS = D / 16, CPR = D / 8;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* sq_ = reinterpret_cast<T*>(smem_raw);  // [DL_ROWS][LDS] queries
  T* sp = sq_ + DL_ROWS * LDS;              // [DL_COLS][LDS] parents
  const int h = blockIdx.x, p0 = blockIdx.y * DL_COLS, b0 = blockIdx.z * DL_ROWS;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int i = tid; i < DL_ROWS * CPR; i += 256) {
    const int r = i / CPR, c = i % CPR, b = b0 + r;
    cp_async16(sq_ + r * LDS + c * 8, q + (long)(b < B ? b : 0) * qs.b + (long)h * qs.h + c * 8, b < B);
  }
  for (int i = tid; i < DL_COLS * CPR; i += 256) {
    const int r = i / CPR, c = i % CPR, p = p0 + r;
    cp_async16(sp + r * LDS + c * 8, parents + ((long)h * M0 + (p < M0 ? p : 0)) * D + c * 8, p < M0);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  const int mt = warp & 3, nh = warp >> 2;  // rows 16 mt .. +16, parents 64 nh .. +64
  float acc[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
#pragma unroll
  for (int k = 0; k < KS; ++k) {
    uint32_t af[4];
    ldsm_x4(af[0], af[1], af[2], af[3], sq_ + (mt * 16 + (lane & 15)) * LDS + k * 16 + (lane >> 4) * 8);
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      uint32_t b0f, b1f, b2f, b3f;
      const int qd = lane >> 3;
      ldsm_x4(b0f, b1f, b2f, b3f, sp + (nh * 64 + jj * 16 + (qd >> 1) * 8 + (lane & 7)) * LDS + k * 16 + (qd & 1) * 8);
      mma16816<DT>(acc[2 * jj], af, b0f, b1f);
      mma16816<DT>(acc[2 * jj + 1], af, b2f, b3f);
    }
  }
  const float inv_sqrtD = 1.f / sqrtD;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int r = mt * 16 + (lane >> 2) + (e >= 2 ? 8 : 0), b = b0 + r;
      const int p = p0 + nh * 64 + j * 8 + (lane & 3) * 2 + (e & 1);
      if (b < B && p < M0) {
        const int g = b * H + h;
        const float x = rnd<DT>(acc[j][e]);
        const bool vis = present_bit(present, (M0 + 31) >> 5, g, p);  // one query: row g
        const float s = pcnt[(long)(g % sG) * M0 + p] > 0 && vis ? scale_logit<DT>(x, sqrtD, inv_sqrtD) : -INFINITY;
        logits[(long)g * M0 + p] = from_f<DT>(s);
      }
    }
  }
}

// Shared memory of decode_route_kernel, in bytes.
// keys [npow2] u64, e [M0] fp32, then (16-byte aligned) the selection
// scratch and the selected keys [SEL_MAX] u64.
__host__ __device__ inline size_t decode_route_sel_offset(int M0) {
  int npow2 = 1;
  while (npow2 < M0) npow2 <<= 1;
  return ((size_t)npow2 * 8 + (size_t)M0 * 4 + 15) & ~(size_t)15;
}
__host__ __device__ inline size_t decode_route_smem(int M0) {
  return decode_route_sel_offset(M0) + (size_t)select_scratch_words(M0, SEL_MAX) * 4 + (size_t)SEL_MAX * 8;
}

// Per (b,h): row max, e = DT(exp(DT(s - m))), l, z, p = DT(e / max(z, eps)),
// w = DT(n p) and the stable top-P.  Writes e [G, M0] fp32, the row's
// (m, l, max(z, eps)) and the selection for decode_value_kernel.
template <int DT>
__global__ void __launch_bounds__(DA_THREADS) decode_route_kernel(
    const typename Storage<DT>::T* __restrict__ logits, int M0, const int* __restrict__ pcnt, int sG,
    const int* __restrict__ min_valid, int P, const uint16_t* __restrict__ exptab, float* __restrict__ ework,
    float* __restrict__ rowstat, int* __restrict__ selwork, float* __restrict__ importance_out,
    int* __restrict__ sel_out, int sel_stride, int* __restrict__ pass_cnt_out) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  int npow2 = 1;
  while (npow2 < M0) npow2 <<= 1;
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(smem_raw);  // [npow2]
  float* ev = reinterpret_cast<float*>(keys + npow2);                          // [M0]
  __shared__ float fred[DA_WARPS];
  __shared__ double dred[2][DA_WARPS];
  __shared__ int sbudget;
  const int g = blockIdx.x, gs = g % sG;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const auto* lrow = logits + (long)g * M0;
  const int* cnt_p = pcnt + (long)gs * M0;

  // row max (pipeline.py:137-141)
  float mx = -INFINITY;
  for (int p = tid; p < M0; p += DA_THREADS) {
    const float s = to_f(lrow[p]);
    ev[p] = s;
    mx = fmax_nan_f(mx, s);
  }
  for (int o = 16; o > 0; o >>= 1) mx = fmax_nan_f(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) fred[warp] = mx;
  __syncthreads();
  mx = fred[0];
  for (int w = 1; w < DA_WARPS; ++w) mx = fmax_nan_f(mx, fred[w]);
  const float safe = mx == -INFINITY ? 0.f : mx;

  // e = DT(exp(DT(s - m))), l = sum DT(e n), z = sum e (pipeline.py:142-150)
  double lz = 0.0, zz = 0.0;
  for (int p = tid; p < M0; p += DA_THREADS) {
    const float e = exp_of_diff<DT>(rnd<DT>(__fsub_rn(ev[p], safe)), exptab);
    lz += (double)rnd<DT>(__fmul_rn(e, count_dt<DT>(cnt_p[p])));
    zz += (double)e;
    ev[p] = e;
    ework[(long)g * M0 + p] = e;
  }
  for (int o = 16; o > 0; o >>= 1) {
    lz += __shfl_xor_sync(0xffffffffu, lz, o);
    zz += __shfl_xor_sync(0xffffffffu, zz, o);
  }
  if (lane == 0) {
    dred[0][warp] = lz;
    dred[1][warp] = zz;
  }
  __syncthreads();
  double lt = 0.0, zt = 0.0;
  for (int w = 0; w < DA_WARPS; ++w) {
    lt += dred[0][w];
    zt += dred[1][w];
  }
  const float zc = clamp_min_nan(rnd64<DT>(zt), eps_dt<DT>());

  // importance w = DT(n * p), p = DT(e / max(z, eps)) (routing.py:61-63; one
  // query, so its sum over queries is p itself)
  for (int p = tid; p < npow2; p += DA_THREADS) {
    if (p < M0) {
      const float pr = rnd<DT>(__fdiv_rn(ev[p], zc));
      const float w = rnd<DT>(__fmul_rn(count_dt<DT>(cnt_p[p]), pr));
      if (importance_out) importance_out[(long)g * M0 + p] = w;
      keys[p] = decode_route_key(w, p);
    } else {
      keys[p] = ~0ull;
    }
  }
  if (tid == 0) {
    const int bud = min(P, *min_valid);  // pipeline.py:340-343
    sbudget = bud;
    if (g == 0 && pass_cnt_out) pass_cnt_out[0] = bud;
    float* rs = rowstat + (long)g * 4;
    rs[0] = safe;
    rs[1] = rnd64<DT>(lt);
    rs[2] = zc;
    rs[3] = __int_as_float(bud);
  }
  __syncthreads();
  const int budget = sbudget;
  // stable descending top-k (routing.py:152-170): a radix select of the
  // budget's keys when it is small, else a bitonic sort of all packed keys
  const unsigned long long* order = keys;
  if (budget <= SEL_MAX) {
    uint32_t* scr = reinterpret_cast<uint32_t*>(smem_raw + decode_route_sel_offset(M0));
    unsigned long long* chosen = reinterpret_cast<unsigned long long*>(scr + select_scratch_words(M0, SEL_MAX));
    select_smallest<DA_THREADS>(keys, M0, budget, chosen, scr);
    order = chosen;
  } else {
  for (int k = 2; k <= npow2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < npow2; i += DA_THREADS) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned long long x = keys[i], y = keys[ixj];
          const bool up = (i & k) == 0;
          if ((x > y) == up) {
            keys[i] = y;
            keys[ixj] = x;
          }
        }
      }
      __syncthreads();
    }
  }
  }
  for (int j = tid; j < P; j += DA_THREADS) {
    const int p = j < budget ? (int)(order[j] & 0xffffffffu) : -1;
    selwork[(long)g * P + j] = p;
    if (sel_out) sel_out[(long)g * sel_stride + j] = p;
  }
}

// Loads EPL consecutive 16-bit elements (8 or 4 bytes) of a row as floats.
template <int DT, int EPL>
__device__ __forceinline__ void load_row_part(const typename Storage<DT>::T* p, float (&x)[EPL]) {
  if constexpr (EPL == 4) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    x[0] = half_lo<DT>(u.x);
    x[1] = half_hi<DT>(u.x);
    x[2] = half_lo<DT>(u.y);
    x[3] = half_hi<DT>(u.y);
  } else {
    const uint32_t u = *reinterpret_cast<const uint32_t*>(p);
    x[0] = half_lo<DT>(u);
    x[1] = half_hi<DT>(u);
  }
}

// Per (b,h): a = DT(e @ V) streamed from HBM (pipeline.py:147), then the child
// correction of the selected parents (refinement.py:165-304,
// attention.py:149-158) and out = a' / max(l', 1e-12).  Slot s of the
// correction is j (1 + C) + k: k = 0 the selected parent j (removed with
// weight exp(p - m) n), k > 0 its child k - 1 (added with exp(u - m) n_c).
template <int DT, int D>
__global__ void __launch_bounds__(DA_THREADS, 3) decode_value_kernel(
    const typename Storage<DT>::T* __restrict__ q, Strides3 qs, int H, int M0, int C, float sqrtD,
    const typename Storage<DT>::T* __restrict__ children, const typename Storage<DT>::T* __restrict__ pagg,
    const typename Storage<DT>::T* __restrict__ cagg, const int* __restrict__ pcnt, const int* __restrict__ ccnt,
    int sG, const float* __restrict__ ework, const float* __restrict__ rowstat, const int* __restrict__ selwork,
    int P, float* __restrict__ out, Strides3 os) {
  using T = typename Storage<DT>::T;
  constexpr int EPL = D / 32;  // elements per lane of a D-row
  __shared__ float red0[DA_WARPS][D], red1[DA_WARPS][D];
  __shared__ float sl[DA_WARPS][2];
  const int g = blockIdx.x, b = g / H, h = g % H, gs = g % sG;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float* er = ework + (long)g * M0;
  const float safe = rowstat[(long)g * 4], l0 = rowstat[(long)g * 4 + 1], zc = rowstat[(long)g * 4 + 2];
  const int budget = __float_as_int(rowstat[(long)g * 4 + 3]);

  // ---- a = sum_p e_p V_p: sixteen rows per warp in flight, kept packed ----
  float acc[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) acc[e] = 0.f;
  {
    using Part = typename std::conditional<EPL == 4, uint2, uint32_t>::type;
    constexpr int NWP = EPL / 2;
    const T* vb = pagg + (long)gs * M0 * D + lane * EPL;
    constexpr int U = 16;
    for (int p0 = warp; p0 < M0; p0 += DA_WARPS * U) {
      Part x[U];
      float ew[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int p = p0 + u * DA_WARPS;
        ew[u] = p < M0 ? er[p] : 0.f;
        x[u] = p < M0 ? *reinterpret_cast<const Part*>(vb + (long)p * D) : Part{};
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint32_t* w = reinterpret_cast<const uint32_t*>(&x[u]);
#pragma unroll
        for (int e = 0; e < NWP; ++e) {
          acc[2 * e] = fmaf(ew[u], half_lo<DT>(w[e]), acc[2 * e]);
          acc[2 * e + 1] = fmaf(ew[u], half_hi<DT>(w[e]), acc[2 * e + 1]);
        }
      }
    }
  }
#pragma unroll
  for (int e = 0; e < EPL; ++e) red0[warp][lane * EPL + e] = acc[e];

  // ---- correction ----
  const float inv_sqrtD = 1.f / sqrtD;
  float ql[EPL];
  load_row_part<DT, EPL>(q + (long)b * qs.b + (long)h * qs.h + lane * EPL, ql);
  const int* sg = selwork + (long)g * P;
  float rl = 0.f, al = 0.f, ra[EPL], aa[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) ra[e] = aa[e] = 0.f;
  // a warp per selected parent: its parent-sum row, its C child codeword rows
  // and child-sum rows are all loaded (packed, EPL/2 words per lane) before
  // any is used
  constexpr int NW = EPL / 2, CM = 8;
  for (int j = warp; j < budget; j += DA_WARPS) {
    const int p = sg[j];
    uint32_t pv[NW], cr[CM][NW], cv[CM][NW];
    const long prow = (long)gs * M0 + p;
    const int np = pcnt[prow];
    const int nc = lane < C ? ccnt[prow * C + lane] : 0;
    const T* pr_ = pagg + prow * D + lane * EPL;
    if constexpr (NW == 2) {
      const uint2 u = *reinterpret_cast<const uint2*>(pr_);
      pv[0] = u.x;
      pv[1] = u.y;
    } else {
      pv[0] = *reinterpret_cast<const uint32_t*>(pr_);
    }
#pragma unroll
    for (int c = 0; c < CM; ++c) {
      if (c < C) {
        const T* a_ = children + (((long)h * M0 + p) * C + c) * D + lane * EPL;
        const T* b_ = cagg + (prow * C + c) * D + lane * EPL;
        if constexpr (NW == 2) {
          const uint2 u = *reinterpret_cast<const uint2*>(a_), w = *reinterpret_cast<const uint2*>(b_);
          cr[c][0] = u.x;
          cr[c][1] = u.y;
          cv[c][0] = w.x;
          cv[c][1] = w.y;
        } else {
          cr[c][0] = *reinterpret_cast<const uint32_t*>(a_);
          cv[c][0] = *reinterpret_cast<const uint32_t*>(b_);
        }
      } else {
#pragma unroll
        for (int e = 0; e < NW; ++e) cr[c][e] = cv[c][e] = 0u;
      }
    }
    float dot[CM];
#pragma unroll
    for (int c = 0; c < CM; ++c) {
      dot[c] = 0.f;
#pragma unroll
      for (int e = 0; e < NW; ++e) {
        dot[c] = fmaf(ql[2 * e], half_lo<DT>(cr[c][e]), dot[c]);
        dot[c] = fmaf(ql[2 * e + 1], half_hi<DT>(cr[c][e]), dot[c]);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int c = 0; c < CM; ++c)
        if (c < C) dot[c] += __shfl_xor_sync(0xffffffffu, dot[c], o);
    // the removed parent: exp(p - m) n with p its probability (refinement.py:233,335)
    const float prb = rnd<DT>(__fdiv_rn(er[p], zc));
    const float wp = __fmul_rn(expf(__fsub_rn(prb, safe)), count_dt<DT>(np));
    rl += wp;
#pragma unroll
    for (int e = 0; e < NW; ++e) {
      ra[2 * e] = fmaf(wp, half_lo<DT>(pv[e]), ra[2 * e]);
      ra[2 * e + 1] = fmaf(wp, half_hi<DT>(pv[e]), ra[2 * e + 1]);
    }
    // its children: u = DT(DT(q.c) / sqrt(D)), -inf for an empty child
    // (pipeline.py:184-189), weight exp(u - m) n_c (refinement.py:341-343)
#pragma unroll
    for (int c = 0; c < CM; ++c) {
      if (c < C) {
        const int n = __shfl_sync(0xffffffffu, nc, c);
        const float lg = n > 0 ? scale_logit<DT>(rnd<DT>(dot[c]), sqrtD, inv_sqrtD) : -INFINITY;
        const float w = __fmul_rn(expf(__fsub_rn(lg, safe)), count_dt<DT>(n));
        al += w;
#pragma unroll
        for (int e = 0; e < NW; ++e) {
          aa[2 * e] = fmaf(w, half_lo<DT>(cv[c][e]), aa[2 * e]);
          aa[2 * e + 1] = fmaf(w, half_hi<DT>(cv[c][e]), aa[2 * e + 1]);
        }
      }
    }
  }
  __syncthreads();  // red0 holds the value sums
#pragma unroll
  for (int e = 0; e < EPL; ++e) red1[warp][lane * EPL + e] = ra[e];
  if (lane == 0) {
    sl[warp][0] = rl;
    sl[warp][1] = al;
  }
  __syncthreads();
  float rlt = 0.f, alt = 0.f;
  for (int w = 0; w < DA_WARPS; ++w) {
    rlt += sl[w][0];
    alt += sl[w][1];
  }
  const float l1 = __fadd_rn(__fsub_rn(l0, rlt), alt);  // OnlineSoftmaxState.replace, unit scales
  const float den = clamp_min_nan(l1, 1e-12f);           // attention_module.py:532-535
  // a = DT(e @ V) and the removed parents' sums per column (each column is
  // read and rewritten by one thread); then the children's sums go through red1
  for (int d = tid; d < D; d += DA_THREADS) {
    float s = 0.f, rs = 0.f;
    for (int w = 0; w < DA_WARPS; ++w) {
      s += red0[w][d];
      rs += red1[w][d];
    }
    red0[0][d] = rnd<DT>(s);
    red0[1][d] = rs;
  }
  __syncthreads();
#pragma unroll
  for (int e = 0; e < EPL; ++e) red1[warp][lane * EPL + e] = aa[e];
  __syncthreads();
  for (int d = tid; d < D; d += DA_THREADS) {
    float as = 0.f;
    for (int w = 0; w < DA_WARPS; ++w) as += red1[w][d];
    const float a1 = __fadd_rn(__fsub_rn(red0[0][d], red0[1][d]), as);
    out[(long)b * os.b + (long)h * os.h + d] = __fdiv_rn(a1, den);
  }
}

}  // namespace

// AVQ_DISABLE_DECODE=1 sends decode steps through the prefill kernels (read at
// every call, so one process can compare both).
bool decode_forward_ok(int dt, int T, int D, int M0, int C, int P, int passes, int hvaq) {
  const char* e = std::getenv("AVQ_DISABLE_DECODE");
  if (e && *e && *e != '0') return false;
  return dt != DT_F32 && T == 1 && passes == 1 && hvaq == 0 && (D == 64 || D == 128) && C >= 1 && C <= 8 &&
         M0 <= 4096 && P <= 1024;
}

size_t decode_work_bytes(int G, int M0, int P) {
  return align_up((size_t)G * M0 * 2) + align_up((size_t)G * M0 * 4) + align_up((size_t)G * 16) +
         align_up((size_t)G * P * 4);
}

template <int DT>
int launch_decode_forward(const ForwardArgs& a, void* work, const void* exptab, int* sel, int sel_stride,
                          int* pass_cnt, float* importance, cudaStream_t st) {
  using T = typename Storage<DT>::T;
  const int G = a.B * a.H, D = a.D, sG = a.state_groups > 0 ? a.state_groups : G;
  if (((uintptr_t)a.q % 16) || a.qs.b % 8 || a.qs.h % 8) return AVQ_ERR_UNSUPPORTED;
  // the workspace: logits [G, M0] dtype, e [G, M0] fp32, row statistics [G, 4], selection [G, P]
  char* wp = static_cast<char*>(work);
  T* dlog = reinterpret_cast<T*>(wp);
  wp += align_up((size_t)G * a.M0 * 2);
  float* ework = reinterpret_cast<float*>(wp);
  wp += align_up((size_t)G * a.M0 * 4);
  float* rowstat = reinterpret_cast<float*>(wp);
  wp += align_up((size_t)G * 16);
  int* selwork = reinterpret_cast<int*>(wp);
  const float sqrtD = (float)std::sqrt((double)D);
  const size_t lsm = (size_t)(DL_ROWS + DL_COLS) * (D + 8) * sizeof(T);
  const size_t rsm = decode_route_smem(a.M0);
  auto go = [&](auto lk, auto vk) {
    {
      AVQ_TIMED("decode_logits", st);
      cudaFuncSetAttribute(lk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lsm);
      lk<<<dim3(a.H, (a.M0 + DL_COLS - 1) / DL_COLS, (a.B + DL_ROWS - 1) / DL_ROWS), 256, lsm, st>>>(
          static_cast<const T*>(a.q), a.qs, a.B, a.H, a.M0, sqrtD, static_cast<const T*>(a.parents_dt), a.pcnt, sG,
          a.present, dlog);
    }
    if (a.min_valid_ready) cudaStreamWaitEvent(st, static_cast<cudaEvent_t>(a.min_valid_ready), 0);
    {
      AVQ_TIMED("decode_route", st);
      auto rk = decode_route_kernel<DT>;
      cudaFuncSetAttribute(rk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rsm);
      rk<<<G, DA_THREADS, rsm, st>>>(dlog, a.M0, a.pcnt, sG, a.min_valid, a.P, static_cast<const uint16_t*>(exptab),
                                     ework, rowstat, selwork, importance, sel, sel_stride, pass_cnt);
    }
    AVQ_TIMED("decode_value", st);
    vk<<<G, DA_THREADS, 0, st>>>(static_cast<const T*>(a.q), a.qs, a.H, a.M0, a.C, sqrtD,
                                 static_cast<const T*>(a.children_dt), static_cast<const T*>(a.pagg),
                                 static_cast<const T*>(a.cagg), a.pcnt, a.ccnt, sG, ework, rowstat, selwork, a.P,
                                 a.out, a.os);
  };
  if (D == 64) go(decode_logits_kernel<DT, 64>, decode_value_kernel<DT, 64>);
  else go(decode_logits_kernel<DT, 128>, decode_value_kernel<DT, 128>);
  return cudaPeekAtLastError() == cudaSuccess ? AVQ_OK : AVQ_ERR_CUDA;
}

template int launch_decode_forward<DT_BF16>(const ForwardArgs&, void*, const void*, int*, int, int*, float*,
                                            cudaStream_t);
template int launch_decode_forward<DT_F16>(const ForwardArgs&, void*, const void*, int*, int, int*, float*,
                                           cudaStream_t);

}  // namespace avq
