// Decode-step attention: one query per (b,h) (T = 1), bf16 / fp16, D in
// {64, 128}, one routing pass without the HVAQ temperature (reference
// pipeline.py:46-189, routing.py:24-170, refinement.py:82-304,
// attention.py:100-163, attention_module.py:532-535).
//
// A decode step's work is dominated by reading every (b,h)'s parent sums
// V = pagg[g] once ([M0, D] in the dtype), plus the selected parents'
// children sums; the arithmetic is small.  Two kernels:
//
//   decode_logits_kernel  per head, the logits of all B queries against a
//       128-parent chunk: S = Q_h P_h^T on mma.sync tensor cores (fp32
//       accumulators, the same K-order as the prefill kernels), narrowed,
//       scaled by 1/sqrt(D) (pipeline.py:81) and masked where the parent is
//       empty (:107).  The codebook tile is read once per head, not once per
//       (b,h).
//   decode_attn_kernel    per (b,h): row max, exponentials, l and z, the
//       probabilities and the importance n * p (with one query, its sum over
//       queries is p itself), the stable top-P over M0 (bitonic sort of
//       packed keys: descending value, NaN first, ascending index), a = e @ V
//       streamed from HBM, then the child correction of the selected parents
//       and out = a' / max(l', 1e-12).
//
// Rounding points are those of the prefill path: DT(exp(DT(s - m))), z and l
// as exactly rounded sums, p = DT(e / max(z, eps)), w = DT(n p); the
// correction weights are fp32 quantities (exp(p - m) n for a parent -- the
// probability used as a logit, refinement.py:233 -- and exp(u - m) n_c for a
// child, u = DT(DT(q.c) / sqrt(D)), -inf for an empty child).
#include <cmath>
#include <cstdlib>

#include "avq_kernels.cuh"
#include "avq_mma.cuh"

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
        const float s = pcnt[(long)(g % sG) * M0 + p] > 0 ? scale_logit<DT>(x, sqrtD, inv_sqrtD) : -INFINITY;
        logits[(long)g * M0 + p] = from_f<DT>(s);
      }
    }
  }
}

// Shared memory of decode_attn_kernel, in bytes.
__host__ __device__ inline size_t decode_attn_smem(int D, int M0, int P) {
  int npow2 = 1;
  while (npow2 < M0) npow2 <<= 1;
  return (size_t)npow2 * 8                 // keys
         + (size_t)M0 * 4                  // e
         + (size_t)DA_WARPS * D * 4 * 2    // warp partials (two sets)
         + (size_t)D * 4 * 2               // q, a
         + (size_t)P * 4                   // selection
         + (size_t)DA_WARPS * 2 * 8 + 64;  // scalar partials
}

template <int DT, int D>
__global__ void __launch_bounds__(DA_THREADS, 4) decode_attn_kernel(
    const typename Storage<DT>::T* __restrict__ logits, const typename Storage<DT>::T* __restrict__ q, Strides3 qs,
    int H, int M0, int C, float sqrtD, const typename Storage<DT>::T* __restrict__ children,
    const typename Storage<DT>::T* __restrict__ pagg, const typename Storage<DT>::T* __restrict__ cagg,
    const int* __restrict__ pcnt, const int* __restrict__ ccnt, int sG, const int* __restrict__ min_valid, int P,
    const uint16_t* __restrict__ exptab, float* __restrict__ out, Strides3 os, float* __restrict__ importance_out,
    int* __restrict__ sel_out, int sel_stride, int* __restrict__ pass_cnt_out) {
  using T = typename Storage<DT>::T;
  constexpr int EPL = D / 32;  // elements per lane of a D-row
  extern __shared__ __align__(128) unsigned char smem_raw[];
  int npow2 = 1;
  while (npow2 < M0) npow2 <<= 1;
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(smem_raw);  // [npow2]
  float* ev = reinterpret_cast<float*>(keys + npow2);                          // [M0]
  float* red0 = ev + M0;                                                       // [DA_WARPS][D]
  float* red1 = red0 + DA_WARPS * D;                                           // [DA_WARPS][D]
  float* qv = red1 + DA_WARPS * D;                                             // [D]
  float* av = qv + D;                                                          // [D]
  int* sel = reinterpret_cast<int*>(av + D);                                   // [P]
  double* dred = reinterpret_cast<double*>(((uintptr_t)(sel + P) + 7) & ~(uintptr_t)7);  // [2][DA_WARPS]
  __shared__ float fred[DA_WARPS];
  __shared__ int sbudget;
  const int g = blockIdx.x, b = g / H, h = g % H, gs = g % sG;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const T* lrow = logits + (long)g * M0;
  const int* cnt_p = pcnt + (long)gs * M0;

  // ---- logits, row max (pipeline.py:137-141) ----
  float mx = -INFINITY;
  for (int p = tid; p < M0; p += DA_THREADS) {
    const float s = to_f(lrow[p]);
    ev[p] = s;
    mx = fmax_nan_f(mx, s);
  }
  for (int d = tid; d < D; d += DA_THREADS) qv[d] = to_f(q[(long)b * qs.b + (long)h * qs.h + d]);
  for (int o = 16; o > 0; o >>= 1) mx = fmax_nan_f(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) fred[warp] = mx;
  __syncthreads();
  mx = fred[0];
  for (int w = 1; w < DA_WARPS; ++w) mx = fmax_nan_f(mx, fred[w]);
  const float safe = mx == -INFINITY ? 0.f : mx;

  // ---- e = DT(exp(DT(s - m))), l = sum DT(e n), z = sum e (pipeline.py:142-150) ----
  double lz = 0.0, zz = 0.0;
  for (int p = tid; p < M0; p += DA_THREADS) {
    const float e = exp_of_diff<DT>(rnd<DT>(__fsub_rn(ev[p], safe)), exptab);
    lz += (double)rnd<DT>(__fmul_rn(e, count_dt<DT>(cnt_p[p])));
    zz += (double)e;
    ev[p] = e;
  }
  for (int o = 16; o > 0; o >>= 1) {
    lz += __shfl_xor_sync(0xffffffffu, lz, o);
    zz += __shfl_xor_sync(0xffffffffu, zz, o);
  }
  if (lane == 0) {
    dred[warp] = lz;
    dred[DA_WARPS + warp] = zz;
  }
  __syncthreads();  // also: every e is in ev
  double lt = 0.0, zt = 0.0;
  for (int w = 0; w < DA_WARPS; ++w) {
    lt += dred[w];
    zt += dred[DA_WARPS + w];
  }
  const float l0 = rnd64<DT>(lt), z0 = rnd64<DT>(zt);
  const float zc = clamp_min_nan(z0, eps_dt<DT>());

  // ---- a = DT(e @ V) (pipeline.py:147): every parent row once, fp32 sums ----
  {
    float acc[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[e] = 0.f;
    // each lane holds EPL consecutive elements (EPL/2 packed pairs) of a row;
    // U rows per warp are loaded before they are used
    const T* vb = pagg + (long)gs * M0 * D + lane * EPL;
    constexpr int U = 8, NW = EPL / 2;
    for (int p0 = warp; p0 < M0; p0 += DA_WARPS * U) {
      uint32_t vr[U][NW];
      float ew[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int p = p0 + u * DA_WARPS;
        ew[u] = p < M0 ? ev[p] : 0.f;
        if constexpr (NW == 2) {
          const uint2 x = p < M0 ? __ldcs(reinterpret_cast<const uint2*>(vb + (long)p * D)) : make_uint2(0u, 0u);
          vr[u][0] = x.x;
          vr[u][1] = x.y;
        } else {
          vr[u][0] = p < M0 ? __ldcs(reinterpret_cast<const unsigned int*>(vb + (long)p * D)) : 0u;
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int e = 0; e < NW; ++e) {
          acc[2 * e] = fmaf(ew[u], half_lo<DT>(vr[u][e]), acc[2 * e]);
          acc[2 * e + 1] = fmaf(ew[u], half_hi<DT>(vr[u][e]), acc[2 * e + 1]);
        }
    }
#pragma unroll
    for (int e = 0; e < EPL; ++e) red0[warp * D + lane * EPL + e] = acc[e];
  }

  // ---- importance w = DT(n * p), p = DT(e / max(z, eps)) (routing.py:61-63) ----
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
  }
  __syncthreads();
  for (int d = tid; d < D; d += DA_THREADS) {
    float s = 0.f;
    for (int w = 0; w < DA_WARPS; ++w) s += red0[w * D + d];
    av[d] = rnd<DT>(s);
  }
  // ---- stable descending top-k (routing.py:152-170): bitonic sort ----
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
  const int budget = sbudget;
  for (int j = tid; j < P; j += DA_THREADS) {
    const int p = j < budget ? (int)(keys[j] & 0xffffffffu) : -1;
    if (j < budget) sel[j] = p;
    if (sel_out) sel_out[(long)g * sel_stride + j] = p;
  }
  __syncthreads();

  // ---- correction (refinement.py:165-304, attention.py:149-158) ----
  // slot s = j (1 + C) + k: k = 0 the selected parent j (removed), k > 0 its
  // child k - 1 (added); a warp per slot
  float rl = 0.f, al = 0.f, ra[EPL], aa[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) ra[e] = aa[e] = 0.f;
  const float inv_sqrtD = 1.f / sqrtD;
  const int nslots = budget * (1 + C);
  float ql[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) ql[e] = qv[lane * EPL + e];
  constexpr int SU = 4;  // slots per warp in flight
  for (int s0 = warp; s0 < nslots; s0 += DA_WARPS * SU) {
    float lr[SU][EPL], vr[SU][EPL];  // logit row (a child), value row
    int kind[SU], pp[SU], n[SU];     // kind: -1 none, 0 parent, 1 child
#pragma unroll
    for (int u = 0; u < SU; ++u) {
      const int s = s0 + u * DA_WARPS;
      kind[u] = -1;
      if (s < nslots) {
        const int j = s / (1 + C), k = s % (1 + C), p = sel[j];
        pp[u] = p;
        const T* vrow_p;
        if (k == 0) {
          kind[u] = 0;
          n[u] = cnt_p[p];
          vrow_p = pagg + ((long)gs * M0 + p) * D;
        } else {
          kind[u] = 1;
          const long crow = ((long)h * M0 + p) * C + (k - 1), vrow = ((long)gs * M0 + p) * C + (k - 1);
          n[u] = ccnt[vrow];
          vrow_p = cagg + vrow * D;
          const T* cr = children + crow * D + lane * EPL;
#pragma unroll
          for (int e = 0; e < EPL; ++e) lr[u][e] = to_f(cr[e]);
        }
        const T* vrl = vrow_p + lane * EPL;
#pragma unroll
        for (int e = 0; e < EPL; ++e) vr[u][e] = to_f(vrl[e]);
      }
    }
    float dot[SU];
#pragma unroll
    for (int u = 0; u < SU; ++u) {
      dot[u] = 0.f;
      if (kind[u] == 1) {
#pragma unroll
        for (int e = 0; e < EPL; ++e) dot[u] = fmaf(ql[e], lr[u][e], dot[u]);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int u = 0; u < SU; ++u) dot[u] += __shfl_xor_sync(0xffffffffu, dot[u], o);
#pragma unroll
    for (int u = 0; u < SU; ++u) {
      if (kind[u] == 0) {
        const float pr = rnd<DT>(__fdiv_rn(ev[pp[u]], zc));
        const float w = __fmul_rn(expf(__fsub_rn(pr, safe)), count_dt<DT>(n[u]));  // refinement.py:335
        rl += w;
#pragma unroll
        for (int e = 0; e < EPL; ++e) ra[e] = fmaf(w, vr[u][e], ra[e]);
      } else if (kind[u] == 1) {
        // pipeline.py:184-189: u = DT(DT(q.c) / sqrt(D)), -inf for an empty child
        const float lg = n[u] > 0 ? scale_logit<DT>(rnd<DT>(dot[u]), sqrtD, inv_sqrtD) : -INFINITY;
        const float w = __fmul_rn(expf(__fsub_rn(lg, safe)), count_dt<DT>(n[u]));  // refinement.py:341-343
        al += w;
#pragma unroll
        for (int e = 0; e < EPL; ++e) aa[e] = fmaf(w, vr[u][e], aa[e]);
      }
    }
  }
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    red0[warp * D + lane * EPL + e] = ra[e];
    red1[warp * D + lane * EPL + e] = aa[e];
  }
  if (lane == 0) {
    dred[warp] = (double)rl;
    dred[DA_WARPS + warp] = (double)al;
  }
  __syncthreads();
  float rlt = 0.f, alt = 0.f;
  for (int w = 0; w < DA_WARPS; ++w) {
    rlt += (float)dred[w];
    alt += (float)dred[DA_WARPS + w];
  }
  const float l1 = __fadd_rn(__fsub_rn(l0, rlt), alt);  // OnlineSoftmaxState.replace, unit scales
  const float den = clamp_min_nan(l1, 1e-12f);           // attention_module.py:532-535
  for (int d = tid; d < D; d += DA_THREADS) {
    float rs = 0.f, as = 0.f;
    for (int w = 0; w < DA_WARPS; ++w) {
      rs += red0[w * D + d];
      as += red1[w * D + d];
    }
    const float a1 = __fadd_rn(__fsub_rn(av[d], rs), as);
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

size_t decode_logits_bytes(int G, int M0) { return (size_t)G * M0 * 2; }

template <int DT>
int launch_decode_forward(const ForwardArgs& a, void* dlog, const void* exptab, int* sel, int sel_stride,
                          int* pass_cnt, float* importance, cudaStream_t st) {
  using T = typename Storage<DT>::T;
  const int G = a.B * a.H, D = a.D, sG = a.state_groups > 0 ? a.state_groups : G;
  if (((uintptr_t)a.q % 16) || a.qs.b % 8 || a.qs.h % 8) return AVQ_ERR_UNSUPPORTED;
  const float sqrtD = (float)std::sqrt((double)D);
  const size_t lsm = (size_t)(DL_ROWS + DL_COLS) * (D + 8) * sizeof(T);
  const size_t asm_ = decode_attn_smem(D, a.M0, a.P);
  auto go = [&](auto lk, auto ak) {
    {
      AVQ_TIMED("decode_logits", st);
      cudaFuncSetAttribute(lk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lsm);
      lk<<<dim3(a.H, (a.M0 + DL_COLS - 1) / DL_COLS, (a.B + DL_ROWS - 1) / DL_ROWS), 256, lsm, st>>>(
          static_cast<const T*>(a.q), a.qs, a.B, a.H, a.M0, sqrtD, static_cast<const T*>(a.parents_dt), a.pcnt, sG,
          static_cast<T*>(dlog));
    }
    if (a.min_valid_ready) cudaStreamWaitEvent(st, static_cast<cudaEvent_t>(a.min_valid_ready), 0);
    AVQ_TIMED("decode_attn", st);
    cudaFuncSetAttribute(ak, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)asm_);
    ak<<<G, DA_THREADS, asm_, st>>>(static_cast<const T*>(dlog), static_cast<const T*>(a.q), a.qs, a.H, a.M0, a.C,
                                    sqrtD, static_cast<const T*>(a.children_dt), static_cast<const T*>(a.pagg),
                                    static_cast<const T*>(a.cagg), a.pcnt, a.ccnt, sG, a.min_valid, a.P,
                                    static_cast<const uint16_t*>(exptab), a.out, a.os, importance, sel, sel_stride,
                                    pass_cnt);
  };
  if (D == 64) go(decode_logits_kernel<DT, 64>, decode_attn_kernel<DT, 64>);
  else go(decode_logits_kernel<DT, 128>, decode_attn_kernel<DT, 128>);
  return cudaPeekAtLastError() == cudaSuccess ? AVQ_OK : AVQ_ERR_CUDA;
}

template int launch_decode_forward<DT_BF16>(const ForwardArgs&, void*, const void*, int*, int, int*, float*,
                                            cudaStream_t);
template int launch_decode_forward<DT_F16>(const ForwardArgs&, void*, const void*, int*, int, int*, float*,
                                           cudaStream_t);

}  // namespace avq
