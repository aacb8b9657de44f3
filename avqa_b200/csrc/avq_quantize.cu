// Hierarchical vector quantization of keys (reference quantizer.py:166-278).
//
//   prep_codebook   : cast the fp32 master codebook to the dtype, squared norms
//   assign          : parent distance + first-argmin, then child distance +
//                     first-argmin inside the assigned parent
//   bucket_hist / bucket_scan / bucket_scatter
//                   : stable counting sort of keys by parent (key order kept
//                     inside every bucket) -> per-parent member lists
//   aggregate       : per parent, fp32 sum of member values in key order,
//                     narrowed once (the reference's 2-D index_add_), plus
//                     the child sums and counts in the same pass
//
// Index work is exact.  Dot products here accumulate in double, so every
// distance equals the exactly rounded reference value.
#include <algorithm>

#include "avq_kernels.cuh"
#include "avq_mma.cuh"

namespace avq {

// ---------------------------------------------------------------------------
// Codebook preparation (attention_module.py:344-348 cast + quantizer.py:208,224 norms)
// ---------------------------------------------------------------------------
template <int DT>
__global__ void prep_codebook_kernel(const float* __restrict__ src, typename Storage<DT>::T* __restrict__ dst,
                                     float* __restrict__ sq, long rows, int D) {
  const int lane = threadIdx.x & 31;
  const long row = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  double acc = 0.0;
  for (int d = lane; d < D; d += 32) {
    const float x = rnd<DT>(src[row * D + d]);
    dst[row * D + d] = from_f<DT>(x);
    acc += (double)rnd<DT>(__fmul_rn(x, x));
  }
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) sq[row] = rnd64<DT>(acc);
}

// ---------------------------------------------------------------------------
// Assignment
// ---------------------------------------------------------------------------
struct ArgMin {
  float v;
  int i;
};

// torch.argmin: the first minimum; a NaN wins over every number.
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  if (bi < 0) return true;
  const bool n = isnan(v), bn = isnan(bv);
  if (n || bn) return n && (!bn || i < bi);
  return v < bv || (v == bv && i < bi);
}

__device__ __forceinline__ ArgMin shfl_best(ArgMin a, int width_mask) {
  for (int o = 1; o <= width_mask; o <<= 1) {
    const float v = __shfl_xor_sync(0xffffffffu, a.v, o);
    const int i = __shfl_xor_sync(0xffffffffu, a.i, o);
    if (i >= 0 && better(v, i, a.v, a.i)) a = {v, i};
  }
  return a;
}

constexpr int AS_ROWS = 64;  // keys per CTA
constexpr int AS_COLS = 32;  // parents per smem tile

template <int DT>
__global__ void __launch_bounds__(256) assign_kernel(const typename Storage<DT>::T* __restrict__ keys, Strides3 ks,
                                                     int H, int S, int D, int M0, int C,
                                                     const typename Storage<DT>::T* __restrict__ parents,
                                                     const float* __restrict__ p_sq,
                                                     const typename Storage<DT>::T* __restrict__ children,
                                                     const float* __restrict__ c_sq, int* __restrict__ passign,
                                                     int* __restrict__ cassign) {
  extern __shared__ float smem[];
  const int ld = D + 1;
  float* kk = smem;                      // [AS_ROWS][ld]
  float* pp = kk + AS_ROWS * ld;         // [AS_COLS][ld]
  float* ksq = pp + AS_COLS * ld;        // [AS_ROWS]
  const int g = blockIdx.y, b = g / H, h = g % H;
  const int s0 = blockIdx.x * AS_ROWS;
  const int tid = threadIdx.x, r = tid >> 2, l4 = tid & 3;
  const long kbase = (long)b * ks.b + (long)h * ks.h;

  for (int e = tid; e < AS_ROWS * D; e += blockDim.x) {
    const int rr = e / D, d = e % D;
    const int s = s0 + rr;
    kk[rr * ld + d] = s < S ? to_f(keys[kbase + (long)s * ks.s + d]) : 0.f;
  }
  __syncthreads();
  if (tid < AS_ROWS) {
    double acc = 0.0;
    for (int d = 0; d < D; ++d) {
      const float x = kk[tid * ld + d];
      acc += (double)rnd<DT>(__fmul_rn(x, x));
    }
    ksq[tid] = rnd64<DT>(acc);
  }
  __syncthreads();
  const float my_ksq = ksq[r];
  ArgMin best = {0.f, -1};
  const long pbase = (long)h * M0;
  for (int p0 = 0; p0 < M0; p0 += AS_COLS) {
    for (int e = tid; e < AS_COLS * D; e += blockDim.x) {
      const int j = e / D, d = e % D;
      pp[j * ld + d] = (p0 + j < M0) ? to_f(parents[(pbase + p0 + j) * D + d]) : 0.f;
    }
    __syncthreads();
    double acc[AS_COLS / 4];
#pragma unroll
    for (int i = 0; i < AS_COLS / 4; ++i) acc[i] = 0.0;
    for (int d = 0; d < D; ++d) {
      const double kv = (double)kk[r * ld + d];
#pragma unroll
      for (int i = 0; i < AS_COLS / 4; ++i) acc[i] = fma(kv, (double)pp[(l4 + 4 * i) * ld + d], acc[i]);
    }
#pragma unroll
    for (int i = 0; i < AS_COLS / 4; ++i) {
      const int p = p0 + l4 + 4 * i;
      if (p < M0) {
        const float cross = rnd64<DT>(acc[i]);
        const float two = rnd<DT>(__fmul_rn(2.f, cross));
        const float t1 = rnd<DT>(__fadd_rn(my_ksq, p_sq[pbase + p]));
        const float dd = rnd<DT>(__fsub_rn(t1, two));
        if (better(dd, p, best.v, best.i)) best = {dd, p};
      }
    }
    __syncthreads();
  }
  best = shfl_best(best, 2);
  const int s = s0 + r;
  // Child stage: children of the assigned parent; the cross term is a sum of
  // dtype-rounded elementwise products (quantizer.py:223-226).
  ArgMin cb = {0.f, -1};
  const int p = best.i;
  for (int c = l4; c < C; c += 4) {
    const long crow = ((pbase + p) * C + c);
    double acc = 0.0;
    for (int d = 0; d < D; ++d) acc += (double)rnd<DT>(__fmul_rn(kk[r * ld + d], to_f(children[crow * D + d])));
    const float cross = rnd64<DT>(acc);
    const float two = rnd<DT>(__fmul_rn(2.f, cross));
    const float t1 = rnd<DT>(__fadd_rn(my_ksq, c_sq[crow]));
    const float dd = rnd<DT>(__fsub_rn(t1, two));
    if (better(dd, c, cb.v, cb.i)) cb = {dd, c};
  }
  cb = shfl_best(cb, 2);
  if (l4 == 0 && s < S) {
    passign[(long)g * S + s] = p;
    cassign[(long)g * S + s] = cb.i;
  }
}

// ---------------------------------------------------------------------------
// Tensor-core assignment (bf16 / fp16).  CTA = 128 keys x all parents in
// chunks of 64; warp w owns keys [16w, 16w+16) and every parent, so each
// key's argmin stays inside one warp (quad shuffles).  The cross term k.p is
// an m16n8k16 MMA with fp32 accumulation, narrowed like the reference's
// bf16/fp16 matmul output; norms and the child stage accumulate in double.
// ---------------------------------------------------------------------------
constexpr int AM_ROWS = 128;
constexpr int AM_CH = 64;

template <int DT, int D>
__global__ void __launch_bounds__(256) assign_mma_kernel(const typename Storage<DT>::T* __restrict__ keys, Strides3 ks,
                                                         int H, int S, int M0, int C,
                                                         const typename Storage<DT>::T* __restrict__ parents,
                                                         const float* __restrict__ p_sq,
                                                         const typename Storage<DT>::T* __restrict__ children,
                                                         const float* __restrict__ c_sq, int* __restrict__ passign,
                                                         int* __restrict__ cassign) {
  using T = typename Storage<DT>::T;
  constexpr int LDS = D + 8, KS = D / 16, CPR = D / 8;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* sk = (T*)smem_raw;                        // [AM_ROWS][LDS]
  T* sp = sk + AM_ROWS * LDS;                  // [2][AM_CH][LDS]
  float* sksq = (float*)(sp + 2 * AM_CH * LDS);  // [AM_ROWS]
  float* spsq = sksq + AM_ROWS;                  // [2][AM_CH]
  int* sbest = (int*)(spsq + 2 * AM_CH);         // [AM_ROWS]
  const int g = blockIdx.y, b = g / H, h = g % H, s0 = blockIdx.x * AM_ROWS;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const T* kb = keys + (long)b * ks.b + (long)h * ks.h;
  const T* pb = parents + (long)h * M0 * D;

  for (int i = tid; i < AM_ROWS * CPR; i += blockDim.x) {
    const int r = i / CPR, c = i % CPR, s = s0 + r;
    cp_async16(sk + r * LDS + c * 8, kb + (long)(s < S ? s : 0) * ks.s + c * 8, s < S);
  }
  auto load_chunk = [&](int buf, int p0) {
    for (int i = tid; i < AM_CH * CPR; i += blockDim.x) {
      const int r = i / CPR, c = i % CPR, p = p0 + r;
      cp_async16(sp + (buf * AM_CH + r) * LDS + c * 8, pb + (long)(p < M0 ? p : 0) * D + c * 8, p < M0);
    }
    if (tid < AM_CH) {
      const int p = p0 + tid;
      if (p < M0) {
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(smem_u32(spsq + buf * AM_CH + tid)),
                     "l"(p_sq + (long)h * M0 + p));
      } else {
        spsq[buf * AM_CH + tid] = INFINITY;
      }
    }
  };
  load_chunk(0, 0);
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  if (tid < AM_ROWS) {
    double acc = 0.0;
#pragma unroll 8
    for (int d = 0; d < D; ++d) {
      const float x = to_f(sk[tid * LDS + d]);
      acc += (double)rnd<DT>(__fmul_rn(x, x));
    }
    sksq[tid] = rnd64<DT>(acc);
  }
  uint32_t af[KS][4];
#pragma unroll
  for (int k = 0; k < KS; ++k)
    ldsm_x4(af[k][0], af[k][1], af[k][2], af[k][3], sk + (warp * 16 + (lane & 15)) * LDS + k * 16 + (lane >> 4) * 8);
  __syncthreads();
  const int rA = warp * 16 + (lane >> 2), rB = rA + 8;
  const float ksqA = sksq[rA], ksqB = sksq[rB];
  float bvA = 0.f, bvB = 0.f;
  int biA = -1, biB = -1;
  const int nch = (M0 + AM_CH - 1) / AM_CH;
  for (int ci = 0; ci < nch; ++ci) {
    const int buf = ci & 1, p0 = ci * AM_CH;
    if (ci + 1 < nch) load_chunk(buf ^ 1, p0 + AM_CH);
    cp_async_commit();
    float acc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    const T* spb = sp + buf * AM_CH * LDS;
#pragma unroll
    for (int k = 0; k < KS; ++k) {
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        uint32_t b0, b1, b2, b3;
        const int q = lane >> 3;
        ldsm_x4(b0, b1, b2, b3, spb + (jj * 16 + (q >> 1) * 8 + (lane & 7)) * LDS + k * 16 + (q & 1) * 8);
        mma16816<DT>(acc[2 * jj], af[k], b0, b1);
        mma16816<DT>(acc[2 * jj + 1], af[k], b2, b3);
      }
    }
    const float* psq = spsq + buf * AM_CH;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int cl = j * 8 + (lane & 3) * 2 + e, p = p0 + cl;
        if (p < M0) {
          const float ps = psq[cl];
          {
            const float cross = rnd<DT>(acc[j][e]);
            const float dd = rnd<DT>(__fsub_rn(rnd<DT>(__fadd_rn(ksqA, ps)), rnd<DT>(__fmul_rn(2.f, cross))));
            if (better(dd, p, bvA, biA)) { bvA = dd; biA = p; }
          }
          {
            const float cross = rnd<DT>(acc[j][2 + e]);
            const float dd = rnd<DT>(__fsub_rn(rnd<DT>(__fadd_rn(ksqB, ps)), rnd<DT>(__fmul_rn(2.f, cross))));
            if (better(dd, p, bvB, biB)) { bvB = dd; biB = p; }
          }
        }
      }
    }
    cp_async_wait<0>();
    __syncthreads();
  }
  ArgMin A = shfl_best({bvA, biA}, 2), Bm = shfl_best({bvB, biB}, 2);
  if ((lane & 3) == 0) {
    sbest[rA] = A.i;
    sbest[rB] = Bm.i;
  }
  __syncwarp();
  // child stage: lane -> key warp*16 + lane/2, children lane&1, +2, ...
  const int r = warp * 16 + (lane >> 1), half = lane & 1, s = s0 + r;
  const int p = sbest[r];
  const float ksq = sksq[r];
  ArgMin cb = {0.f, -1};
  for (int c = half; c < C; c += 2) {
    const long crow = ((long)h * M0 + p) * C + c;
    const uint4* cr = reinterpret_cast<const uint4*>(children + crow * D);
    const uint4* kr = reinterpret_cast<const uint4*>(sk + r * LDS);
    double acc = 0.0;
#pragma unroll 4
    for (int v = 0; v < D / 8; ++v) {
      const uint4 cv = __ldg(cr + v), kv = kr[v];
      const T* ce = reinterpret_cast<const T*>(&cv);
      const T* ke = reinterpret_cast<const T*>(&kv);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc += (double)rnd<DT>(__fmul_rn(to_f(ke[e]), to_f(ce[e])));
    }
    const float cross = rnd64<DT>(acc);
    const float dd = rnd<DT>(__fsub_rn(rnd<DT>(__fadd_rn(ksq, c_sq[crow])), rnd<DT>(__fmul_rn(2.f, cross))));
    if (better(dd, c, cb.v, cb.i)) cb = {dd, c};
  }
  {
    const float v = __shfl_xor_sync(0xffffffffu, cb.v, 1);
    const int i = __shfl_xor_sync(0xffffffffu, cb.i, 1);
    if (i >= 0 && better(v, i, cb.v, cb.i)) cb = {v, i};
  }
  if (half == 0 && s < S) {
    passign[(long)(blockIdx.y) * S + s] = p;
    cassign[(long)(blockIdx.y) * S + s] = cb.i;
  }
}

// ---------------------------------------------------------------------------
// Stable counting sort by parent
// ---------------------------------------------------------------------------
// hist[g][seg][p] = number of keys of segment seg assigned to parent p.
__global__ void bucket_hist_kernel(const int* __restrict__ passign, int S, int M0, int nseg, int seg_len,
                                   int* __restrict__ hist) {
  extern __shared__ int sh[];
  const int g = blockIdx.y, seg = blockIdx.x;
  for (int p = threadIdx.x; p < M0; p += blockDim.x) sh[p] = 0;
  __syncthreads();
  const int s_end = min(S, (seg + 1) * seg_len);
  for (int s = seg * seg_len + threadIdx.x; s < s_end; s += blockDim.x) atomicAdd(&sh[passign[(long)g * S + s]], 1);
  __syncthreads();
  int* out = hist + ((long)g * nseg + seg) * M0;
  for (int p = threadIdx.x; p < M0; p += blockDim.x) out[p] = sh[p];
}

// Per g: bucket totals -> exclusive offsets; hist rewritten in place as each
// segment's first slot per bucket.  Writes parent offsets/counts, the number
// of non-empty parents and folds it into the global minimum.  The segment
// counts of a bucket are read in batches of independent loads, and the
// totals are scanned with warp shuffles.
__global__ void __launch_bounds__(1024) bucket_scan_kernel(int* __restrict__ hist, int M0, int nseg,
                                                           int* __restrict__ poff, int* __restrict__ pcnt,
                                                           int* __restrict__ nvalid, int* __restrict__ gmin_valid) {
  extern __shared__ int sh[];  // [M0] bucket totals, then the buckets' first slots
  __shared__ int wsum[32];
  constexpr unsigned full = 0xffffffffu;
  const int g = blockIdx.x, tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5;
  int* base = hist + (long)g * nseg * M0;
  for (int p = tid; p < M0; p += nt) {
    int tot = 0;
    for (int s0 = 0; s0 < nseg; s0 += 8) {
      int c[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) c[k] = s0 + k < nseg ? base[(long)(s0 + k) * M0 + p] : 0;
#pragma unroll
      for (int k = 0; k < 8; ++k) tot += c[k];
    }
    sh[p] = tot;
  }
  __syncthreads();
  // exclusive scan of the totals (M0 <= 8192): a contiguous chunk per thread,
  // an inclusive shuffle scan over the warp, then over the warp sums
  const int per = (M0 + nt - 1) / nt, lo = min(M0, tid * per), hi = min(M0, lo + per);
  int acc = 0, nz = 0;
  for (int p = lo; p < hi; ++p) {
    acc += sh[p];
    nz += sh[p] > 0;
  }
  int incl = acc;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(full, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int v = lane < nt / 32 ? wsum[lane] : 0;
    int iv = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(full, iv, o);
      if (lane >= o) iv += y;
    }
    if (lane < nt / 32) wsum[lane] = iv - v;
  }
  __syncthreads();
  int run = wsum[warp] + incl - acc;
  for (int p = lo; p < hi; ++p) {
    const int c = sh[p];
    poff[(long)g * M0 + p] = run;
    pcnt[(long)g * M0 + p] = c;
    sh[p] = run;
    run += c;
  }
  __syncthreads();
  // each segment's first slot per bucket: the bucket start plus the counts of
  // the segments before it
  for (int p = tid; p < M0; p += nt) {
    int r = sh[p];
    for (int s0 = 0; s0 < nseg; s0 += 8) {
      int c[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) c[k] = s0 + k < nseg ? base[(long)(s0 + k) * M0 + p] : 0;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (s0 + k < nseg) base[(long)(s0 + k) * M0 + p] = r;
        r += c[k];
      }
    }
  }
  // number of valid parents
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) nz += __shfl_xor_sync(full, nz, o);
  __syncthreads();
  if (lane == 0) wsum[warp] = nz;
  __syncthreads();
  if (tid == 0) {
    int tot = 0;
    for (int w = 0; w < nt / 32; ++w) tot += wsum[w];
    nvalid[g] = tot;
    if (gmin_valid) atomicMin(gmin_valid, tot);
  }
}

// One warp per segment walks its keys in order; ranks inside a 32-key group
// come from __match_any_sync, so the order inside every bucket is key order.
__global__ void bucket_scatter_kernel(const int* __restrict__ passign, const int* __restrict__ hist, int S, int M0,
                                      int nseg, int seg_len, int* __restrict__ order) {
  extern __shared__ int run[];  // [M0]
  const int g = blockIdx.y, seg = blockIdx.x, lane = threadIdx.x;
  const int* off = hist + ((long)g * nseg + seg) * M0;
  for (int p = lane; p < M0; p += 32) run[p] = off[p];
  __syncwarp();
  const int s_begin = seg * seg_len, s_end = min(S, s_begin + seg_len);
  for (int s0 = s_begin; s0 < s_end; s0 += 32) {
    const int s = s0 + lane;
    const bool act = s < s_end;
    const int p = act ? passign[(long)g * S + s] : -1 - lane;  // inactive lanes never match
    const unsigned peers = __match_any_sync(0xffffffffu, p);
    const unsigned lower = peers & ((1u << lane) - 1u);
    if (act) {
      const int pos = run[p] + __popc(lower);
      order[(long)g * S + pos] = s;
    }
    __syncwarp();
    if (act && (peers >> lane) == 1u) run[p] += __popc(peers);  // highest lane of the group
    __syncwarp();
  }
}

// One warp per parent: members in key order; lane owns dims lane, lane+32, ...
template <int DT, int CMAX, int DMAX>
__global__ void __launch_bounds__(256) aggregate_kernel(
    const typename Storage<DT>::T* __restrict__ values, Strides3 vs, int H, int S, int D, int M0, int C,
    const int* __restrict__ order, const int* __restrict__ poff, const int* __restrict__ pcnt,
    const int* __restrict__ cassign, typename Storage<DT>::T* __restrict__ pagg,
    typename Storage<DT>::T* __restrict__ cagg, float* __restrict__ pacc, float* __restrict__ cacc,
    int* __restrict__ ccnt, long rows) {
  constexpr int NJ = DMAX / 32;
  const int lane = threadIdx.x & 31;
  const long gp = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gp >= rows) return;
  const int g = (int)(gp / M0);
  const int b = g / H, h = g % H;
  const long vbase = (long)b * vs.b + (long)h * vs.h;
  float ap[NJ];
  float ac[CMAX][NJ];
  int cn[CMAX];
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    ap[j] = 0.f;
#pragma unroll
    for (int c = 0; c < CMAX; ++c) ac[c][j] = 0.f;
  }
#pragma unroll
  for (int c = 0; c < CMAX; ++c) cn[c] = 0;
  const int beg = poff[gp], n = pcnt[gp];
  for (int i = 0; i < n; ++i) {
    const int s = order[(long)g * S + beg + i];
    const int cc = cassign[(long)g * S + s];
#pragma unroll
    for (int c = 0; c < CMAX; ++c) cn[c] += (c == cc);
    const typename Storage<DT>::T* row = values + vbase + (long)s * vs.s;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int d = lane + 32 * j;
      if (d < D) {
        const float v = to_f(row[d]);
        ap[j] = __fadd_rn(ap[j], v);
#pragma unroll
        for (int c = 0; c < CMAX; ++c)
          if (c == cc) ac[c][j] = __fadd_rn(ac[c][j], v);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    const int d = lane + 32 * j;
    if (d < D) {
      pagg[gp * D + d] = from_f<DT>(ap[j]);
      if (pacc) pacc[gp * D + d] = ap[j];
#pragma unroll
      for (int c = 0; c < CMAX; ++c)
        if (c < C) {
          cagg[(gp * C + c) * D + d] = from_f<DT>(ac[c][j]);
          if (cacc) cacc[(gp * C + c) * D + d] = ac[c][j];
        }
    }
  }
  if (lane == 0)
#pragma unroll
    for (int c = 0; c < CMAX; ++c)
      if (c < C) ccnt[gp * C + c] = cn[c];
}

template <int DT>
__device__ __forceinline__ float half_bits_to_f(uint32_t u) {
  if (DT == DT_BF16) return __uint_as_float(u << 16);
  return __half2float(__ushort_as_half((unsigned short)u));
}

// VPL consecutive dtype elements with one 4/8/16-byte load.
template <int DT, int VPL>
__device__ __forceinline__ void load_row_elems(const typename Storage<DT>::T* p, float* out) {
  if constexpr (DT == DT_F32) {
    if constexpr (VPL == 4) {
      const float4 w = *reinterpret_cast<const float4*>(p);
      out[0] = w.x; out[1] = w.y; out[2] = w.z; out[3] = w.w;
    } else {
      const float2 w = *reinterpret_cast<const float2*>(p);
      out[0] = w.x; out[1] = w.y;
    }
  } else if constexpr (VPL == 4) {
    const uint2 w = *reinterpret_cast<const uint2*>(p);
    out[0] = half_bits_to_f<DT>(w.x & 0xffffu); out[1] = half_bits_to_f<DT>(w.x >> 16);
    out[2] = half_bits_to_f<DT>(w.y & 0xffffu); out[3] = half_bits_to_f<DT>(w.y >> 16);
  } else {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(p);
    out[0] = half_bits_to_f<DT>(w & 0xffffu); out[1] = half_bits_to_f<DT>(w >> 16);
  }
}

// Vectorised aggregation for D = 32 * VPL (VPL = 2 or 4 dtype elements per
// lane).  One warp per parent; the member rows stream through a per-warp
// ring of AG_RING rows in shared memory filled with cp.async, so AG_RING rows
// per warp are in flight independently of the register budget.  Lane l copies
// and later reads only its own VPL-element slice of every row, so the ring
// needs no cross-lane synchronisation.  The fp32 additions stay in key order
// (index_add_, quantizer.py:241-262).
constexpr int AG_WARPS = 8;
constexpr int AG_BATCH = 4;  // parents per work-counter increment

template <int BYTES>
__device__ __forceinline__ void cp_async_slice(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], %2;\n" ::"r"(smem_u32(smem)), "l"(gmem), "n"(BYTES));
}

template <int DT, int CMAX, int VPL>
__global__ void __launch_bounds__(AG_WARPS * 32) aggregate_vec_kernel(
    const typename Storage<DT>::T* __restrict__ values, Strides3 vs, int H, int S, int M0, int C,
    const int* __restrict__ order, const int* __restrict__ poff, const int* __restrict__ pcnt,
    const int* __restrict__ cassign, typename Storage<DT>::T* __restrict__ pagg,
    typename Storage<DT>::T* __restrict__ cagg, float* __restrict__ pacc, float* __restrict__ cacc,
    int* __restrict__ ccnt, long rows, int* __restrict__ next_row) {
  using T = typename Storage<DT>::T;
  struct alignas(VPL * sizeof(T)) V {
    T e[VPL];
  };
  constexpr int D = 32 * VPL, AG_RING = sizeof(T) == 4 ? 8 : 16, SB = VPL * (int)sizeof(T);
  __shared__ __align__(16) T ring_all[AG_WARPS][AG_RING][D];
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  T (*ring)[D] = ring_all[wib];
  // persistent warps: each takes the next AG_BATCH parents from a counter, so a
  // long member list never holds up the other warps of its block; the batch's
  // member offsets and counts come in one load
  for (;;) {
  int gnext = 0;
  if (lane == 0) gnext = atomicAdd(next_row, AG_BATCH);
  const long gb = __shfl_sync(0xffffffffu, gnext, 0);
  if (gb >= rows) break;
  const int bpoff = lane < AG_BATCH && gb + lane < rows ? poff[gb + lane] : 0;
  const int bpcnt = lane < AG_BATCH && gb + lane < rows ? pcnt[gb + lane] : 0;
  for (int kb = 0; kb < AG_BATCH && gb + kb < rows; ++kb) {
  const long gp = gb + kb;
  const int g = (int)(gp / M0), b = g / H, h = g % H;
  const T* vbase = values + (long)b * vs.b + (long)h * vs.h + lane * VPL;
  float ap[VPL], ac[CMAX][VPL];
  int cn = 0;  // lane c < CMAX counts child c
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    ap[j] = 0.f;
#pragma unroll
    for (int c = 0; c < CMAX; ++c) ac[c][j] = 0.f;
  }
  const int beg = __shfl_sync(0xffffffffu, bpoff, kb), n = __shfl_sync(0xffffffffu, bpcnt, kb);
  const int* ord = order + (long)g * S + beg;
  const int* cas = cassign + (long)g * S;
  // member ids: batch i0 in (cur_s, cur_c), the next batch in (nxt_s)
  int cur_s = lane < n ? ord[lane] : 0;
  int cur_c = lane < n ? cas[cur_s] : -1;
  int nxt_s = lane + 32 < n ? ord[lane + 32] : 0;
  // prologue: the first AG_RING rows
  const int pre = min(n, AG_RING);
  for (int i = 0; i < AG_RING; ++i) {
    if (i < pre) {
      const int s = __shfl_sync(0xffffffffu, cur_s, i);
      cp_async_slice<SB>(&ring[i][lane * VPL], vbase + (long)s * vs.s);
    }
    cp_async_commit();
  }
  for (int i0 = 0; i0 < n; i0 += 32) {
    const int m = min(32, n - i0);
#pragma unroll
    for (int c = 0; c < CMAX; ++c) {
      const int k = __popc(__ballot_sync(0xffffffffu, cur_c == c));
      if (lane == c) cn += k;
    }
    for (int j = 0; j < m; ++j) {
      const int i = i0 + j;
      cp_async_wait<AG_RING - 1>();  // row i has landed (groups complete in order)
      float v[VPL];
      load_row_elems<DT, VPL>(&ring[i % AG_RING][lane * VPL], v);
      const int cc = __shfl_sync(0xffffffffu, cur_c, j);
#pragma unroll
      for (int q = 0; q < VPL; ++q) ap[q] = __fadd_rn(ap[q], v[q]);
      // the row's child, the same in every lane (a shuffled member id), so each
      // test is a uniform branch and only that child's sums take the row
#pragma unroll
      for (int c = 0; c < CMAX; ++c)
        if (c == cc)
#pragma unroll
          for (int q = 0; q < VPL; ++q) ac[c][q] = __fadd_rn(ac[c][q], v[q]);
      // refill the slot with row i + AG_RING (after the slot's value was used)
      const int ni = i + AG_RING;
      if (ni < n) {
        const int nj = ni - i0;  // < 32 + AG_RING: in this batch or the next
        const int a = __shfl_sync(0xffffffffu, cur_s, nj & 31), bb = __shfl_sync(0xffffffffu, nxt_s, nj & 31);
        cp_async_slice<SB>(&ring[i % AG_RING][lane * VPL], vbase + (long)(nj < 32 ? a : bb) * vs.s);
      }
      cp_async_commit();
    }
    // advance the id batches
    cur_s = nxt_s;
    cur_c = (lane + i0 + 32 < n) ? cas[cur_s] : -1;
    nxt_s = lane + i0 + 64 < n ? ord[i0 + 64 + lane] : 0;
  }
  cp_async_wait<0>();
  const long o = gp * D + lane * VPL;
  V pv;
#pragma unroll
  for (int q = 0; q < VPL; ++q) pv.e[q] = from_f<DT>(ap[q]);
  *reinterpret_cast<V*>(pagg + o) = pv;
  if (pacc)
#pragma unroll
    for (int q = 0; q < VPL; ++q) pacc[o + q] = ap[q];
#pragma unroll
  for (int c = 0; c < CMAX; ++c) {
    if (c < C) {
      const long oc = (gp * C + c) * D + lane * VPL;
#pragma unroll
      for (int q = 0; q < VPL; ++q) pv.e[q] = from_f<DT>(ac[c][q]);
      *reinterpret_cast<V*>(cagg + oc) = pv;
      if (cacc)
#pragma unroll
        for (int q = 0; q < VPL; ++q) cacc[oc + q] = ac[c][q];
    }
  }
  if (lane < C) ccnt[gp * C + lane] = cn;
  }
  }
}

// ---------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------
template <int DT>
int launch_prep_codebook(const float* parents32, const float* children32, int H, int M0, int C, int D,
                         void* parents_dt, void* children_dt, float* p_sq, float* c_sq, cudaStream_t st) {
  using T = typename Storage<DT>::T;
  const long rp = (long)H * M0, rc = rp * C;
  prep_codebook_kernel<DT><<<(unsigned)((rp + 7) / 8), 256, 0, st>>>(parents32, (T*)parents_dt, p_sq, rp, D);
  prep_codebook_kernel<DT><<<(unsigned)((rc + 7) / 8), 256, 0, st>>>(children32, (T*)children_dt, c_sq, rc, D);
  return cudaPeekAtLastError() == cudaSuccess ? AVQ_OK : AVQ_ERR_CUDA;
}

int bucket_segments(int S, int M0, int* seg_len) {
  int nseg = S / 256;
  if (nseg < 1) nseg = 1;
  if (nseg > 64) nseg = 64;
  *seg_len = (S + nseg - 1) / nseg;
  if (*seg_len < 1) *seg_len = 1;
  return nseg;
}

size_t quantize_workspace_bytes(int G, int S, int M0) {
  int seg_len;
  const int nseg = bucket_segments(S, M0, &seg_len);
  return align_up((size_t)G * nseg * M0 * sizeof(int)) + align_up((size_t)G * (S > 0 ? S : 1) * sizeof(int)) +
         align_up((size_t)G * M0 * sizeof(int)) + align_up(sizeof(int));
}

template <int DT>
int launch_quantize(const QuantizeArgs& a, cudaStream_t st) {
  using T = typename Storage<DT>::T;
  const int G = a.B * a.H;
  if (a.D > 256 || a.C > 8 || a.M0 > 8192) return AVQ_ERR_UNSUPPORTED;
  int seg_len;
  const int nseg = bucket_segments(a.S, a.M0, &seg_len);
  char* ws = (char*)a.workspace;
  int* hist = (int*)ws;
  ws += align_up((size_t)G * nseg * a.M0 * sizeof(int));
  int* order = (int*)ws;
  ws += align_up((size_t)G * (a.S > 0 ? a.S : 1) * sizeof(int));
  int* poff = (int*)ws;
  ws += align_up((size_t)G * a.M0 * sizeof(int));
  int* agg_next = (int*)ws;  // work counter of the persistent aggregation warps
  bool child_later = false;  // the tcgen05 parent pass leaves the children to launch_child_bucket
  if (a.S > 0) {
    const bool aligned = ((uintptr_t)a.keys % 16 == 0) && a.ks.s % 8 == 0 && a.ks.h % 8 == 0 && a.ks.b % 8 == 0;
    bool done = false;
    if constexpr (DT != DT_F32) {
      if (aligned && assign_tc_ok(DT, a.D, a.M0)) {
        const int rc = launch_assign_tc<DT>(a, st);
        if (rc != AVQ_OK && rc != AVQ_ERR_UNSUPPORTED) return rc;
        done = rc == AVQ_OK;
        child_later = done;
      }
      if (!done && aligned && (a.D == 64 || a.D == 128)) {
        done = true;
      auto launch_mma = [&](auto kfn, int D) {
        AVQ_TIMED("assign", st);
        const size_t smem = (size_t)(AM_ROWS + 2 * AM_CH) * (D + 8) * sizeof(T) +
                            (AM_ROWS + 2 * AM_CH) * sizeof(float) + AM_ROWS * sizeof(int);
        cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        kfn<<<dim3((a.S + AM_ROWS - 1) / AM_ROWS, G), 256, smem, st>>>(
            (const T*)a.keys, a.ks, a.H, a.S, a.M0, a.C, (const T*)a.parents_dt, a.p_sq, (const T*)a.children_dt,
            a.c_sq, a.passign, a.cassign);
      };
        if (a.D == 64) launch_mma(assign_mma_kernel<DT, 64>, 64);
        else launch_mma(assign_mma_kernel<DT, 128>, 128);
      }
    }
    if (!done) {
      AVQ_TIMED("assign_exact", st);
      const size_t smem = (size_t)((AS_ROWS + AS_COLS) * (a.D + 1) + AS_ROWS) * sizeof(float);
      auto kfn = assign_kernel<DT>;
      cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      dim3 grid((a.S + AS_ROWS - 1) / AS_ROWS, G);
      kfn<<<grid, 256, smem, st>>>((const T*)a.keys, a.ks, a.H, a.S, a.D, a.M0, a.C, (const T*)a.parents_dt, a.p_sq,
                                   (const T*)a.children_dt, a.c_sq, a.passign, a.cassign);
    }
  }
  {
    AVQ_TIMED("bucket_sort", st);
    if (a.S > 0)
      bucket_hist_kernel<<<dim3(nseg, G), 256, a.M0 * sizeof(int), st>>>(a.passign, a.S, a.M0, nseg, seg_len, hist);
    else
      cudaMemsetAsync(hist, 0, (size_t)G * nseg * a.M0 * sizeof(int), st);
    bucket_scan_kernel<<<G, 1024, a.M0 * sizeof(int), st>>>(hist, a.M0, nseg, poff, a.pcnt, a.nvalid, a.gmin_valid);
    if (a.S > 0)
      bucket_scatter_kernel<<<dim3(nseg, G), 32, a.M0 * sizeof(int), st>>>(a.passign, hist, a.S, a.M0, nseg, seg_len,
                                                                           order);
  }
  if constexpr (DT != DT_F32) {
    if (child_later) {
      const int rc = launch_child_bucket<DT>(a, order, st);
      if (rc != AVQ_OK) return rc;
    }
  }
  AVQ_TIMED("aggregate", st);
  const long rows = (long)G * a.M0;
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  const bool valigned = ((uintptr_t)a.values % 16 == 0) && a.vs.s % 8 == 0 && a.vs.h % 8 == 0 && a.vs.b % 8 == 0;
  if (valigned && (a.D == 64 || a.D == 128)) {
    int dev = 0, nsm = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    const unsigned pblocks = (unsigned)std::min<long>((long)blocks, (long)nsm * 8);
    cudaMemsetAsync(agg_next, 0, sizeof(int), st);
#define AVQ_AGGV(CM, VP)                                                                                         \
  aggregate_vec_kernel<DT, CM, VP><<<pblocks, 256, 0, st>>>((const T*)a.values, a.vs, a.H, a.S, a.M0, a.C, order, \
                                                            poff, a.pcnt, a.cassign, (T*)a.pagg, (T*)a.cagg,     \
                                                            a.pacc, a.cacc, a.ccnt, rows, agg_next)
    if (a.C <= 4) {
      if (a.D == 64) AVQ_AGGV(4, 2); else AVQ_AGGV(4, 4);
    } else {
      if (a.D == 64) AVQ_AGGV(8, 2); else AVQ_AGGV(8, 4);
    }
#undef AVQ_AGGV
    return cudaPeekAtLastError() == cudaSuccess ? AVQ_OK : AVQ_ERR_CUDA;
  }
#define AVQ_AGG(CM, DM)                                                                                         \
  aggregate_kernel<DT, CM, DM><<<blocks, 256, 0, st>>>((const T*)a.values, a.vs, a.H, a.S, a.D, a.M0, a.C, order, \
                                                       poff, a.pcnt, a.cassign, (T*)a.pagg, (T*)a.cagg, a.pacc,  \
                                                       a.cacc, a.ccnt, rows)
  if (a.C <= 4) {
    if (a.D <= 64) AVQ_AGG(4, 64); else if (a.D <= 128) AVQ_AGG(4, 128); else AVQ_AGG(4, 256);
  } else {
    if (a.D <= 64) AVQ_AGG(8, 64); else if (a.D <= 128) AVQ_AGG(8, 128); else AVQ_AGG(8, 256);
  }
#undef AVQ_AGG
  return cudaPeekAtLastError() == cudaSuccess ? AVQ_OK : AVQ_ERR_CUDA;
}

template int launch_prep_codebook<DT_F32>(const float*, const float*, int, int, int, int, void*, void*, float*, float*,
                                          cudaStream_t);
template int launch_prep_codebook<DT_BF16>(const float*, const float*, int, int, int, int, void*, void*, float*,
                                           float*, cudaStream_t);
template int launch_prep_codebook<DT_F16>(const float*, const float*, int, int, int, int, void*, void*, float*, float*,
                                          cudaStream_t);
template int launch_quantize<DT_F32>(const QuantizeArgs&, cudaStream_t);
template int launch_quantize<DT_BF16>(const QuantizeArgs&, cudaStream_t);
template int launch_quantize<DT_F16>(const QuantizeArgs&, cudaStream_t);

}  // namespace avq
