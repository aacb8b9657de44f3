// Decode: incremental quantization of appended tokens and the paged KV write
// (reference attention_module.py:350-367 resolve_kv_cache + cache.py:246-299,
// then quantizer.py:166-278 on the grown key set).
//
// The reference re-quantizes every cached key on every decode step.  With a
// static codebook the old keys keep their assignments, and each bucket's fp32
// key-order sum only gains the new key at its end, so the incremental update
//     acc32[bucket] += v ;  agg[bucket] = dtype(acc32[bucket]) ;  count += 1
// is bit-identical to the full recomputation.
#include "avq_kernels.cuh"

namespace avq {

__device__ __forceinline__ bool better_d(float v, int i, float bv, int bi) {
  if (bi < 0) return true;
  const bool n = isnan(v), bn = isnan(bv);
  if (n || bn) return n && (!bn || i < bi);
  return v < bv || (v == bv && i < bi);
}

// One CTA per (b,h); the new tokens are processed one after another in order.
template <int DT>
__global__ void __launch_bounds__(128) append_kernel(
    const typename Storage<DT>::T* __restrict__ knew, Strides3 ks, const typename Storage<DT>::T* __restrict__ vnew,
    Strides3 vs, int H, int Tn, int D, int M0, int C, const typename Storage<DT>::T* __restrict__ parents,
    const float* __restrict__ p_sq, const typename Storage<DT>::T* __restrict__ children,
    const float* __restrict__ c_sq, float* __restrict__ pacc, float* __restrict__ cacc,
    typename Storage<DT>::T* __restrict__ pagg, typename Storage<DT>::T* __restrict__ cagg, int* __restrict__ pcnt,
    int* __restrict__ ccnt, int* __restrict__ nvalid, typename Storage<DT>::T* __restrict__ kpage,
    typename Storage<DT>::T* __restrict__ vpage, Strides3 pgs, int slot0) {
  extern __shared__ float sm[];
  float* kk = sm;           // [D]
  float* red_v = kk + D;    // [128]
  int* red_i = (int*)(red_v + 128);
  __shared__ float ksq_s;
  __shared__ int bestp_s, bestc_s;
  const int g = blockIdx.x, b = g / H, h = g % H, tid = threadIdx.x;
  const long ph = (long)h * M0;
  for (int i = 0; i < Tn; ++i) {
    const typename Storage<DT>::T* krow = knew + (long)b * ks.b + (long)h * ks.h + (long)i * ks.s;
    const typename Storage<DT>::T* vrow = vnew + (long)b * vs.b + (long)h * vs.h + (long)i * vs.s;
    for (int d = tid; d < D; d += blockDim.x) {
      kk[d] = to_f(krow[d]);
      if (kpage) {
        const long o = (long)b * pgs.b + (long)h * pgs.h + (long)(slot0 + i) * pgs.s + d;
        kpage[o] = krow[d];
        vpage[o] = vrow[d];
      }
    }
    __syncthreads();
    if (tid == 0) {
      double acc = 0.0;
      for (int d = 0; d < D; ++d) acc += (double)rnd<DT>(__fmul_rn(kk[d], kk[d]));
      ksq_s = rnd64<DT>(acc);
    }
    __syncthreads();
    const float ksq = ksq_s;
    float bv = 0.f;
    int bi = -1;
    for (int p = tid; p < M0; p += blockDim.x) {
      const typename Storage<DT>::T* prow = parents + (ph + p) * D;
      double acc = 0.0;
      for (int d = 0; d < D; ++d) acc = fma((double)kk[d], (double)to_f(prow[d]), acc);
      const float cross = rnd64<DT>(acc);
      const float dd = rnd<DT>(__fsub_rn(rnd<DT>(__fadd_rn(ksq, p_sq[ph + p])), rnd<DT>(__fmul_rn(2.f, cross))));
      if (better_d(dd, p, bv, bi)) {
        bv = dd;
        bi = p;
      }
    }
    red_v[tid] = bv;
    red_i[tid] = bi;
    __syncthreads();
    if (tid == 0) {
      float v = red_v[0];
      int ix = red_i[0];
      for (int k = 1; k < blockDim.x; ++k)
        if (red_i[k] >= 0 && better_d(red_v[k], red_i[k], v, ix)) {
          v = red_v[k];
          ix = red_i[k];
        }
      bestp_s = ix;
    }
    __syncthreads();
    const int p = bestp_s;
    if (tid < 32) {
      float cv = 0.f;
      int ci = -1;
      for (int c = tid; c < C; c += 32) {
        const long crow = (ph + p) * C + c;
        double acc = 0.0;
        for (int d = 0; d < D; ++d) acc += (double)rnd<DT>(__fmul_rn(kk[d], to_f(children[crow * D + d])));
        const float cross = rnd64<DT>(acc);
        const float dd = rnd<DT>(__fsub_rn(rnd<DT>(__fadd_rn(ksq, c_sq[crow])), rnd<DT>(__fmul_rn(2.f, cross))));
        if (better_d(dd, c, cv, ci)) {
          cv = dd;
          ci = c;
        }
      }
      for (int o = 16; o > 0; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, cv, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, ci, o);
        if (i2 >= 0 && better_d(v2, i2, cv, ci)) {
          cv = v2;
          ci = i2;
        }
      }
      if (tid == 0) bestc_s = ci;
    }
    __syncthreads();
    const int c = bestc_s;
    const long gp = (long)g * M0 + p;
    for (int d = tid; d < D; d += blockDim.x) {
      const float v = to_f(vrow[d]);
      const float ap = __fadd_rn(pacc[gp * D + d], v);
      pacc[gp * D + d] = ap;
      pagg[gp * D + d] = from_f<DT>(ap);
      const float ac = __fadd_rn(cacc[(gp * C + c) * D + d], v);
      cacc[(gp * C + c) * D + d] = ac;
      cagg[(gp * C + c) * D + d] = from_f<DT>(ac);
    }
    if (tid == 0) {
      if (pcnt[gp]++ == 0) nvalid[g] += 1;
      ccnt[gp * C + c] += 1;
    }
    __syncthreads();
  }
}

__global__ void reduce_min_kernel(const int* __restrict__ v, int n, int* __restrict__ out) {
  __shared__ int red[1024];
  int m = 0x7fffffff;
  for (int i = threadIdx.x; i < n; i += blockDim.x) m = min(m, v[i]);
  red[threadIdx.x] = m;
  __syncthreads();
  for (int s = blockDim.x >> 1; s > 0; s >>= 1) {
    if (threadIdx.x < s) red[threadIdx.x] = min(red[threadIdx.x], red[threadIdx.x + s]);
    __syncthreads();
  }
  if (threadIdx.x == 0) *out = red[0];
}

template <int DT>
int launch_append(const AppendArgs& a, cudaStream_t st) {
  using T = typename Storage<DT>::T;
  const int G = a.B * a.H;
  if (G == 0 || a.Tn == 0) return AVQ_OK;
  const size_t smem = sizeof(float) * (a.D + 128) + sizeof(int) * 128;
  AVQ_TIMED("append", st);
  append_kernel<DT><<<G, 128, smem, st>>>((const T*)a.k, a.ks, (const T*)a.v, a.vs, a.H, a.Tn, a.D, a.M0, a.C,
                                          (const T*)a.parents_dt, a.p_sq, (const T*)a.children_dt, a.c_sq, a.pacc,
                                          a.cacc, (T*)a.pagg, (T*)a.cagg, a.pcnt, a.ccnt, a.nvalid, (T*)a.kpage,
                                          (T*)a.vpage, a.pgs, a.slot0);
  return cudaPeekAtLastError() == cudaSuccess ? AVQ_OK : AVQ_ERR_CUDA;
}

int launch_reduce_min(const int* v, int n, int* out, cudaStream_t st) {
  reduce_min_kernel<<<1, 1024, 0, st>>>(v, n, out);
  return cudaPeekAtLastError() == cudaSuccess ? AVQ_OK : AVQ_ERR_CUDA;
}

template int launch_append<DT_F32>(const AppendArgs&, cudaStream_t);
template int launch_append<DT_BF16>(const AppendArgs&, cudaStream_t);
template int launch_append<DT_F16>(const AppendArgs&, cudaStream_t);

}  // namespace avq
