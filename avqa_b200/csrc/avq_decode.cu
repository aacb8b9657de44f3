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

// The 16-bit halves of a packed pair as floats (bf16 or fp16 storage).
template <int DT>
__device__ __forceinline__ float half_lo_bits(uint32_t w) {
  return DT == DT_BF16 ? __uint_as_float(w << 16) : __half2float(__ushort_as_half((unsigned short)(w & 0xffffu)));
}
template <int DT>
__device__ __forceinline__ float half_hi_bits(uint32_t w) {
  return DT == DT_BF16 ? __uint_as_float(w & 0xffff0000u) : __half2float(__ushort_as_half((unsigned short)(w >> 16)));
}

__device__ __forceinline__ bool better_d(float v, int i, float bv, int bi) {
  if (bi < 0) return true;
  const bool n = isnan(v), bn = isnan(bv);
  if (n || bn) return n && (!bn || i < bi);
  return v < bv || (v == bv && i < bi);
}

// One CTA per (b,h) (256 threads); the new tokens are processed one after
// another in order.  Parent distances: 8 lanes per parent (lane j of the group
// takes elements j, j+8, ...), four parents per warp at a time, the cross term
// k.p summed exactly in fp64 (products of two dtype values are exact) and
// narrowed fp64 -> fp32 -> dtype, as the reference's fp32 matmul rounds its
// exact value when no accumulation error reaches a rounding point.  Children:
// one warp per child with the products rounded to the dtype first
// (quantizer.py:223-226).  First minimum wins, NaN first (torch.argmin).
constexpr int AP_THREADS = 256;

template <int DT>
__global__ void __launch_bounds__(AP_THREADS) append_kernel(
    const typename Storage<DT>::T* __restrict__ knew, Strides3 ks, const typename Storage<DT>::T* __restrict__ vnew,
    Strides3 vs, int H, int Tn, int D, int M0, int C, const typename Storage<DT>::T* __restrict__ parents,
    const float* __restrict__ p_sq, const typename Storage<DT>::T* __restrict__ children,
    const float* __restrict__ c_sq, float* __restrict__ pacc, float* __restrict__ cacc,
    typename Storage<DT>::T* __restrict__ pagg, typename Storage<DT>::T* __restrict__ cagg, int* __restrict__ pcnt,
    int* __restrict__ ccnt, int* __restrict__ nvalid, typename Storage<DT>::T* __restrict__ kpage,
    typename Storage<DT>::T* __restrict__ vpage, Strides3 pgs, int slot0) {
  extern __shared__ float sm[];
  float* kk = sm;  // [D]
  __shared__ float red_v[AP_THREADS / 32][4];
  __shared__ int red_i[AP_THREADS / 32][4];
  __shared__ float cd_v[8];
  __shared__ double ksq_part[AP_THREADS / 32];
  __shared__ int bestp_s, bestc_s;
  const int g = blockIdx.x, b = g / H, h = g % H, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int sub = lane >> 3, l8 = lane & 7;
  const long ph = (long)h * M0;
  for (int i = 0; i < Tn; ++i) {
    const typename Storage<DT>::T* krow = knew + (long)b * ks.b + (long)h * ks.h + (long)i * ks.s;
    const typename Storage<DT>::T* vrow = vnew + (long)b * vs.b + (long)h * vs.h + (long)i * vs.s;
    double sq = 0.0;
    for (int d = tid; d < D; d += AP_THREADS) {
      const float x = to_f(krow[d]);
      kk[d] = x;
      sq += (double)rnd<DT>(__fmul_rn(x, x));  // quantizer.py:207-208 (products rounded, summed in fp32)
      if (kpage) {
        const long o = (long)b * pgs.b + (long)h * pgs.h + (long)(slot0 + i) * pgs.s + d;
        kpage[o] = krow[d];
        vpage[o] = vrow[d];
      }
    }
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    if (lane == 0) ksq_part[warp] = sq;
    __syncthreads();
    double sqt = 0.0;
    for (int w = 0; w < AP_THREADS / 32; ++w) sqt += ksq_part[w];
    const float ksq = rnd64<DT>(sqt);
    // parents: group `sub` of warp `warp` takes parents warp*4 + sub + 32*it,
    // two at a time; with 16-bit elements and D a multiple of 64 a lane reads
    // 16-byte chunks l8, l8 + 8, ... of the row
    float bv = 0.f;
    int bi = -1;
    auto consider = [&](int p, double acc) {
      const float cross = rnd64<DT>(acc);
      const float dd = rnd<DT>(__fsub_rn(rnd<DT>(__fadd_rn(ksq, p_sq[ph + p])), rnd<DT>(__fmul_rn(2.f, cross))));
      if (better_d(dd, p, bv, bi)) {
        bv = dd;
        bi = p;
      }
    };
    const bool vec = DT != DT_F32 && D % 64 == 0;
    for (int p0 = warp * 4; p0 < M0; p0 += 2 * (AP_THREADS / 8)) {
      const int pa = p0 + sub, pb = pa + AP_THREADS / 8;
      double acc0 = 0.0, acc1 = 0.0;
      if (vec) {
        for (int c = l8; c < D / 8; c += 8) {
          const uint4 x0 = pa < M0 ? *reinterpret_cast<const uint4*>(parents + (ph + pa) * D + c * 8) : make_uint4(0, 0, 0, 0);
          const uint4 x1 = pb < M0 ? *reinterpret_cast<const uint4*>(parents + (ph + pb) * D + c * 8) : make_uint4(0, 0, 0, 0);
          const uint32_t w0[4] = {x0.x, x0.y, x0.z, x0.w}, w1[4] = {x1.x, x1.y, x1.z, x1.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const double k0 = (double)kk[c * 8 + 2 * e], k1 = (double)kk[c * 8 + 2 * e + 1];
            acc0 = fma(k0, (double)half_lo_bits<DT>(w0[e]), acc0);
            acc0 = fma(k1, (double)half_hi_bits<DT>(w0[e]), acc0);
            acc1 = fma(k0, (double)half_lo_bits<DT>(w1[e]), acc1);
            acc1 = fma(k1, (double)half_hi_bits<DT>(w1[e]), acc1);
          }
        }
      } else {
        for (int d = l8; d < D; d += 8) {
          const double kd = (double)kk[d];
          if (pa < M0) acc0 = fma(kd, (double)to_f(parents[(ph + pa) * D + d]), acc0);
          if (pb < M0) acc1 = fma(kd, (double)to_f(parents[(ph + pb) * D + d]), acc1);
        }
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, o);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, o);
      }
      if (pa < M0) consider(pa, acc0);
      if (pb < M0) consider(pb, acc1);
    }
    if (l8 == 0) {
      red_v[warp][sub] = bv;
      red_i[warp][sub] = bi;
    }
    __syncthreads();
    if (tid == 0) {
      float v = 0.f;
      int ix = -1;
      for (int w = 0; w < AP_THREADS / 32; ++w)
        for (int k = 0; k < 4; ++k)
          if (red_i[w][k] >= 0 && better_d(red_v[w][k], red_i[w][k], v, ix)) {
            v = red_v[w][k];
            ix = red_i[w][k];
          }
      bestp_s = ix;
    }
    __syncthreads();
    const int p = bestp_s;
    // children: warp c takes child c
    if (warp < C) {
      const long crow = (ph + p) * C + warp;
      double acc = 0.0;
      for (int d = lane; d < D; d += 32) acc += (double)rnd<DT>(__fmul_rn(kk[d], to_f(children[crow * D + d])));
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0) {
        const float cross = rnd64<DT>(acc);
        cd_v[warp] = rnd<DT>(__fsub_rn(rnd<DT>(__fadd_rn(ksq, c_sq[crow])), rnd<DT>(__fmul_rn(2.f, cross))));
      }
    }
    __syncthreads();
    if (tid == 0) {
      float v = 0.f;
      int ix = -1;
      for (int c = 0; c < C; ++c)
        if (better_d(cd_v[c], c, v, ix)) {
          v = cd_v[c];
          ix = c;
        }
      bestc_s = ix;
    }
    __syncthreads();
    const int c = bestc_s;
    const long gp = (long)g * M0 + p;
    for (int d = tid; d < D; d += AP_THREADS) {
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
  if (a.C > 8) return AVQ_ERR_UNSUPPORTED;  // one warp per child
  const size_t smem = sizeof(float) * a.D;
  AVQ_TIMED("append", st);
  append_kernel<DT><<<G, AP_THREADS, smem, st>>>((const T*)a.k, a.ks, (const T*)a.v, a.vs, a.H, a.Tn, a.D, a.M0, a.C,
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
