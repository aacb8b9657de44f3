// Dense attention (reference backend.py:190-203 naive_attention and
// :105-156 online_softmax_attention): softmax(mask(DT(DT(q k^T) * D^-1/2))) v.
// It is the reference's execution.mode = "reference" path, the path with
// refinement disabled, and the budget-0 fallback (pipeline.py:261-273, 310-345).
//
//   without a mask, bf16 / fp16, D in {64, 128}: the tcgen05 parent-attention
//       kernel in its dense mode (avq_parent_tc.cu): keys and values as its
//       parent and parent-sum tiles, two passes (row max, then e = DT(exp(
//       DT(s - m))) and O += e V on the tensor cores), out = DT(O / z);
//   dense_attn_mma_kernel   bf16 / fp16, D in {64, 128}: one CTA per 64
//       queries of one (b,h), 64-key tiles double-buffered with cp.async,
//       S = Q K^T and O += P V on mma.sync (fp32 accumulators), the softmax
//       online in fp32 (FlashAttention-2 order: running max, rescaled sums).
//   dense_attn_simt_kernel  every other shape and fp32: a warp per query, the
//       dot products and the online softmax in fp32.
//
// The logits are rounded where the reference rounds them (the matmul result
// to the dtype, then the scaled logit); the probabilities stay fp32 until the
// P V product (bf16 / fp16 operands), which the output tolerance of the
// dtype covers.  A query whose keys are all masked gets NaN, as softmax over
// -inf does; the output is in the input dtype.
#include <cmath>

#include "avq_kernels.cuh"
#include "avq_mma.cuh"

namespace avq {

namespace {

constexpr int DQ = 64, DK = 64;  // queries per CTA, keys per tile

template <int DT, int D>
__global__ void __launch_bounds__(128) dense_attn_mma_kernel(
    const typename Storage<DT>::T* __restrict__ q, Strides3 qs, const typename Storage<DT>::T* __restrict__ k,
    Strides3 ks, const typename Storage<DT>::T* __restrict__ v, Strides3 vs, int H, int T, int N, float scale,
    const unsigned char* __restrict__ mask, long long mb, long long mh, long long mt,
    typename Storage<DT>::T* __restrict__ out, Strides3 os) {
  using T_ = typename Storage<DT>::T;
  constexpr int LDS = D + 8, KS = D / 16, CPR = D / 8, NT = D / 8;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T_* sq_ = reinterpret_cast<T_*>(smem_raw);  // [DQ][LDS]
  T_* sk = sq_ + DQ * LDS;                   // [2][DK][LDS]
  T_* sv = sk + 2 * DK * LDS;                // [2][DK][LDS]
  const int g = blockIdx.y, b = g / H, h = g % H, t0 = blockIdx.x * DQ;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r0 = warp * 16 + (lane >> 2), r1 = r0 + 8, cq = (lane & 3) * 2;
  const T_* qb = q + (long)b * qs.b + (long)h * qs.h;
  const T_* kb = k + (long)b * ks.b + (long)h * ks.h;
  const T_* vb = v + (long)b * vs.b + (long)h * vs.h;
  for (int i = tid; i < DQ * CPR; i += 128) {
    const int r = i / CPR, c = i % CPR, t = t0 + r;
    cp_async16(sq_ + r * LDS + c * 8, qb + (long)(t < T ? t : 0) * qs.s + c * 8, t < T);
  }
  auto load_kv = [&](int tile, int buf) {
    for (int i = tid; i < DK * CPR; i += 128) {
      const int r = i / CPR, c = i % CPR, n = tile * DK + r;
      cp_async16(sk + (buf * DK + r) * LDS + c * 8, kb + (long)(n < N ? n : 0) * ks.s + c * 8, n < N);
      cp_async16(sv + (buf * DK + r) * LDS + c * 8, vb + (long)(n < N ? n : 0) * vs.s + c * 8, n < N);
    }
  };
  const int ntile = (N + DK - 1) / DK;
  load_kv(0, 0);
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  uint32_t af[KS][4];
#pragma unroll
  for (int kk = 0; kk < KS; ++kk)
    ldsm_x4(af[kk][0], af[kk][1], af[kk][2], af[kk][3], sq_ + (warp * 16 + (lane & 15)) * LDS + kk * 16 + (lane >> 4) * 8);
  float oacc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) oacc[j][0] = oacc[j][1] = oacc[j][2] = oacc[j][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const unsigned char* mrow0 = mask ? mask + b * mb + h * mh + (long)(t0 + r0 < T ? t0 + r0 : 0) * mt : nullptr;
  const unsigned char* mrow1 = mask ? mask + b * mb + h * mh + (long)(t0 + r1 < T ? t0 + r1 : 0) * mt : nullptr;
  for (int tile = 0; tile < ntile; ++tile) {
    const int buf = tile & 1;
    if (tile + 1 < ntile) load_kv(tile + 1, buf ^ 1);
    cp_async_commit();
    const T_* skb = sk + buf * DK * LDS;
    const T_* svb = sv + buf * DK * LDS;
    // S = Q K^T (16 rows x 64 keys per warp)
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        uint32_t b0, b1, b2, b3;
        const int qd = lane >> 3;
        ldsm_x4(b0, b1, b2, b3, skb + (jj * 16 + (qd >> 1) * 8 + (lane & 7)) * LDS + kk * 16 + (qd & 1) * 8);
        mma16816<DT>(s[2 * jj], af[kk], b0, b1);
        mma16816<DT>(s[2 * jj + 1], af[kk], b2, b3);
      }
    }
    // logits DT(DT(acc) * scale) (backend.py:197), masked (:199), tile row max
    float tm0 = -INFINITY, tm1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int n = tile * DK + j * 8 + cq + (e & 1);
        const unsigned char* mr = e >= 2 ? mrow1 : mrow0;
        float x = rnd<DT>(__fmul_rn(rnd<DT>(s[j][e]), scale));
        if (n >= N || (mr && !mr[n])) x = -INFINITY;
        s[j][e] = x;
        if (e >= 2) tm1 = fmaxf(tm1, x);
        else tm0 = fmaxf(tm0, x);
      }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      tm0 = fmaxf(tm0, __shfl_xor_sync(0xffffffffu, tm0, o));
      tm1 = fmaxf(tm1, __shfl_xor_sync(0xffffffffu, tm1, o));
    }
    const float n0 = fmaxf(m0, tm0), n1 = fmaxf(m1, tm1);
    // the fast exponential (within 2 ulp): the probabilities feed the P V product
    // in the dtype, far coarser than fp32
    const float c0 = n0 == -INFINITY ? 1.f : __expf(m0 - n0), c1 = n1 == -INFINITY ? 1.f : __expf(m1 - n1);
    m0 = n0;
    m1 = n1;
    l0 *= c0;
    l1 *= c1;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      oacc[j][0] *= c0;
      oacc[j][1] *= c0;
      oacc[j][2] *= c1;
      oacc[j][3] *= c1;
    }
    // P = exp(s - m) as the A operand of O += P V (16 keys per k step)
    uint32_t pa[4][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float p[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mm = e >= 2 ? m1 : m0;
        p[e] = s[j][e] == -INFINITY ? 0.f : __expf(s[j][e] - mm);
      }
      l0 += p[0] + p[1];
      l1 += p[2] + p[3];
      const int kk = j >> 1, hi = j & 1;
      pa[kk][2 * hi] = pack2<DT>(p[0], p[1]);
      pa[kk][2 * hi + 1] = pack2<DT>(p[2], p[3]);
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t a2[4] = {pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3]};
#pragma unroll
      for (int jj = 0; jj < NT / 2; ++jj) {
        uint32_t b0, b1, b2, b3;
        const int qd = lane >> 3;
        ldsm_x4_t(b0, b1, b2, b3, svb + (kk * 16 + (qd & 1) * 8 + (lane & 7)) * LDS + jj * 16 + (qd >> 1) * 8);
        mma16816<DT>(oacc[2 * jj], a2, b0, b1);
        mma16816<DT>(oacc[2 * jj + 1], a2, b2, b3);
      }
    }
    cp_async_wait<0>();
    __syncthreads();
  }
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, o);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o);
  }
  // softmax over a row of -inf is NaN (torch.softmax)
  const float i0 = m0 == -INFINITY ? NAN : 1.f / l0, i1 = m1 == -INFINITY ? NAN : 1.f / l1;
  T_* o0 = out + (long)b * os.b + (long)h * os.h + (long)(t0 + r0) * os.s;
  T_* o1 = out + (long)b * os.b + (long)h * os.h + (long)(t0 + r1) * os.s;
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int d = j * 8 + cq;
    if (t0 + r0 < T) *reinterpret_cast<uint32_t*>(o0 + d) = pack2<DT>(oacc[j][0] * i0, oacc[j][1] * i0);
    if (t0 + r1 < T) *reinterpret_cast<uint32_t*>(o1 + d) = pack2<DT>(oacc[j][2] * i1, oacc[j][3] * i1);
  }
}

// A warp per query; lane j holds dimensions j, j + 32, ... (D <= 256).
template <int DT>
__global__ void __launch_bounds__(256) dense_attn_simt_kernel(
    const typename Storage<DT>::T* __restrict__ q, Strides3 qs, const typename Storage<DT>::T* __restrict__ k,
    Strides3 ks, const typename Storage<DT>::T* __restrict__ v, Strides3 vs, int H, int T, int N, int D, float scale,
    const unsigned char* __restrict__ mask, long long mb, long long mh, long long mt,
    typename Storage<DT>::T* __restrict__ out, Strides3 os) {
  const int g = blockIdx.y, b = g / H, h = g % H, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= T) return;
  float qv[8], o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int d = lane + 32 * i;
    qv[i] = d < D ? to_f(q[(long)b * qs.b + (long)h * qs.h + (long)t * qs.s + d]) : 0.f;
    o[i] = 0.f;
  }
  const unsigned char* mr = mask ? mask + b * mb + h * mh + (long)t * mt : nullptr;
  float m = -INFINITY, l = 0.f;
  for (int n = 0; n < N; ++n) {
    const auto* kr = k + (long)b * ks.b + (long)h * ks.h + (long)n * ks.s;
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int d = lane + 32 * i;
      if (d < D) dot = fmaf(qv[i], to_f(kr[d]), dot);
    }
    for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
    float x = rnd<DT>(__fmul_rn(rnd<DT>(dot), scale));
    if (mr && !mr[n]) x = -INFINITY;
    if (x == -INFINITY) continue;
    const float mn = fmaxf(m, x), c = m == -INFINITY ? 0.f : expf(m - mn), p = expf(x - mn);
    m = mn;
    l = l * c + p;
    const auto* vr = v + (long)b * vs.b + (long)h * vs.h + (long)n * vs.s;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int d = lane + 32 * i;
      if (d < D) o[i] = fmaf(p, to_f(vr[d]), o[i] * c);
    }
  }
  const float inv = m == -INFINITY ? NAN : 1.f / l;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int d = lane + 32 * i;
    if (d < D) out[(long)b * os.b + (long)h * os.h + (long)t * os.s + d] = from_f<DT>(o[i] * inv);
  }
}

}  // namespace

template <int DT>
int launch_dense_attention(const void* q, Strides3 qs, const void* k, Strides3 ks, const void* v, Strides3 vs, int B,
                           int H, int T, int N, int D, const unsigned char* mask, const long long* mst, void* out,
                           Strides3 os, cudaStream_t st) {
  using T_ = typename Storage<DT>::T;
  const int G = B * H;
  if (G == 0 || T == 0) return AVQ_OK;
  if (D > 256) return AVQ_ERR_UNSUPPORTED;
  const float scale = (float)std::pow((double)D, -0.5);  // scale_for (backend.py:43-45)
  const long long mb = mask ? mst[0] : 0, mh = mask ? mst[1] : 0, mt = mask ? mst[2] : 0;
  auto aligned = [](const void* p, Strides3 s) {
    return ((uintptr_t)p % 16) == 0 && s.b % 8 == 0 && s.h % 8 == 0 && s.s % 8 == 0;
  };
  bool mma = DT != DT_F32 && (D == 64 || D == 128) && aligned(q, qs) && aligned(k, ks) && aligned(v, vs) &&
             ((uintptr_t)out % 4) == 0 && os.s % 2 == 0 && os.h % 2 == 0 && os.b % 2 == 0;
  AVQ_TIMED("dense_attn", st);
  if constexpr (DT != DT_F32) {
    if (!mask) {  // the tcgen05 parent-attention kernel in its dense mode
      const int rc = launch_dense_tc<DT>(q, qs, k, ks, v, vs, B, H, T, N, D, scale, out, os, st);
      if (rc != AVQ_ERR_UNSUPPORTED) return rc;
    }
    if (mma) {
      const size_t smem = (size_t)(DQ + 4 * DK) * (D + 8) * sizeof(T_);
      auto go = [&](auto kfn) {
        cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        kfn<<<dim3((T + DQ - 1) / DQ, G), 128, smem, st>>>(
            static_cast<const T_*>(q), qs, static_cast<const T_*>(k), ks, static_cast<const T_*>(v), vs, H, T, N,
            scale, mask, mb, mh, mt, static_cast<T_*>(out), os);
      };
      if (D == 64) go(dense_attn_mma_kernel<DT, 64>);
      else go(dense_attn_mma_kernel<DT, 128>);
      return cudaPeekAtLastError() == cudaSuccess ? AVQ_OK : AVQ_ERR_CUDA;
    }
  }
  dense_attn_simt_kernel<DT><<<dim3((T + 7) / 8, G), 256, 0, st>>>(
      static_cast<const T_*>(q), qs, static_cast<const T_*>(k), ks, static_cast<const T_*>(v), vs, H, T, N, D, scale,
      mask, mb, mh, mt, static_cast<T_*>(out), os);
  return cudaPeekAtLastError() == cudaSuccess ? AVQ_OK : AVQ_ERR_CUDA;
}

template int launch_dense_attention<DT_F32>(const void*, Strides3, const void*, Strides3, const void*, Strides3, int,
                                            int, int, int, int, const unsigned char*, const long long*, void*,
                                            Strides3, cudaStream_t);
template int launch_dense_attention<DT_BF16>(const void*, Strides3, const void*, Strides3, const void*, Strides3, int,
                                             int, int, int, int, const unsigned char*, const long long*, void*,
                                             Strides3, cudaStream_t);
template int launch_dense_attention<DT_F16>(const void*, Strides3, const void*, Strides3, const void*, Strides3, int,
                                            int, int, int, int, const unsigned char*, const long long*, void*,
                                            Strides3, cudaStream_t);

}  // namespace avq
