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
#include "avq_mma.cuh"

namespace avq {

__device__ __forceinline__ bool better_d(float v, int i, float bv, int bi) {
  if (bi < 0) return true;
  const bool n = isnan(v), bn = isnan(bv);
  if (n || bn) return n && (!bn || i < bi);
  return v < bv || (v == bv && i < bi);
}

// ---------------------------------------------------------------------------
// Parent assignment of the appended keys on mma.sync tensor cores: one CTA per
// (head, 128-parent chunk, 64 appended rows), the cross terms k.p as the fp32
// accumulators of the same MMA K-order as the prefill quantizer, then
// d = DT(DT(k_sq + p_sq) - DT(2 DT(k.p))) (quantizer.py:207-210) and the first
// minimum over the chunk, merged across chunks by an atomicMin on packed
// (distance order, index) keys; a NaN distance wins, the lowest index first
// (torch.argmin).  Rows are (b, token) pairs of one head.
constexpr int AA_ROWS = 64, AA_COLS = 128;

// Packed argmin key: a NaN distance first, then ascending distance, then index.
__device__ __forceinline__ unsigned long long argmin_key(float d, int p) {
  const unsigned long long o = isnan(d) ? 0ull : (unsigned long long)float_order_key(d) + 1ull;
  return (o << 32) | (unsigned)p;
}

template <int DT, int D>
__global__ void __launch_bounds__(256) append_assign_kernel(const typename Storage<DT>::T* __restrict__ knew,
                                                            Strides3 ks, int B, int H, int Tn, int M0,
                                                            const typename Storage<DT>::T* __restrict__ parents,
                                                            const float* __restrict__ p_sq,
                                                            unsigned long long* __restrict__ best) {
  using T = typename Storage<DT>::T;
  constexpr int LDS = D + 8, KS = D / 16, CPR = D / 8;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* sk = reinterpret_cast<T*>(smem_raw);  // [AA_ROWS][LDS] keys
  T* sp = sk + AA_ROWS * LDS;              // [AA_COLS][LDS] parents
  float* ksq = reinterpret_cast<float*>(sp + AA_COLS * LDS);  // [AA_ROWS]
  const int h = blockIdx.x, p0 = blockIdx.y * AA_COLS, r0 = blockIdx.z * AA_ROWS, NR = B * Tn;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  auto key_ptr = [&](int r) {  // row r = b * Tn + i
    const int b = r / Tn, i = r % Tn;
    return knew + (long)b * ks.b + (long)h * ks.h + (long)i * ks.s;
  };
  for (int x = tid; x < AA_ROWS * CPR; x += 256) {
    const int r = x / CPR, c = x % CPR, rr = r0 + r;
    cp_async16(sk + r * LDS + c * 8, key_ptr(rr < NR ? rr : 0) + c * 8, rr < NR);
  }
  for (int x = tid; x < AA_COLS * CPR; x += 256) {
    const int r = x / CPR, c = x % CPR, p = p0 + r;
    cp_async16(sp + r * LDS + c * 8, parents + ((long)h * M0 + (p < M0 ? p : 0)) * D + c * 8, p < M0);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  // k_sq: the dtype-rounded squares summed exactly (quantizer.py:207-208), a warp per row
  for (int r = warp; r < AA_ROWS; r += 8) {
    double sq = 0.0;
    for (int d = lane; d < D; d += 32) {
      const float x = to_f(sk[r * LDS + d]);
      sq += (double)rnd<DT>(__fmul_rn(x, x));
    }
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    if (lane == 0) ksq[r] = rnd64<DT>(sq);
  }
  const int mt = warp & 3, nh = warp >> 2;  // rows 16 mt .. +16, parents 64 nh .. +64
  float acc[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
#pragma unroll
  for (int k = 0; k < KS; ++k) {
    uint32_t af[4];
    ldsm_x4(af[0], af[1], af[2], af[3], sk + (mt * 16 + (lane & 15)) * LDS + k * 16 + (lane >> 4) * 8);
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      uint32_t b0f, b1f, b2f, b3f;
      const int qd = lane >> 3;
      ldsm_x4(b0f, b1f, b2f, b3f, sp + (nh * 64 + jj * 16 + (qd >> 1) * 8 + (lane & 7)) * LDS + k * 16 + (qd & 1) * 8);
      mma16816<DT>(acc[2 * jj], af, b0f, b1f);
      mma16816<DT>(acc[2 * jj + 1], af, b2f, b3f);
    }
  }
  __syncthreads();  // ksq complete
  // rows (lane >> 2) and +8 of the warp's 16; the four lanes of a row cover its 64 columns
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int r = mt * 16 + (lane >> 2) + half * 8, rr = r0 + r;
    unsigned long long kb = ~0ull;
    if (rr < NR) {
      const float kq = ksq[r];
#pragma unroll
      for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int p = p0 + nh * 64 + j * 8 + (lane & 3) * 2 + e;
          if (p < M0) {
            const float cross = rnd<DT>(acc[j][half * 2 + e]);
            const float dd =
                rnd<DT>(__fsub_rn(rnd<DT>(__fadd_rn(kq, p_sq[(long)h * M0 + p])), rnd<DT>(__fmul_rn(2.f, cross))));
            const unsigned long long key = argmin_key(dd, p);
            kb = key < kb ? key : kb;
          }
        }
    }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, kb, o);
      kb = other < kb ? other : kb;
    }
    if ((lane & 3) == 0 && rr < NR) {
      const int b = rr / Tn, i = rr % Tn;
      atomicMin(best + ((long)b * H + h) * Tn + i, kb);
    }
  }
}

// One CTA per (b,h) (256 threads); the new tokens are processed one after
// another in order.  The parent of each new key comes from
// append_assign_kernel (`best`); without it (fp32, or D not in {64, 128}) the
// CTA scans the parents itself: 8 lanes per parent, the cross term k.p summed
// exactly in fp64.  Children: one warp per child with the products rounded to
// the dtype first (quantizer.py:223-226).  First minimum wins, NaN first
// (torch.argmin).
constexpr int AP_THREADS = 256;

template <int DT>
__global__ void __launch_bounds__(AP_THREADS) append_kernel(
    const typename Storage<DT>::T* __restrict__ knew, Strides3 ks, const typename Storage<DT>::T* __restrict__ vnew,
    Strides3 vs, int H, int Tn, int D, int M0, int C, const typename Storage<DT>::T* __restrict__ parents,
    const float* __restrict__ p_sq, const typename Storage<DT>::T* __restrict__ children,
    const float* __restrict__ c_sq, float* __restrict__ pacc, float* __restrict__ cacc,
    typename Storage<DT>::T* __restrict__ pagg, typename Storage<DT>::T* __restrict__ cagg, int* __restrict__ pcnt,
    int* __restrict__ ccnt, int* __restrict__ nvalid, typename Storage<DT>::T* __restrict__ kpage,
    typename Storage<DT>::T* __restrict__ vpage, Strides3 pgs, int slot0,
    const unsigned long long* __restrict__ best) {
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
    if (tid == 0) bestp_s = best ? (int)(best[(long)g * Tn + i] & 0xffffffffu) : -1;
    if (!best) {
      // parents: group `sub` of warp `warp` takes parents warp*4 + sub + 32*it,
      // two at a time; with 16-bit elements and D a multiple of 64 a lane reads
      // 16-byte chunks l8, l8 + 8, ... of the row (fp32 path and unsupported D)
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
      for (int p0 = warp * 4; p0 < M0; p0 += 2 * (AP_THREADS / 8)) {
        const int pa = p0 + sub, pb = pa + AP_THREADS / 8;
        double acc0 = 0.0, acc1 = 0.0;
        for (int d = l8; d < D; d += 8) {
          const double kd = (double)kk[d];
          if (pa < M0) acc0 = fma(kd, (double)to_f(parents[(ph + pa) * D + d]), acc0);
          if (pb < M0) acc1 = fma(kd, (double)to_f(parents[(ph + pb) * D + d]), acc1);
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

size_t append_workspace_bytes(int B, int H, int Tn) { return (size_t)B * H * (Tn > 0 ? Tn : 1) * 8; }

template <int DT>
int launch_append(const AppendArgs& a, cudaStream_t st) {
  using T = typename Storage<DT>::T;
  const int G = a.B * a.H;
  if (G == 0 || a.Tn == 0) return AVQ_OK;
  if (a.C > 8) return AVQ_ERR_UNSUPPORTED;  // one warp per child
  unsigned long long* best = nullptr;
  const bool tc = DT != DT_F32 && (a.D == 64 || a.D == 128) && a.workspace &&
                  a.workspace_bytes >= append_workspace_bytes(a.B, a.H, a.Tn) && ((uintptr_t)a.k % 16) == 0 &&
                  a.ks.b % 8 == 0 && a.ks.h % 8 == 0 && a.ks.s % 8 == 0;
  if constexpr (DT != DT_F32) {
    if (tc) {
      best = static_cast<unsigned long long*>(a.workspace);
      if (cudaMemsetAsync(best, 0xFF, append_workspace_bytes(a.B, a.H, a.Tn), st) != cudaSuccess) return AVQ_ERR_CUDA;
      const size_t smem = (size_t)(AA_ROWS + AA_COLS) * (a.D + 8) * sizeof(T) + AA_ROWS * sizeof(float);
      AVQ_TIMED("append_assign", st);
      auto go = [&](auto kfn) {
        cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        kfn<<<dim3(a.H, (a.M0 + AA_COLS - 1) / AA_COLS, (a.B * a.Tn + AA_ROWS - 1) / AA_ROWS), 256, smem, st>>>(
            (const T*)a.k, a.ks, a.B, a.H, a.Tn, a.M0, (const T*)a.parents_dt, a.p_sq, best);
      };
      if (a.D == 64) go(append_assign_kernel<DT, 64>);
      else go(append_assign_kernel<DT, 128>);
    }
  }
  const size_t smem = sizeof(float) * a.D;
  AVQ_TIMED("append", st);
  append_kernel<DT><<<G, AP_THREADS, smem, st>>>((const T*)a.k, a.ks, (const T*)a.v, a.vs, a.H, a.Tn, a.D, a.M0, a.C,
                                                 (const T*)a.parents_dt, a.p_sq, (const T*)a.children_dt, a.c_sq,
                                                 a.pacc, a.cacc, (T*)a.pagg, (T*)a.cagg, a.pcnt, a.ccnt, a.nvalid,
                                                 (T*)a.kpage, (T*)a.vpage, a.pgs, a.slot0, best);
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
