// Streaming VQ (reference streaming_vq.py:109-229, StreamingVQBuffer.extend):
// a batch of B new keys [B, D] -- the same keys for every head -- is assigned
// to the per-head codebook, and the keys are added to running per-codeword
// sums and counts.
//
//   stream_parent : distance DT(DT(k_sq - DT(2 DT(k.p))) + p_sq) in that
//                   order (:172-177); the dot products accumulate in double,
//                   so each term is the exactly rounded value; first argmin
//                   over parents (a NaN wins) via a 64-bit atomicMin of
//                   (order key, index) per (b, h).  A thread per parent, a CTA
//                   per (128 parents, head, 8 keys), so a single key still
//                   spreads the codebook read over the SMs.
//   stream_child  : DT(sum DT(DT(k - c)^2)) over the assigned parent's
//                   children (:183-188), first argmin; writes the [B, H]
//                   int64 results and appends them to the running record,
//                   which the reference lays out as assign.reshape(1, H, B):
//                   flat result i goes to record row i / B, column size + i % B.
//                   With one key per call it also does the aggregation below
//                   (each head then has exactly one row).
//   stream_aggregate : index_add_ of the keys (:191-213).  Row i of the flat
//                   [B*H] order adds key i / H to head i / B
//                   (arange(H).repeat_interleave(B)) at codeword
//                   assign.reshape(-1)[i].  torch's CPU index_add_ accumulates
//                   the rows of one call in fp32, in row order, starting from
//                   the stored value, and narrows once: one CTA per
//                   (destination head, parent | child) groups its B rows by
//                   codeword and a warp sums each group in row order.  Counts
//                   are exact int64.
#include "avq_kernels.cuh"

namespace avq {

namespace {

constexpr int SP_KEYS = 8;      // keys per CTA
constexpr int SP_THREADS = 128;  // parents per CTA: one thread per parent
constexpr int SP_CHUNK = 32;     // dimensions per register chunk of a parent row
constexpr int ST_MAX_D = 512;

// (order key, index) for a 64-bit atomicMin: the smallest distance, then the
// smallest index; a NaN distance sorts below every number (torch.argmin).
__device__ __forceinline__ unsigned long long argmin_key(float d, int i) {
  const uint32_t k = isnan(d) ? 0u : float_order_key(__fadd_rn(d, 0.f));  // -0 -> +0
  return ((unsigned long long)k << 32) | (uint32_t)i;
}

// One thread per parent: the parent row streams through registers in
// 32-element chunks (16-byte loads, all issued before use), the dot products
// with the CTA's keys (shared memory, read as broadcasts) accumulate in
// double, so no cross-lane reduction is needed per parent; the per-key
// minimum goes through one warp reduction and one atomicMin per warp.
template <int DT>
__global__ void __launch_bounds__(SP_THREADS) stream_parent_kernel(const typename Storage<DT>::T* __restrict__ keys,
                                                                   long long kstride, int B, int M0, int D,
                                                                   const typename Storage<DT>::T* __restrict__ parents,
                                                                   unsigned long long* __restrict__ best, int H) {
  using T = typename Storage<DT>::T;
  constexpr int EW = 16 / sizeof(T);  // elements per 16-byte load
  __shared__ double kk[SP_KEYS][ST_MAX_D];  // held as double: one conversion per key element, not per product
  __shared__ float ksq[SP_KEYS];
  const int h = blockIdx.y, p = blockIdx.x * SP_THREADS + threadIdx.x, b0 = blockIdx.z * SP_KEYS;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nk = min(SP_KEYS, B - b0);
  for (int e = tid; e < SP_KEYS * D; e += blockDim.x) {
    const int r = e / D, d = e % D;
    kk[r][d] = r < nk ? (double)to_f(keys[(long long)(b0 + r) * kstride + d]) : 0.0;
  }
  __syncthreads();
  for (int r = warp; r < nk; r += SP_THREADS / 32) {  // k_sq = (keys * keys).sum(1), narrowed once
    double acc = 0.0;
    for (int d = lane; d < D; d += 32) {
      const float kv = (float)kk[r][d];
      acc += (double)rnd<DT>(__fmul_rn(kv, kv));
    }
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) ksq[r] = rnd64<DT>(acc);
  }
  __syncthreads();
  const bool live = p < M0;
  double psq = 0.0, acc[SP_KEYS];
#pragma unroll
  for (int r = 0; r < SP_KEYS; ++r) acc[r] = 0.0;
  const T* prow = parents + ((long long)h * M0 + (live ? p : 0)) * D;
  // 16-byte loads when every row starts on a 16-byte boundary
  const bool vec = D % EW == 0 && (reinterpret_cast<uintptr_t>(parents) & 15u) == 0u;
  for (int d0 = 0; d0 < D; d0 += SP_CHUNK) {
    T pc[SP_CHUNK];
    if (vec) {
      uint4 raw[SP_CHUNK / EW];
#pragma unroll
      for (int i = 0; i < SP_CHUNK / EW; ++i)
        raw[i] = (live && d0 + i * EW < D) ? *reinterpret_cast<const uint4*>(prow + d0 + i * EW)
                                           : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int i = 0; i < SP_CHUNK / EW; ++i)
#pragma unroll
        for (int e = 0; e < EW; ++e) pc[i * EW + e] = reinterpret_cast<const T*>(&raw[i])[e];
    } else {
#pragma unroll
      for (int e = 0; e < SP_CHUNK; ++e) pc[e] = (live && d0 + e < D) ? prow[d0 + e] : prow[0];
    }
#pragma unroll
    for (int e = 0; e < SP_CHUNK; ++e) {
      const int d = d0 + e;
      if (d < D) {
        const float pv = to_f(pc[e]);
        const double pvd = (double)pv;
        psq += (double)rnd<DT>(__fmul_rn(pv, pv));
#pragma unroll
        for (int r = 0; r < SP_KEYS; ++r)
          if (r < nk) acc[r] = fma(kk[r][d], pvd, acc[r]);
      }
    }
  }
  const float p_sq = rnd64<DT>(psq);
#pragma unroll
  for (int r = 0; r < SP_KEYS; ++r) {
    if (r < nk) {
      unsigned long long key = ~0ull;
      if (live) {
        const float cross = rnd64<DT>(acc[r]);
        const float two = rnd<DT>(__fmul_rn(2.f, cross));
        const float t1 = rnd<DT>(__fsub_rn(ksq[r], two));
        key = argmin_key(rnd<DT>(__fadd_rn(t1, p_sq)), p);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other < key ? other : key;
      }
      if (lane == 0 && key != ~0ull) atomicMin(best + (long long)(b0 + r) * H + h, key);
    }
  }
}

// A warp per flat result i = b H + h: the child argmin over the assigned
// parent's children (their rows loaded before any is used), the [B, H]
// outputs and the record.  FUSED (one key per call): row i = h is then the
// only row of head h, so the warp also adds the key to its parent and child
// sums (fp32 sum of the stored value and the key, narrowed once) and counts.
// PER: key elements per lane (D <= 32 PER).
template <int DT, bool FUSED, int PER>
__global__ void __launch_bounds__(256) stream_child_kernel(const typename Storage<DT>::T* __restrict__ keys,
                                                           long long kstride, int B, int H, int M0, int C, int D,
                                                           const typename Storage<DT>::T* __restrict__ children,
                                                           const unsigned long long* __restrict__ best,
                                                           long long* __restrict__ pout, long long* __restrict__ cout_,
                                                           long long* __restrict__ prec, long long* __restrict__ crec,
                                                           long long rec_stride, long long rec_size,
                                                           typename Storage<DT>::T* __restrict__ pagg,
                                                           typename Storage<DT>::T* __restrict__ cagg,
                                                           long long* __restrict__ pcnt, long long* __restrict__ ccnt) {
  constexpr int CMAX = 4;  // children per batch of row loads
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long i = (long long)blockIdx.x * 8 + warp;  // flat [B, H] index
  if (i >= (long long)B * H) return;
  const int b = (int)(i / H), h = (int)(i % H);
  const int p = (int)(uint32_t)(best[i] & 0xffffffffu);
  const typename Storage<DT>::T* krow = keys + (long long)b * kstride;
  float kv[PER];
#pragma unroll
  for (int e = 0; e < PER; ++e) kv[e] = lane + 32 * e < D ? to_f(krow[lane + 32 * e]) : 0.f;
  float bv = 0.f;
  int bi = -1;
  for (int c0 = 0; c0 < C; c0 += CMAX) {
    double acc[CMAX];
    float cv[CMAX][PER];
#pragma unroll
    for (int c = 0; c < CMAX; ++c) {
      const typename Storage<DT>::T* crow = children + (((long long)h * M0 + p) * C + (c0 + c < C ? c0 + c : 0)) * D;
#pragma unroll
      for (int e = 0; e < PER; ++e) cv[c][e] = (c0 + c < C && lane + 32 * e < D) ? to_f(crow[lane + 32 * e]) : 0.f;
    }
#pragma unroll
    for (int c = 0; c < CMAX; ++c) {
      acc[c] = 0.0;
#pragma unroll
      for (int e = 0; e < PER; ++e)
        if (lane + 32 * e < D) {
          const float df = rnd<DT>(__fsub_rn(kv[e], cv[c][e]));
          acc[c] += (double)rnd<DT>(__fmul_rn(df, df));
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int c = 0; c < CMAX; ++c) acc[c] += __shfl_xor_sync(0xffffffffu, acc[c], o);
#pragma unroll
    for (int c = 0; c < CMAX; ++c) {
      if (c0 + c < C) {
        const float v = rnd64<DT>(acc[c]);
        // first minimum; a NaN wins over every number (and the first NaN stays)
        const bool take = bi < 0 || (isnan(v) ? !isnan(bv) : (!isnan(bv) && v < bv));
        if (take) {
          bv = v;
          bi = c0 + c;
        }
      }
    }
  }
  if (lane == 0) {
    pout[i] = p;
    cout_[i] = bi;
    if (prec) {
      const long long r = i / B, j = i % B;
      prec[r * rec_stride + rec_size + j] = p;
      crec[r * rec_stride + rec_size + j] = bi;
    }
  }
  if constexpr (FUSED) {
    typename Storage<DT>::T* pa = pagg + ((long long)h * M0 + p) * D;
    typename Storage<DT>::T* ca = cagg + (((long long)h * M0 + p) * C + bi) * D;
#pragma unroll
    for (int e = 0; e < PER; ++e) {
      const int d = lane + 32 * e;
      if (d < D) {
        pa[d] = from_f<DT>(__fadd_rn(to_f(pa[d]), kv[e]));
        ca[d] = from_f<DT>(__fadd_rn(to_f(ca[d]), kv[e]));
      }
    }
    if (lane == 0) {
      pcnt[(long long)h * M0 + p] += 1;
      ccnt[((long long)h * M0 + p) * C + bi] += 1;
    }
  }
}

// One CTA per (destination head hd, kind): kind 0 adds into the parent sums
// [H, M0, D] / counts [H, M0], kind 1 into the child sums [H, M0*C, D] /
// counts [H, M0*C].  Rows i = hd*B + j, j = 0..B-1.
//   1. tab[dest_j] = j for every row (racing stores: each codeword's slot
//      ends up holding one of its rows), lead = INT_MAX, last = -1;
//   2. rep_j = tab[dest_j] names row j's group; lead / last = min / max row;
//   3. the group's first row's warp walks rows lead..last in order (ballot
//      over 32 rows at a time), summing the members' keys in fp32 from the
//      stored value, then narrows once and adds the member count.
template <int DT>
__global__ void __launch_bounds__(256) stream_aggregate_kernel(
    const typename Storage<DT>::T* __restrict__ keys, long long kstride, int B, int H, int M0, int C, int D,
    const long long* __restrict__ pout, const long long* __restrict__ cout_, typename Storage<DT>::T* __restrict__ pagg,
    typename Storage<DT>::T* __restrict__ cagg, long long* __restrict__ pcnt, long long* __restrict__ ccnt,
    int* __restrict__ tab_p, int* __restrict__ tab_c, int* __restrict__ rows) {
  using T = typename Storage<DT>::T;
  const int hd = blockIdx.x, kind = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nwarps = blockDim.x >> 5;
  const long long nd = kind ? (long long)M0 * C : (long long)M0;  // codewords per head
  int* tab = kind ? tab_c + (long long)hd * nd : tab_p + (long long)hd * nd;
  int* rep = rows + ((long long)(kind * H + hd) * 3) * B;
  int* lead = rep + B;
  int* last = lead + B;
  T* agg = (kind ? cagg : pagg) + (long long)hd * nd * D;
  long long* cnt = (kind ? ccnt : pcnt) + (long long)hd * nd;
  const long long i0 = (long long)hd * B;
  auto dest = [&](int j) -> long long {
    const long long p = pout[i0 + j];
    return kind ? p * C + cout_[i0 + j] : p;
  };
  for (int j = tid; j < B; j += blockDim.x) {
    tab[dest(j)] = j;
    lead[j] = INT_MAX;
    last[j] = -1;
  }
  __syncthreads();
  for (int j = tid; j < B; j += blockDim.x) {
    const int r = tab[dest(j)];
    rep[j] = r;
    atomicMin(lead + r, j);
    atomicMax(last + r, j);
  }
  __syncthreads();
  constexpr int PER = ST_MAX_D / 32;
  for (int j = warp; j < B; j += nwarps) {
    const int r = rep[j];
    if (lead[r] != j) continue;
    const long long dj = dest(j);
    T* arow = agg + dj * D;
    float acc[PER];
#pragma unroll
    for (int e = 0; e < PER; ++e) acc[e] = (lane + 32 * e < D) ? to_f(arow[lane + 32 * e]) : 0.f;
    int members = 0;
    const int end = last[r];
    for (int base = j; base <= end; base += 32) {
      const int jj = base + lane;
      unsigned int m = __ballot_sync(0xffffffffu, jj <= end && rep[jj] == r);
      members += __popc(m);
      while (m) {
        const int s = __ffs(m) - 1;
        m &= m - 1;
        const T* krow = keys + ((i0 + base + s) / H) * kstride;  // key (hd*B + row) / H
#pragma unroll
        for (int e = 0; e < PER; ++e)
          if (lane + 32 * e < D) acc[e] = __fadd_rn(acc[e], to_f(krow[lane + 32 * e]));
      }
    }
#pragma unroll
    for (int e = 0; e < PER; ++e)
      if (lane + 32 * e < D) arow[lane + 32 * e] = from_f<DT>(acc[e]);
    if (lane == 0) cnt[dj] += members;
  }
}

}  // namespace

int stream_max_head_dim() { return ST_MAX_D; }

size_t stream_workspace_bytes(int B, int H, int M0, int C) {
  return align_up((size_t)B * H * sizeof(unsigned long long)) + align_up((size_t)H * M0 * sizeof(int)) +
         align_up((size_t)H * M0 * C * sizeof(int)) + align_up((size_t)2 * H * 3 * B * sizeof(int));
}

template <int DT>
int launch_stream_extend(const void* keys, long long kstride, int B, int H, int M0, int C, int D, const void* parents,
                         const void* children, long long* pout, long long* cout_, long long* prec, long long* crec,
                         long long rec_stride, long long rec_size, long long* pcnt, long long* ccnt, void* pagg,
                         void* cagg, void* workspace, cudaStream_t st) {
  using T = typename Storage<DT>::T;
  if (B == 0) return AVQ_OK;
  char* w = static_cast<char*>(workspace);
  auto* best = reinterpret_cast<unsigned long long*>(w);
  w += align_up((size_t)B * H * sizeof(unsigned long long));
  int* tab_p = reinterpret_cast<int*>(w);
  w += align_up((size_t)H * M0 * sizeof(int));
  int* tab_c = reinterpret_cast<int*>(w);
  w += align_up((size_t)H * M0 * C * sizeof(int));
  int* rows = reinterpret_cast<int*>(w);
  if (cudaMemsetAsync(best, 0xff, (size_t)B * H * sizeof(unsigned long long), st) != cudaSuccess)
    return AVQ_ERR_CUDA;
  const T* k = static_cast<const T*>(keys);
  {
    AVQ_TIMED("stream_parent", st);
    stream_parent_kernel<DT><<<dim3((M0 + SP_THREADS - 1) / SP_THREADS, H, (B + SP_KEYS - 1) / SP_KEYS), SP_THREADS, 0,
                               st>>>(
        k, kstride, B, M0, D, static_cast<const T*>(parents), best, H);
  }
  {
    AVQ_TIMED("stream_child", st);
    const long long rows_bh = (long long)B * H;
    auto kfn = D <= 128 ? (B == 1 ? stream_child_kernel<DT, true, 4> : stream_child_kernel<DT, false, 4>)
                        : (B == 1 ? stream_child_kernel<DT, true, ST_MAX_D / 32>
                                  : stream_child_kernel<DT, false, ST_MAX_D / 32>);
    kfn<<<(unsigned)((rows_bh + 7) / 8), 256, 0, st>>>(k, kstride, B, H, M0, C, D, static_cast<const T*>(children),
                                                       best, pout, cout_, prec, crec, rec_stride, rec_size,
                                                       static_cast<T*>(pagg), static_cast<T*>(cagg), pcnt, ccnt);
  }
  if (B > 1) {
    AVQ_TIMED("stream_aggregate", st);
    stream_aggregate_kernel<DT><<<dim3(H, 2), 256, 0, st>>>(k, kstride, B, H, M0, C, D, pout, cout_,
                                                             static_cast<T*>(pagg), static_cast<T*>(cagg), pcnt, ccnt,
                                                             tab_p, tab_c, rows);
  }
  return cudaPeekAtLastError() == cudaSuccess ? AVQ_OK : AVQ_ERR_CUDA;
}

#define AVQ_STREAM_INST(DT)                                                                                         \
  template int launch_stream_extend<DT>(const void*, long long, int, int, int, int, int, const void*, const void*,  \
                                        long long*, long long*, long long*, long long*, long long, long long,       \
                                        long long*, long long*, void*, void*, void*, cudaStream_t);
AVQ_STREAM_INST(DT_F32)
AVQ_STREAM_INST(DT_BF16)
AVQ_STREAM_INST(DT_F16)
#undef AVQ_STREAM_INST

}  // namespace avq
