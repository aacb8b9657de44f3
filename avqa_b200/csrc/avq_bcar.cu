// BCAR online codebook adaptation (reference online_adaptation.py:37-127):
// after a quantization, every child codeword moves toward the mean of the
// keys assigned to it,
//     c' = c + DT(w * DT(mean - c)),  w = DT(fp32(1 - decay)) where the cell
//     received keys, else 0,
// the updated children are averaged over the batch, and every parent becomes
// the mean of its children.  All arithmetic is in the codebook dtype with the
// reference's rounding points:
//   * the cell sums of the keys are exact (fp64 atomics of dtype values; the
//     reference's one-hot einsum sums them exactly in fp32 for bf16 / fp16)
//     and narrowed fp64 -> fp32 -> DT; the count is narrowed to DT;
//   * mean = DT(DT(sum) * DT(1 / DT(count)));
//   * the codebook is tiled over the batch as children.repeat_interleave(B)
//     while the groups are ordered g = b H + h, so group i updates the
//     children of head i / B, and the batch mean reads the groups as
//     view(B, H): head h averages groups b H + h over b (for B > 1 this is the
//     reference's own pairing);
//   * a cell that received no key in any batch keeps its children;
//   * parents = DT(fp32 sum over c / C).
#include "avq_kernels.cuh"

namespace avq {

namespace {

// Cell sums of the keys: a warp per key, a lane per 32 dimensions.
template <int DT>
__global__ void __launch_bounds__(256) bcar_sum_kernel(const typename Storage<DT>::T* __restrict__ keys, Strides3 ks,
                                                       int H, int S, int D, int MC, int C,
                                                       const int* __restrict__ passign,
                                                       const int* __restrict__ cassign, double* __restrict__ sums,
                                                       int* __restrict__ cnts) {
  const int g = blockIdx.y, b = g / H, h = g % H, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int s = blockIdx.x * 8 + warp;
  if (s >= S) return;
  const int cell = passign[(long)g * S + s] * C + cassign[(long)g * S + s];
  const typename Storage<DT>::T* kr = keys + (long)b * ks.b + (long)h * ks.h + (long)s * ks.s;
  double* dst = sums + ((long)g * MC + cell) * D;
  for (int d = lane; d < D; d += 32) atomicAdd(dst + d, (double)to_f(kr[d]));
  if (lane == 0) atomicAdd(cnts + (long)g * MC + cell, 1);
}

// One CTA per (cell, head), a thread per dimension.
template <int DT>
__global__ void bcar_child_kernel(int B, int H, int D, int MC, float w_dt, const double* __restrict__ sums,
                                  const int* __restrict__ cnts, const typename Storage<DT>::T* __restrict__ ch_in,
                                  typename Storage<DT>::T* __restrict__ ch_out) {
  const int cell = blockIdx.x, h = blockIdx.y;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    bool any = false;
    for (int b = 0; b < B; ++b) {
      const int i = b * H + h;  // the group whose update lands in head h's batch mean
      const float src = to_f(ch_in[((long)(i / B) * MC + cell) * D + d]);  // repeat_interleave(B)
      const int n = cnts[(long)i * MC + cell];
      const float sum = rnd64<DT>(sums[((long)i * MC + cell) * D + d]);
      const float inv = n > 0 ? rnd<DT>(__fdiv_rn(1.f, rnd<DT>((float)n))) : 0.f;
      const float mean = rnd<DT>(__fmul_rn(sum, inv));
      const float w = n > 0 ? w_dt : 0.f;
      const float upd = rnd<DT>(__fmul_rn(w, rnd<DT>(__fsub_rn(mean, src))));
      acc = __fadd_rn(acc, rnd<DT>(__fadd_rn(src, upd)));
      any |= n > 0;
    }
    const long o = ((long)h * MC + cell) * D + d;
    ch_out[o] = any ? from_f<DT>(__fdiv_rn(acc, (float)B)) : ch_in[o];
  }
}

// One CTA per (parent, head): parents = DT(fp32 sum of the C children / C).
template <int DT>
__global__ void bcar_parent_kernel(int M0, int C, int D, const typename Storage<DT>::T* __restrict__ ch,
                                   typename Storage<DT>::T* __restrict__ parents) {
  const int p = blockIdx.x, h = blockIdx.y;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int c = 0; c < C; ++c) acc = __fadd_rn(acc, to_f(ch[(((long)h * M0 + p) * C + c) * D + d]));
    parents[((long)h * M0 + p) * D + d] = from_f<DT>(__fdiv_rn(acc, (float)C));
  }
}

}  // namespace

size_t bcar_workspace_bytes(int G, int M0, int C, int D) {
  return align_up((size_t)G * M0 * C * D * sizeof(double)) + align_up((size_t)G * M0 * C * sizeof(int));
}

template <int DT>
int launch_bcar(const void* keys, Strides3 ks, const int* passign, const int* cassign, int B, int H, int S, int D,
                int M0, int C, float decay, const void* ch_in, void* ch_out, void* parents_out, void* workspace,
                cudaStream_t st) {
  using T = typename Storage<DT>::T;
  const int G = B * H, MC = M0 * C;
  double* sums = static_cast<double*>(workspace);
  int* cnts = reinterpret_cast<int*>(static_cast<char*>(workspace) + align_up((size_t)G * MC * D * sizeof(double)));
  if (cudaMemsetAsync(workspace, 0, bcar_workspace_bytes(G, M0, C, D), st) != cudaSuccess) return AVQ_ERR_CUDA;
  // DT(fp32(1 - decay)): the reference multiplies a Python float by a bool tensor
  // (fp32), then casts to the codebook dtype
  float w_dt;
  {
    const float w32 = (float)(1.0 - (double)decay);
    if (DT == DT_BF16) w_dt = __bfloat162float(__float2bfloat16_rn(w32));
    else if (DT == DT_F16) w_dt = __half2float(__float2half_rn(w32));
    else w_dt = w32;
  }
  const int th = D < 256 ? ((D + 31) / 32) * 32 : 256;
  {
    AVQ_TIMED("bcar", st);
    if (S > 0 && G > 0)
      bcar_sum_kernel<DT><<<dim3((S + 7) / 8, G), 256, 0, st>>>(static_cast<const T*>(keys), ks, H, S, D, MC, C,
                                                                 passign, cassign, sums, cnts);
    bcar_child_kernel<DT><<<dim3(MC, H), th, 0, st>>>(B, H, D, MC, w_dt, sums, cnts, static_cast<const T*>(ch_in),
                                                      static_cast<T*>(ch_out));
    bcar_parent_kernel<DT><<<dim3(M0, H), th, 0, st>>>(M0, C, D, static_cast<const T*>(ch_out),
                                                       static_cast<T*>(parents_out));
  }
  return cudaPeekAtLastError() == cudaSuccess ? AVQ_OK : AVQ_ERR_CUDA;
}

template int launch_bcar<DT_F32>(const void*, Strides3, const int*, const int*, int, int, int, int, int, int, float,
                                 const void*, void*, void*, void*, cudaStream_t);
template int launch_bcar<DT_BF16>(const void*, Strides3, const int*, const int*, int, int, int, int, int, int, float,
                                  const void*, void*, void*, void*, cudaStream_t);
template int launch_bcar<DT_F16>(const void*, Strides3, const int*, const int*, int, int, int, int, int, int, float,
                                 const void*, void*, void*, void*, cudaStream_t);

}  // namespace avq
