// Codeword visibility under a user or causal mask (reference
// pipeline.py:82-106, attention_module.py:210-223, 369-390).
//
// The reference masks parent p for query t when no key assigned to p is
// allowed by the mask: codeword_present = (mask @ one_hot(assign)) > 0, a
// [T, S] x [S, M0] product per (b,h).  Here the same predicate becomes a bit
// per (g, t, p): bit p % 32 of word present[(g T + t) W + p / 32],
// W = ceil(M0 / 32).  The attention kernels test it beside the count mask.
//
//   causal: key j is visible to query t iff j <= t + offset, so parent p is
//       present iff its first key position f_p <= t + offset.  One CTA per
//       (b,h) finds f (shared-memory atomicMin over the assignments), then a
//       warp ballot per (t, word) sets the bits: lane i tests parent 32 w + i.
//   user mask: a warp per query row scans the row's keys (coalesced mask and
//       assignment reads) and ORs the assigned parents' bits into a shared
//       row of words.
#include <climits>

#include "avq_kernels.cuh"

namespace avq {

namespace {

constexpr int PR_THREADS = 256;

__global__ void __launch_bounds__(PR_THREADS) causal_presence_kernel(const int* __restrict__ passign, int S, int M0,
                                                                     int T, int offset, int W, int sG,
                                                                     unsigned int* __restrict__ present) {
  extern __shared__ int first[];  // [M0]
  const int g = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int p = tid; p < M0; p += PR_THREADS) first[p] = INT_MAX;
  __syncthreads();
  const int* pa = passign + (long)(g % sG) * S;
  for (int j = tid; j < S; j += PR_THREADS) atomicMin(&first[pa[j]], j);
  __syncthreads();
  unsigned int* out = present + (long)g * T * W;
  for (int w = warp; w < W; w += PR_THREADS / 32) {
    const int p = 32 * w + lane;
    const long f = p < M0 ? (long)first[p] : (long)INT_MAX + 1;
    for (int t = 0; t < T; ++t) {
      const unsigned int bits = __ballot_sync(0xffffffffu, f <= (long)t + offset);
      if (lane == 0) out[(long)t * W + w] = bits;
    }
  }
}

// One CTA per (group, 8 query rows); mask element (b, h, t, j) at
// b mb + h mh + t mt + j.
__global__ void __launch_bounds__(PR_THREADS) mask_presence_kernel(const int* __restrict__ passign, int H, int S,
                                                                   int T, int W, int sG,
                                                                   const unsigned char* __restrict__ mask,
                                                                   long long mb, long long mh, long long mt,
                                                                   unsigned int* __restrict__ present) {
  extern __shared__ unsigned int words[];  // [8][W]
  const int g = blockIdx.y, b = g / H, h = g % H, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t = blockIdx.x * 8 + warp;
  for (int i = tid; i < 8 * W; i += PR_THREADS) words[i] = 0u;
  __syncthreads();
  if (t < T) {
    const unsigned char* mrow = mask + b * mb + h * mh + t * mt;
    const int* pa = passign + (long)(g % sG) * S;
    unsigned int* row = words + warp * W;
    for (int j = lane; j < S; j += 32)
      if (mrow[j]) {
        const int p = pa[j];
        atomicOr(&row[p >> 5], 1u << (p & 31));
      }
  }
  __syncthreads();
  for (int i = tid; i < 8 * W; i += PR_THREADS) {
    const int r = i / W, w = i % W, tt = blockIdx.x * 8 + r;
    if (tt < T) present[((long)g * T + tt) * W + w] = words[i];
  }
}

}  // namespace

int presence_words(int M0) { return (M0 + 31) / 32; }

int launch_presence(const int* passign, int B, int H, int S, int M0, int T, const unsigned char* mask,
                    const long long* mask_strides, int causal_offset, int sG, unsigned int* present, cudaStream_t st) {
  const int G = B * H, W = presence_words(M0);
  if (G == 0 || T == 0) return AVQ_OK;
  if (S == 0) {  // no keys: no parent is present
    return cudaMemsetAsync(present, 0, (size_t)G * T * W * sizeof(unsigned int), st) == cudaSuccess ? AVQ_OK
                                                                                                     : AVQ_ERR_CUDA;
  }
  if (!mask) {
    AVQ_TIMED("presence", st);
    causal_presence_kernel<<<G, PR_THREADS, (size_t)M0 * sizeof(int), st>>>(passign, S, M0, T, causal_offset, W, sG,
                                                                            present);
  } else {
    const size_t smem = (size_t)8 * W * sizeof(unsigned int);
    AVQ_TIMED("presence", st);
    mask_presence_kernel<<<dim3((T + 7) / 8, G), PR_THREADS, smem, st>>>(passign, H, S, T, W, sG, mask,
                                                                        mask_strides[0], mask_strides[1],
                                                                        mask_strides[2], present);
  }
  return cudaPeekAtLastError() == cudaSuccess ? AVQ_OK : AVQ_ERR_CUDA;
}

}  // namespace avq
