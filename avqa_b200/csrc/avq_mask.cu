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
//       present iff its first key position f_p <= t + offset.  A first kernel
//       finds f per key set (global atomicMin over the assignments, S spread
//       over many CTAs); the second writes the bits, one CTA per (b,h) and 64
//       queries: a warp takes a query row, lane i tests parent 32 w + i of
//       word w (one ballot per word), and lane w % 32 stores the word, so a
//       row's words go out in whole 128-byte pieces.
//   user mask: a warp per query row scans the row's keys (coalesced mask and
//       assignment reads) and ORs the assigned parents' bits into a shared
//       row of words.
#include <climits>

#include "avq_kernels.cuh"

namespace avq {

namespace {

constexpr int PR_THREADS = 256;

constexpr int CP_ROWS = 64;      // query rows per bits CTA
constexpr int FK_KEYS = 4096;    // keys per first-position CTA

// first[gs * M0 + p] = min over keys j of key set gs assigned to p (INT_MAX
// when none; the buffer starts at INT_MAX).
__global__ void __launch_bounds__(PR_THREADS) first_key_kernel(const int* __restrict__ passign, int S, int M0,
                                                               int* __restrict__ first) {
  const int gs = blockIdx.y, j0 = blockIdx.x * FK_KEYS;
  const int* pa = passign + (long)gs * S;
  const int j1 = min(S, j0 + FK_KEYS);
  for (int j = j0 + threadIdx.x; j < j1; j += PR_THREADS) atomicMin(first + (long)gs * M0 + pa[j], j);
}

__global__ void __launch_bounds__(PR_THREADS) causal_bits_kernel(const int* __restrict__ first, int M0, int T,
                                                                 int offset, int W, int sG,
                                                                 unsigned int* __restrict__ present) {
  extern __shared__ int fs[];  // [W * 32] first positions of this key set, INT_MAX past M0
  const int g = blockIdx.y, t0 = blockIdx.x * CP_ROWS, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int* f = first + (long)(g % sG) * M0;
  for (int p = tid; p < W * 32; p += PR_THREADS) fs[p] = p < M0 ? f[p] : INT_MAX;
  __syncthreads();
  for (int r = warp; r < CP_ROWS; r += PR_THREADS / 32) {
    const int t = t0 + r;
    if (t >= T) break;
    const long lim = (long)t + offset;
    unsigned int* out = present + ((long)g * T + t) * W;
    for (int w0 = 0; w0 < W; w0 += 32) {
      unsigned int mine = 0u;
      const int nw = min(32, W - w0);
      for (int i = 0; i < nw; ++i) {
        const unsigned int bits = __ballot_sync(0xffffffffu, (long)fs[32 * (w0 + i) + lane] <= lim);
        if (lane == i) mine = bits;
      }
      if (lane < nw) out[w0 + lane] = mine;
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

// The causal path's first key position per (key set, parent).
size_t presence_workspace_bytes(int sG, int M0) { return align_up((size_t)sG * M0 * sizeof(int)); }

int launch_presence(const int* passign, int B, int H, int S, int M0, int T, const unsigned char* mask,
                    const long long* mask_strides, int causal_offset, int sG, unsigned int* present, void* scratch,
                    cudaStream_t st) {
  const int G = B * H, W = presence_words(M0);
  if (G == 0 || T == 0) return AVQ_OK;
  if (S == 0) {  // no keys: no parent is present
    return cudaMemsetAsync(present, 0, (size_t)G * T * W * sizeof(unsigned int), st) == cudaSuccess ? AVQ_OK
                                                                                                     : AVQ_ERR_CUDA;
  }
  if (!mask) {
    int* first = static_cast<int*>(scratch);
    if (cudaMemsetAsync(first, 0x7F, (size_t)sG * M0 * sizeof(int), st) != cudaSuccess) return AVQ_ERR_CUDA;
    AVQ_TIMED("presence", st);
    first_key_kernel<<<dim3((S + FK_KEYS - 1) / FK_KEYS, sG), PR_THREADS, 0, st>>>(passign, S, M0, first);
    causal_bits_kernel<<<dim3((T + CP_ROWS - 1) / CP_ROWS, G), PR_THREADS, (size_t)W * 32 * sizeof(int), st>>>(
        first, M0, T, causal_offset, W, sG, present);
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
