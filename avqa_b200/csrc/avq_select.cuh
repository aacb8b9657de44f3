// Stable top-k of the routing kernels: the `need` smallest of n unique 64-bit
// keys, in ascending order, by one CTA of NT threads.
//
// The routing keys pack (descending importance, NaN first) in the high word
// and the parent index in the low word (route_key), so the k smallest keys in
// ascending order are torch.topk's stable descending selection
// (routing.py:152-170).  A full bitonic sort of n keys costs n log^2 n / 4
// compare-exchanges and a barrier per stage; selecting k << n needs far less:
//
//   1. radix select on the high word, 8 bits per round from the top: a
//      256-bin histogram of the candidates that match the digits fixed so
//      far (warp-aggregated shared atomics), one warp scans it and picks the
//      bin that holds the k-th smallest; after four rounds the boundary value
//      hw* is known, with `less` keys below it and `tie` more wanted among the
//      keys equal to it;
//   2. the keys below hw* are taken, and of the keys equal to it the `tie`
//      smallest indices (the low word), ranked by a prefix popcount over a
//      bitmask of the tied indices;
//   3. the k chosen keys are placed by rank (each counts the chosen keys
//      below it; the keys are unique, so the ranks are a permutation).
//
// Every loop runs the same trip count in every thread of a warp, so the
// warp-collective calls see their whole warp.
#pragma once

#include <cstdint>

namespace avq {

// Largest k for which the routing kernels select instead of sorting every key
// (the rank placement costs k^2 / NT comparisons per thread).
constexpr int SEL_MAX = 256;

// Shared scratch of select_smallest, in 32-bit words, for n keys and k <= kmax
// (an even count, so that a 64-bit array can follow).
__host__ __device__ inline int select_scratch_words(int n, int kmax) {
  const int nw = (n + 31) / 32;
  return 256 + 8 + 2 * nw + 2 * kmax;  // histogram, scalars, tie bits and prefixes, the chosen keys
}

// keys[0, n): unique keys with key i's low word == i (the parent index).
// Writes the k smallest keys, ascending, to out[0, k) (shared or global).
// scratch: select_scratch_words(n, k) words of shared memory, 8-byte aligned.
template <int NT>
__device__ void select_smallest(const unsigned long long* keys, int n, int k, unsigned long long* out,
                                uint32_t* scratch) {
  static_assert(NT % 32 == 0, "whole warps");
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nw = (n + 31) / 32;
  int* hist = reinterpret_cast<int*>(scratch);          // [256]
  int* sc = hist + 256;                                 // [8]: digit, before, count
  uint32_t* tie_bits = scratch + 256 + 8;               // [nw]
  int* tie_pre = reinterpret_cast<int*>(tie_bits + nw);  // [nw]
  unsigned long long* chosen = reinterpret_cast<unsigned long long*>(tie_bits + 2 * nw);  // [k], 8-byte aligned
  if (k <= 0) return;
  uint32_t prefix = 0u, pmask = 0u;
  int remaining = k;
  const int iters = (n + NT - 1) / NT;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += NT) hist[i] = 0;
    __syncthreads();
    for (int it = 0; it < iters; ++it) {
      const int i = it * NT + tid;
      const uint32_t hw = i < n ? (uint32_t)(keys[i] >> 32) : 0u;
      const bool cand = i < n && (hw & pmask) == prefix;
      const uint32_t digit = (hw >> shift) & 255u;
      const uint32_t cmask = __ballot_sync(0xffffffffu, cand);
      if (cand) {
        const uint32_t same = __match_any_sync(cmask, digit);
        if (lane == __ffs(same) - 1) atomicAdd(hist + digit, __popc(same));
      }
    }
    __syncthreads();
    if (warp == 0) {
      int c[8], s = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = hist[lane * 8 + j];
        s += c[j];
      }
      int incl = s;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      int before = incl - s;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (before < remaining && remaining <= before + c[j]) {
          sc[0] = lane * 8 + j;
          sc[1] = before;
        }
        before += c[j];
      }
    }
    __syncthreads();
    const uint32_t d = (uint32_t)sc[0];
    remaining -= sc[1];
    prefix |= d << shift;
    pmask |= 255u << shift;
    __syncthreads();  // sc is rewritten by the next round
  }
  // prefix is the boundary high word; `remaining` keys equal to it are wanted
  if (tid == 0) sc[2] = 0;
  for (int it = 0; it < (nw * 32 + NT - 1) / NT; ++it) {
    const int i = it * NT + tid;
    const bool tie = i < n && (uint32_t)(keys[i] >> 32) == prefix;
    const uint32_t b = __ballot_sync(0xffffffffu, tie);
    if (lane == 0 && (i >> 5) < nw) tie_bits[i >> 5] = b;
  }
  __syncthreads();
  if (warp == 0) {
    int run = 0;
    for (int w0 = 0; w0 < nw; w0 += 32) {
      const int w = w0 + lane;
      const int c = w < nw ? __popc(tie_bits[w]) : 0;
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      if (w < nw) tie_pre[w] = run + incl - c;
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
  }
  __syncthreads();
  for (int i = tid; i < n; i += NT) {
    const unsigned long long key = keys[i];
    const uint32_t hw = (uint32_t)(key >> 32);
    bool take = hw < prefix;
    if (hw == prefix) {
      const int rank = tie_pre[i >> 5] + __popc(tie_bits[i >> 5] & ((1u << (i & 31)) - 1u));
      take = rank < remaining;
    }
    if (take) {
      const int slot = atomicAdd(sc + 2, 1);
      if (slot < k) chosen[slot] = key;  // exactly k are taken; the guard keeps the store in bounds regardless
    }
  }
  __syncthreads();
  for (int j = tid; j < k; j += NT) {
    const unsigned long long key = chosen[j];
    int pos = 0;
    for (int i = 0; i < k; ++i) pos += chosen[i] < key;
    if (pos < k) out[pos] = key;
  }
  __syncthreads();
}

}  // namespace avq
