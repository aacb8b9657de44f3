// Key -> parent -> child assignment on the sm_100a tensor cores for bf16 /
// fp16 and D in {64, 128} (reference quantizer.py:166-226).
//
// CTA = 128 keys of one (b,h); thread r of warps 0-3 owns key r (TMEM lane r);
// warp 4 issues tcgen05.mma, warp 5 streams the key tile and 64- or
// 128-parent chunks of the head's codebook with TMA.  TMEM holds two buffers
// of fp32 cross terms K P_c^T, one column per parent of a chunk.
//
// Parent distance (quantizer.py:207-210), each op rounded to the dtype:
//   d = DT(DT(k_sq + p_sq) - DT(2 * DT(k . p)))
// computed with packed dtype x2 arithmetic: for dtype operands the exact sum
// or difference either fits fp32 or is dominated by one operand, so a single
// dtype rounding equals the reference's fp32-then-dtype rounding.
// torch.argmin (first minimum, NaN wins) becomes a signed min over 32-bit
// keys: the order-preserving integer form of the 16-bit distance in the high
// half and the parent index in the low half.  A row with a NaN
// distance (only possible with non-finite inputs) takes a scalar path.
// Child stage (quantizer.py:218-226): a later kernel, once the keys are sorted
// by parent (child_bucket_kernel); the cross term is a sum of dtype-rounded
// elementwise products, rounded once as its exact value would be (fp32 with
// an error bound, fp64 where the bound cannot decide).
#include <cuda.h>

#include <algorithm>

#include "avq_kernels.cuh"
#include "avq_mma.cuh"
#include "avq_tc.cuh"

namespace avq {

namespace {
// Bit 0: a CTA of this file gave up on a bounded wait.
__device__ int g_fault;
}  // namespace

namespace {

constexpr int AR = 128;        // keys per CTA
// parents per chunk: 64 (two 64-column TMEM buffers, three CTAs per SM) up to
// A_SMALL_M0 parents, else 128 (two 128-column buffers, two CTAs per SM: half
// as many chunk hand-overs for a large codebook)
constexpr int A_SMALL_M0 = 1024;
constexpr int ATHREADS = 192;  // 4 row warps + MMA warp + TMA warp
constexpr int A_MAX_M0 = 4096;
constexpr int A_MAX_C = 8;           // children per parent on this path

constexpr int AB_K = 0, AB_PFULL = 1, AB_PEMPTY = 3, AB_SFULL = 5, AB_SCONS = 7, AB_END = 9, AN_BARS = 10;

struct AssignLayout {
  int k, p[2], ps2, bars, misc, total;
};

__host__ __device__ inline AssignLayout assign_layout(int D, int M0, int ACH) {
  AssignLayout L;
  const int nch = (M0 + ACH - 1) / ACH;
  int o = 0;
  L.k = o;
  o += AR * D * 2;
  for (int i = 0; i < 2; ++i) {
    L.p[i] = o;
    o += ACH * D * 2;
  }
  L.ps2 = o;
  o += nch * (ACH / 2) * 4;
  L.bars = o;
  o += AN_BARS * 8;
  L.misc = o;
  o += 32;  // TMEM slot, abort flag, per-warp maxima of the parent norms
  L.total = o;
  return L;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

template <int DT>
__device__ __forceinline__ uint32_t hfma2_dt(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  if (DT == DT_BF16) asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  else asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

// A quarter of the dtype's largest finite value.
template <int DT>
struct DtQuarterMax {
  static constexpr float v = DT == DT_F16 ? 16376.f : 0x1.FEp125f;
};

template <int DT>
__device__ __forceinline__ uint32_t hadd2_dt(uint32_t a, uint32_t b) {
  uint32_t r;
  if (DT == DT_BF16) asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  else asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Both halves of a dtype x2 word mapped to order-preserving signed 16-bit
// integers (negative values: magnitude bits flipped).
__device__ __forceinline__ uint32_t order2(uint32_t d2) {
  const uint32_t neg = prmt(d2, 0u, 0xBB99u);  // 0xFFFF in each half whose sign bit is set
  return d2 ^ (neg & 0x7FFF7FFFu);
}

__device__ __forceinline__ int key_lo(uint32_t k2, uint32_t idx2) { return (int)prmt(k2, idx2, 0x1054u); }
__device__ __forceinline__ int key_hi(uint32_t k2, uint32_t idx2) { return (int)prmt(k2, idx2, 0x3276u); }

__device__ __forceinline__ void drain(uint64_t* bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!tc::mbar_try(bar, parity) && clock64() - t0 < tc::kWaitCycles / 8) {
  }
}

// Bound on sum_d |DT(k_d c_d)| from the dtype norms: |k_d c_d| <= (k_d^2 +
// c_d^2) / 2, and k_sq, c_sq are the once-rounded exact sums of the dtype
// squares, so sum_d k_d^2 <= k_sq (1 + 2.1 u) + D eta (u the dtype's unit
// roundoff, eta half its smallest subnormal).  Scaled by 2^-21 >= gamma_7:
//   err <= 2^-21 * (0.52 (k_sq + c_sq) + 4 D eta).
template <int DT>
struct ChildBound {
  static constexpr float scale = 0.52f * 0x1p-21f;
  static constexpr float slack = DT == DT_F16 ? 0x1p-36f : 0x1p-140f;  // >= 2^-21 * 4 * 128 * eta
};

// Child assignment in bucket order (quantizer.py:218-227), after the parent
// pass and the counting sort by parent: a warp takes 32 consecutive keys of
// the sorted order of one (b,h), so neighbouring keys mostly share their
// parent and its C child rows (one contiguous block) are read from L2 once
// for many keys instead of once per key.  Each key's dtype k_sq comes from
// the parent pass, parked in the key's cassign word as float bits, and is
// overwritten by the key's child index here.
//
// A key's child rows are spread over the warp R = 32/G rows at a time (NP
// passes of R rows), G lanes to a row, lane (rsub, vg) holding the 16-byte
// chunks vg + G*t (t < NV) of row ps*R + rsub in pass ps; the warp takes its
// keys four at a time.
//
// cross = DT(fp32(sum_d DT(k_d c_d))) with the sum exact (what the fp64 sum
// of the dtype products gives) is evaluated in fp32: each lane sums its 8*NV
// products pairwise and the row's G lanes combine by butterfly, a tree of
// depth 3 + log2(NV*G) <= 7, so the fp32 result S' lies within
// gamma_7 * sum|t| of the exact sum, bounded by ChildBound.  fp32 and dtype
// rounding are monotone, so when both ends of [S' - b, S' + b] (rounded
// outwards) round to the same dtype value that value is the exact sum's
// rounding; otherwise (close to a dtype rounding boundary, or non-finite)
// the row is summed again in fp64.  The row's lanes reduce-scatter the four
// keys' sums, so each lane finishes one key: the rounding test, the distance
// and the argmin run once per lane, not once per key.  torch.argmin over the
// children (first minimum, a NaN wins) is a signed min over 32-bit keys: the
// order-preserving integer form of the distance, whose low 13 bits are zero
// for dtype values, or'ed with the child index.
constexpr int CB_WARPS = 8;  // warps per CTA of the child kernel

template <int DT, int D, int NV, int NP>
__global__ void __launch_bounds__(CB_WARPS * 32, NP > 1 ? 2 : 3) child_bucket_kernel(
    const typename Storage<DT>::T* __restrict__ keys, Strides3 ks, int H, int S, int M0, int C,
    const int* __restrict__ order, const int* __restrict__ passign, const typename Storage<DT>::T* __restrict__ children,
    const float* __restrict__ c_sq, int* __restrict__ cassign) {
  using T = typename Storage<DT>::T;
  constexpr int CPR = D / 8, G = CPR / NV, KP = 4, NGRP = 32 / KP;
  static_assert(G >= KP && G % KP == 0 && 32 % G == 0, "lanes per row");
  constexpr int R = 32 / G;       // child rows per pass
  constexpr int CQ = R * NP;      // the largest C this split serves
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = blockIdx.y, b = g / H, h = g % H;
  const int i0 = (blockIdx.x * CB_WARPS + warp) * 32;
  if (i0 >= S) return;  // whole warps leave together
  const int vg = lane % G, rsub = lane / G;
  const bool hb1 = (vg & (G / 2)) != 0, hb2 = (vg & (G / 4)) != 0;
  const int kq = (hb1 ? 2 : 0) + (hb2 ? 1 : 0);  // the key of the group this lane finishes
  // this lane's own key: sorted position i0 + lane
  const bool live = i0 + lane < S;
  const int s_mine = live ? order[(long)g * S + i0 + lane] : 0;
  const int p_mine = live ? passign[(long)g * S + s_mine] : 0;
  const float ksq_mine = live ? __int_as_float(cassign[(long)g * S + s_mine]) : 0.f;
  float cq[CQ];  // the lane's key's child norms; the finishing lanes take them by shuffle
#pragma unroll
  for (int c = 0; c < CQ; ++c) cq[c] = live && c < C ? c_sq[((long)h * M0 + p_mine) * C + c] : 0.f;
  const T* kbase = keys + (long)b * ks.b + (long)h * ks.h;
  const T* cbase = children + (long)h * M0 * C * D;
  // the warp's 32 key rows, staged in shared memory at once (one gather
  // latency for the warp instead of one per group of four)
  extern __shared__ __align__(16) unsigned char cb_smem[];
  unsigned char* krows = cb_smem + warp * 32 * D * 2;
#pragma unroll
  for (int c = 0; c < CPR; ++c)
    cp_async16(krows + lane * D * 2 + 16 * c, kbase + (long)s_mine * ks.s + 8 * c, live);
  cp_async_commit();
  auto key_chunk = [&](int j, int t) -> uint4 {  // chunk vg + G t of the warp's key j
    return *reinterpret_cast<const uint4*>(krows + j * D * 2 + 16 * (vg + G * t));
  };
  cp_async_wait<0>();
  __syncwarp();
  // the child rows of the parent in hand, reloaded only where the sorted keys
  // move on to the next parent (warp-uniform)
  auto blk_chunk = [&](int p, int ps, int t) -> uint4 {
    const int crow = ps * R + rsub;
    return crow < C ? *reinterpret_cast<const uint4*>(cbase + ((long)p * C + crow) * D + 8 * (vg + G * t))
                    : make_uint4(0u, 0u, 0u, 0u);
  };
  int cur_p = -1;
  uint4 wc[NP][NV];
  int mine = 0;
#pragma unroll 1
  for (int gq = 0; gq < NGRP; ++gq) {
    if (i0 + gq * KP >= S) break;  // warp-uniform
    int pk[KP];
#pragma unroll
    for (int kk = 0; kk < KP; ++kk) pk[kk] = __shfl_sync(full, p_mine, gq * KP + kk);  // 0 past S
    const float ksk = __shfl_sync(full, ksq_mine, gq * KP + kq);
    float sxa[NP][KP];
#pragma unroll
    for (int kk = 0; kk < KP; ++kk) {
      if (pk[kk] != cur_p) {
        cur_p = pk[kk];
#pragma unroll
        for (int ps = 0; ps < NP; ++ps)
#pragma unroll
          for (int t = 0; t < NV; ++t) wc[ps][t] = blk_chunk(cur_p, ps, t);
      }
#pragma unroll
      for (int ps = 0; ps < NP; ++ps) {
        float2 acc[NV * 4];
#pragma unroll
        for (int t = 0; t < NV; ++t) {
          const uint4 u = key_chunk(gq * KP + kk, t), w = wc[ps][t];
          const uint32_t ku[4] = {u.x, u.y, u.z, u.w}, cw[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const uint32_t pr = hmul2_dt<DT>(ku[e], cw[e]);  // DT(k_d * c_d)
            acc[4 * t + e] = make_float2(half_lo<DT>(pr), half_hi<DT>(pr));
          }
        }
#pragma unroll
        for (int st = 1; st < NV * 4; st <<= 1)
#pragma unroll
          for (int i = 0; i + st < NV * 4; i += 2 * st) acc[i] = add_f32x2(acc[i], acc[i + st]);
        sxa[ps][kk] = acc[0].x + acc[0].y;
      }
    }
    int best = 0x7FFFFFFF;  // over the passes: the key of this lane's key kq
#pragma unroll
    for (int ps = 0; ps < NP; ++ps) {
      const int crow = ps * R + rsub;  // the child row of this lane in this pass
      const bool rowon = crow < C;
      const float* sx = sxa[ps];
      // reduce-scatter of the four keys' row sums over the row's G lanes: the
      // lanes G/2 apart swap a pair of keys and keep the other, the lanes G/4
      // apart one key of the pair, and a butterfly over the rest completes the
      // lane's key kq (every lane of it then holds the same sum)
      float sv;
      {
        const float s0 = hb1 ? sx[0] : sx[2], s1 = hb1 ? sx[1] : sx[3];
        const float r0 = __shfl_xor_sync(full, s0, G / 2), r1 = __shfl_xor_sync(full, s1, G / 2);
        const float w0 = (hb1 ? sx[2] : sx[0]) + r0, w1 = (hb1 ? sx[3] : sx[1]) + r1;
        const float r = __shfl_xor_sync(full, hb2 ? w0 : w1, G / 4);
        sv = (hb2 ? w1 : w0) + r;
      }
#pragma unroll
      for (int o = 1; o < G / 4; o <<= 1) sv += __shfl_xor_sync(full, sv, o);
      float cs = 0.f;  // c_sq of this lane's (key, child) pair, from the key's owner lane
#pragma unroll
      for (int c = ps * R; c < ps * R + R; ++c) {
        const float v = __shfl_sync(full, cq[c], gq * KP + kq);
        cs = crow == c ? v : cs;
      }
      const float bnd = __fmaf_ru(__fadd_ru(ksk, cs), ChildBound<DT>::scale, ChildBound<DT>::slack);
      float cross = rnd<DT>(__fsub_rd(sv, bnd));
      const bool bad = rowon && !(cross == rnd<DT>(__fadd_ru(sv, bnd)));
      if (__any_sync(full, bad)) {
#pragma unroll
        for (int kk = 0; kk < KP; ++kk) {
          if (!__any_sync(full, bad && kq == kk)) continue;
          double e64 = 0.0;
#pragma unroll
          for (int t = 0; t < NV; ++t) {
            const uint4 u = key_chunk(gq * KP + kk, t), w = blk_chunk(pk[kk], ps, t);
            const uint32_t ku[4] = {u.x, u.y, u.z, u.w}, cw[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const uint32_t pr = hmul2_dt<DT>(ku[e], cw[e]);
              e64 += (double)half_lo<DT>(pr) + (double)half_hi<DT>(pr);
            }
          }
#pragma unroll
          for (int o = 1; o < G; o <<= 1) e64 += __shfl_xor_sync(full, e64, o);
          if (bad && kq == kk) cross = rnd64<DT>(e64);
        }
      }
      // d = DT(DT(k_sq + c_sq) - DT(2 * cross)); + 0 turns a -0 into +0 (torch compares them equal)
      const float dd =
          __fadd_rn(rnd<DT>(__fsub_rn(rnd<DT>(__fadd_rn(ksk, cs)), rnd<DT>(__fmul_rn(2.f, cross)))), 0.f);
      const int bits = __float_as_int(dd);
      const int ord = bits >= 0 ? bits : (bits ^ 0x7FFFE000);
      int key = !rowon ? 0x7FFFFFFF : isnan(dd) ? (int)(0x80000000u | (uint32_t)crow) : (ord & ~0x1FFF) | crow;
#pragma unroll
      for (int o = G; o < 32; o <<= 1) key = min(key, __shfl_xor_sync(full, key, o));
      best = min(best, key);  // the child index in the low bits keeps the first minimum
    }
    // row 0's lane vg = (kk >> 1) G/2 + (kk & 1) G/4 now holds key kk of the group
    const int kk_own = lane % KP;
    const int res = __shfl_sync(full, best, (kk_own >> 1) * (G / 2) + (kk_own & 1) * (G / 4));
    if (lane / KP == gq) mine = res & 0x1FFF;
  }
  if (live) cassign[(long)g * S + s_mine] = mine;
}

template <int DT, int D, int ACH>
__global__ void __launch_bounds__(ATHREADS, ACH == 64 ? 3 : 2) assign_tc_kernel(
    const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_p, int4 kpos, int H, int S,
    int M0, const typename Storage<DT>::T* __restrict__ parents, const float* __restrict__ p_sq,
    int* __restrict__ passign, int* __restrict__ cassign) {
  using T = typename Storage<DT>::T;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = tc::smem_addr(smem_raw);
  unsigned char* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  constexpr int A_TMEM_COLS = 2 * ACH;
  const AssignLayout L = assign_layout(D, M0, ACH);
  const int g = blockIdx.y, b = g / H, h = g % H, s0 = blockIdx.x * AR;
  const int nch = (M0 + ACH - 1) / ACH;
  // the CTA's i-th chunk is chunk (i + rot) mod nch: the CTAs of a head that
  // run together start at different chunks, so that they do not all request
  // the same codebook lines from L2 at once (the argmin keys carry the parent
  // index, so the order of the chunks does not change the result)
  const int rot = blockIdx.x % nch;
  auto chunk_of = [&](int i) { return i + rot < nch ? i + rot : i + rot - nch; };
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L.bars);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + L.misc);
  volatile int* abort = reinterpret_cast<volatile int*>(sm + L.misc + 4);
  float* psq_wmax = reinterpret_cast<float*>(sm + L.misc + 16);
  uint32_t* ps2 = reinterpret_cast<uint32_t*>(sm + L.ps2);
  int np[2] = {0, 0};  // parent chunks issued per buffer (TMA producer)

  if (warp == 5 && lane == 0) {
    // the producer initialises the barriers and starts the key tile and the
    // first two parent chunks while the other warps set up
    for (int i = 0; i < AN_BARS; ++i) tc::mbar_init(&bars[i], (i == AB_SCONS || i == AB_SCONS + 1) ? AR : 1);
    *abort = 0;
    tc::fence_mbar_init();
    tc::tma_prefetch_desc(&tm_k);
    tc::tma_prefetch_desc(&tm_p);
    tc::mbar_expect_tx(&bars[AB_K], AR * D * 2);
    for (int kb = 0; kb < D / 64; ++kb) {
      int c[4];
      c[0] = kb * 64;
      c[kpos.x] = s0;
      c[kpos.y] = h;
      c[kpos.z] = b;
      tc::tma_load_4d(sm + L.k + kb * AR * 128, &tm_k, c[0], c[1], c[2], c[3], &bars[AB_K]);
    }
    for (int ci = 0; ci < 2 && ci < nch; ++ci) {
      tc::mbar_expect_tx(&bars[AB_PFULL + ci], ACH * D * 2);
      for (int kb = 0; kb < D / 64; ++kb)
        tc::tma_load_3d(sm + L.p[ci] + kb * ACH * 128, &tm_p, kb * 64, chunk_of(ci) * ACH, h, &bars[AB_PFULL + ci]);
      ++np[ci];
    }
  }
  if (warp == 4) tc::tmem_alloc(tslot, A_TMEM_COLS);
  if (tid < AR) {
    // squared parent norms as dtype pairs; +inf beyond M0 (never the minimum)
    float mx = 0.f;
    for (int j = tid; j < nch * (ACH / 2); j += AR) {
      const int p = 2 * j;
      const float a0 = p < M0 ? p_sq[(long)h * M0 + p] : INFINITY;
      const float a1 = p + 1 < M0 ? p_sq[(long)h * M0 + p + 1] : INFINITY;
      ps2[j] = pack2<DT>(a0, a1);
      // largest real norm; a NaN sticks (fmaxf would drop it)
      if (p < M0) mx = (a0 > mx || isnan(a0)) ? a0 : mx;
      if (p + 1 < M0) mx = (a1 > mx || isnan(a1)) ? a1 : mx;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float y = __shfl_xor_sync(0xffffffffu, mx, o);
      mx = (y > mx || isnan(y)) ? y : mx;
    }
    if (lane == 0) psq_wmax[warp] = mx;
  }
  tc::tc_before_sync();
  __syncthreads();
  tc::tc_after_sync();
  const uint32_t tbase = *tslot;

  if (warp == 5) {
    if (lane == 0) {  // ---- TMA producer: parent chunks from the third on ----
      for (int ci = 2; ci < nch; ++ci) {
        const int s = ci & 1;
        if (!tc::mbar_wait(&bars[AB_PEMPTY + s], ((ci - 2) >> 1) & 1, abort)) break;
        tc::mbar_expect_tx(&bars[AB_PFULL + s], ACH * D * 2);
        for (int kb = 0; kb < D / 64; ++kb)
          tc::tma_load_3d(sm + L.p[s] + kb * ACH * 128, &tm_p, kb * 64, chunk_of(ci) * ACH, h, &bars[AB_PFULL + s]);
        ++np[s];
      }
      if (*abort) {
        drain(&bars[AB_K], 0);
        for (int s = 0; s < 2; ++s)
          if (np[s]) drain(&bars[AB_PFULL + s], (np[s] - 1) & 1);
      }
    }
  } else if (warp == 4) {
    if (lane == 0) {  // ---- MMA issuer ----
      const uint32_t idS = tc::idesc_f16(DT == DT_BF16 ? 1 : 0, AR, ACH, false);
      const uint32_t ka = tc::smem_addr(sm + L.k);
      const uint32_t pa[2] = {tc::smem_addr(sm + L.p[0]), tc::smem_addr(sm + L.p[1])};
      auto issue = [&](int ci) {
        const int s = ci & 1;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t ad = tc::sdesc_sw128(ka + (kk >> 2) * AR * 128 + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = tc::sdesc_sw128(pa[s] + (kk >> 2) * ACH * 128 + (kk & 3) * 32, 16, 1024);
          tc::mma_ss(tbase + ACH * s, ad, bd, idS, kk > 0);
        }
        tc::mma_commit(&bars[AB_SFULL + s]);
        tc::mma_commit(&bars[AB_PEMPTY + s]);
      };
      bool ok = tc::mbar_wait(&bars[AB_K], 0, abort);
      for (int ci = 0; ok && ci < 2 && ci < nch; ++ci) {
        ok = tc::mbar_wait(&bars[AB_PFULL + ci], 0, abort);
        if (ok) {
          tc::tc_after_sync();
          issue(ci);
        }
      }
      for (int ci = 0; ok && ci + 2 < nch; ++ci) {
        const int s = ci & 1;
        if (!(ok = tc::mbar_wait(&bars[AB_SCONS + s], (ci >> 1) & 1, abort))) break;
        if (!(ok = tc::mbar_wait(&bars[AB_PFULL + s], ((ci + 2) >> 1) & 1, abort))) break;
        tc::tc_after_sync();
        issue(ci + 2);
      }
      tc::mma_commit(&bars[AB_END]);
      if (!ok) drain(&bars[AB_END], 0);
    }
  } else {
    // ---- row threads: key r ----
    const int r = tid, s = s0 + r;
    const bool live = s < S;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    bool ok = __all_sync(0xffffffffu, tc::mbar_wait(&bars[AB_K], 0, abort));
    // the key row in the swizzled tile: 16-byte chunk j of slab kb at (j ^ (r & 7))
    auto key_chunk = [&](int v) -> uint4 {
      const int kb = v >> 3, j = v & 7;
      return *reinterpret_cast<const uint4*>(sm + L.k + kb * AR * 128 + r * 128 + ((j ^ (r & 7)) << 4));
    };
    float ksq = 0.f;
    if (ok) {
      // k_sq = DT(sum DT(k_d^2)) with the sum exact (quantizer.py:208): fp32
      // pairs accumulate D/8 terms each, then three more additions, so the
      // rounding error of the nonnegative sum is at most gamma_18 S <= 2^-19 S';
      // where that interval straddles a dtype rounding boundary, fp64
      float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll 4
      for (int v = 0; v < D / 8; ++v) {
        const uint4 u = key_chunk(v);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t sq = hmul2_dt<DT>(w[e], w[e]);
          acc[e] = add_f32x2(acc[e], make_float2(half_lo<DT>(sq), half_hi<DT>(sq)));
        }
      }
      const float2 t2 = add_f32x2(add_f32x2(acc[0], acc[1]), add_f32x2(acc[2], acc[3]));
      const float s32 = t2.x + t2.y;
      const float bnd = __fmul_ru(s32, 0x1p-19f);
      ksq = rnd<DT>(__fsub_rd(s32, bnd));
      if (!(ksq == rnd<DT>(__fadd_ru(s32, bnd)))) {
        double a64 = 0.0;
        for (int v = 0; v < D / 8; ++v) {
          const uint4 u = key_chunk(v);
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
          for (int e = 0; e < 4; ++e) {
            const uint32_t sq = hmul2_dt<DT>(w[e], w[e]);
            a64 += (double)half_lo<DT>(sq) + (double)half_hi<DT>(sq);
          }
        }
        ksq = rnd64<DT>(a64);
      }
    }
    const uint32_t ksq2 = dup2<DT>(ksq);
    // every distance of the warp's keys is finite when k_sq + max p_sq stays
    // below a quarter of the dtype's range (|2 k.p| <= k_sq + p_sq up to
    // rounding): then no NaN can win, and DT(s - DT(2x)) = fma(-2, x, s) as
    // doubling is exact
    const float psqmax = fmaxf(fmaxf(psq_wmax[0], psq_wmax[1]), fmaxf(psq_wmax[2], psq_wmax[3]));
    const bool finite_w =
        __all_sync(0xffffffffu, !isnan(psq_wmax[0] + psq_wmax[1] + psq_wmax[2] + psq_wmax[3]) &&
                                    ksq + psqmax <= DtQuarterMax<DT>::v);
    int best = 0x7FFFFFFF;
    uint32_t nanacc = 0u;
    for (int ci = 0; ok && ci < nch; ++ci) {
      const int sb = ci & 1;
      ok = __all_sync(0xffffffffu, tc::mbar_wait(&bars[AB_SFULL + sb], (ci >> 1) & 1, abort));
      if (!ok) break;
      tc::tc_after_sync();
      // two 32-column quarters; the second quarter's TMEM load is in flight
      // while the first one is scanned
      const uint32_t col = tbase + lane_off + ACH * sb;
      uint32_t qa[32], qb[32];
      auto scan = [&](const uint32_t (&r)[32], int quarter) {
        const int cid = chunk_of(ci);
        const uint4* pp = reinterpret_cast<const uint4*>(ps2 + cid * (ACH / 2) + 16 * quarter);
        if (finite_w) {
          // keys with the index within the quarter.  While no distance of the
          // warp's quarter has its sign bit set (distances are >= +0 unless a
          // key nearly equals a parent), the raw dtype bits order as signed
          // 16-bit integers already, so the order transform is skipped and
          // only the sign bits are gathered; otherwise the quarter is scanned
          // again with the transform (the same keys for the >= +0 halves)
          auto quarter_min = [&](auto ordered) -> int {
            constexpr bool ORD = decltype(ordered)::value;
            int qbest = 0x7FFFFFFF;
            uint32_t sgn = 0u;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint4 pq = pp[q];
              const uint32_t pv[4] = {pq.x, pq.y, pq.z, pq.w};
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const int j = 4 * q + k;
                const uint32_t x2 = pack2<DT>(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));  // DT(k . p)
                const uint32_t d2 = hfma2_dt<DT>(x2, 0xC000C000u, hadd2_dt<DT>(ksq2, pv[k]));
                uint32_t k2 = d2;
                if constexpr (ORD) k2 = order2(d2);
                else sgn |= d2;
                const uint32_t il = (uint32_t)(2 * j) | ((uint32_t)(2 * j + 1) << 16);
                qbest = min(qbest, min(key_lo(k2, il), key_hi(k2, il)));
              }
            }
            if constexpr (!ORD) {
              if (__any_sync(0xffffffffu, (sgn & 0x80008000u) != 0u)) return -1;
            }
            return qbest;
          };
          int qbest = quarter_min(std::false_type{});
          if (qbest < 0) qbest = quarter_min(std::true_type{});  // warp-uniform: the vote above
          best = min(best, qbest + (cid * ACH + 32 * quarter));  // the index half has room: M0 <= 4096
          return;
        }
        const uint32_t base2 = (uint32_t)(cid * ACH + 32 * quarter) * 0x10001u + 0x10000u;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 pq = pp[q];
          const uint32_t pv[4] = {pq.x, pq.y, pq.z, pq.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int j = 4 * q + k;
            const uint32_t x2 = pack2<DT>(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));  // DT(k . p)
            const uint32_t d2 = hsub2_dt<DT>(hadd2_dt<DT>(ksq2, pv[k]), hadd2_dt<DT>(x2, x2));
            nanacc = hmax2_nan_dt<DT>(nanacc, d2);
            const uint32_t k2 = order2(d2), idx2 = base2 + 0x20002u * (uint32_t)j;
            best = min(best, min(key_lo(k2, idx2), key_hi(k2, idx2)));
          }
        }
      };
      static_assert(ACH == 64 || ACH == 128, "chunk size");
      tc::tmem_ld32(col, qa);
      tc::tmem_wait_ld();
      tc::tmem_ld32(col + 32, qb);
      scan(qa, 0);
      tc::tmem_wait_ld();
      if constexpr (ACH == 128) {
        tc::tmem_ld32(col + 64, qa);
        scan(qb, 1);
        tc::tmem_wait_ld();
        tc::tmem_ld32(col + 96, qb);
        scan(qa, 2);
        tc::tmem_wait_ld();
      }
      tc::tc_before_sync();
      tc::mbar_arrive(&bars[AB_SCONS + sb]);
      scan(qb, ACH / 32 - 1);
    }
    int pbest = best & 0xFFFF;
    const bool has_nan = isnan(half_lo<DT>(nanacc)) || isnan(half_hi<DT>(nanacc));
    if (ok && live && has_nan) {
      // a NaN distance wins (torch.argmin): the first parent whose distance is
      // NaN; NaN-ness does not depend on the summation order of k . p
      const T* pb = parents + (long)h * M0 * D;
      for (int p = 0; p < M0; ++p) {
        float cr = 0.f;
        for (int v = 0; v < D / 8; ++v) {
          const uint4 u = key_chunk(v);
          const uint4 w = *reinterpret_cast<const uint4*>(pb + (long)p * D + 8 * v);
          const uint32_t ku[4] = {u.x, u.y, u.z, u.w}, pw[4] = {w.x, w.y, w.z, w.w};
          for (int e = 0; e < 4; ++e)
            cr += half_lo<DT>(ku[e]) * half_lo<DT>(pw[e]) + half_hi<DT>(ku[e]) * half_hi<DT>(pw[e]);
        }
        const float dd = rnd<DT>(__fsub_rn(rnd<DT>(__fadd_rn(ksq, p_sq[(long)h * M0 + p])),
                                           rnd<DT>(__fmul_rn(2.f, rnd<DT>(cr)))));
        if (isnan(dd)) {
          pbest = p;
          break;
        }
      }
    }
    // the child stage runs later, in bucket order (child_bucket_kernel); it
    // finds this key's k_sq in the key's cassign word
    if (live) {  // a CTA that gave up on a wait still leaves indices in range for the later kernels
      passign[(long)g * S + s] = ok ? pbest : 0;
      cassign[(long)g * S + s] = __float_as_int(ok ? ksq : 0.f);
    }
  }

  tc::tc_before_sync();
  __syncthreads();
  if (warp == 4) {
    tc::tc_after_sync();
    tc::tmem_free(tbase, A_TMEM_COLS);
  }
  if (tid == 0 && *abort) atomicOr(&g_fault, 1);
}

}  // namespace

bool assign_tc_ok(int dt, int D, int M0) {
  const char* e = std::getenv("AVQ_DISABLE_TCGEN05");
  const bool off = e && *e && *e != '0';
  return !off && dt != DT_F32 && (D == 64 || D == 128) && M0 <= A_MAX_M0;
}

template <int DT>
int launch_assign_tc(const QuantizeArgs& a, cudaStream_t st) {
  using T = typename Storage<DT>::T;
  const int G = a.B * a.H, D = a.D;
  CUtensorMap tk, tp;
  int4 kpos;
  if (!tc::map_rows4(&tk, DT, a.keys, a.ks, a.B, a.H, a.S, D, AR, &kpos) ||
      !tc::map_rows3(&tp, DT, a.parents_dt, a.H, a.M0, D, a.M0 <= A_SMALL_M0 ? 64 : 128))
    return AVQ_ERR_UNSUPPORTED;
  // the child kernel reads child rows with 16-byte loads: aligned rows, at most A_MAX_C children
  if (a.C < 1 || a.C > A_MAX_C || (uintptr_t)a.children_dt % 16 != 0 || (uintptr_t)a.c_sq % 4 != 0)
    return AVQ_ERR_UNSUPPORTED;
  const int ach = a.M0 <= A_SMALL_M0 ? 64 : 128;
  const AssignLayout L = assign_layout(D, a.M0, ach);
  // 64-parent chunks: at least 60 KB, so at most 3 CTAs (3 x 128 TMEM columns) per SM;
  // 128-parent chunks: at least 80 KB, at most 2 CTAs (2 x 256 columns): tcgen05.alloc never waits
  const size_t smem = std::max<size_t>((size_t)L.total + 1024, (ach == 64 ? 60 : 80) * 1024);
  auto go = [&](auto kfn) {
    AVQ_TIMED("assign_tc", st);
    cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kfn<<<dim3((a.S + AR - 1) / AR, G), ATHREADS, smem, st>>>(tk, tp, kpos, a.H, a.S, a.M0,
                                                                static_cast<const T*>(a.parents_dt), a.p_sq,
                                                                a.passign, a.cassign);
  };
  if (ach == 64) {
    if (D == 64) go(assign_tc_kernel<DT, 64, 64>);
    else go(assign_tc_kernel<DT, 128, 64>);
  } else {
    if (D == 64) go(assign_tc_kernel<DT, 64, 128>);
    else go(assign_tc_kernel<DT, 128, 128>);
  }
  return cudaPeekAtLastError() == cudaSuccess ? AVQ_OK : AVQ_ERR_CUDA;
}

template int launch_assign_tc<DT_BF16>(const QuantizeArgs&, cudaStream_t);
template int launch_assign_tc<DT_F16>(const QuantizeArgs&, cudaStream_t);

// The child stage of a launch_assign_tc pass, once `order` holds each (b,h)'s
// keys sorted by parent.
template <int DT>
int launch_child_bucket(const QuantizeArgs& a, const int* order, cudaStream_t st) {
  using T = typename Storage<DT>::T;
  const int G = a.B * a.H;
  if (a.S <= 0) return AVQ_OK;
  const dim3 grid((a.S + 32 * CB_WARPS - 1) / (32 * CB_WARPS), G);
  AVQ_TIMED("child", st);
#define AVQ_CB(D_, NV, NP)                                                                                          \
  do {                                                                                                              \
    cudaFuncSetAttribute(child_bucket_kernel<DT, D_, NV, NP>, cudaFuncAttributeMaxDynamicSharedMemorySize,        \
                         CB_WARPS * 32 * (D_) * 2);                                                                 \
    child_bucket_kernel<DT, D_, NV, NP><<<grid, CB_WARPS * 32, CB_WARPS * 32 * (D_) * 2, st>>>(                    \
        static_cast<const T*>(a.keys), a.ks, a.H, a.S, a.M0, a.C, order, a.passign,                               \
        static_cast<const T*>(a.children_dt), a.c_sq, a.cassign);                                                 \
  } while (0)
  // rows per pass 32 / (D / 8 / NV): 2 or 4 at D = 128, 4 or 8 at D = 64
  if (a.D == 128) {
    if (a.C <= 2) AVQ_CB(128, 1, 1);
    else if (a.C <= 4) AVQ_CB(128, 2, 1);
    else AVQ_CB(128, 2, 2);
  } else {
    if (a.C <= 4) AVQ_CB(64, 1, 1);
    else AVQ_CB(64, 2, 1);
  }
#undef AVQ_CB
  return cudaPeekAtLastError() == cudaSuccess ? AVQ_OK : AVQ_ERR_CUDA;
}

template int launch_child_bucket<DT_BF16>(const QuantizeArgs&, const int*, cudaStream_t);
template int launch_child_bucket<DT_F16>(const QuantizeArgs&, const int*, cudaStream_t);


// Reads and clears this file's fault word (device code without relocatable
// linking keeps one copy per file, so every kernel file has its own).
int read_fault_assign(int* code, cudaStream_t st) {
  int v = 0;
  if (cudaMemcpyFromSymbolAsync(&v, g_fault, sizeof(int), 0, cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return AVQ_ERR_CUDA;
  const int zero = 0;
  if (cudaMemcpyToSymbolAsync(g_fault, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st) != cudaSuccess)
    return AVQ_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return AVQ_ERR_CUDA;
  *code = v;
  return AVQ_OK;
}

}  // namespace avq
