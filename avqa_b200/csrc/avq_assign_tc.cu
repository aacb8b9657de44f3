// Key -> parent -> child assignment on the sm_100a tensor cores for bf16 /
// fp16 and D in {64, 128} (reference quantizer.py:166-226).
//
// CTA = 128 keys of one (b,h); thread r of warps 0-3 owns key r (TMEM lane r);
// warp 4 issues tcgen05.mma, warp 5 streams the key tile and 128-parent
// chunks of the head's codebook with TMA.  TMEM holds two 128-column buffers
// of fp32 cross terms K P_c^T.
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
// Child stage (quantizer.py:218-226): each row warp then takes its 32 keys
// one group of four at a time, the keys' child blocks arriving by bulk copy
// in the idle parent buffers; the cross term is a sum of dtype-rounded
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
constexpr int ACH = 128;       // parents per chunk
constexpr int ATHREADS = 192;  // 4 row warps + MMA warp + TMA warp
constexpr int A_TMEM_COLS = 256;
constexpr int A_MAX_M0 = 4096;
constexpr int A_MAX_C = 8;           // children per parent on this path
constexpr int A_KP = 4;              // keys per ring group of the child stage
constexpr int A_RING_GROUPS = 4;     // most ring groups of a row warp's child stage

constexpr int AB_K = 0, AB_PFULL = 1, AB_PEMPTY = 3, AB_SFULL = 5, AB_SCONS = 7, AB_END = 9, AN_BARS = 10;

struct AssignLayout {
  int k, p[2], ps2, rbar, bars, misc, total;
};

__host__ __device__ inline AssignLayout assign_layout(int D, int M0) {
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
  L.rbar = o;  // child-stage ring barriers, A_RING_GROUPS per row warp
  o += 4 * A_RING_GROUPS * 8;
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

// Global -> shared bulk copy (TMA engine, no tensor map), completing on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   tc::smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(tc::smem_addr(bar))
               : "memory");
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

// Child stage of one warp's 32 keys (quantizer.py:218-227).  A key's C child
// rows form one contiguous block; its rows are spread over the warp, G lanes
// to a row, lane (rsub, vg) holding the 16-byte chunks vg + G*t (t < NV) of
// row rsub.  The blocks stream through a per-warp ring of NG groups of A_KP
// keys in shared memory, one bulk copy per key issued by the key's own lane,
// NG - 1 groups ahead of the one being reduced; each key's C child norms sit
// in its lane's registers.
//
// cross = DT(fp32(sum_d DT(k_d c_d))) with the sum exact (what the fp64 sum
// of the dtype products gives) is evaluated in fp32: each lane sums its 8*NV
// products pairwise and the row's G lanes combine by butterfly, a tree of
// depth 3 + log2(NV*G) <= 7, so the fp32 result S' lies within
// gamma_7 * sum|t| of the exact sum, bounded by ChildBound.  fp32 and dtype
// rounding are monotone, so when both ends of [S' - b, S' + b] (rounded
// outwards) round to the same dtype value that value is the exact sum's
// rounding; otherwise (close to a dtype rounding boundary, or non-finite)
// the row is summed again in fp64.  The row's lanes reduce-scatter the A_KP
// keys' sums, so each lane finishes one key: the rounding test, the distance
// and the argmin run once per lane, not once per key.  torch.argmin over the children (first minimum, a NaN wins) is a
// signed min over 32-bit keys: the order-preserving integer form of the
// distance, whose low 13 bits are zero for dtype values, or'ed with the
// child index.
template <int DT, int D, int NV, int NG>
__device__ __forceinline__ int child_stage(unsigned char* ring, uint64_t* rbar, volatile int* abort,
                                           const unsigned char* ktile, int warp, int lane, uint32_t livemask, int pbest,
                                           float ksq, const unsigned char* __restrict__ chh,
                                           const float* __restrict__ csqh, int C) {
  static_assert(NG <= A_RING_GROUPS, "ring barriers");
  constexpr int CPR = D / 8, G = CPR / NV, KP = A_KP, NGRP = 32 / KP;
  static_assert(G >= KP && G % KP == 0 && 32 % G == 0, "lanes per row");
  constexpr int RB = D * 2;  // bytes per child row
  const unsigned full = 0xffffffffu;
  static_assert(KP == 4, "two halving levels");
  const int vg = lane % G, rsub = lane / G;
  const bool hb1 = (vg & (G / 2)) != 0, hb2 = (vg & (G / 4)) != 0;
  const int kq = (hb1 ? 2 : 0) + (hb2 ? 1 : 0);  // the key of the group this lane finishes
  const bool rowon = rsub < C;
  const int blk = C * RB;
  const int boff_mine = pbest * blk;  // byte offset of this lane's key's child block in the head
  const int lane_off = rsub * RB + vg * 16;
  (void)warp;
  // keys KP*grp .. KP*grp+KP-1 into ring group grp % NG: each live key's
  // owner lane copies its block with one bulk copy; the group's first owner
  // arms the barrier.  Every lane's reads of the slot fed the shuffles of the
  // reductions before, so they are complete when the owner's copy is issued.
  auto issue = [&](int grp) {
    const int sg = grp % NG, kk = lane % KP;
    const uint32_t gl = (livemask >> (grp * KP)) & ((1u << KP) - 1u);
    if (lane == grp * KP) tc::mbar_expect_tx(&rbar[sg], (uint32_t)__popc(gl) * (uint32_t)blk);
    __syncwarp();
    if (lane / KP == grp && ((gl >> kk) & 1u))
      bulk_g2s(ring + (sg * KP + kk) * blk, chh + boff_mine, (uint32_t)blk, &rbar[sg]);
  };
  // this lane's key's child norms, read once; the epilogue takes them from the
  // key's owner lane
  // the largest C that this lane split serves (the dispatch picks NV from C)
  constexpr int CQ = D == 128 ? (NV >= 4 ? 8 : (NV == 2 ? 4 : 2)) : (NV >= 2 ? 8 : 4);
  float cq[CQ];
  const bool live_mine = ((livemask >> lane) & 1u) != 0u;
#pragma unroll
  for (int c = 0; c < CQ; ++c) cq[c] = live_mine && c < C ? csqh[pbest * C + c] : 0.f;
  uint32_t koff[NV];  // this lane's key chunks in the swizzled key tile, before the row swizzle
#pragma unroll
  for (int t = 0; t < NV; ++t) {
    const int v = vg + G * t;
    koff[t] = (uint32_t)((v >> 3) * AR * 128 + ((v & 7) << 4));
  }
  auto key_chunk = [&](int rk, int t) -> uint4 {  // chunk j of slab v/8 sits at j ^ (rk & 7)
    return *reinterpret_cast<const uint4*>(ktile + rk * 128 + (koff[t] ^ ((rk & 7) << 4)));
  };
  auto blk_chunk = [&](int slot, int t) -> uint4 {
    return rowon ? *reinterpret_cast<const uint4*>(ring + slot * blk + lane_off + G * 16 * t)
                 : make_uint4(0u, 0u, 0u, 0u);
  };

  int mine = -1;
#pragma unroll 1
  for (int gq = 0; gq < NG; ++gq) issue(gq);
  int gq = 0;
#pragma unroll 1
  for (; gq < NGRP; ++gq) {
    const int sg = gq % NG;
    if (!__all_sync(full, tc::mbar_wait(&rbar[sg], (gq / NG) & 1, abort))) break;
    float sx[KP];
#pragma unroll
    for (int kk = 0; kk < KP; ++kk) {
      const int rk = warp * 32 + gq * KP + kk;
      float2 acc[NV * 4];
#pragma unroll
      for (int t = 0; t < NV; ++t) {
        const uint4 u = key_chunk(rk, t), w = blk_chunk(sg * KP + kk, t);
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
      sx[kk] = acc[0].x + acc[0].y;
    }
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
    const float ksk = __shfl_sync(full, ksq, gq * KP + kq);
    float cs = 0.f;  // c_sq of this lane's (key, child) pair, from the key's owner lane
#pragma unroll
    for (int c = 0; c < CQ; ++c) {
      if (c < C) {
        const float v = __shfl_sync(full, cq[c], gq * KP + kq);
        cs = rsub == c ? v : cs;
      }
    }
    const float bnd = __fmaf_ru(__fadd_ru(ksk, cs), ChildBound<DT>::scale, ChildBound<DT>::slack);
    float cross = rnd<DT>(__fsub_rd(sv, bnd));
    const bool bad = rowon && !(cross == rnd<DT>(__fadd_ru(sv, bnd)));
    if (__any_sync(full, bad)) {
#pragma unroll
      for (int kk = 0; kk < KP; ++kk) {
        if (!__any_sync(full, bad && kq == kk)) continue;
        const int rk = warp * 32 + gq * KP + kk;
        double e64 = 0.0;
#pragma unroll
        for (int t = 0; t < NV; ++t) {
          const uint4 u = key_chunk(rk, t), w = blk_chunk(sg * KP + kk, t);
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
    const float dd = __fadd_rn(rnd<DT>(__fsub_rn(rnd<DT>(__fadd_rn(ksk, cs)), rnd<DT>(__fmul_rn(2.f, cross)))), 0.f);
    const int bits = __float_as_int(dd);
    const int ord = bits >= 0 ? bits : (bits ^ 0x7FFFE000);
    int key = !rowon ? 0x7FFFFFFF : isnan(dd) ? (int)(0x80000000u | (uint32_t)rsub) : (ord & ~0x1FFF) | rsub;
#pragma unroll
    for (int o = G; o < 32; o <<= 1) key = min(key, __shfl_xor_sync(full, key, o));
    // row 0's lane vg = (kk >> 1) G/2 + (kk & 1) G/4 now holds key kk of the group
    const int kk_own = lane % KP;
    const int res = __shfl_sync(full, key, (kk_own >> 1) * (G / 2) + (kk_own & 1) * (G / 4));
    if (lane / KP == gq) mine = res & 0x1FFF;
    // every value read from this ring group fed the reductions above: refill it
    if (gq + NG < NGRP) issue(gq + NG);
  }
  if (gq < NGRP) {  // a wait gave up: let the copies in flight land before the CTA exits
    for (int g2 = gq; g2 < NGRP && g2 < gq + NG; ++g2) drain(&rbar[g2 % NG], (g2 / NG) & 1);
    return -1;
  }
  return mine;
}

template <int DT, int D>
__global__ void __launch_bounds__(ATHREADS, 2) assign_tc_kernel(
    const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_p, int4 kpos, int H, int S,
    int M0, int C, const typename Storage<DT>::T* __restrict__ parents, const float* __restrict__ p_sq,
    const typename Storage<DT>::T* __restrict__ children, const float* __restrict__ c_sq, int* __restrict__ passign,
    int* __restrict__ cassign) {
  using T = typename Storage<DT>::T;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = tc::smem_addr(smem_raw);
  unsigned char* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  const AssignLayout L = assign_layout(D, M0);
  const int g = blockIdx.y, b = g / H, h = g % H, s0 = blockIdx.x * AR;
  const int nch = (M0 + ACH - 1) / ACH;
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
    for (int i = 0; i < 4 * A_RING_GROUPS; ++i) tc::mbar_init(reinterpret_cast<uint64_t*>(sm + L.rbar) + i, 1);
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
        tc::tma_load_3d(sm + L.p[ci] + kb * ACH * 128, &tm_p, kb * 64, ci * ACH, h, &bars[AB_PFULL + ci]);
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
          tc::tma_load_3d(sm + L.p[s] + kb * ACH * 128, &tm_p, kb * 64, ci * ACH, h, &bars[AB_PFULL + s]);
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
      // four 32-column quarters; the next quarter's TMEM load is in flight
      // while the current one is scanned
      const uint32_t col = tbase + lane_off + ACH * sb;
      uint32_t qa[32], qb[32];
      auto scan = [&](const uint32_t (&r)[32], int quarter) {
        const uint4* pp = reinterpret_cast<const uint4*>(ps2 + ci * (ACH / 2) + 16 * quarter);
        if (finite_w) {
          int qbest = 0x7FFFFFFF;  // keys with the index within the quarter
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 pq = pp[q];
            const uint32_t pv[4] = {pq.x, pq.y, pq.z, pq.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int j = 4 * q + k;
              const uint32_t x2 = pack2<DT>(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));  // DT(k . p)
              const uint32_t d2 = hfma2_dt<DT>(x2, 0xC000C000u, hadd2_dt<DT>(ksq2, pv[k]));
              const uint32_t k2 = order2(d2), il = (uint32_t)(2 * j) | ((uint32_t)(2 * j + 1) << 16);
              qbest = min(qbest, min(key_lo(k2, il), key_hi(k2, il)));
            }
          }
          best = min(best, qbest + (ci * ACH + 32 * quarter));  // the index half has room: M0 <= 4096
          return;
        }
        const uint32_t base2 = (uint32_t)(ci * ACH + 32 * quarter) * 0x10001u + 0x10000u;
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
      tc::tmem_ld32(col, qa);
      tc::tmem_wait_ld();
      tc::tmem_ld32(col + 32, qb);
      scan(qa, 0);
      tc::tmem_wait_ld();
      tc::tmem_ld32(col + 64, qa);
      scan(qb, 1);
      tc::tmem_wait_ld();
      tc::tmem_ld32(col + 96, qb);
      scan(qa, 2);
      tc::tmem_wait_ld();
      tc::tc_before_sync();
      tc::mbar_arrive(&bars[AB_SCONS + sb]);
      scan(qb, 3);
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
    // child stage: the assigned parent's children (quantizer.py:218-226), a
    // warp's 32 keys through a cp.async ring in the now idle parent buffers
    int bi = -1;
    if (ok) {
      const uint32_t livemask = __ballot_sync(0xffffffffu, live);
      unsigned char* ring = sm + L.p[0] + warp * (ACH * D);
      uint64_t* rbar = reinterpret_cast<uint64_t*>(sm + L.rbar) + warp * A_RING_GROUPS;
      const unsigned char* chh = reinterpret_cast<const unsigned char*>(children + (long)h * M0 * C * D);
      const float* csqh = c_sq + (long)h * M0 * C;
      const unsigned char* kt = sm + L.k;
      if constexpr (D == 128)
        bi = C <= 2 ? child_stage<DT, D, 1, 4>(ring, rbar, abort, kt, warp, lane, livemask, pbest, ksq, chh, csqh, C)
             : C <= 4 ? child_stage<DT, D, 2, 4>(ring, rbar, abort, kt, warp, lane, livemask, pbest, ksq, chh, csqh, C)
                      : child_stage<DT, D, 4, 2>(ring, rbar, abort, kt, warp, lane, livemask, pbest, ksq, chh, csqh, C);
      else
        bi = C <= 4 ? child_stage<DT, D, 1, 4>(ring, rbar, abort, kt, warp, lane, livemask, pbest, ksq, chh, csqh, C)
                    : child_stage<DT, D, 2, 2>(ring, rbar, abort, kt, warp, lane, livemask, pbest, ksq, chh, csqh, C);
    }
    if (live) {  // a CTA that gave up on a wait still leaves indices in range for the later kernels
      const bool good = ok && bi >= 0;
      passign[(long)g * S + s] = good ? pbest : 0;
      cassign[(long)g * S + s] = good ? bi : 0;
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
      !tc::map_rows3(&tp, DT, a.parents_dt, a.H, a.M0, D, ACH))
    return AVQ_ERR_UNSUPPORTED;
  // the child blocks move with bulk copies: 16-byte aligned rows
  if (a.C < 1 || a.C > A_MAX_C || (uintptr_t)a.children_dt % 16 != 0 || (uintptr_t)a.c_sq % 4 != 0)
    return AVQ_ERR_UNSUPPORTED;
  const AssignLayout L = assign_layout(D, a.M0);
  const size_t smem = std::max<size_t>((size_t)L.total + 1024, 80 * 1024);  // <= 2 CTAs (2 x 256 TMEM columns) per SM
  auto go = [&](auto kfn) {
    AVQ_TIMED("assign_tc", st);
    cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kfn<<<dim3((a.S + AR - 1) / AR, G), ATHREADS, smem, st>>>(tk, tp, kpos, a.H, a.S, a.M0, a.C,
                                                                static_cast<const T*>(a.parents_dt), a.p_sq,
                                                                static_cast<const T*>(a.children_dt), a.c_sq,
                                                                a.passign, a.cassign);
  };
  if (D == 64) go(assign_tc_kernel<DT, 64>);
  else go(assign_tc_kernel<DT, 128>);
  return cudaPeekAtLastError() == cudaSuccess ? AVQ_OK : AVQ_ERR_CUDA;
}

template int launch_assign_tc<DT_BF16>(const QuantizeArgs&, cudaStream_t);
template int launch_assign_tc<DT_F16>(const QuantizeArgs&, cudaStream_t);


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
