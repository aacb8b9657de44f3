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
// Child stage (quantizer.py:218-226): the cross term is a sum of
// dtype-rounded elementwise products, rounded once as its exact value would
// be (fp32 with an error bound, fp64 where the bound cannot decide).
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
constexpr int A_KP = 4;              // keys per cp.async group of the child stage
constexpr int A_CSQ_PER_WARP = 64;   // staged child norms per warp: ring slots x C <= 64

constexpr int AB_K = 0, AB_PFULL = 1, AB_PEMPTY = 3, AB_SFULL = 5, AB_SCONS = 7, AB_END = 9, AN_BARS = 10;

struct AssignLayout {
  int k, p[2], ps2, csq, bars, misc, total;
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
  L.csq = o;
  o += 4 * A_CSQ_PER_WARP * 4;
  L.bars = o;
  o += AN_BARS * 8;
  L.misc = o;
  o += 16;
  L.total = o;
  return L;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

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

// cp.async with memory clobbers: shared-memory reads of a ring slot stay
// between the wait that fills it and the copy that refills it.
__device__ __forceinline__ void ring_cp16(void* smem, const void* gmem, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem), "r"(pred ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void ring_cp4(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void ring_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void ring_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Packed fp32 pair addition (one instruction for both lanes, IEEE
// round-to-nearest per element).
__device__ __forceinline__ float2 add_f32x2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
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
// row rsub, so one key costs the warp NV coalesced 16-byte copies a lane.
// The blocks stream through a per-warp ring of NG groups of A_KP keys in
// shared memory (cp.async), NG - 1 groups ahead of the one being reduced.
//
// cross = DT(fp32(sum_d DT(k_d c_d))) with the sum exact (what the fp64 sum
// of the dtype products gives) is evaluated in fp32: each lane sums its 8*NV
// products pairwise and the row's G lanes combine by butterfly, a tree of
// depth 3 + log2(NV*G) <= 7, so the fp32 result S' lies within
// gamma_7 * sum|t| of the exact sum, bounded by ChildBound.  fp32 and dtype
// rounding are monotone, so when both ends of [S' - b, S' + b] (rounded
// outwards) round to the same dtype value that value is the exact sum's
// rounding; otherwise (close to a dtype rounding boundary, or non-finite)
// the row is summed again in fp64.  After the butterfly every lane of a row
// holds the row's sums of all A_KP keys, so lane vg finishes key vg % A_KP:
// the rounding test, the distance and the argmin run once per lane, not once
// per key.  torch.argmin over the children (first minimum, a NaN wins) is a
// signed min over 32-bit keys: the order-preserving integer form of the
// distance, whose low 13 bits are zero for dtype values, or'ed with the
// child index.
template <int DT, int D, int NV, int NG>
__device__ __forceinline__ int child_stage(unsigned char* ring, float* csr, const unsigned char* ktile, int warp,
                                           int lane, uint32_t livemask, int pbest, float ksq,
                                           const unsigned char* __restrict__ chh, const float* __restrict__ csqh,
                                           int C) {
  constexpr int CPR = D / 8, G = CPR / NV, KP = A_KP, NGRP = 32 / KP;
  static_assert(G >= KP && G % KP == 0 && 32 % G == 0, "lanes per row");
  constexpr int RB = D * 2;  // bytes per child row
  const unsigned full = 0xffffffffu;
  const int vg = lane % G, rsub = lane / G, kq = lane % KP;
  const bool rowon = rsub < C;
  const int blk = C * RB;
  const int boff_mine = pbest * blk;  // byte offset of this lane's key's child block in the head
  const int lane_off = rsub * RB + vg * 16;
  auto issue = [&](int grp) {  // keys KP*grp .. KP*grp+KP-1 into ring group grp % NG
    const int sg = grp % NG;
#pragma unroll
    for (int kk = 0; kk < KP; ++kk) {
      const int k = grp * KP + kk;
      const int boff = __shfl_sync(full, boff_mine, k);
      const bool on = ((livemask >> k) & 1u) != 0u;
      if (rowon) {
        unsigned char* dst = ring + (sg * KP + kk) * blk + lane_off;
        const unsigned char* src = on ? chh + boff + lane_off : chh;
#pragma unroll
        for (int t = 0; t < NV; ++t) ring_cp16(dst + G * 16 * t, src + (on ? G * 16 * t : 0), on);
        if (vg == 0 && on) ring_cp4(csr + (sg * KP + kk) * C + rsub, csqh + boff / RB + rsub);
      }
    }
    ring_commit();
  };
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
#pragma unroll 1
  for (int gq = 0; gq < NGRP; ++gq) {
    ring_wait<NG - 1>();
    __syncwarp();  // the child norms come from other lanes' copies
    const int sg = gq % NG;
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
#pragma unroll
    for (int o = 1; o < G; o <<= 1)
#pragma unroll
      for (int kk = 0; kk < KP; ++kk) sx[kk] += __shfl_xor_sync(full, sx[kk], o);
    // this lane's key: kq = vg % KP
    float sv = sx[0];
#pragma unroll
    for (int kk = 1; kk < KP; ++kk) sv = kq == kk ? sx[kk] : sv;
    const float ksk = __shfl_sync(full, ksq, gq * KP + kq);
    const float cs = rowon ? csr[(sg * KP + kq) * C + rsub] : 0.f;
    const float bnd = __fmaf_ru(__fadd_ru(ksk, cs), ChildBound<DT>::scale, ChildBound<DT>::slack);
    float cross = rnd<DT>(__fsub_rd(sv, bnd));
    const bool bad = rowon && !(cross == rnd<DT>(__fadd_ru(sv, bnd)));
    const uint32_t badb = __ballot_sync(full, bad);
    if (badb) {
#pragma unroll
      for (int kk = 0; kk < KP; ++kk) {
        if (!(badb & (0x11111111u << kk))) continue;  // lanes finishing key kk: lane % KP == kk
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
    // lanes 0 .. KP-1 (row 0, vg = kk) now hold keys 0 .. KP-1 of the group
    const int res = __shfl_sync(full, key, kq);
    if (lane / KP == gq) mine = res & 0x1FFF;
    // every value read from this ring group fed the reductions above: refill it
    if (gq + NG < NGRP) issue(gq + NG);
    else ring_commit();
  }
  return mine;
}

__device__ __forceinline__ void drain(uint64_t* bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!tc::mbar_try(bar, parity) && clock64() - t0 < tc::kWaitCycles / 8) {
  }
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
  uint32_t* ps2 = reinterpret_cast<uint32_t*>(sm + L.ps2);

  if (tid == 0) {
    for (int i = 0; i < AN_BARS; ++i) tc::mbar_init(&bars[i], (i == AB_SCONS || i == AB_SCONS + 1) ? AR : 1);
    *abort = 0;
    tc::fence_mbar_init();
  }
  if (warp == 4) tc::tmem_alloc(tslot, A_TMEM_COLS);
  if (tid < AR) {
    // squared parent norms as dtype pairs; +inf beyond M0 (never the minimum)
    for (int j = tid; j < nch * (ACH / 2); j += AR) {
      const int p = 2 * j;
      const float a0 = p < M0 ? p_sq[(long)h * M0 + p] : INFINITY;
      const float a1 = p + 1 < M0 ? p_sq[(long)h * M0 + p + 1] : INFINITY;
      ps2[j] = pack2<DT>(a0, a1);
    }
  }
  tc::tc_before_sync();
  __syncthreads();
  tc::tc_after_sync();
  const uint32_t tbase = *tslot;

  if (warp == 5) {
    if (lane == 0) {  // ---- TMA producer ----
      tc::tma_prefetch_desc(&tm_k);
      tc::tma_prefetch_desc(&tm_p);
      int np[2] = {0, 0};
      tc::mbar_expect_tx(&bars[AB_K], AR * D * 2);
      for (int kb = 0; kb < D / 64; ++kb) {
        int c[4];
        c[0] = kb * 64;
        c[kpos.x] = s0;
        c[kpos.y] = h;
        c[kpos.z] = b;
        tc::tma_load_4d(sm + L.k + kb * AR * 128, &tm_k, c[0], c[1], c[2], c[3], &bars[AB_K]);
      }
      for (int ci = 0; ci < nch; ++ci) {
        const int s = ci & 1;
        if (ci >= 2 && !tc::mbar_wait(&bars[AB_PEMPTY + s], ((ci - 2) >> 1) & 1, abort)) break;
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
    if (ok) {  // k_sq = DT(sum DT(k_d^2)) (quantizer.py:208), fp64 partial sums
      double acc[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll 4
      for (int v = 0; v < D / 8; ++v) {
        const uint4 u = key_chunk(v);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t sq = hmul2_dt<DT>(w[e], w[e]);
          acc[e] += (double)half_lo<DT>(sq) + (double)half_hi<DT>(sq);
        }
      }
      ksq = rnd64<DT>((acc[0] + acc[1]) + (acc[2] + acc[3]));
    }
    const uint32_t ksq2 = dup2<DT>(ksq);
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
    if (ok) {
      const uint32_t livemask = __ballot_sync(0xffffffffu, live);
      unsigned char* ring = sm + L.p[0] + warp * (ACH * D);
      float* csr = reinterpret_cast<float*>(sm + L.csq) + warp * A_CSQ_PER_WARP;
      const unsigned char* chh = reinterpret_cast<const unsigned char*>(children + (long)h * M0 * C * D);
      const float* csqh = c_sq + (long)h * M0 * C;
      const unsigned char* kt = sm + L.k;
      int bi;
      if constexpr (D == 128)
        bi = C <= 2 ? child_stage<DT, D, 1, 4>(ring, csr, kt, warp, lane, livemask, pbest, ksq, chh, csqh, C)
             : C <= 4 ? child_stage<DT, D, 2, 4>(ring, csr, kt, warp, lane, livemask, pbest, ksq, chh, csqh, C)
                      : child_stage<DT, D, 4, 2>(ring, csr, kt, warp, lane, livemask, pbest, ksq, chh, csqh, C);
      else
        bi = C <= 4 ? child_stage<DT, D, 1, 4>(ring, csr, kt, warp, lane, livemask, pbest, ksq, chh, csqh, C)
                    : child_stage<DT, D, 2, 2>(ring, csr, kt, warp, lane, livemask, pbest, ksq, chh, csqh, C);
      if (live) {
        passign[(long)g * S + s] = pbest;
        cassign[(long)g * S + s] = bi;
      }
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
  if (a.C < 1 || a.C > A_MAX_C) return AVQ_ERR_UNSUPPORTED;
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
