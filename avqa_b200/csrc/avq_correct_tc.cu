// Child correction on the sm_100a tensor cores for bf16 / fp16 and D in {64, 128}
// (reference refinement.py:82-304, attention.py:100-163, multipass.py:207-262,
// attention_module.py:532-535).
//
// CTA = 128 queries of one (b,h); thread r of warps 0-3 owns query r (TMEM
// lane r) and 96 of them also gather one slot row of the group after next with
// cp.async; warp 4 loads the query tile with TMA and issues tcgen05.mma.  The
// slot descriptors (rows, counts, masks) of every group come from a small
// kernel run before, so the gathers need no dependent loads.
// The selected parents of a pass are taken J = 48 / (1 + C) at a time with
// their children: 48 slots (J parents, J*C children, zero padding).
//
// TMEM (256 columns): O [0, D) -- the fp32 state a, seeded from the parent
// pass -- then the 48 slot logits Q L^T and the slot weights as three bf16
// parts (hi, mid, lo: 24 significant bits, two per column) that are the A
// operand of O += W V.  Per slot and query, with m, z the parent-pass row max
// and normaliser:
//   parent  pi = DT(e / max(z, eps)), e = DT(exp(DT(s - m)));  w = -exp(pi - m) n
//   child   w = exp(u - m) n_c            (u = -inf for an empty child)
// and l' = l - sum w_parent + sum w_child per pass; out = O / max(l', 1e-12).
// The weights are fp32 quantities of the reference's fp32 correction; they use
// the fast exponential (relative error a few 1e-7), far inside the bf16
// output tolerance, and never feed a routing decision.
//
// fp16: the logit MMA runs on fp16 operands; the weights stay three bf16 parts
// (one MMA kind takes one operand type), so each gathered fp16 value row is
// split exactly into two bf16 planes, v = hi + lo (11 significant bits = 8 +
// at most 3), by the thread that gathered it, and O += W V takes six MMAs.
#include <cuda.h>

#include <algorithm>
#include <type_traits>
#include <cstdlib>

#include "avq_kernels.cuh"
#include "avq_mma.cuh"
#include "avq_tc.cuh"

namespace avq {

namespace {
// Bit 0: a CTA of this file gave up on a bounded wait.
__device__ int g_fault;
}  // namespace

namespace {

constexpr int CR = 128;        // queries per CTA
constexpr int NS = 48;         // slots per group
constexpr int C_TMEM_COLS = 256;
constexpr uint32_t EXPB = 0x3AFF;  // exponential table (same layout as the parent-attention table)
constexpr int EXPN = 2051;

constexpr int CB_Q = 0, CB_FULL = 1, CB_EMPTY = 4, CB_SFULL = 7, CB_SFREE = 8, CB_WFULL = 9, CB_WFREE = 10,
              CB_OFULL = 11, CB_XCH = 12, CB_XFREE = 13, CN_BARS = 14;

constexpr int NBUF = 3;         // gathered slot buffers
constexpr int CTHREADS2 = 288;  // 8 row warps (two threads per query) + the MMA / TMA warp
constexpr int MW = 8;           // the MMA / TMA warp

struct CorrLayout {
  int q, l[NBUF], v[NBUF], vlo[NBUF], meta[NBUF], exptab, bars, misc, total;
};

// split_v: fp16 value rows, stored as two bf16 planes (v and vlo).
// masked: a third meta array holds each parent slot's parent index (for the
// mask bits); unmasked calls keep the two-array layout.
__host__ __device__ inline CorrLayout corr_layout(int D, bool split_v, bool masked) {
  CorrLayout L;
  int o = 0;
  L.q = o;
  o += CR * D * 2;
  for (int i = 0; i < NBUF; ++i) {
    L.l[i] = o;
    o += NS * D * 2;
  }
  for (int i = 0; i < NBUF; ++i) {
    L.v[i] = o;
    o += NS * D * 2;
  }
  for (int i = 0; i < NBUF; ++i) {
    L.vlo[i] = o;
    if (split_v) o += NS * D * 2;
  }
  for (int i = 0; i < NBUF; ++i) {
    L.meta[i] = o;
    o += (masked ? 3 : 2) * NS * 4;  // n [48], logit mask [48], (masked) parent index of a parent slot or -1 [48]
  }
  L.exptab = o;
  o += ((EXPN + 1) / 2) * 4;
  o = (o + 15) & ~15;
  L.bars = o;
  o += CN_BARS * 8;
  L.misc = o;
  o += 16;
  L.total = o;
  return L;
}

// Barrier of the 256 row threads (the MMA / TMA warp does not take part), and
// the same barrier returning whether `p` holds in every row thread.
__device__ __forceinline__ void corr_rows_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
__device__ __forceinline__ bool corr_rows_all(bool p) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred a, b;\n\tsetp.ne.u32 a, %1, 0;\n\tbar.red.and.pred b, 1, 256, a;\n\tselp.u32 %0, 1, 0, b;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)p)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void drain_c(uint64_t* bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!tc::mbar_try(bar, parity) && clock64() - t0 < tc::kWaitCycles / 8) {
  }
}

__device__ __forceinline__ float exp_bf16_tab(float d, const uint16_t* tab) {
  // DT(exp(d)) for a bf16 value d <= 0 or NaN (NaN -> 0), from the table
  uint32_t a = (__float_as_uint(d) >> 16) & 0x7FFFu;
  a = a < EXPB ? EXPB : (a > EXPB + EXPN - 1 ? EXPB + EXPN - 1 : a);
  return __uint_as_float((uint32_t)tab[a - EXPB] << 16);
}

// Slot descriptor of (slice g, group, slot): the logit row (>= 0 a parent row
// of the codebook, <= -2 the child row -2 - x, -1 zeros), the value row (same
// encoding over the parent / child sums), the count in the dtype (-1: empty
// slot) and the logit mask.
struct SlotDesc {
  int lrow, vrow;
  float n, mk;
};

template <int DT, int C>
__global__ void corr_desc_kernel(const int* __restrict__ sel, int sel_stride, const int* __restrict__ pass_cnt,
                                 int npass, PassOffsets po, int multipass, int H, int M0,
                                 const int* __restrict__ pcnt, const int* __restrict__ ccnt, int maxgroups,
                                 SlotDesc* __restrict__ desc, int sG) {
  constexpr int J = NS / (1 + C), NREAL = J * (1 + C);
  const int g = blockIdx.x, h = g % H, gs = g % sG;
  const int* sg = sel + (long)g * sel_stride;
  int kg = 0;
  for (int ps = 0; ps < npass; ++ps) {
    const int cnt = pass_cnt[ps];
    if (cnt <= 0) break;
    const bool quirk = multipass && cnt == M0;  // refinement.py:256-260
    for (int j0 = 0; j0 < cnt && kg < maxgroups; j0 += J, ++kg) {
      for (int r = threadIdx.x; r < NS; r += blockDim.x) {
        SlotDesc d{-1, -1, -1.f, 0.f};
        if (r < J) {
          const int j = j0 + r;
          if (j < cnt) {
            const int p = sg[po.off[ps] + j];
            d.lrow = h * M0 + p;
            d.vrow = gs * M0 + p;
            d.n = count_dt<DT>(pcnt[(long)gs * M0 + p]);
            d.mk = d.n > 0.f ? 1.f : 0.f;
          }
        } else if (r < NREAL) {
          const int jj = (r - J) / C, c = (r - J) % C, j = j0 + jj;
          if (j < cnt) {
            const int p = sg[po.off[ps] + j];
            const int pl = quirk ? j : p;
            d.lrow = -2 - ((h * M0 + pl) * C + c);
            d.vrow = -2 - ((gs * M0 + p) * C + c);
            d.n = count_dt<DT>(ccnt[((long)gs * M0 + p) * C + c]);
            d.mk = ccnt[((long)gs * M0 + pl) * C + c] > 0 ? 1.f : 0.f;
          }
        }
        desc[((long)g * maxgroups + kg) * NS + r] = d;
      }
    }
  }
}

// MK: a user / causal mask is applied (present != nullptr); compiled out otherwise.
template <int DT, int D, int C, bool MK>
__global__ void __launch_bounds__(CTHREADS2, 2) correct_tc_kernel(
    const __grid_constant__ CUtensorMap tm_q, int4 qpos, int H, int Tq, float sqrtD,
    const typename Storage<DT>::T* __restrict__ parents, const typename Storage<DT>::T* __restrict__ children,
    const typename Storage<DT>::T* __restrict__ pagg, const typename Storage<DT>::T* __restrict__ cagg,
    const float* __restrict__ m_in, const float* __restrict__ l_in, const float* __restrict__ z_in,
    const float* __restrict__ beta_in, const typename Storage<DT>::T* __restrict__ a_in,
    const int* __restrict__ pass_cnt, int npass, int maxgroups, const SlotDesc* __restrict__ desc,
    const uint16_t* __restrict__ exptab_g, float* __restrict__ out, Strides3 os, int M0,
    const unsigned int* __restrict__ present) {
  using T = typename Storage<DT>::T;
  constexpr bool SPLIT = DT == DT_F16;  // fp16 value rows become two bf16 planes
  constexpr int J = NS / (1 + C), NREAL = J * (1 + C), CPR = D / 8;
  constexpr int OCOL = 0, SCOL = D, WCOL = D + NS;  // TMEM columns
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = tc::smem_addr(smem_raw);
  unsigned char* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  const CorrLayout L = corr_layout(D, SPLIT, MK);
  const int g = blockIdx.y, b = g / H, h = g % H, t0 = blockIdx.x * CR;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L.bars);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + L.misc);
  volatile int* abort = reinterpret_cast<volatile int*>(sm + L.misc + 4);
  const uint16_t* exptab = reinterpret_cast<const uint16_t*>(sm + L.exptab);

  // groups per pass (the same sequence on every thread)
  int ngroups = 0;
  for (int ps = 0; ps < npass; ++ps) {
    const int cnt = pass_cnt[ps];
    if (cnt <= 0) break;
    ngroups += (cnt + J - 1) / J;
  }
  ngroups = min(ngroups, maxgroups);

  if (tid == 0) {
    for (int i = 0; i < CN_BARS; ++i) {
      const int cnt = ((i >= CB_FULL && i < CB_FULL + NBUF) || i == CB_SFREE || i == CB_WFULL || i == CB_XCH ||
                       i == CB_XFREE)
                          ? 2 * CR
                          : 1;
      tc::mbar_init(&bars[i], cnt);
    }
    *abort = 0;
    tc::fence_mbar_init();
    // the Q tile, issued at once
    tc::tma_prefetch_desc(&tm_q);
    tc::mbar_expect_tx(&bars[CB_Q], CR * D * 2);
    for (int kb = 0; kb < D / 64; ++kb) {
      int c[4];
      c[0] = kb * 64;
      c[qpos.x] = t0;
      c[qpos.y] = h;
      c[qpos.z] = b;
      tc::tma_load_4d(sm + L.q + kb * CR * 128, &tm_q, c[0], c[1], c[2], c[3], &bars[CB_Q]);
    }
  }
  if (warp == MW) tc::tmem_alloc(tslot, C_TMEM_COLS);
  if (DT == DT_BF16 && tid < 2 * CR) {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(exptab_g);
    uint32_t* dst = reinterpret_cast<uint32_t*>(sm + L.exptab);
    for (int i = tid; i < (EXPN + 1) / 2; i += 2 * CR) dst[i] = src[i];
  }
  // ---- the row threads' prologue, before the CTA barrier so that its loads
  // (row statistics, the seed a, the first two groups' slot rows) overlap
  // the set-up: two threads per query.  Warps 0-3 (half 0) and 4-7 (half 1)
  // both reach TMEM lane r; half h takes slots 24h..24h+23 of every group
  // and the output columns [h D/2, (h+1) D/2).  Threads r < 48 of half 0
  // gather the logit row of slot r, those of half 1 its value row.
  const bool rowt = warp != MW;
  const int hf = tid >> 7, r = tid & (CR - 1), t = t0 + r;
  const bool live = rowt && t < Tq;
  const long row = (long)g * Tq + (live ? t : 0);
  const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
  constexpr int XCOL = WCOL + 3 * (NS / 2);  // 8 free columns: the halves' weight sums
  static_assert(XCOL + 8 <= C_TMEM_COLS, "TMEM columns");
  const float inv_sqrtD = 1.f / sqrtD;
  const float2 invl2 = make_float2(next_down(inv_sqrtD), next_down(inv_sqrtD));  // <= 1/sqrt(D)
  const float2 invh2 = make_float2(next_up(inv_sqrtD), next_up(inv_sqrtD));      // >= 1/sqrt(D)
  const float m = live ? m_in[row] : 0.f;
  const float zc = clamp_min_nan(live ? z_in[row] : 1.f, eps_dt<DT>()), rz = 1.f / zc;
  const float zl = next_down(rz), zh = next_up(rz);  // bracket 1 / zc
  const float bt = beta_in && live ? beta_in[row] : 0.f;
  // the row's mask words (pipeline.py:82-106): a masked parent has probability 0
  const unsigned int* prow = (MK && live) ? present + row * ((M0 + 31) >> 5) : nullptr;
  float l = live ? l_in[row] : 1.f;
  const int gslot = r;
  const bool gathers = rowt && r < NS, isv = hf == 1;
  const SlotDesc* dg = desc + (long)g * maxgroups * NS + gslot;
  auto gather = [&](int kg, const SlotDesc& d) {
    const int bf = kg % NBUF;
    if (gathers) {
      const int x = isv ? d.vrow : d.lrow;
      const T* src = x >= 0 ? (isv ? pagg : parents) + (long)x * D
                            : (isv ? cagg : children) + (long)(x <= -2 ? -2 - x : 0) * D;
      unsigned char* dst = sm + (isv ? L.v[bf] : L.l[bf]) + gslot * 128;
#pragma unroll
      for (int ch = 0; ch < CPR; ++ch)
        cp_async16(dst + (ch >> 3) * NS * 128 + (((ch & 7) ^ (gslot & 7)) << 4), src + ch * 8, x != -1);
      if (!isv) {
        float* meta = reinterpret_cast<float*>(sm + L.meta[bf]);
        meta[gslot] = d.n;
        meta[NS + gslot] = d.mk;
        if constexpr (MK)
          reinterpret_cast<int*>(meta)[2 * NS + gslot] = (gslot < J && d.lrow >= 0) ? d.lrow - h * M0 : -1;
      }
    }
    cp_async_commit();
  };
  auto publish = [&](int kg) {  // copies of group kg have landed (this thread's part)
    if constexpr (SPLIT) {
      // the value row this thread gathered: fp16 -> bf16 hi (in place) + bf16 lo
      if (gathers && isv) {
        const int bf = kg % NBUF;
#pragma unroll
        for (int ch = 0; ch < CPR; ++ch) {
          const int off = (ch >> 3) * NS * 128 + gslot * 128 + (((ch & 7) ^ (gslot & 7)) << 4);
          uint4* vh = reinterpret_cast<uint4*>(sm + L.v[bf] + off);
          uint4* vl = reinterpret_cast<uint4*>(sm + L.vlo[bf] + off);
          const uint4 u = *vh;
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
          uint32_t hi[4], lo[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float a0 = half_lo<DT_F16>(w[e]), a1 = half_hi<DT_F16>(w[e]);
            hi[e] = pack2<DT_BF16>(a0, a1);
            // exact remainders; an infinite sum keeps lo = 0 so that w * v stays infinite
            const float r0 = isinf(a0) ? 0.f : a0 - half_lo<DT_BF16>(hi[e]);
            const float r1 = isinf(a1) ? 0.f : a1 - half_hi<DT_BF16>(hi[e]);
            lo[e] = pack2<DT_BF16>(r0, r1);
          }
          *vh = make_uint4(hi[0], hi[1], hi[2], hi[3]);
          *vl = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
      }
    }
    tc::fence_async_smem();
    tc::mbar_arrive(&bars[CB_FULL + kg % NBUF]);
  };
  // this half's columns of the parent pass's a (attention.py:154-158), loaded
  // first so that their latency overlaps the first gathers
  uint4 a_seed[D / 16];
#pragma unroll
  for (int k = 0; k < D / 16; ++k)
    a_seed[k] = live ? reinterpret_cast<const uint4*>(a_in + row * D + hf * (D / 2))[k] : make_uint4(0u, 0u, 0u, 0u);
  SlotDesc dn1{-1, -1, -1.f, 0.f}, dn2{-1, -1, -1.f, 0.f};  // descriptors of the next groups
  if (gathers) {
    // the first descriptors at once, then the first two groups' rows
    const SlotDesc d0 = ngroups > 0 ? dg[0] : SlotDesc{-1, -1, -1.f, 0.f};
    if (ngroups > 1) dn1 = dg[NS];
    if (ngroups > 2) dn2 = dg[2 * NS];
    if (ngroups > 0) gather(0, d0);
    else cp_async_commit();
  } else if (rowt) {
    cp_async_commit();
  }
  if (rowt) {
    if (ngroups > 1) gather(1, dn1);
    else cp_async_commit();
  }
  tc::tc_before_sync();
  __syncthreads();
  tc::tc_after_sync();
  const uint32_t tbase = *tslot;

  if (warp == MW) {
    // ---- MMA issue (thread 0 issued the Q tile) ----
    if (lane == 0) {
      const uint32_t idS = tc::idesc_f16(DT == DT_BF16 ? 1 : 0, CR, NS, false);
      const uint32_t idO = tc::idesc_f16(1, CR, D, true);  // bf16 weights x bf16 value planes
      const uint32_t qa = tc::smem_addr(sm + L.q);
      uint32_t la[NBUF], va[NBUF], vla[NBUF];
      for (int i = 0; i < NBUF; ++i) {
        la[i] = tc::smem_addr(sm + L.l[i]);
        va[i] = tc::smem_addr(sm + L.v[i]);
        vla[i] = tc::smem_addr(sm + L.vlo[i]);
      }
      auto issue_S = [&](int kg) -> bool {
        const int bf = kg % NBUF;
        if (!tc::mbar_wait(&bars[CB_FULL + bf], (kg / NBUF) & 1, abort)) return false;
        tc::tc_after_sync();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t ad = tc::sdesc_sw128(qa + (kk >> 2) * CR * 128 + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = tc::sdesc_sw128(la[bf] + (kk >> 2) * NS * 128 + (kk & 3) * 32, 16, 1024);
          tc::mma_ss(tbase + SCOL, ad, bd, idS, kk > 0);
        }
        tc::mma_commit(&bars[CB_SFULL]);
        return true;
      };
      bool ok = tc::mbar_wait(&bars[CB_Q], 0, abort);
      if (ok && ngroups > 0) ok = issue_S(0);
      for (int kg = 0; ok && kg < ngroups; ++kg) {
        const int bf = kg % NBUF;
        if (kg + 1 < ngroups) {
          if (!(ok = tc::mbar_wait(&bars[CB_SFREE], kg & 1, abort))) break;
          if (!(ok = issue_S(kg + 1))) break;
        }
        if (!(ok = tc::mbar_wait(&bars[CB_WFULL], kg & 1, abort))) break;
        tc::tc_after_sync();
#pragma unroll
        for (int vp = 0; vp < (SPLIT ? 2 : 1); ++vp)
#pragma unroll
          for (int part = 0; part < 3; ++part)
#pragma unroll
            for (int kk = 0; kk < NS / 16; ++kk) {
              const uint64_t bd = tc::sdesc_sw128((vp ? vla[bf] : va[bf]) + kk * 16 * 128, NS * 128, 1024);
              tc::mma_ts(tbase + OCOL, tbase + WCOL + part * (NS / 2) + kk * 8, bd, idO, true);
            }
        tc::mma_commit(&bars[CB_WFREE]);
        tc::mma_commit(&bars[CB_EMPTY + bf]);
      }
      tc::mma_commit(&bars[CB_OFULL]);
      if (!ok) drain_c(&bars[CB_OFULL], 0);
    }
  } else {
    // ---- row threads ----
    cp_async_wait<1>();
    if (ngroups > 0) publish(0);
    // O = a, this half's columns
#pragma unroll
    for (int d0 = 0; d0 < D / 2; d0 += 32) {
      const int dc = hf * (D / 2) + d0;
      uint32_t o[32];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint4 u = a_seed[d0 / 8 + k];
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          o[8 * k + 2 * e] = __float_as_uint(half_lo<DT>(w[e]));
          o[8 * k + 2 * e + 1] = __float_as_uint(half_hi<DT>(w[e]));
        }
      }
      tc::tmem_st32(tbase + lane_off + OCOL + dc, o);
    }
    tc::tmem_wait_st();
    bool ok = true;
    int kg = 0, npass_done = 0;
    for (int ps = 0; ok && ps < npass; ++ps) {
      const int cnt = pass_cnt[ps];
      if (cnt <= 0) break;
      double rl = 0.0, al = 0.0;
      for (int j0 = 0; j0 < cnt && kg < ngroups; j0 += J, ++kg) {
        const int bf = kg % NBUF;
        ok = __all_sync(0xffffffffu, tc::mbar_wait(&bars[CB_SFULL], kg & 1, abort) &&
                                         tc::mbar_wait(&bars[CB_FULL + bf], (kg / NBUF) & 1, abort));
        if (!ok) break;
        tc::tc_after_sync();
        uint32_t sv[24];
        {
          uint32_t sa[16], sb[8];
          tc::tmem_ld16(tbase + lane_off + SCOL + 24 * hf, sa);
          tc::tmem_ld8(tbase + lane_off + SCOL + 24 * hf + 16, sb);
          tc::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 24; ++i) sv[i] = i < 16 ? sa[i] : sb[i - 16];
        }
        tc::tc_before_sync();
        tc::mbar_arrive(&bars[CB_SFREE]);
        // publish group kg + 1 (gathered a group ago); group kg + 2 is gathered
        // after the weights, when the value MMAs of group kg - 1 that read its
        // buffer have had time to finish
        cp_async_wait<0>();
        if (kg + 1 < ngroups) publish(kg + 1);
        const float* meta = reinterpret_cast<const float*>(sm + L.meta[bf]);
        // logits DT(DT(acc) / sqrt(D)): |x| / sqrt(D) lies between RD(|x| invl)
        // and RU(|x| invh); when both round to the same dtype value, so does
        // the correctly rounded quotient (sign copied back); else exact redo
        float sl[24];
        bool near = false;
        if constexpr (D == 64) {
          // sqrt(64) = 8: DT(x / 8) is exact in fp32, one packed multiply by 1/8
#pragma unroll
          for (int i2 = 0; i2 < 12; ++i2) {
            const int i = 2 * i2;
            const uint32_t s2 = hmul2_dt<DT>(pack2<DT>(__uint_as_float(sv[i]), __uint_as_float(sv[i + 1])),
                                             dup2<DT>(0.125f));
            sl[i] = half_lo<DT>(s2);
            sl[i + 1] = half_hi<DT>(s2);
          }
        } else {
#pragma unroll
        for (int i2 = 0; i2 < 12; ++i2) {
          const int i = 2 * i2;
          const uint32_t x2 = pack2<DT>(__uint_as_float(sv[i]), __uint_as_float(sv[i + 1]));
          const uint32_t a2 = x2 & 0x7FFF7FFFu;
          const float2 av = make_float2(half_lo<DT>(a2), half_hi<DT>(a2));
          const float2 ylo = mul_f32x2_rd(av, invl2), yhi = mul_f32x2_ru(av, invh2);
          const uint32_t qlo = pack2<DT>(ylo.x, ylo.y);
          near |= qlo != pack2<DT>(yhi.x, yhi.y);
          const uint32_t s2 = qlo | (x2 & 0x80008000u);
          sl[i] = half_lo<DT>(s2);
          sl[i + 1] = half_hi<DT>(s2);
        }
        }
        if (near) {
#pragma unroll
          for (int i = 0; i < 24; ++i) sl[i] = scale_logit<DT>(rnd<DT>(__uint_as_float(sv[i])), sqrtD, inv_sqrtD);
        }
        // weights (fp32; refinement.py:335,341-343): -exp(pi - m) n for a parent,
        // exp(u - m) n_c for a child, 0 for an empty slot
        float wv[24];
        float rlg = 0.f, alg = 0.f;
        uint32_t pbad = 0u;  // parent slots whose quotient is redone
        float pe[J];         // their exponentials
        // the slot kinds of a half are fixed: one copy of the loop per half
        auto weights = [&](auto hfc) {
          constexpr int HF = decltype(hfc)::value;
          const float4* mn4 = reinterpret_cast<const float4*>(meta + 24 * HF);
          const float4* mk4 = reinterpret_cast<const float4*>(meta + NS + 24 * HF);
#pragma unroll
          for (int q = 0; q < 6; ++q) {
            const float4 n4 = mn4[q], k4 = mk4[q];
            const float nv[4] = {n4.x, n4.y, n4.z, n4.w}, kv[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int i = 4 * q + e, k = 24 * HF + i;
              float w = 0.f;
              if (k < NREAL) {
                float s = kv[e] > 0.f ? sl[i] : -INFINITY;
                if constexpr (MK) {
                  if (k < J && prow) {
                    const int pp = reinterpret_cast<const int*>(meta)[2 * NS + k];
                    if (pp >= 0 && !((prow[pp >> 5] >> (pp & 31)) & 1u)) s = -INFINITY;
                  }
                }
                if (k < J) {
                  if (beta_in) s = rnd<DT>(__fmul_rn(bt, rnd<DT>(__fmul_rn(s, sqrtD))));
                  float ex;
                  if constexpr (DT == DT_BF16) ex = exp_bf16_tab(rnd<DT>(s - m), exptab);
                  else ex = fmaxf(exp_dt_fast<DT>(rnd<DT>(s - m)), 0.f);  // NaN -> 0
                  // pi = DT(e / z): e / z lies between RD(e zl) and RU(e zh)
                  // (e >= 0); ends that round apart are redone exactly below
                  const float pi = rnd<DT>(__fmul_rd(ex, zl));
                  if (pi != rnd<DT>(__fmul_ru(ex, zh))) pbad |= 1u << i;
                  pe[i] = ex;
                  w = nv[e] >= 0.f ? -__expf(pi - m) * nv[e] : 0.f;  // summed into rlg below
                } else {
                  w = nv[e] >= 0.f ? __expf(s - m) * nv[e] : 0.f;
                  alg += w;
                }
              }
              wv[i] = w;
            }
          }
        };
        if (hf == 0) weights(std::integral_constant<int, 0>{});
        else weights(std::integral_constant<int, 1>{});
        if (__any_sync(0xffffffffu, pbad != 0u)) {
#pragma unroll
          for (int i = 0; i < J; ++i) {
            if ((pbad >> i) & 1u) {  // only half 0 holds parent slots
              const float pi = rnd<DT>(__fdiv_rn(pe[i], zc));
              const float nvi = meta[i];
              wv[i] = nvi >= 0.f ? -__expf(pi - m) * nvi : 0.f;
            }
          }
        }
        if (hf == 0) {
#pragma unroll
          for (int i = 0; i < J; ++i) rlg += -wv[i];  // slot order, as the weights were made
        }
        rl += (double)rlg;
        al += (double)alg;
        if (kg + 2 < ngroups) {
          const int nb = (kg + 2) % NBUF;
          if (kg + 2 >= NBUF) {
            ok = __all_sync(0xffffffffu, tc::mbar_wait(&bars[CB_EMPTY + nb], ((kg + 2) / NBUF - 1) & 1, abort));
            if (!ok) break;
          }
          gather(kg + 2, dn2);
          if (gathers && kg + 3 < ngroups) dn2 = dg[(long)(kg + 3) * NS];
        }
        // three bf16 parts per weight (w = hi + mid + lo to 24 bits), packed in pairs
        uint32_t wp[3][12];
#pragma unroll
        for (int i2 = 0; i2 < 12; ++i2) {
          const float w0 = wv[2 * i2], w1 = wv[2 * i2 + 1];
          const uint32_t h2 = pack2<DT_BF16>(w0, w1);
          const float r0 = w0 - half_lo<DT_BF16>(h2), r1 = w1 - half_hi<DT_BF16>(h2);
          const uint32_t m2 = pack2<DT_BF16>(r0, r1);
          wp[0][i2] = h2;
          wp[1][i2] = m2;
          wp[2][i2] = pack2<DT_BF16>(r0 - half_lo<DT_BF16>(m2), r1 - half_hi<DT_BF16>(m2));
        }
        if (kg > 0) {  // the previous group's value MMAs have read the weight columns
          ok = __all_sync(0xffffffffu, tc::mbar_wait(&bars[CB_WFREE], (kg - 1) & 1, abort));
          if (!ok) break;
          tc::tc_after_sync();
        }
#pragma unroll
        for (int part = 0; part < 3; ++part) {
          tc::tmem_st8(tbase + lane_off + WCOL + part * (NS / 2) + 12 * hf, wp[part]);
          tc::tmem_st4(tbase + lane_off + WCOL + part * (NS / 2) + 12 * hf + 8, wp[part] + 8);
        }
        tc::tmem_wait_st();
        tc::tc_before_sync();
        tc::mbar_arrive(&bars[CB_WFULL]);
      }
      if (!ok) break;
      // the two halves' weight sums meet in TMEM; OnlineSoftmaxState.replace
      // with unit scales (attention.py:149-153)
      if (npass_done > 0) {
        ok = __all_sync(0xffffffffu, tc::mbar_wait(&bars[CB_XFREE], (npass_done - 1) & 1, abort));
        if (!ok) break;
        tc::tc_after_sync();
      }
      {
        const unsigned long long rb = __double_as_longlong(rl), ab = __double_as_longlong(al);
        const uint32_t xv[4] = {(uint32_t)rb, (uint32_t)(rb >> 32), (uint32_t)ab, (uint32_t)(ab >> 32)};
        tc::tmem_st4(tbase + lane_off + XCOL + 4 * hf, xv);
        tc::tmem_wait_st();
      }
      tc::tc_before_sync();
      tc::mbar_arrive(&bars[CB_XCH]);
      ok = __all_sync(0xffffffffu, tc::mbar_wait(&bars[CB_XCH], npass_done & 1, abort));
      if (!ok) break;
      tc::tc_after_sync();
      uint32_t xo[4];
      tc::tmem_ld4(tbase + lane_off + XCOL + 4 * (1 - hf), xo);
      tc::tmem_wait_ld();
      tc::tc_before_sync();
      tc::mbar_arrive(&bars[CB_XFREE]);
      const double rlo = __longlong_as_double((long long)(((unsigned long long)xo[1] << 32) | xo[0]));
      const double alo = __longlong_as_double((long long)(((unsigned long long)xo[3] << 32) | xo[2]));
      const double rlt = hf == 0 ? rl + rlo : rlo + rl, alt = hf == 0 ? al + alo : alo + al;
      l = __fadd_rn(__fsub_rn(l, __double2float_rn(rlt)), __double2float_rn(alt));
      ++npass_done;
    }
    cp_async_wait<0>();
    if (ok) ok = __all_sync(0xffffffffu, tc::mbar_wait(&bars[CB_OFULL], 0, abort));
    // every row thread takes the same branch below (one vote), so the barrier matches
    if (corr_rows_all(ok)) {
      tc::tc_after_sync();
      // the output tile goes through the idle Q, slot-row and value buffers, so
      // that each warp stores whole rows (512 contiguous bytes) instead of 32
      // rows' 16-byte pieces
      constexpr int SLD = D + 4;  // padded row: the 16-byte writes of a warp hit distinct banks
      static_assert(CR * SLD * 4 <= CR * D * 2 + 2 * NBUF * NS * D * 2, "output staging");
      float* stg = reinterpret_cast<float*>(sm + L.q);
      const float rden = __fdiv_rn(1.f, clamp_min_nan(l, 1e-12f));
#pragma unroll
      for (int d0 = 0; d0 < D / 2; d0 += 32) {
        const int dc = hf * (D / 2) + d0;
        uint32_t o[32];
        tc::tmem_ld32(tbase + lane_off + OCOL + dc, o);
        tc::tmem_wait_ld();
#pragma unroll
        for (int k = 0; k < 8; ++k)
          *reinterpret_cast<float4*>(stg + r * SLD + dc + 4 * k) =
              make_float4(__uint_as_float(o[4 * k]) * rden, __uint_as_float(o[4 * k + 1]) * rden,
                          __uint_as_float(o[4 * k + 2]) * rden, __uint_as_float(o[4 * k + 3]) * rden);
      }
      corr_rows_sync();
      constexpr int F4 = D / 4, RPI = 32 / F4;  // float4 per row, rows per warp instruction
      const int c4 = lane % F4;
#pragma unroll 4
      for (int i = 0; i < CR / 8; i += RPI) {
        const int rr = warp * (CR / 8) + i + lane / F4, tt = t0 + rr;
        if (tt < Tq)
          *reinterpret_cast<float4*>(out + (long)b * os.b + (long)tt * os.s + (long)h * os.h + 4 * c4) =
              *reinterpret_cast<const float4*>(stg + rr * SLD + 4 * c4);
      }
    }
  }

  tc::tc_before_sync();
  __syncthreads();
  if (warp == MW) {
    tc::tc_after_sync();
    tc::tmem_free(tbase, C_TMEM_COLS);
  }
  if (tid == 0 && *abort) atomicOr(&g_fault, 1);
}

}  // namespace

bool correct_tc_ok(int dt, int D, int C) {
  const char* e = std::getenv("AVQ_DISABLE_TCGEN05");
  const bool off = e && *e && *e != '0';
  return !off && (dt == DT_BF16 || dt == DT_F16) && (D == 64 || D == 128) && (C == 4 || C == 8);
}

int correct_tc_groups(int sel_stride, int C) {
  const int J = NS / (1 + C);
  return (sel_stride + 8 * (J - 1)) / J;  // every pass (at most 8) may end in a partial group
}

size_t correct_tc_desc_bytes(int G, int sel_stride, int C) {
  return (size_t)G * correct_tc_groups(sel_stride, C) * NS * sizeof(SlotDesc);
}

template <int DT>
int launch_correct_tc(const CorrArgs& a, const void* exptab, void* desc, cudaStream_t st) {
  using T = typename Storage<DT>::T;
  const int G = a.B * a.H, D = a.D;
  CUtensorMap tq;
  int4 qpos;
  if (!tc::map_rows4(&tq, DT, a.q, a.qs, a.B, a.H, a.T, D, CR, &qpos)) return AVQ_ERR_UNSUPPORTED;
  if (((uintptr_t)a.out % 16) || a.os.s % 4 || a.os.h % 4 || a.os.b % 4) return AVQ_ERR_UNSUPPORTED;
  PassOffsets po;
  for (int k = 0; k < 8; ++k) po.off[k] = a.pass_off[k];
  const int maxgroups = correct_tc_groups(a.sel_stride, a.C);
  SlotDesc* sd = static_cast<SlotDesc*>(desc);
  const bool mk = a.present != nullptr;
  const CorrLayout L = corr_layout(D, DT == DT_F16, mk);
  const size_t smem = std::max<size_t>((size_t)L.total + 1024, 80 * 1024);  // <= 2 CTAs (2 x 256 TMEM columns) per SM
  auto go = [&](auto dfn, auto kfn) {
    AVQ_TIMED("correct_tc", st);
    dfn<<<G, 64, 0, st>>>(a.sel, a.sel_stride, a.pass_cnt, a.npass, po, a.multipass, a.H, a.M0, a.pcnt, a.ccnt,
                          maxgroups, sd, a.sG > 0 ? a.sG : G);
    cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kfn<<<dim3((a.T + CR - 1) / CR, G), CTHREADS2, smem, st>>>(
        tq, qpos, a.H, a.T, a.sqrtD, static_cast<const T*>(a.parents), static_cast<const T*>(a.children),
        static_cast<const T*>(a.pagg), static_cast<const T*>(a.cagg), a.m, a.l, a.z, a.beta,
        static_cast<const T*>(a.a), a.pass_cnt, a.npass, maxgroups, sd, static_cast<const uint16_t*>(exptab), a.out,
        a.os, a.M0, a.present);
  };
  auto pick = [&](auto dfn, auto k_plain, auto k_masked) { mk ? go(dfn, k_masked) : go(dfn, k_plain); };
  if (a.C == 4) {
    if (D == 64) pick(corr_desc_kernel<DT, 4>, correct_tc_kernel<DT, 64, 4, false>, correct_tc_kernel<DT, 64, 4, true>);
    else pick(corr_desc_kernel<DT, 4>, correct_tc_kernel<DT, 128, 4, false>, correct_tc_kernel<DT, 128, 4, true>);
  } else {
    if (D == 64) pick(corr_desc_kernel<DT, 8>, correct_tc_kernel<DT, 64, 8, false>, correct_tc_kernel<DT, 64, 8, true>);
    else pick(corr_desc_kernel<DT, 8>, correct_tc_kernel<DT, 128, 8, false>, correct_tc_kernel<DT, 128, 8, true>);
  }
  return cudaPeekAtLastError() == cudaSuccess ? AVQ_OK : AVQ_ERR_CUDA;
}

template int launch_correct_tc<DT_BF16>(const CorrArgs&, const void*, void*, cudaStream_t);
template int launch_correct_tc<DT_F16>(const CorrArgs&, const void*, void*, cudaStream_t);

// Reads and clears this file's fault word (device code without relocatable
// linking keeps one copy per file, so every kernel file has its own).
int read_fault_correct(int* code, cudaStream_t st) {
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
