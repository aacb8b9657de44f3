// Parent attention on the sm_100a tensor cores (tcgen05 + TMEM + TMA) for
// bf16 / fp16 and D in {64, 128} (reference pipeline.py:46-151, :322-339 and
// routing.py:61-63): the parent logits, their softmax statistics, the value
// sums a = e @ V and the per-parent importance partials of the first routing
// pass.
//
// CTA = 128 queries of one (b,h) = one UMMA M tile.  Each query row has two
// threads (warps w and w+4 share TMEM lane quarter w): half hf takes parents
// 32hf..32hf+31 of every 64-parent chunk, and the halves combine their row
// statistics once per pass.  Warp 8 issues the tcgen05.mma instructions;
// warp 9 streams Q, parent and parent-sum tiles with TMA into
// 128-byte-swizzled shared memory: after Q, one ring of four tile buffers
// takes the parent tiles of pass 1 and then the parent and parent-sum tiles
// of pass 2 alternately, in that order.
//
// TMEM, 256 columns: the fp32 accumulator O = e @ V in [0, D) and two
// 64-column logit slots at [D, D+64) and [D+64, D+128).  A slot receives one
// 64-parent chunk of Q P^T; in the second pass half hf overwrites the first
// 16 of its 32 columns with its 32 dtype exponentials (two per column), the A
// operand of the e @ V MMA (K steps at columns 0, 8, 32, 40).  Pass 1, which
// leaves O unused, has two more logit slots in O's columns (and past D + 128
// for D = 64), so four chunks are in flight.
//
//   pass 1  S_c = Q P_c^T for every chunk c; row max of the narrowed,
//           scaled, masked logits.
//   pass 2  S_c again (the tensor cores recompute it instead of a round trip
//           through memory); e = DT(exp(DT(s - m))), l += DT(e * n), z += e;
//           e -> TMEM -> O += e V_c; e -> the scratch slice that the routing
//           kernel reads for its exact fallback.
//   pass 3  probs = DT(e / max(z, eps)) summed over each 64-query tile per
//           parent (fp32 partials, within 2^-19 relative of the exact sums).
//
// Rounding points are those of the reference (see avq_common.cuh); for bf16
// the exponential comes from a table of DT(correctly rounded fp32 exp(x))
// over every bf16 x in [-128, -2^-9].
#include <cuda.h>

#include <algorithm>
#include <cstdlib>

#include "avq_kernels.cuh"
#include "avq_mma.cuh"
#include "avq_tc.cuh"

namespace avq {

namespace {
// Bit 0: a CTA of this file gave up on a bounded wait (read by avq_device_fault).
__device__ int g_fault;
}  // namespace

namespace {

constexpr int TR = 128;        // queries per CTA
constexpr int TCH = 64;        // parents per chunk
constexpr int TROW = 256;      // two row threads per query
constexpr int TTHREADS = 320;  // 8 row warps + MMA warp + TMA warp
constexpr int W_MMA = 8, W_TMA = 9;
constexpr int TC_TMEM_COLS = 256;
constexpr uint32_t EXP_BASE = 0x3AFF;  // bf16 bits of the largest |d| whose exp rounds to 1
constexpr int EXP_N = 2051;            // entries 0..2049: |d| bits EXP_BASE + i; 2050: |d| > 128, inf, NaN
constexpr int EXP_WORDS = (EXP_N + 1) / 2;
constexpr int TC_MAX_M0 = 8192;  // above 2048 the shared memory allows one CTA per SM

// Barrier slots: the tile ring's full and empty barriers, the logit slots'
// full (MMA done) and consumed (row threads done) barriers.
// HVAQ mode adds the gathered selected-parent tile (B_SEL: its 32 gathering
// lanes) and the row threads' temperatures (B_BETA: all 256 row threads).
constexpr int B_Q = 0, B_RFULL = 1, B_REMPTY = 5, B_SFULL = 9, B_EFULL = 13, B_SFREE = 17, B_OFULL = 18, B_SEL = 19,
              B_BETA = 20, N_BARS = 21;
constexpr int NRING = 4;  // tile ring buffers (the layout's p[0], p[1], v[0], v[1], contiguous)

// TMEM column of logit slot k; slots 2 and 3 only in pass 1.
template <int D>
__device__ __forceinline__ uint32_t s_col(int k) {
  return k < 2 ? D + 64 * k : (D == 128 ? 64 * (k - 2) : (k == 2 ? 0 : D + 128));
}

struct TcLayout {
  int q, p[2], v[2], sel, exptab, pm2, n2, srow, scomb, xch, bars, misc, total;
};

// hv: the HVAQ rescaling pass, which also holds one tile of gathered parent
// rows (the first routing pass's selection).
__host__ __device__ inline TcLayout tc_layout(int D, int M0, bool hv = false) {
  TcLayout L;
  const int nch = (M0 + TCH - 1) / TCH;
  int o = 0;
  L.q = o;
  o += TR * D * 2;
  for (int i = 0; i < 2; ++i) {
    L.p[i] = o;
    o += TCH * D * 2;
  }
  for (int i = 0; i < 2; ++i) {
    L.v[i] = o;
    o += TCH * D * 2;
  }
  L.sel = o;
  if (hv) o += TCH * D * 2;
  L.exptab = o;
  o += EXP_WORDS * 4;
  o = (o + 15) & ~15;
  L.pm2 = o;
  o += nch * 32 * 4;
  L.n2 = o;
  o += nch * 32 * 4;
  L.srow = o;
  o += TR * 4 * 4;
  L.scomb = o;
  o += 2 * 8 * 64 * 4;
  // the halves' row statistics [3][2][TR] before pass 3: pass 3 writes the
  // combine buffers only after its first staging barrier, which every row
  // thread reaches after its last exchange read
  L.xch = L.scomb;
  L.bars = o;
  o += N_BARS * 8;
  L.misc = o;
  o += 16;
  L.total = o;
  return L;
}

// DT(x / sqrt(D)) of the dtype-narrowed fp32 accumulators a0, a1, with -inf
// where `keep` (0xFFFF per live half) is clear -- empty parents
// (pipeline.py:81,107).
template <int DT>
__device__ __forceinline__ uint32_t logit2(uint32_t a0, uint32_t a1, float sqrtD, float inv, uint32_t keep) {
  const uint32_t x2 = pack2<DT>(__uint_as_float(a0), __uint_as_float(a1));
  const float x0 = half_lo<DT>(x2), x1 = half_hi<DT>(x2);
  float y0 = x0 * inv, y1 = x1 * inv;  // within 2 ulp of the correctly rounded quotient
  if (near_midpoint<DT>(y0)) y0 = __fdiv_rn(x0, sqrtD);
  if (near_midpoint<DT>(y1)) y1 = __fdiv_rn(x1, sqrtD);
  const uint32_t s2 = pack2<DT>(y0, y1);
  const uint32_t ninf = DT == DT_BF16 ? 0xFF80FF80u : 0xFC00FC00u;
  return (s2 & keep) | (ninf & ~keep);
}

// DT(exp(d)) for both halves of d2 (every d <= 0 or NaN); NaN -> 0
// (pipeline.py:143-145).
template <int DT>
__device__ __forceinline__ uint32_t exp2_dt(uint32_t d2, const uint16_t* tab) {
  if constexpr (DT == DT_BF16) {
    uint32_t c;
    asm("max.u16x2 %0, %1, %2;" : "=r"(c) : "r"(d2 & 0x7FFF7FFFu), "r"(EXP_BASE * 0x10001u));
    asm("min.u16x2 %0, %1, %2;" : "=r"(c) : "r"(c), "r"((EXP_BASE + EXP_N - 1) * 0x10001u));
    const uint32_t lo = tab[(c & 0xFFFFu) - EXP_BASE], hi = tab[(c >> 16) - EXP_BASE];
    return lo | (hi << 16);
  } else {
    const float e0 = fmaxf(exp_dt_fast<DT>(half_lo<DT>(d2)), 0.f);
    const float e1 = fmaxf(exp_dt_fast<DT>(half_hi<DT>(d2)), 0.f);
    return pack2<DT>(e0, e1);
  }
}

__global__ void exp_table_kernel(uint16_t* __restrict__ tab) {
  for (int i = threadIdx.x; i < 2 * EXP_WORDS; i += blockDim.x) {
    uint16_t v = 0;
    if (i < EXP_N - 1) {
      const float x = __uint_as_float((EXP_BASE + (uint32_t)i) << 16);
      v = __bfloat16_as_ushort(__float2bfloat16_rn(__double2float_rn(exp(-(double)x))));
    }
    tab[i] = v;
  }
}

__device__ __forceinline__ float fmax_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Bounded wait that ignores the abort flag (draining copies in flight).
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!tc::mbar_try(bar, parity) && clock64() - t0 < tc::kWaitCycles / 8) {
  }
}

// Barrier of the 256 row threads (the MMA and TMA warps do not take part).
__device__ __forceinline__ void rows_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
// The same barrier, returning whether `p` holds in every row thread.
__device__ __forceinline__ bool rows_all(bool p) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred a, b;\n\tsetp.ne.u32 a, %1, 0;\n\tbar.red.and.pred b, 1, 256, a;\n\tselp.u32 %0, 1, 0, b;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)p)
      : "memory");
  return r != 0;
}

// HV: the HVAQ rescaling pass (pipeline.py:192-258, hopfield.py:55-144).  It
// reads the plain pass's row max and normaliser from m_out / z_out (the same
// rows it then overwrites), the plain pass's selection sel0 (at most 64
// parents), and writes the per-query temperature beta_out; the logits of every
// later step are DT(beta * DT(s * sqrt(D))).
// MK: a user / causal mask is applied (present != nullptr); without it the
// mask code is compiled out, so unmasked calls run the same instructions as a
// kernel without mask support.
// DN: dense attention (the reference's naive_attention, backend.py:190-203):
// the "parents" and "parent sums" are the (b,h)'s own keys and values (4-D
// maps tm_p / tm_v at kvpos), every key counts once, the logits are
// DT(DT(acc) * scale) as the reference multiplies by its scale, and instead of
// the routing state the kernel writes out = DT(O / z) at `dout` (strides os);
// passes 1 and 2 only (no exponential slices, no importance partials).
template <int DT, int D, bool HV, bool MK, bool DN = false>
__global__ void __launch_bounds__(TTHREADS, 2) parent_attn_tc_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_p,
    const __grid_constant__ CUtensorMap tm_v, int4 qpos, int H, int Tq, int M0, float sqrtD,
    const int* __restrict__ pcnt, const uint16_t* __restrict__ exptab_g, typename Storage<DT>::T* __restrict__ scratch,
    float* __restrict__ m_out, float* __restrict__ l_out, float* __restrict__ z_out,
    typename Storage<DT>::T* __restrict__ a_out, float* __restrict__ colpart, int sG,
    const typename Storage<DT>::T* __restrict__ parents_g, const int* __restrict__ sel0, int sel_stride,
    const int* __restrict__ pass_cnt, int hvaq, float beta0, float alpha, float* __restrict__ beta_out,
    const unsigned int* __restrict__ present, int4 kvpos, float dscale, typename Storage<DT>::T* __restrict__ dout,
    Strides3 os) {
  static_assert(!DN || (!HV && !MK), "the dense mode has no HVAQ pass and no mask bits");
  using T = typename Storage<DT>::T;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = tc::smem_addr(smem_raw);
  unsigned char* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  const TcLayout L = tc_layout(D, M0, HV);
  const int g = blockIdx.y, b = g / H, h = g % H, qt = blockIdx.x, t0 = qt * TR, gs = g % sG;
  const int nch = (M0 + TCH - 1) / TCH, nv = 2 * nch;
  const int ntiles = (Tq + 63) / 64, LDL = exp_slice_pitch(M0);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L.bars);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + L.misc);
  volatile int* abort = reinterpret_cast<volatile int*>(sm + L.misc + 4);
  const uint16_t* exptab = reinterpret_cast<const uint16_t*>(sm + L.exptab);
  uint32_t* pm2 = reinterpret_cast<uint32_t*>(sm + L.pm2);
  uint32_t* n2 = reinterpret_cast<uint32_t*>(sm + L.n2);
  float* srow = reinterpret_cast<float*>(sm + L.srow);
  float* scomb = reinterpret_cast<float*>(sm + L.scomb);
  float* xch = reinterpret_cast<float*>(sm + L.xch);

  const int ntl = nch + nv;  // ring tiles: P_0..P_{nch-1}, then P_0, V_0, P_1, V_1, ...
  constexpr int RB = TCH * D * 2;
  // ring tile i into buffer i % NRING (expect_tx, then the 64-column boxes)
  auto load_tile = [&](int i) {
    const int k = i & (NRING - 1);
    unsigned char* buf = sm + L.p[0] + k * RB;
    tc::mbar_expect_tx(&bars[B_RFULL + k], RB);
    const bool par = i < nch || ((i - nch) & 1) == 0;
    const int c = i < nch ? i : (i - nch) >> 1;
    for (int kb = 0; kb < D / 64; ++kb) {
      if constexpr (DN) {  // keys / values of this (b,h): rows c*TCH.. of the 4-D map
        int cc[4];
        cc[0] = kb * 64;
        cc[kvpos.x] = c * TCH;
        cc[kvpos.y] = h;
        cc[kvpos.z] = b;
        tc::tma_load_4d(buf + kb * TCH * 128, par ? &tm_p : &tm_v, cc[0], cc[1], cc[2], cc[3], &bars[B_RFULL + k]);
      } else {
        if (par) tc::tma_load_3d(buf + kb * TCH * 128, &tm_p, kb * 64, c * TCH, h, &bars[B_RFULL + k]);
        else tc::tma_load_3d(buf + kb * TCH * 128, &tm_v, kb * 64, c * TCH, gs, &bars[B_RFULL + k]);
      }
    }
  };

  // ---- setup: barriers, TMEM, tables ----
  // The producer thread initialises the barriers and issues Q and the first
  // ring tiles at once, so the copies overlap the table fill.
  if (warp == W_TMA && lane == 0) {
    for (int i = 0; i < N_BARS; ++i)
      tc::mbar_init(&bars[i], ((i >= B_EFULL && i < B_EFULL + 4) || i == B_BETA) ? TROW : (i == B_SEL ? 32 : 1));
    *abort = 0;
    tc::fence_mbar_init();
    tc::tma_prefetch_desc(&tm_q);
    tc::tma_prefetch_desc(&tm_p);
    tc::tma_prefetch_desc(&tm_v);
    tc::mbar_expect_tx(&bars[B_Q], TR * D * 2);
    for (int kb = 0; kb < D / 64; ++kb) {
      int c[4];
      c[0] = kb * 64;
      c[qpos.x] = t0;
      c[qpos.y] = h;
      c[qpos.z] = b;
      tc::tma_load_4d(sm + L.q + kb * TR * 128, &tm_q, c[0], c[1], c[2], c[3], &bars[B_Q]);
    }
    for (int i = 0; i < NRING && i < ntl; ++i) load_tile(i);
  }
  if (warp == W_MMA) tc::tmem_alloc(tslot, TC_TMEM_COLS);
  if (tid < TROW) {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(exptab_g);
    uint32_t* dst = reinterpret_cast<uint32_t*>(sm + L.exptab);
    for (int i = tid; i < EXP_WORDS; i += TROW) dst[i] = src[i];
    for (int j = tid; j < nch * 32; j += TROW) {
      const int p = 2 * j;
      int c0, c1;
      if constexpr (DN) {  // every key counts once
        c0 = p < M0 ? 1 : 0;
        c1 = p + 1 < M0 ? 1 : 0;
      } else {
        c0 = p < M0 ? pcnt[(long)gs * M0 + p] : 0;
        c1 = p + 1 < M0 ? pcnt[(long)gs * M0 + p + 1] : 0;
      }
      pm2[j] = (c0 > 0 ? 0xFFFFu : 0u) | (c1 > 0 ? 0xFFFF0000u : 0u);
      n2[j] = pack2<DT>(count_dt<DT>(c0), count_dt<DT>(c1));
    }
  }
  tc::tc_before_sync();
  __syncthreads();
  tc::tc_after_sync();
  const uint32_t tbase = *tslot;

  if (warp == W_TMA) {
    if constexpr (HV) {
      // the plain pass's selected parents (head h rows), gathered in the
      // 128-byte-swizzled K-major layout of a TMA box: row j, 16-byte chunk c
      // of 64-column block kb at kb*TCH*128 + j*128 + ((c ^ j) & 7)*16; rows
      // past the selection are zero-filled
      const int nsel = min(pass_cnt[0], TCH);
      const int* sl = sel0 + (long)g * sel_stride;
      unsigned char* sb = sm + L.sel;
      for (int i = lane; i < TCH * (D / 8); i += 32) {
        const int j = i / (D / 8), c = i % (D / 8);
        const bool in = j < nsel;
        const int p = in ? sl[j] : 0;
        cp_async16(sb + (c >> 3) * TCH * 128 + j * 128 + (((c & 7) ^ (j & 7)) << 4),
                   parents_g + ((long)h * M0 + p) * D + c * 8, in);
      }
      cp_async_commit();
      cp_async_wait<0>();
      tc::fence_async_smem();
      tc::mbar_arrive(&bars[B_SEL]);
    }
    // ---- TMA producer: the rest of the ring, each buffer once its last tile is consumed ----
    if (lane == 0) {
      int issued = ntl < NRING ? ntl : NRING;
      for (int i = NRING; i < ntl; ++i) {
        if (!tc::mbar_wait(&bars[B_REMPTY + (i & (NRING - 1))], ((i >> 2) - 1) & 1, abort)) break;
        load_tile(i);
        issued = i + 1;
      }
      if (*abort) {  // let the copies in flight land before the CTA exits
        drain_wait(&bars[B_Q], 0);
        for (int k = 0; k < NRING && k < issued; ++k) drain_wait(&bars[B_RFULL + k], ((issued - 1 - k) >> 2) & 1);
      }
    }
  } else if (warp == W_MMA) {
    // ---- MMA issuer ----
    if (lane == 0) {
      const int fmt = DT == DT_BF16 ? 1 : 0;
      const uint32_t idS = tc::idesc_f16(fmt, TR, TCH, false);
      const uint32_t idO = tc::idesc_f16(fmt, TR, D, true);
      const uint32_t qa = tc::smem_addr(sm + L.q), ra0 = tc::smem_addr(sm + L.p[0]);
      // chunk w's logits in logit slot slot(w), from ring tile s_tile(w); the
      // e @ V MMA of second-pass chunk u reads ring tile nch + 2u + 1
      auto slot = [&](int w) { return w < nch ? (w & 3) : (w & 1); };
      auto s_tile = [&](int w) { return w < nch ? w : nch + 2 * (w - nch); };
      auto issue_S = [&](int w) {
        const int i = s_tile(w), k = i & (NRING - 1), sl = slot(w);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t ad = tc::sdesc_sw128(qa + (kk >> 2) * TR * 128 + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = tc::sdesc_sw128(ra0 + k * RB + (kk >> 2) * TCH * 128 + (kk & 3) * 32, 16, 1024);
          tc::mma_ss(tbase + s_col<D>(sl), ad, bd, idS, kk > 0);
        }
        tc::mma_commit(&bars[B_SFULL + sl]);
        tc::mma_commit(&bars[B_REMPTY + k]);
      };
      auto tile_ready = [&](int i) { return tc::mbar_wait(&bars[B_RFULL + (i & (NRING - 1))], (i >> 2) & 1, abort); };
      // the next chunk to use chunk v's logit slot, or -1.  The second pass
      // takes slots 0 and 1 after the first pass's last chunks there.
      auto next_user = [&](int v) {
        if (v >= nch) return v + 2 < nv ? v + 2 : -1;
        if (v + 4 < nch) return v + 4;
        const int k = v & 3, w = nch + ((k - nch) & 1);
        return k < 2 && w < nv ? w : -1;
      };
      bool ok = tc::mbar_wait(&bars[B_Q], 0, abort);
      if constexpr (HV) {
        // logits of the selected parents into slot 0; the first chunk takes the
        // slot again once every row thread has its temperature
        if (ok && (ok = tc::mbar_wait(&bars[B_SEL], 0, abort))) {
          tc::tc_after_sync();
          const uint32_t sa = tc::smem_addr(sm + L.sel);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint64_t ad = tc::sdesc_sw128(qa + (kk >> 2) * TR * 128 + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = tc::sdesc_sw128(sa + (kk >> 2) * TCH * 128 + (kk & 3) * 32, 16, 1024);
            tc::mma_ss(tbase + s_col<D>(0), ad, bd, idS, kk > 0);
          }
          tc::mma_commit(&bars[B_SFULL]);
          ok = tc::mbar_wait(&bars[B_BETA], 0, abort);
          tc::tc_after_sync();
        }
      }
      // the chunks whose slot has no earlier user: the first four, and the
      // second pass's chunk 1 when there is one parent chunk
      for (int w = 0; ok && w < 4 && w < nch; ++w) {
        if ((ok = tile_ready(s_tile(w)))) {
          tc::tc_after_sync();
          issue_S(w);
        }
      }
      if (ok && nch == 1 && (ok = tile_ready(s_tile(1)))) {
        tc::tc_after_sync();
        issue_S(1);
      }
      int nfree = 0;
      uint32_t eph = 0u;  // phase bit per logit slot's consumed barrier
      for (int v = 0; ok && v < nv; ++v) {
        const int sl = slot(v);
        if (!(ok = tc::mbar_wait(&bars[B_EFULL + sl], (eph >> sl) & 1u, abort))) break;
        eph ^= 1u << sl;
        tc::tc_after_sync();
        if (v >= nch) {
          const int u = v - nch, i = nch + 2 * u + 1, k = i & (NRING - 1);
          if (!(ok = tile_ready(i))) break;
          tc::tc_after_sync();
          // K steps of 16 parents: columns 0, 8 (half 0) and 32, 40 (half 1)
#pragma unroll
          for (int kk = 0; kk < TCH / 16; ++kk) {
            const uint64_t bd = tc::sdesc_sw128(ra0 + k * RB + kk * 16 * 128, TCH * 128, 1024);
            tc::mma_ts(tbase, tbase + D + 64 * sl + (kk >> 1) * 32 + (kk & 1) * 8, bd, idO, u > 0 || kk > 0);
          }
          tc::mma_commit(&bars[B_REMPTY + k]);
        }
        const int w = next_user(v);
        if (w >= 0) {
          if (v >= nch) {  // the e @ V MMA still reads this slot
            tc::mma_commit(&bars[B_SFREE]);
            if (!(ok = tc::mbar_wait(&bars[B_SFREE], nfree & 1, abort))) break;
            ++nfree;
          }
          if (!(ok = tile_ready(s_tile(w)))) break;
          tc::tc_after_sync();
          issue_S(w);
        }
      }
      tc::mma_commit(&bars[B_OFULL]);  // arrives once every MMA above has completed
      if (!ok) drain_wait(&bars[B_OFULL], 0);
    }
  } else {
    // ---- row threads: query r, half hf (parents 32hf..32hf+31 of each chunk) ----
    const int r = tid & (TR - 1), hf = tid >> 7, t = t0 + r;
    const bool live = t < Tq;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const float inv_sqrtD = 1.f / sqrtD;
    const float2 invl2 = make_float2(next_down(inv_sqrtD), next_down(inv_sqrtD));  // <= 1/sqrt(D)
    const float2 invh2 = make_float2(next_up(inv_sqrtD), next_up(inv_sqrtD));      // >= 1/sqrt(D)
    const uint32_t ninf2 = DT == DT_BF16 ? 0xFF80FF80u : 0xFC00FC00u;
    const long row = (long)g * Tq + t;
    T* srow_g = DN ? nullptr : scratch + (((long)g * ntiles + (t >> 6)) * 64 + (t & 63)) * LDL;
    // the row's mask words (pipeline.py:82-106); none for rows past T
    const int PW = (M0 + 31) >> 5;
    const unsigned int* prow = (MK && live) ? present + row * PW : nullptr;
    auto pword = [&](int wi) -> uint32_t {
      if constexpr (!MK) return 0xFFFFFFFFu;
      return prow ? (wi < PW ? prow[wi] : 0u) : 0xFFFFFFFFu;
    };
    const bool sector_stores = (reinterpret_cast<uintptr_t>(scratch) & 31u) == 0u;
    bool ok = true;
    float beta = 0.f;
    if constexpr (HV) {
      // pass 0: each query's temperature from its plain-pass probabilities of
      // the selected parents: p = DT(e / max(z, eps)) with the plain pass's m
      // and z, renormalised over the selection, entropy H = -sum p log p,
      // beta = DT(beta0 * schedule(H)) (pipeline.py:222-258, hopfield.py:55-102)
      ok = __all_sync(0xffffffffu, tc::mbar_wait(&bars[B_SFULL], 0u, abort));
      uint32_t ra[32];
      if (ok) {
        tc::tc_after_sync();
        tc::tmem_ld32(tbase + lane_off + s_col<D>(0) + 32 * hf, ra);
        tc::tmem_wait_ld();
      }
      // every row thread takes the same branch (one vote), so the barriers match
      if (rows_all(ok)) {
        const int nsel = min(pass_cnt[0], TCH);
        const int* sl = sel0 + (long)g * sel_stride;
        const float m0 = live ? m_out[row] : 0.f;
        const float zc0 = clamp_min_nan(live ? z_out[row] : 1.f, eps_dt<DT>());
        // DT(x / d) for x >= 0: x / d lies between RD(x dl) and RU(x dh), dl, dh
        // the fp32 neighbours of RN(1 / d); when both round to the same dtype
        // value so does the correctly rounded quotient, else divide exactly
        auto div_pos = [](float x, float d, float dl, float dh) -> float {
          const float lo = rnd<DT>(__fmul_rd(x, dl));
          return lo == rnd<DT>(__fmul_ru(x, dh)) ? lo : rnd<DT>(__fdiv_rn(x, d));
        };
        const float zi0 = 1.f / zc0, zl0 = next_down(zi0), zh0 = next_up(zi0);
        float pis[32];
        double gsp = 0.0;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int j = 32 * hf + i;
          float pi = 0.f;
          if (j < nsel) {
            const int pj = sl[j];
            const bool keep = pcnt[(long)gs * M0 + pj] > 0 && (!MK || !prow || ((prow[pj >> 5] >> (pj & 31)) & 1u));
            const float s = keep ? scale_logit<DT>(rnd<DT>(__uint_as_float(ra[i])), sqrtD, inv_sqrtD) : -INFINITY;
            const float e = fmaxf(exp_dt_fast<DT>(rnd<DT>(__fsub_rn(s, m0))), 0.f);  // NaN -> 0 (pipeline.py:143-145)
            pi = div_pos(e, zc0, zl0, zh0);
            gsp += (double)pi;
          }
          pis[i] = pi;
        }
        // the halves' sums meet in srow (free until pass 3), half 0's part first
        double* xd = reinterpret_cast<double*>(srow);
        xd[hf * TR + r] = gsp;
        rows_sync();
        const float gsc = clamp_min_nan(rnd64<DT>(xd[r] + xd[TR + r]), eps_dt<DT>());
        const float gi = 1.f / gsc, gl = next_down(gi), gh = next_up(gi);
        double ent = 0.0;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if (32 * hf + i < nsel) {
            const float top = div_pos(pis[i], gsc, gl, gh);  // pipeline.py:238
            const float lp = top > 0.f ? log_rn<DT>(top) : 0.f;
            ent += (double)rnd<DT>(__fmul_rn(top, lp));  // hopfield.py:100
          }
        }
        rows_sync();
        xd[hf * TR + r] = ent;
        rows_sync();
        const float hq = -rnd64<DT>(xd[r] + xd[TR + r]);
        const float sched = hvaq == 1 ? rnd<DT>(__fadd_rn(1.f, rnd<DT>(__fdiv_rn(1.f, rnd<DT>(__fadd_rn(1.f, hq))))))
                                      : rnd<DT>(__fadd_rn(1.f, rnd<DT>(__fmul_rn(alpha, hq))));
        beta = rnd<DT>(__fmul_rn(beta0, sched));  // hopfield.py:102
        if (live && hf == 0) beta_out[row] = beta;
      }
      tc::tc_before_sync();
      tc::mbar_arrive(&bars[B_BETA]);
    }
    const float2 sqd2 = make_float2(sqrtD, sqrtD);
    const uint32_t beta2 = dup2<DT>(beta);
    // pass 1: the row max of the logits (pipeline.py:107,137).  Narrowing and
    // scaling are monotone (so is the HVAQ rescaling, beta > 0), so it is the
    // logit of the largest raw accumulator over the non-empty parents
    // (NaN-propagating, as torch.max).
    float mxa[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    uint32_t sph = HV ? 1u : 0u;  // phase bit per logit slot's full barrier (HVAQ: slot 0 served pass 0)
    for (int v = 0; v < nch; ++v) {
      const int sl = v & 3;
      ok = __all_sync(0xffffffffu, tc::mbar_wait(&bars[B_SFULL + sl], (sph >> sl) & 1u, abort));
      sph ^= 1u << sl;
      if (!ok) break;
      tc::tc_after_sync();
      uint32_t ra[32];
      tc::tmem_ld32(tbase + lane_off + s_col<D>(sl) + 32 * hf, ra);
      tc::tmem_wait_ld();
      tc::tc_before_sync();
      tc::mbar_arrive(&bars[B_EFULL + sl]);
      const uint32_t* pm = pm2 + v * 32 + 16 * hf;
      const uint4* pm4 = reinterpret_cast<const uint4*>(pm);
      const uint32_t pb = pword(2 * v + hf);  // parent 64 v + 32 hf + i is bit i
      uint32_t all = pb;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 u = pm4[q];
        all &= u.x & u.y & u.z & u.w;
      }
      if (all == 0xFFFFFFFFu) {
#pragma unroll
        for (int i = 0; i < 32; ++i) mxa[i & 3] = fmax_nan(mxa[i & 3], __uint_as_float(ra[i]));
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const bool keep = ((pm[i >> 1] >> ((i & 1) * 16)) & 1u) && ((pb >> i) & 1u);
          mxa[i & 3] = fmax_nan(mxa[i & 3], keep ? __uint_as_float(ra[i]) : -INFINITY);
        }
      }
    }
    xch[hf * TR + r] = fmax_nan(fmax_nan(mxa[0], mxa[1]), fmax_nan(mxa[2], mxa[3]));
    rows_sync();
    const float amax = fmax_nan(xch[r], xch[TR + r]);
    float rm = DN ? rnd<DT>(__fmul_rn(rnd<DT>(amax), dscale)) : rnd<DT>(__fdiv_rn(rnd<DT>(amax), sqrtD));
    if constexpr (HV) rm = rnd<DT>(__fmul_rn(beta, rnd<DT>(__fmul_rn(rm, sqrtD))));  // pipeline.py:256, hopfield.py:144
    const float safe = rm == -INFINITY ? 0.f : rm;  // pipeline.py:137-141
    const uint32_t m2 = dup2<DT>(safe);
    // pass 2: exponentials, sums, e @ V
    float2 la2 = make_float2(0.f, 0.f);
    float za = 0.f;
    for (int v = nch; ok && v < nv; ++v) {
      const int c = v - nch, s = v & 1;
      ok = __all_sync(0xffffffffu, tc::mbar_wait(&bars[B_SFULL + s], (sph >> s) & 1u, abort));
      sph ^= 1u << s;
      if (!ok) break;
      tc::tc_after_sync();
      const uint32_t col = tbase + lane_off + D + 64 * s + 32 * hf;
      const uint32_t pb = pword(2 * c + hf);
      float zh[2];
      // 16 parents at a time; the second block's TMEM load is in flight while
      // the first is computed (its exponentials go to columns 0-7, the load
      // reads 16-31)
      uint32_t rh[2][16];
      tc::tmem_ld16(col, rh[0]);
      tc::tmem_wait_ld();
      tc::tmem_ld16(col + 16, rh[1]);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        if (hh == 1) tc::tmem_wait_ld();
        const uint32_t (&ra)[16] = rh[hh];
        // logits: DT(DT(acc) / sqrt(D)) (pipeline.py:81).  |x| / sqrt(D) lies
        // between RD(|x| invl) and RU(|x| invh); when both round to the same
        // dtype value, so does the correctly rounded quotient, and rounding to
        // nearest is symmetric, so the sign is copied back.  A block where
        // some pair's ends disagree is redone with correctly rounded quotients.
        uint32_t s2[8];
        if constexpr (DN) {
          // DT(DT(acc) * scale), the reference's own product (backend.py:197)
          const float2 sc2 = make_float2(dscale, dscale);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t x2 = pack2<DT>(__uint_as_float(ra[2 * j]), __uint_as_float(ra[2 * j + 1]));
            const float2 y = mul_f32x2_rn(make_float2(half_lo<DT>(x2), half_hi<DT>(x2)), sc2);
            s2[j] = pack2<DT>(y.x, y.y);
          }
        } else if constexpr (D == 64) {
          // sqrt(64) = 8: the quotient is exact in fp32, so DT(x / 8) is one
          // packed multiply by 1/8 (a single rounding, as the reference's)
#pragma unroll
          for (int j = 0; j < 8; ++j)
            s2[j] = hmul2_dt<DT>(pack2<DT>(__uint_as_float(ra[2 * j]), __uint_as_float(ra[2 * j + 1])), dup2<DT>(0.125f));
        } else {
        uint32_t near = 0u;  // bits where some pair's ends disagree (one LOP3 per pair)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t x2 = pack2<DT>(__uint_as_float(ra[2 * j]), __uint_as_float(ra[2 * j + 1]));
          const uint32_t a2 = x2 & 0x7FFF7FFFu;
          const float2 av = make_float2(half_lo<DT>(a2), half_hi<DT>(a2));
          const float2 ylo = mul_f32x2_rd(av, invl2), yhi = mul_f32x2_ru(av, invh2);
          const uint32_t qlo = pack2<DT>(ylo.x, ylo.y);
          near |= qlo ^ pack2<DT>(yhi.x, yhi.y);
          s2[j] = qlo | (x2 & 0x80008000u);
        }
        if (near != 0u) {
#pragma unroll
          for (int j = 0; j < 8; ++j) s2[j] = logit2<DT>(ra[2 * j], ra[2 * j + 1], sqrtD, inv_sqrtD, 0xFFFFFFFFu);
        }
        }
        if constexpr (HV) {
          // DT(beta * DT(s * sqrt(D))): the fp32 product narrowed, then the exact
          // DT product rounded once
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if constexpr (D == 64) {  // s * 8 is exact: one packed multiply
              s2[j] = hmul2_dt<DT>(hmul2_dt<DT>(s2[j], dup2<DT>(8.f)), beta2);
            } else {
              const float2 sc = mul_f32x2_rn(make_float2(half_lo<DT>(s2[j]), half_hi<DT>(s2[j])), sqd2);
              s2[j] = hmul2_dt<DT>(pack2<DT>(sc.x, sc.y), beta2);
            }
          }
        }
        const int pw = c * 32 + hf * 16 + hh * 8;  // first parent pair of the block
        const uint4* pm4 = reinterpret_cast<const uint4*>(pm2 + pw);
        const uint4* nn4 = reinterpret_cast<const uint4*>(n2 + pw);
        uint32_t e2[8];
        float zs[8];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const uint4 pmq = pm4[q], nnq = nn4[q];
          const uint32_t pmv[4] = {pmq.x, pmq.y, pmq.z, pmq.w}, nnv[4] = {nnq.x, nnq.y, nnq.z, nnq.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int j = 4 * q + k;
            uint32_t keepm = pmv[k];
            if constexpr (MK) {  // the pair's two mask bits, widened to its halves (pipeline.py:106)
              const uint32_t two = (pb >> (hh * 16 + 2 * j)) & 3u;
              keepm &= ((two & 1u) ? 0xFFFFu : 0u) | ((two & 2u) ? 0xFFFF0000u : 0u);
            }
            const uint32_t sm2 = (s2[j] & keepm) | (ninf2 & ~keepm);  // -inf for empty parents (pipeline.py:107)
            const uint32_t ee = exp2_dt<DT>(hsub2_dt<DT>(sm2, m2), exptab);
            e2[j] = ee;
            if constexpr (!DN) {  // every dense key counts once: l is z
              const uint32_t w2 = hmul2_dt<DT>(ee, nnv[k]);  // DT(e * n), pipeline.py:146
              la2 = add_f32x2(la2, make_float2(half_lo<DT>(w2), half_hi<DT>(w2)));
            }
            zs[j] = half_lo<DT>(ee) + half_hi<DT>(ee);
          }
        }
#pragma unroll
        for (int w = 4; w >= 1; w >>= 1)
#pragma unroll
          for (int j = 0; j < w; ++j) zs[j] += zs[j + w];
        zh[hh] = zs[0];
        tc::tmem_st8(col + 8 * hh, e2);
        // a block of 16 starting below M0 is stored whole: when M0 % 16 == 8 the
        // last block spills 8 columns past M0, into the row pitch's padding
        // (exp_slice_pitch(M0) >= round_up(M0, 16), asserted on the host)
        if (!DN && live && 2 * pw < M0) {
          // one whole 32-byte sector per store when the slices are 32-byte
          // aligned (the pitch keeps every row so), else two 16-byte halves
          T* dst = srow_g + 2 * pw;
          if (sector_stores) {
            asm volatile("st.global.L1::no_allocate.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst),
                         "r"(e2[0]), "r"(e2[1]), "r"(e2[2]), "r"(e2[3]), "r"(e2[4]), "r"(e2[5]), "r"(e2[6]), "r"(e2[7])
                         : "memory");
          } else {
            uint4* d4 = reinterpret_cast<uint4*>(dst);
            d4[0] = make_uint4(e2[0], e2[1], e2[2], e2[3]);
            d4[1] = make_uint4(e2[4], e2[5], e2[6], e2[7]);
          }
        }
      }
      za += zh[0] + zh[1];
      tc::tmem_wait_st();
      tc::tc_before_sync();
      tc::mbar_arrive(&bars[B_EFULL + s]);
    }
    // the halves' sums: z and l are the half-0 part plus the half-1 part in
    // both threads of the row
    xch[2 * TR + hf * TR + r] = za;
    xch[4 * TR + hf * TR + r] = la2.x + la2.y;
    rows_sync();
    const float zsum = xch[2 * TR + r] + xch[3 * TR + r];
    const float lsum = xch[4 * TR + r] + xch[5 * TR + r];
    // z feeds the probabilities.  Each half sums a chunk's 32 exponentials as
    // a pairwise tree (depth 5), the halves' chunk sums add in sequence and
    // the two halves once more, so the fp32 sum is within (6 + nch) * 2^-24
    // relative of the exact one; when the window straddles a dtype rounding
    // point the row is summed again exactly (by both threads, alike).
    float z = rnd<DT>(zsum);
    if (!DN && ok && live) {
      const float eps = zsum * (float)(nch + 8) * 5.9604645e-8f;
      if (rnd<DT>(zsum - eps) != rnd<DT>(zsum + eps)) {
        double ex = 0.0;
        const uint4* src = reinterpret_cast<const uint4*>(srow_g);
        for (int k = 0; k < M0 / 8; ++k) {
          const uint4 u = src[k];
          ex += (double)half_lo<DT>(u.x) + (double)half_hi<DT>(u.x) + (double)half_lo<DT>(u.y) +
                (double)half_hi<DT>(u.y) + (double)half_lo<DT>(u.z) + (double)half_hi<DT>(u.z) +
                (double)half_lo<DT>(u.w) + (double)half_hi<DT>(u.w);
        }
        z = rnd64<DT>(ex);
      }
    }
    if (ok) ok = __all_sync(0xffffffffu, tc::mbar_wait(&bars[B_OFULL], 0, abort));
    // every row thread takes the same branch below (one vote), so the barrier matches
    if (rows_all(ok)) {
      tc::tc_after_sync();
      // the tile of a goes through the idle Q, P and V buffers (pass 3 refills
      // them only after its own vote), so that each warp stores whole rows
      // instead of 32 rows' 16-byte pieces; half hf stages columns
      // [hf D/2, (hf+1) D/2) of its row
      constexpr int SLDB = D * 2 + 16;  // padded row bytes: a warp's 16-byte writes hit distinct banks
      static_assert(TR * SLDB <= TR * D * 2 + 4 * TCH * D * 2, "output staging");
      unsigned char* stga = sm + L.q;
      const float iz = 1.f / zsum;  // the dense output is O / z
#pragma unroll
      for (int d0 = 0; d0 < D / 2; d0 += 32) {
        uint32_t oa[32];
        const int dc = hf * (D / 2) + d0;
        tc::tmem_ld32(tbase + lane_off + dc, oa);
        tc::tmem_wait_ld();
        if constexpr (DN) {
#pragma unroll
          for (int k = 0; k < 32; ++k) oa[k] = __float_as_uint(__uint_as_float(oa[k]) * iz);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t* src = oa + 8 * k;
          *reinterpret_cast<uint4*>(stga + r * SLDB + dc * 2 + 16 * k) =
              make_uint4(pack2<DT>(__uint_as_float(src[0]), __uint_as_float(src[1])),
                         pack2<DT>(__uint_as_float(src[2]), __uint_as_float(src[3])),
                         pack2<DT>(__uint_as_float(src[4]), __uint_as_float(src[5])),
                         pack2<DT>(__uint_as_float(src[6]), __uint_as_float(src[7])));
        }
      }
      rows_sync();
      constexpr int U4 = D / 8, RPI = 32 / U4;  // 16-byte pieces per row, rows per warp instruction
      const int c16 = lane % U4;
#pragma unroll 4
      for (int i = 0; i < TR / 8; i += RPI) {
        const int rr = (warp & 7) * (TR / 8) + i + lane / U4, tt = t0 + rr;
        if (tt < Tq) {
          T* dst = DN ? dout + (long)b * os.b + (long)h * os.h + (long)tt * os.s : a_out + ((long)g * Tq + tt) * D;
          reinterpret_cast<uint4*>(dst)[c16] = *reinterpret_cast<const uint4*>(stga + rr * SLDB + 16 * c16);
        }
      }
      if (!DN && live && hf == 0) {
        m_out[row] = safe;
        l_out[row] = rnd<DT>(lsum);
        z_out[row] = z;
      }
    }
    if constexpr (!DN) {
    const float zc = clamp_min_nan(z, eps_dt<DT>());
    if (hf == 0) {  // z and the fp32 neighbours of RN(1/z), which bracket 1/z
      const float zi = 1.f / zc;
      srow[r * 4] = zc;
      srow[r * 4 + 1] = next_down(zi);
      srow[r * 4 + 2] = next_up(zi);
    }
    // pass 3: importance partials (routing.py:61-63).  The CTA's exponential
    // rows stream through the idle Q, P and V tile buffers in 64-column
    // blocks (cp.async, NSTG block buffers); each iteration takes two blocks
    // between two row-thread barriers.  Lane = 2 columns, each thread sums 16
    // rows in order (rows 32(w%4) + 16hf + i), and the four 16-row sums of
    // each 64-query tile are added in row order.  Rows beyond T stage as zeros
    // and add 0.  Every row thread runs the same iterations (one vote first),
    // so the barriers match.
    constexpr int PB = 64, BLK = TR * PB * 2;
    constexpr int NSTG = (TR * D * 2 + 4 * TCH * D * 2) / BLK;  // Q, P, V buffers: 6 blocks (D 128), 3 (D 64)
    static_assert(NSTG >= 3, "staging depth");
    unsigned char* stg = sm + L.q;
    const int nblk = (M0 + PB - 1) / PB;
    const int rbase = 32 * (warp & 3) + 16 * hf;
    auto stage = [&](int blk) {  // one cp.async group, empty beyond the last block
      if (blk < nblk) {
        unsigned char* buf = stg + (blk % NSTG) * BLK;
        const int pc = blk * PB, ch = tid & 7;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int rr = (tid >> 3) + 32 * k, tw = t0 + rr;
          const bool in = tw < Tq && pc + ch * 8 < M0;
          const int ts = in ? tw : t0;
          cp_async16(buf + rr * (PB * 2) + ch * 16,
                     scratch + (((long)g * ntiles + (ts >> 6)) * 64 + (ts & 63)) * LDL + (in ? pc + ch * 8 : 0), in);
        }
      }
      cp_async_commit();
    };
    // the column sums of one block over this thread's 16 rows
    auto block_sums = [&](int blk) -> float2 {
      const unsigned char* buf = stg + (blk % NSTG) * BLK;
      float2 c2 = make_float2(0.f, 0.f);
#pragma unroll 1
      for (int g8 = 0; g8 < 2; ++g8) {
        uint32_t w[8], q[8], bad = 0u;  // bits where some pair's ends disagree
        float4 zr[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int rw = rbase + g8 * 8 + i;
          w[i] = *reinterpret_cast<const uint32_t*>(buf + rw * (PB * 2) + lane * 4);
          zr[i] = *reinterpret_cast<const float4*>(srow + rw * 4);
        }
        // DT(e / z), e >= 0: e / z lies between RD(e zl) and RU(e zh); when
        // both round to the same dtype value so does the correctly rounded
        // quotient, else the pair is divided exactly
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float2 ev = make_float2(half_lo<DT>(w[i]), half_hi<DT>(w[i]));
          const float2 ylo = mul_f32x2_rd(ev, make_float2(zr[i].y, zr[i].y));
          const float2 yhi = mul_f32x2_ru(ev, make_float2(zr[i].z, zr[i].z));
          q[i] = pack2<DT>(ylo.x, ylo.y);
          bad |= q[i] ^ pack2<DT>(yhi.x, yhi.y);
        }
        if (bad) {  // rare: the eight pairs divided exactly (the agreeing ones give the same values)
#pragma unroll
          for (int i = 0; i < 8; ++i)
            q[i] = pack2<DT>(__fdiv_rn(half_lo<DT>(w[i]), zr[i].x), __fdiv_rn(half_hi<DT>(w[i]), zr[i].x));
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) c2 = add_f32x2(c2, make_float2(half_lo<DT>(q[i]), half_hi<DT>(q[i])));
      }
      return c2;
    };
    const bool ok3 = rows_all(ok);
    if (ok3)
      for (int i = 0; i < NSTG - 2; ++i) stage(i);
    for (int blk = 0; ok3 && blk < nblk; blk += 2) {
      // the buffers of blocks blk - 2 and blk - 1 were read before the last barrier
      stage(blk + NSTG - 2);
      stage(blk + NSTG - 1);
      cp_async_wait<NSTG - 2>();
      rows_sync();  // every thread's copies of blocks blk and blk + 1 have landed
      const float2 s0 = block_sums(blk);
      const float2 s1 = blk + 1 < nblk ? block_sums(blk + 1) : make_float2(0.f, 0.f);
      scomb[warp * 64 + 2 * lane] = s0.x;
      scomb[warp * 64 + 2 * lane + 1] = s0.y;
      scomb[512 + warp * 64 + 2 * lane] = s1.x;
      scomb[512 + warp * 64 + 2 * lane + 1] = s1.y;
      rows_sync();  // the partials are visible, and both blocks' buffers are read
      {
        // tile tl: rows 64tl + [0,16) warp 2tl, [16,32) warp 2tl+4, [32,48) warp 2tl+1, [48,64) warp 2tl+5;
        // thread tid handles block blk + (tid >> 7)
        const int bb = tid >> 7, t2 = tid & 127, tl = t2 >> 6, cl = t2 & 63, pcol = (blk + bb) * PB + cl;
        const int tile = 2 * qt + tl;
        const float* sc = scomb + 512 * bb;
        if (tile < ntiles && pcol < M0)
          colpart[((long)g * ntiles + tile) * M0 + pcol] =
              (sc[(2 * tl) * 64 + cl] + sc[(2 * tl + 4) * 64 + cl]) + (sc[(2 * tl + 1) * 64 + cl] + sc[(2 * tl + 5) * 64 + cl]);
      }
    }
    cp_async_wait<0>();
    }  // !DN
  }

  // ---- teardown ----
  tc::tc_before_sync();
  __syncthreads();
  if (warp == W_MMA) {
    tc::tc_after_sync();
    tc::tmem_free(tbase, TC_TMEM_COLS);
  }
  if (tid == 0 && *abort) atomicOr(&g_fault, 1);
}

// ---- host side ----------------------------------------------------------------
// AVQ_DISABLE_TCGEN05=1 selects the mma.sync parent-attention kernel (read at
// every launch, so one process can run both).
bool tc_disabled() {
  const char* e = std::getenv("AVQ_DISABLE_TCGEN05");
  return e && *e && *e != '0';
}

}  // namespace

bool parent_attn_tc_ok(int dt, int D, int M0) {
  return !tc_disabled() && dt != DT_F32 && (D == 64 || D == 128) && M0 % 8 == 0 && M0 <= TC_MAX_M0;
}

bool parent_attn_tc_hvaq_ok(int dt, int D, int M0, int P) { return parent_attn_tc_ok(dt, D, M0) && P <= TCH; }

size_t parent_attn_tc_table_bytes() { return (size_t)EXP_WORDS * 4; }

void launch_exp_table(void* tab, cudaStream_t st) { exp_table_kernel<<<1, 256, 0, st>>>(static_cast<uint16_t*>(tab)); }

template <int DT>
int launch_parent_attn_tc(const PAArgs& a, void* exptab, cudaStream_t st) {
  using T = typename Storage<DT>::T;
  const int G = a.B * a.H, D = a.D, M0 = a.M0, sG = a.sG > 0 ? a.sG : G;
  const bool hv = a.mode == 1;
  if (hv && (!a.sel0 || !a.pass_cnt || !a.beta)) return AVQ_ERR_UNSUPPORTED;
  // Q [B,H,T,D] strided, P [H, M0, D], V [sG, M0, D]; 128-byte swizzled boxes
  CUtensorMap tq, tp, tv;
  int4 qpos;
  if (!tc::map_rows4(&tq, DT, a.q, a.qs, a.B, a.H, a.T, D, TR, &qpos) ||
      !tc::map_rows3(&tp, DT, a.parents, a.H, M0, D, TCH) || !tc::map_rows3(&tv, DT, a.pagg, sG, M0, D, TCH))
    return AVQ_ERR_UNSUPPORTED;
  if (exp_slice_pitch(M0) < ((M0 + 15) & ~15)) return AVQ_ERR_UNSUPPORTED;  // whole 16-column stores
  const TcLayout L = tc_layout(D, M0, hv);
  // at least 80 KB so that no more than two CTAs (2 x 256 TMEM columns) share an SM
  const size_t smem = std::max<size_t>((size_t)L.total + 1024, 80 * 1024);
  auto go = [&](auto kfn) {
    AVQ_TIMED(hv ? "parent_attn_hvaq_tc" : "parent_attn_tc", st);
    cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kfn<<<dim3((a.T + TR - 1) / TR, G), TTHREADS, smem, st>>>(
        tq, tp, tv, qpos, a.H, a.T, M0, a.sqrtD, a.pcnt, static_cast<const uint16_t*>(exptab),
        static_cast<T*>(a.sglobal), a.m, a.l, a.z, static_cast<T*>(a.a), a.colpart, sG,
        static_cast<const T*>(a.parents), a.sel0, a.sel_stride, a.pass_cnt, a.hvaq, a.beta0, a.alpha, a.beta,
        a.present, make_int4(0, 0, 0, 0), 0.f, nullptr, Strides3{0, 0, 0});
  };
  const bool mk = a.present != nullptr;
  if (hv) {
    if (D == 64) mk ? go(parent_attn_tc_kernel<DT, 64, true, true>) : go(parent_attn_tc_kernel<DT, 64, true, false>);
    else mk ? go(parent_attn_tc_kernel<DT, 128, true, true>) : go(parent_attn_tc_kernel<DT, 128, true, false>);
  } else {
    if (D == 64) mk ? go(parent_attn_tc_kernel<DT, 64, false, true>) : go(parent_attn_tc_kernel<DT, 64, false, false>);
    else mk ? go(parent_attn_tc_kernel<DT, 128, false, true>) : go(parent_attn_tc_kernel<DT, 128, false, false>);
  }
  return cudaPeekAtLastError() == cudaSuccess ? AVQ_OK : AVQ_ERR_CUDA;
}

template int launch_parent_attn_tc<DT_BF16>(const PAArgs&, void*, cudaStream_t);
template int launch_parent_attn_tc<DT_F16>(const PAArgs&, void*, cudaStream_t);

namespace {
// The bf16 exponential table of the dense path, rewritten by every call (the
// same 4 KB each time), so the dense entry needs no caller workspace.
__device__ uint16_t g_dense_exptab[2 * EXP_WORDS];
}  // namespace

// Dense attention on the parent-attention kernel (DN mode): keys and values
// are the parent and parent-sum operands, one CTA per 128 queries of a (b,h).
template <int DT>
int launch_dense_tc(const void* q, Strides3 qs, const void* k, Strides3 ks, const void* v, Strides3 vs, int B, int H,
                    int T, int N, int D, float scale, void* out, Strides3 os, cudaStream_t st) {
  using T_ = typename Storage<DT>::T;
  if (tc_disabled() || (D != 64 && D != 128) || N < 1 || N > TC_MAX_M0 || N % 8 || T < 1) return AVQ_ERR_UNSUPPORTED;
  // whole-row 16-byte output stores
  if ((reinterpret_cast<uintptr_t>(out) & 15u) || os.b % 8 || os.h % 8 || os.s % 8) return AVQ_ERR_UNSUPPORTED;
  CUtensorMap tq, tk, tv;
  int4 qpos, kpos, vpos;
  if (!tc::map_rows4(&tq, DT, q, qs, B, H, T, D, TR, &qpos) || !tc::map_rows4(&tk, DT, k, ks, B, H, N, D, TCH, &kpos) ||
      !tc::map_rows4(&tv, DT, v, vs, B, H, N, D, TCH, &vpos))
    return AVQ_ERR_UNSUPPORTED;
  if (kpos.x != vpos.x || kpos.y != vpos.y || kpos.z != vpos.z) return AVQ_ERR_UNSUPPORTED;
  // the kernel copies the table into shared memory whatever the dtype (fp16
  // does not read it), so the address is always a filled device array
  void* tab = nullptr;
  if (cudaGetSymbolAddress(&tab, g_dense_exptab) != cudaSuccess) return AVQ_ERR_CUDA;
  launch_exp_table(tab, st);
  const TcLayout L = tc_layout(D, N, false);
  const size_t smem = std::max<size_t>((size_t)L.total + 1024, 80 * 1024);
  auto go = [&](auto kfn) {
    cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kfn<<<dim3((T + TR - 1) / TR, B * H), TTHREADS, smem, st>>>(
        tq, tk, tv, qpos, H, T, N, (float)std::sqrt((double)D), nullptr, static_cast<const uint16_t*>(tab), nullptr,
        nullptr, nullptr, nullptr, nullptr, nullptr, 1, nullptr, nullptr, 0, nullptr, 0, 0.f, 0.f, nullptr, nullptr,
        kpos, scale, static_cast<T_*>(out), os);
  };
  if (D == 64) go(parent_attn_tc_kernel<DT, 64, false, false, true>);
  else go(parent_attn_tc_kernel<DT, 128, false, false, true>);
  return cudaPeekAtLastError() == cudaSuccess ? AVQ_OK : AVQ_ERR_CUDA;
}

template int launch_dense_tc<DT_BF16>(const void*, Strides3, const void*, Strides3, const void*, Strides3, int, int,
                                      int, int, int, float, void*, Strides3, cudaStream_t);
template int launch_dense_tc<DT_F16>(const void*, Strides3, const void*, Strides3, const void*, Strides3, int, int,
                                     int, int, int, float, void*, Strides3, cudaStream_t);

int read_device_fault(int* code, cudaStream_t st) {
  int v = 0, va = 0, vc = 0;
  if (cudaMemcpyFromSymbolAsync(&v, g_fault, sizeof(int), 0, cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return AVQ_ERR_CUDA;
  const int zero = 0;
  if (cudaMemcpyToSymbolAsync(g_fault, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st) != cudaSuccess)
    return AVQ_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return AVQ_ERR_CUDA;
  if (read_fault_assign(&va, st) != AVQ_OK || read_fault_correct(&vc, st) != AVQ_OK) return AVQ_ERR_CUDA;
  *code = v | va | vc;
  return AVQ_OK;
}

}  // namespace avq
