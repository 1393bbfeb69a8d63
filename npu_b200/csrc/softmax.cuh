// Device helpers shared by the prefill kernels (prefill.cu, prefill_d256.cu):
// the exp2 split between the MUFU and FMA pipes, 3-input max, and the output
// store of one 32-column chunk of a query row.
#pragma once

#include "prefill.cuh"

namespace b2a {

// Of every 4 column pairs of S, this many have their exp2 evaluated on the
// FMA pipe (exp2_fma2) instead of the MUFU unit; the rest use ex2.approx.
// Spreading the exponentials over both pipes keeps MUFU off the critical path.
#ifndef B2A_EXP2_EMU
#define B2A_EXP2_EMU 1
#endif
constexpr int kExp2EmuPairs = B2A_EXP2_EMU;
static_assert(kExp2EmuPairs >= 0 && kExp2EmuPairs <= 4, "B2A_EXP2_EMU is a count out of 4 pairs");

// The split that measured fastest per head dim on B200 (causal prefill,
// T = 1k-8k): at D = 64, where the exponentials are the largest share of a
// block's work, one pair in four on the FMA pipe is ~5 % faster; at D = 128
// all on MUFU is 2-4 % faster; D = 256 measures the same either way.
template <int D>
__host__ __device__ constexpr int exp2_emu_pairs() {
  return D == 128 ? 0 : kExp2EmuPairs;
}

__device__ __forceinline__ float u2f(uint32_t x) { return __uint_as_float(x); }
__device__ __forceinline__ uint32_t f2u(float x) { return __float_as_uint(x); }

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

#ifndef B2A_EXP2_DEG
#define B2A_EXP2_DEG 2
#endif
static_assert(B2A_EXP2_DEG == 2 || B2A_EXP2_DEG == 3, "exp2 polynomial degree is 2 or 3");

// 2^x for a pair, on the FMA pipe: x = n + f with n = round(x) (adding the
// 1.5 * 2^23 rounding constant leaves n in the low mantissa bits of t) and
// f in [-1/2, 1/2]; 2^f comes from a polynomial fitted for relative error by
// npu_b200/csrc/exp2_poly_fit.py (cubic: max rel. error 7.5e-5; quadratic:
// 1.7e-3, below the 2^-9 rounding of the bf16 P tile); 2^n is added to the
// exponent field with one shift-add of n << 23. Inputs are clamped at -120 so
// the exponent arithmetic cannot wrap. The caller only uses this on key
// blocks without masked entries (no -inf inputs); it returns 2^-120, not 0,
// for anything below the clamp.
__device__ __forceinline__ uint32_t shl23_add(uint32_t t, uint32_t p) {
  uint32_t r;
  asm("mad.lo.u32 %0, %1, 8388608, %2;" : "=r"(r) : "r"(t), "r"(p));
  return r;
}

__device__ __forceinline__ float2 exp2_fma2(float2 xin) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  const float2 x = make_float2(fmaxf(xin.x, -120.f), fmaxf(xin.y, -120.f));
  const float2 t = __fadd2_rn(x, make_float2(kRound, kRound));
  const float2 n = __fadd2_rn(t, make_float2(-kRound, -kRound));
  const float2 f = __ffma2_rn(n, make_float2(-1.f, -1.f), x);
#if B2A_EXP2_DEG == 3
  constexpr float c0 = 9.999281168e-01f, c1 = 6.932609677e-01f, c2 = 2.426105440e-01f, c3 = 5.517132208e-02f;
  float2 p = __ffma2_rn(f, make_float2(c3, c3), make_float2(c2, c2));
  p = __ffma2_rn(p, f, make_float2(c1, c1));
  p = __ffma2_rn(p, f, make_float2(c0, c0));
#else
  constexpr float c0 = 1.000442982e+00f, c1 = 7.034428120e-01f, c2 = 2.384257019e-01f;
  float2 p = __ffma2_rn(f, make_float2(c2, c2), make_float2(c1, c1));
  p = __ffma2_rn(p, f, make_float2(c0, c0));
#endif
  return make_float2(__uint_as_float(shl23_add(__float_as_uint(t.x), __float_as_uint(p.x))),
                     __uint_as_float(shl23_add(__float_as_uint(t.y), __float_as_uint(p.y))));
}

// One row of P for a key block: x = S * scale * log2e - m, P = 2^x as bf16
// into the 128B-swizzled K-major tile (16-byte stores, chunk index XOR row),
// returns the fp32 row sum. With kEmu, kExp2EmuPairs of every 4 column pairs
// take exp2 on the FMA pipe; callers pass kEmu only for blocks with no masked
// key (all x finite), the others use ex2.approx throughout (exact 0 for -inf).
template <int BN, bool kEmu>
__device__ __forceinline__ float softmax_p_row(const uint32_t (&s)[BN / 32][32], float sl2, float m_use,
                                               uint32_t pbase, int chunk_bytes, int row) {
  const float2 sc2 = make_float2(sl2, sl2);
  const float2 nm2 = make_float2(-m_use, -m_use);
  float2 acc[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) acc[k] = make_float2(0.f, 0.f);
#pragma unroll
  for (int c8 = 0; c8 < BN / 8; ++c8) {
    uint32_t wv[4];
#pragma unroll
    for (int pp = 0; pp < 4; ++pp) {
      const int i = c8 * 8 + pp * 2;
      const float2 x = __ffma2_rn(make_float2(u2f(s[i >> 5][i & 31]), u2f(s[(i + 1) >> 5][(i + 1) & 31])), sc2, nm2);
      float2 e;
      if (kEmu && pp < kExp2EmuPairs)
        e = exp2_fma2(x);
      else
        e = make_float2(ex2(x.x), ex2(x.y));
      acc[pp] = __fadd2_rn(acc[pp], e);
      wv[pp] = pack_bf16x2(e.x, e.y);
    }
    st_shared_v4(pbase + (c8 >> 3) * chunk_bytes + row * 128 + (((c8 & 7) ^ (row & 7)) << 4), wv[0], wv[1], wv[2],
                 wv[3]);
  }
  const float2 r2 = __fadd2_rn(__fadd2_rn(acc[0], acc[1]), __fadd2_rn(acc[2], acc[3]));
  return r2.x + r2.y;
}

// Same as softmax_p_row, but P goes to tensor memory for an MMA that reads its
// A operand from TMEM: columns tP .. tP + BN/2 of this thread's lane, two bf16
// per 32-bit column (even key in the low half). The caller waits for the
// stores (tcgen05.wait::st) before publishing P. The TMEM stores are
// warp-collective: every lane of the warp must call this with the same kEmu.
// With kTrackMax the raw (unscaled) row max of S is accumulated into *smax
// alongside, so a caller can compute P with a running max from earlier blocks
// and only redo the row when this block's max turns out to be much larger.
// kLean trades ILP for registers: two partial sums and maxima instead of
// four, and P stored 8 columns (16 keys) at a time instead of 16.
template <int BN, bool kEmu, bool kTrackMax = false, bool kLean = false>
__device__ __forceinline__ float softmax_p_row_tmem(const uint32_t (&s)[BN / 32][32], float sl2, float m_use,
                                                    uint32_t tP, float* smax = nullptr) {
  constexpr int NACC = kLean ? 2 : 4;
  constexpr int NST = kLean ? 8 : 16;  // packed columns per TMEM store
  const float2 sc2 = make_float2(sl2, sl2);
  const float2 nm2 = make_float2(-m_use, -m_use);
  float2 acc[NACC];
#pragma unroll
  for (int k = 0; k < NACC; ++k) acc[k] = make_float2(0.f, 0.f);
  float mx[NACC];
#pragma unroll
  for (int k = 0; k < NACC; ++k) mx[k] = -INFINITY;
#pragma unroll
  for (int g = 0; g < BN / (2 * NST); ++g) {
    uint32_t wv[NST];
#pragma unroll
    for (int e = 0; e < NST; ++e) {
      const int pp = g * NST + e;  // column pair index within the row
      const int q = pp >> 4, i = 2 * (pp & 15);
      if (kTrackMax) mx[pp % NACC] = fmax3(mx[pp % NACC], u2f(s[q][i]), u2f(s[q][i + 1]));
      const float2 x = __ffma2_rn(make_float2(u2f(s[q][i]), u2f(s[q][i + 1])), sc2, nm2);
      float2 e2;
      if (kEmu && (pp & 3) < kExp2EmuPairs)
        e2 = exp2_fma2(x);
      else
        e2 = make_float2(ex2(x.x), ex2(x.y));
      acc[pp % NACC] = __fadd2_rn(acc[pp % NACC], e2);
      wv[e] = pack_bf16x2(e2.x, e2.y);
    }
    if constexpr (NST == 8)
      tmem_st8(tP + NST * g, wv);
    else
      tmem_st16(tP + NST * g, wv);
  }
  float2 r2 = acc[0];
#pragma unroll
  for (int k = 1; k < NACC; ++k) r2 = __fadd2_rn(r2, acc[k]);
  if (kTrackMax) {
    float m = mx[0];
#pragma unroll
    for (int k = 1; k < NACC; ++k) m = fmaxf(m, mx[k]);
    *smax = m;
  }
  return r2.x + r2.y;
}

// P for 32-key chunks [Q0, Q0 + NQ) of a row whose S values are in s, with
// partial row sums and (optionally) raw maxima accumulated into acc / mx.
// Lets a caller start on the first chunks while TMEM loads of the later ones
// are still in flight (the P columns written here, tP + 16 q, lie below the
// S columns of any later chunk). Same pipe split and TMEM store rules as
// softmax_p_row_tmem.
template <int NCH, int Q0, int NQ, int kEmuPairs, bool kTrackMax>
__device__ __forceinline__ void softmax_p_chunks_tmem(const uint32_t (&s)[NCH][32], float sl2, float m_use,
                                                      uint32_t tP, float2 (&acc)[4], float (&mx)[4]) {
  const float2 sc2 = make_float2(sl2, sl2);
  const float2 nm2 = make_float2(-m_use, -m_use);
#pragma unroll
  for (int q = Q0; q < Q0 + NQ; ++q) {
    uint32_t wv[16];
#pragma unroll
    for (int pp = 0; pp < 16; ++pp) {
      if (kTrackMax) mx[pp & 3] = fmax3(mx[pp & 3], u2f(s[q][2 * pp]), u2f(s[q][2 * pp + 1]));
      const float2 x = __ffma2_rn(make_float2(u2f(s[q][2 * pp]), u2f(s[q][2 * pp + 1])), sc2, nm2);
      float2 e;
      if ((pp & 3) < kEmuPairs)
        e = exp2_fma2(x);
      else
        e = make_float2(ex2(x.x), ex2(x.y));
      acc[pp & 3] = __fadd2_rn(acc[pp & 3], e);
      wv[pp] = pack_bf16x2(e.x, e.y);
    }
    tmem_st16(tP + 16 * q, wv);
  }
}

// The running max of a row is only moved (and everything summed so far
// rescaled) when a block's max exceeds it by more than 2^8 in the exp2
// domain; otherwise P values stay <= 256, which bf16 and the fp32 row sum
// hold exactly enough. This keeps the rescale off the common path.
constexpr float kRescaleThreshold = 8.0f;

// P for one 64-key half of a row's key block into TMEM columns tP .. tP + 32
// (two bf16 per column), with the row's running max m_run (exp2 domain).
// Keys past `lim` (relative to the half's first key) are masked. With a
// running max present, P is computed with it and the half's max taken
// alongside; only if that max exceeds m_run by more than the threshold is
// m_run moved and the half redone (MUFU only). Rows without a running max
// take the max first. Returns the factor (<= 1) by which everything summed
// for this row before this half (earlier blocks, the block's earlier half,
// their P and O) has to be scaled: 1 unless m_run moved. `hsum` receives the
// half's sum of P. kEmuPairs of every 4 column pairs use the FMA-pipe exp2 on
// unmasked halves. Warp-collective (TMEM stores, votes): all lanes call it.
template <int kEmuPairs>
__device__ __forceinline__ float softmax_half_tmem(uint32_t (&s)[2][32], int lim, float sl2, float& m_run,
                                                   uint32_t tP, float& hsum) {
  const bool full = __all_sync(0xffffffffu, lim >= 63);
  if (!full) {
#pragma unroll
    for (int i = 0; i < 64; ++i)
      if (i > lim) s[i >> 5][i & 31] = f2u(-INFINITY);
  }
  float a = 1.f;
  float2 acc[4];
  float mx[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    acc[k] = make_float2(0.f, 0.f);
    mx[k] = -INFINITY;
  }
  if (__all_sync(0xffffffffu, m_run != -INFINITY)) {
    // exp2 on both pipes only when no key is masked (no -inf inputs).
    if (full)
      softmax_p_chunks_tmem<2, 0, 2, kEmuPairs, true>(s, sl2, m_run, tP, acc, mx);
    else
      softmax_p_chunks_tmem<2, 0, 2, 0, true>(s, sl2, m_run, tP, acc, mx);
    const float m_blk = fmaxf(fmax3(mx[0], mx[1], mx[2]), mx[3]) * sl2;
    const bool jump = m_blk > m_run + kRescaleThreshold;
    if (__any_sync(0xffffffffu, jump)) {
      if (jump) {
        a = ex2(m_run - m_blk);
        m_run = m_blk;
      }
      tmem_wait_st();  // the first pass's stores land before they are overwritten
#pragma unroll
      for (int k = 0; k < 4; ++k) acc[k] = make_float2(0.f, 0.f);
      softmax_p_chunks_tmem<2, 0, 2, 0, false>(s, sl2, m_run, tP, acc, mx);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 64; i += 8) {
      mx[0] = fmax3(mx[0], u2f(s[i >> 5][(i & 31)]), u2f(s[i >> 5][(i & 31) + 1]));
      mx[1] = fmax3(mx[1], u2f(s[i >> 5][(i & 31) + 2]), u2f(s[i >> 5][(i & 31) + 3]));
      mx[2] = fmax3(mx[2], u2f(s[i >> 5][(i & 31) + 4]), u2f(s[i >> 5][(i & 31) + 5]));
      mx[3] = fmax3(mx[3], u2f(s[i >> 5][(i & 31) + 6]), u2f(s[i >> 5][(i & 31) + 7]));
    }
    const float m_new = fmaxf(m_run, fmaxf(fmax3(mx[0], mx[1], mx[2]), mx[3]) * sl2);
    if (m_run == -INFINITY) {
      if (m_new != -INFINITY) a = 0.f;  // everything before was computed from masked keys: zeros
      m_run = m_new;
    } else if (m_new > m_run + kRescaleThreshold) {
      a = ex2(m_run - m_new);
      m_run = m_new;
    }
    const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
    softmax_p_chunks_tmem<2, 0, 2, 0, false>(s, sl2, m_use, tP, acc, mx);
  }
  const float2 r2 = __fadd2_rn(__fadd2_rn(acc[0], acc[1]), __fadd2_rn(acc[2], acc[3]));
  hsum = r2.x + r2.y;
  return a;
}

// sigmoid(g) = 1 / (1 + e^-g) in fp32 (torch.sigmoid, qwen/forward.py:226).
__device__ __forceinline__ float sigmoidf_(float g) { return __fdividef(1.f, 1.f + __expf(-g)); }

// One 32-column chunk of an output row: O scaled by inv_l and, with a gate,
// by sigmoid(gate). Only called for rows that exist (the gate is read).
__device__ __forceinline__ void out_chunk_values(const PrefillParams& p, int b, int h, int grow, int c,
                                                 const uint32_t (&o)[32], float inv_l, float (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = u2f(o[i]) * inv_l;
  if (p.gate) {
    const long long gi = (long long)b * p.g_sb + (long long)h * p.g_sh + (long long)grow * p.g_st + 32 * c;
    if (p.gate_bf16) {
      const uint4* g4 = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.gate) + gi);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 w = g4[i];
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          v[8 * i + 2 * k] *= sigmoidf_(u2f(ws[k] << 16));
          v[8 * i + 2 * k + 1] *= sigmoidf_(u2f(ws[k] & 0xffff0000u));
        }
      }
    } else {
      const float4* g4 = reinterpret_cast<const float4*>(static_cast<const float*>(p.gate) + gi);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 w = g4[i];
        v[4 * i] *= sigmoidf_(w.x);
        v[4 * i + 1] *= sigmoidf_(w.y);
        v[4 * i + 2] *= sigmoidf_(w.z);
        v[4 * i + 3] *= sigmoidf_(w.w);
      }
    }
  }
}

// Scale one 32-column chunk of an output row (out_chunk_values) and store it
// (fp32 or bf16) with 32-byte stores where O is aligned for them (p.o_v8: a
// warp's row-per-thread stores then write whole 32-byte sectors, with half
// the store instructions), else 16-byte stores.
__device__ __forceinline__ void store_out_chunk(const PrefillParams& p, int b, int h, int grow, int c,
                                                const uint32_t (&o)[32], float inv_l) {
  float v[32];
  out_chunk_values(p, b, h, grow, c, o, inv_l, v);
  const long long base = (long long)b * p.o_sb + (long long)h * p.o_sh + (long long)grow * p.o_st + 32 * c;
  if (p.o_v8) {
    if (p.out_fp32) {
      float* dst = reinterpret_cast<float*>(p.o) + base;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        st_global_v8(dst + 8 * i, f2u(v[8 * i]), f2u(v[8 * i + 1]), f2u(v[8 * i + 2]), f2u(v[8 * i + 3]),
                     f2u(v[8 * i + 4]), f2u(v[8 * i + 5]), f2u(v[8 * i + 6]), f2u(v[8 * i + 7]));
    } else {
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.o) + base;
#pragma unroll
      for (int i = 0; i < 2; ++i)
        st_global_v8(dst + 16 * i, pack_bf16x2(v[16 * i], v[16 * i + 1]), pack_bf16x2(v[16 * i + 2], v[16 * i + 3]),
                     pack_bf16x2(v[16 * i + 4], v[16 * i + 5]), pack_bf16x2(v[16 * i + 6], v[16 * i + 7]),
                     pack_bf16x2(v[16 * i + 8], v[16 * i + 9]), pack_bf16x2(v[16 * i + 10], v[16 * i + 11]),
                     pack_bf16x2(v[16 * i + 12], v[16 * i + 13]), pack_bf16x2(v[16 * i + 14], v[16 * i + 15]));
    }
  } else if (p.out_fp32) {
    float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.o) + base);
#pragma unroll
    for (int i = 0; i < 8; ++i) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  } else {
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.o) + base);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint4 w;
      w.x = pack_bf16x2(v[8 * i + 0], v[8 * i + 1]);
      w.y = pack_bf16x2(v[8 * i + 2], v[8 * i + 3]);
      w.z = pack_bf16x2(v[8 * i + 4], v[8 * i + 5]);
      w.w = pack_bf16x2(v[8 * i + 6], v[8 * i + 7]);
      dst[i] = w;
    }
  }
}

}  // namespace b2a
