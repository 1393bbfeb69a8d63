// Kernel body of the tcgen05 causal GQA prefill; see prefill.cuh for the
// design. The host-side launcher (tensor maps, argument checks) is at the end
// of this file and is called from capi.cu.
#include "prefill.cuh"
#include "softmax.cuh"

namespace b2a {

// The running max is only moved (and O rescaled) when the block max exceeds
// it by more than 2^8 in the exp2 domain; otherwise P values stay <= 256,
// which bf16 and the fp32 row sum hold exactly enough. This keeps the
// TMEM round trip for the O rescale off the common path.
constexpr float kRescaleThreshold = 8.0f;

template <int D>
__global__ void __launch_bounds__(384, 1)
    fa_prefill_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ PrefillParams p) {
  using C = PrefillCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  uint8_t* sQ = smem + C::OFF_Q;
  uint8_t* sKV = smem + C::OFF_KV;
  PrefillBars* bars = reinterpret_cast<PrefillBars*>(smem + C::OFF_BAR);
  volatile int* abort_flag = &bars->abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Block -> (query block, head, batch). The heaviest causal query blocks are
  // launched first; the Hq heads of one batch are adjacent so the query heads
  // that share a KV head run together and re-read K/V from L2.
  const int hb = p.Hq * p.B;
  const int lin = blockIdx.x;
  const int qblk = p.n_qblk - 1 - lin / hb;
  const int rem = lin % hb;
  const int h = rem % p.Hq;
  const int b = rem / p.Hq;
  const int hk = h / (p.Hq / p.Hkv);
  const int q0 = qblk * 256;
  const int sp = p.start_pos_arr ? p.start_pos_arr[b] : p.start_pos;
  // Key blocks each query tile needs: n_t[t] for tile t; tile 0 (earlier rows)
  // never needs more blocks than tile 1, and under the causal mask at most one
  // fewer. n_kv = n_t[1] is what gets loaded.
  int n_t[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    if (p.causal) {
      const int last_row = min(q0 + (t + 1) * C::BM - 1, p.Tq - 1);
      const long long kv_end = min((long long)p.Tk, (long long)sp + last_row + 1);
      n_t[t] = kv_end <= 0 ? 0 : (int)((kv_end + C::BN - 1) / C::BN);
    } else {
      n_t[t] = (p.Tk + C::BN - 1) / C::BN;
    }
  }
  const int n_kv = n_t[1];
  const int n0 = n_t[0];

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
#pragma unroll
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      mbar_init(&bars->s_full[t], 1);
      mbar_init(&bars->p_full[t], 4);  // one arrive per softmax warp
      mbar_init(&bars->o_full[t], 1);
    }
    mbar_init(&bars->drain, 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  // Each role's code sits entirely inside the branch that set its register
  // budget, so the compiler allocates it against that budget.
  if (warp < 4) {
  setmaxnreg_dec<C::REGS_LOW>();
  // The producer and the MMA issuer run as whole warps: every lane walks the
  // loop and waits, one elected lane issues each copy / MMA / commit (the *_w
  // helpers), which keeps the operands in uniform registers.
  if (n_kv > 0 && warp == 0) {
    // ------------------------------------------------------------ producer
    mbar_arrive_expect_tx_w(&bars->q_full, C::NQT * C::Q_TILE_BYTES);
#pragma unroll
    for (int t = 0; t < C::NQT; ++t)
#pragma unroll
      for (int c = 0; c < C::KCH; ++c)
        tma_load_4d_w(sQ + t * C::Q_TILE_BYTES + c * C::CHUNK_BYTES, &tm_q, &bars->q_full, c * 64, q0 + t * C::BM,
                      h, b);
    int issued = 0;
    for (int i = 0; i < 2 * n_kv; ++i) {
      const int slot = i % C::STAGES;
      const uint32_t ph = (uint32_t)(i / C::STAGES) & 1u;
      if (!__all_sync(0xffffffffu, mbar_wait(&bars->kv_empty[slot], ph ^ 1u, abort_flag, p.err))) break;
      const int j = i >> 1;
      const CUtensorMap* m = (i & 1) ? &tm_v : &tm_k;
      uint8_t* dst = sKV + slot * C::KV_TILE_BYTES;
      mbar_arrive_expect_tx_w(&bars->kv_full[slot], C::KV_TILE_BYTES);
#pragma unroll
      for (int c = 0; c < C::KCH; ++c)
        tma_load_4d_w(dst + c * C::CHUNK_BYTES, m, &bars->kv_full[slot], c * 64, j * C::BN, hk, b);
      issued = i + 1;
    }
    if (*abort_flag && lane == 0) {
      // Let every copy still in flight land before the CTA releases smem.
      mbar_wait_quiet(&bars->q_full, 0);
      for (int i = max(0, issued - C::STAGES); i < issued; ++i)
        mbar_wait_quiet(&bars->kv_full[i % C::STAGES], (uint32_t)(i / C::STAGES) & 1u);
    }
  } else if (n_kv > 0 && warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    constexpr uint32_t IDESC_S = umma_idesc_bf16(128, C::BN, false);
    constexpr uint32_t IDESC_PV = umma_idesc_bf16(128, D, true);
    // Descriptors are built once; stepping through a tile adds the byte
    // offset >> 4 to the 14-bit start-address field (smem addresses stay
    // below 256 KB, so the field never carries into the next one).
    const uint64_t dQ = make_sdesc_sw128(smem_u32(sQ), 16, 1024);
    const uint64_t dK = make_sdesc_sw128(smem_u32(sKV), 16, 1024);
    const uint64_t dV = make_sdesc_sw128(smem_u32(sKV), C::CHUNK_BYTES, 1024);
    // S_t = Q_t K^T: A = Q tile (K-major), B = K tile (K-major); 16-wide K
    // steps walk 32 bytes inside a 128-byte swizzle row, then the next chunk.
    auto issue_S = [&](int t, int slot) {
      const uint64_t qa = dQ + (uint64_t)((t * C::Q_TILE_BYTES) >> 4);
      const uint64_t ka = dK + (uint64_t)((slot * C::KV_TILE_BYTES) >> 4);
      const uint32_t d = tmem + C::S_COL + t * C::BN;
#pragma unroll
      for (int k = 0; k < D / 16; ++k) {
        const uint64_t off = (uint64_t)(((k >> 2) * C::CHUNK_BYTES + (k & 3) * 32) >> 4);
        umma_bf16_ss_w(d, qa + off, ka + off, IDESC_S, k > 0 ? 1u : 0u);
      }
    };
    // O_t (+)= P_t V: A = P_t in TMEM (16 keys = 8 columns per step), B = V
    // tile read MN-major (head_dim contiguous); a 16-key step is 16 rows =
    // 2048 bytes, 64-column head_dim chunks sit CHUNK_BYTES apart (LBO of dV).
    auto issue_PV = [&](int t, int slot, bool acc) {
      const uint32_t pa = tmem + C::S_COL + t * C::BN;
      const uint64_t va = dV + (uint64_t)((slot * C::KV_TILE_BYTES) >> 4);
      const uint32_t d = tmem + C::O_COL + t * D;
#pragma unroll
      for (int s = 0; s < C::BN / 16; ++s)
        umma_bf16_ts_w(d, pa + 8 * s, va + (uint64_t)((s * 2048) >> 4), IDESC_PV, (acc || s > 0) ? 1u : 0u);
    };
    auto wait_all = [&](uint64_t* bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, p.err));
    };
    auto wait_load = [&](int i) -> bool {
      return wait_all(&bars->kv_full[i % C::STAGES], (uint32_t)(i / C::STAGES) & 1u);
    };

    // Tile 0 runs n0 blocks, tile 1 runs n_kv (n0 <= n_kv): a tile-0 block
    // that lies entirely above the diagonal is neither computed nor waited on.
    if (wait_all(&bars->q_full, 0) && wait_load(0)) {
      tc_fence_after();
      if (n0 > 0) {
        issue_S(0, 0);
        tc_commit_w(&bars->s_full[0]);
      }
      issue_S(1, 0);
      tc_commit_w(&bars->s_full[1]);
      tc_commit_w(&bars->kv_empty[0]);
      // Per key block j: the V_j and K_{j+1} tiles are waited for first
      // (normally long landed; the MMA warp is idle here anyway, waiting for
      // the softmax), so that nothing but the softmax handoffs sits between
      // a tile's PV MMAs and its next S MMAs.
      for (int j = 0; j < n_kv; ++j) {
        const int vslot = (2 * j + 1) % C::STAGES;
        const bool has_next = j + 1 < n_kv;
        const int kslot = (2 * j + 2) % C::STAGES;
        if (!wait_load(2 * j + 1)) break;
        if (has_next && !wait_load(2 * j + 2)) break;
        if (j < n0) {
          if (!wait_all(&bars->p_full[0], (uint32_t)j & 1u)) break;
          tc_fence_after();
          issue_PV(0, vslot, j > 0);
          if (j + 1 == n0) tc_commit_w(&bars->o_full[0]);
          if (j + 1 < n0) {
            issue_S(0, kslot);
            tc_commit_w(&bars->s_full[0]);
          }
        }
        if (!wait_all(&bars->p_full[1], (uint32_t)j & 1u)) break;
        tc_fence_after();
        issue_PV(1, vslot, j > 0);
        tc_commit_w(&bars->kv_empty[vslot]);
        if (!has_next) {
          tc_commit_w(&bars->o_full[1]);
        } else {
          issue_S(1, kslot);
          tc_commit_w(&bars->s_full[1]);
          tc_commit_w(&bars->kv_empty[kslot]);
        }
      }
    }
    // Every MMA issued above must finish before TMEM is deallocated.
    tc_commit_w(&bars->drain);
    mbar_wait_quiet(&bars->drain, 0);
  }
  } else {
    setmaxnreg_inc<C::REGS_HIGH>();
    // ------------------------------------------------------------ softmax + epilogue
    const int t = (warp - 4) >> 2;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    const uint32_t tS = tmem + lane_off + C::S_COL + t * C::BN;
    const uint32_t tO = tmem + lane_off + C::O_COL + t * D;
    const int grow = q0 + t * C::BM + row;
    const bool valid = grow < p.Tq;
    // Last visible key of this row (fits in int: it is below Tk).
    const int kv_last = p.causal ? (int)min((long long)sp + grow, (long long)p.Tk - 1) : p.Tk - 1;
    const float sl2 = p.scale_log2;
    float m_run = -INFINITY;
    float l_run = 0.f;
    bool ok = true;
    const int n_mine = t == 0 ? n0 : n_kv;

    for (int j = 0; j < n_mine; ++j) {
      const bool w = mbar_wait(&bars->s_full[t], (uint32_t)j & 1u, abort_flag, p.err);
      if (!__all_sync(0xffffffffu, w)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // Keys past the row's last visible key are masked; only blocks that
      // cross the diagonal (or the end of K) have any. `full` is warp-uniform:
      // it picks the exp2 pipe split, and the TMEM stores inside the P
      // routines are warp-wide; full blocks skip the mask pass entirely.
      const int lim = max(-1, min(C::BN - 1, kv_last - j * C::BN));
      const bool full = __all_sync(0xffffffffu, lim == C::BN - 1);
      const bool seen = __all_sync(0xffffffffu, m_run != -INFINITY);
      uint32_t s[4][32];
      bool rescale = false;
      float alpha = 1.f;
#define S_AT(i) u2f(s[(i) >> 5][(i) & 31])
      if (full && seen) {
        // Common case: P = exp2(S * scale * log2e - m_run) with the running
        // max of earlier blocks, this block's max tracked on the side. The
        // second half of S is still loading while the first half is done.
        // Only if the block max exceeds m_run by more than the threshold is
        // the row redone with the new max (the first pass's P is overwritten
        // before it is published).
        tmem_ld32(tS, s[0]);
        tmem_ld32(tS + 32, s[1]);
        tmem_wait_ld();
        tmem_ld32(tS + 64, s[2]);
        tmem_ld32(tS + 96, s[3]);
        float2 acc[4];
        float mx[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          acc[k] = make_float2(0.f, 0.f);
          mx[k] = -INFINITY;
        }
        softmax_p_chunks_tmem<4, 0, 2, true, true>(s, sl2, m_run, tS, acc, mx);
        tmem_wait_ld();
        softmax_p_chunks_tmem<4, 2, 2, true, true>(s, sl2, m_run, tS, acc, mx);
        const float2 r2 = __fadd2_rn(__fadd2_rn(acc[0], acc[1]), __fadd2_rn(acc[2], acc[3]));
        float rs = r2.x + r2.y;
        const float m_blk = fmaxf(fmax3(mx[0], mx[1], mx[2]), mx[3]) * sl2;
        const bool jump = m_blk > m_run + kRescaleThreshold;
        if (__any_sync(0xffffffffu, jump)) {
          if (jump) {
            alpha = ex2(m_run - m_blk);
            l_run *= alpha;
            m_run = m_blk;
            rescale = true;
          }
          tmem_wait_st();
          rs = softmax_p_row_tmem<C::BN, false>(s, sl2, m_run, tS);  // rare: MUFU only
        }
        l_run += rs;
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) tmem_ld32(tS + 32 * q, s[q]);
        tmem_wait_ld();
        if (!full) {
#pragma unroll
          for (int i = 0; i < C::BN; ++i)
            if (i > lim) s[i >> 5][i & 31] = f2u(-INFINITY);
        }
        if (seen) {
          // Diagonal block: as above with the exp2 on MUFU only (masked keys
          // give exact zeros).
          float smax;
          float rs = softmax_p_row_tmem<C::BN, false, true>(s, sl2, m_run, tS, &smax);
          const float m_blk = smax * sl2;
          const bool jump = m_blk > m_run + kRescaleThreshold;
          if (__any_sync(0xffffffffu, jump)) {
            if (jump) {
              alpha = ex2(m_run - m_blk);
              l_run *= alpha;
              m_run = m_blk;
              rescale = true;
            }
            tmem_wait_st();
            rs = softmax_p_row_tmem<C::BN, false>(s, sl2, m_run, tS);
          }
          l_run += rs;
        } else {
          // First block (or a row that has seen no key yet): row max first.
          float a0 = -INFINITY, a1 = -INFINITY, a2 = -INFINITY, a3 = -INFINITY;
#pragma unroll
          for (int i = 0; i < C::BN; i += 8) {
            a0 = fmax3(a0, S_AT(i), S_AT(i + 1));
            a1 = fmax3(a1, S_AT(i + 2), S_AT(i + 3));
            a2 = fmax3(a2, S_AT(i + 4), S_AT(i + 5));
            a3 = fmax3(a3, S_AT(i + 6), S_AT(i + 7));
          }
          const float m_new = fmaxf(m_run, fmaxf(fmax3(a0, a1, a2), a3) * sl2);
          if (j == 0) {
            m_run = m_new;
          } else if (m_new > m_run + kRescaleThreshold) {
            alpha = ex2(m_run - m_new);
            l_run *= alpha;
            m_run = m_new;
            rescale = true;
          }
          const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
          l_run += softmax_p_row_tmem<C::BN, false>(s, sl2, m_use, tS);  // once per row: MUFU only
        }
      }
#undef S_AT

      // O_t holds the sum through block j-1 (its last PV finished before
      // S_t(j) did); rescale it before the MMA adds block j.
      if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + 32 * c, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = f2u(u2f(o[i]) * alpha);
          tmem_st32(tO + 32 * c, o);
        }
      }
      // P and any O rescale are in TMEM before the MMA may read them: every
      // lane completes its stores and fences, then one arrive per warp.
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[t]);
    }

    if (n_mine == 0) {
      if (valid) {
        uint32_t z[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) z[i] = 0u;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) store_out_chunk(p, b, h, grow, c, z, 0.f);
        if (p.lse) p.lse[((long long)b * p.Hq + h) * p.Tq + grow] = -INFINITY;
      }
    } else if (ok) {
      const bool w = mbar_wait(&bars->o_full[t], 0, abort_flag, p.err);
      if (__all_sync(0xffffffffu, w)) {
        tc_fence_after();
        const float inv_l = l_run > 0.f ? 1.f / l_run : 0.f;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + 32 * c, o);
          tmem_wait_ld();
          if (valid) store_out_chunk(p, b, h, grow, c, o, inv_l);
        }
        if (p.lse && valid) {
          p.lse[((long long)b * p.Hq + h) * p.Tq + grow] =
              l_run > 0.f ? (m_run + __log2f(l_run)) * 0.69314718055994531f : -INFINITY;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ launcher
template <int D>
static int launch_prefill_t(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                            const PrefillParams& p, cudaStream_t st) {
  using C = PrefillCfg<D>;
  cudaError_t e = cudaFuncSetAttribute(fa_prefill_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       C::SMEM_BYTES);
  if (e != cudaSuccess) return -1;
  // The in-kernel register split needs at least MIN_LAUNCH_REGS per thread.
  cudaFuncAttributes fa{};
  if (cudaFuncGetAttributes(&fa, fa_prefill_kernel<D>) != cudaSuccess || fa.numRegs < C::MIN_LAUNCH_REGS)
    return -1;
  const long long nblk = (long long)p.n_qblk * p.Hq * p.B;
  if (nblk <= 0 || nblk > 0x7fffffffLL) return -2;
  fa_prefill_kernel<D><<<(unsigned)nblk, C::THREADS, C::SMEM_BYTES, st>>>(tq, tk, tv, p);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int launch_prefill(int D, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                   const PrefillParams& p, cudaStream_t st) {
  switch (D) {
    case 64: return launch_prefill_t<64>(tq, tk, tv, p, st);
    case 128: return launch_prefill_t<128>(tq, tk, tv, p, st);
    default: return -3;
  }
}

}  // namespace b2a
