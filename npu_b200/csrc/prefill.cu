// Kernel body of the tcgen05 causal GQA prefill; see prefill.cuh for the
// design. The host-side launcher (tensor maps, argument checks) is at the end
// of this file and is called from capi.cu.
#include "prefill.cuh"
#include "softmax.cuh"

namespace b2a {

#ifndef B2A_ONE_TILE_MAX_ROWS
#define B2A_ONE_TILE_MAX_ROWS 1024
#endif
// Longest query length served by one-tile CTAs (prefill_rows_per_cta).
constexpr int kOneTileMaxRows = B2A_ONE_TILE_MAX_ROWS;


template <int D, int NQT>
__global__ void __launch_bounds__(PrefillCfg<D, NQT>::THREADS, PrefillCfg<D, NQT>::CTAS_PER_SM)
    fa_prefill_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                      const __grid_constant__ PrefillParams p) {
  using C = PrefillCfg<D, NQT>;
  constexpr int kEmuPairs = exp2_emu_pairs<D>();
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
  const int q0 = qblk * (C::BM * C::NQT);
  const int sp = p.start_pos_arr ? p.start_pos_arr[b] : p.start_pos;
  // Key blocks each query tile needs: n_t[t] for tile t; tile 0 (earlier rows)
  // never needs more blocks than tile 1, and under the causal mask at most one
  // fewer. n_kv = n_t[1] is what gets loaded.
  int n_t[C::NQT];
#pragma unroll
  for (int t = 0; t < C::NQT; ++t) {
    if (p.causal) {
      const int last_row = min(q0 + (t + 1) * C::BM - 1, p.Tq - 1);
      const long long kv_end = min((long long)p.Tk, (long long)sp + last_row + 1);
      n_t[t] = kv_end <= 0 ? 0 : (int)((kv_end + C::BN - 1) / C::BN);
    } else {
      n_t[t] = (p.Tk + C::BN - 1) / C::BN;
    }
  }
  const int n_kv = n_t[C::NQT - 1];
  const int n0 = n_t[0];

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
#pragma unroll
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], C::NQT);  // released by every UMMA issuer
    }
#pragma unroll
    for (int t = 0; t < C::NQT; ++t) {
      mbar_init(&bars->sa_full[t], 1);
      mbar_init(&bars->sb_full[t], 1);
      mbar_init(&bars->mid[t], 4);       // one arrive per softmax warp
      mbar_init(&bars->p_full[t], 4);    // one arrive per softmax warp
      mbar_init(&bars->pva_done[t], 1);
      mbar_init(&bars->o_full[t], 1);
    }
#pragma unroll
    for (int t = 0; t < C::NQT; ++t) mbar_init(&bars->drain[t], 1);
    bars->abort_flag = 0;
    fence_mbar_init();
    // The Q tiles and the first ring of K/V tiles are requested here, so
    // their latency overlaps the TMEM allocation and the block barrier below
    // (the producer warp issues the rest). The ring slots are all free.
    if (n_kv > 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(&bars->q_full, C::NQT * C::Q_TILE_BYTES);
#pragma unroll
      for (int t = 0; t < C::NQT; ++t)
#pragma unroll
        for (int c = 0; c < C::KCH; ++c)
          tma_load_4d(sQ + t * C::Q_TILE_BYTES + c * C::CHUNK_BYTES, &tm_q, &bars->q_full, c * 64,
                      q0 + t * C::BM, h, b);
      for (int i = 0; i < min(C::STAGES, 2 * n_kv); ++i) {
        uint8_t* dst = sKV + i * C::KV_TILE_BYTES;
        mbar_arrive_expect_tx(&bars->kv_full[i], C::KV_TILE_BYTES);
#pragma unroll
        for (int c = 0; c < C::KCH; ++c)
          tma_load_4d(dst + c * C::CHUNK_BYTES, (i & 1) ? &tm_v : &tm_k, &bars->kv_full[i], c * 64,
                      (i >> 1) * C::BN, hk, b);
      }
    }
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
    // Q and the first STAGES K/V tiles were requested during set-up.
    int issued = min(C::STAGES, 2 * n_kv);
    for (int i = issued; i < 2 * n_kv; ++i) {
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
  } else if (n_kv > 0 && warp >= 1 && warp <= C::NQT) {
    // ------------------------------------------------------------ UMMA issuers
    // Warp 1 issues tile 0's MMAs, warp 2 (NQT = 2) tile 1's. Each reads
    // every K/V tile it needs and releases it (kv_empty counts NQT arrivals).
    const int t = warp - 1;
    const int nt = t == 0 ? n0 : n_kv;
    constexpr uint32_t IDESC_S = umma_idesc_bf16(128, C::HALF, false);
    constexpr uint32_t IDESC_PV = umma_idesc_bf16(128, D, true);
    // Descriptors are built once; stepping through a tile adds the byte
    // offset >> 4 to the 14-bit start-address field (smem addresses stay
    // below 256 KB, so the field never carries into the next one).
    const uint64_t dQ = make_sdesc_sw128(smem_u32(sQ + t * C::Q_TILE_BYTES), 16, 1024);
    const uint64_t dK = make_sdesc_sw128(smem_u32(sKV), 16, 1024);
    const uint64_t dV = make_sdesc_sw128(smem_u32(sKV), C::CHUNK_BYTES, 1024);
    const uint32_t dS = tmem + C::S_COL + t * C::BN;
    const uint32_t dO = tmem + C::O_COL + t * D;
    // Half h of S_t = Q_t K^T over keys [64 h, 64 h + 64) of the K tile into
    // columns [col, col + 64) of R_t: A = Q tile (K-major), B = 64 K rows
    // (K-major; row 64 starts 8 KB into each 128-row chunk); 16-wide K steps
    // walk 32 bytes inside a 128-byte swizzle row, then the next chunk.
    auto issue_S_half = [&](int slot, int h, uint32_t col) {
      const uint64_t ka = dK + (uint64_t)((slot * C::KV_TILE_BYTES + h * C::HALF * 128) >> 4);
#pragma unroll
      for (int k = 0; k < D / 16; ++k) {
        const uint64_t off = (uint64_t)(((k >> 2) * C::CHUNK_BYTES + (k & 3) * 32) >> 4);
        umma_bf16_ss_w(dS + col, dQ + off, ka + off, IDESC_S, k > 0 ? 1u : 0u);
      }
    };
    // O_t (+)= P_t V over keys [64 h, 64 h + 64): A = P_t in TMEM at columns
    // [pcol + 32 h, pcol + 32 h + 32) of R_t (16 keys = 8 columns per step),
    // B = V rows of those keys read MN-major (head_dim contiguous); a 16-key
    // step is 16 rows = 2048 bytes, 64-column head_dim chunks sit CHUNK_BYTES
    // apart (LBO of dV).
    auto issue_PV_half = [&](int slot, uint32_t pcol, int h, bool acc) {
      const uint64_t va = dV + (uint64_t)((slot * C::KV_TILE_BYTES) >> 4);
#pragma unroll
      for (int s = 4 * h; s < 4 * h + 4; ++s)
        umma_bf16_ts_w(dO, dS + pcol + 8 * s, va + (uint64_t)((s * 2048) >> 4), IDESC_PV, (acc || s > 0) ? 1u : 0u);
    };
    auto wait_all = [&](uint64_t* bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, p.err));
    };
    auto wait_load = [&](int i) -> bool {
      return wait_all(&bars->kv_full[i % C::STAGES], (uint32_t)(i / C::STAGES) & 1u);
    };

    // Per key block j: once the softmax has taken the second half of S_t(j),
    // the first half of S_t(j+1) goes into its columns; once P_t(j) is
    // published, PV_t(j) and then the second half of S_t(j+1) (over P_t(j)'s
    // columns). V_j and K_{j+1} are waited for first (normally long landed).
    // K/V load items are K_j = 2 j, V_j = 2 j + 1; `used` counts the items
    // this warp has released so far, in order.
    bool ok = wait_all(&bars->q_full, 0);
    int used = 0;
    if (ok && nt > 0) {
      ok = wait_load(0);
      if (ok) {
        tc_fence_after();
        issue_S_half(0, 0, 0);
        tc_commit_w(&bars->sa_full[t]);
        issue_S_half(0, 1, C::HALF);
        tc_commit_w(&bars->sb_full[t]);
        tc_commit_w(&bars->kv_empty[0]);
        used = 1;
      }
    }
    for (int j = 0; ok && j < nt; ++j) {
      const int vslot = (2 * j + 1) % C::STAGES;
      const bool next = j + 1 < nt;
      const int kslot = (2 * j + 2) % C::STAGES;
      const uint32_t fcol = (j & 1) ? C::HALF : 0;  // P_t(j), then S_t(j+1)'s second half
      if (!wait_load(2 * j + 1) || (next && !wait_load(2 * j + 2))) break;
      // Mid-block handoff: the next block's first S half (needed first by
      // the softmax), then the first PV half.
      if (!wait_all(&bars->mid[t], (uint32_t)j & 1u)) break;
      tc_fence_after();
      if (next) {
        issue_S_half(kslot, 0, C::HALF - fcol);
        tc_commit_w(&bars->sa_full[t]);
      }
      issue_PV_half(vslot, fcol, 0, j > 0);
      tc_commit_w(&bars->pva_done[t]);
      if (!wait_all(&bars->p_full[t], (uint32_t)j & 1u)) break;
      tc_fence_after();
      issue_PV_half(vslot, fcol, 1, true);
      tc_commit_w(&bars->kv_empty[vslot]);
      if (next) {
        issue_S_half(kslot, 1, fcol);
        tc_commit_w(&bars->sb_full[t]);
        tc_commit_w(&bars->kv_empty[kslot]);
        used = 2 * j + 3;
      } else {
        tc_commit_w(&bars->o_full[t]);
        used = 2 * j + 2;
      }
    }
    // K/V tiles of blocks this tile never reaches (tile 0 stops one block
    // short at the diagonal) are released once they have landed: landing
    // means the slot is in the phase of exactly that tile.
    for (int i = used; ok && i < 2 * n_kv; ++i) {
      if (!wait_load(i)) break;
      if (lane == 0) mbar_arrive(&bars->kv_empty[i % C::STAGES]);
    }
    // Every MMA issued above must finish before TMEM is deallocated.
    tc_commit_w(&bars->drain[t]);
    mbar_wait_quiet(&bars->drain[t], 0);
  }
  } else {
    setmaxnreg_inc<C::REGS_HIGH>();
    // ------------------------------------------------------------ softmax + epilogue
    const int t = (warp - 4) >> 2;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    const uint32_t tR = tmem + lane_off + C::S_COL + t * C::BN;  // this row's S/P region
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
      const uint32_t fcol = (j & 1) ? C::HALF : 0;  // first half of S_t(j); P_t(j) goes here
      const uint32_t scol = C::HALF - fcol;         // second half of S_t(j)
      if (!__all_sync(0xffffffffu, mbar_wait(&bars->sa_full[t], (uint32_t)j & 1u, abort_flag, p.err))) {
        ok = false;
        break;
      }
      tc_fence_after();
      // Keys of block j past the row's last visible key are masked.
      const int lim = kv_last - j * C::BN;
      // One 64-key half at a time (64 registers of S): the first half's P
      // is done while the second half may still be on the tensor core.
      uint32_t s[2][32];
      tmem_ld32(tR + fcol, s[0]);
      tmem_ld32(tR + fcol + 32, s[1]);
      tmem_wait_ld();
      float hs0, hs1;
      const float a0 = softmax_half_tmem<kEmuPairs>(s, lim, sl2, m_run, tR + fcol, hs0);
      auto rescale_O = [&](float f) {
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + 32 * c, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = f2u(u2f(o[i]) * f);
          tmem_st32(tO + 32 * c, o);
        }
      };
      // Second half of S_t(j) (PV_t(j-1) is complete once it is, since it
      // was issued after it).
      if (!__all_sync(0xffffffffu, mbar_wait(&bars->sb_full[t], (uint32_t)j & 1u, abort_flag, p.err))) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (j > 0 && __any_sync(0xffffffffu, a0 != 1.f)) {
        // Rare: the running max moved; O (blocks < j) is brought to it before
        // the first PV half adds block j.
        rescale_O(a0);
      }
      tmem_ld32(tR + scol, s[0]);
      tmem_ld32(tR + scol + 32, s[1]);
      tmem_wait_ld();
      // One handoff: P for keys 0-63 is in TMEM (the first PV half can go)
      // and the second S half is in registers (its columns can take the
      // first half of S_t(j+1)).
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->mid[t]);
      const float a1 = softmax_half_tmem<kEmuPairs>(s, lim - C::HALF, sl2, m_run, tR + fcol + 32, hs1);
      if (__any_sync(0xffffffffu, a1 != 1.f)) {
        // Rare: the second half moved the running max. O then holds blocks
        // < j and the first half of block j (once its PV half completes);
        // bring it to the new max before the second PV half adds to it.
        if (!__all_sync(0xffffffffu, mbar_wait(&bars->pva_done[t], (uint32_t)j & 1u, abort_flag, p.err))) {
          ok = false;
          break;
        }
        tc_fence_after();
        rescale_O(a1);
      }
      l_run = (l_run * a0 + hs0) * a1 + hs1;

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
    } else {
      const bool w = ok && mbar_wait(&bars->o_full[t], 0, abort_flag, p.err);
      // With o_tma the tile's rows are staged in its Q buffer, which no MMA
      // reads any more (all of tile t's S MMAs completed before o_full[t]),
      // and written out by one TMA store; rows past Tq are clipped by it.
      const uint32_t stage = smem_u32(sQ + t * C::Q_TILE_BYTES);
      if (__all_sync(0xffffffffu, w)) {
        tc_fence_after();
        const float inv_l = l_run > 0.f ? 1.f / l_run : 0.f;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + 32 * c, o);
          tmem_wait_ld();
          if (p.o_tma) {
            float v[32];
            if (valid) {
              out_chunk_values(p, b, h, grow, c, o, inv_l, v);
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = 0.f;
            }
            stage_out_chunk_bf16(stage, C::CHUNK_BYTES, row, c, v);
          } else if (valid) {
            store_out_chunk(p, b, h, grow, c, o, inv_l);
          }
        }
        if (p.lse && valid) {
          p.lse[((long long)b * p.Hq + h) * p.Tq + grow] =
              l_run > 0.f ? (m_run + __log2f(l_run)) * 0.69314718055994531f : -INFINITY;
        }
      }
      if (p.o_tma) {
        // Every thread of the tile's warpgroup arrives here exactly once
        // (this branch is tile-uniform), also on the abort path.
        fence_proxy_async_smem();
        named_bar_sync(1 + t, 128);
        if (row == 0 && !*abort_flag) {
#pragma unroll
          for (int c = 0; c < C::KCH; ++c)
            tma_store_4d(&tm_o, sQ + t * C::Q_TILE_BYTES + c * C::CHUNK_BYTES, c * 64, q0 + t * C::BM, h, b);
          tma_store_commit();
          tma_store_wait_read();  // the staging buffer must outlive the copy's reads
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
template <int D, int NQT>
static int launch_prefill_t(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                            const CUtensorMap& to, const PrefillParams& p, cudaStream_t st) {
  using C = PrefillCfg<D, NQT>;
  cudaError_t e = cudaFuncSetAttribute(fa_prefill_kernel<D, NQT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       C::SMEM_BYTES);
  if (e != cudaSuccess) return -1;
  // The in-kernel register split needs at least MIN_LAUNCH_REGS per thread.
  cudaFuncAttributes fa{};
  if (cudaFuncGetAttributes(&fa, fa_prefill_kernel<D, NQT>) != cudaSuccess || fa.numRegs < C::MIN_LAUNCH_REGS)
    return -1;
  const long long nblk = (long long)p.n_qblk * p.Hq * p.B;
  if (nblk <= 0 || nblk > 0x7fffffffLL) return -2;
  fa_prefill_kernel<D, NQT><<<(unsigned)nblk, C::THREADS, C::SMEM_BYTES, st>>>(tq, tk, tv, to, p);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// One-tile CTAs (two per SM) pay off when a CTA sees few key blocks, so that
// its start-up and epilogue are a large share of its time.
int prefill_rows_per_cta(int D, int Tq, int Tk) {
  (void)D;
  (void)Tk;
  return Tq <= kOneTileMaxRows ? 128 : 256;
}

int launch_prefill(int D, int rows_per_cta, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                   const CUtensorMap& to, const PrefillParams& p, cudaStream_t st) {
  const bool one = rows_per_cta == 128;
  switch (D) {
    case 64:
      return one ? launch_prefill_t<64, 1>(tq, tk, tv, to, p, st) : launch_prefill_t<64, 2>(tq, tk, tv, to, p, st);
    case 128:
      return one ? launch_prefill_t<128, 1>(tq, tk, tv, to, p, st)
                 : launch_prefill_t<128, 2>(tq, tk, tv, to, p, st);
    default: return -3;
  }
}

}  // namespace b2a
