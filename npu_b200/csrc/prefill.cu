// Kernel body of the tcgen05 causal GQA prefill; see prefill.cuh for the
// design. The host-side launcher (tensor maps, argument checks) is at the end
// of this file and is called from capi.cu.
#include "prefill.cuh"

namespace b2a {

// The running max is only moved (and O rescaled) when the block max exceeds
// it by more than 2^8 in the exp2 domain; otherwise P values stay <= 256,
// which bf16 and the fp32 row sum hold exactly enough. This keeps the
// TMEM round trip for the O rescale off the common path.
constexpr float kRescaleThreshold = 8.0f;

__device__ __forceinline__ float u2f(uint32_t x) { return __uint_as_float(x); }
__device__ __forceinline__ uint32_t f2u(float x) { return __float_as_uint(x); }

template <int D>
__device__ __forceinline__ void prefill_store_chunk(const PrefillParams& p, int b, int h, int grow, int c,
                                                    const uint32_t (&o)[32], float inv_l) {
  const long long base = (long long)b * p.o_sb + (long long)h * p.o_sh + (long long)grow * p.o_st + 32 * c;
  if (p.out_fp32) {
    float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.o) + base);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      dst[i] = make_float4(u2f(o[4 * i]) * inv_l, u2f(o[4 * i + 1]) * inv_l, u2f(o[4 * i + 2]) * inv_l,
                           u2f(o[4 * i + 3]) * inv_l);
    }
  } else {
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.o) + base);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint4 w;
      w.x = pack_bf16x2(u2f(o[8 * i + 0]) * inv_l, u2f(o[8 * i + 1]) * inv_l);
      w.y = pack_bf16x2(u2f(o[8 * i + 2]) * inv_l, u2f(o[8 * i + 3]) * inv_l);
      w.z = pack_bf16x2(u2f(o[8 * i + 4]) * inv_l, u2f(o[8 * i + 5]) * inv_l);
      w.w = pack_bf16x2(u2f(o[8 * i + 6]) * inv_l, u2f(o[8 * i + 7]) * inv_l);
      dst[i] = w;
    }
  }
}

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
  uint8_t* sP = smem + C::OFF_P;
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
  int n_kv;
  if (p.causal) {
    const int last_row = min(q0 + 255, p.Tq - 1);
    const long long kv_end = min((long long)p.Tk, (long long)sp + last_row + 1);
    n_kv = kv_end <= 0 ? 0 : (int)((kv_end + C::BN - 1) / C::BN);
  } else {
    n_kv = (p.Tk + C::BN - 1) / C::BN;
  }

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
      mbar_init(&bars->p_full[t], 128);
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

  if (n_kv > 0 && warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      mbar_arrive_expect_tx(&bars->q_full, C::NQT * C::Q_TILE_BYTES);
#pragma unroll
      for (int t = 0; t < C::NQT; ++t)
#pragma unroll
        for (int c = 0; c < C::KCH; ++c)
          tma_load_4d(sQ + t * C::Q_TILE_BYTES + c * C::CHUNK_BYTES, &tm_q, &bars->q_full, c * 64,
                      q0 + t * C::BM, h, b);
      int issued = 0;
      for (int i = 0; i < 2 * n_kv; ++i) {
        const int slot = i % C::STAGES;
        const uint32_t ph = (uint32_t)(i / C::STAGES) & 1u;
        if (!mbar_wait(&bars->kv_empty[slot], ph ^ 1u, abort_flag, p.err)) break;
        const int j = i >> 1;
        const CUtensorMap* m = (i & 1) ? &tm_v : &tm_k;
        uint8_t* dst = sKV + slot * C::KV_TILE_BYTES;
        mbar_arrive_expect_tx(&bars->kv_full[slot], C::KV_TILE_BYTES);
#pragma unroll
        for (int c = 0; c < C::KCH; ++c)
          tma_load_4d(dst + c * C::CHUNK_BYTES, m, &bars->kv_full[slot], c * 64, j * C::BN, hk, b);
        issued = i + 1;
      }
      if (*abort_flag) {
        // Let every copy still in flight land before the CTA releases smem.
        mbar_wait_quiet(&bars->q_full, 0);
        for (int i = max(0, issued - C::STAGES); i < issued; ++i)
          mbar_wait_quiet(&bars->kv_full[i % C::STAGES], (uint32_t)(i / C::STAGES) & 1u);
      }
    }
  } else if (n_kv > 0 && warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC_S = umma_idesc_bf16(128, C::BN, false);
      constexpr uint32_t IDESC_PV = umma_idesc_bf16(128, D, true);
      const uint32_t sQa = smem_u32(sQ), sKVa = smem_u32(sKV), sPa = smem_u32(sP);
      // S_t = Q_t K^T: A = Q tile (K-major), B = K tile (K-major); 16-wide K
      // steps walk 32 bytes inside a 128-byte swizzle row, then the next chunk.
      auto issue_S = [&](int t, int slot) {
        const uint32_t qa = sQa + t * C::Q_TILE_BYTES;
        const uint32_t ka = sKVa + slot * C::KV_TILE_BYTES;
        const uint32_t d = tmem + C::S_COL + t * C::BN;
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off = (k >> 2) * C::CHUNK_BYTES + (k & 3) * 32;
          umma_bf16_ss(d, make_sdesc_sw128(qa + off, 16, 1024), make_sdesc_sw128(ka + off, 16, 1024), IDESC_S,
                       k > 0 ? 1u : 0u);
        }
      };
      // O_t (+)= P_t V: A = P tile (K-major over keys), B = V tile read
      // MN-major (head_dim contiguous); a 16-key step is 16 rows = 2048 bytes,
      // 64-column head_dim chunks sit CHUNK_BYTES apart.
      auto issue_PV = [&](int t, int slot, bool acc) {
        const uint32_t pa = sPa + t * C::P_TILE_BYTES;
        const uint32_t va = sKVa + slot * C::KV_TILE_BYTES;
        const uint32_t d = tmem + C::O_COL + t * D;
#pragma unroll
        for (int s = 0; s < C::BN / 16; ++s) {
          const uint32_t aoff = (s >> 2) * C::CHUNK_BYTES + (s & 3) * 32;
          umma_bf16_ss(d, make_sdesc_sw128(pa + aoff, 16, 1024),
                       make_sdesc_sw128(va + s * 2048, C::CHUNK_BYTES, 1024), IDESC_PV,
                       (acc || s > 0) ? 1u : 0u);
        }
      };
      auto wait_load = [&](int i) -> bool {
        return mbar_wait(&bars->kv_full[i % C::STAGES], (uint32_t)(i / C::STAGES) & 1u, abort_flag, p.err);
      };

      bool ok = mbar_wait(&bars->q_full, 0, abort_flag, p.err) && wait_load(0);
      if (ok) {
        tc_fence_after();
        issue_S(0, 0);
        tc_commit(&bars->s_full[0]);
        issue_S(1, 0);
        tc_commit(&bars->s_full[1]);
        tc_commit(&bars->kv_empty[0]);
        for (int j = 0; j < n_kv; ++j) {
          const int vi = 2 * j + 1;
          const int vslot = vi % C::STAGES;
          if (!wait_load(vi)) break;
          if (!mbar_wait(&bars->p_full[0], (uint32_t)j & 1u, abort_flag, p.err)) break;
          tc_fence_after();
          issue_PV(0, vslot, j > 0);
          if (j + 1 == n_kv) tc_commit(&bars->o_full[0]);
          int kslot = 0;
          if (j + 1 < n_kv) {
            const int ki = 2 * j + 2;
            kslot = ki % C::STAGES;
            if (!wait_load(ki)) break;
            tc_fence_after();
            issue_S(0, kslot);
            tc_commit(&bars->s_full[0]);
          }
          if (!mbar_wait(&bars->p_full[1], (uint32_t)j & 1u, abort_flag, p.err)) break;
          tc_fence_after();
          issue_PV(1, vslot, j > 0);
          tc_commit(&bars->kv_empty[vslot]);
          if (j + 1 == n_kv) {
            tc_commit(&bars->o_full[1]);
          } else {
            issue_S(1, kslot);
            tc_commit(&bars->s_full[1]);
            tc_commit(&bars->kv_empty[kslot]);
          }
        }
      }
      // Every MMA issued above must finish before TMEM is deallocated.
      tc_commit(&bars->drain);
      mbar_wait_quiet(&bars->drain, 0);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax + epilogue
    const int t = (warp - 4) >> 2;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    const uint32_t tS = tmem + lane_off + C::S_COL + t * C::BN;
    const uint32_t tO = tmem + lane_off + C::O_COL + t * D;
    const int grow = q0 + t * C::BM + row;
    const bool valid = grow < p.Tq;
    const long long row_pos = (long long)sp + grow;
    const long long kv_last = p.causal ? min(row_pos, (long long)p.Tk - 1) : (long long)p.Tk - 1;
    const float sl2 = p.scale_log2;
    float m_run = -INFINITY;
    float l_run = 0.f;
    const uint32_t pbase = smem_u32(sP) + t * C::P_TILE_BYTES;
    bool ok = true;

    for (int j = 0; j < n_kv; ++j) {
      const bool w = mbar_wait(&bars->s_full[t], (uint32_t)j & 1u, abort_flag, p.err);
      if (!__all_sync(0xffffffffu, w)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t s[4][32];
#pragma unroll
      for (int q = 0; q < 4; ++q) tmem_ld32(tS + 32 * q, s[q]);
      tmem_wait_ld();

      const long long lim_ll = kv_last - (long long)j * C::BN;
      const int lim = lim_ll < -1 ? -1 : (lim_ll > C::BN - 1 ? C::BN - 1 : (int)lim_ll);
      float mx = -INFINITY;
      if (lim == C::BN - 1) {
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int i = 0; i < 32; ++i) mx = fmaxf(mx, u2f(s[q][i]));
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            float v = u2f(s[q][i]);
            if (32 * q + i > lim) v = -INFINITY;
            s[q][i] = f2u(v);
            mx = fmaxf(mx, v);
          }
      }
      const float m_blk = mx * sl2;
      const float m_new = fmaxf(m_run, m_blk);
      bool rescale = false;
      float alpha = 1.f;
      if (j == 0) {
        m_run = m_new;
      } else if (m_new > m_run + kRescaleThreshold) {
        alpha = ex2(m_run - m_new);
        l_run *= alpha;
        m_run = m_new;
        rescale = true;
      }
      const float m_use = (m_run == -INFINITY) ? 0.f : m_run;

      // P = exp2(S * scale * log2e - m), bf16, into the swizzled K-major tile.
      float rs = 0.f;
#pragma unroll
      for (int c8 = 0; c8 < 16; ++c8) {
        float pv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          pv[i] = ex2(fmaf(u2f(s[c8 >> 2][(c8 & 3) * 8 + i]), sl2, -m_use));
          rs += pv[i];
        }
        const int region = c8 >> 3, jj = c8 & 7;
        const uint32_t addr = pbase + region * C::CHUNK_BYTES + row * 128 + ((jj ^ (row & 7)) << 4);
        st_shared_v4(addr, pack_bf16x2(pv[0], pv[1]), pack_bf16x2(pv[2], pv[3]), pack_bf16x2(pv[4], pv[5]),
                     pack_bf16x2(pv[6], pv[7]));
      }
      l_run += rs;

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
        tmem_wait_st();
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->p_full[t]);
    }

    if (n_kv == 0) {
      if (valid) {
        uint32_t z[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) z[i] = 0u;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) prefill_store_chunk<D>(p, b, h, grow, c, z, 0.f);
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
          if (valid) prefill_store_chunk<D>(p, b, h, grow, c, o, inv_l);
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
