// Causal GQA prefill for head_dim 256 (the Qwen3.6 attention geometry,
// qwen/forward.py:6-7: 16 query heads over 2 KV heads, D=256), sm_100a.
//
// Same semantics as fa_prefill_kernel (prefill.cu). TMEM cannot hold two
// 128 x 256 fp32 output tiles plus scores, so one CTA owns ONE 128-row query
// tile and overlaps across key blocks instead of across query tiles:
//   TMEM: S[0], S[1] (64 fp32 columns each, double-buffered; P[b] is written
//         over the first 32 columns of S[b]), Q (128 columns of packed bf16,
//         copied in once), O (256 columns)
//   smem: Q staging (64 KB), a 5-stage ring of 64-key K / V tiles (32 KB each)
// Both MMAs take their A operand from TMEM (Q for S = Q K^T, P for O += P V),
// so shared memory only carries K and V: its bandwidth, shared by the
// tensor core's operand reads and the TMA fills, is what bounds this kernel.
// MMA order: S(0), S(1), then per block j: PV(j), S(j+2). While the softmax
// warpgroup turns S(j) into P(j), the tensor core runs PV(j-1) and S(j+1).
// Warps: 0 TMA, 1 TMEM + MMA issue, 2-3 idle, 4-7 softmax + epilogue.
#include "prefill.cuh"
#include "softmax.cuh"

namespace b2a {

struct D256Cfg {
  static constexpr int D = 256;
  static constexpr int BM = 128;
  static constexpr int BN = 64;
  static constexpr int KCH = D / 64;                  // 4 swizzle chunks per row
  static constexpr int Q_CHUNK = BM * 128;            // 16 KB: 128 rows x 128 B
  static constexpr int KV_CHUNK = BN * 128;           // 8 KB: 64 rows x 128 B
  static constexpr int Q_BYTES = KCH * Q_CHUNK;       // 64 KB
  static constexpr int KV_TILE_BYTES = KCH * KV_CHUNK;  // 32 KB
  static constexpr int STAGES = 5;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_KV = OFF_Q + Q_BYTES;
  static constexpr int OFF_BAR = OFF_KV + STAGES * KV_TILE_BYTES;
  static constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;
  static constexpr int TMEM_COLS = 512;
  static constexpr int S_COL = 0;    // S[b] at b * BN, P[b] over its first BN / 2
  static constexpr int Q_COL = 128;  // Q (bf16 pairs) at 128 .. 255
  static constexpr int O_COL = 256;  // O at 256 .. 511
  static constexpr int THREADS = 256;  // 1 CTA per SM: up to 255 registers per thread
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

struct D256Bars {
  uint64_t q_full;
  uint64_t q_tmem;
  uint64_t kv_full[8];
  uint64_t kv_empty[8];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t pv_done;
  uint64_t o_full;
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};

// The running max moves (and O is rescaled) only past a 2^8 gap; see prefill.cu.
constexpr float kRescaleThresholdD256 = 8.0f;

// Order in which the producer loads tiles and the MMA issuer consumes them:
// K0, K1, then for each block j: V_j followed by K_{j+2} (when it exists).
// Returns true for a V tile; *blk receives the key block index.
__device__ __forceinline__ bool d256_load_item(int i, int n, int* blk) {
  if (n == 1) {
    *blk = 0;
    return i == 1;
  }
  if (i < 2) {
    *blk = i;
    return false;
  }
  // After K0, K1 the sequence is V0, K2, V1, K3, ..., V_{n-3}, K_{n-1}, V_{n-2}, V_{n-1}.
  const int r = i - 2;
  const int pairs = n - 2;  // (V_j, K_{j+2}) for j < n - 2
  if (r < 2 * pairs) {
    *blk = (r & 1) ? (r >> 1) + 2 : (r >> 1);
    return (r & 1) == 0;
  }
  *blk = (n - 2) + (r - 2 * pairs);
  return true;
}

__global__ void __launch_bounds__(256, 1)
    fa_prefill_d256_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                           const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ PrefillParams p) {
  using C = D256Cfg;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  uint8_t* sQ = smem + C::OFF_Q;
  uint8_t* sKV = smem + C::OFF_KV;
  D256Bars* bars = reinterpret_cast<D256Bars*>(smem + C::OFF_BAR);
  volatile int* abort_flag = &bars->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // Block -> (query tile, head, batch), heaviest causal tiles first.
  const int hb = p.Hq * p.B;
  const int lin = blockIdx.x;
  const int qt = p.n_qblk - 1 - lin / hb;
  const int rem = lin % hb;
  const int h = rem % p.Hq, b = rem / p.Hq;
  const int hk = h / (p.Hq / p.Hkv);
  const int q0 = qt * C::BM;
  const int sp = p.start_pos_arr ? p.start_pos_arr[b] : p.start_pos;
  int n;
  if (p.causal) {
    const int last_row = min(q0 + C::BM - 1, p.Tq - 1);
    const long long kv_end = min((long long)p.Tk, (long long)sp + last_row + 1);
    n = kv_end <= 0 ? 0 : (int)((kv_end + C::BN - 1) / C::BN);
  } else {
    n = (p.Tk + C::BN - 1) / C::BN;
  }
  const int n_items = n == 0 ? 0 : 2 * n;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->q_tmem, 128);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->s_full[s], 1);
      mbar_init(&bars->p_full[s], 128);
    }
    mbar_init(&bars->pv_done, 1);
    mbar_init(&bars->o_full, 1);
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

  if (warp < 4) {
    // Producer and MMA issuer run as whole warps; one elected lane issues
    // each copy / MMA / commit (the *_w helpers).
    if (n > 0 && warp == 0) {
      // -------------------------------------------------------- producer
      mbar_arrive_expect_tx_w(&bars->q_full, C::Q_BYTES);
      for (int c = 0; c < C::KCH; ++c)
        tma_load_4d_w(sQ + c * C::Q_CHUNK, &tm_q, &bars->q_full, c * 64, q0, h, b);
      int issued = 0;
      for (int i = 0; i < n_items; ++i) {
        const int slot = i % C::STAGES;
        if (!__all_sync(0xffffffffu,
                        mbar_wait(&bars->kv_empty[slot], ((uint32_t)(i / C::STAGES) & 1u) ^ 1u, abort_flag, p.err)))
          break;
        int blk;
        const bool is_v = d256_load_item(i, n, &blk);
        uint8_t* dst = sKV + slot * C::KV_TILE_BYTES;
        mbar_arrive_expect_tx_w(&bars->kv_full[slot], C::KV_TILE_BYTES);
        for (int c = 0; c < C::KCH; ++c)
          tma_load_4d_w(dst + c * C::KV_CHUNK, is_v ? &tm_v : &tm_k, &bars->kv_full[slot], c * 64, blk * C::BN, hk,
                      b);
        issued = i + 1;
      }
      if (*abort_flag && lane == 0) {
        mbar_wait_quiet(&bars->q_full, 0);
        for (int i = max(0, issued - C::STAGES); i < issued; ++i)
          mbar_wait_quiet(&bars->kv_full[i % C::STAGES], (uint32_t)(i / C::STAGES) & 1u);
      }
    } else if (n > 0 && warp == 1) {
      // -------------------------------------------------------- UMMA issuer
      constexpr uint32_t IDESC_S = umma_idesc_bf16(128, C::BN, false);
      constexpr uint32_t IDESC_PV = umma_idesc_bf16(128, C::D, true);
      const uint64_t dK = make_sdesc_sw128(smem_u32(sKV), 16, 1024);
      const uint64_t dV = make_sdesc_sw128(smem_u32(sKV), C::KV_CHUNK, 1024);
      int li = 0;  // next load item to consume
      auto wait_item = [&]() -> int {
        const int slot = li % C::STAGES;
        const bool ok = __all_sync(
            0xffffffffu, mbar_wait(&bars->kv_full[slot], (uint32_t)(li / C::STAGES) & 1u, abort_flag, p.err));
        ++li;
        return ok ? slot : -1;
      };
      // S[buf] = Q K^T: A = Q in TMEM (8 columns per 16-wide K-step), B = the
      // K tile in smem (4 chunks of 128 B rows, 32 B per K-step inside one).
      auto issue_S = [&](int buf, int slot) {
        const uint64_t ka = dK + (uint64_t)((slot * C::KV_TILE_BYTES) >> 4);
        const uint32_t d = tmem + C::S_COL + buf * C::BN;
#pragma unroll
        for (int k = 0; k < C::D / 16; ++k) {
          const uint64_t ko = (uint64_t)(((k >> 2) * C::KV_CHUNK + (k & 3) * 32) >> 4);
          umma_bf16_ts_w(d, tmem + C::Q_COL + 8 * k, ka + ko, IDESC_S, k > 0 ? 1u : 0u);
        }
      };
      // O (+)= P[buf] V: A = P[buf] in TMEM (4 K-steps of 16 keys), B = V read
      // MN-major with its four 64-column head_dim chunks KV_CHUNK apart.
      auto issue_PV = [&](int buf, int slot, bool acc) {
        const uint32_t pa = tmem + C::S_COL + buf * C::BN;
        const uint64_t va = dV + (uint64_t)((slot * C::KV_TILE_BYTES) >> 4);
#pragma unroll
        for (int s = 0; s < C::BN / 16; ++s)
          umma_bf16_ts_w(tmem + C::O_COL, pa + 8 * s, va + (uint64_t)((s * 2048) >> 4), IDESC_PV,
                       (acc || s > 0) ? 1u : 0u);
      };
      bool ok = __all_sync(0xffffffffu, mbar_wait(&bars->q_tmem, 0, abort_flag, p.err));
      for (int j0 = 0; ok && j0 < min(n, 2); ++j0) {
        const int slot = wait_item();
        if (slot < 0) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_S(j0, slot);
        tc_commit_w(&bars->s_full[j0]);
        tc_commit_w(&bars->kv_empty[slot]);
      }
      for (int j = 0; ok && j < n; ++j) {
        const int vslot = wait_item();
        if (vslot < 0) break;
        if (!__all_sync(0xffffffffu, mbar_wait(&bars->p_full[j & 1], (uint32_t)(j >> 1) & 1u, abort_flag, p.err)))
          break;
        tc_fence_after();
        issue_PV(j & 1, vslot, j > 0);
        tc_commit_w(&bars->pv_done);
        tc_commit_w(&bars->kv_empty[vslot]);
        if (j + 2 < n) {
          const int kslot = wait_item();
          if (kslot < 0) break;
          tc_fence_after();
          issue_S(j & 1, kslot);
          tc_commit_w(&bars->s_full[j & 1]);
          tc_commit_w(&bars->kv_empty[kslot]);
        }
      }
      tc_commit_w(&bars->o_full);
      tc_commit_w(&bars->drain);
      mbar_wait_quiet(&bars->drain, 0);
    }
  } else {
    // ---------------------------------------------------------- softmax + epilogue
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    const uint32_t tO = tmem + lane_off + C::O_COL;
    const int grow = q0 + row;
    const bool valid = grow < p.Tq;
    const long long row_pos = (long long)sp + grow;
    const long long kv_last = p.causal ? min(row_pos, (long long)p.Tk - 1) : (long long)p.Tk - 1;
    const float sl2 = p.scale_log2;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    if (n > 0) {
      // Copy this thread's row of Q from the swizzled staging tile into TMEM
      // (bf16 pairs, 128 columns) for the S MMA's A operand.
      const bool w = mbar_wait(&bars->q_full, 0, abort_flag, p.err);
      ok = __all_sync(0xffffffffu, w);
      if (ok) {
        const uint32_t qrow = smem_u32(sQ) + row * 128;
#pragma unroll
        for (int c = 0; c < C::KCH; ++c) {
          uint32_t r[32];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const uint32_t a = qrow + c * C::Q_CHUNK + ((u ^ (row & 7)) << 4);
            asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(r[4 * u]), "=r"(r[4 * u + 1]), "=r"(r[4 * u + 2]), "=r"(r[4 * u + 3])
                         : "r"(a));
          }
          tmem_st32(tmem + lane_off + C::Q_COL + 32 * c, r);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&bars->q_tmem);
      }
    }
    for (int j = 0; ok && j < n; ++j) {
      const int buf = j & 1;
      const bool w = mbar_wait(&bars->s_full[buf], (uint32_t)(j >> 1) & 1u, abort_flag, p.err);
      if (!__all_sync(0xffffffffu, w)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t s[2][32];
      tmem_ld32(tmem + lane_off + C::S_COL + buf * C::BN, s[0]);
      tmem_ld32(tmem + lane_off + C::S_COL + buf * C::BN + 32, s[1]);
      tmem_wait_ld();
#define S_AT(i) u2f(s[(i) >> 5][(i) & 31])
      const long long lim_ll = kv_last - (long long)j * C::BN;
      const int lim = lim_ll < -1 ? -1 : (lim_ll > C::BN - 1 ? C::BN - 1 : (int)lim_ll);
      if (lim < C::BN - 1) {
#pragma unroll
        for (int i = 0; i < C::BN; ++i)
          if (i > lim) s[i >> 5][i & 31] = f2u(-INFINITY);
      }
      float a0 = -INFINITY, a1 = -INFINITY, a2 = -INFINITY, a3 = -INFINITY;
#pragma unroll
      for (int i = 0; i < C::BN; i += 8) {
        a0 = fmax3(a0, S_AT(i), S_AT(i + 1));
        a1 = fmax3(a1, S_AT(i + 2), S_AT(i + 3));
        a2 = fmax3(a2, S_AT(i + 4), S_AT(i + 5));
        a3 = fmax3(a3, S_AT(i + 6), S_AT(i + 7));
      }
      const float m_new = fmaxf(m_run, fmaxf(fmax3(a0, a1, a2), a3) * sl2);
      bool rescale = false;
      float alpha = 1.f;
      if (j == 0) {
        m_run = m_new;
      } else if (m_new > m_run + kRescaleThresholdD256) {
        alpha = ex2(m_run - m_new);
        l_run *= alpha;
        m_run = m_new;
        rescale = true;
      }
      const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
      const uint32_t tP = tmem + lane_off + C::S_COL + buf * C::BN;
      // Warp-uniform choice: the TMEM stores inside are warp-wide.
      if (__all_sync(0xffffffffu, lim == C::BN - 1))
        l_run += softmax_p_row_tmem<C::BN, true>(s, sl2, m_use, tP);
      else
        l_run += softmax_p_row_tmem<C::BN, false>(s, sl2, m_use, tP);
#undef S_AT
      if (__any_sync(0xffffffffu, rescale)) {
        // O holds blocks up to j-1 once PV(j-1) has completed.
        const bool pw = mbar_wait(&bars->pv_done, (uint32_t)(j - 1) & 1u, abort_flag, p.err);
        if (!__all_sync(0xffffffffu, pw)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < C::D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + 32 * c, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = f2u(u2f(o[i]) * alpha);
          tmem_st32(tO + 32 * c, o);
        }
      }
      tmem_wait_st();  // P and any O rescale are in TMEM before the MMA reads them
      tc_fence_before();
      mbar_arrive(&bars->p_full[buf]);
    }
    if (n == 0) {
      if (valid) {
        uint32_t z[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) z[i] = 0u;
        for (int c = 0; c < C::D / 32; ++c) store_out_chunk(p, b, h, grow, c, z, 0.f);
        if (p.lse) p.lse[((long long)b * p.Hq + h) * p.Tq + grow] = -INFINITY;
      }
    } else if (ok) {
      const bool w = mbar_wait(&bars->o_full, 0, abort_flag, p.err);
      if (__all_sync(0xffffffffu, w)) {
        tc_fence_after();
        const float inv_l = l_run > 0.f ? 1.f / l_run : 0.f;
#pragma unroll 1
        for (int c = 0; c < C::D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + 32 * c, o);
          tmem_wait_ld();
          if (valid) store_out_chunk(p, b, h, grow, c, o, inv_l);
        }
        if (p.lse && valid)
          p.lse[((long long)b * p.Hq + h) * p.Tq + grow] =
              l_run > 0.f ? (m_run + __log2f(l_run)) * 0.69314718055994531f : -INFINITY;
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

int launch_prefill_d256(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                        const PrefillParams& p, cudaStream_t st) {
  using C = D256Cfg;
  if (cudaFuncSetAttribute(fa_prefill_d256_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES) !=
      cudaSuccess)
    return -1;
  const long long nblk = (long long)p.n_qblk * p.Hq * p.B;
  if (nblk <= 0 || nblk > 0x7fffffffLL) return -2;
  fa_prefill_d256_kernel<<<(unsigned)nblk, C::THREADS, C::SMEM_BYTES, st>>>(tq, tk, tv, p);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace b2a
