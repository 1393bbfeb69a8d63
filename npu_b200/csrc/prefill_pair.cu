// Causal GQA prefill on SM pairs (head_dim 128): tcgen05.mma.cta_group::2.
//
// Same semantics as fa_prefill_kernel (prefill.cu): causal mask on absolute
// positions (npu/fa_ref.py:57-60), rows with no unmasked key give 0
// (npu/fa_ref.py:112-128), query head h reads KV head h / (Hq / Hkv).
//
// A work item runs on a cluster of two CTAs on two SMs. Both CTAs take the
// same 256 query rows: CTA r of the pair takes query head 2 i + r of a GQA
// group, so they read the same K/V. Each CTA holds its own two 128-row Q
// tiles, and every UMMA is M = 256 over the pair, rows 0-127 from CTA 0 and
// rows 128-255 from CTA 1. The B operand is split across the two SMs:
//  - S = Q K^T runs as two N = 64 halves per key block. CTA r holds keys
//    64 h + 32 r .. + 32 of half h.
//  - O += P V runs with N = D = 128. CTA r holds head_dim columns
//    64 r .. + 64 of V.
// So each SM loads half of every K/V tile (32 KB per key block instead of
// 64 KB) and its tensor core reads half of every B operand from its own
// shared memory. The per-SM shared-memory traffic that co-bounds the one-SM
// kernel (the N = 64 SS UMMAs re-read Q, plus the K/V fills) drops by ~30 %,
// and the K/V ring holds twice the key blocks.
//
// Roles. CTA 0 of the pair (the leader) issues every UMMA for both CTAs
// (warp 1: tile 0, warp 2: tile 1). Warp 0 of each CTA loads that CTA's Q
// tiles and K/V halves; the TMA completes on the leader's barriers
// (cp.async.bulk.tensor .cta_group::2, no multicast). The leader's commits
// arrive on the barrier at the same offset in both CTAs (tcgen05.commit with
// a CTA mask of 0b11). Each CTA's softmax warps arrive on the leader's mid /
// p_full barriers (remote mbarrier.arrive through mapa). Warps 4-11 of each
// CTA run the softmax and epilogue on their own TMEM exactly as the one-SM
// kernel does: the S-half / P / O column plan, the mid-block handoff and the
// rescale rules are the same. Every wait is bounded. TMEM is allocated and
// freed for the pair (tcgen05.alloc .cta_group::2, issued by warp 1 of both
// CTAs). A cluster barrier after set-up and another before the free keep
// either CTA's shared memory alive while the other can still reach it.
// Limitation of the abort path (a wait past its bound, which sets the error
// word): the peer CTA's K/V loads complete on the leader's barriers. So the
// peer cannot wait for its own copies in flight before it leaves, as the
// one-SM kernel's producer does. A late copy can then land in shared memory
// that the SM has already given to a later CTA. The launch has failed by
// then (the host reads the error word), and nothing leaves the SM's own
// shared memory.
//
// Measured slower than the one-SM kernel (every half-block handoff waits for
// both SMs). It is selected only when the caller sets B2A_PREFILL_SM_PAIRS
// (prefill.cu, prefill_plan).
#include "prefill.cuh"
#include "softmax.cuh"

namespace b2a {

// ------------------------------------------------------------ pair PTX
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of `addr` (a shared::cta address) in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// All threads of both CTAs.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::
          : "memory");
}

// Arrive on an mbarrier given by its shared::cluster address (this CTA's or
// the peer's).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t caddr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(caddr) : "memory");
}

// 4-D tiled load into this CTA's shared memory whose completion bytes go to
// an mbarrier of either CTA of the pair (shared::cluster address). Warp-wide:
// one elected lane issues.
__device__ __forceinline__ void tma_load_4d_pair_w(void* smem_dst, const CUtensorMap* map, uint32_t bar_caddr,
                                                   int c0, int c1, int c2, int c3) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];\n\t}\n" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_caddr), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// TMEM allocation for the pair: warp 1 of both CTAs issues each of these.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// M = 256 UMMAs over the pair (issued by the leader; warp-wide, elected lane).
__device__ __forceinline__ void umma_pair_ss_w(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_pair_ts_w(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the barrier at this offset in both CTAs once every UMMA the
// leader issued so far has completed (CTA mask 0b11).
__device__ __forceinline__ void tc_commit_both_w(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t.reg .b16 m;\n\t"
      "mov.b16 m, 3;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}\n" ::
          "r"(smem_u32(bar))
      : "memory");
}
// The same, on this (the leader's) CTA only.
__device__ __forceinline__ void tc_commit_own_w(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}\n" ::"r"(
          smem_u32(bar))
      : "memory");
}

// ------------------------------------------------------------ configuration
struct PairCfg {
  static constexpr int D = 128;
  static constexpr int BM = 128, BN = 128, NQT = 2;
  static constexpr int KCH = D / 64;                 // 128-byte chunks per Q / K row
  static constexpr int Q_CHUNK = BM * 128;           // 16 KB: 128 rows x 128 B
  static constexpr int Q_TILE_BYTES = BM * D * 2;    // 32 KB
  static constexpr int KH_ROWS = 32;                 // keys of an S half held per CTA
  static constexpr int K_CHUNK = KH_ROWS * 128;      // 4 KB: 32 rows x 128 B
  static constexpr int KH_BYTES = KCH * K_CHUNK;     // 8 KB: one S half's keys, all of D
  static constexpr int KV_TILE_BYTES = 2 * KH_BYTES; // 16 KB: a K half-tile or a V half-tile
  static_assert(KV_TILE_BYTES == BN * 64 * 2, "a V half-tile is 128 keys x 64 head_dim columns");
  static constexpr int STAGES = 10;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_KV = OFF_Q + NQT * Q_TILE_BYTES;
  static constexpr int OFF_BAR = OFF_KV + STAGES * KV_TILE_BYTES;
  static constexpr int BAR_BYTES = 512;
  static constexpr int SMEM_BYTES = OFF_BAR + BAR_BYTES + 1024;
  static constexpr int TMEM_COLS = 512;
  static constexpr int S_COL = 0, HALF = BN / 2, O_COL = NQT * BN;
  static constexpr int THREADS = 384;
  static constexpr int REGS_LOW = 112, REGS_HIGH = 184;
  static constexpr int MIN_LAUNCH_REGS = (128 * REGS_LOW + 256 * REGS_HIGH + THREADS - 1) / THREADS;
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static_assert(O_COL + NQT * D <= TMEM_COLS, "TMEM budget");
};

struct PairBars {
  uint64_t q_full;       // leader: both CTAs' Q tiles landed
  uint64_t kv_full[10];  // leader: both CTAs' halves of a load item landed
  uint64_t kv_empty[10]; // both: the leader's MMAs that read the slot completed
  uint64_t sa_full[2], sb_full[2], pva_done[2], o_full[2];  // both
  uint64_t mid[2], p_full[2];  // leader: 8 softmax warps (4 per CTA)
  uint64_t drain[2];     // leader
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(PairBars) <= PairCfg::BAR_BYTES, "barrier area");

// ------------------------------------------------------------ kernel
// Work item -> (query block, batch, head pair). Heaviest query blocks first;
// the head pairs of a KV head adjacent, so they share K/V through L2.
struct PairItem {
  int h, b, hk, q0, sp;
  int n_t[2];  // key blocks each 128-row tile needs (tile 0 never more)
};

__device__ __forceinline__ PairItem pair_item(const PrefillParams& p, int item, int rank) {
  constexpr int BM = 128, BN = 128;
  PairItem it;
  const int np = p.Hq / p.Hkv / 2;  // head pairs per KV head
  const int per = p.B * p.Hkv * np;
  const int qblk = p.n_qblk - 1 - item / per;
  const int rem = item % per;
  const int pair = rem % np;
  const int bk = rem / np;
  it.hk = bk % p.Hkv;
  it.b = bk / p.Hkv;
  it.h = it.hk * (2 * np) + 2 * pair + rank;
  it.q0 = qblk * 2 * BM;
  it.sp = p.start_pos_arr ? p.start_pos_arr[it.b] : p.start_pos;
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    if (p.causal) {
      const int last_row = min(it.q0 + BM * t + BM - 1, p.Tq - 1);
      const long long kv_end = min((long long)p.Tk, (long long)it.sp + last_row + 1);
      it.n_t[t] = kv_end <= 0 ? 0 : (int)((kv_end + BN - 1) / BN);
    } else {
      it.n_t[t] = (p.Tk + BN - 1) / BN;
    }
  }
  return it;
}

__global__ void __launch_bounds__(PairCfg::THREADS, 1)
    fa_prefill_pair_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                           const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ PrefillParams p) {
  using C = PairCfg;
  constexpr int D = C::D;
  constexpr int kEmuPairs = exp2_emu_pairs<D>();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  uint8_t* sQ = smem + C::OFF_Q;
  uint8_t* sKV = smem + C::OFF_KV;
  PairBars* bars = reinterpret_cast<PairBars*>(smem + C::OFF_BAR);
  volatile int* abort_flag = &bars->abort_flag;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool lead = rank == 0;
  // shared::cluster address of a barrier in the leader's shared memory.
  auto at_lead = [&](uint64_t* bar) -> uint32_t { return mapa_shared(smem_u32(bar), 0); };
  auto wait_all = [&](uint64_t* bar, uint32_t parity) -> bool {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, p.err));
  };

  const PairItem it = pair_item(p, (int)(blockIdx.x >> 1), (int)rank);
  const int n_kv = it.n_t[1];

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
#pragma unroll
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], C::NQT);  // one commit per UMMA issuer warp
    }
#pragma unroll
    for (int t = 0; t < C::NQT; ++t) {
      mbar_init(&bars->sa_full[t], 1);
      mbar_init(&bars->sb_full[t], 1);
      mbar_init(&bars->pva_done[t], 1);
      mbar_init(&bars->o_full[t], 1);
      mbar_init(&bars->mid[t], 8);  // 4 softmax warps in each CTA
      mbar_init(&bars->p_full[t], 8);
      mbar_init(&bars->drain[t], 1);
    }
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  if (warp == 1) {
    tmem_alloc_pair(&bars->tmem_base, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  // Both CTAs' barriers are initialised (and TMEM allocated) before either
  // CTA signals the other's.
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp < 4) {
    setmaxnreg_dec<C::REGS_LOW>();
    if (warp == 0 && n_kv > 0) {
      // -------------------------------------------------------- producer
      // This CTA's Q tiles, then its halves of K_j and V_j through the ring
      // (load item 2 j is K_j, 2 j + 1 is V_j); bytes complete on the
      // leader's barriers, which expect both CTAs' halves.
      const uint32_t q_bar = at_lead(&bars->q_full);
      if (lead) mbar_arrive_expect_tx_w(&bars->q_full, 2 * C::NQT * C::Q_TILE_BYTES);
#pragma unroll
      for (int t = 0; t < C::NQT; ++t)
#pragma unroll
        for (int c = 0; c < C::KCH; ++c)
          tma_load_4d_pair_w(sQ + t * C::Q_TILE_BYTES + c * C::Q_CHUNK, &tm_q, q_bar, c * 64, it.q0 + 128 * t,
                             it.h, it.b);
      for (int i = 0; i < 2 * n_kv; ++i) {
        const int slot = i % C::STAGES;
        if (!wait_all(&bars->kv_empty[slot], ((uint32_t)(i / C::STAGES) & 1u) ^ 1u)) break;
        if (lead) mbar_arrive_expect_tx_w(&bars->kv_full[slot], 2 * C::KV_TILE_BYTES);
        const uint32_t bar = at_lead(&bars->kv_full[slot]);
        uint8_t* dst = sKV + slot * C::KV_TILE_BYTES;
        const int j = i >> 1;
        if ((i & 1) == 0) {
          // K_j: keys 64 h + 32 rank .. + 32 of each S half h, all of D.
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int c = 0; c < C::KCH; ++c)
              tma_load_4d_pair_w(dst + h * C::KH_BYTES + c * C::K_CHUNK, &tm_k, bar, c * 64,
                                 j * C::BN + 64 * h + 32 * (int)rank, it.hk, it.b);
        } else {
          // V_j: all 128 keys, head_dim columns 64 rank .. + 64.
          tma_load_4d_pair_w(dst, &tm_v, bar, 64 * (int)rank, j * C::BN, it.hk, it.b);
        }
      }
    } else if (lead && (warp == 1 || warp == 2) && n_kv > 0) {
      // -------------------------------------------------------- UMMA issuers (leader)
      const int t = warp - 1;
      constexpr uint32_t IDESC_S = umma_idesc_bf16(256, C::HALF, false);
      constexpr uint32_t IDESC_PV = umma_idesc_bf16(256, D, true);
      const uint64_t dQ = make_sdesc_sw128(smem_u32(sQ + t * C::Q_TILE_BYTES), 16, 1024);
      const uint64_t dK = make_sdesc_sw128(smem_u32(sKV), 16, 1024);
      const uint64_t dV = make_sdesc_sw128(smem_u32(sKV), C::KV_TILE_BYTES, 1024);
      const uint32_t dS = tmem + C::S_COL + t * C::BN;
      const uint32_t dO = tmem + C::O_COL + t * D;
      // Half h of S_t over keys [64 h, 64 h + 64) into columns [col, col + 64):
      // A = the pair's Q tiles t, B = each CTA's 32 keys of that half.
      auto issue_S_half = [&](int slot, int h, uint32_t col) {
        const uint64_t kb = dK + (uint64_t)((slot * C::KV_TILE_BYTES + h * C::KH_BYTES) >> 4);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint64_t qo = (uint64_t)(((k >> 2) * C::Q_CHUNK + (k & 3) * 32) >> 4);
          const uint64_t ko = (uint64_t)(((k >> 2) * C::K_CHUNK + (k & 3) * 32) >> 4);
          umma_pair_ss_w(dS + col, dQ + qo, kb + ko, IDESC_S, k > 0 ? 1u : 0u);
        }
      };
      // O_t (+)= P_t V over keys [64 h, 64 h + 64): A = P_t in TMEM, B = each
      // CTA's 64 head_dim columns of V (MN-major, 16 keys = 2 KB per K-step).
      auto issue_PV_half = [&](int slot, uint32_t pcol, int h, bool acc) {
        const uint64_t va = dV + (uint64_t)((slot * C::KV_TILE_BYTES) >> 4);
#pragma unroll
        for (int s = 4 * h; s < 4 * h + 4; ++s)
          umma_pair_ts_w(dO, dS + pcol + 8 * s, va + (uint64_t)((s * 2048) >> 4), IDESC_PV,
                         (acc || s > 0) ? 1u : 0u);
      };
      const int nt = t == 0 ? it.n_t[0] : n_kv;
      auto wait_load = [&](int i) -> bool {
        return wait_all(&bars->kv_full[i % C::STAGES], (uint32_t)(i / C::STAGES) & 1u);
      };
      bool ok = wait_all(&bars->q_full, 0);
      int used = 0;
      if (ok && nt > 0) {
        ok = wait_load(0);
        if (ok) {
          tc_fence_after();
          issue_S_half(0, 0, 0);
          tc_commit_both_w(&bars->sa_full[t]);
          issue_S_half(0, 1, C::HALF);
          tc_commit_both_w(&bars->sb_full[t]);
          tc_commit_both_w(&bars->kv_empty[0]);
          used = 1;
        }
      }
      for (int j = 0; ok && j < nt; ++j) {
        const uint32_t par = (uint32_t)j & 1u;
        const int vslot = (2 * j + 1) % C::STAGES;
        const bool next = j + 1 < nt;
        const int kslot = (2 * j + 2) % C::STAGES;
        const uint32_t fcol = (j & 1) ? C::HALF : 0;  // P_t(j), then S_t(j+1)'s second half
        if (!wait_load(2 * j + 1) || (next && !wait_load(2 * j + 2))) {
          ok = false;
          break;
        }
        if (!wait_all(&bars->mid[t], par)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (next) {
          issue_S_half(kslot, 0, C::HALF - fcol);
          tc_commit_both_w(&bars->sa_full[t]);
        }
        issue_PV_half(vslot, fcol, 0, j > 0);
        tc_commit_both_w(&bars->pva_done[t]);
        if (!wait_all(&bars->p_full[t], par)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_PV_half(vslot, fcol, 1, true);
        tc_commit_both_w(&bars->kv_empty[vslot]);
        if (next) {
          issue_S_half(kslot, 1, fcol);
          tc_commit_both_w(&bars->sb_full[t]);
          tc_commit_both_w(&bars->kv_empty[kslot]);
          used = 2 * j + 3;
        } else {
          tc_commit_both_w(&bars->o_full[t]);
          used = 2 * j + 2;
        }
      }
      // K/V items this tile never reaches (tile 0 stops one block short on
      // the diagonal) are released once they have landed, for both CTAs.
      for (int i = used; ok && i < 2 * n_kv; ++i) {
        if (!wait_load(i)) {
          ok = false;
          break;
        }
        tc_commit_both_w(&bars->kv_empty[i % C::STAGES]);
      }
      // Every UMMA issued above completes before the cluster barrier and the
      // TMEM free.
      tc_commit_own_w(&bars->drain[t]);
      mbar_wait_quiet(&bars->drain[t], 0);
    }
  } else {
    setmaxnreg_inc<C::REGS_HIGH>();
    // ------------------------------------------------------------ softmax + epilogue
    const int t = (warp - 4) >> 2;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    const uint32_t tR = tmem + lane_off + C::S_COL + t * C::BN;
    const uint32_t tO = tmem + lane_off + C::O_COL + t * D;
    const float sl2 = p.scale_log2;
    const uint32_t mid_bar = at_lead(&bars->mid[t]), pfull_bar = at_lead(&bars->p_full[t]);
    const int grow = it.q0 + 128 * t + row;
    const bool valid = grow < p.Tq;
    const int kv_last = p.causal ? (int)min((long long)it.sp + grow, (long long)p.Tk - 1) : p.Tk - 1;
    float m_run = -INFINITY;
    float l_run = 0.f;
    const int n_mine = t == 0 ? it.n_t[0] : n_kv;
    bool ok = true;
    for (int j = 0; j < n_mine; ++j) {
      const uint32_t par = (uint32_t)j & 1u;
      const uint32_t fcol = (j & 1) ? C::HALF : 0;  // first half of S_t(j); P_t(j) goes here
      const uint32_t scol = C::HALF - fcol;         // second half of S_t(j)
      if (!wait_all(&bars->sa_full[t], par)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int lim = kv_last - j * C::BN;
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
      // Second half of S_t(j); PV_t(j-1) is complete once it is.
      if (!wait_all(&bars->sb_full[t], par)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (j > 0 && __any_sync(0xffffffffu, a0 != 1.f)) rescale_O(a0);
      tmem_ld32(tR + scol, s[0]);
      tmem_ld32(tR + scol + 32, s[1]);
      tmem_wait_ld();
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mid_bar);
      const float a1 = softmax_half_tmem<kEmuPairs>(s, lim - C::HALF, sl2, m_run, tR + fcol + 32, hs1);
      if (__any_sync(0xffffffffu, a1 != 1.f)) {
        if (!wait_all(&bars->pva_done[t], par)) {
          ok = false;
          break;
        }
        tc_fence_after();
        rescale_O(a1);
      }
      l_run = (l_run * a0 + hs0) * a1 + hs1;
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(pfull_bar);
    }
    if (n_mine == 0) {
      if (valid) {
        uint32_t z[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) z[i] = 0u;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) store_out_chunk(p, it.b, it.h, grow, c, z, 0.f);
        if (p.lse) p.lse[((long long)it.b * p.Hq + it.h) * p.Tq + grow] = -INFINITY;
      }
    } else if (ok && wait_all(&bars->o_full[t], 0)) {
      tc_fence_after();
      const float inv_l = l_run > 0.f ? 1.f / l_run : 0.f;
#pragma unroll
      for (int c = 0; c < D / 32; c += 2) {
        uint32_t o[2][32];
        tmem_ld32(tO + 32 * c, o[0]);
        tmem_ld32(tO + 32 * c + 32, o[1]);
        tmem_wait_ld();
        if (valid) {
          store_out_chunk(p, it.b, it.h, grow, c, o[0], inv_l);
          store_out_chunk(p, it.b, it.h, grow, c + 1, o[1], inv_l);
        }
      }
      if (p.lse && valid)
        p.lse[((long long)it.b * p.Hq + it.h) * p.Tq + grow] =
            l_run > 0.f ? (m_run + __log2f(l_run)) * 0.69314718055994531f : -INFINITY;
    }
  }

  // Neither CTA frees TMEM or leaves while the other may still read its
  // shared memory (the leader's UMMAs read both CTAs' operands; the peer's
  // softmax warps arrive on the leader's barriers).
  tc_fence_before();
  cluster_sync_all();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ launcher
int launch_prefill_pair(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const PrefillParams& p,
                        cudaStream_t st) {
  using C = PairCfg;
  if (cudaFuncSetAttribute(fa_prefill_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES) !=
      cudaSuccess)
    return -1;
  cudaFuncAttributes fa{};
  if (cudaFuncGetAttributes(&fa, fa_prefill_pair_kernel) != cudaSuccess || fa.numRegs < C::MIN_LAUNCH_REGS)
    return -1;
  if (p.Hkv <= 0 || (p.Hq / p.Hkv) % 2) return -2;
  const long long items = (long long)p.n_qblk * p.B * (p.Hq / 2);
  if (items <= 0 || 2 * items > 0x7fffffffLL) return -2;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(2 * items));
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, fa_prefill_pair_kernel, tq, tk, tv, p) != cudaSuccess) return -1;
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace b2a
