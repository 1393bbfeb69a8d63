// Kernel body of the tcgen05 causal GQA prefill; see prefill.cuh for the
// design. The host-side launcher (tensor maps, argument checks) is at the end
// of this file and is called from capi.cu.
#include <cstdlib>

#include "prefill.cuh"
#include "softmax.cuh"

namespace b2a {

#ifndef B2A_ONE_TILE_MAX_ROWS
#define B2A_ONE_TILE_MAX_ROWS 1024
#endif
// Longest query length served by one-tile CTAs (prefill_plan).
constexpr int kOneTileMaxRows = B2A_ONE_TILE_MAX_ROWS;
#ifndef B2A_HEAD_PAIRS
#define B2A_HEAD_PAIRS 1
#endif
// Two-tile items pair query heads when the GQA group size is even and the
// query is at most this long; longer queries use row-pair items.
constexpr bool kHeadPairs = B2A_HEAD_PAIRS != 0;
constexpr int kHeadPairMaxRows = 3072;
// With an even GQA group, queries longer than this use head-pair items
// instead of one-tile CTAs.
constexpr int kHeadPairMinRows = 513;


// Work item -> (query block, batch, heads) and the key blocks its query tiles
// need. The heaviest causal query blocks come first in launch order; the
// query heads that share a KV head are adjacent, so they run together and
// re-read K/V from L2. Row mode: tile t covers rows [q0 + 128 t, +128) of
// query head h. Head-pair mode (NQT = 2, head_pairs): tile t covers rows
// [q0, q0 + 128) of query head h + t.
template <int NQT, bool PAIRS>
struct PrefillItem {
  static_assert(!PAIRS || NQT == 2, "head-pair items have two tiles");
  int h, b, hk, q0, sp;
  int n_t[NQT];  // key blocks query tile t needs; tile 0 never more than
                 // tile 1 and, under the causal mask, at most one fewer
  int n_kv;      // n_t[NQT - 1]: the key blocks that get loaded
  __device__ __forceinline__ int head(int t) const { return h + (PAIRS ? t : 0); }
  __device__ __forceinline__ int row0(int t) const { return q0 + (PAIRS ? 0 : 128 * t); }
};

template <int NQT, bool PAIRS>
__device__ __forceinline__ PrefillItem<NQT, PAIRS> prefill_item(const PrefillParams& p, int lin) {
  constexpr int BM = 128, BN = 128;
  PrefillItem<NQT, PAIRS> it;
  int qblk;
  if (PAIRS) {
    // Heaviest row blocks first; the head pairs of one KV head adjacent.
    const int np = p.Hq / p.Hkv / 2;  // head pairs per KV head
    const int per = p.B * p.Hkv * np;
    qblk = p.n_qblk - 1 - lin / per;
    const int rem = lin % per;
    const int pair = rem % np;
    const int bk = rem / np;
    it.hk = bk % p.Hkv;
    it.b = bk / p.Hkv;
    it.h = it.hk * (2 * np) + 2 * pair;
    it.q0 = qblk * BM;
  } else {
    const int hb = p.Hq * p.B;
    qblk = p.n_qblk - 1 - lin / hb;
    const int rem = lin % hb;
    it.h = rem % p.Hq;
    it.b = rem / p.Hq;
    it.hk = it.h / (p.Hq / p.Hkv);
    it.q0 = qblk * (BM * NQT);
  }
  it.sp = p.start_pos_arr ? p.start_pos_arr[it.b] : p.start_pos;
#pragma unroll
  for (int t = 0; t < NQT; ++t) {
    if (p.causal) {
      const int last_row = min(it.row0(t) + BM - 1, p.Tq - 1);
      const long long kv_end = min((long long)p.Tk, (long long)it.sp + last_row + 1);
      it.n_t[t] = kv_end <= 0 ? 0 : (int)((kv_end + BN - 1) / BN);
    } else {
      it.n_t[t] = (p.Tk + BN - 1) / BN;
    }
  }
  it.n_kv = it.n_t[NQT - 1];
  return it;
}

// PAIRS: head-pair work items (NQT = 2 only), else row blocks.
template <int D, int NQT, bool PAIRS>
__global__ void __launch_bounds__(PrefillCfg<D, NQT>::THREADS, PrefillCfg<D, NQT>::CTAS_PER_SM)
    fa_prefill_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ PrefillParams p) {
  using C = PrefillCfg<D, NQT>;
  constexpr int kEmuPairs = exp2_emu_pairs<D>();
  // Warps that take every work item from the scheduler: the producer, the
  // UMMA issuers and the softmax warps.
  constexpr int kConsumerWarps = 1 + NQT + 4 * NQT;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  uint8_t* sQ = smem + C::OFF_Q;
  uint8_t* sKV = smem + C::OFF_KV;
  PrefillBars* bars = reinterpret_cast<PrefillBars*>(smem + C::OFF_BAR);
  volatile int* abort_flag = &bars->abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  auto wait_all = [&](uint64_t* bar, uint32_t parity) -> bool {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, p.err));
  };
  // The CTA's work item number n (n >= 1; item 0 is its own blockIdx.x),
  // published by the scheduler warp in slot (n - 1) & 1: the blockIdx.x of a
  // CTA it took over, or -1 when there is none (or on abort). Every consumer
  // warp calls this once per item it finishes, in order.
  auto next_item = [&](int n) -> int {
    const int slot = (n - 1) & 1;
    if (!wait_all(&bars->item_full[slot], (uint32_t)((n - 1) >> 1) & 1u)) return -1;
    const int id = *reinterpret_cast<volatile int*>(&bars->item_id[slot]);
    __syncwarp();
    if (lane == 0) mbar_arrive(&bars->item_empty[slot]);
    return id;
  };

  const PrefillItem<NQT, PAIRS> first = prefill_item<NQT, PAIRS>(p, blockIdx.x);
  const int first_loads = min(C::STAGES, 2 * first.n_kv);
  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    // Every UMMA issuer commits once its last S MMA of an item is issued.
    mbar_init(&bars->q_free, C::NQT);
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
    mbar_init(&bars->stagger, 4);
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->item_full[s], 1);
      mbar_init(&bars->item_empty[s], kConsumerWarps);
    }
    mbar_init(&bars->clc_bar, 1);
    bars->abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    // The first item's Q tiles and first ring of K/V tiles are requested
    // here, so their latency overlaps the TMEM allocation and the block
    // barrier below (the producer warp issues the rest). The ring is free.
    if (first.n_kv > 0) {
      mbar_arrive_expect_tx(&bars->q_full, C::NQT * C::Q_TILE_BYTES);
#pragma unroll
      for (int t = 0; t < C::NQT; ++t)
#pragma unroll
        for (int c = 0; c < C::KCH; ++c)
          tma_load_4d(sQ + t * C::Q_TILE_BYTES + c * C::CHUNK_BYTES, &tm_q, &bars->q_full, c * 64,
                      first.row0(t), first.head(t), first.b);
      for (int i = 0; i < first_loads; ++i) {
        uint8_t* dst = sKV + i * C::KV_TILE_BYTES;
        mbar_arrive_expect_tx(&bars->kv_full[i], C::KV_TILE_BYTES);
#pragma unroll
        for (int c = 0; c < C::KCH; ++c)
          tma_load_4d(dst + c * C::CHUNK_BYTES, (i & 1) ? &tm_v : &tm_k, &bars->kv_full[i], c * 64,
                      (i >> 1) * C::BN, first.hk, first.b);
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
  // The producer, the MMA issuers and the scheduler run as whole warps:
  // every lane walks the loop and waits, one elected lane issues each copy /
  // MMA / commit (the *_w helpers), which keeps the operands in uniform
  // registers.
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // K/V loads run through the ring across work items: load g (counted
    // from the CTA's first item) uses slot g % STAGES in round g / STAGES.
    int lin = blockIdx.x;
    int ld = 0;        // loads of earlier items
    int issued = 0;    // loads issued in total
    int q_rounds = 0;  // items with keys (one Q load each)
    bool ok = true;
    for (int n = 1;; ++n) {
      const PrefillItem<NQT, PAIRS> it = prefill_item<NQT, PAIRS>(p, lin);
      if (it.n_kv > 0) {
        int i0 = 0;
        if (n == 1) {
          i0 = first_loads;  // requested during set-up
          issued = first_loads;
        } else {
          // The Q buffer is free once every S MMA of the previous item with
          // keys has completed.
          if (!wait_all(&bars->q_free, (uint32_t)(q_rounds - 1) & 1u)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx_w(&bars->q_full, C::NQT * C::Q_TILE_BYTES);
#pragma unroll
          for (int t = 0; t < C::NQT; ++t)
#pragma unroll
            for (int c = 0; c < C::KCH; ++c)
              tma_load_4d_w(sQ + t * C::Q_TILE_BYTES + c * C::CHUNK_BYTES, &tm_q, &bars->q_full, c * 64,
                            it.row0(t), it.head(t), it.b);
        }
        ++q_rounds;
        for (int i = i0; i < 2 * it.n_kv; ++i) {
          const int g = ld + i;
          const int slot = g % C::STAGES;
          const uint32_t ph = (uint32_t)(g / C::STAGES) & 1u;
          if (!wait_all(&bars->kv_empty[slot], ph ^ 1u)) {
            ok = false;
            break;
          }
          const CUtensorMap* m = (i & 1) ? &tm_v : &tm_k;
          uint8_t* dst = sKV + slot * C::KV_TILE_BYTES;
          mbar_arrive_expect_tx_w(&bars->kv_full[slot], C::KV_TILE_BYTES);
#pragma unroll
          for (int c = 0; c < C::KCH; ++c)
            tma_load_4d_w(dst + c * C::CHUNK_BYTES, m, &bars->kv_full[slot], c * 64, (i >> 1) * C::BN, it.hk,
                          it.b);
          issued = g + 1;
        }
        if (!ok) break;
        ld += 2 * it.n_kv;
      }
      lin = next_item(n);
      if (lin < 0) break;
    }
    if (*abort_flag && lane == 0) {
      // Let every copy still in flight land before the CTA releases smem.
      if (q_rounds > 0) mbar_wait_quiet(&bars->q_full, (uint32_t)(q_rounds - 1) & 1u);
      for (int g = max(0, issued - C::STAGES); g < issued; ++g)
        mbar_wait_quiet(&bars->kv_full[g % C::STAGES], (uint32_t)(g / C::STAGES) & 1u);
    }
  } else if (warp >= 1 && warp <= C::NQT) {
    // ------------------------------------------------------------ UMMA issuers
    // Warp 1 issues tile 0's MMAs, warp 2 (NQT = 2) tile 1's. Each reads
    // every K/V tile it needs and releases it (kv_empty counts NQT arrivals).
    const int t = warp - 1;
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

    int lin = blockIdx.x;
    int G = 0;         // ring position of the current item's first load
    int J = 0;         // key blocks of this tile in earlier items (barrier rounds)
    int q_rounds = 0;  // items with keys so far
    int stg = 0;       // head-pair items with keys so far (stagger rounds)
    bool ok = true;
    for (int n = 1;; ++n) {
      const PrefillItem<NQT, PAIRS> it = prefill_item<NQT, PAIRS>(p, lin);
      const int nt = t == 0 ? it.n_t[0] : it.n_kv;
      if (it.n_kv > 0) {
        auto slot_of = [&](int i) { return (G + i) % C::STAGES; };
        auto wait_load = [&](int i) -> bool {
          return wait_all(&bars->kv_full[slot_of(i)], (uint32_t)((G + i) / C::STAGES) & 1u);
        };
        // Per key block j: once the softmax has taken the second half of
        // S_t(j), the first half of S_t(j+1) goes into its columns; once
        // P_t(j) is published, PV_t(j) and then the second half of S_t(j+1)
        // (over P_t(j)'s columns). V_j and K_{j+1} are waited for first
        // (normally long landed). K/V load items are K_j = 2 j,
        // V_j = 2 j + 1; `used` counts the items this warp has released so
        // far, in order. The previous item's last PV MMAs were issued by this
        // thread before this item's S MMAs overwrite their P columns (UMMAs
        // from one thread execute in order), and its O was read out by the
        // softmax warps before they publish this item's first `mid`, which
        // the first PV (the one that overwrites O) waits for.
        ok = wait_all(&bars->q_full, (uint32_t)q_rounds & 1u);
        ++q_rounds;
        // Head-pair items: tile 1 starts one block behind tile 0 (its first S
        // MMAs wait for tile 0's first mid), so the two tiles' epilogues,
        // whose row stores would otherwise hit the memory pipe at the same
        // moment, fall into the other tile's key loop (row-pair items are
        // offset by the diagonal block already). Measured +5 % at T = 1024,
        // +2.5 % at T = 2048. Tile 0 cannot publish the next item's first mid
        // before this wait has passed: that needs the next Q, which needs
        // q_free, which needs this warp's S MMAs of this item.
        if (PAIRS && t == 1 && it.n_t[0] > 0) {
          ok = ok && wait_all(&bars->stagger, (uint32_t)stg & 1u);
          ++stg;
        }
        int used = 0;
        if (ok && nt > 0) {
          ok = wait_load(0);
          if (ok) {
            tc_fence_after();
            issue_S_half(slot_of(0), 0, 0);
            tc_commit_w(&bars->sa_full[t]);
            issue_S_half(slot_of(0), 1, C::HALF);
            tc_commit_w(&bars->sb_full[t]);
            tc_commit_w(&bars->kv_empty[slot_of(0)]);
            used = 1;
            if (nt == 1) tc_commit_w(&bars->q_free);  // this item's last S MMA is issued
          }
        }
        for (int j = 0; ok && j < nt; ++j) {
          const uint32_t par = (uint32_t)(J + j) & 1u;
          const int vslot = slot_of(2 * j + 1);
          const bool next = j + 1 < nt;
          const int kslot = slot_of(2 * j + 2);
          const uint32_t fcol = (j & 1) ? C::HALF : 0;  // P_t(j), then S_t(j+1)'s second half
          if (!wait_load(2 * j + 1) || (next && !wait_load(2 * j + 2))) {
            ok = false;
            break;
          }
          // Mid-block handoff: the next block's first S half (needed first by
          // the softmax), then the first PV half.
          if (!wait_all(&bars->mid[t], par)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (next) {
            issue_S_half(kslot, 0, C::HALF - fcol);
            tc_commit_w(&bars->sa_full[t]);
          }
          issue_PV_half(vslot, fcol, 0, j > 0);
          tc_commit_w(&bars->pva_done[t]);
          if (!wait_all(&bars->p_full[t], par)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_PV_half(vslot, fcol, 1, true);
          tc_commit_w(&bars->kv_empty[vslot]);
          if (next) {
            issue_S_half(kslot, 1, fcol);
            tc_commit_w(&bars->sb_full[t]);
            tc_commit_w(&bars->kv_empty[kslot]);
            used = 2 * j + 3;
            if (j + 2 == nt) tc_commit_w(&bars->q_free);  // this item's last S MMA is issued
          } else {
            tc_commit_w(&bars->o_full[t]);
            used = 2 * j + 2;
          }
        }
        if (ok && nt == 0) tc_commit_w(&bars->q_free);  // this tile reads no Q in this item
        // K/V tiles of blocks this tile never reaches (tile 0 stops one block
        // short at the diagonal) are released once they have landed: landing
        // means the slot is in the round of exactly that load.
        for (int i = used; ok && i < 2 * it.n_kv; ++i) {
          if (!wait_load(i)) {
            ok = false;
            break;
          }
          if (lane == 0) mbar_arrive(&bars->kv_empty[slot_of(i)]);
        }
        G += 2 * it.n_kv;
        J += nt;
      }
      if (!ok) break;
      lin = next_item(n);
      if (lin < 0) break;
    }
    // Every MMA issued above must finish before TMEM is deallocated.
    tc_commit_w(&bars->drain[t]);
    mbar_wait_quiet(&bars->drain[t], 0);
  } else if (warp == 3) {
    // ------------------------------------------------------------ scheduler
    // Item n (n >= 1) is claimed once every consumer warp has taken item
    // n - 1, i.e. has started working on it: one item of look-ahead, so the
    // next Q and K/V can stream in early while the claim stays late enough
    // for the last items to spread over the CTAs that finish first.
    for (int n = 1;; ++n) {
      if (n >= 2 && !wait_all(&bars->item_empty[(n - 2) & 1], (uint32_t)((n - 2) >> 1) & 1u)) break;
      const uint32_t cpar = (uint32_t)(n - 1) & 1u;
      if (lane == 0) {
        fence_proxy_async_smem();  // the previous response was read through the generic proxy
        mbar_arrive_expect_tx(&bars->clc_bar, 16);
        clc_try_cancel(bars->clc_resp, &bars->clc_bar);
      }
      __syncwarp();
      if (!wait_all(&bars->clc_bar, cpar)) {
        // Abort: the response must still land before shared memory goes away.
        if (lane == 0) mbar_wait_quiet(&bars->clc_bar, cpar);
        break;
      }
      const int id = clc_cancelled_ctaid_x(bars->clc_resp);
      __syncwarp();
      if (lane == 0) {
        bars->item_id[(n - 1) & 1] = id;
        mbar_arrive(&bars->item_full[(n - 1) & 1]);
      }
      __syncwarp();
      if (id < 0) break;
    }
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
    const float sl2 = p.scale_log2;
    int lin = blockIdx.x;
    int J = 0;         // key blocks of this tile in earlier items (barrier rounds)
    int o_rounds = 0;  // earlier items in which this tile had key blocks
    bool ok = true;
    for (int n = 1;; ++n) {
      const PrefillItem<NQT, PAIRS> it = prefill_item<NQT, PAIRS>(p, lin);
      const int b = it.b, h = it.head(t);
      const int grow = it.row0(t) + row;
      const bool valid = grow < p.Tq;
      // Last visible key of this row (fits in int: it is below Tk).
      const int kv_last = p.causal ? (int)min((long long)it.sp + grow, (long long)p.Tk - 1) : p.Tk - 1;
      float m_run = -INFINITY;
      float l_run = 0.f;
      const int n_mine = t == 0 ? it.n_t[0] : it.n_kv;

      for (int j = 0; j < n_mine; ++j) {
        const uint32_t par = (uint32_t)(J + j) & 1u;
        const uint32_t fcol = (j & 1) ? C::HALF : 0;  // first half of S_t(j); P_t(j) goes here
        const uint32_t scol = C::HALF - fcol;         // second half of S_t(j)
        if (!__all_sync(0xffffffffu, mbar_wait(&bars->sa_full[t], par, abort_flag, p.err))) {
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
        if (!__all_sync(0xffffffffu, mbar_wait(&bars->sb_full[t], par, abort_flag, p.err))) {
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
        if (PAIRS && t == 0 && j == 0 && lane == 0) mbar_arrive(&bars->stagger);
        const float a1 = softmax_half_tmem<kEmuPairs>(s, lim - C::HALF, sl2, m_run, tR + fcol + 32, hs1);
        if (__any_sync(0xffffffffu, a1 != 1.f)) {
          // Rare: the second half moved the running max. O then holds blocks
          // < j and the first half of block j (once its PV half completes);
          // bring it to the new max before the second PV half adds to it.
          if (!__all_sync(0xffffffffu, mbar_wait(&bars->pva_done[t], par, abort_flag, p.err))) {
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
        const bool w = ok && mbar_wait(&bars->o_full[t], (uint32_t)o_rounds & 1u, abort_flag, p.err);
        if (__all_sync(0xffffffffu, w)) {
          tc_fence_after();
          const float inv_l = l_run > 0.f ? 1.f / l_run : 0.f;
          // Two 32-column TMEM loads per wait: the second load's latency
          // hides behind the first.
#pragma unroll
          for (int c = 0; c < D / 32; c += 2) {
            uint32_t o[2][32];
            tmem_ld32(tO + 32 * c, o[0]);
            tmem_ld32(tO + 32 * c + 32, o[1]);
            tmem_wait_ld();
            if (valid) {
              store_out_chunk(p, b, h, grow, c, o[0], inv_l);
              store_out_chunk(p, b, h, grow, c + 1, o[1], inv_l);
            }
          }
          if (p.lse && valid) {
            p.lse[((long long)b * p.Hq + h) * p.Tq + grow] =
                l_run > 0.f ? (m_run + __log2f(l_run)) * 0.69314718055994531f : -INFINITY;
          }
        }
      }
      J += n_mine;
      if (n_mine > 0) ++o_rounds;
      if (!ok) break;
      lin = next_item(n);
      if (lin < 0) break;
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
template <int D, int NQT, bool PAIRS>
static int launch_prefill_t(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                            const PrefillParams& p, cudaStream_t st) {
  using C = PrefillCfg<D, NQT>;
  cudaError_t e = cudaFuncSetAttribute(fa_prefill_kernel<D, NQT, PAIRS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       C::SMEM_BYTES);
  if (e != cudaSuccess) return -1;
  // The in-kernel register split needs at least MIN_LAUNCH_REGS per thread.
  cudaFuncAttributes fa{};
  if (cudaFuncGetAttributes(&fa, fa_prefill_kernel<D, NQT, PAIRS>) != cudaSuccess || fa.numRegs < C::MIN_LAUNCH_REGS)
    return -1;
  // One CTA per work item (query blocks x query heads, or x head pairs).
  const long long nblk = (long long)p.n_qblk * p.B * (p.head_pairs ? p.Hq / 2 : p.Hq);
  if (nblk <= 0 || nblk > 0x7fffffffLL) return -2;
  fa_prefill_kernel<D, NQT, PAIRS><<<(unsigned)nblk, C::THREADS, C::SMEM_BYTES, st>>>(tq, tk, tv, p);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// One-tile CTAs (two per SM) pay off when a CTA sees few key blocks, so that
// its start-up and epilogue are a large share of its time. Beyond that, up to
// kHeadPairMaxRows, two-tile items pair query heads when the GQA group size is
// even: both tiles then walk the same key blocks (row-pair items leave tile 0
// one block short on the diagonal, ~10 % at T = 2048), and one K/V stream
// feeds two tiles through the 5-slot ring, where a one-tile CTA's 2-slot ring
// leaves each block's loads exposed. Measured on B200 (config 3 heads,
// TFLOP/s, interleaved A/B, medians): one-tile CTAs against head pairs
// T=256 347 / 323, T=512 547 / 551, T=768 657 / 697, T=1024 696 / 744;
// head pairs against row pairs T=2048 918 / 787, T=3072 896 / 876; at T=4096
// and 8192 head pairs ran 1-3 % slower (more KV heads in flight at once:
// their K/V no longer fit in L2). Odd groups keep one-tile CTAs up to
// kOneTileMaxRows (measured against row pairs: T=1024 +2-3 %, T=2048 -10 %).
// Queries of at least this many rows (head dim 128, even GQA group) run on SM
// pairs (prefill_pair.cu) when the environment variable B2A_PREFILL_SM_PAIRS
// holds a positive row count; unset or 0 (the default): never. The SM-pair
// kernel gives the same results bit for bit but measured slower (config 3:
// 825 against 1065 TFLOP/s at T=8192), so it is opt-in.
static int sm_pairs_min_rows() {
  const char* s = std::getenv("B2A_PREFILL_SM_PAIRS");
  if (!s || !*s) return 0;
  const long v = std::strtol(s, nullptr, 10);
  return v > 0 && v < (1L << 30) ? (int)v : 0;
}

PrefillPlan prefill_plan(int D, int Hq, int Hkv, int Tq, int Tk) {
  (void)Tk;
  const bool even_group = Hkv > 0 && Hq % Hkv == 0 && (Hq / Hkv) % 2 == 0;
  const int pair_min = D == 128 && even_group ? sm_pairs_min_rows() : 0;
  if (pair_min > 0 && Tq >= pair_min) return PrefillPlan{256, 2, 0, 1};
  if (kHeadPairs && even_group && Tq >= kHeadPairMinRows && Tq <= kHeadPairMaxRows)
    return PrefillPlan{128, 2, 1, 0};
  if (Tq <= kOneTileMaxRows) return PrefillPlan{128, 1, 0, 0};
  return PrefillPlan{256, 2, 0, 0};
}

int launch_prefill(int D, const PrefillPlan& plan, const CUtensorMap& tq, const CUtensorMap& tk,
                   const CUtensorMap& tv, const PrefillParams& p, cudaStream_t st) {
  const bool one = plan.tiles == 1;
  const bool pairs = !one && plan.head_pairs;
  switch (D) {
    case 64:
      return one ? launch_prefill_t<64, 1, false>(tq, tk, tv, p, st)
                 : (pairs ? launch_prefill_t<64, 2, true>(tq, tk, tv, p, st)
                          : launch_prefill_t<64, 2, false>(tq, tk, tv, p, st));
    case 128:
      return one ? launch_prefill_t<128, 1, false>(tq, tk, tv, p, st)
                 : (pairs ? launch_prefill_t<128, 2, true>(tq, tk, tv, p, st)
                          : launch_prefill_t<128, 2, false>(tq, tk, tv, p, st));
    default: return -3;
  }
}

}  // namespace b2a
