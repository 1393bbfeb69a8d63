// Causal GQA prefill attention for sm_100a (tcgen05 + TMEM + TMA).
//
// Semantics follow the reference's FlashAttention-2 forward
// (npu/fa_ref.py:42-131, flash_attention_ref): for query row r with absolute
// position start_pos + r and key column c, the key is masked iff
// c > start_pos + r (causal); rows with no unmasked key produce 0
// (npu/fa_ref.py:112-128); the softmax scale is a runtime argument (the
// reference kernel hard-codes 1/sqrt(64), npu/fa_kernel.cc:37-38). Query head h
// reads key/value head h / (Hq / Hkv), the repeat_interleave mapping of
// smollm.py:205-207, without materialising the expanded K/V.
//
// A work item is two 128-row query tiles that ping-pong on the tensor core,
// so one tile's softmax overlaps the other tile's MMAs: a 256-row query block
// of one (batch, query head), or, for queries of 513-3072 rows with an even
// GQA group, the same 128 rows of two query heads that share a KV head (both
// tiles then walk the same key blocks). The grid has one CTA per work item, but a CTA does not
// stop after its own: it takes over CTAs that have not started yet (cluster
// launch control, clusterlaunchcontrol.try_cancel), in launch order, until
// none is left. Each resident CTA thus walks items heaviest first, with its
// TMEM, barriers and K/V ring set up once, the next item's K/V streaming in
// while the current one finishes, and the next item's Q loaded and first S
// MMAs issued while the current item's epilogue runs. Warp roles (12 warps):
//   warp 0      TMA producer: Q once, then K_j / V_j tiles through a ring
//   warp 1      TMEM owner + UMMA issuer for tile 0
//   warp 2      UMMA issuer for tile 1 (each tile's MMAs wait only on that
//               tile's softmax, so one tile's handoffs never stall the other's)
//   warp 3      scheduler: claims the next work item (try_cancel) as soon as
//               every role has started the current one
//   warps 4-7   softmax + epilogue for tile 0 (thread = row = TMEM lane)
//   warps 8-11  softmax + epilogue for tile 1
// TMEM (512 columns): a 128-column S/P region per tile (R_t = [128 t,
// 128 t + 128)) and O_0, O_1 (D columns each). S_t(j) is computed as two
// 64-key halves (N = 64 UMMAs) into the two 64-column halves of R_t, whose
// roles alternate with the parity of j: the first half lands in
// first(j) = 64 * (j & 1), the second in the other half. The softmax writes
// P_t(j) (bf16, two keys per 32-bit column, 64 columns) over first(j), which
// the PV UMMA reads as its A operand. As soon as the softmax has read the
// second half of S_t(j) into registers, the first half of S_t(j+1) can go
// into it; the second half of S_t(j+1) replaces P_t(j) once PV_t(j) is
// issued (UMMAs from one thread execute in order). So a tile's softmax can
// start on block j+1 right after publishing P_t(j), instead of waiting for
// PV_t(j) and a whole S_t(j+1) to run on the tensor core. PV_t(j) itself is
// issued in two K = 64 halves: the first as soon as P for keys 0-63 is
// written (mid-block), so only the second half and S_t(j+1)'s second half
// sit between the end of block j and the middle of block j+1. P never touches
// shared memory (whose bandwidth, shared by the tensor core's operand reads
// and the TMA fills, is the next bound).
#pragma once

#include "common.cuh"

namespace b2a {

struct PrefillParams {
  void* o;             // [B, Hq, Tq, D], innermost stride 1
  long long o_sb, o_sh, o_st;  // element strides
  float* lse;          // optional [B, Hq, Tq] natural-log LSE (nullptr = skip)
  const int* start_pos_arr;  // optional per-batch start position (device)
  int start_pos;
  int B, Hq, Hkv, Tq, Tk;
  float scale_log2;    // softmax scale * log2(e)
  int causal;
  int out_fp32;
  int n_qblk;          // query blocks per head: ceil(Tq / rows per work item)
  // Two-tile work items (NQT = 2) pair query heads instead of row blocks:
  // tile t is query head 2 i + t of a KV head's group over the same 128 rows,
  // so both tiles walk the same key blocks and share every K/V tile. Needs an
  // even group size (Hq / Hkv); n_qblk then counts 128-row blocks.
  int head_pairs;
  int* err;            // device error word (may be nullptr)
  // Optional output gate [B, Hq, Tq, D] (element strides g_sb, g_sh, g_st,
  // innermost 1; fp32 or bf16): o = attention * sigmoid(gate), the gated
  // attention epilogue of qwen/forward.py:223-226. nullptr = no gate.
  const void* gate;
  long long g_sb, g_sh, g_st;
  int gate_bf16;
  // 1: O's base and strides are 32-byte aligned, so the epilogue's
  // row-per-thread stores may be 32-byte vector stores.
  int o_v8;
};

// NQT query tiles of 128 rows per CTA. NQT = 2: the two tiles' softmax and
// MMAs interleave inside one CTA (one CTA per SM). NQT = 1: half the shared
// memory and TMEM, so two CTAs share an SM and one's start-up and epilogue
// overlap the other's steady state — the better choice when each CTA sees
// few key blocks (short sequences).
template <int D, int NQT_ = 2>
struct PrefillCfg {
  static constexpr int BM = 128;  // rows per Q tile == TMEM lanes
  static constexpr int BN = 128;  // keys per K/V tile
  static constexpr int NQT = NQT_;  // Q tiles per CTA
  static constexpr int KCH = D / 64;  // 128-byte swizzle chunks per row
  static constexpr int CHUNK_BYTES = 128 * 128;  // 128 rows x 128 B
  static constexpr int Q_TILE_BYTES = BM * D * 2;
  static constexpr int KV_TILE_BYTES = BN * D * 2;
  static constexpr int STAGES = NQT == 2 ? ((D == 64) ? 8 : 5) : ((D == 64) ? 4 : 2);
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_KV = OFF_Q + NQT * Q_TILE_BYTES;
  static constexpr int OFF_BAR = OFF_KV + STAGES * KV_TILE_BYTES;
  static constexpr int BAR_BYTES = 512;
  static constexpr int SMEM_BYTES = OFF_BAR + BAR_BYTES + 1024;  // + alignment slack
  static constexpr int CTAS_PER_SM = NQT == 2 ? 1 : 2;
  static constexpr int TMEM_COLS = NQT == 2 ? 512 : 256;
  static constexpr int S_COL = 0;          // S/P region R_t at S_COL + t * BN
  static constexpr int HALF = BN / 2;      // keys per S half (one N = 64 UMMA group)
  static constexpr int O_COL = NQT * BN;   // O_t at O_COL + t * D
  static constexpr int THREADS = 128 + 128 * NQT;
  // setmaxnreg split: warpgroup 0 (TMA + MMA issue) gives registers to the
  // softmax warpgroups. The sum 128 * REGS_LOW + 128 * NQT * REGS_HIGH stays
  // within THREADS * MIN_LAUNCH_REGS, so any launch with >= MIN_LAUNCH_REGS
  // registers per thread covers it (the launcher refuses to launch otherwise;
  // 168 for NQT = 2, 128 for NQT = 1 at two CTAs per SM).
  static constexpr int REGS_LOW = NQT == 2 ? 112 : 88;
  static constexpr int REGS_HIGH = NQT == 2 ? 184 : 168;
  static constexpr int MIN_LAUNCH_REGS = (128 * REGS_LOW + 128 * NQT * REGS_HIGH + THREADS - 1) / THREADS;
  static_assert(D == 64 || D == 128, "two-tile prefill supports head_dim 64 and 128");
  static_assert(NQT == 1 || NQT == 2, "one or two query tiles per CTA");
  static_assert(O_COL + NQT * D <= TMEM_COLS, "TMEM budget");
  static_assert(SMEM_BYTES * CTAS_PER_SM <= 232448 - 1024 * (CTAS_PER_SM - 1), "shared memory budget");
  static_assert(MIN_LAUNCH_REGS * THREADS * CTAS_PER_SM <= 65536, "register budget");
};

// Barrier slots inside the OFF_BAR region.
struct PrefillBars {
  uint64_t q_full;
  uint64_t q_free;       // the Q buffer may be refilled for the next work
                         // item: every S MMA of the current one has completed
  uint64_t kv_full[8];
  uint64_t kv_empty[8];
  uint64_t sa_full[2];   // first 64-key half of S_t(j) is in TMEM
  uint64_t sb_full[2];   // second half of S_t(j) is in TMEM
  uint64_t mid[2];       // P_t(j) for keys 0-63 is in TMEM and the second
                         // S half has been read into registers
  uint64_t pva_done[2];  // the PV MMAs of that first half have completed
  uint64_t p_full[2];
  uint64_t o_full[2];
  uint64_t drain[2];     // per UMMA issuer warp
  uint64_t stagger;      // head-pair items: tile 0's softmax warps have
                         // published the item's first mid
  // Work items beyond the CTA's own are taken from CTAs of the grid that have
  // not started yet (cluster launch control); the scheduler warp publishes
  // each one in a two-slot ring read by every other warp.
  uint64_t item_full[2];
  uint64_t item_empty[2];
  uint64_t clc_bar;
  alignas(16) uint8_t clc_resp[16];
  int item_id[2];
  uint32_t tmem_base;
  int abort_flag;
};

// Head dim 256 variant (one query tile per CTA, prefill_d256.cu).
int launch_prefill_d256(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                        const PrefillParams& p, cudaStream_t st);

// How the D <= 128 kernel cuts this problem into work items: rows per item
// and per query head (256 or 128: PrefillParams::n_qblk must be computed
// with it) and whether two-tile items pair query heads (head_pairs, rows per
// item then 128 with two tiles).
struct PrefillPlan {
  int rows_per_item;
  int tiles;       // query tiles per CTA (NQT)
  int head_pairs;
  int sm_pairs;    // 1: fa_prefill_pair_kernel (prefill_pair.cu), D = 128
};
PrefillPlan prefill_plan(int D, int Hq, int Hkv, int Tq, int Tk);

// Head dim 128 on SM pairs (prefill_pair.cu): cluster launch, 256 rows of two
// query heads per item; K's tensor map has 32-row boxes, Q's and V's 128.
int launch_prefill_pair(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                        const PrefillParams& p, cudaStream_t st);

// Launch the prefill kernel on `st` for the given plan.
// Returns 0 on success, -3 for an unsupported head_dim, another negative
// value on launch failure.
int launch_prefill(int D, const PrefillPlan& plan, const CUtensorMap& tq, const CUtensorMap& tk,
                   const CUtensorMap& tv, const PrefillParams& p, cudaStream_t st);

}  // namespace b2a
