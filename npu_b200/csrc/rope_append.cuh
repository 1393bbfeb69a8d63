// Attention prologue: per-head RMSNorm (optional), rotary embedding on the
// first rope_dim lanes of each head, and an in-place KV-cache append. Takes
// the q/k/v projections in their natural [B, T, H, D] layout (views into one
// fused QKV output or separate ones; q may be every other D-block of a
// [q | gate] projection) and writes
//   q  -> [B, Hq, T, D] bf16, the prefill/decode kernels' query layout;
//   k, v -> rows start_pos[b] .. start_pos[b] + T - 1 of a preallocated
//           device-resident cache [B, Hkv, Lmax, D] bf16, in place.
// SmolLM (smollm.py:186-208): no norm, rope_dim = D. Qwen gated attention
// (qwen/forward.py:178-204): per-head Q/K RMSNorm, rope_dim = 64 of 256.
// One launch replaces the reference's transposes, norms, rotations,
// torch.cat of the cache and repeat_interleave; GQA heads are never expanded.
#pragma once

#include "common.cuh"

namespace b2a {

struct RopeAppendParams {
  const void* q;
  const void* k;
  const void* v;
  long long qs[3], ks[3], vs[3];  // element strides of (b, t, h); d is contiguous
  const void* cos;                // [max_pos, rope_dim], same dtype as q/k/v, contiguous
  const void* sin;
  int max_pos;
  int rope_dim;                   // rotated lanes per head: 0 or a power of two in [16, D]
  const void* q_norm;             // optional per-head RMSNorm weights [D] (same dtype as q)
  const void* k_norm;
  float norm_eps;
  void* q_out;                    // [B, Hq, T, D] bf16, contiguous
  void* k_cache;                  // [B, Hkv, Lmax, D] bf16 with element strides kcs (b, h, l)
  void* v_cache;
  long long kcs[3], vcs[3];
  int B, T, Hq, Hkv, D, Lmax;
  int start_pos;                  // used when start_pos_arr is null
  const int* start_pos_arr;       // optional per-batch first position (device)
  int* seqlens_out;               // optional: seqlens_out[b] = start_pos[b] + T (device)
  int src_bf16;                   // 1: q/k/v/cos/sin/norms are bf16, 0: fp32
  int* err;                       // device error word
};

// Returns 0, -3 for an unsupported head_dim, another negative value on launch
// failure.
int launch_rope_append(const RopeAppendParams& p, cudaStream_t st);

}  // namespace b2a
