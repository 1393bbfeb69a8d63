// Parameters and launcher of the split-KV decode kernels (decode.cu).
#pragma once

#include "common.cuh"

namespace b2a {

struct DecodeParams {
  const __nv_bfloat16* q;  // [B, Hq, D]
  long long q_sb, q_sh;
  const int* seqlens;      // [B], device
  float* part_o;           // [B, Hkv, max_splits, group, D]
  float* part_lse;         // [B, Hkv, max_splits, group]
  void* o;                 // [B, Hq, D]
  long long o_sb, o_sh;
  int B, Hq, Hkv, Lmax, group, split_len, max_splits;
  float scale_log2;
  int out_fp32;
  int* err;
  // Optional output gate [B, Hq, D] (element strides g_sb, g_sh; fp32 or
  // bf16): o = attention * sigmoid(gate) (qwen/forward.py:223-226).
  const void* gate;
  long long g_sb, g_sh;
  int gate_bf16;
  // Optional fused output projection with residual add (b2a_decode_proj):
  // x[b, :] += o_b @ wo^T, where o_b is sequence b's (gated) attention output
  // flattened over heads, [Hq * D], and wo is [dim, Hq * D] with row stride
  // wo_ld elements (the F.linear weight of the output projection). x is
  // [B, dim] with row stride x_sb. The combine then runs per (block of
  // outputs, sequence) and each output has one writer; `o` is not written
  // when it is nullptr.
  const void* wo;
  long long wo_ld;
  int dim, wo_fp32;
  void* x;
  long long x_sb;
  int x_fp32;
};

// Launch the split kernel and the LSE combine on `st`. Returns 0 on success,
// -3 for an unsupported head_dim, -4 for a fused projection whose attention
// row does not fit in shared memory, another negative value on launch failure.
int launch_decode(int D, const CUtensorMap& tk, const CUtensorMap& tv, const DecodeParams& p, cudaStream_t st);

}  // namespace b2a
