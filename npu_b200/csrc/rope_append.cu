// Attention prologue: RMSNorm + rotary + KV-cache append (see
// rope_append.cuh). Memory-bound: every source element is read once and
// every output element written once.
//
// Thread layout: a "row" is one (b, t, head) vector of D elements among the
// Hq query, Hkv key and Hkv value heads; D / 8 threads share a row (8, 16 or
// 32 lanes of one warp), thread i owning elements [8 i, 8 i + 8). The row's
// sum of squares is a shuffle reduction over those lanes; the rotate-half
// partner of element e < rope_dim / 2 is e + rope_dim / 2, held by thread
// i ^ (rope_dim / 16), so pairs are exchanged with one shuffle.
//
// Arithmetic follows the reference op by op in the source dtype:
//   rms_norm (smollm.py:37-42, qwen/forward.py:58-61): fp32 statistics,
//     (x * rsqrt(mean(x^2) + eps)) * w, rounded to the source dtype;
//   rotary (smollm.py:53-58, qwen/forward.py:81-95): x * cos +
//     rotate_half(x) * sin with each product and the sum a separately
//     rounded operation (no fused multiply-add), products and sum rounded to
//     bf16 for bf16 sources as eager PyTorch does.
// Results are rounded to bf16 for the attention kernels. Without a norm the
// rotation is bit-exact against the reference; the norm's reduction order
// differs from torch's, so normed rows agree to rounding.
#include "rope_append.cuh"

namespace b2a {

namespace {

__device__ __forceinline__ void load8(const float* p, float (&x)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  x[0] = a.x;
  x[1] = a.y;
  x[2] = a.z;
  x[3] = a.w;
  x[4] = b.x;
  x[5] = b.y;
  x[6] = b.z;
  x[7] = b.w;
}

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&x)[8]) {
  const uint4 v = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[2 * i] = __uint_as_float(w[i] << 16);
    x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

__device__ __forceinline__ float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ void store8_bf16(__nv_bfloat16* p, const float (&x)[8]) {
  uint4 v;
  v.x = pack_bf16x2(x[0], x[1]);
  v.y = pack_bf16x2(x[2], x[3]);
  v.z = pack_bf16x2(x[4], x[5]);
  v.w = pack_bf16x2(x[6], x[7]);
  *reinterpret_cast<uint4*>(p) = v;
}

template <typename Src, int D>
__global__ void __launch_bounds__(256) rope_append_kernel(const RopeAppendParams p) {
  constexpr int TPR = D / 8;  // threads per row, a power of two <= 32
  constexpr bool kBf16 = sizeof(Src) == 2;
  const long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int heads = p.Hq + 2 * p.Hkv;
  const long long rows = (long long)p.B * p.T * heads;
  const long long row = g / TPR;
  const int part = (int)(g % TPR);
  // Every lane takes part in the shuffles below; lanes past the last row or on
  // a rejected row compute on zeros and store nothing.
  bool active = row < rows;
  const long long r = active ? row : 0;
  const int j = (int)(r % heads);
  const long long bt = r / heads;
  const int t = (int)(bt % p.T);
  const int b = (int)(bt / p.T);
  const int pos0 = p.start_pos_arr ? p.start_pos_arr[b] : p.start_pos;
  const long long pos = (long long)pos0 + t;
  const int kind = j < p.Hq ? 0 : (j < p.Hq + p.Hkv ? 1 : 2);  // q, k, v
  const int h = kind == 0 ? j : (kind == 1 ? j - p.Hq : j - p.Hq - p.Hkv);
  if (active && kind == 0 && h == 0 && t == 0 && part == 0 && p.seqlens_out) p.seqlens_out[b] = pos0 + p.T;
  const bool rotated = kind != 2 && p.rope_dim > 0;
  if (active && (pos < 0 || (rotated && pos >= p.max_pos) || (kind != 0 && pos >= p.Lmax))) {
    if (p.err && part == 0) atomicOr(p.err, kErrBadArgs);
    active = false;
  }

  const int i0 = 8 * part;
  float x[8];
  if (active) {
    const Src* src;
    if (kind == 0)
      src = static_cast<const Src*>(p.q) + b * p.qs[0] + t * p.qs[1] + h * p.qs[2];
    else if (kind == 1)
      src = static_cast<const Src*>(p.k) + b * p.ks[0] + t * p.ks[1] + h * p.ks[2];
    else
      src = static_cast<const Src*>(p.v) + b * p.vs[0] + t * p.vs[1] + h * p.vs[2];
    load8(src + i0, x);
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = 0.f;
  }

  // Per-head RMSNorm over the D lanes of the row.
  if (p.q_norm || p.k_norm) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = __fmaf_rn(x[e], x[e], ss);
#pragma unroll
    for (int off = TPR / 2; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const void* wp = kind == 0 ? p.q_norm : (kind == 1 ? p.k_norm : nullptr);
    if (wp) {
      const float rms = rsqrtf(__fadd_rn(__fdiv_rn(ss, (float)D), p.norm_eps));
      float w[8];
      load8(static_cast<const Src*>(wp) + i0, w);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        x[e] = __fmul_rn(__fmul_rn(x[e], rms), w[e]);
        if (kBf16) x[e] = round_bf16(x[e]);
      }
    }
  }

  // Rotate-half on the first rope_dim lanes.
  if (p.rope_dim > 0) {
    const int xo = p.rope_dim / 16;  // lane distance of a rotate-half pair
    float y[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) y[e] = __shfl_xor_sync(0xffffffffu, x[e], xo);
    if (active && rotated && i0 < p.rope_dim) {
      const bool first = (part & xo) == 0;  // lanes [0, rope_dim/2): partner term is -x[e + rope_dim/2]
      float c[8], s[8];
      load8(static_cast<const Src*>(p.cos) + pos * p.rope_dim + i0, c);
      load8(static_cast<const Src*>(p.sin) + pos * p.rope_dim + i0, s);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float a = __fmul_rn(x[e], c[e]);
        float bb = __fmul_rn(first ? -y[e] : y[e], s[e]);
        if (kBf16) {
          a = round_bf16(a);
          bb = round_bf16(bb);
        }
        x[e] = __fadd_rn(a, bb);
      }
    }
  }
  if (!active) return;

  __nv_bfloat16* dst;
  if (kind == 0)
    dst = static_cast<__nv_bfloat16*>(p.q_out) + (((long long)b * p.Hq + h) * p.T + t) * D;
  else if (kind == 1)
    dst = static_cast<__nv_bfloat16*>(p.k_cache) + b * p.kcs[0] + h * p.kcs[1] + pos * p.kcs[2];
  else
    dst = static_cast<__nv_bfloat16*>(p.v_cache) + b * p.vcs[0] + h * p.vcs[1] + pos * p.vcs[2];
  store8_bf16(dst + i0, x);
}

template <typename Src, int D>
int launch_t(const RopeAppendParams& p, cudaStream_t st) {
  const long long rows = (long long)p.B * p.T * (p.Hq + 2 * p.Hkv);
  const long long threads = rows * (D / 8);
  const long long blocks = (threads + 255) / 256;
  if (blocks <= 0 || blocks > 0x7fffffffLL) return -2;
  rope_append_kernel<Src, D><<<(unsigned)blocks, 256, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

template <typename Src>
int launch_src(const RopeAppendParams& p, cudaStream_t st) {
  switch (p.D) {
    case 64: return launch_t<Src, 64>(p, st);
    case 128: return launch_t<Src, 128>(p, st);
    case 256: return launch_t<Src, 256>(p, st);
    default: return -3;
  }
}

}  // namespace

int launch_rope_append(const RopeAppendParams& p, cudaStream_t st) {
  return p.src_bf16 ? launch_src<__nv_bfloat16>(p, st) : launch_src<float>(p, st);
}

}  // namespace b2a
