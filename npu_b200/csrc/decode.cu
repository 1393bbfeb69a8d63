// Split-KV flash-decode for sm_100a: one query token per sequence against a
// contiguous bf16 KV cache [B, Hkv, Lmax, D] with per-sequence lengths.
//
// Semantics: the decode step of the reference (smollm.py:222-234 with T=1,
// where no mask is applied and the token attends to all Tk cached keys;
// qwen/forward.py:206-221 likewise). Query head h uses KV head
// h / (Hq / Hkv) (repeat_interleave, smollm.py:205-207).
//
// Kernel 1 (split): grid (split, kv_head, seq). A producer warp streams
// 64-key K/V tiles with TMA into a 128B-swizzled shared-memory ring; four
// compute warps each take 16 keys of every tile. The GQA group (up to 16 query
// heads of one KV head) is the M=16 side of mma.sync m16n8k16, so every KV byte
// read from HBM serves the whole group. Each split writes an fp32 partial O
// (normalised) and its log2-domain LSE per query head.
// Kernel 2 (combine): per (seq, query head), merge the splits' partials by LSE.
#include "decode.cuh"

namespace b2a {

template <int D>
struct DecodeCfg {
  static constexpr int TK = 64;  // keys per tile
  static constexpr int KCH = D / 64;
  static constexpr int CHUNK_BYTES = TK * 128;  // 64 rows x 128 B
  static constexpr int TILE_BYTES = TK * D * 2;  // K or V tile
  static constexpr int STAGES = (D == 256) ? 2 : (D == 128 ? 3 : 4);
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES;
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
  static constexpr int SCRATCH_BYTES = 4 * 16 * D * 4 + 2 * 4 * 16 * 4;  // O, m, l per warp
  static constexpr int BODY_BYTES = RING_BYTES > SCRATCH_BYTES ? RING_BYTES : SCRATCH_BYTES;
  static constexpr int OFF_BAR = BODY_BYTES;
  static constexpr int SMEM_BYTES = OFF_BAR + 128 + 1024;
  static constexpr int THREADS = 160;  // 4 compute warps + 1 producer warp
  static_assert(D == 64 || D == 128 || D == 256, "decode supports head_dim 64, 128, 256");
};

struct DecodeBars {
  uint64_t full[4];
  uint64_t empty[4];
  int abort_flag;
};

__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}

// Byte address of (key row r, 16-byte unit U along head_dim) in a 64-key tile
// loaded by TMA with SWIZZLE_128B: 64-column chunks of 64 rows x 128 B, the
// unit index XORed with (row & 7).
template <int D>
__device__ __forceinline__ uint32_t tile_addr(uint32_t base, int r, int U) {
  return base + (U >> 3) * DecodeCfg<D>::CHUNK_BYTES + r * 128 + (((U & 7) ^ (r & 7)) << 4);
}

__device__ __forceinline__ uint32_t ld_q_pair(const __nv_bfloat16* p) {
  return *reinterpret_cast<const uint32_t*>(p);
}

template <int D>
__global__ void __launch_bounds__(160)
    decode_split_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                        const __grid_constant__ DecodeParams p) {
  using C = DecodeCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  DecodeBars* bars = reinterpret_cast<DecodeBars*>(smem + C::OFF_BAR);
  volatile int* abort_flag = &bars->abort_flag;

  // Launched as a programmatic dependent of the previous kernel in the
  // stream: nothing that kernel may write is read before this wait.
  grid_dep_wait();
  // The combine kernel may launch now; it waits for this whole grid in its
  // own grid_dep_wait, so its CTAs only take SM slots that split CTAs free.
  grid_dep_launch();
  const int split = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  int L = p.seqlens[b];
  if (L > p.Lmax || L < 0) {
    if (threadIdx.x == 0 && split == 0 && g == 0 && p.err) atomicOr(p.err, kErrBadArgs);
    L = L < 0 ? 0 : p.Lmax;
  }
  const int kb = split * p.split_len;
  if (kb >= L) return;  // this split has no keys; the combine ignores it
  const int ke = min(L, kb + p.split_len);
  const int n_tiles = (ke - kb + C::TK - 1) / C::TK;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 4);
    }
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      int issued = 0;
      for (int i = 0; i < n_tiles; ++i) {
        const int slot = i % C::STAGES;
        const uint32_t ph = (uint32_t)(i / C::STAGES) & 1u;
        if (!mbar_wait(&bars->empty[slot], ph ^ 1u, abort_flag, p.err)) break;
        uint8_t* kdst = smem + slot * C::STAGE_BYTES;
        uint8_t* vdst = kdst + C::TILE_BYTES;
        mbar_arrive_expect_tx(&bars->full[slot], 2 * C::TILE_BYTES);
        const int row = kb + i * C::TK;
#pragma unroll
        for (int c = 0; c < C::KCH; ++c) {
          tma_load_4d(kdst + c * C::CHUNK_BYTES, &tm_k, &bars->full[slot], c * 64, row, g, b);
          tma_load_4d(vdst + c * C::CHUNK_BYTES, &tm_v, &bars->full[slot], c * 64, row, g, b);
        }
        issued = i + 1;
      }
      if (*abort_flag) {
        for (int i = max(0, issued - C::STAGES); i < issued; ++i)
          mbar_wait_quiet(&bars->full[i % C::STAGES], (uint32_t)(i / C::STAGES) & 1u);
      }
    }
  } else {
    // ------------------------------------------------------------ compute warps
    const int gr = lane >> 2, tq = lane & 3;
    const int rows_valid = p.group;
    // Q as the A operand of m16n8k16: rows = query heads of this KV group.
    uint32_t qa[D / 16][4];
    {
      const int h0 = g * p.group + gr, h1 = h0 + 8;
      const bool v0 = gr < rows_valid, v1 = gr + 8 < rows_valid;
      const __nv_bfloat16* q0 = p.q + (long long)b * p.q_sb + (long long)h0 * p.q_sh;
      const __nv_bfloat16* q1 = p.q + (long long)b * p.q_sb + (long long)h1 * p.q_sh;
#pragma unroll
      for (int k = 0; k < D / 16; ++k) {
        qa[k][0] = v0 ? ld_q_pair(q0 + 16 * k + 2 * tq) : 0u;
        qa[k][1] = v1 ? ld_q_pair(q1 + 16 * k + 2 * tq) : 0u;
        qa[k][2] = v0 ? ld_q_pair(q0 + 16 * k + 2 * tq + 8) : 0u;
        qa[k][3] = v1 ? ld_q_pair(q1 + 16 * k + 2 * tq + 8) : 0u;
      }
    }
    float acc[D / 8][4];
#pragma unroll
    for (int n = 0; n < D / 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    const float sl2 = p.scale_log2;
    const int mi = lane >> 3, mr = lane & 7;  // ldmatrix: matrix index / row in it

    for (int i = 0; i < n_tiles; ++i) {
      const int slot = i % C::STAGES;
      const bool w = mbar_wait(&bars->full[slot], (uint32_t)(i / C::STAGES) & 1u, abort_flag, p.err);
      if (!__all_sync(0xffffffffu, w)) break;
      const uint32_t kbase = smem_u32(smem + slot * C::STAGE_BYTES);
      const uint32_t vbase = kbase + C::TILE_BYTES;

      // S = Q K^T for this warp's 16 keys: two n8 groups.
      float s[2][4];
#pragma unroll
      for (int ng = 0; ng < 2; ++ng) {
        s[ng][0] = s[ng][1] = s[ng][2] = s[ng][3] = 0.f;
        const int r = 16 * warp + 8 * ng + mr;
#pragma unroll
        for (int kp = 0; kp < D / 32; ++kp) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4(tile_addr<D>(kbase, r, 4 * kp + mi), b0, b1, b2, b3);
          mma_bf16_16816(s[ng], qa[2 * kp], b0, b1);
          mma_bf16_16816(s[ng], qa[2 * kp + 1], b2, b3);
        }
      }
      // Mask keys past this split's end (and past the sequence length).
      const int key0 = kb + i * C::TK + 16 * warp + 2 * tq;
#pragma unroll
      for (int ng = 0; ng < 2; ++ng)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          if (key0 + 8 * ng + e >= ke) {
            s[ng][e] = -INFINITY;
            s[ng][2 + e] = -INFINITY;
          }
        }
      float mx0 = fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1]));
      float mx1 = fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3]));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m0, mx0 * sl2), mn1 = fmaxf(m1, mx1 * sl2);
      const float u0 = (mn0 == -INFINITY) ? 0.f : mn0, u1 = (mn1 == -INFINITY) ? 0.f : mn1;
      const float a0 = ex2(m0 - u0), a1 = ex2(m1 - u1);
      m0 = mn0;
      m1 = mn1;
      float pr[2][4];
#pragma unroll
      for (int ng = 0; ng < 2; ++ng) {
        pr[ng][0] = ex2(fmaf(s[ng][0], sl2, -u0));
        pr[ng][1] = ex2(fmaf(s[ng][1], sl2, -u0));
        pr[ng][2] = ex2(fmaf(s[ng][2], sl2, -u1));
        pr[ng][3] = ex2(fmaf(s[ng][3], sl2, -u1));
      }
      l0 = l0 * a0 + pr[0][0] + pr[0][1] + pr[1][0] + pr[1][1];
      l1 = l1 * a1 + pr[0][2] + pr[0][3] + pr[1][2] + pr[1][3];
#pragma unroll
      for (int n = 0; n < D / 8; ++n) {
        acc[n][0] *= a0;
        acc[n][1] *= a0;
        acc[n][2] *= a1;
        acc[n][3] *= a1;
      }
      uint32_t pa[4];
      pa[0] = pack_bf16x2(pr[0][0], pr[0][1]);
      pa[1] = pack_bf16x2(pr[0][2], pr[0][3]);
      pa[2] = pack_bf16x2(pr[1][0], pr[1][1]);
      pa[3] = pack_bf16x2(pr[1][2], pr[1][3]);
      // O += P V: V rows are keys, transposed ldmatrix gives the k16 x n8 B operand.
      const int vr = 16 * warp + 8 * (mi & 1) + mr;
#pragma unroll
      for (int dn = 0; dn < D / 8; dn += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(tile_addr<D>(vbase, vr, dn + (mi >> 1)), b0, b1, b2, b3);
        mma_bf16_16816(acc[dn], pa, b0, b1);
        mma_bf16_16816(acc[dn + 1], pa, b2, b3);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->empty[slot]);
    }

    // Merge the four warps' (m, l, O) for every query head of the group.
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    asm volatile("bar.sync 1, 128;" ::: "memory");  // all compute warps done reading the ring
    float* so = reinterpret_cast<float*>(smem);     // [4][16][D]
    float* sm = so + 4 * 16 * D;                    // [4][16]
    float* sl = sm + 4 * 16;                        // [4][16]
#pragma unroll
    for (int n = 0; n < D / 8; ++n) {
      float* r0p = so + (warp * 16 + gr) * D + 8 * n + 2 * tq;
      float* r1p = so + (warp * 16 + gr + 8) * D + 8 * n + 2 * tq;
      r0p[0] = acc[n][0];
      r0p[1] = acc[n][1];
      r1p[0] = acc[n][2];
      r1p[1] = acc[n][3];
    }
    if (tq == 0) {
      sm[warp * 16 + gr] = m0;
      sm[warp * 16 + gr + 8] = m1;
      sl[warp * 16 + gr] = l0;
      sl[warp * 16 + gr + 8] = l1;
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    const long long pidx = ((long long)b * p.Hkv + g) * p.max_splits + split;
    for (int e = threadIdx.x; e < rows_valid * D; e += 128) {
      const int r = e / D, d = e % D;
      float M = -INFINITY;
#pragma unroll
      for (int w2 = 0; w2 < 4; ++w2) M = fmaxf(M, sm[w2 * 16 + r]);
      const float Mu = (M == -INFINITY) ? 0.f : M;
      float lsum = 0.f, osum = 0.f;
#pragma unroll
      for (int w2 = 0; w2 < 4; ++w2) {
        const float f = ex2(sm[w2 * 16 + r] - Mu);
        lsum += f * sl[w2 * 16 + r];
        osum += f * so[(w2 * 16 + r) * D + d];
      }
      p.part_o[(pidx * p.group + r) * D + d] = lsum > 0.f ? osum / lsum : 0.f;
      if (d == 0) p.part_lse[pidx * p.group + r] = lsum > 0.f ? M + __log2f(lsum) : -INFINITY;
    }
  }
  __syncthreads();
}

// One CTA per (sequence, query head); thread d owns output column d.
__global__ void decode_combine_kernel(const __grid_constant__ DecodeParams p, int D) {
  grid_dep_wait();  // every split's partials are written and visible
  const int bh = blockIdx.x;
  const int b = bh / p.Hq, h = bh % p.Hq;
  const int g = h / p.group, r = h % p.group;
  int L = p.seqlens[b];
  L = L < 0 ? 0 : (L > p.Lmax ? p.Lmax : L);
  int ns = (L + p.split_len - 1) / p.split_len;
  ns = ns > p.max_splits ? p.max_splits : ns;
  const long long base = ((long long)b * p.Hkv + g) * p.max_splits;
  float M = -INFINITY;
  for (int s = 0; s < ns; ++s) M = fmaxf(M, p.part_lse[(base + s) * p.group + r]);
  const float Mu = (M == -INFINITY) ? 0.f : M;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float wsum = 0.f, osum = 0.f;
    for (int s = 0; s < ns; ++s) {
      const float w = ex2(p.part_lse[(base + s) * p.group + r] - Mu);
      wsum += w;
      osum += w * p.part_o[((base + s) * p.group + r) * D + d];
    }
    float v = wsum > 0.f ? osum / wsum : 0.f;
    if (p.gate) {
      const long long gi = (long long)b * p.g_sb + (long long)h * p.g_sh + d;
      const float gv = p.gate_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(p.gate)[gi])
                                   : static_cast<const float*>(p.gate)[gi];
      v *= __fdividef(1.f, 1.f + __expf(-gv));  // sigmoid, as torch.sigmoid in fp32
    }
    if (p.o) {
      const long long oi = (long long)b * p.o_sb + (long long)h * p.o_sh + d;
      if (p.out_fp32)
        reinterpret_cast<float*>(p.o)[oi] = v;
      else
        reinterpret_cast<__nv_bfloat16*>(p.o)[oi] = __float2bfloat16_rn(v);
    }
  }
}

// Combine fused with the output projection and residual add (b2a_decode_proj):
// one CTA per (block of PROJ_N outputs, sequence). It merges the splits of
// every query head of its sequence into the attention output o [Hq * D]
// (shared memory; the same per-element arithmetic as decode_combine_kernel,
// then rounded to x's dtype), and adds o @ wo^T for its outputs into the
// residual stream: warp w takes outputs n0 + w, n0 + w + 4, ..., its lanes
// stride over o and the weight row, and a fixed shuffle tree sums them. Every
// output has one writer and a fixed summation order, so the result does not
// depend on scheduling.
constexpr int kProjN = 32;  // outputs per CTA
constexpr int kProjMaxSmem = 200 * 1024;  // attention output row of one sequence, Hq * D floats

__global__ void decode_combine_proj_kernel(const __grid_constant__ DecodeParams p, int D) {
  extern __shared__ float sm_proj[];
  grid_dep_wait();  // every split's partials are written and visible
  const int b = blockIdx.y;
  const int HD = p.Hq * D;
  float* so = sm_proj;             // [Hq * D] attention output of sequence b
  float* sM = so + HD;             // [Hq] per-head max LSE (log2 domain)
  float* sW = sM + p.Hq;           // [Hq] per-head sum of split weights
  int L = p.seqlens[b];
  L = L < 0 ? 0 : (L > p.Lmax ? p.Lmax : L);
  int ns = (L + p.split_len - 1) / p.split_len;
  ns = ns > p.max_splits ? p.max_splits : ns;
  for (int h = threadIdx.x; h < p.Hq; h += blockDim.x) {
    const int g = h / p.group, r = h % p.group;
    const long long base = ((long long)b * p.Hkv + g) * p.max_splits;
    float M = -INFINITY;
    for (int sp = 0; sp < ns; ++sp) M = fmaxf(M, p.part_lse[(base + sp) * p.group + r]);
    const float Mu = (M == -INFINITY) ? 0.f : M;
    float wsum = 0.f;
    for (int sp = 0; sp < ns; ++sp) wsum += ex2(p.part_lse[(base + sp) * p.group + r] - Mu);
    sM[h] = Mu;
    sW[h] = wsum;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < HD; e += blockDim.x) {
    const int h = e / D, d = e % D;
    const int g = h / p.group, r = h % p.group;
    const long long base = ((long long)b * p.Hkv + g) * p.max_splits;
    float osum = 0.f;
    for (int sp = 0; sp < ns; ++sp)
      osum += ex2(p.part_lse[(base + sp) * p.group + r] - sM[h]) * p.part_o[((base + sp) * p.group + r) * D + d];
    const float v = sW[h] > 0.f ? osum / sW[h] : 0.f;
    so[e] = p.x_fp32 ? v : __bfloat162float(__float2bfloat16_rn(v));
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const int n0 = blockIdx.x * kProjN;
  for (int n = n0 + warp; n < min(n0 + kProjN, p.dim); n += nwarps) {
    float acc = 0.f;
    if (p.wo_fp32) {
      const float* w = static_cast<const float*>(p.wo) + (long long)n * p.wo_ld;
      for (int k = lane; k < HD; k += 32) acc = fmaf(so[k], w[k], acc);
    } else {
      const __nv_bfloat16* w = static_cast<const __nv_bfloat16*>(p.wo) + (long long)n * p.wo_ld;
      for (int k = lane; k < HD; k += 32) acc = fmaf(so[k], __bfloat162float(w[k]), acc);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) {
      const long long xi = (long long)b * p.x_sb + n;
      if (p.x_fp32) {
        float* xp = reinterpret_cast<float*>(p.x) + xi;
        *xp = *xp + acc;
      } else {
        __nv_bfloat16* xp = reinterpret_cast<__nv_bfloat16*>(p.x) + xi;
        *xp = __float2bfloat16_rn(__bfloat162float(*xp) + acc);
      }
    }
  }
}

// ------------------------------------------------------------------ launchers
template <int D>
static int launch_decode_t(const CUtensorMap& tk, const CUtensorMap& tv, const DecodeParams& p,
                           cudaStream_t st) {
  using C = DecodeCfg<D>;
  cudaError_t e = cudaFuncSetAttribute(decode_split_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       C::SMEM_BYTES);
  if (e != cudaSuccess) return -1;
  // Both kernels are launched with programmatic stream serialization: each
  // may be scheduled while the kernel before it drains, and waits for it in
  // grid_dep_wait before reading anything (split: the previous kernel's
  // outputs, e.g. q or a cache append; combine: the split's partials).
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)p.max_splits, (unsigned)p.Hkv, (unsigned)p.B);
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, decode_split_kernel<D>, tk, tv, p) != cudaSuccess) return -1;
  if (p.wo) {
    const size_t smem = ((size_t)p.Hq * D + 2 * (size_t)p.Hq) * sizeof(float);
    if (smem > (size_t)kProjMaxSmem) return -4;
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(decode_combine_proj_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
      return -1;
    cfg.gridDim = dim3((unsigned)((p.dim + kProjN - 1) / kProjN), (unsigned)p.B);
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = smem;
    if (cudaLaunchKernelEx(&cfg, decode_combine_proj_kernel, p, D) != cudaSuccess) return -1;
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
  }
  cfg.gridDim = dim3((unsigned)(p.B * p.Hq));
  cfg.blockDim = dim3(D < 128 ? 64 : 128);
  cfg.dynamicSmemBytes = 0;
  if (cudaLaunchKernelEx(&cfg, decode_combine_kernel, p, D) != cudaSuccess) return -1;
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int launch_decode(int D, const CUtensorMap& tk, const CUtensorMap& tv, const DecodeParams& p, cudaStream_t st) {
  switch (D) {
    case 64: return launch_decode_t<64>(tk, tv, p, st);
    case 128: return launch_decode_t<128>(tk, tv, p, st);
    case 256: return launch_decode_t<256>(tk, tv, p, st);
    default: return -3;
  }
}

}  // namespace b2a
