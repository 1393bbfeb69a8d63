// Diagnostic: one 128x128x128 bf16 UMMA through the same descriptor and
// swizzle conventions the prefill kernel uses, so a layout error shows up as a
// wrong GEMM rather than as a wrong attention output.
//   b_mn_major = 0: C = A * B^T with B given as [N=128][K=128] (the S = Q K^T path)
//   b_mn_major = 1: C = A * B   with B given as [K=128][N=128] (the O = P V path)
//   b_mn_major = 2: as 1, but A is read from TMEM (the P-in-TMEM path): each
//                   thread stores its row of A into TMEM with tcgen05.st.
// A is [M=128][K=128] row-major. Operands are written into shared memory by
// threads using the 128-byte swizzle formula.
#include "b2attn_diag.h"
#include "common.cuh"

namespace b2a {

__global__ void __launch_bounds__(128) diag_umma_kernel(const __nv_bfloat16* A, const __nv_bfloat16* Bm, float* C,
                                                        int b_mn, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  uint8_t* sA = smem;
  uint8_t* sB = smem + 32768;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 65536);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 65536 + 64);
  int* abort_flag = reinterpret_cast<int*>(smem + 65536 + 128);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int CH = 16384;

  // Row r (M or N, or K for the MN-major B), 64-element chunk c / 64.
  auto sw = [&](uint8_t* base, int r, int c) -> __nv_bfloat16* {
    const int unit = (c & 63) >> 3;
    return reinterpret_cast<__nv_bfloat16*>(base + (c >> 6) * CH + r * 128 + ((unit ^ (r & 7)) << 4) +
                                            (c & 7) * 2);
  };
  for (int i = tid; i < 128 * 128; i += 128) {
    const int r = i >> 7, c = i & 127;
    *sw(sA, r, c) = A[i];
    *sw(sB, r, c) = Bm[i];  // K-major: r = n, c = k; MN-major: r = k, c = n
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  fence_proxy_async_smem();
  if (warp == 0) tmem_alloc(tmem_slot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  constexpr uint32_t kACol = 128;  // A (packed bf16) at TMEM columns [128, 192)
  if (b_mn == 2) {
    const uint32_t* arow = reinterpret_cast<const uint32_t*>(A) + tid * 64;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t r[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) r[i] = arow[half * 32 + i];
      tmem_st32(tmem + lane_off + kACol + half * 32, r);
    }
    tmem_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid == 0) {
    const uint32_t a = smem_u32(sA), b = smem_u32(sB);
    const uint32_t idesc = umma_idesc_bf16(128, 128, b_mn != 0);
    for (int k = 0; k < 8; ++k) {
      const uint32_t off = (k >> 2) * CH + (k & 3) * 32;
      const uint64_t bd = b_mn ? make_sdesc_sw128(b + k * 2048, CH, 1024) : make_sdesc_sw128(b + off, 16, 1024);
      if (b_mn == 2)
        umma_bf16_ts(tmem, tmem + kACol + k * 8, bd, idesc, k > 0 ? 1u : 0u);
      else
        umma_bf16_ss(tmem, make_sdesc_sw128(a + off, 16, 1024), bd, idesc, k > 0 ? 1u : 0u);
    }
    tc_commit(bar);
  }
  __syncwarp();
  const bool ok = mbar_wait(bar, 0, abort_flag, err);
  if (__all_sync(0xffffffffu, ok)) {
    tc_fence_after();
    const int row = warp * 32 + lane;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t r[32];
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + 32 * q, r);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) C[row * 128 + 32 * q + i] = __uint_as_float(r[i]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// A wait on an mbarrier that nothing ever arrives on, bounded by `limit`
// cycles: the failure path every kernel's waits take (abort flag, error word,
// orderly exit) exercised on purpose, without faulting or hanging the GPU.
__global__ void __launch_bounds__(32) diag_wait_timeout_kernel(long long limit, int* err) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncwarp();
  const bool ok = mbar_wait_limit(&bar, 0, &abort_flag, threadIdx.x == 0 ? err : nullptr, limit);
  (void)ok;
}

}  // namespace b2a

extern "C" int b2a_diag_wait_timeout(long long limit_cycles, void* stream) {
  if (limit_cycles <= 0 || limit_cycles > 4000000000LL) return -1;
  int* err = b2a::device_error_word();
  if (!err) return -11;
  b2a::diag_wait_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_cycles, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

extern "C" int b2a_diag_umma_gemm(const void* a, const void* b, float* c, int b_mn_major, void* stream) {
  if (!a || !b || !c) return -1;
  constexpr int smem = 65536 + 256 + 1024;
  if (cudaFuncSetAttribute(b2a::diag_umma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
      cudaSuccess)
    return -6;
  b2a::diag_umma_kernel<<<1, 128, smem, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(a), static_cast<const __nv_bfloat16*>(b), c, b_mn_major, nullptr);
  return cudaGetLastError() == cudaSuccess ? 0 : -6;
}
