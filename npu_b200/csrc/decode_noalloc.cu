// b2a_decode_noalloc: the split-KV decode for callers that cannot allocate
// device memory.
//
// b2a_decode needs caller-provided scratch for the per-split partial results.
// Some callers have no way to provide it: hosts that reserve all device
// memory at start-up for their own pool and forbid any later cudaMalloc (it
// would fail, or fragment a pool sized to the byte), hosts that must not pay
// the implicit device-wide synchronisation a cudaFree brings, and plugin / FFI
// callers that only hold raw input and output pointers with no handle to an
// allocator. This entry point takes the same inputs and outputs as b2a_decode
// and uses a fixed scratch buffer compiled into the library instead.
//
// The buffer is a file-scope device array of B2A_NOALLOC_SCRATCH_BYTES: every
// GPU that loads the library holds it until the process exits. A problem whose
// scratch would exceed it is rejected with B2A_ERR_WORKSPACE (pass a larger
// split_len, or use b2a_decode with your own workspace).
//
// The host-side name of the array is not a device address (handing it to a
// kernel would fault, or on systems where the GPU can reach host memory,
// silently use the wrong memory). The device address is looked up with
// cudaGetSymbolAddress the first time this entry point runs on a device, with
// that device current; make that first call outside any stream capture. All
// calls on a device share the one buffer, which keeps whatever the last call
// left there: calls whose kernels overlap on the GPU (different streams with
// no ordering between them) race on it. Nothing in it has to start at zero —
// each call writes every partial its combine step reads.
#include <mutex>

#include "b2attn.h"
#include "decode.cuh"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[B2A_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDev = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDev] = {};

// Device address of g_noalloc_scratch on the current device (looked up once
// per device).
int noalloc_scratch(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return B2A_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return B2A_ERR_CUDA;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return B2A_OK;
}

}  // namespace

extern "C" int b2a_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, const int* seqlens,
                                  void* o, int B, int Hq, int Hkv, int Lmax, int D, const long long* q_strides,
                                  const long long* k_strides, const long long* v_strides,
                                  const long long* o_strides, float scale, int split_len, int out_fp32,
                                  void* stream) {
  if (split_len == 0) split_len = b2a_decode_default_split(B, Hkv, Lmax);
  if (b2a_decode_workspace_bytes(B, Hq, Hkv, D, Lmax, split_len) > (size_t)B2A_NOALLOC_SCRATCH_BYTES)
    return B2A_ERR_WORKSPACE;
  void* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  return b2a_decode(q, k_cache, v_cache, seqlens, o, B, Hq, Hkv, Lmax, D, q_strides, k_strides, v_strides,
                    o_strides, scale, split_len, out_fp32, scratch, (size_t)B2A_NOALLOC_SCRATCH_BYTES, stream);
}
