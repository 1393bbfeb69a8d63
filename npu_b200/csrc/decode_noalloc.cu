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
// GPU that loads the library holds it until the process exits. With
// split_len = 0 the default split length is doubled until the partial results
// fit; a problem whose scratch exceeds the buffer even then (or with the
// split_len the caller chose) is rejected with B2A_ERR_WORKSPACE before any
// launch.
//
// The host-side name of the array is not a device address (handing it to a
// kernel would fault, or on systems where the GPU can reach host memory,
// silently use the wrong memory). The device address is looked up with
// cudaGetSymbolAddress the first time this entry point runs in a device's
// context, with that device current; make that first call outside any stream
// capture. The address is cached per device together with the context it
// belongs to, so a new context (after cudaDeviceReset) triggers a fresh
// lookup. All calls on a device share the one buffer, which keeps whatever the
// last call left there: calls whose kernels overlap on the GPU (different
// streams with no ordering between them) race on it. Nothing in it has to
// start at zero — each call writes every partial its combine step reads.
#include <cuda.h>

#include <mutex>

#include "b2attn.h"
#include "decode.cuh"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[B2A_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDev = 64;
std::mutex g_scratch_mu;
struct ScratchAddr {
  CUcontext ctx;
  void* addr;
};
ScratchAddr g_scratch[kMaxDev] = {};

using PfnCtxGetCurrent = CUresult (*)(CUcontext*);

// The calling thread's current driver context (nullptr if none or if the
// driver entry point is unavailable).
CUcontext current_context() {
  static std::once_flag once;
  static PfnCtxGetCurrent fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PfnCtxGetCurrent>(p);
  });
  CUcontext c = nullptr;
  if (fn && fn(&c) != CUDA_SUCCESS) c = nullptr;
  return c;
}

// Device address of g_noalloc_scratch on the current device. The library
// holds code for sm_100 only, so the compute capability is checked first: on
// another GPU the symbol lookup would fail and leave a sticky-looking CUDA
// error behind.
int noalloc_scratch(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) {
    cudaGetLastError();
    return B2A_ERR_CUDA;
  }
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) {
    cudaGetLastError();
    return B2A_ERR_CUDA;
  }
  if (major != 10 || minor != 0) return B2A_ERR_DEVICE;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  const CUcontext ctx = current_context();
  if (!g_scratch[dev].addr || !ctx || g_scratch[dev].ctx != ctx) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();  // leave no error for the caller's next runtime call to pick up
      g_scratch[dev] = ScratchAddr{};
      return B2A_ERR_CUDA;
    }
    // The lookup creates the primary context if the caller had none yet.
    g_scratch[dev] = ScratchAddr{ctx ? ctx : current_context(), p};
  }
  *out = g_scratch[dev].addr;
  return B2A_OK;
}

}  // namespace

extern "C" int b2a_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, const int* seqlens,
                                  void* o, int B, int Hq, int Hkv, int Lmax, int D, const long long* q_strides,
                                  const long long* k_strides, const long long* v_strides,
                                  const long long* o_strides, float scale, int split_len, int out_fp32,
                                  void* stream) {
  constexpr size_t kCap = (size_t)B2A_NOALLOC_SCRATCH_BYTES;
  if (split_len == 0) {
    // The speed-tuned default ignores the fixed buffer: lengthen the splits
    // (fewer partials) until they fit, up to one split per sequence.
    long long s = b2a_decode_default_split(B, Hkv, Lmax);
    while (s < Lmax && b2a_decode_workspace_bytes(B, Hq, Hkv, D, Lmax, (int)s) > kCap) s *= 2;
    split_len = (int)(s <= 0x7fffffc0LL ? s : 0x7fffffc0LL);  // a multiple of 64 that fits an int
  }
  const size_t need = b2a_decode_workspace_bytes(B, Hq, Hkv, D, Lmax, split_len);
  if (need > kCap) return B2A_ERR_WORKSPACE;
  // need == 0 means the geometry is invalid: b2a_decode reports which check
  // failed, before touching the scratch.
  void* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  return b2a_decode(q, k_cache, v_cache, seqlens, o, B, Hq, Hkv, Lmax, D, q_strides, k_strides, v_strides,
                    o_strides, scale, split_len, out_fp32, scratch, kCap, stream);
}
