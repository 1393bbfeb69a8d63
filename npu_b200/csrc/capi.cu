// extern "C" boundary of libb2attn (declared in include/b2attn.h): argument
// validation, TMA tensor-map encoding and kernel launch. Stateless apart from
// per-device caches (driver entry point, error-word address, arch check).
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdint>
#include <mutex>

#include "b2attn.h"
#include "decode.cuh"
#include "prefill.cuh"
#include "rope_append.cuh"

namespace {

constexpr int kMaxDevices = 64;

// Error word the kernels OR their device-side failure bits into. One per
// device (module-scope __device__ variable); read by b2a_get_device_error.
__device__ int g_b2a_err_word;

std::mutex g_mu;
int* g_err_ptr[kMaxDevices] = {};
int g_arch_ok[kMaxDevices] = {};  // 0 unknown, 1 sm_100, -1 other

int current_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
  return dev;
}

bool device_is_sm100(int dev) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_arch_ok[dev] == 0) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    g_arch_ok[dev] = (major == 10 && minor == 0) ? 1 : -1;
  }
  return g_arch_ok[dev] == 1;
}

// Device address of g_b2a_err_word for the current device (the host-side
// name of a __device__ variable is not a device address).
int* device_err_ptr(int dev) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_err_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_b2a_err_word) != cudaSuccess) return nullptr;
    g_err_ptr[dev] = static_cast<int*>(p);
  }
  return g_err_ptr[dev];
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// bf16 tensor [n3, n2, rows, D] (innermost D contiguous) with element strides
// s_row, s_2, s_3; box = 64 columns x box_rows rows, 128-byte swizzle,
// out-of-range elements read as zero.
int tmap_bf16_4d(CUtensorMap* m, const void* base, int D, long long rows, long long n2, long long n3,
                 long long s_row, long long s_2, long long s_3, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return B2A_ERR_TMA;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)(rows > 0 ? rows : 1), (cuuint64_t)n2, (cuuint64_t)n3};
  cuuint64_t strides[3] = {(cuuint64_t)(s_row * 2), (cuuint64_t)(s_2 * 2), (cuuint64_t)(s_3 * 2)};
  cuuint32_t box[4] = {64u, (cuuint32_t)box_rows, 1u, 1u};
  cuuint32_t es[4] = {1u, 1u, 1u, 1u};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? B2A_OK : B2A_ERR_TMA;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool strides_ok(const long long* s, int n, long long mult) {
  for (int i = 0; i < n; ++i)
    if (s[i] < 0 || (s[i] % mult) != 0) return false;
  return true;
}

// Per-device prologue shared by every entry point: arch check and the
// device error-word address.
int prologue(int** err) {
  const int dev = current_device();
  if (dev < 0) return B2A_ERR_CUDA;
  if (!device_is_sm100(dev)) return B2A_ERR_DEVICE;
  *err = device_err_ptr(dev);
  return *err ? B2A_OK : B2A_ERR_CUDA;
}

constexpr float kLog2e = 1.4426950408889634f;

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

int decode_geometry(int B, int Hq, int Hkv, int D, int Lmax, int split_len, int* group, int* max_splits) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Lmax <= 0 || split_len <= 0 || split_len % 64) return B2A_ERR_INVALID_ARG;
  if (D != 64 && D != 128 && D != 256) return B2A_ERR_HEAD_DIM;
  if (Hq % Hkv) return B2A_ERR_GQA;
  *group = Hq / Hkv;
  if (*group > 16) return B2A_ERR_GQA;
  *max_splits = (Lmax + split_len - 1) / split_len;
  return B2A_OK;
}

}  // namespace

namespace {

int rope_append_impl(const void* q, const void* k, const void* v, const long long* qs, const long long* ks,
                     const long long* vs, int src_bf16, const void* cos_tab, const void* sin_tab, int max_pos,
                     int rope_dim, const void* q_norm, const void* k_norm, float eps, void* q_out, void* k_cache,
                     void* v_cache, const long long* kcs, const long long* vcs, int B, int T, int Hq, int Hkv,
                     int D, int Lmax, int start_pos, const int* start_pos_per_batch, int* seqlens_out,
                     void* stream) {
  if (!q || !k || !v || !qs || !ks || !vs || !q_out || !k_cache || !v_cache || !kcs || !vcs)
    return B2A_ERR_INVALID_ARG;
  if (B <= 0 || T <= 0 || Hq <= 0 || Hkv <= 0 || Lmax <= 0) return B2A_ERR_INVALID_ARG;
  if (D != 64 && D != 128 && D != 256) return B2A_ERR_HEAD_DIM;
  // rope_dim: 0 (no rotation) or a power of two in [16, D] (a rotate-half pair
  // is then one lane-xor apart in the kernel's layout).
  if (rope_dim != 0 && (rope_dim < 16 || rope_dim > D || (rope_dim & (rope_dim - 1))))
    return B2A_ERR_INVALID_ARG;
  if (rope_dim && (!cos_tab || !sin_tab || max_pos <= 0)) return B2A_ERR_INVALID_ARG;
  if ((q_norm || k_norm) && !(eps >= 0.f && std::isfinite(eps))) return B2A_ERR_INVALID_ARG;
  if (!start_pos_per_batch &&
      (start_pos < 0 || (long long)start_pos + T > Lmax || (rope_dim && (long long)start_pos + T > max_pos)))
    return B2A_ERR_INVALID_ARG;
  const uintptr_t src_align = 15u;  // 8 consecutive elements per thread: 32 B (fp32) or 16 B (bf16)
  for (const void* ptr : {q, k, v, cos_tab, sin_tab, q_norm, k_norm})
    if (reinterpret_cast<uintptr_t>(ptr) & src_align) return B2A_ERR_ALIGNMENT;
  for (const void* ptr : {(const void*)q_out, (const void*)k_cache, (const void*)v_cache})
    if (reinterpret_cast<uintptr_t>(ptr) & 15u) return B2A_ERR_ALIGNMENT;
  const long long mult = src_bf16 ? 8 : 4;
  if (!strides_ok(qs, 3, mult) || !strides_ok(ks, 3, mult) || !strides_ok(vs, 3, mult) ||
      !strides_ok(kcs, 3, 8) || !strides_ok(vcs, 3, 8))
    return B2A_ERR_ALIGNMENT;

  int* err = nullptr;
  int rc = prologue(&err);
  if (rc) return rc;
  b2a::RopeAppendParams p{};
  p.q = q;
  p.k = k;
  p.v = v;
  for (int i = 0; i < 3; ++i) {
    p.qs[i] = qs[i];
    p.ks[i] = ks[i];
    p.vs[i] = vs[i];
    p.kcs[i] = kcs[i];
    p.vcs[i] = vcs[i];
  }
  p.cos = cos_tab;
  p.sin = sin_tab;
  p.max_pos = max_pos;
  p.rope_dim = rope_dim;
  p.q_norm = q_norm;
  p.k_norm = k_norm;
  p.norm_eps = eps;
  p.q_out = q_out;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.B = B;
  p.T = T;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.D = D;
  p.Lmax = Lmax;
  p.start_pos = start_pos;
  p.start_pos_arr = start_pos_per_batch;
  p.seqlens_out = seqlens_out;
  p.src_bf16 = src_bf16 ? 1 : 0;
  p.err = err;
  rc = b2a::launch_rope_append(p, static_cast<cudaStream_t>(stream));
  if (rc == -3) return B2A_ERR_HEAD_DIM;
  return rc ? B2A_ERR_LAUNCH : B2A_OK;
}

}  // namespace

namespace {

int prefill_impl(const void* q, const void* k, const void* v, void* o, float* lse, int B, int Hq, int Hkv, int Tq,
                 int Tk, int D, const long long* qs, const long long* ks, const long long* vs, const long long* os,
                 int start_pos, const int* start_pos_per_batch, float scale, int causal, int out_fp32,
                 const void* gate, const long long* gs, int gate_bf16, void* stream) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Tq <= 0 || Tk < 0) return B2A_ERR_INVALID_ARG;
  // With no keys, K and V are never read (every row outputs 0); an empty
  // tensor may come with a null pointer, so give the tensor maps q instead.
  if (Tk == 0) {
    k = q;
    v = q;
    ks = qs;
    vs = qs;
  }
  if (!q || !k || !v || !o || !qs || !ks || !vs || !os) return B2A_ERR_INVALID_ARG;
  if (!(scale > 0.f) || !std::isfinite(scale)) return B2A_ERR_INVALID_ARG;
  if (D != 64 && D != 128 && D != 256) return B2A_ERR_HEAD_DIM;
  if (Hq % Hkv) return B2A_ERR_GQA;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o)) return B2A_ERR_ALIGNMENT;
  if (lse && (reinterpret_cast<uintptr_t>(lse) & 3u)) return B2A_ERR_ALIGNMENT;
  if (!strides_ok(qs, 3, 8) || !strides_ok(ks, 3, 8) || !strides_ok(vs, 3, 8) ||
      !strides_ok(os, 3, out_fp32 ? 4 : 8))
    return B2A_ERR_ALIGNMENT;
  if (gate && (!gs || !aligned16(gate) || !strides_ok(gs, 3, gate_bf16 ? 8 : 4))) return B2A_ERR_ALIGNMENT;
  // Work items: 128 query rows for D = 256; for D <= 128 two 128-row tiles
  // (two row blocks of one head, or one row block of two heads of a GQA
  // group), or one tile for short sequences (prefill_plan).
  const b2a::PrefillPlan plan = D == 256 ? b2a::PrefillPlan{128, 1, 0, 0} : b2a::prefill_plan(D, Hq, Hkv, Tq, Tk);
  const int rows_per_cta = plan.rows_per_item;
  const long long n_qblk = (Tq + rows_per_cta - 1) / rows_per_cta;
  if (n_qblk * Hq * (long long)B > 0x7fffffffLL) return B2A_ERR_INVALID_ARG;

  int* err = nullptr;
  int rc = prologue(&err);
  if (rc) return rc;

  CUtensorMap tq, tk, tv;
  if ((rc = tmap_bf16_4d(&tq, q, D, Tq, Hq, B, qs[2], qs[1], qs[0], 128))) return rc;
  const int kv_heads_map = Tk == 0 ? Hq : Hkv;  // Tk == 0: maps describe q, never loaded
  // Key-tile rows per TMA box: 128 for the two-tile kernel, 64 for D = 256;
  // on SM pairs each CTA loads 32-key pieces of K and 128-key halves of V.
  const int kv_box = D == 256 ? 64 : 128;
  const int k_box = plan.sm_pairs ? 32 : kv_box;
  if ((rc = tmap_bf16_4d(&tk, k, D, Tk, kv_heads_map, B, ks[2], ks[1], ks[0], k_box))) return rc;
  if ((rc = tmap_bf16_4d(&tv, v, D, Tk, kv_heads_map, B, vs[2], vs[1], vs[0], kv_box))) return rc;
  // Per-row stores use 32-byte vector stores when O and its strides allow.
  const int esz = out_fp32 ? 4 : 2;
  const int o_v8 = (reinterpret_cast<uintptr_t>(o) % 32 == 0 && (os[0] * esz) % 32 == 0 &&
                    (os[1] * esz) % 32 == 0 && (os[2] * esz) % 32 == 0)
                       ? 1
                       : 0;

  b2a::PrefillParams p{};
  p.o = o;
  p.o_sb = os[0];
  p.o_sh = os[1];
  p.o_st = os[2];
  p.lse = lse;
  p.start_pos_arr = start_pos_per_batch;
  p.start_pos = start_pos;
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.Tq = Tq;
  p.Tk = Tk;
  p.scale_log2 = scale * kLog2e;
  p.causal = causal ? 1 : 0;
  p.out_fp32 = out_fp32 ? 1 : 0;
  p.n_qblk = (int)n_qblk;
  p.head_pairs = plan.head_pairs;
  p.err = err;
  p.gate = gate;
  if (gate) {
    p.g_sb = gs[0];
    p.g_sh = gs[1];
    p.g_st = gs[2];
    p.gate_bf16 = gate_bf16 ? 1 : 0;
  }
  p.o_v8 = o_v8;
  rc = D == 256        ? b2a::launch_prefill_d256(tq, tk, tv, p, static_cast<cudaStream_t>(stream))
       : plan.sm_pairs ? b2a::launch_prefill_pair(tq, tk, tv, p, static_cast<cudaStream_t>(stream))
                       : b2a::launch_prefill(D, plan, tq, tk, tv, p, static_cast<cudaStream_t>(stream));
  if (rc == -3) return B2A_ERR_HEAD_DIM;
  return rc ? B2A_ERR_LAUNCH : B2A_OK;
}

// Fused output projection of b2a_decode_proj (nullptr: plain decode).
struct DecodeProj {
  const void* wo;
  long long wo_ld;
  int dim, wo_fp32;
  void* x;
  long long x_sb;
  int x_fp32;
};

int decode_impl(const void* q, const void* k_cache, const void* v_cache, const int* seqlens, void* o, int B,
                int Hq, int Hkv, int Lmax, int D, const long long* qs, const long long* ks, const long long* vs,
                const long long* os, float scale, int split_len, int out_fp32, void* workspace,
                size_t workspace_bytes, const void* gate, const long long* gs, int gate_bf16, void* stream,
                const DecodeProj* proj = nullptr) {
  if (!q || !k_cache || !v_cache || !seqlens || !qs || !ks || !vs) return B2A_ERR_INVALID_ARG;
  if (!proj && (!o || !os)) return B2A_ERR_INVALID_ARG;
  if (!(scale > 0.f) || !std::isfinite(scale)) return B2A_ERR_INVALID_ARG;
  if (split_len == 0) split_len = b2a_decode_default_split(B, Hkv, Lmax);
  int group = 0, max_splits = 0;
  int rc = decode_geometry(B, Hq, Hkv, D, Lmax, split_len, &group, &max_splits);
  if (rc) return rc;
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || (o && !aligned16(o))) return B2A_ERR_ALIGNMENT;
  if (!strides_ok(qs, 2, 8) || !strides_ok(ks, 3, 8) || !strides_ok(vs, 3, 8) || (o && !strides_ok(os, 2, 1)))
    return B2A_ERR_ALIGNMENT;
  if (proj) {
    if (!proj->wo || !proj->x || proj->dim <= 0 || proj->wo_ld < (long long)Hq * D || proj->x_sb < proj->dim)
      return B2A_ERR_INVALID_ARG;
    // The combine holds one sequence's attention output (Hq * D floats) in
    // shared memory.
    if (((long long)Hq * D + 2LL * Hq) * 4 > 200LL * 1024) return B2A_ERR_INVALID_ARG;
    // 16-byte vector reads of each weight row segment; element-aligned x.
    if (!aligned16(proj->wo) || proj->wo_ld % (proj->wo_fp32 ? 4 : 8) ||
        (reinterpret_cast<uintptr_t>(proj->x) & (proj->x_fp32 ? 3u : 1u)))
      return B2A_ERR_ALIGNMENT;
  }
  const size_t need = b2a_decode_workspace_bytes(B, Hq, Hkv, D, Lmax, split_len);
  if (!workspace || workspace_bytes < need || !aligned16(workspace)) return B2A_ERR_WORKSPACE;

  int* err = nullptr;
  if ((rc = prologue(&err))) return rc;

  CUtensorMap tk, tv;
  if ((rc = tmap_bf16_4d(&tk, k_cache, D, Lmax, Hkv, B, ks[2], ks[1], ks[0], 64))) return rc;
  if ((rc = tmap_bf16_4d(&tv, v_cache, D, Lmax, Hkv, B, vs[2], vs[1], vs[0], 64))) return rc;

  const size_t n = (size_t)B * Hkv * max_splits * group;
  b2a::DecodeParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_sb = qs[0];
  p.q_sh = qs[1];
  p.seqlens = seqlens;
  p.part_o = static_cast<float*>(workspace);
  p.part_lse = reinterpret_cast<float*>(static_cast<char*>(workspace) + align256(n * D * sizeof(float)));
  p.o = o;
  p.o_sb = o ? os[0] : 0;
  p.o_sh = o ? os[1] : 0;
  if (proj) {
    p.wo = proj->wo;
    p.wo_ld = proj->wo_ld;
    p.dim = proj->dim;
    p.wo_fp32 = proj->wo_fp32 ? 1 : 0;
    p.x = proj->x;
    p.x_sb = proj->x_sb;
    p.x_fp32 = proj->x_fp32 ? 1 : 0;
  }
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.Lmax = Lmax;
  p.group = group;
  p.split_len = split_len;
  p.max_splits = max_splits;
  p.scale_log2 = scale * kLog2e;
  p.out_fp32 = out_fp32 ? 1 : 0;
  p.err = err;
  p.gate = gate;
  if (gate) {
    if (!gs) return B2A_ERR_INVALID_ARG;
    p.g_sb = gs[0];
    p.g_sh = gs[1];
    p.gate_bf16 = gate_bf16 ? 1 : 0;
  }
  rc = b2a::launch_decode(D, tk, tv, p, static_cast<cudaStream_t>(stream));
  if (rc == -3) return B2A_ERR_HEAD_DIM;
  if (rc == -4) return B2A_ERR_INVALID_ARG;
  return rc ? B2A_ERR_LAUNCH : B2A_OK;
}

}  // namespace

namespace b2a {
int* device_error_word() {
  const int dev = current_device();
  return dev < 0 ? nullptr : device_err_ptr(dev);
}
}  // namespace b2a

extern "C" {

const char* b2a_strerror(int code) {
  switch (code) {
    case B2A_OK: return "ok";
    case B2A_ERR_INVALID_ARG: return "invalid argument (null pointer, non-positive size or scale)";
    case B2A_ERR_HEAD_DIM: return "unsupported head_dim";
    case B2A_ERR_GQA: return "query heads must be a multiple of KV heads (group <= 16 for decode)";
    case B2A_ERR_ALIGNMENT: return "pointer or stride not 16-byte aligned / innermost stride not 1";
    case B2A_ERR_TMA: return "TMA tensor map encoding failed";
    case B2A_ERR_LAUNCH: return "kernel launch failed";
    case B2A_ERR_WORKSPACE: return "decode workspace missing or too small";
    case B2A_ERR_DEVICE: return "current CUDA device is not sm_100 (B200)";
    case B2A_ERR_DEVICE_TIMEOUT: return "a kernel's bounded wait ran out (device-side abort)";
    case B2A_ERR_DEVICE_BAD_LEN: return "a sequence length exceeded the KV cache length";
    case B2A_ERR_CUDA: return "CUDA runtime error";
    default: return "unknown b2attn status";
  }
}

int b2a_version(void) { return 100; }

int b2a_decode_default_split(int B, int Hkv, int Lmax) {
  if (B <= 0 || Hkv <= 0 || Lmax <= 0) return 512;
  // Keys x KV heads to stream, assuming caches half full (lengths are on the
  // device), spread over about one wave of CTAs (two per SM on 148 SMs).
  // Measured on B200 (config 4 heads, D = 128): each split CTA pays a fixed
  // cost (pipeline fill, its partial O and LSE, one more input to the
  // combine), so few long splits beat many short ones. A split that leaves a
  // few CTAs for a second, nearly empty wave is much slower: at 16
  // sequences 4096 keys ran 5.9 TB/s, 3072 4.8 and 512 4.6. The measured
  // optima sat at powers of two, hence the rounding. With several waves of
  // work anyway, 2048 is best (128 sequences: 6.85 TB/s against 6.74 at
  // 4096).
  const long long slots = 2LL * 148;
  const long long work = (long long)B * Hkv * ((Lmax + 1) / 2);
  const long long want = work / slots;
  int split = 512;
  while (split < 4096 && (long long)split * 3 / 2 < want) split *= 2;  // nearest power of two
  if (split > 2048 && work / 2048 >= 4 * slots) split = 2048;
  return split;
}

size_t b2a_decode_workspace_bytes(int B, int Hq, int Hkv, int D, int Lmax, int split_len) {
  if (split_len == 0) split_len = b2a_decode_default_split(B, Hkv, Lmax);
  int group = 0, max_splits = 0;
  if (decode_geometry(B, Hq, Hkv, D, Lmax, split_len, &group, &max_splits)) return 0;
  const size_t n = (size_t)B * Hkv * max_splits * group;
  return align256(n * D * sizeof(float)) + align256(n * sizeof(float));
}

int b2a_prefill(const void* q, const void* k, const void* v, void* o, float* lse, int B, int Hq, int Hkv, int Tq,
                int Tk, int D, const long long* qs, const long long* ks, const long long* vs, const long long* os,
                int start_pos, const int* start_pos_per_batch, float scale, int causal, int out_fp32,
                void* stream) {
  return prefill_impl(q, k, v, o, lse, B, Hq, Hkv, Tq, Tk, D, qs, ks, vs, os, start_pos, start_pos_per_batch,
                      scale, causal, out_fp32, nullptr, nullptr, 0, stream);
}

int b2a_prefill_gated(const void* q, const void* k, const void* v, const void* gate, void* o, float* lse, int B,
                      int Hq, int Hkv, int Tq, int Tk, int D, const long long* qs, const long long* ks,
                      const long long* vs, const long long* gs, const long long* os, int gate_bf16,
                      int start_pos, const int* start_pos_per_batch, float scale, int causal, int out_fp32,
                      void* stream) {
  if (!gate || !gs) return B2A_ERR_INVALID_ARG;
  return prefill_impl(q, k, v, o, lse, B, Hq, Hkv, Tq, Tk, D, qs, ks, vs, os, start_pos, start_pos_per_batch,
                      scale, causal, out_fp32, gate, gs, gate_bf16, stream);
}

int b2a_decode(const void* q, const void* k_cache, const void* v_cache, const int* seqlens, void* o, int B,
               int Hq, int Hkv, int Lmax, int D, const long long* qs, const long long* ks, const long long* vs,
               const long long* os, float scale, int split_len, int out_fp32, void* workspace,
               size_t workspace_bytes, void* stream) {
  return decode_impl(q, k_cache, v_cache, seqlens, o, B, Hq, Hkv, Lmax, D, qs, ks, vs, os, scale, split_len,
                     out_fp32, workspace, workspace_bytes, nullptr, nullptr, 0, stream);
}

int b2a_decode_gated(const void* q, const void* k_cache, const void* v_cache, const int* seqlens,
                     const void* gate, void* o, int B, int Hq, int Hkv, int Lmax, int D, const long long* qs,
                     const long long* ks, const long long* vs, const long long* gs, const long long* os,
                     int gate_bf16, float scale, int split_len, int out_fp32, void* workspace,
                     size_t workspace_bytes, void* stream) {
  if (!gate || !gs) return B2A_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(gate) & (gate_bf16 ? 1u : 3u)) return B2A_ERR_ALIGNMENT;
  return decode_impl(q, k_cache, v_cache, seqlens, o, B, Hq, Hkv, Lmax, D, qs, ks, vs, os, scale, split_len,
                     out_fp32, workspace, workspace_bytes, gate, gs, gate_bf16, stream);
}

int b2a_decode_proj(const void* q, const void* k_cache, const void* v_cache, const int* seqlens, const void* wo,
                    long long wo_ld, int wo_fp32, int dim, void* x, long long x_sb, int x_fp32, int B, int Hq,
                    int Hkv, int Lmax, int D, const long long* qs, const long long* ks, const long long* vs,
                    float scale, int split_len, void* workspace, size_t workspace_bytes, void* stream) {
  const DecodeProj proj{wo, wo_ld, dim, wo_fp32, x, x_sb, x_fp32};
  // The attention output is rounded to x's dtype before the projection, as
  // an unfused caller storing it in the model dtype would.
  return decode_impl(q, k_cache, v_cache, seqlens, nullptr, B, Hq, Hkv, Lmax, D, qs, ks, vs, nullptr, scale,
                     split_len, x_fp32 ? 1 : 0, workspace, workspace_bytes, nullptr, nullptr, 0, stream, &proj);
}

int b2a_rope_append(const void* q, const void* k, const void* v, const long long* qs, const long long* ks,
                    const long long* vs, int src_bf16, const void* cos_tab, const void* sin_tab, int max_pos,
                    void* q_out, void* k_cache, void* v_cache, const long long* kcs, const long long* vcs, int B,
                    int T, int Hq, int Hkv, int D, int Lmax, int start_pos, const int* start_pos_per_batch,
                    int* seqlens_out, void* stream) {
  if (!cos_tab || !sin_tab || max_pos <= 0) return B2A_ERR_INVALID_ARG;
  return rope_append_impl(q, k, v, qs, ks, vs, src_bf16, cos_tab, sin_tab, max_pos, D, nullptr, nullptr, 0.f,
                          q_out, k_cache, v_cache, kcs, vcs, B, T, Hq, Hkv, D, Lmax, start_pos,
                          start_pos_per_batch, seqlens_out, stream);
}

int b2a_qk_norm_rope_append(const void* q, const void* k, const void* v, const long long* qs,
                            const long long* ks, const long long* vs, int src_bf16, const void* q_norm,
                            const void* k_norm, float eps, const void* cos_tab, const void* sin_tab,
                            int max_pos, int rope_dim, void* q_out, void* k_cache, void* v_cache,
                            const long long* kcs, const long long* vcs, int B, int T, int Hq, int Hkv, int D,
                            int Lmax, int start_pos, const int* start_pos_per_batch, int* seqlens_out,
                            void* stream) {
  return rope_append_impl(q, k, v, qs, ks, vs, src_bf16, cos_tab, sin_tab, max_pos, rope_dim, q_norm, k_norm,
                          eps, q_out, k_cache, v_cache, kcs, vcs, B, T, Hq, Hkv, D, Lmax, start_pos,
                          start_pos_per_batch, seqlens_out, stream);
}

int b2a_get_device_error(int* status, int clear, void* stream) {
  if (!status) return B2A_ERR_INVALID_ARG;
  const int dev = current_device();
  if (dev < 0) return B2A_ERR_CUDA;
  int* err = device_err_ptr(dev);
  if (!err) return B2A_ERR_CUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int word = 0;
  if (cudaMemcpyAsync(&word, err, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess) return B2A_ERR_CUDA;
  if (clear && cudaMemsetAsync(err, 0, sizeof(int), st) != cudaSuccess) return B2A_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return B2A_ERR_CUDA;
  *status = (word & b2a::kErrWaitTimeout) ? B2A_ERR_DEVICE_TIMEOUT
            : (word & b2a::kErrBadArgs)   ? B2A_ERR_DEVICE_BAD_LEN
                                          : B2A_OK;
  return B2A_OK;
}

}  // extern "C"
