/*
 * b2attn — C ABI of the B200 (sm_100a) attention engine.
 *
 * This is the boundary that replaces the reference's FlashAttention-2 device
 * path: the host wrapper NpuAttention.run_batch (npu/fa.py:206-323), which
 * packs Q/K/V, dispatches the AIE kernel entry points attn_block /
 * attn_finalise (npu/fa_kernel.cc:68-217, :219-227) and reads the output back.
 * Those entry points keep per-dispatch running state in static tile memory
 * (npu/fa_kernel.cc:59-64); every function here is instead stateless,
 * re-entrant and ordered on the caller's CUDA stream.
 *
 * Conventions
 *  - All tensor pointers are caller-owned device memory; nothing here
 *    allocates on the call path. Decode scratch comes from the caller
 *    (b2a_decode_workspace_bytes).
 *  - Element types: Q/K/V and the KV cache are bf16. Outputs are bf16 or fp32
 *    (out_fp32). Innermost (head_dim) stride is 1; every other stride is given
 *    in ELEMENTS and must be a multiple of 8 (16 bytes). Base pointers must be
 *    16-byte aligned.
 *  - `stream` is a cudaStream_t (NULL = legacy default stream).
 *  - Return value: B2A_OK (0) or a negative B2A_ERR_* code; no C++ exception
 *    crosses this boundary. Device-side faults that kernels detect (a bounded
 *    wait that ran out, a sequence length larger than the cache) are reported
 *    through b2a_get_device_error.
 *  - GQA: query head h reads KV head h / (Hq / Hkv) — the repeat_interleave
 *    mapping of smollm.py:205-207 and qwen/forward.py:194-197.
 */
#ifndef B2ATTN_H
#define B2ATTN_H

#include <stddef.h>

#if defined(__GNUC__)
#define B2A_API __attribute__((visibility("default")))
#else
#define B2A_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  B2A_OK = 0,
  B2A_ERR_INVALID_ARG = -1,      /* null pointer, non-positive size, scale <= 0 */
  B2A_ERR_HEAD_DIM = -2,         /* head_dim not supported by this entry point */
  B2A_ERR_GQA = -3,              /* Hq not a multiple of Hkv, or group too large */
  B2A_ERR_ALIGNMENT = -4,        /* pointer or stride not 16-byte aligned */
  B2A_ERR_TMA = -5,              /* tensor-map encoding failed or unavailable */
  B2A_ERR_LAUNCH = -6,           /* kernel launch failed (cudaGetLastError) */
  B2A_ERR_WORKSPACE = -7,        /* decode workspace missing or too small */
  B2A_ERR_DEVICE = -8,           /* current device is not sm_100 */
  B2A_ERR_DEVICE_TIMEOUT = -9,   /* a kernel's bounded wait ran out */
  B2A_ERR_DEVICE_BAD_LEN = -10,  /* a sequence length exceeded the cache */
  B2A_ERR_CUDA = -11             /* another CUDA runtime error */
};

/* Human-readable text for a status code. Never NULL. */
B2A_API const char* b2a_strerror(int code);

/* ABI version (major * 100 + minor). */
B2A_API int b2a_version(void);

/*
 * Causal (or full) GQA attention prefill.
 * Replaces: NpuAttention.run_batch (npu/fa.py:206-323) driving attn_block /
 * attn_finalise (npu/fa_kernel.cc:68-227); arithmetic follows
 * flash_attention_ref (npu/fa_ref.py:42-131).
 *
 *   q   [B, Hq,  Tq, D]  strides q_strides  = {batch, head, row}
 *   k   [B, Hkv, Tk, D]  strides k_strides
 *   v   [B, Hkv, Tk, D]  strides v_strides
 *   o   [B, Hq,  Tq, D]  strides o_strides  (bf16, or fp32 if out_fp32)
 *   lse optional [B, Hq, Tq] fp32 contiguous: natural-log sum of
 *       exp(scale * s) over unmasked keys (-inf for fully masked rows).
 *
 * Query row r sits at absolute position start + r, where start is
 * start_pos_per_batch[b] (device int32 array) when that pointer is non-NULL,
 * else start_pos. With causal != 0, key c is masked iff c > start + r
 * (npu/fa_ref.py:57-60, :102-108). Rows with no unmasked key output 0
 * (npu/fa_ref.py:112-128). scale is the softmax scale (1/sqrt(D) in the
 * reference, npu/fa_ref.py:68). Tk may be 0: every row is then 0 and k / v
 * are not read (they may be NULL).
 * Supported D: 64, 128, 256.
 */
B2A_API int b2a_prefill(const void* q, const void* k, const void* v, void* o, float* lse, int B, int Hq, int Hkv,
                int Tq, int Tk, int D, const long long* q_strides, const long long* k_strides,
                const long long* v_strides, const long long* o_strides, int start_pos,
                const int* start_pos_per_batch, float scale, int causal, int out_fp32, void* stream);

/*
 * Bytes of caller-provided device scratch that b2a_decode needs for the given
 * geometry and split length (0 split_len = the default chosen by b2a_decode).
 */
B2A_API size_t b2a_decode_workspace_bytes(int B, int Hq, int Hkv, int D, int Lmax, int split_len);

/* The split length b2a_decode uses when called with split_len = 0. */
B2A_API int b2a_decode_default_split(int B, int Hkv, int Lmax);

/*
 * Single-token decode attention over a contiguous KV cache (split-KV
 * flash-decode + log-sum-exp combine, two launches on `stream`).
 * Replaces: the T=1 attention step of smollm.py:222-234 (and the bucketed
 * decode route through run_batch, smollm.py:144,212-221).
 *
 *   q        [B, Hq, D]        strides q_strides = {batch, head}
 *   k_cache  [B, Hkv, Lmax, D] strides k_strides = {batch, head, position}
 *   v_cache  [B, Hkv, Lmax, D] strides v_strides
 *   seqlens  [B] int32 device  keys 0 .. seqlens[b]-1 are attended (no mask)
 *   o        [B, Hq, D]        strides o_strides = {batch, head}
 *
 * split_len: keys per split CTA, a multiple of 64 (0 = default).
 * Supported D: 64, 128, 256; Hq / Hkv <= 16.
 */
B2A_API int b2a_decode(const void* q, const void* k_cache, const void* v_cache, const int* seqlens, void* o, int B,
               int Hq, int Hkv, int Lmax, int D, const long long* q_strides, const long long* k_strides,
               const long long* v_strides, const long long* o_strides, float scale, int split_len,
               int out_fp32, void* workspace, size_t workspace_bytes, void* stream);

/* Size of the fixed device scratch buffer behind b2a_decode_noalloc. */
#define B2A_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)

/*
 * b2a_decode without caller scratch, for callers that cannot allocate device
 * memory (hosts that reserve all device memory up front and forbid later
 * cudaMalloc/cudaFree, plugin/FFI callers holding only input and output
 * pointers). No counterpart in the reference.
 * Same arguments and results as b2a_decode minus the workspace. Scratch is a
 * device array of B2A_NOALLOC_SCRATCH_BYTES inside this library, held by every
 * GPU that loads it until exit; problems needing more return
 * B2A_ERR_WORKSPACE (use a larger split_len, or b2a_decode). The first call on
 * a device looks up the array's device address (cudaGetSymbolAddress): make
 * it outside any stream capture. All calls on a device share the buffer, so
 * calls that overlap on the GPU race; nothing in it needs to start at zero.
 */
B2A_API int b2a_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, const int* seqlens,
                               void* o, int B, int Hq, int Hkv, int Lmax, int D, const long long* q_strides,
                               const long long* k_strides, const long long* v_strides,
                               const long long* o_strides, float scale, int split_len, int out_fp32,
                               void* stream);

/*
 * Read (and optionally clear) the device error word the kernels set on the
 * current device. Synchronises `stream`. *status receives B2A_OK,
 * B2A_ERR_DEVICE_TIMEOUT or B2A_ERR_DEVICE_BAD_LEN.
 */
B2A_API int b2a_get_device_error(int* status, int clear, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B2ATTN_H */
