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
 *  - All tensor pointers are caller-owned device memory (b2a_prefill_host:
 *    host memory, plus a device workspace); nothing here allocates on the
 *    call path. Scratch comes from the caller (b2a_decode_workspace_bytes,
 *    b2a_prefill_host_workspace_bytes).
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
 * With the environment variable B2A_PREFILL_SM_PAIRS set to a positive row
 * count, head dim 128 queries with an even GQA group and at least that many
 * rows run on SM pairs (a two-CTA cluster per 256 rows of two query heads,
 * tcgen05.mma.cta_group::2): same results bit for bit, measured slower than
 * the default one-SM kernel, so off unless asked for. Read on every call.
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

/*
 * The split length b2a_decode uses when called with split_len = 0: keys per
 * split CTA such that the estimated work (B x Hkv x Lmax / 2 keys, since the
 * lengths are on the device) fills about one wave of CTAs, rounded to a
 * power of two in [512, 4096], and 2048 when that still leaves several
 * waves. Pass an explicit split_len when the lengths are known to be far
 * from half the cache.
 */
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

/*
 * b2a_prefill / b2a_decode with the gated-attention epilogue of Qwen3.5/3.6
 * (qwen/forward.py:223-226): the output is attention * sigmoid(gate), fused
 * into the kernels' output stores (no extra pass over O).
 *   prefill: gate [B, Hq, Tq, D], element strides gate_strides = {batch,
 *            head, row}, 16-byte aligned, strides multiples of 16 bytes;
 *   decode:  gate [B, Hq, D], gate_strides = {batch, head}.
 * gate_bf16: 1 for bf16, 0 for fp32. The q projection of the reference holds
 * [q_h | gate_h] per head, so the gate is usually a strided view of it
 * (head stride 2 D). All other arguments as the ungated calls.
 */
B2A_API int b2a_prefill_gated(const void* q, const void* k, const void* v, const void* gate, void* o, float* lse,
                              int B, int Hq, int Hkv, int Tq, int Tk, int D, const long long* q_strides,
                              const long long* k_strides, const long long* v_strides,
                              const long long* gate_strides, const long long* o_strides, int gate_bf16,
                              int start_pos, const int* start_pos_per_batch, float scale, int causal,
                              int out_fp32, void* stream);

B2A_API int b2a_decode_gated(const void* q, const void* k_cache, const void* v_cache, const int* seqlens,
                             const void* gate, void* o, int B, int Hq, int Hkv, int Lmax, int D,
                             const long long* q_strides, const long long* k_strides, const long long* v_strides,
                             const long long* gate_strides, const long long* o_strides, int gate_bf16,
                             float scale, int split_len, int out_fp32, void* workspace, size_t workspace_bytes,
                             void* stream);

/*
 * b2a_decode followed by the output projection and residual add, fused into
 * the combine kernel: x[b, :] += o_b @ wo^T, where o_b is sequence b's
 * attention output [Hq * D] (rounded to x's dtype) and wo [dim, Hq * D] the
 * output projection weight (F.linear layout, row stride wo_ld elements, fp32
 * with wo_fp32 = 1 else bf16; 16-byte aligned, wo_ld a multiple of 16 bytes).
 * x: the residual stream [B, dim] (row stride x_sb elements, fp32 with
 * x_fp32 = 1 else bf16), updated in place; the attention output itself is not
 * stored. Replaces: the attention core plus `x = x + wo(o)` of the T=1 layer
 * step (smollm.py:222-236, where the output projection follows attention at
 * :235-236). The combine runs per (block of 32 outputs, sequence): every
 * output of x has one writer and a fixed summation order, so results are
 * reproducible. Hq * D <= ~51k (one sequence's attention output in shared
 * memory). Workspace as b2a_decode.
 */
B2A_API int b2a_decode_proj(const void* q, const void* k_cache, const void* v_cache, const int* seqlens,
                            const void* wo, long long wo_ld, int wo_fp32, int dim, void* x, long long x_sb,
                            int x_fp32, int B, int Hq, int Hkv, int Lmax, int D, const long long* q_strides,
                            const long long* k_strides, const long long* v_strides, float scale, int split_len,
                            void* workspace, size_t workspace_bytes, void* stream);

/* Size of the fixed device scratch buffer behind b2a_decode_noalloc. */
#define B2A_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)

/*
 * b2a_decode without caller scratch, for callers that cannot allocate device
 * memory (hosts that reserve all device memory up front and forbid later
 * cudaMalloc/cudaFree, plugin/FFI callers holding only input and output
 * pointers). No counterpart in the reference.
 * Same arguments and results as b2a_decode minus the workspace. Scratch is a
 * device array of B2A_NOALLOC_SCRATCH_BYTES inside this library, held by every
 * GPU that loads it until exit. With split_len = 0 the default split length
 * is doubled until the partial results fit; problems that need more even with
 * one split per sequence (or with the caller's split_len) return
 * B2A_ERR_WORKSPACE before any launch (use a larger split_len, or b2a_decode).
 * A non-sm_100 device returns B2A_ERR_DEVICE. The first call in a device's
 * context looks up the array's device address (cudaGetSymbolAddress): make it
 * outside any stream capture; a new context (after cudaDeviceReset) is
 * detected and looked up again. All calls on a device share the buffer, so
 * calls that overlap on the GPU race; nothing in it needs to start at zero.
 */
B2A_API int b2a_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, const int* seqlens,
                               void* o, int B, int Hq, int Hkv, int Lmax, int D, const long long* q_strides,
                               const long long* k_strides, const long long* v_strides,
                               const long long* o_strides, float scale, int split_len, int out_fp32,
                               void* stream);

/*
 * Fused RoPE + in-place KV-cache append, one launch per layer and step.
 * Replaces: the per-step projection transposes, the two apply_rope calls,
 * torch.cat of the layer cache and repeat_interleave of smollm.py:186-208
 * (and the Tk buckets of smollm.py:17-20,144): the cache is a preallocated
 * device buffer written in place and read by b2a_prefill / b2a_decode
 * without expanding GQA heads.
 *
 *   q, k, v  [B, T, H, D] views (H = Hq, Hkv, Hkv), element strides
 *            {batch, token, head} in q/k/v_strides, D contiguous; fp32
 *            (src_bf16 = 0) or bf16 (src_bf16 = 1); 16-byte aligned, strides
 *            multiples of 16 bytes
 *   cos_tab, sin_tab [max_pos, D] contiguous, same dtype as q/k/v: the
 *            model's rotary tables (build_rope_cache, smollm.py:45-50)
 *   q_out    [B, Hq, T, D] bf16 contiguous: q rotated (the attention
 *            kernels' query layout)
 *   k_cache, v_cache [B, Hkv, Lmax, D] bf16, element strides {batch, head,
 *            position} in k/v_cache_strides (multiples of 8): rows
 *            p_b .. p_b + T - 1 receive k rotated and v, where p_b =
 *            start_pos_per_batch[b] (device int32) or start_pos
 *   seqlens_out [B] int32 device, optional: set to p_b + T
 *
 * Rotation is rotate-half (smollm.py:53-58), computed op by op in the source
 * dtype as the reference does, then rounded to bf16. Positions must satisfy
 * 0 <= p_b and p_b + T <= min(Lmax, max_pos): checked on the host for a
 * scalar start_pos (B2A_ERR_INVALID_ARG), on the device for per-batch
 * positions (rows out of range are skipped and the device error word reports
 * B2A_ERR_DEVICE_BAD_LEN). Supported D: 64, 128, 256.
 */
B2A_API int b2a_rope_append(const void* q, const void* k, const void* v, const long long* q_strides,
                            const long long* k_strides, const long long* v_strides, int src_bf16,
                            const void* cos_tab, const void* sin_tab, int max_pos, void* q_out, void* k_cache,
                            void* v_cache, const long long* k_cache_strides, const long long* v_cache_strides,
                            int B, int T, int Hq, int Hkv, int D, int Lmax, int start_pos,
                            const int* start_pos_per_batch, int* seqlens_out, void* stream);

/*
 * b2a_rope_append with the gated-attention prologue of Qwen3.5/3.6
 * (qwen/forward.py:178-204): each q and k head is RMS-normalised over its D
 * lanes with the weights q_norm / k_norm ([D], source dtype; either may be
 * null to skip; fp32 statistics, (x * rsqrt(mean(x^2) + eps)) * w as
 * qwen/forward.py:58-61) and then rotated on its first rope_dim lanes only
 * (partial rotate-half, qwen/forward.py:81-95; cos_tab/sin_tab are
 * [max_pos, rope_dim]). rope_dim is 0 (no rotation) or a power of two in
 * [16, D]. q may be a strided view of the [q_h | gate_h] per-head layout of
 * the gated q projection (head stride 2 D). Sources need 16-byte alignment
 * and strides that are multiples of 16 bytes; caches and q_out likewise.
 * Otherwise as b2a_rope_append (which is this call with rope_dim = D and no
 * norms).
 */
B2A_API int b2a_qk_norm_rope_append(const void* q, const void* k, const void* v, const long long* q_strides,
                                    const long long* k_strides, const long long* v_strides, int src_bf16,
                                    const void* q_norm, const void* k_norm, float eps, const void* cos_tab,
                                    const void* sin_tab, int max_pos, int rope_dim, void* q_out, void* k_cache,
                                    void* v_cache, const long long* k_cache_strides,
                                    const long long* v_cache_strides, int B, int T, int Hq, int Hkv, int D,
                                    int Lmax, int start_pos, const int* start_pos_per_batch, int* seqlens_out,
                                    void* stream);

/*
 * Prefill with inputs and result in HOST memory: the call surface of the
 * reference's NpuAttention.run_batch (npu/fa.py:206-323), which takes host
 * Q/K/V stacks and returns the host O stack.
 *
 *   q   [B, Hq,  Tq, D]  bf16, contiguous, host memory
 *   k   [B, Hkv, Tk, D]  bf16, contiguous, host memory (may be NULL if Tk == 0)
 *   v   [B, Hkv, Tk, D]
 *   o   [B, Hq,  Tq, D]  bf16 (fp32 if out_fp32), contiguous, host memory
 *   start_pos_per_batch  optional HOST int32 [B]; else start_pos for all
 *   workspace  device memory of b2a_prefill_host_workspace_bytes(...) bytes,
 *              256-byte aligned
 *
 * Same arithmetic, masking and results as b2a_prefill. The problem is cut
 * into n_chunks pieces of (batch, KV head) units (0 = 32): whole batches
 * when there are enough, else KV heads of one batch. Each piece is copied in
 * on a library-owned copy stream, computed on `stream`, and copied out on a
 * second copy stream, with two workspace slots alternating, so uploads,
 * kernels and downloads of neighbouring pieces overlap. The call is
 * asynchronous and ordered on `stream`: it returns once everything is
 * queued, and work queued on `stream` afterwards (a synchronize, an event)
 * sees the complete o. Host buffers must stay valid and unmodified until
 * then. Page-locked host memory is needed for the copies to overlap;
 * pageable buffers give the same result with the copies serialised.
 * Concurrent calls on one device are serialised while queueing and must not
 * share a workspace unless ordered on one stream.
 */
B2A_API size_t b2a_prefill_host_workspace_bytes(int B, int Hq, int Hkv, int Tq, int Tk, int D, int out_fp32,
                                                int n_chunks);
B2A_API int b2a_prefill_host(const void* q, const void* k, const void* v, void* o, int B, int Hq, int Hkv, int Tq,
                             int Tk, int D, int start_pos, const int* start_pos_per_batch, float scale, int causal,
                             int out_fp32, int n_chunks, void* workspace, size_t workspace_bytes, void* stream);

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
