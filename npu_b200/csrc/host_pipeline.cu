// Host-buffer prefill (b2a_prefill_host): the call surface of the reference's
// NpuAttention.run_batch (npu/fa.py:206-323), whose inputs and result live in
// host memory (it packs and syncs the Q/K/V buffers to the device,
// npu/fa.py:266-311, runs, and syncs and reads O back, :313-323). The problem
// is cut into chunks of (batch, KV head) units; each chunk's Q/K/V go
// host -> device on one copy stream, the prefill kernel runs on the caller's
// stream, and the output goes device -> host on a second copy stream. Two
// device slots alternate between chunks, so chunk i+1's upload and chunk
// i-1's download run while chunk i computes; upload and download use the two
// directions of the host link at the same time.
//
// Stream protocol (all waits are stream-side, nothing blocks the host):
//   fork        recorded on the caller's stream; both copy streams wait on it
//   in_ready[s] upload of the chunk in slot s done      -> compute waits
//   comp[s]     kernel of the chunk in slot s done      -> download waits,
//                                                          next upload to s waits
//   out_done[s] download of the chunk in slot s done    -> next kernel into s waits
//   join        the caller's stream waits on the last download (and upload),
//               so work queued after the call sees the whole output.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <vector>

#include "b2attn.h"

namespace {

constexpr int kMaxDev = 64;
constexpr int kSlots = 2;

struct CopyEngines {
  bool ready = false;
  cudaStream_t up = nullptr, down = nullptr;
  cudaEvent_t fork = nullptr, up_last = nullptr;
  cudaEvent_t in_ready[kSlots] = {}, comp[kSlots] = {}, out_done[kSlots] = {};
};

std::mutex g_host_mu[kMaxDev];
CopyEngines g_eng[kMaxDev];

int engines(int dev, CopyEngines** out) {
  CopyEngines& e = g_eng[dev];
  if (!e.ready) {
    const unsigned ef = cudaEventDisableTiming;
    if (cudaStreamCreateWithFlags(&e.up, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&e.down, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&e.fork, ef) != cudaSuccess ||
        cudaEventCreateWithFlags(&e.up_last, ef) != cudaSuccess)
      return B2A_ERR_CUDA;
    for (int s = 0; s < kSlots; ++s)
      if (cudaEventCreateWithFlags(&e.in_ready[s], ef) != cudaSuccess ||
          cudaEventCreateWithFlags(&e.comp[s], ef) != cudaSuccess ||
          cudaEventCreateWithFlags(&e.out_done[s], ef) != cudaSuccess)
        return B2A_ERR_CUDA;
    e.ready = true;
  }
  *out = &e;
  return B2A_OK;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// A chunk is either whole batches [b0, b0 + nb) (nh == Hkv) or KV heads
// [h0, h0 + nh) of the single batch b0 (nb == 1).
struct Chunk {
  int b0, nb, h0, nh;
};

struct Plan {
  std::vector<Chunk> chunks;
  long long max_units = 0;  // largest chunk in (batch, KV head) units
  size_t q_bytes = 0, kv_bytes = 0, o_bytes = 0, slot_bytes = 0, pos_off = 0, total = 0;
};

bool make_plan(int B, int Hq, int Hkv, int Tq, int Tk, int D, int out_fp32, int n_chunks, Plan* pl) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Tq <= 0 || Tk < 0 || n_chunks < 0 || Hq % Hkv) return false;
  if (D != 64 && D != 128 && D != 256) return false;
  const long long units = (long long)B * Hkv;
  if (n_chunks == 0) n_chunks = 32;
  long long per = (units + n_chunks - 1) / n_chunks;
  pl->chunks.clear();
  if (per >= Hkv) {
    const int nb = (int)((per + Hkv - 1) / Hkv);
    for (int b = 0; b < B; b += nb) pl->chunks.push_back({b, nb < B - b ? nb : B - b, 0, Hkv});
    // Taper: the last chunk's kernel and download run after every upload is
    // done, with nothing left to overlap them. Split its last batch into one
    // chunk per KV head, so only a small piece remains in that tail.
    if (pl->chunks.size() > 1 && Hkv > 1) {
      Chunk& last = pl->chunks.back();
      const int bl = last.b0 + last.nb - 1;
      if (--last.nb == 0) pl->chunks.pop_back();
      for (int h = 0; h < Hkv; ++h) pl->chunks.push_back({bl, 1, h, 1});
    }
  } else {
    const int nh = (int)per;
    for (int b = 0; b < B; ++b)
      for (int h = 0; h < Hkv; h += nh) pl->chunks.push_back({b, 1, h, nh < Hkv - h ? nh : Hkv - h});
  }
  pl->max_units = 0;
  for (const Chunk& c : pl->chunks) {
    const long long u = (long long)c.nb * c.nh;
    if (u > pl->max_units) pl->max_units = u;
  }
  const long long G = Hq / Hkv;
  pl->q_bytes = align256((size_t)pl->max_units * G * Tq * D * 2);
  pl->kv_bytes = align256((size_t)pl->max_units * (Tk > 0 ? Tk : 1) * D * 2);
  pl->o_bytes = align256((size_t)pl->max_units * G * Tq * D * (out_fp32 ? 4 : 2));
  pl->slot_bytes = pl->q_bytes + 2 * pl->kv_bytes + pl->o_bytes;
  pl->pos_off = kSlots * pl->slot_bytes;
  pl->total = pl->pos_off + align256((size_t)B * sizeof(int));
  return true;
}

}  // namespace

extern "C" {

size_t b2a_prefill_host_workspace_bytes(int B, int Hq, int Hkv, int Tq, int Tk, int D, int out_fp32,
                                        int n_chunks) {
  Plan pl;
  return make_plan(B, Hq, Hkv, Tq, Tk, D, out_fp32, n_chunks, &pl) ? pl.total : 0;
}

int b2a_prefill_host(const void* q, const void* k, const void* v, void* o, int B, int Hq, int Hkv, int Tq,
                     int Tk, int D, int start_pos, const int* start_pos_per_batch, float scale, int causal,
                     int out_fp32, int n_chunks, void* workspace, size_t workspace_bytes, void* stream) {
  Plan pl;
  if (!make_plan(B, Hq, Hkv, Tq, Tk, D, out_fp32, n_chunks, &pl)) {
    if (D != 64 && D != 128 && D != 256) return B2A_ERR_HEAD_DIM;
    if (Hq > 0 && Hkv > 0 && Hq % Hkv) return B2A_ERR_GQA;
    return B2A_ERR_INVALID_ARG;
  }
  if (!q || !o || (Tk > 0 && (!k || !v))) return B2A_ERR_INVALID_ARG;
  if (!(scale > 0.f)) return B2A_ERR_INVALID_ARG;
  if (!workspace || workspace_bytes < pl.total || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return B2A_ERR_WORKSPACE;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return B2A_ERR_CUDA;

  std::lock_guard<std::mutex> lk(g_host_mu[dev]);
  CopyEngines* e = nullptr;
  int rc = engines(dev, &e);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  int* pos_dev = reinterpret_cast<int*>(ws + pl.pos_off);
  const long long G = Hq / Hkv;
  const size_t esz_o = out_fp32 ? 4 : 2;
  const size_t q_unit = (size_t)G * Tq * D * 2, kv_unit = (size_t)Tk * D * 2, o_unit = (size_t)G * Tq * D * esz_o;

  bool ok = cudaEventRecord(e->fork, st) == cudaSuccess && cudaStreamWaitEvent(e->up, e->fork, 0) == cudaSuccess &&
            cudaStreamWaitEvent(e->down, e->fork, 0) == cudaSuccess;
  const bool any_whole = pl.chunks[0].nh == Hkv;  // whole-batch chunks come first
  if (ok && start_pos_per_batch && any_whole)
    ok = cudaMemcpyAsync(pos_dev, start_pos_per_batch, (size_t)B * sizeof(int), cudaMemcpyHostToDevice, e->up) ==
         cudaSuccess;

  const int n = (int)pl.chunks.size();
  auto upload = [&](int i) -> bool {
    const Chunk& c = pl.chunks[i];
    const int s = i % kSlots;
    char* slot = ws + (size_t)s * pl.slot_bytes;
    const size_t u0 = (size_t)c.b0 * Hkv + c.h0, nu = (size_t)c.nb * c.nh;
    if (i >= kSlots && cudaStreamWaitEvent(e->up, e->comp[s], 0) != cudaSuccess) return false;
    if (cudaMemcpyAsync(slot, static_cast<const char*>(q) + u0 * q_unit, nu * q_unit, cudaMemcpyHostToDevice,
                        e->up) != cudaSuccess)
      return false;
    if (Tk > 0) {
      if (cudaMemcpyAsync(slot + pl.q_bytes, static_cast<const char*>(k) + u0 * kv_unit, nu * kv_unit,
                          cudaMemcpyHostToDevice, e->up) != cudaSuccess ||
          cudaMemcpyAsync(slot + pl.q_bytes + pl.kv_bytes, static_cast<const char*>(v) + u0 * kv_unit,
                          nu * kv_unit, cudaMemcpyHostToDevice, e->up) != cudaSuccess)
        return false;
    }
    return cudaEventRecord(e->in_ready[s], e->up) == cudaSuccess;
  };

  if (ok) ok = upload(0);
  for (int i = 0; ok && i < n; ++i) {
    // Queue the next upload first: with pageable host memory a copy call
    // returns only when its transfer is done, and this order still keeps
    // one upload ahead of the kernel.
    if (i + 1 < n && !(ok = upload(i + 1))) break;
    const Chunk& c = pl.chunks[i];
    const int s = i % kSlots;
    char* slot = ws + (size_t)s * pl.slot_bytes;
    const size_t u0 = (size_t)c.b0 * Hkv + c.h0, nu = (size_t)c.nb * c.nh;
    if (cudaStreamWaitEvent(st, e->in_ready[s], 0) != cudaSuccess ||
        (i >= kSlots && cudaStreamWaitEvent(st, e->out_done[s], 0) != cudaSuccess)) {
      ok = false;
      break;
    }
    const int hq = c.nh * (int)G;
    const long long qs_c[3] = {(long long)hq * Tq * D, (long long)Tq * D, D};
    const long long ks_c[3] = {(long long)c.nh * Tk * D, (long long)Tk * D, D};
    int sp = start_pos;
    const int* sp_arr = nullptr;
    if (start_pos_per_batch) {
      if (c.nh == Hkv)
        sp_arr = pos_dev + c.b0;
      else
        sp = start_pos_per_batch[c.b0];
    }
    rc = b2a_prefill(slot, Tk > 0 ? slot + pl.q_bytes : nullptr, Tk > 0 ? slot + pl.q_bytes + pl.kv_bytes : nullptr,
                     slot + pl.q_bytes + 2 * pl.kv_bytes, nullptr, c.nb, hq, c.nh, Tq, Tk, D, qs_c, ks_c, ks_c,
                     qs_c, sp, sp_arr, scale, causal, out_fp32, st);
    if (rc) break;
    if (cudaEventRecord(e->comp[s], st) != cudaSuccess || cudaStreamWaitEvent(e->down, e->comp[s], 0) != cudaSuccess ||
        cudaMemcpyAsync(static_cast<char*>(o) + u0 * o_unit, slot + pl.q_bytes + 2 * pl.kv_bytes, nu * o_unit,
                        cudaMemcpyDeviceToHost, e->down) != cudaSuccess ||
        cudaEventRecord(e->out_done[s], e->down) != cudaSuccess) {
      ok = false;
      break;
    }
  }
  // Join both copy streams back into the caller's stream, also on failure,
  // so no copy into or out of the workspace outlives the call's stream order.
  const bool joined = cudaEventRecord(e->up_last, e->up) == cudaSuccess &&
                      cudaStreamWaitEvent(st, e->up_last, 0) == cudaSuccess &&
                      cudaEventRecord(e->fork, e->down) == cudaSuccess &&
                      cudaStreamWaitEvent(st, e->fork, 0) == cudaSuccess;
  if (rc) return rc;
  return ok && joined ? B2A_OK : B2A_ERR_CUDA;
}

}  // extern "C"
