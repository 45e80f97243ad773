// Allocation-free C entry point for split-KV paged decode attention.
//
// This entry point has no counterpart in the reference; it exists for callers
// of this library that cannot allocate GPU memory themselves: code running
// while a CUDA stream is being captured by someone else's graph, runtimes
// that hand out only caller-owned buffers (custom allocators, plugin hosts,
// other languages calling through the C ABI), or hot paths where a
// cudaMalloc/cudaFree would synchronise the device.  The torch-facing
// `attn_decode` takes its split-KV scratch from the caller's workspace tensor;
// this variant keeps that scratch in a fixed device array instead, so it
// allocates nothing and needs no torch.
//
// Scratch: one file-scope device array of kNoAllocScratchFloats floats
// (16 MiB).  Every GPU that loads the library holds it until the process
// exits.  A call needs B * Hq * splits * (D + 1) floats of it; larger requests
// are rejected (return code 2, see mb_noalloc_last_error()).
//
// Sharing: all calls on a device use the same array and it keeps the last
// call's contents.  Every (sequence, head, split) partial and its log-sum-exp
// is written by the split kernel before the combine kernel reads it, so
// nothing has to start at zero.  Calls whose kernels overlap on the GPU (two
// streams, or two host threads) race on the array: serialise them.
//
// Set-up: the first call on a device resolves the array's device address with
// cudaGetSymbolAddress while that device is current, and caches it.  Make that
// first call before any stream capture begins.  In host code the array's name
// is only a host-side stand-in, never a device pointer, so the resolved
// address is what the kernels receive.
#include <cuda_runtime.h>
#include <cstdio>
#include <mutex>
#include "attn_decode.cuh"
#include "mb_noalloc.h"

namespace {

constexpr size_t kNoAllocScratchFloats = size_t(4) << 20;  // 16 MiB
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

constexpr int kMaxDevices = 64;
float* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_mu;
thread_local char g_err[256] = "";

int fail(int code, const char* msg) {
  std::snprintf(g_err, sizeof(g_err), "%s", msg);
  return code;
}

// Device address of the scratch array for the current device.
float* scratch_for_current_device(int* rc) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *rc = fail(4, "mb_attn_decode_noalloc: no current CUDA device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      *rc = fail(4, "mb_attn_decode_noalloc: cudaGetSymbolAddress failed for the scratch array");
      return nullptr;
    }
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  return g_scratch_ptr[dev];
}

template <int D, int G>
void launch_split(dim3 grid, cudaStream_t st, const __nv_bfloat16* q, const __nv_bfloat16* k,
                  const __nv_bfloat16* v, const int* bt, const int* cl, __nv_bfloat16* out, float* po, float* pl,
                  int Hkv, int mbk, int splits, float sl2) {
  mb::attn_decode_kernel<D, G><<<grid, mb::kWarps * 32, 0, st>>>(q, k, v, bt, cl, out, po, pl, Hkv, mbk, splits, sl2);
}

}  // namespace

extern "C" {

// Human-readable reason for the last non-zero return code on this thread.
__attribute__((visibility("default"))) const char* mb_noalloc_last_error() { return g_err; }

// Largest scratch request (in floats) the entry point accepts.
__attribute__((visibility("default"))) size_t mb_attn_decode_noalloc_max_scratch_floats() {
  return kNoAllocScratchFloats;
}

// Paged decode attention, split-KV, with no allocation.
//   q          [B, Hq, D] bf16           out  [B, Hq, D] bf16
//   k cache [num_blocks, Hkv, 16, D], v cache [num_blocks, Hkv, D, 16] bf16
//   block_tables [B, max_blocks] int32,  ctx_lens [B] int32
// All pointers are device pointers owned by the caller; `stream` is a
// cudaStream_t (0 = legacy default stream).  Returns 0 on success, 1 for bad
// arguments, 2 when B*Hq*splits*(D+1) exceeds the scratch array, 3 for a
// head_dim / group size without a compiled kernel, 4 for a CUDA error.
// Every ctx_lens[b] must be <= 16 * max_blocks; a longer one is clamped on the
// device to the tokens its block-table row addresses.
__attribute__((visibility("default"))) int mb_attn_decode_noalloc(
    const void* q, const void* k_cache, const void* v_cache, const int* block_tables, const int* ctx_lens, void* out,
    int B, int Hq, int Hkv, int D, int max_blocks, int splits, float scale, void* stream) {
  if (!q || !k_cache || !v_cache || !block_tables || !ctx_lens || !out || B <= 0 || Hq <= 0 || Hkv <= 0 ||
      Hq % Hkv != 0 || max_blocks <= 0 || splits <= 0)
    return fail(1, "mb_attn_decode_noalloc: invalid argument");
  if (D != 64 && D != 128 && D != 256) return fail(3, "mb_attn_decode_noalloc: head_dim must be 64, 128 or 256");
  {
    // an error left by earlier, unrelated work on this thread is reported as such (and cleared),
    // so that it is not mistaken for this call's launch failure below
    const cudaError_t pending = cudaGetLastError();
    if (pending != cudaSuccess) {
      char m[200];
      std::snprintf(m, sizeof(m), "mb_attn_decode_noalloc: CUDA error pending before the call: %s",
                    cudaGetErrorString(pending));
      return fail(4, m);
    }
  }
  const size_t need = (size_t)B * Hq * splits * (D + 1);
  if (need > kNoAllocScratchFloats) {
    char m[160];
    std::snprintf(m, sizeof(m), "mb_attn_decode_noalloc: needs %zu scratch floats, maximum is %zu", need,
                  kNoAllocScratchFloats);
    return fail(2, m);
  }
  int rc = 0;
  float* scratch = scratch_for_current_device(&rc);
  if (!scratch) return rc;
  float* po = scratch;
  float* pl = scratch + (size_t)B * Hq * splits * D;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int G = Hq / Hkv;
  const float sl2 = scale * 1.4426950408889634f;
  auto pq = static_cast<const __nv_bfloat16*>(q);
  auto pk = static_cast<const __nv_bfloat16*>(k_cache);
  auto pv = static_cast<const __nv_bfloat16*>(v_cache);
  auto pout = static_cast<__nv_bfloat16*>(out);
  dim3 grid(B, Hkv, splits);
  bool ok = true;
#define MB_NA(DD, GG) \
  else if (D == DD && G == GG) launch_split<DD, GG>(grid, st, pq, pk, pv, block_tables, ctx_lens, pout, po, pl, Hkv, max_blocks, splits, sl2);
  if (false) {
  }
  MB_NA(128, 1) MB_NA(128, 2) MB_NA(128, 4) MB_NA(128, 8) MB_NA(128, 16)
  MB_NA(256, 1) MB_NA(256, 2) MB_NA(256, 4) MB_NA(256, 8)
  MB_NA(64, 1) MB_NA(64, 2) MB_NA(64, 4) MB_NA(64, 8)
  else ok = false;
#undef MB_NA
  if (!ok) return fail(3, "mb_attn_decode_noalloc: unsupported head_dim / group size");
  if (cudaGetLastError() != cudaSuccess) return fail(4, "mb_attn_decode_noalloc: split kernel launch failed");
  if (splits > 1) {
    if (D == 128) mb::attn_combine_kernel<128><<<B * Hq, 128, 0, st>>>(po, pl, pout, splits);
    else if (D == 256) mb::attn_combine_kernel<256><<<B * Hq, 128, 0, st>>>(po, pl, pout, splits);
    else mb::attn_combine_kernel<64><<<B * Hq, 64, 0, st>>>(po, pl, pout, splits);
    if (cudaGetLastError() != cudaSuccess) return fail(4, "mb_attn_decode_noalloc: combine kernel launch failed");
  }
  g_err[0] = '\0';
  return 0;
}

}  // extern "C"
