// Expert-parallel MoE dispatch / combine fused with the all-to-all over
// NVLink peer memory (P2P loads and stores issued from inside the kernels; no
// NCCL on this path).
//
// Every rank owns one "exchange" buffer, mapped into every other rank with
// CUDA IPC, laid out as
//   recv_x [N*C, H] bf16  rows sent to this rank (source r uses rows r*C ..)
//   comb   [N*C, H] bf16  expert outputs returned to this rank (owner o uses rows o*C ..)
//   meta   [N*C]    int32 local expert id of each received row
//   cnt    [N]      int32 rows received from each source
//   flag_d [N]      u32   dispatch epoch written by each source
//   flag_c [N]      u32   combine epoch written by each owner
//   cntm   [N][1024] int32 per-expert counts of each source (direct dispatch)
//   flag_n [N]      u32   counts epoch written by each source
// C = capacity per (source, owner) = max tokens per call x top-k, so a call can
// never overflow.  The product path (ep_dispatch2 / ep_combine2) is
//   ep_dispatch2        counts all-gather, then each row stored straight into
//                       its owner's expert-ordered receive region (+ its return
//                       address in meta); flag_d released at every owner.
//   grouped GEMMs       gate/up waits on flag_d in its TMA producer; down.
//   ep_combine_send2    result rows back to their sources' comb slots.
//   ep_combine_reduce   as below.
// The three-kernel receive path below (dispatch, recv, permute) is kept for
// the bounded-wait fault test.  One MoE call:
//   ep_dispatch      (source) each (token, k) pair claims a slot in its owner's
//                    receive region and stores the hidden row there; the last
//                    CTA publishes counts and releases flag_d at the owner.
//   ep_recv          (owner)  bounded wait for every source's flag, histogram
//                    of local experts, expert-ordered position of each row.
//   ep_permute       (owner)  copy received rows into expert order.
//   grouped GEMMs    (owner)  gate/up + SwiGLU, down (gemm.cu).
//   ep_combine_send  (owner)  store each result row into its source's comb
//                    region; the last CTA releases flag_c at every source.
//   ep_combine_reduce(source) bounded wait for every owner's flag, then
//                    out[t] = residual[t] + sum_k w[t,k] * comb[map[t,k]] in a
//                    fixed k order; the last CTA advances the epoch.
// Flags carry a monotonically increasing epoch kept in device memory, so the
// sequence is replayable inside a CUDA graph without host work.  Buffer reuse
// across consecutive calls is safe: a source only dispatches call i+1 after
// its combine of call i has seen every owner's flag, and an owner only sends
// combine results after receiving every source's dispatch.
//
// The reference has no distributed code; its MoE loops over experts on one
// device with a host sync per top-k slot (pio/models/qwen3_coder_30b/model.py:308-353).
#include <cstring>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "launch.cuh"
#include "status.h"

namespace mb {

constexpr int kEpMaxExperts = 1024;  // global experts covered by the count matrix

struct EpLayout {
  int64_t recv_x, comb, meta, cnt, flag_d, flag_c, cntm, flag_n, total;
};

static EpLayout ep_layout(int64_t N, int64_t C, int64_t H) {
  auto al = [](int64_t x) { return (x + 255) / 256 * 256; };
  EpLayout L;
  L.recv_x = 0;
  L.comb = al(L.recv_x + N * C * H * 2);
  L.meta = al(L.comb + N * C * H * 2);
  L.cnt = al(L.meta + N * C * 4);
  L.flag_d = al(L.cnt + N * 4);
  L.flag_c = al(L.flag_d + N * 4);
  L.cntm = al(L.flag_c + N * 4);           // [N][kEpMaxExperts] int32: every source's per-expert counts
  L.flag_n = al(L.cntm + N * kEpMaxExperts * 4);
  L.total = al(L.flag_n + N * 4);
  return L;
}

int64_t ep_buffer_bytes(int64_t N, int64_t C, int64_t H) { return ep_layout(N, C, H).total; }

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Bounded spin until *p >= want (wrap-safe compare).  Returns false on timeout.
__device__ __forceinline__ bool wait_flag(const uint32_t* p, uint32_t want, int* status, int code) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0;; ++i) {
    if ((int32_t)(ld_acquire_sys(p) - want) >= 0) return true;
    if ((i & 63) == 63 && globaltimer_ns() - t0 > kWaitLimitNs) {
      set_status(status, code);
      return false;
    }
  }
}

template <typename T>
__device__ __forceinline__ T* at_off(uint64_t base, int64_t off) {
  return reinterpret_cast<T*>(base + off);
}

// Warp copies one row of n16 16-byte chunks: per lane 8 loads in flight, then
// 8 stores (a load-store loop over possibly aliasing pointers would serialise
// on every chunk).  L2 loads (.cg) for data other GPUs wrote.
template <bool CG>
__device__ __forceinline__ void copy_row(uint4* __restrict__ d, const uint4* __restrict__ s, int n16, int lane) {
  for (int base = 0; base < n16; base += 32 * 8) {
    uint4 r[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = base + j * 32 + lane;
      if (i < n16) r[j] = CG ? __ldcg(s + i) : s[i];
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = base + j * 32 + lane;
      if (i < n16) d[i] = r[j];
    }
  }
}

struct EpArgs {
  const uint64_t* peers;  // [N] base address of every rank's exchange buffer (own rank included)
  int rank, N, C, H, El;
  EpLayout L;
  uint32_t* epoch;        // [1] local
  int* send_cnt;          // [N] local, zero between calls
  int* done;              // [4] local CTA-completion counters, zero between calls
  int* status;
};

// ---------------------------------------------------------------- dispatch
__global__ void ep_dispatch_kernel(EpArgs a, const __nv_bfloat16* __restrict__ x, const int* __restrict__ ids,
                                   int TK, int K, int* __restrict__ map) {
  pdl_wait();
  pdl_trigger();
  const uint32_t epoch = *a.epoch + 1;
  const int warps = blockDim.x / 32, warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  for (int pair = blockIdx.x * warps + warp; pair < TK; pair += gridDim.x * warps) {
    int e = ids[pair];
    if (e < 0 || e >= a.El * a.N) {  // defensive: an invalid id must never become an address
      set_status(a.status, kErrBounds);
      e = 0;
    }
    const int dst = e / a.El;
    int slot = 0;
    if (lane == 0) {
      slot = atomicAdd(&a.send_cnt[dst], 1);
      map[pair] = dst * a.C + slot;
      at_off<int>(a.peers[dst], a.L.meta)[a.rank * a.C + slot] = e % a.El;
    }
    slot = __shfl_sync(0xffffffffu, slot, 0);
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(pair / K) * a.H);
    uint4* dstp = reinterpret_cast<uint4*>(at_off<__nv_bfloat16>(a.peers[dst], a.L.recv_x) +
                                           ((size_t)a.rank * a.C + slot) * a.H);
    copy_row<false>(dstp, src, a.H / 8, lane);
  }
  // CTA barrier, then one system-scope fence + arrive per CTA (cumulative over the CTA's stores)
  __syncthreads();
  __shared__ int last;
  if (threadIdx.x == 0) {
    __threadfence_system();
    last = atomicAdd(&a.done[0], 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence_system();
  for (int dst = threadIdx.x; dst < a.N; dst += blockDim.x) {
    at_off<int>(a.peers[dst], a.L.cnt)[a.rank] = atomicAdd(&a.send_cnt[dst], 0);
  }
  __threadfence_system();
  __syncthreads();
  for (int dst = threadIdx.x; dst < a.N; dst += blockDim.x) {
    st_release_sys(at_off<uint32_t>(a.peers[dst], a.L.flag_d) + a.rank, epoch);
    a.send_cnt[dst] = 0;
  }
  if (threadIdx.x == 0) a.done[0] = 0;
}

// ---------------------------------------------------------------- receive
// One CTA of 1024 threads: waits for all sources, orders rows by local expert.
__global__ void __launch_bounds__(1024) ep_recv_kernel(EpArgs a, int* __restrict__ row_pos, int* __restrict__ offs, int* __restrict__ abort) {
  pdl_wait();
  pdl_trigger();
  const uint32_t epoch = *a.epoch + 1;
  const uint64_t self = a.peers[a.rank];
  __shared__ int hist[1024];
  __shared__ int cursor[1024];
  __shared__ int cnts[64];
  __shared__ int ok_all;
  if (threadIdx.x == 0) ok_all = 1;
  for (int e = threadIdx.x; e < a.El; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  for (int src = threadIdx.x; src < a.N; src += blockDim.x) {
    if (!wait_flag(at_off<uint32_t>(self, a.L.flag_d) + src, epoch, a.status, kErrPeerTimeout)) ok_all = 0;
    cnts[src] = ld_acquire_sys(reinterpret_cast<const uint32_t*>(at_off<int>(self, a.L.cnt) + src));
  }
  __syncthreads();
  __threadfence();  // order this thread's reads after the flag acquires above
  if (!ok_all) {
    if (threadIdx.x == 0) *abort = 1;
  }
  const int* meta = at_off<int>(self, a.L.meta);
  const int rows = a.N * a.C;
  for (int i = threadIdx.x; i < rows; i += blockDim.x) {
    const int src = i / a.C, slot = i % a.C;
    if (ok_all && slot < cnts[src]) atomicAdd(&hist[__ldcg(meta + i)], 1);
  }
  __syncthreads();
  {  // exclusive scan of hist over El <= 1024 experts: warp scans, then a scan of the warp totals
    __shared__ int wsum[32];
    const int e = threadIdx.x, lane = e & 31, wid = e >> 5;
    const int h = e < a.El ? hist[e] : 0;
    int incl = h;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (lane == 31) wsum[wid] = incl;
    __syncthreads();
    if (wid == 0) {
      int w = lane < (int)(blockDim.x >> 5) ? wsum[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += n;
      }
      wsum[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    const int excl = incl - h + (wid > 0 ? wsum[wid - 1] : 0);
    if (e < a.El) {
      offs[e] = excl;
      cursor[e] = excl;
    }
    if (e == a.El - 1) offs[a.El] = excl + h;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < rows; i += blockDim.x) {
    const int src = i / a.C, slot = i % a.C;
    row_pos[i] = (ok_all && slot < cnts[src]) ? atomicAdd(&cursor[__ldcg(meta + i)], 1) : -1;
  }
}

// warp per received row: recv_x[i] -> xs[row_pos[i]]
__global__ void ep_permute_kernel(EpArgs a, const int* __restrict__ row_pos, __nv_bfloat16* __restrict__ xs) {
  pdl_wait();
  pdl_trigger();
  const int warps = blockDim.x / 32, lane = threadIdx.x & 31;
  const uint64_t self = a.peers[a.rank];
  const __nv_bfloat16* rx = at_off<__nv_bfloat16>(self, a.L.recv_x);
  for (int i = blockIdx.x * warps + threadIdx.x / 32; i < a.N * a.C; i += gridDim.x * warps) {
    const int p = row_pos[i];
    if (p < 0) continue;
    const uint4* s = reinterpret_cast<const uint4*>(rx + (size_t)i * a.H);
    uint4* d = reinterpret_cast<uint4*>(xs + (size_t)p * a.H);
    copy_row<true>(d, s, a.H / 8, lane);
  }
}

// ---------------------------------------------------------------- combine
__global__ void ep_combine_send_kernel(EpArgs a, const int* __restrict__ row_pos, const __nv_bfloat16* __restrict__ y) {
  pdl_wait();
  pdl_trigger();
  const uint32_t epoch = *a.epoch + 1;
  const int warps = blockDim.x / 32, lane = threadIdx.x & 31;
  for (int i = blockIdx.x * warps + threadIdx.x / 32; i < a.N * a.C; i += gridDim.x * warps) {
    const int p = row_pos[i];
    if (p < 0) continue;
    const int src = i / a.C, slot = i % a.C;
    const uint4* s = reinterpret_cast<const uint4*>(y + (size_t)p * a.H);
    uint4* d = reinterpret_cast<uint4*>(at_off<__nv_bfloat16>(a.peers[src], a.L.comb) +
                                        ((size_t)a.rank * a.C + slot) * a.H);
    copy_row<false>(d, s, a.H / 8, lane);
  }
  __syncthreads();
  __shared__ int last;
  if (threadIdx.x == 0) {
    __threadfence_system();
    last = atomicAdd(&a.done[1], 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence_system();
  for (int src = threadIdx.x; src < a.N; src += blockDim.x)
    st_release_sys(at_off<uint32_t>(a.peers[src], a.L.flag_c) + a.rank, epoch);
  if (threadIdx.x == 0) a.done[1] = 0;
}

// CTA per token: wait for every owner, weighted sum in k order, + residual.
__global__ void ep_combine_reduce_kernel(EpArgs a, const int* __restrict__ map, const float* __restrict__ wts, int T,
                                         int K, const __nv_bfloat16* __restrict__ residual,
                                         __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const uint32_t epoch = *a.epoch + 1;
  const uint64_t self = a.peers[a.rank];
  __shared__ int ok_all;
  if (threadIdx.x == 0) ok_all = 1;
  __syncthreads();
  for (int o = threadIdx.x; o < a.N; o += blockDim.x)
    if (!wait_flag(at_off<uint32_t>(self, a.L.flag_c) + o, epoch, a.status, kErrPeerTimeout)) ok_all = 0;
  __syncthreads();
  __threadfence();
  const __nv_bfloat16* comb = at_off<__nv_bfloat16>(self, a.L.comb);
  for (int t = blockIdx.x; t < T; t += gridDim.x) {
    for (int c = threadIdx.x * 8; c < a.H; c += blockDim.x * 8) {
      float acc[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] = residual ? __bfloat162float(residual[(size_t)t * a.H + c + q]) : 0.f;
      if (ok_all) {
        for (int k0 = 0; k0 < K; k0 += 8) {  // 8 expert rows in flight, summed in k order
          uint4 raw[8];
          float wk[8];
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if (k0 + j < K) {
              raw[j] = __ldcg(reinterpret_cast<const uint4*>(comb + (size_t)map[t * K + k0 + j] * a.H + c));
              wk[j] = wts[t * K + k0 + j];
            }
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if (k0 + j < K) {
              const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw[j]);
#pragma unroll
              for (int q = 0; q < 8; ++q) acc[q] += wk[j] * __bfloat162float(h[q]);
            }
        }
      }
      __align__(16) __nv_bfloat16 o8[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) o8[q] = __float2bfloat16(acc[q]);
      *reinterpret_cast<uint4*>(out + (size_t)t * a.H + c) = *reinterpret_cast<uint4*>(o8);
    }
  }
  __syncthreads();
  __shared__ int last;
  if (threadIdx.x == 0) last = atomicAdd(&a.done[2], 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (last && threadIdx.x == 0) {
    *a.epoch = epoch;  // every kernel of this call has read the old value
    a.done[2] = 0;
  }
}

// ------------------------------------------------ direct-placement dispatch
// One kernel replaces dispatch + receive + permute.  Every rank broadcasts its
// per-expert counts (CTA 0: the [N][E] count matrix lands in every buffer, then
// flag_n); every CTA waits for the other ranks' counts (its own come from the
// local routing output, so no CTA waits on another CTA of this GPU), derives
//   base[e]  first row of expert e in its owner's expert-ordered GEMM input
//   pre[e]   rows of expert e sent by lower ranks
//   sbase[e] this rank's rows for lower experts of the same owner
// and a warp per (token, k) pair stores the hidden row at row
// base[e] + pre[e] + idx of the owner's xs (idx = order among this rank's
// pairs of expert e), and its return address (rank, slot) into the owner's
// meta.  The last CTA releases flag_d at every owner; the owner's gate/up GEMM
// waits on those flags in its TMA producer.  CTA 0 also writes this rank's
// offs[El + 1] (expert row offsets of its own xs).
__device__ __forceinline__ int block_excl_scan(int v, int* sh) {  // blockDim <= 1024, sh >= 32 ints
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  __syncthreads();
  if (lane == 31) sh[wid] = incl;
  __syncthreads();
  if (wid == 0) {
    int w = lane < (int)(blockDim.x >> 5) ? sh[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += n;
    }
    sh[lane] = w;
  }
  __syncthreads();
  return incl - v + (wid > 0 ? sh[wid - 1] : 0);
}

__global__ void __launch_bounds__(1024)
    ep_dispatch2_kernel(EpArgs a, const __nv_bfloat16* __restrict__ x, const int* __restrict__ ids,
                        const int* __restrict__ counts, const int* __restrict__ offs_g, int* __restrict__ cursor,
                        int TK, int K, int* __restrict__ map, int* __restrict__ offs) {
  pdl_wait();
  pdl_trigger();
  const uint32_t epoch = *a.epoch + 1;
  const int E = a.El * a.N, tid = threadIdx.x;
  extern __shared__ int sm[];
  int* base = sm;           // [E]
  int* pre = base + E;      // [E]
  int* sbase = pre + E;     // [E]
  int* col = sbase + E;     // [E]
  int* scan_sh = col + E;   // [32]
  __shared__ int ok_all;
  const uint64_t self = a.peers[a.rank];
  if (blockIdx.x == 0) {  // publish this rank's counts to every rank
    for (int d = 0; d < a.N; ++d) {
      int* dst = at_off<int>(a.peers[d], a.L.cntm) + a.rank * kEpMaxExperts;
      for (int e = tid; e < E; e += blockDim.x) dst[e] = counts[e];
    }
    __syncthreads();
    if (tid == 0) {
      __threadfence_system();
      for (int d = 0; d < a.N; ++d) st_release_sys(at_off<uint32_t>(a.peers[d], a.L.flag_n) + a.rank, epoch);
    }
  }
  if (tid == 0) ok_all = 1;
  __syncthreads();
  for (int src = tid; src < a.N; src += blockDim.x)
    if (src != a.rank && !wait_flag(at_off<uint32_t>(self, a.L.flag_n) + src, epoch, a.status, kErrPeerTimeout))
      ok_all = 0;
  __syncthreads();
  __threadfence();
  const int* cntm = at_off<int>(self, a.L.cntm);
  // per expert: column sum and lower-rank prefix; every thread owns experts tid, tid + blockDim, ...
  // (E <= blockDim is enforced on the host, so one expert per thread)
  int colsum = 0, mine = 0, lower = 0;
  const int e = tid;
  if (e < E) {
    for (int src = 0; src < a.N; ++src) {
      const int c = src == a.rank ? counts[e] : (ok_all ? __ldcg(cntm + src * kEpMaxExperts + e) : 0);
      colsum += c;
      if (src < a.rank) lower += c;
      if (src == a.rank) mine = c;
    }
  }
  // global exclusive scans, then rebased to the start of each owner's expert segment
  const int gcol = block_excl_scan(e < E ? colsum : 0, scan_sh);
  if (e < E) base[e] = gcol;
  const int gmine = block_excl_scan(e < E ? mine : 0, scan_sh);
  if (e < E) sbase[e] = gmine;
  if (e < E) {
    pre[e] = lower;
    col[e] = colsum;
  }
  __syncthreads();
  int seg_col = 0, seg_mine = 0;  // scan values at the first expert of this owner's segment
  if (e < E) {
    const int seg = (e / a.El) * a.El;
    seg_col = base[seg];
    seg_mine = sbase[seg];
  }
  __syncthreads();
  if (e < E) {
    base[e] = gcol - seg_col;
    sbase[e] = gmine - seg_mine;
  }
  __syncthreads();
  if (blockIdx.x == 0 && tid <= a.El) {  // this rank's own xs offsets
    const int g0 = a.rank * a.El;
    offs[tid] = tid < a.El ? base[g0 + tid] : base[g0 + a.El - 1] + col[g0 + a.El - 1];
  }
  // rows
  const int warps = blockDim.x / 32, warp = tid / 32, lane = tid & 31;
  for (int pair = blockIdx.x * warps + warp; pair < TK; pair += gridDim.x * warps) {
    int ex = ids[pair];
    if (ex < 0 || ex >= E) {  // defensive: an invalid id must never become an address
      set_status(a.status, kErrBounds);
      ex = 0;
    }
    const int dst = ex / a.El;
    int idx = 0;
    if (lane == 0) idx = atomicAdd(&cursor[ex], 1);  // the routing step leaves cursor[] at zero
    idx = __shfl_sync(0xffffffffu, idx, 0);
    const int pos = base[ex] + pre[ex] + idx;    // row in the owner's xs
    const int slot = sbase[ex] + idx;            // row in this rank's comb region of that owner
    if (!ok_all || idx < 0 || idx >= counts[ex] || pos < 0 || pos >= a.N * a.C || slot < 0 || slot >= a.C) {
      if (lane == 0) {  // status set: the host raises after the step
        if (ok_all) set_status(a.status, kErrCapacity);
        map[pair] = 0;  // a valid comb row, so the combine never indexes out of bounds
      }
      continue;
    }
    if (lane == 0) {
      map[pair] = dst * a.C + slot;
      at_off<int>(a.peers[dst], a.L.meta)[pos] = a.rank * a.C + slot;
    }
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(pair / K) * a.H);
    uint4* dstp = reinterpret_cast<uint4*>(at_off<__nv_bfloat16>(a.peers[dst], a.L.recv_x) + (size_t)pos * a.H);
    copy_row<false>(dstp, src, a.H / 8, lane);
  }
  __syncthreads();
  __shared__ int last;
  if (tid == 0) {
    __threadfence_system();
    last = atomicAdd(&a.done[0], 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  if (tid == 0) {
    __threadfence_system();
    for (int d = 0; d < a.N; ++d) st_release_sys(at_off<uint32_t>(a.peers[d], a.L.flag_d) + a.rank, epoch);
    a.done[0] = 0;
  }
}

// ------------------------------------------- fused route + dispatch (one launch)
// Router GEMV, softmax top-k, the per-expert count exchange and the direct
// placement of every (token, k) row in its owner's expert-ordered receive
// region, in one kernel.  Phases, separated by grid barriers (the grid is at
// most one CTA per SM, so every CTA is resident; waits are bounded):
//   1. logits[t][e] = x[t] . Wr[e] in fp32, tiles of 8 experts x 16 tokens;
//   2. a warp per token: softmax, top-k (ties to the lower expert id),
//      optional renormalisation; ids / wts written, counts[e] += 1;
//   3. the last CTA to arrive publishes this rank's counts to every rank and
//      releases flag_n; every CTA waits for all ranks' counts, derives the
//      expert bases (as ep_dispatch2 does) and a warp per pair stores the row
//      into its owner's buffer.  The last CTA to finish releases flag_d at
//      every owner, and zeroes counts / cursors / barrier counters for the
//      next call.
// Scratch (device, zero between calls): counts [E], cursor [E]; logits [T, E] f32.
constexpr int kRdThreads = 1024;

// Orders this thread's earlier writes before a later flag store: at system scope when peers read
// them over NVLink, at device scope on a single rank (a system-scope fence costs microseconds).
__device__ __forceinline__ void fence_peers(int nranks) {
  if (nranks > 1) __threadfence_system();
  else __threadfence();
}
constexpr int kRdTileE = 8, kRdTileT = 16;

__device__ __forceinline__ bool grid_arrive_wait(int* ctr, int target, int* status) {
  __syncthreads();
  __shared__ int ok;
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(ctr, 1);
    ok = 1;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 0;; ++i) {
      int v;
      asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
      if (v >= target) break;
      if ((i & 63) == 63 && globaltimer_ns() - t0 > kWaitLimitNs) {
        set_status(status, kErrPeerTimeout);
        ok = 0;
        break;
      }
    }
    __threadfence();
  }
  __syncthreads();
  return ok != 0;
}

template <int EPL>
__global__ void __launch_bounds__(kRdThreads)
    ep_route_dispatch_kernel(EpArgs a, const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ wr,
                             int T, int K, int renorm, float* __restrict__ logits, int* __restrict__ ids,
                             float* __restrict__ wts, int* __restrict__ counts, int* __restrict__ cursor,
                             int* __restrict__ map, int* __restrict__ offs, int* __restrict__ bar,
                             int* __restrict__ pos_map, uint64_t* __restrict__ trace) {
  // trace (optional, [8]): %globaltimer of CTA 0 at the phase boundaries, for latency attribution
  auto mark = [&](int i) {
    if (trace && blockIdx.x == 0 && threadIdx.x == 0) trace[i] = globaltimer_ns();
  };
  mark(0);
  pdl_wait();
  pdl_trigger();
  mark(1);
  const uint32_t epoch = *a.epoch + 1;
  const int E = a.El * a.N, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, H = a.H;
  // ---------------- 1. router logits
  // A tile is 8 experts x 16 tokens: its 8 router rows and 16 token rows are brought into shared
  // memory with 16-byte cp.async copies (one round of memory latency), then warp w forms the dot
  // products of expert w % 8 with tokens 4*(w / 8) .. +3 from shared memory.
  {
    extern __shared__ __align__(16) uint8_t rd_dyn[];
    __nv_bfloat16* sw = reinterpret_cast<__nv_bfloat16*>(rd_dyn);          // [8][H]
    __nv_bfloat16* sx = sw + kRdTileE * H;                                  // [16][H]
    const int tiles_e = (E + kRdTileE - 1) / kRdTileE, tiles_t = (T + kRdTileT - 1) / kRdTileT;
    const int e_in = warp % kRdTileE, t_grp = warp / kRdTileE;  // 4 token groups of 4 tokens
    const int n16 = H / 8;                                      // 16-byte pieces per row
    for (int tile = blockIdx.x; tile < tiles_e * tiles_t; tile += G) {
      const int e_base = (tile % tiles_e) * kRdTileE, t_base = (tile / tiles_e) * kRdTileT;
      __syncthreads();  // the previous tile's reads are done
      for (int i = tid; i < (kRdTileE + kRdTileT) * n16; i += blockDim.x) {
        const int row = i / n16, piece = i % n16;
        const bool is_w = row < kRdTileE;
        const int src_row = is_w ? e_base + row : t_base + row - kRdTileE;
        const bool in = is_w ? src_row < E : src_row < T;
        const __nv_bfloat16* src = (is_w ? wr : x) + (in ? (size_t)src_row * H + piece * 8 : 0);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(sw + (size_t)row * H + piece * 8)),
                     "l"(src), "r"(in ? 16 : 0) : "memory");
      }
      asm volatile("cp.async.commit_group;\n\tcp.async.wait_all;" ::: "memory");
      __syncthreads();
      const int e = e_base + e_in, t0 = t_base + t_grp * 4;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      for (int c = lane * 8; c < H; c += 256) {
        const uint4 wv = *reinterpret_cast<const uint4*>(sw + (size_t)e_in * H + c);
        const __nv_bfloat16* wh = reinterpret_cast<const __nv_bfloat16*>(&wv);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 xv = *reinterpret_cast<const uint4*>(sx + (size_t)(t_grp * 4 + j) * H + c);
          const __nv_bfloat16* xh = reinterpret_cast<const __nv_bfloat16*>(&xv);
#pragma unroll
          for (int q = 0; q < 8; ++q) acc[j] += __bfloat162float(wh[q]) * __bfloat162float(xh[q]);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float v = warp_sum(acc[j]);
        if (lane == 0 && e < E && t0 + j < T) logits[(size_t)(t0 + j) * E + e] = v;
      }
    }
  }
  mark(2);
  if (!grid_arrive_wait(bar, G, a.status)) return;
  mark(3);
  // ---------------- 2. top-k per token (warp per token)
  for (int t = blockIdx.x + G * warp; t < T; t += G * (kRdThreads / 32)) {  // spread over the CTAs
    float v[EPL];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = i * 32 + lane;
      v[i] = e < E ? __ldcg(logits + (size_t)t * E + e) : -INFINITY;
      mx = fmaxf(mx, v[i]);
    }
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = i * 32 + lane;
      v[i] = e < E ? __expf(v[i] - mx) : -1.f;  // probabilities; -1 marks padding
      sum += e < E ? v[i] : 0.f;
    }
    sum = warp_sum(sum);
    float picked = 0.f, my_w = 0.f;
    int my_id = -1;
    for (int k = 0; k < K; ++k) {
      float bv = -2.f;
      int bi = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < EPL; ++i)
        if (v[i] > bv) { bv = v[i]; bi = i * 32 + lane; }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      if (lane == k) { my_w = bv / sum; my_id = bi; }
      picked += bv / sum;
#pragma unroll
      for (int i = 0; i < EPL; ++i)
        if (i * 32 + lane == bi) v[i] = -2.f;
    }
    if (lane < K) {
      if (my_id < 0 || my_id >= E) {  // non-finite logits: never index with an invalid id
        set_status(a.status, kErrBounds);
        my_id = 0;
        my_w = 0.f;
      }
      ids[(size_t)t * K + lane] = my_id;
      wts[(size_t)t * K + lane] = renorm ? my_w / picked : my_w;
      atomicAdd(&counts[my_id], 1);
    }
  }
  // ---------------- 3. count exchange, then placement
  __shared__ int last_in;
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    last_in = atomicAdd(bar + 1, 1) == G - 1;
  }
  __syncthreads();
  if (last_in) {  // every CTA's counts are in: publish them to every rank
    __threadfence();
    for (int d = 0; d < a.N; ++d) {
      int* dst = at_off<int>(a.peers[d], a.L.cntm) + a.rank * kEpMaxExperts;
      for (int e = tid; e < E; e += blockDim.x) dst[e] = __ldcg(counts + e);
    }
    __syncthreads();
    if (tid == 0) {
      fence_peers(a.N);
      for (int d = 0; d < a.N; ++d) st_release_sys(at_off<uint32_t>(a.peers[d], a.L.flag_n) + a.rank, epoch);
    }
  }
  __shared__ int ok_all;
  __shared__ int sh[5 * kEpMaxExperts + 32];
  int* base = sh;
  int* pre = base + kEpMaxExperts;
  int* sbase = pre + kEpMaxExperts;
  int* col = sbase + kEpMaxExperts;
  int* own = col + kEpMaxExperts;
  int* scan_sh = own + kEpMaxExperts;
  if (tid == 0) ok_all = 1;
  __syncthreads();
  const uint64_t self = a.peers[a.rank];
  mark(4);
  for (int src = tid; src < a.N; src += blockDim.x)  // own counts included: they arrive through the same path
    if (!wait_flag(at_off<uint32_t>(self, a.L.flag_n) + src, epoch, a.status, kErrPeerTimeout)) ok_all = 0;
  __syncthreads();
  __threadfence();
  mark(5);
  const int* cntm = at_off<int>(self, a.L.cntm);
  int colsum = 0, mine = 0, lower = 0;
  const int e = tid;
  if (e < E && ok_all) {
    for (int src = 0; src < a.N; ++src) {
      const int c = __ldcg(cntm + src * kEpMaxExperts + e);
      colsum += c;
      if (src < a.rank) lower += c;
      if (src == a.rank) mine = c;
    }
  }
  const int gcol = block_excl_scan(e < E ? colsum : 0, scan_sh);
  if (e < E) base[e] = gcol;
  const int gmine = block_excl_scan(e < E ? mine : 0, scan_sh);
  if (e < E) {
    sbase[e] = gmine;
    pre[e] = lower;
    col[e] = colsum;
    own[e] = mine;
  }
  __syncthreads();
  int seg_col = 0, seg_mine = 0;
  if (e < E) {
    const int seg = (e / a.El) * a.El;
    seg_col = base[seg];
    seg_mine = sbase[seg];
  }
  __syncthreads();
  if (e < E) {
    base[e] = gcol - seg_col;
    sbase[e] = gmine - seg_mine;
  }
  __syncthreads();
  if (blockIdx.x == 0 && tid <= a.El) {
    const int g0 = a.rank * a.El;
    offs[tid] = tid < a.El ? base[g0 + tid] : base[g0 + a.El - 1] + col[g0 + a.El - 1];
  }
  const int TK = T * K;
  for (int pair = blockIdx.x + G * warp; pair < TK; pair += G * (kRdThreads / 32)) {  // spread over the CTAs
    int ex = __ldcg(ids + pair);
    if (ex < 0 || ex >= E) ex = 0;
    const int dst = ex / a.El;
    int idx = 0;
    if (lane == 0) idx = atomicAdd(&cursor[ex], 1);
    idx = __shfl_sync(0xffffffffu, idx, 0);
    const int pos = base[ex] + pre[ex] + idx;
    const int slot = sbase[ex] + idx;
    if (!ok_all || idx < 0 || idx >= own[ex] || pos < 0 || pos >= a.N * a.C || slot < 0 || slot >= a.C) {
      if (lane == 0) {
        if (ok_all) set_status(a.status, kErrCapacity);
        map[pair] = 0;
      }
      continue;
    }
    if (lane == 0) {
      map[pair] = dst * a.C + slot;
      if (pos_map) pos_map[pair] = pos;  // single rank: the combine reads the expert rows in place
      at_off<int>(a.peers[dst], a.L.meta)[pos] = a.rank * a.C + slot;
    }
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(pair / K) * H);
    uint4* dstp = reinterpret_cast<uint4*>(at_off<__nv_bfloat16>(a.peers[dst], a.L.recv_x) + (size_t)pos * H);
    copy_row<false>(dstp, src, H / 8, lane);
  }
  mark(6);
  __syncthreads();
  __shared__ int last;
  if (tid == 0) {
    fence_peers(a.N);
    last = atomicAdd(&a.done[0], 1) == G - 1;
  }
  __syncthreads();
  mark(7);
  if (!last) return;
  // every CTA is past its last use of counts / cursor / the barrier counters
  for (int i = tid; i < E; i += blockDim.x) {
    counts[i] = 0;
    cursor[i] = 0;
  }
  if (tid == 0) {
    bar[0] = 0;
    bar[1] = 0;
    fence_peers(a.N);
    for (int d = 0; d < a.N; ++d) st_release_sys(at_off<uint32_t>(a.peers[d], a.L.flag_d) + a.rank, epoch);
    a.done[0] = 0;
  }
}

// Owner: expert outputs y (xs order, offs[El] rows) back to their sources' comb slots.
__global__ void ep_combine_send2_kernel(EpArgs a, const int* __restrict__ offs, const __nv_bfloat16* __restrict__ y) {
  pdl_wait();
  pdl_trigger();
  const uint32_t epoch = *a.epoch + 1;
  const uint64_t self = a.peers[a.rank];
  __shared__ int ok_all;
  if (threadIdx.x == 0) ok_all = 1;
  __syncthreads();
  for (int src = threadIdx.x; src < a.N; src += blockDim.x)  // already complete: orders the meta reads
    if (!wait_flag(at_off<uint32_t>(self, a.L.flag_d) + src, epoch, a.status, kErrPeerTimeout)) ok_all = 0;
  __syncthreads();
  __threadfence();
  const int rows = min(offs[a.El], a.N * a.C);
  const int* meta = at_off<int>(self, a.L.meta);
  const int warps = blockDim.x / 32, lane = threadIdx.x & 31;
  for (int p = blockIdx.x * warps + threadIdx.x / 32; ok_all && p < rows; p += gridDim.x * warps) {
    const int dst = __ldcg(meta + p);
    const int src = dst / a.C, slot = dst - src * a.C;
    if (src < 0 || src >= a.N) continue;
    const uint4* s = reinterpret_cast<const uint4*>(y + (size_t)p * a.H);
    uint4* d = reinterpret_cast<uint4*>(at_off<__nv_bfloat16>(a.peers[src], a.L.comb) +
                                        ((size_t)a.rank * a.C + slot) * a.H);
    copy_row<false>(d, s, a.H / 8, lane);
  }
  __syncthreads();
  __shared__ int last;
  if (threadIdx.x == 0) {
    __threadfence_system();
    last = atomicAdd(&a.done[1], 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int src = 0; src < a.N; ++src) st_release_sys(at_off<uint32_t>(a.peers[src], a.L.flag_c) + a.rank, epoch);
    a.done[1] = 0;
  }
}

// ------------------------------------------- combine fused with add + RMSNorm
// Replaces ep_combine_reduce + the next layer's add + RMSNorm: a warp per
// token waits (bounded) for every owner's flag_c, forms
//   h = bf16(sum_k w[t,k] * comb[map[t,k]])      (fixed k order)
//   residual[t] = bf16(residual[t] + h);  out[t] = rmsnorm(residual[t]) * nw
// which is exactly what the two kernels computed.  The last CTA advances the
// epoch.  H is a compile-time multiple of 256.
template <int H>
__global__ void __launch_bounds__(H / 8)
    ep_combine_norm_kernel(EpArgs a, const int* __restrict__ map, const float* __restrict__ wts, int T,
                           int K, __nv_bfloat16* __restrict__ residual,
                           const __nv_bfloat16* __restrict__ nw, __nv_bfloat16* __restrict__ out,
                           float eps, const __nv_bfloat16* __restrict__ rows) {
  // CTA per token, H/8 threads, 8 columns per thread: the K expert rows, the residual and the norm
  // weight of a thread's columns are all requested before any is used (one round of latency),
  // then a block reduction forms the RMS.
  pdl_wait();
  pdl_trigger();
  constexpr int kThreadsCN = H / 8, kWarpsCN = kThreadsCN / 32 > 0 ? kThreadsCN / 32 : 1;
  const uint32_t epoch = *a.epoch + 1;
  const uint64_t self = a.peers[a.rank];
  __shared__ int ok_all;
  __shared__ float red[kWarpsCN];
  if (threadIdx.x == 0) ok_all = 1;
  __syncthreads();
  // rows != nullptr (single rank): the expert outputs are read where the down GEMM wrote them
  for (int o = threadIdx.x; o < a.N && !rows; o += blockDim.x)
    if (!wait_flag(at_off<uint32_t>(self, a.L.flag_c) + o, epoch, a.status, kErrPeerTimeout)) ok_all = 0;
  __syncthreads();
  __threadfence();
  const __nv_bfloat16* comb = rows ? rows : at_off<__nv_bfloat16>(self, a.L.comb);
  const int c = threadIdx.x * 8, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int t = blockIdx.x; t < T; t += gridDim.x) {
    const uint4 rr = *reinterpret_cast<const uint4*>(residual + (size_t)t * H + c);
    const uint4 wr = *reinterpret_cast<const uint4*>(nw + c);
    float v[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) v[q] = 0.f;
    if (ok_all) {
      for (int k0 = 0; k0 < K; k0 += 8) {  // up to 8 expert rows in flight, summed in k order
        uint4 raw[8];
        float wk[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (k0 + j < K) {
            raw[j] = __ldcg(reinterpret_cast<const uint4*>(comb + (size_t)map[t * K + k0 + j] * H + c));
            wk[j] = wts[t * K + k0 + j];
          }
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (k0 + j < K) {
            const __nv_bfloat16* hh = reinterpret_cast<const __nv_bfloat16*>(&raw[j]);
#pragma unroll
            for (int q = 0; q < 8; ++q) v[q] += wk[j] * __bfloat162float(hh[q]);
          }
      }
    }
    const __nv_bfloat16* r = reinterpret_cast<const __nv_bfloat16*>(&rr);
    __align__(16) __nv_bfloat16 sum8[8];
    float ss = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float hq = __bfloat162float(__float2bfloat16(v[q]));  // the combined row, rounded as stored
      sum8[q] = __float2bfloat16(hq + __bfloat162float(r[q]));
      v[q] = __bfloat162float(sum8[q]);
      ss += v[q] * v[q];
    }
    *reinterpret_cast<uint4*>(residual + (size_t)t * H + c) = *reinterpret_cast<uint4*>(sum8);
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kWarpsCN; ++w) tot += red[w];
    const float inv = rsqrtf(tot / H + eps);
    const __nv_bfloat16* wh = reinterpret_cast<const __nv_bfloat16*>(&wr);
    __align__(16) __nv_bfloat16 o8[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) o8[q] = __float2bfloat16(v[q] * inv * __bfloat162float(wh[q]));
    *reinterpret_cast<uint4*>(out + (size_t)t * H + c) = *reinterpret_cast<uint4*>(o8);
    __syncthreads();  // red[] is reused by the next token
  }
  __syncthreads();
  __shared__ int last;
  if (threadIdx.x == 0) last = atomicAdd(&a.done[2], 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (last && threadIdx.x == 0) {
    *a.epoch = epoch;  // every kernel of this call has read the old value
    a.done[2] = 0;
  }
}

// ---------------------------------------------------------------- host
static EpArgs make_args(const at::Tensor& peers, int64_t rank, int64_t N, int64_t C, int64_t H, int64_t El,
                        at::Tensor& state) {
  TORCH_CHECK(peers.scalar_type() == at::kLong && peers.numel() == N && peers.is_cuda());
  TORCH_CHECK(state.scalar_type() == at::kInt && state.numel() >= 8 + N && state.is_cuda());
  TORCH_CHECK(H % 8 == 0 && N <= 64 && El <= 1024);
  EpArgs a;
  a.peers = reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>());
  a.rank = (int)rank;
  a.N = (int)N;
  a.C = (int)C;
  a.H = (int)H;
  a.El = (int)El;
  a.L = ep_layout(N, C, H);
  int* s = state.data_ptr<int>();
  a.epoch = reinterpret_cast<uint32_t*>(s);  // state[0]
  a.done = s + 4;                             // state[4..7]
  a.send_cnt = s + 8;                         // state[8..8+N)
  a.status = status_ptr(peers.device().index());
  return a;
}

// Runs the dispatch half: ids [T, K] int32 (global expert ids) -> rows in the
// owners' exchange buffers; on return (stream order) this rank's xs holds its
// received rows in local-expert order with offs [El+1].
void ep_dispatch(const at::Tensor& peers, at::Tensor& state, int64_t rank, int64_t C, int64_t El,
                 const at::Tensor& x, const at::Tensor& ids, at::Tensor& map, at::Tensor& row_pos, at::Tensor& offs,
                 at::Tensor& xs, at::Tensor& abort) {
  const int64_t N = peers.numel(), T = x.size(0), H = x.size(1), K = ids.size(1);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && ids.scalar_type() == at::kInt);
  TORCH_CHECK(T * K <= C, "ep_dispatch: T*K (", T * K, ") exceeds capacity ", C);
  TORCH_CHECK(row_pos.numel() >= N * C && offs.numel() >= El + 1 && xs.size(0) >= N * C && map.numel() >= T * K);
  EpArgs a = make_args(peers, rank, N, C, H, El, state);
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int TK = (int)(T * K);
  const int grid = std::max(1, std::min(148, (TK + 7) / 8));
  launch_k(ep_dispatch_kernel, grid, 256, 0, st, a, reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
           ids.data_ptr<int>(), TK, (int)K, map.data_ptr<int>());
  launch_k(ep_recv_kernel, 1, 1024, 0, st, a, row_pos.data_ptr<int>(), offs.data_ptr<int>(), abort.data_ptr<int>());
  const int rows = (int)(N * C);
  launch_k(ep_permute_kernel, std::max(1, std::min(296, (rows + 7) / 8)), 256, 0, st, a,
           (const int*)row_pos.data_ptr<int>(), reinterpret_cast<__nv_bfloat16*>(xs.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Direct-placement dispatch: routing outputs (ids [T, K], per-expert counts [E],
// offs_g [E+1], cursor [E] zeroed by the routing step) -> rows in the owners' expert-ordered
// xs (this rank's own xs is the exchange buffer's receive region, offsets in
// offs [El+1]).  The owner's gate/up GEMM must wait on flag_d (see
// ep_flag_addr) before reading xs.
void ep_dispatch2(const at::Tensor& peers, at::Tensor& state, int64_t rank, int64_t C, int64_t El,
                  const at::Tensor& x, const at::Tensor& ids, const at::Tensor& counts, const at::Tensor& offs_g,
                  at::Tensor& cursor, at::Tensor& map, at::Tensor& offs) {
  const int64_t N = peers.numel(), T = x.size(0), H = x.size(1), K = ids.size(1);
  const int64_t E = N * El;
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && ids.scalar_type() == at::kInt);
  TORCH_CHECK(T * K <= C, "ep_dispatch2: T*K (", T * K, ") exceeds capacity ", C);
  TORCH_CHECK(E <= kEpMaxExperts && counts.numel() >= E && offs_g.numel() >= E && cursor.numel() >= E &&
              offs.numel() >= El + 1 && map.numel() >= T * K);
  EpArgs a = make_args(peers, rank, N, C, H, El, state);
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int TK = (int)(T * K);
  const int threads = (int)std::max<int64_t>(256, (E + 31) / 32 * 32);
  const int grid = std::max(1, std::min(148, (TK + threads / 32 - 1) / (threads / 32)));
  const size_t smem = (size_t)(4 * E + 32) * sizeof(int);
  launch_k(ep_dispatch2_kernel, grid, threads, smem, st, a, reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
           (const int*)ids.data_ptr<int>(), (const int*)counts.data_ptr<int>(), (const int*)offs_g.data_ptr<int>(),
           cursor.data_ptr<int>(), TK, (int)K, map.data_ptr<int>(), offs.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Fused route + dispatch: x [T, H] bf16, router weight wr [E, H] bf16 ->
// ids / wts [T, K], map [T*K], this rank's xs offsets offs [El + 1], rows in the
// owners' receive regions.  scratch: int32 [2E + 2] (counts, cursor, barrier
// counters; zero before the first call, left zero by every call), logits f32 [>= T*E].
void ep_route_dispatch(const at::Tensor& peers, at::Tensor& state, int64_t rank, int64_t C, int64_t El,
                       const at::Tensor& x, const at::Tensor& wr, int64_t K, bool renorm, at::Tensor& ids,
                       at::Tensor& wts, at::Tensor& map, at::Tensor& offs, at::Tensor& scratch, at::Tensor& logits,
                       const c10::optional<at::Tensor>& pos_map, const c10::optional<at::Tensor>& trace) {
  const int64_t N = peers.numel(), T = x.size(0), H = x.size(1);
  const int64_t E = N * El;
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && wr.scalar_type() == at::kBFloat16 &&
              wr.is_contiguous() && wr.size(0) == E && wr.size(1) == H);
  TORCH_CHECK(H % 256 == 0, "ep_route_dispatch: hidden size must be a multiple of 256");
  TORCH_CHECK(T * K <= C, "ep_route_dispatch: T*K (", T * K, ") exceeds capacity ", C);
  TORCH_CHECK(E <= kEpMaxExperts && K <= 32 && K <= E);
  TORCH_CHECK(ids.numel() >= T * K && wts.numel() >= T * K && map.numel() >= T * K && offs.numel() >= El + 1 &&
              scratch.scalar_type() == at::kInt && scratch.numel() >= 2 * E + 2 &&
              logits.scalar_type() == at::kFloat && logits.numel() >= T * E);
  if (T == 0) return;
  EpArgs a = make_args(peers, rank, N, C, H, El, state);
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  int sms = 0;
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, x.device().index()));
  const int64_t tiles = ((E + kRdTileE - 1) / kRdTileE) * ((T + kRdTileT - 1) / kRdTileT);
  const int64_t pair_ctas = (T * K + kRdThreads / 32 - 1) / (kRdThreads / 32);
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(sms, std::max(tiles, pair_ctas)));
  int* sc = scratch.data_ptr<int>();
  uint64_t* tr = nullptr;
  if (trace && trace->defined()) {
    TORCH_CHECK(trace->scalar_type() == at::kLong && trace->numel() >= 8);
    tr = reinterpret_cast<uint64_t*>(trace->data_ptr<int64_t>());
  }
  int* pm = nullptr;
  if (pos_map && pos_map->defined()) {
    TORCH_CHECK(pos_map->scalar_type() == at::kInt && pos_map->numel() >= T * K);
    pm = pos_map->data_ptr<int>();
  }
  const int epl = (int)((E + 31) / 32);
  const size_t rd_smem = (size_t)(kRdTileE + kRdTileT) * H * 2;  // router rows + token rows of one tile
  TORCH_CHECK(rd_smem <= 160 * 1024, "ep_route_dispatch: hidden size too large for the router tile");
  static bool rd_attr[4] = {false, false, false, false};
#define MB_RD(P)                                                                                                   \
  do {                                                                                                             \
  {                                                                                                                \
    const int ai = P == 4 ? 0 : P == 8 ? 1 : P == 16 ? 2 : 3;                                                      \
    if (!rd_attr[ai]) {                                                                                            \
      C10_CUDA_CHECK(cudaFuncSetAttribute(ep_route_dispatch_kernel<P>, cudaFuncAttributeMaxDynamicSharedMemorySize,  \
                                          160 * 1024));                                                            \
      rd_attr[ai] = true;                                                                                          \
    }                                                                                                              \
  }                                                                                                                \
  launch_k(ep_route_dispatch_kernel<P>, grid, kRdThreads, rd_smem, st, a, reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), \
           reinterpret_cast<const __nv_bfloat16*>(wr.data_ptr()), (int)T, (int)K, (int)renorm, logits.data_ptr<float>(), \
           ids.data_ptr<int>(), wts.data_ptr<float>(), sc, sc + E, map.data_ptr<int>(), offs.data_ptr<int>(), sc + 2 * E, \
           pm, tr);                                                                                                 \
  } while (0)
  if (epl <= 4) MB_RD(4);
  else if (epl <= 8) MB_RD(8);
  else if (epl <= 16) MB_RD(16);
  else MB_RD(32);
#undef MB_RD
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Byte address of this rank's flag_d array (the gate/up GEMM waits on it).
int64_t ep_flag_addr(const at::Tensor& peers, int64_t rank, int64_t C, int64_t H) {
  const EpLayout L = ep_layout(peers.numel(), C, H);
  const int64_t own = peers.to(at::kCPU).data_ptr<int64_t>()[rank];
  return own + L.flag_d;
}

// Byte address of this rank's receive region (the expert-ordered xs of the direct dispatch).
int64_t ep_recv_addr(const at::Tensor& peers, int64_t rank, int64_t C, int64_t H) {
  const EpLayout L = ep_layout(peers.numel(), C, H);
  return peers.to(at::kCPU).data_ptr<int64_t>()[rank] + L.recv_x;
}

// Combine after the direct dispatch: y [>= offs[El], H] in xs order.
void ep_combine2(const at::Tensor& peers, at::Tensor& state, int64_t rank, int64_t C, int64_t El,
                 const at::Tensor& offs, const at::Tensor& y, const at::Tensor& map, const at::Tensor& wts,
                 const c10::optional<at::Tensor>& residual, at::Tensor& out) {
  const int64_t N = peers.numel(), T = out.size(0), H = out.size(1), K = wts.size(1);
  TORCH_CHECK(y.scalar_type() == at::kBFloat16 && y.is_contiguous() && out.is_contiguous());
  EpArgs a = make_args(peers, rank, N, C, H, El, state);
  c10::cuda::CUDAGuard guard(y.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int rows = (int)(N * C);
  launch_k(ep_combine_send2_kernel, std::max(1, std::min(296, (rows + 7) / 8)), 256, 0, st, a,
           (const int*)offs.data_ptr<int>(), reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()));
  const __nv_bfloat16* r =
      (residual && residual->defined()) ? reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr()) : nullptr;
  launch_k(ep_combine_reduce_kernel, (int)std::max<int64_t>(1, T), 256, 0, st, a, (const int*)map.data_ptr<int>(),
           (const float*)wts.data_ptr<float>(), (int)T, (int)K, r, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Combine, first half: the owner returns its expert outputs y to their
// sources' comb slots (the weighted sum follows in ep_combine_norm).
void ep_combine_send(const at::Tensor& peers, at::Tensor& state, int64_t rank, int64_t C, int64_t El,
                     const at::Tensor& offs, const at::Tensor& y, int64_t H) {
  const int64_t N = peers.numel();
  TORCH_CHECK(y.scalar_type() == at::kBFloat16 && y.is_contiguous() && y.size(1) == H);
  EpArgs a = make_args(peers, rank, N, C, H, El, state);
  c10::cuda::CUDAGuard guard(y.device());
  const int rows = (int)(N * C);
  launch_k(ep_combine_send2_kernel, std::max(1, std::min(296, (rows + 7) / 8)), 256, 0,
           at::cuda::getCurrentCUDAStream(), a, (const int*)offs.data_ptr<int>(),
           reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Combine, second half, fused with the next add + RMSNorm:
// residual [T, H] += sum_k wts * comb rows; out = rmsnorm(residual) * w.
void ep_combine_norm(const at::Tensor& peers, at::Tensor& state, int64_t rank, int64_t C, int64_t El,
                     const at::Tensor& map, const at::Tensor& wts, at::Tensor& residual, const at::Tensor& w,
                     at::Tensor& out, double eps, const c10::optional<at::Tensor>& rows) {
  const int64_t N = peers.numel(), T = out.size(0), H = out.size(1), K = wts.size(1);
  TORCH_CHECK(residual.scalar_type() == at::kBFloat16 && residual.is_contiguous() && residual.size(0) == T &&
              residual.size(1) == H && out.is_contiguous() && w.numel() == H && w.is_contiguous());
  EpArgs a = make_args(peers, rank, N, C, H, El, state);
  c10::cuda::CUDAGuard guard(out.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int grid = (int)std::max<int64_t>(1, T);  // CTA per token
  auto r = reinterpret_cast<__nv_bfloat16*>(residual.data_ptr());
  auto pw = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  auto po = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  const __nv_bfloat16* pr = nullptr;
  if (rows && rows->defined()) {
    TORCH_CHECK(N == 1 && rows->scalar_type() == at::kBFloat16 && rows->is_contiguous() && rows->size(1) == H,
                "ep_combine_norm: local rows only on a single rank");
    pr = reinterpret_cast<const __nv_bfloat16*>(rows->data_ptr());
  }
#define MB_CN(HH)                                                                                               \
  case HH:                                                                                                      \
    launch_k(ep_combine_norm_kernel<HH>, grid, HH / 8, 0, st, a, (const int*)map.data_ptr<int>(),              \
             (const float*)wts.data_ptr<float>(), (int)T, (int)K, r, pw, po, (float)eps, pr);                  \
    break;
  switch (H) {
    MB_CN(256) MB_CN(512) MB_CN(1024) MB_CN(2048) MB_CN(3072) MB_CN(4096)
    default:
      TORCH_CHECK(false, "ep_combine_norm: hidden size ", H, " not compiled");
  }
#undef MB_CN
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Receive step alone (fault tests: a wait for flags no peer writes must time
// out, record kErrPeerTimeout and return, leaving the context usable).
void ep_recv_only(const at::Tensor& peers, at::Tensor& state, int64_t rank, int64_t C, int64_t El, int64_t H,
                  at::Tensor& row_pos, at::Tensor& offs, at::Tensor& abort) {
  EpArgs a = make_args(peers, rank, peers.numel(), C, H, El, state);
  c10::cuda::CUDAGuard guard(peers.device());
  launch_k(ep_recv_kernel, 1, 1024, 0, at::cuda::getCurrentCUDAStream(), a, row_pos.data_ptr<int>(),
           offs.data_ptr<int>(), abort.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Combine half: y [N*C, H] expert outputs in xs order -> out [T, H].
void ep_combine(const at::Tensor& peers, at::Tensor& state, int64_t rank, int64_t C, int64_t El,
                const at::Tensor& row_pos, const at::Tensor& y, const at::Tensor& map, const at::Tensor& wts,
                const c10::optional<at::Tensor>& residual, at::Tensor& out) {
  const int64_t N = peers.numel(), T = out.size(0), H = out.size(1), K = wts.size(1);
  TORCH_CHECK(y.scalar_type() == at::kBFloat16 && y.is_contiguous() && out.is_contiguous());
  EpArgs a = make_args(peers, rank, N, C, H, El, state);
  c10::cuda::CUDAGuard guard(y.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int rows = (int)(N * C);
  launch_k(ep_combine_send_kernel, std::max(1, std::min(296, (rows + 7) / 8)), 256, 0, st, a,
           (const int*)row_pos.data_ptr<int>(), reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()));
  const __nv_bfloat16* r =
      (residual && residual->defined()) ? reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr()) : nullptr;
  launch_k(ep_combine_reduce_kernel, (int)std::max<int64_t>(1, T), 256, 0, st, a, (const int*)map.data_ptr<int>(),
           (const float*)wts.data_ptr<float>(), (int)T, (int)K, r, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ---------------------------------------------------------------- IPC buffers
// Exchange buffers are plain cudaMalloc allocations shared with CUDA IPC
// handles (no multicast objects).
std::tuple<int64_t, std::string> ipc_alloc(int64_t bytes) {
  void* p = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&p, bytes));
  C10_CUDA_CHECK(cudaMemset(p, 0, bytes));
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, p));
  return {reinterpret_cast<int64_t>(p), std::string(reinterpret_cast<const char*>(&h), sizeof(h))};
}

int64_t ipc_open(const std::string& handle) {
  TORCH_CHECK(handle.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr) { C10_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr))); }
void ipc_free(int64_t ptr) { C10_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(ptr))); }

}  // namespace mb
