// Tensor-parallel plumbing over NVLink peer memory (no NCCL on these paths).
//
// Every rank owns an exchange buffer (CUDA IPC, mapped into every peer):
//   ag    [peer_rows, H] bf16   this rank's normed activation shard (read by peers' GEMMs)
//   rs    [N, peer_rows, H]     reduce-scatter slots: partial rows from each source rank
//   ag_flags [N] u32            ag_flags[p] = boundary epoch once rank p's shard is published
//   rs_flags [N] u32            rs_flags[p] = epoch once rank p's partials for this rank are stored
// Sequence parallelism: the residual stream is split by tokens, rank r owns
// rows [r*peer_rows, (r+1)*peer_rows).  A layer boundary is
//   gather-GEMM (gemm.cu, activations loaded from the peers' ag buffers)
//   -> local attention / MLP math
//   -> scatter-GEMM (partials P2P-stored into the owners' rs slots)
//   -> tp_reduce (owner: wait flags, sum partials in rank order + residual,
//      RMSNorm, write its ag shard, advance the epoch, release ag flags).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "launch.cuh"
#include "status.h"

namespace mb {

CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dt, int64_t rows, int64_t cols, int64_t ld_bytes,
                         int box_cols, int box_rows, CUtensorMapSwizzle sw);

__device__ __forceinline__ uint32_t ld_acq(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// CTA per local row, H/8 threads, one 16-byte column chunk per thread: every
// load of the row (residual, x_add, the nsrc partial slots) is issued before
// any store, so a row costs about one memory round trip instead of one per
// chunk.  nsrc == 0: publish only (no partials to wait for).
__global__ void __launch_bounds__(1024)
    tp_reduce_kernel(const uint64_t* __restrict__ peers, int rank, int nranks, int nsrc, int rows, int H,
                     int64_t ag_off, int64_t rs_off, int64_t ag_flag_off, int64_t rs_flag_off, uint32_t* epoch,
                     int* done, const __nv_bfloat16* __restrict__ x_add, __nv_bfloat16* __restrict__ residual,
                     const __nv_bfloat16* __restrict__ w, float eps, __nv_bfloat16* __restrict__ local_out,
                     int* status) {
  pdl_wait();
  pdl_trigger();
  const uint32_t e = *epoch;
  const int t = blockIdx.x, tid = threadIdx.x;
  const int col = tid * 8;
  const uint64_t self = peers[rank];
  __shared__ float red[32];
  __shared__ int ok_all;
  if (tid == 0) ok_all = 1;
  __syncthreads();
  if (nsrc > 0) {
    const uint32_t* rf = reinterpret_cast<const uint32_t*>(self + rs_flag_off);
    for (int s = tid; s < nranks; s += blockDim.x) {
      const uint64_t t0 = globaltimer_ns();
      while ((int32_t)(ld_acq(rf + s) - e) < 0) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          set_status(status, kErrPeerTimeout);
          ok_all = 0;
          break;
        }
      }
    }
    __syncthreads();
    __threadfence();
  }
  const size_t off = (size_t)t * H + col;
  const uint4 rr = *reinterpret_cast<const uint4*>(residual + off);
  const uint4 xa = x_add ? *reinterpret_cast<const uint4*>(x_add + off) : make_uint4(0, 0, 0, 0);
  const uint4 wr = *reinterpret_cast<const uint4*>(w + col);
  float acc[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    acc[q] = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(&rr)[q]);
    if (x_add) acc[q] += __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(&xa)[q]);
  }
  if (ok_all && nsrc > 0) {
    const __nv_bfloat16* slots = reinterpret_cast<const __nv_bfloat16*>(self + rs_off);
    constexpr int kBatch = 8;  // partial loads in flight together; summed in fixed rank order
    for (int s0 = 0; s0 < nsrc; s0 += kBatch) {
      uint4 pr[kBatch];
#pragma unroll
      for (int j = 0; j < kBatch; ++j)
        if (s0 + j < nsrc) pr[j] = __ldcg(reinterpret_cast<const uint4*>(slots + ((size_t)(s0 + j) * rows + t) * H + col));
#pragma unroll
      for (int j = 0; j < kBatch; ++j)
        if (s0 + j < nsrc) {
#pragma unroll
          for (int q = 0; q < 8; ++q) acc[q] += __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(&pr[j])[q]);
        }
    }
  }
  __align__(16) __nv_bfloat16 hb[8];
  float v[8], ss = 0.f;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    hb[q] = __float2bfloat16(acc[q]);
    v[q] = __bfloat162float(hb[q]);
    ss += v[q] * v[q];
  }
  *reinterpret_cast<uint4*>(residual + off) = *reinterpret_cast<uint4*>(hb);
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
  const float inv = rsqrtf(tot / H + eps);
  __align__(16) __nv_bfloat16 o[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) o[q] = __float2bfloat16(v[q] * inv * __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(&wr)[q]));
  // all-gather by push: this row lands at gathered row rank*rows + t in every rank's buffer
  const size_t grow = (size_t)rank * rows + t;
  for (int p = 0; p < nranks; ++p)
    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(peers[p] + ag_off) + grow * H + col) =
        *reinterpret_cast<uint4*>(o);
  if (local_out) *reinterpret_cast<uint4*>(local_out + off) = *reinterpret_cast<uint4*>(o);
  // last CTA: advance the epoch and publish this rank's shard to every peer
  // CTA barrier, then one system-scope fence + arrive per CTA (cumulative over the CTA's stores)
  __syncthreads();
  __shared__ int last;
  if (threadIdx.x == 0) {
    __threadfence_system();
    last = atomicAdd(done, 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence_system();
  const uint32_t ne = e + 1;
  for (int p = threadIdx.x; p < nranks; p += blockDim.x) {
    uint32_t* f = reinterpret_cast<uint32_t*>(peers[p] + ag_flag_off) + rank;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(ne) : "memory");
  }
  if (threadIdx.x == 0) {
    *epoch = ne;
    *done = 0;
  }
}

void tp_reduce(const at::Tensor& peers, int64_t rank, bool with_partials, int64_t rows, int64_t H, int64_t ag_off,
               int64_t rs_off, int64_t ag_flag_off, int64_t rs_flag_off, at::Tensor& state,
               const c10::optional<at::Tensor>& x_add, at::Tensor& residual, const at::Tensor& w, double eps,
               const c10::optional<at::Tensor>& local_out) {
  TORCH_CHECK(H % 256 == 0 && H / 256 <= 32, "tp_reduce: hidden size must be a multiple of 256 (<= 8192)");
  TORCH_CHECK(residual.is_contiguous() && residual.size(0) == rows && residual.size(1) == H);
  const int N = (int)peers.numel();
  c10::cuda::CUDAGuard guard(residual.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  int* s = state.data_ptr<int>();
  auto bf = [](const c10::optional<at::Tensor>& t) -> __nv_bfloat16* {
    return (t && t->defined()) ? reinterpret_cast<__nv_bfloat16*>(t->data_ptr()) : nullptr;
  };
  const uint64_t* pp = reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>());
  auto* res = reinterpret_cast<__nv_bfloat16*>(residual.data_ptr());
  auto* ww = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  const int grid = (int)std::max<int64_t>(1, rows);
  launch_k(tp_reduce_kernel, grid, (int)(H / 8), 0, st, pp, (int)rank, N, with_partials ? N : 0, (int)rows, (int)H,
           ag_off, rs_off, ag_flag_off, rs_flag_off, reinterpret_cast<uint32_t*>(s), s + 5,
           (const __nv_bfloat16*)bf(x_add), res, ww, (float)eps, bf(local_out), status_ptr(residual.device().index()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Split-K reduce-scatter: sums the fp32 partials of the row-parallel GEMM,
// rounds to bf16 and stores each row once, into its owner's slot for this
// rank; the last CTA releases the owners' flags.  CTA per token row.
__global__ void __launch_bounds__(1024) tp_splitk_scatter_kernel(const float* __restrict__ ws, int splits, int T, int H, int peer_rows,
                                         const uint64_t* __restrict__ peers, int rank, int nranks, int64_t rs_off,
                                         int64_t rs_flag_off, const uint32_t* epoch, int* done) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const int d = t / peer_rows, jl = t - d * peer_rows;
  __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(peers[d] + rs_off) + ((size_t)rank * peer_rows + jl) * H;
  for (int c = threadIdx.x * 4; c < H; c += blockDim.x * 4) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < splits; s0 += 8) {  // 8 split partials in flight, summed in split order
      float4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (s0 + j < splits) v[j] = *reinterpret_cast<const float4*>(ws + ((size_t)(s0 + j) * T + t) * H + c);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (s0 + j < splits) {
          acc.x += v[j].x; acc.y += v[j].y; acc.z += v[j].z; acc.w += v[j].w;
        }
    }
    __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
    reinterpret_cast<__nv_bfloat162*>(dst + c)[0] = lo;
    reinterpret_cast<__nv_bfloat162*>(dst + c)[1] = hi;
  }
  // CTA barrier, then one system-scope fence + arrive per CTA (cumulative over the CTA's stores)
  __syncthreads();
  __shared__ int last;
  if (threadIdx.x == 0) {
    __threadfence_system();
    last = atomicAdd(done, 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence_system();
  const uint32_t e = *epoch;
  for (int p = threadIdx.x; p < nranks; p += blockDim.x) {
    uint32_t* f = reinterpret_cast<uint32_t*>(peers[p] + rs_flag_off) + rank;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(e) : "memory");
  }
  if (threadIdx.x == 0) *done = 0;
}

void tp_splitk_scatter(const at::Tensor& ws, int64_t splits, int64_t T, int64_t H, int64_t peer_rows,
                       const at::Tensor& peers, int64_t rank, int64_t rs_off, int64_t rs_flag_off, at::Tensor& state) {
  c10::cuda::CUDAGuard guard(ws.device());
  int* s = state.data_ptr<int>();
  const int threads = (int)std::min<int64_t>(1024, std::max<int64_t>(32, H / 4));
  launch_k(tp_splitk_scatter_kernel, (int)T, threads, 0, at::cuda::getCurrentCUDAStream(), (const float*)ws.data_ptr<float>(),
           (int)splits, (int)T, (int)H, (int)peer_rows, reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>()),
           (int)rank, (int)peers.numel(), rs_off, rs_flag_off, reinterpret_cast<const uint32_t*>(s), s + 6);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Bounded wait, one warp: every rank's shard of the current epoch is published
// (flags live in this rank's own buffer, written by the peers).
__global__ void tp_wait_flags_kernel(const uint64_t* __restrict__ peers, int rank, int nranks, int64_t ag_flag_off,
                                     const uint32_t* epoch, int* status) {
  pdl_wait();
  pdl_trigger();
  const uint32_t e = *epoch;
  const uint32_t* f = reinterpret_cast<const uint32_t*>(peers[rank] + ag_flag_off);
  for (int p = threadIdx.x; p < nranks; p += blockDim.x) {
    const uint64_t t0 = globaltimer_ns();
    while ((int32_t)(ld_acq(f + p) - e) < 0) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        set_status(status, kErrPeerTimeout);
        break;
      }
    }
  }
}

// out[i] = row idx[i] of the gathered (published) shards, read over NVLink.
__global__ void tp_gather_rows_kernel(const uint64_t* __restrict__ peers, int peer_rows, int64_t ag_off,
                                      const int64_t* __restrict__ idx, int H, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int64_t g = idx[blockIdx.x];
  (void)peer_rows;
  const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(peers[0] + ag_off) + (size_t)g * H;
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8)
    *reinterpret_cast<uint4*>(out + (size_t)blockIdx.x * H + c) = __ldcg(reinterpret_cast<const uint4*>(src + c));
}

void tp_gather_rows(const at::Tensor& peers, int64_t rank, int64_t peer_rows, int64_t ag_off, int64_t ag_flag_off,
                    at::Tensor& state, const at::Tensor& idx, at::Tensor& out) {
  const int B = (int)idx.numel(), H = (int)out.size(1);
  if (B == 0) return;
  c10::cuda::CUDAGuard guard(out.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const uint64_t* pp = reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>());
  launch_k(tp_wait_flags_kernel, 1, 32, 0, st, pp, (int)rank, (int)peers.numel(), ag_flag_off,
           reinterpret_cast<const uint32_t*>(state.data_ptr<int>()), status_ptr(out.device().index()));
  launch_k(tp_gather_rows_kernel, B, 128, 0, st, pp + rank, (int)peer_rows, ag_off, (const int64_t*)idx.data_ptr<int64_t>(), H,
           reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------ vision -> LLM rows
// Release only (a rank with no visual rows in this step): flags[rank] = state[0] + 1 at every rank.
__global__ void vis_release_kernel(const uint64_t* __restrict__ peers, int rank, int nranks, int64_t flag_off,
                                   const uint32_t* epoch) {
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const uint32_t e = *epoch + 1;
    for (int p = 0; p < nranks; ++p)
      asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(reinterpret_cast<uint32_t*>(peers[p] + flag_off) + rank),
                   "r"(e)
                   : "memory");
  }
}

// One CTA: bounded wait until every rank released this step's visual rows, then
// h[rows[i]] = buf[rows[i]] (this rank's shard rows that hold image tokens), then
// advance the epoch.
__global__ void __launch_bounds__(1024)
    vis_wait_merge_kernel(const uint64_t* __restrict__ peers, int rank, int nranks, int64_t off, int64_t flag_off,
                          uint32_t* epoch, const int* __restrict__ rows, int nrows, int H,
                          __nv_bfloat16* __restrict__ h, int* status) {
  pdl_wait();
  pdl_trigger();
  const uint32_t e = *epoch + 1;
  const uint64_t self = peers[rank];
  __shared__ int ok_all;
  if (threadIdx.x == 0) ok_all = 1;
  __syncthreads();
  const uint32_t* f = reinterpret_cast<const uint32_t*>(self + flag_off);
  for (int p = threadIdx.x; p < nranks; p += blockDim.x) {
    const uint64_t t0 = globaltimer_ns();
    while ((int32_t)(ld_acq(f + p) - e) < 0) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        set_status(status, kErrPeerTimeout);
        ok_all = 0;
        break;
      }
    }
  }
  __syncthreads();
  __threadfence();
  const __nv_bfloat16* buf = reinterpret_cast<const __nv_bfloat16*>(self + off);
  const int n16 = H / 8;
  for (int i = threadIdx.x; ok_all && i < nrows * n16; i += blockDim.x) {
    const int r = rows[i / n16], c = i % n16;
    reinterpret_cast<uint4*>(h + (size_t)r * H)[c] = __ldcg(reinterpret_cast<const uint4*>(buf + (size_t)r * H) + c);
  }
  __syncthreads();
  if (threadIdx.x == 0) *epoch = e;
}

void vis_release(const at::Tensor& peers, int64_t rank, int64_t flag_off, at::Tensor& state) {
  c10::cuda::CUDAGuard guard(peers.device());
  launch_k(vis_release_kernel, 1, 32, 0, at::cuda::getCurrentCUDAStream(),
           reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>()), (int)rank, (int)peers.numel(), flag_off,
           reinterpret_cast<const uint32_t*>(state.data_ptr<int>()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void vis_wait_merge(const at::Tensor& peers, int64_t rank, int64_t off, int64_t flag_off, at::Tensor& state,
                    const at::Tensor& rows, at::Tensor& h) {
  TORCH_CHECK(h.scalar_type() == at::kBFloat16 && h.is_contiguous() && h.size(1) % 8 == 0);
  TORCH_CHECK(rows.scalar_type() == at::kInt && rows.is_contiguous());
  c10::cuda::CUDAGuard guard(h.device());
  launch_k(vis_wait_merge_kernel, 1, 1024, 0, at::cuda::getCurrentCUDAStream(),
           reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>()), (int)rank, (int)peers.numel(), off, flag_off,
           reinterpret_cast<uint32_t*>(state.data_ptr<int>()), (const int*)rows.data_ptr<int>(), (int)rows.numel(),
           (int)h.size(1), reinterpret_cast<__nv_bfloat16*>(h.data_ptr()), status_ptr(h.device().index()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------ vocab-parallel greedy LM head
// Each rank holds rows [r*V/N, (r+1)*V/N) of the LM head and has found, per
// token row, the best logit of its slice (value + global index, argmax kernel
// with an index offset).  One CTA: the pairs are stored into slot [rank][t] of
// every rank's exchange buffer over NVLink, one fence + release flag per rank,
// then a bounded wait for every peer's flag and a reduction over the ranks in
// order (strictly greater wins, so a tie keeps the lower rank = lower index, as
// a full-vocabulary argmax does).  8 bytes per token row cross each link
// instead of the all-gathered logits.
struct ValIdx {
  float v;
  int i;
};

__global__ void __launch_bounds__(1024)
    tp_argmax_exchange_kernel(const uint64_t* __restrict__ peers, int rank, int nranks, int cap, int64_t slot_off,
                              int64_t flag_off, uint32_t* epoch, const float* __restrict__ vals,
                              const int64_t* __restrict__ idxs, int T, int64_t* __restrict__ out, int* status) {
  pdl_wait();
  pdl_trigger();
  const uint32_t e = *epoch + 1;
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    ValIdx vi;
    vi.v = vals[t];
    vi.i = (int)idxs[t];
    const uint64_t packed = *reinterpret_cast<const uint64_t*>(&vi);
    for (int p = 0; p < nranks; ++p)
      reinterpret_cast<uint64_t*>(peers[p] + slot_off)[(size_t)rank * cap + t] = packed;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int p = 0; p < nranks; ++p)
      asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(reinterpret_cast<uint32_t*>(peers[p] + flag_off) + rank),
                   "r"(e)
                   : "memory");
  }
  __shared__ int ok_all;
  if (threadIdx.x == 0) ok_all = 1;
  __syncthreads();
  const uint64_t self = peers[rank];
  const uint32_t* f = reinterpret_cast<const uint32_t*>(self + flag_off);
  for (int p = threadIdx.x; p < nranks; p += blockDim.x) {
    const uint64_t t0 = globaltimer_ns();
    while ((int32_t)(ld_acq(f + p) - e) < 0) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        set_status(status, kErrPeerTimeout);
        ok_all = 0;
        break;
      }
    }
  }
  __syncthreads();
  __threadfence();
  const uint64_t* slots = reinterpret_cast<const uint64_t*>(self + slot_off);
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    float bv = -INFINITY;
    int bi = 0;
    for (int p = 0; ok_all && p < nranks; ++p) {
      const uint64_t raw = __ldcg(reinterpret_cast<const unsigned long long*>(slots + (size_t)p * cap + t));
      const ValIdx vi = *reinterpret_cast<const ValIdx*>(&raw);
      if (p == 0 || vi.v > bv) {
        bv = vi.v;
        bi = vi.i;
      }
    }
    out[t] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) *epoch = e;
}

void tp_argmax_exchange(const at::Tensor& peers, int64_t rank, int64_t cap, int64_t slot_off, int64_t flag_off,
                        at::Tensor& state, const at::Tensor& vals, const at::Tensor& idxs, at::Tensor& out) {
  const int T = (int)vals.numel();
  TORCH_CHECK(vals.scalar_type() == at::kFloat && idxs.scalar_type() == at::kLong && out.scalar_type() == at::kLong);
  TORCH_CHECK(idxs.numel() == T && out.numel() == T && T <= cap, "tp_argmax_exchange: ", T, " rows > capacity ", cap);
  TORCH_CHECK(slot_off % 8 == 0 && flag_off % 4 == 0);
  if (T == 0) return;
  c10::cuda::CUDAGuard guard(out.device());
  const int threads = std::min(1024, std::max(32, (T + 31) / 32 * 32));
  launch_k(tp_argmax_exchange_kernel, 1, threads, 0, at::cuda::getCurrentCUDAStream(),
           reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>()), (int)rank, (int)peers.numel(), (int)cap,
           slot_off, flag_off, reinterpret_cast<uint32_t*>(state.data_ptr<int>()), vals.data_ptr<float>(),
           idxs.data_ptr<int64_t>(), T, out.data_ptr<int64_t>(), status_ptr(out.device().index()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mb
