// Expert parallelism as all-gather -> local experts -> reduce-scatter over
// NVLink multicast (NVLS), for decode-sized steps.
//
// The residual stream stays sharded by token (data-parallel attention: rank r
// owns its T_r tokens).  One MoE layer:
//   1. publish (ep_agrs_publish_kernel, CTA per own token): the token's normed
//      row, its top-k expert ids and routing weights are written into every
//      rank's gathered arrays with multimem stores (each byte leaves the GPU
//      once; the switch replicates it), plus this rank's token count; the last
//      CTA releases this rank's all-gather flag with one multicast store.
//   2. place (ep_agrs_place_kernel): after a bounded wait for every rank's
//      flag, each CTA computes the same deterministic placement of the pairs
//      (token, k) whose expert is local: expert-major, then rank, token and k
//      order.  CTA c then copies its share of the rows from the local gathered
//      buffer into the grouped GEMM input and records each pair's row.
//   3. grouped gate/up + SwiGLU and down GEMMs over the local experts (gemm.cu).
//   4. combine (ep_agrs_combine_kernel, CTA per gathered token): this rank's
//      weighted sum over the token's local pairs, in k order, into its `part`
//      row (zeros for a token with no local expert).
//   5. reduce (tp_nvls_reduce_kernel, tp_nvls.cu, no all-gather publish): the
//      owner of each token reads the sum of every rank's `part` row with one
//      multimem.ld_reduce, adds the residual and applies the next RMSNorm.
// Two cross-rank waits per layer (steps 2 and 5); routing needs no count
// exchange because every rank sees every token's expert ids.
//
// Buffer reuse: a rank overwrites its peers' gathered arrays (step 1 of the
// next layer) only after its own step 5, which waited for every rank's
// announcement of step 5, made after that rank's steps 2 and 4 (the only
// readers).  `part` is rewritten (next step 4) only after next step 2 waited
// for every rank's next step 1, which follows that rank's step 5 reads.
//
// The reference's MoE block (pio/models/qwen3_coder_30b/model.py:308-353)
// loops over experts on one device.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "launch.cuh"
#include "multimem.cuh"
#include "status.h"

namespace mb {

struct AgrsArgs {
  uint64_t self, mc;       // unicast base of this rank's symmetric buffer, multicast base
  int rank, N, cap, K, El, H;
  int64_t gx_off;          // [N*cap, H] bf16 gathered normed rows (row r*cap + t)
  int64_t gid_off;         // [N*cap, K] int32 global expert ids
  int64_t gw_off;          // [N*cap, K] fp32 routing weights
  int64_t gcnt_off;        // [N] u32 tokens published by each rank
  int64_t part_off;        // [N*cap, H] bf16 this rank's weighted expert sums
  int64_t ag_flag_off;     // [N] u32
  const uint32_t* epoch;   // state[0]; advanced by the reduce kernel
  int* done;               // CTA-completion counter of the publish kernel
  int* status;
};

template <typename T>
__device__ __forceinline__ const T* loc(const AgrsArgs& a, int64_t off) {
  return reinterpret_cast<const T*>(a.self + off);
}

// Bounded wait for every rank's flag >= want; returns false (status recorded) on timeout.
__device__ bool agrs_wait_all(const AgrsArgs& a, uint32_t want) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  const uint32_t* f = loc<uint32_t>(a, a.ag_flag_off);
  for (int p = threadIdx.x; p < a.N; p += blockDim.x) {
    const uint64_t t0 = globaltimer_ns();
    while ((int32_t)(ld_acquire_sys_u32(f + p) - want) < 0) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        set_status(a.status, kErrPeerTimeout);
        ok = 0;
        break;
      }
    }
  }
  __syncthreads();
  __threadfence();
  return ok != 0;
}

// ------------------------------------------------------------------ 1. publish
// EPL logits per lane (E <= 32 * EPL).  Softmax over all E, top-K by repeated
// warp arg-max (ties: the lower expert id), weights p / sum or p / sum(top-K).
template <int EPL>
__global__ void __launch_bounds__(1024)
    ep_agrs_publish_kernel(AgrsArgs a, const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ logits,
                           int T, int E, int renorm) {
  pdl_wait();
  pdl_trigger();
  const uint32_t ne = *a.epoch + 1;
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, H = a.H, K = a.K;
  if (t < T) {
    const size_t g = (size_t)a.rank * a.cap + t;
    for (int c = tid * 8; c < H; c += blockDim.x * 8)
      mc_store_16(a.mc + a.gx_off + (g * H + c) * 2, *reinterpret_cast<const uint4*>(x + (size_t)t * H + c));
    if (tid < 32) {
      float v[EPL];
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < EPL; ++i) {
        const int e = i * 32 + lane;
        v[i] = e < E ? __bfloat162float(logits[(size_t)t * E + e]) : -INFINITY;
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
        if (my_id < 0 || my_id >= E || !(my_w == my_w)) {  // non-finite logits: never route with an invalid id
          set_status(a.status, kErrBounds);
          my_id = 0;
          my_w = 0.f;
        }
        mc_store_u32(a.mc + a.gid_off + (g * K + lane) * 4, (uint32_t)my_id);
        mc_store_f32(a.mc + a.gw_off + (g * K + lane) * 4, renorm ? my_w / picked : my_w);
      }
    }
  }
  if (t == 0 && tid == 0) mc_store_u32(a.mc + a.gcnt_off + 4ull * a.rank, (uint32_t)T);
  __shared__ int last;
  __syncthreads();
  if (tid == 0) {
    __threadfence_system();
    last = atomicAdd(a.done, 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (last && tid == 0) {
    __threadfence_system();
    mc_store_release_u32(a.mc + a.ag_flag_off + 4ull * a.rank, ne);
    *a.done = 0;
  }
}

// ------------------------------------------------------------------ 2. place
// Deterministic placement, computed identically by every CTA (1024 threads):
// pair p enumerates (rank r, token t < T_r, k) in that order; warp w owns the
// contiguous pair range [w*ch, (w+1)*ch).  Pass 1 counts each warp's local
// pairs per expert (lanes with equal experts found with __match_any_sync),
// a scan over (expert, warp) gives every warp's first row per expert, and
// pass 2 assigns rows in pair order.  Rows of expert e are
// [eoff[e], eoff[e+1]) of xs.
__global__ void __launch_bounds__(1024)
    ep_agrs_place_kernel(AgrsArgs a, __nv_bfloat16* __restrict__ xs, int xs_cap, int* __restrict__ slot_of,
                         int* __restrict__ offs, int max_pairs) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ int sm_place[];
  const int El = a.El, K = a.K, H = a.H;
  int* wbase = sm_place;                 // [32][El]: warp counts, then warp running rows
  int* eoff = wbase + 32 * El;           // [El + 1]
  int* place = eoff + El + 1;            // [max_pairs] row of each pair, -1 when not local
  __shared__ int pstart[65];             // first pair of each rank's tokens
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t ne = *a.epoch + 1;
  const bool ok = agrs_wait_all(a, ne);
  if (tid == 0) {
    const uint32_t* gcnt = loc<uint32_t>(a, a.gcnt_off);
    int acc = 0;
    for (int r = 0; r < a.N; ++r) {
      int c = ok ? (int)__ldcg(gcnt + r) : 0;
      c = c < 0 ? 0 : (c > a.cap ? a.cap : c);
      if (acc + c * K > max_pairs) {  // cannot happen when cap * N * K <= max_pairs (checked on the host)
        set_status(a.status, kErrCapacity);
        c = 0;
      }
      pstart[r] = acc;
      acc += c * K;
    }
    pstart[a.N] = acc;
  }
  for (int i = tid; i < 32 * El; i += blockDim.x) wbase[i] = 0;
  __syncthreads();
  const int P = pstart[a.N];
  const int ch = (P + 31) / 32;
  const int* gid = loc<int>(a, a.gid_off);
  // pair index -> (gathered row g, k, local expert or -1)
  auto pair_at = [&](int p, int& g, int& k) -> int {
    int r = 0;
    while (r + 1 < a.N && pstart[r + 1] <= p) ++r;
    const int q = p - pstart[r];
    const int t = q / K;
    k = q - t * K;
    g = r * a.cap + t;
    const int e = __ldcg(gid + (size_t)g * K + k) - a.rank * El;
    return (e >= 0 && e < El) ? e : -1;
  };
  const int p_lo = warp * ch, p_hi = min(P, p_lo + ch);
  // pass 1: per-warp counts
  for (int p0 = p_lo; p0 < p_hi; p0 += 32) {
    const int p = p0 + lane;
    int g = 0, k = 0;
    const int e = p < p_hi ? pair_at(p, g, k) : -1;
    const unsigned m = __match_any_sync(0xffffffffu, e);
    if (e >= 0 && lane == __ffs(m) - 1) wbase[warp * El + e] += __popc(m);
    __syncwarp();
  }
  __syncthreads();
  // scan: warp-major within each expert, then over experts
  for (int e = tid; e < El; e += blockDim.x) {
    int run = 0;
    for (int w = 0; w < 32; ++w) {
      const int c = wbase[w * El + e];
      wbase[w * El + e] = run;
      run += c;
    }
    eoff[e + 1] = run;  // count for now
  }
  __syncthreads();
  if (tid == 0) {
    eoff[0] = 0;
    for (int e = 0; e < El; ++e) eoff[e + 1] += eoff[e];
    if (eoff[El] > xs_cap) set_status(a.status, kErrCapacity);
  }
  __syncthreads();
  // pass 2: rows in pair order
  for (int p0 = p_lo; p0 < p_hi; p0 += 32) {
    const int p = p0 + lane;
    int g = 0, k = 0;
    const int e = p < p_hi ? pair_at(p, g, k) : -1;
    const unsigned m = __match_any_sync(0xffffffffu, e);
    int row = -1;
    if (e >= 0) {
      row = eoff[e] + wbase[warp * El + e] + __popc(m & ((1u << lane) - 1u));
      if (row >= xs_cap) row = -1;
    }
    if (p < p_hi) place[p] = row;
    __syncwarp();
    if (e >= 0 && lane == __ffs(m) - 1) wbase[warp * El + e] += __popc(m);
    __syncwarp();
  }
  __syncthreads();
  if (blockIdx.x == 0)
    for (int e = tid; e <= El; e += blockDim.x) offs[e] = min(eoff[e], xs_cap);
  // this CTA's share: the pair map and the local rows
  const __nv_bfloat16* gx = loc<__nv_bfloat16>(a, a.gx_off);
  for (int p = blockIdx.x * 32 + warp; p < P; p += gridDim.x * 32) {
    int g = 0, k = 0;
    pair_at(p, g, k);
    const int row = place[p];
    if (lane == 0) slot_of[(size_t)g * K + k] = row;
    if (row < 0) continue;
    const uint4* src = reinterpret_cast<const uint4*>(gx + (size_t)g * H);
    uint4* dst = reinterpret_cast<uint4*>(xs + (size_t)row * H);
    for (int c = lane; c < H / 8; c += 32) dst[c] = __ldcg(src + c);
  }
}

// ------------------------------------------------------------------ 4. combine
// part[g] = bf16(sum_k w[g,k] * y[slot[g,k]]) over the local pairs of gathered
// token g, in k order (zeros when none).  CTA per gathered token, H/8 threads.
__global__ void __launch_bounds__(1024)
    ep_agrs_combine_kernel(AgrsArgs a, const int* __restrict__ slot_of, const __nv_bfloat16* __restrict__ y) {
  pdl_wait();
  pdl_trigger();
  const int g = blockIdx.x, r = g / a.cap, t = g - r * a.cap, K = a.K, H = a.H;
  const int tr = (int)__ldcg(loc<uint32_t>(a, a.gcnt_off) + r);
  if (t >= tr) return;  // no token there: the owner never reads this row
  const float* gw = loc<float>(a, a.gw_off);
  const int c = threadIdx.x * 8;
  float acc[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) acc[q] = 0.f;
  for (int k0 = 0; k0 < K; k0 += 8) {  // up to 8 expert rows in flight, summed in k order
    uint4 raw[8];
    float wk[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int k = k0 + j;
      const int s = k < K ? slot_of[(size_t)g * K + k] : -1;
      wk[j] = s >= 0 ? __ldcg(gw + (size_t)g * K + k) : 0.f;
      raw[j] = s >= 0 ? __ldcg(reinterpret_cast<const uint4*>(y + (size_t)s * H + c)) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const __nv_bfloat16* hh = reinterpret_cast<const __nv_bfloat16*>(&raw[j]);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += wk[j] * __bfloat162float(hh[q]);
    }
  }
  __align__(16) __nv_bfloat16 o[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) o[q] = __float2bfloat16(acc[q]);
  *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.self + a.part_off) + (size_t)g * H + c) =
      *reinterpret_cast<const uint4*>(o);
}

// ------------------------------------------------------------------ host
namespace {

AgrsArgs make_agrs(int64_t self, int64_t mc, int64_t rank, int64_t N, int64_t cap, int64_t K, int64_t El, int64_t H,
                   const at::Tensor& offsets, at::Tensor& state) {
  TORCH_CHECK(offsets.scalar_type() == at::kLong && offsets.numel() == 6 && offsets.device().is_cpu(),
              "ep_agrs: offsets = [gx, gid, gw, gcnt, part, ag_flag] (CPU int64)");
  TORCH_CHECK(state.scalar_type() == at::kInt && state.numel() >= 8 && state.is_cuda());
  TORCH_CHECK(self && mc, "ep_agrs: no symmetric / multicast mapping");
  TORCH_CHECK(N >= 1 && N <= 64 && K >= 1 && K <= 32 && El >= 1 && cap >= 1, "ep_agrs: bad sizes");
  TORCH_CHECK(H % 256 == 0 && H <= 8192, "ep_agrs: hidden size must be a multiple of 256 (<= 8192)");
  const int64_t* o = offsets.data_ptr<int64_t>();
  for (int i = 0; i < 6; ++i) TORCH_CHECK(o[i] % 16 == 0, "ep_agrs: misaligned buffer offset");
  AgrsArgs a{};
  a.self = (uint64_t)self;
  a.mc = (uint64_t)mc;
  a.rank = (int)rank;
  a.N = (int)N;
  a.cap = (int)cap;
  a.K = (int)K;
  a.El = (int)El;
  a.H = (int)H;
  a.gx_off = o[0];
  a.gid_off = o[1];
  a.gw_off = o[2];
  a.gcnt_off = o[3];
  a.part_off = o[4];
  a.ag_flag_off = o[5];
  int* s = state.data_ptr<int>();
  a.epoch = reinterpret_cast<const uint32_t*>(s);
  a.done = s + 6;
  a.status = status_ptr(state.device().index());
  return a;
}

}  // namespace

// x [T, H] normed rows of this rank's tokens, logits [T, E] (bf16 router output).
void ep_agrs_publish(int64_t self, int64_t mc, int64_t rank, int64_t N, int64_t cap, int64_t K, int64_t El,
                     const at::Tensor& offsets, at::Tensor& state, const at::Tensor& x, const at::Tensor& logits,
                     bool renorm) {
  const int64_t T = x.size(0), H = x.size(1), E = El * N;
  AgrsArgs a = make_agrs(self, mc, rank, N, cap, K, El, H, offsets, state);
  TORCH_CHECK(T <= cap, "ep_agrs_publish: ", T, " tokens exceed the per-rank capacity ", cap);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous());
  TORCH_CHECK(T == 0 || (logits.scalar_type() == at::kBFloat16 && logits.is_contiguous() && logits.size(0) == T &&
                         logits.size(1) == E));
  TORCH_CHECK(E <= 512 && K <= 32 && K <= E, "ep_agrs_publish: at most 512 experts");
  c10::cuda::CUDAGuard guard(state.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int grid = (int)std::max<int64_t>(T, 1), threads = (int)(H / 8);
  const auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  const auto* lp = T ? reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()) : nullptr;
  if (E <= 128)
    launch_k(ep_agrs_publish_kernel<4>, grid, threads, 0, st, a, xp, lp, (int)T, (int)E, renorm ? 1 : 0);
  else if (E <= 256)
    launch_k(ep_agrs_publish_kernel<8>, grid, threads, 0, st, a, xp, lp, (int)T, (int)E, renorm ? 1 : 0);
  else
    launch_k(ep_agrs_publish_kernel<16>, grid, threads, 0, st, a, xp, lp, (int)T, (int)E, renorm ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// xs [xs_cap, H] grouped GEMM input (local rows in expert order), slot_of [N*cap*K], offs [El + 1].
void ep_agrs_place(int64_t self, int64_t mc, int64_t rank, int64_t N, int64_t cap, int64_t K, int64_t El,
                   int64_t H, const at::Tensor& offsets, at::Tensor& state, at::Tensor& xs, at::Tensor& slot_of,
                   at::Tensor& offs, int64_t grid) {
  AgrsArgs a = make_agrs(self, mc, rank, N, cap, K, El, H, offsets, state);
  const int64_t max_pairs = N * cap * K;
  TORCH_CHECK(xs.scalar_type() == at::kBFloat16 && xs.is_contiguous() && xs.size(1) == H);
  TORCH_CHECK(slot_of.scalar_type() == at::kInt && slot_of.numel() >= max_pairs);
  TORCH_CHECK(offs.scalar_type() == at::kInt && offs.numel() >= El + 1);
  const int64_t smem = (32 * El + El + 1 + max_pairs) * 4;
  TORCH_CHECK(smem <= 200 * 1024, "ep_agrs_place: ", max_pairs, " pairs and ", El, " local experts exceed shared memory");
  c10::cuda::CUDAGuard guard(state.device());
  if (smem > 48 * 1024)
    C10_CUDA_CHECK(cudaFuncSetAttribute(ep_agrs_place_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  launch_k(ep_agrs_place_kernel, (int)std::max<int64_t>(1, grid), 1024, (size_t)smem, at::cuda::getCurrentCUDAStream(),
           a, reinterpret_cast<__nv_bfloat16*>(xs.data_ptr()), (int)xs.size(0), slot_of.data_ptr<int>(),
           offs.data_ptr<int>(), (int)max_pairs);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// y [rows, H] down-GEMM output (xs order) -> this rank's part rows.
void ep_agrs_combine(int64_t self, int64_t mc, int64_t rank, int64_t N, int64_t cap, int64_t K, int64_t El,
                     int64_t H, const at::Tensor& offsets, at::Tensor& state, const at::Tensor& slot_of,
                     const at::Tensor& y) {
  AgrsArgs a = make_agrs(self, mc, rank, N, cap, K, El, H, offsets, state);
  TORCH_CHECK(y.scalar_type() == at::kBFloat16 && y.is_contiguous() && y.size(1) == H);
  TORCH_CHECK(slot_of.scalar_type() == at::kInt && slot_of.numel() >= N * cap * K);
  c10::cuda::CUDAGuard guard(state.device());
  launch_k(ep_agrs_combine_kernel, (int)(N * cap), (int)(H / 8), 0, at::cuda::getCurrentCUDAStream(), a,
           (const int*)slot_of.data_ptr<int>(), reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mb
