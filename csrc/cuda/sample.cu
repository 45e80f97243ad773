// Fused token sampling over LM-head logits: temperature, top-k, top-p, greedy.
//
// One CTA per row, no sort (every pass streams the row with 16-byte loads, several in flight
// per thread).  With x = logit / T:
//   pass 1      row max m and Z = sum exp(x - m)
//   passes 2-8  the largest t_k with count{x >= t_k} >= k (k > 0) and the
//               largest t_p with mass{x >= t_p} >= p, each by 8-way refinement
//               of [m - 40, m]; the kept set is {x >= max(t_k, t_p)}
//               (each pass evaluates 8 thresholds at once and keeps the bracket
//               around the last feasible one; 9^7 ~ 4.8M steps).  Entries above
//               the bracket only add to one running total and entries below it
//               are skipped, so after the first pass a pass costs little more
//               than the read.
//   last pass   Gumbel-max over {x >= t}: argmax x + G, G = -log(-log u), which
//               draws exactly from the softmax restricted to the kept set.
// Entries more than 40 below the max carry < e^-40 relative mass and cannot win
// the Gumbel race, so the window loses nothing.  T <= 0 selects greedy argmax.
// u comes from a counter-based hash (SplitMix64 finaliser, Steele, Lea & Flood,
// "Fast splittable pseudorandom number generators", 2014) of (seed, step,
// index), so a seeded request replays identically.
//
// The reference has only greedy argmax (tensor_ops_cuda.cu:786, undefined) and a
// host-side top-k (pio/plugins/cpu/c_src/tensor_ops.c topk).
#include <type_traits>

#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "launch.cuh"

namespace mb {

namespace {

constexpr int kThreads = 1024;
constexpr int kWays = 8;
constexpr int kPasses = 7;
constexpr float kWindow = 40.f;

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// uniform in (0, 1): 24 random bits, centred in their bin
__device__ __forceinline__ float uniform01(uint64_t seed, uint64_t step, uint32_t idx) {
  const uint64_t h = splitmix64(seed ^ splitmix64(step * 0x100000001B3ull + idx));
  return ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
}

template <typename T>
__device__ __forceinline__ float ld(const T* p, int64_t i);
template <>
__device__ __forceinline__ float ld<float>(const float* p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}

__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
  for (int i = 1; i < kThreads / 32; ++i) r = fmaxf(r, red[i]);
  return r;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = 0.f;
  for (int i = 0; i < kThreads / 32; ++i) r += red[i];
  return r;
}

// Calls f(value, index) for every entry of a row, this thread's share.  bf16 rows whose
// length is a multiple of 8 and whose start is 16-byte aligned (the LM head's output) are read
// as 16-byte vectors, kUnroll of them in flight per thread before any is used: a pass is then
// bound by L2 bandwidth instead of one load latency per element.
constexpr int kUnroll = 4;
template <typename T, typename F>
__device__ __forceinline__ void row_for_each(const T* __restrict__ x, int64_t V, F&& f) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    if ((V & 7) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
      const uint4* x4 = reinterpret_cast<const uint4*>(x);
      const int64_t n4 = V >> 3;
      for (int64_t b = threadIdx.x; b < n4; b += (int64_t)kThreads * kUnroll) {
        uint4 r[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int64_t j = b + (int64_t)u * kThreads;
          r[u] = j < n4 ? __ldg(x4 + j) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int64_t j = b + (int64_t)u * kThreads;
          if (j < n4) {
            const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&r[u]);
#pragma unroll
            for (int q = 0; q < 8; ++q) f(__bfloat162float(h[q]), j * 8 + q);
          }
        }
      }
      return;
    }
  }
  for (int64_t i = threadIdx.x; i < V; i += kThreads) f(ld(x, i), i);
}

}  // namespace

template <typename T>
__global__ void __launch_bounds__(kThreads)
    sample_kernel(const T* __restrict__ logits, int64_t V, const float* __restrict__ temperature,
                  const int* __restrict__ top_k, const float* __restrict__ top_p, const int64_t* __restrict__ seeds,
                  const int64_t* __restrict__ steps, int64_t* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[kThreads / 32];
  __shared__ float cnt_s[kWays], mass_s[kWays];
  __shared__ float bi_v[kThreads / 32];
  __shared__ int bi_i[kThreads / 32];
  const int row = blockIdx.x, tid = threadIdx.x;
  const T* x = logits + (int64_t)row * V;
  const float temp = temperature[row];
  const bool greedy = !(temp > 0.f);
  const float inv_t = greedy ? 1.f : 1.f / temp;
  // ---- pass 1: max and normaliser
  float m = -INFINITY;
  row_for_each(x, V, [&](float v, int64_t) { m = fmaxf(m, v); });
  m = block_max(m, red) * inv_t;
  float tau = -INFINITY;
  if (!greedy) {
    float z = 0.f;
    row_for_each(x, V, [&](float v, int64_t) { z += __expf(v * inv_t - m); });
    z = block_sum(z, red);
    const int k = top_k[row];
    const float p = top_p[row];
    const float inv_z = 1.f / z;
    // Kept set = {x >= tk} intersect {x >= tp}: tk is the largest t with count{x >= t} >= k,
    // tp the largest t with mass{x >= t} >= p.  Both are refined in the same passes, each in
    // its own bracket [lo, hi).  A bracket bottom that is not itself feasible means the filter
    // keeps (practically) everything: nothing below m - 40 can win the Gumbel race.
    const bool use_k = k > 0, use_p = p < 1.f;
    float lo_k = m - kWindow, hi_k = m + 1e-6f, lo_p = m - kWindow, hi_p = m + 1e-6f;
    {
      float c = 0.f, ms = 0.f;
      row_for_each(x, V, [&](float raw, int64_t) {
        const float v = raw * inv_t;
        if (v >= lo_k) {
          c += 1.f;
          ms += __expf(v - m);
        }
      });
      c = block_sum(c, red);
      ms = block_sum(ms, red) * inv_z;
      if (!use_k || c < (float)k) lo_k = -INFINITY;
      if (!use_p || ms < p * (1.f - 1e-6f)) lo_p = -INFINITY;
    }
    const bool ref_k = lo_k > -INFINITY, ref_p = lo_p > -INFINITY;
    if (ref_k || ref_p) {
      for (int pass = 0; pass < kPasses; ++pass) {
        const float sk = (hi_k - lo_k) / (kWays + 1), sp = (hi_p - lo_p) / (kWays + 1);
        const float floor_k = ref_k ? lo_k + sk : INFINITY, floor_p = ref_p ? lo_p + sp : INFINITY;
        const float lowest = fminf(floor_k, floor_p);
        float c[kWays], ms[kWays];
        float ca = 0.f, ma = 0.f;  // entries at or above a bracket's top count for all its thresholds
#pragma unroll
        for (int w = 0; w < kWays; ++w) c[w] = ms[w] = 0.f;
        row_for_each(x, V, [&](float raw, int64_t) {
          const float v = raw * inv_t;
          if (v < lowest) return;
          if (v >= floor_k) {  // thresholds lo_k + (w+1) sk; v counts for every one <= v
            if (v >= hi_k) {
              ca += 1.f;
            } else {
              const int top = min(kWays - 1, (int)floorf((v - lo_k) / sk) - 1);
#pragma unroll
              for (int w = 0; w < kWays; ++w)
                if (w <= top) c[w] += 1.f;
            }
          }
          if (v >= floor_p) {
            const float e = __expf(v - m);
            if (v >= hi_p) {
              ma += e;
            } else {
              const int top = min(kWays - 1, (int)floorf((v - lo_p) / sp) - 1);
#pragma unroll
              for (int w = 0; w < kWays; ++w)
                if (w <= top) ms[w] += e;
            }
          }
        });
#pragma unroll
        for (int w = 0; w < kWays; ++w) {
          c[w] += ca;
          ms[w] += ma;
        }
        if (tid < kWays) {
          cnt_s[tid] = 0.f;
          mass_s[tid] = 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int w = 0; w < kWays; ++w) {
          const float cw = warp_sum(c[w]), mw = warp_sum(ms[w]);
          if ((tid & 31) == 0) {
            atomicAdd(&cnt_s[w], cw);
            atomicAdd(&mass_s[w], mw);
          }
        }
        __syncthreads();
        // largest feasible threshold of each bracket (feasibility is monotone in w)
        int bk = -1, bp = -1;
        for (int w = 0; w < kWays; ++w) {
          if (cnt_s[w] >= (float)k) bk = w;
          if (mass_s[w] * inv_z >= p * (1.f - 1e-6f)) bp = w;
        }
        if (ref_k) {
          const float nlo = bk >= 0 ? lo_k + (bk + 1) * sk : lo_k;
          hi_k = bk + 1 < kWays ? lo_k + (bk + 2) * sk : hi_k;
          lo_k = nlo;
        }
        if (ref_p) {
          const float nlo = bp >= 0 ? lo_p + (bp + 1) * sp : lo_p;
          hi_p = bp + 1 < kWays ? lo_p + (bp + 2) * sp : hi_p;
          lo_p = nlo;
        }
        __syncthreads();
      }
    }
    tau = fmaxf(lo_k, lo_p);
  }
  // ---- final pass: greedy argmax or Gumbel-max over {x >= tau}
  const uint64_t seed = (uint64_t)seeds[row], stp = (uint64_t)steps[row];
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  row_for_each(x, V, [&](float raw, int64_t i) {
    const float v = raw * inv_t;
    float s;
    if (greedy) {
      s = v;
    } else {
      if (!(v >= tau)) return;
      const float u = uniform01(seed, stp, (uint32_t)i);
      s = v - __logf(-__logf(u));
    }
    if (s > bv || (s == bv && (int)i < bi)) {
      bv = s;
      bi = (int)i;
    }
  });
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if ((tid & 31) == 0) {
    bi_v[tid >> 5] = bv;
    bi_i[tid >> 5] = bi;
  }
  __syncthreads();
  if (tid == 0) {
    float v = bi_v[0];
    int i0 = bi_i[0];
    for (int w = 1; w < kThreads / 32; ++w)
      if (bi_v[w] > v || (bi_v[w] == v && bi_i[w] < i0)) {
        v = bi_v[w];
        i0 = bi_i[w];
      }
    out[row] = i0 == 0x7fffffff ? 0 : i0;
  }
}

void sample_tokens(const at::Tensor& logits, const at::Tensor& temperature, const at::Tensor& top_k,
                   const at::Tensor& top_p, const at::Tensor& seeds, const at::Tensor& steps, at::Tensor& out) {
  TORCH_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.stride(1) == 1);
  TORCH_CHECK(temperature.scalar_type() == at::kFloat && top_p.scalar_type() == at::kFloat &&
              top_k.scalar_type() == at::kInt && seeds.scalar_type() == at::kLong && steps.scalar_type() == at::kLong &&
              out.scalar_type() == at::kLong);
  const int B = (int)logits.size(0);
  TORCH_CHECK(temperature.numel() == B && top_k.numel() == B && top_p.numel() == B && seeds.numel() == B &&
              steps.numel() == B && out.numel() == B);
  TORCH_CHECK(logits.size(1) < (1ll << 31), "vocab too large");
  if (B == 0) return;
  c10::cuda::CUDAGuard guard(logits.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int64_t V = logits.size(1);
  TORCH_CHECK(logits.stride(0) == V, "logits rows must be contiguous");
  if (logits.scalar_type() == at::kBFloat16) {
    launch_k(sample_kernel<__nv_bfloat16>, dim3(B), kThreads, 0, st,
             reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), V, temperature.data_ptr<float>(),
             top_k.data_ptr<int>(), top_p.data_ptr<float>(), seeds.data_ptr<int64_t>(), steps.data_ptr<int64_t>(),
             out.data_ptr<int64_t>());
  } else {
    TORCH_CHECK(logits.scalar_type() == at::kFloat, "sample_tokens: bf16 or f32 logits");
    launch_k(sample_kernel<float>, dim3(B), kThreads, 0, st, logits.data_ptr<float>(), V,
             temperature.data_ptr<float>(), top_k.data_ptr<int>(), top_p.data_ptr<float>(), seeds.data_ptr<int64_t>(),
             steps.data_ptr<int64_t>(), out.data_ptr<int64_t>());
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mb
