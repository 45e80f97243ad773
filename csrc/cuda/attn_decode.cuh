// Device code of the paged decode attention (split-KV + combine), shared by
// the torch-facing entry point (attn_decode.cu) and the allocation-free C
// entry point (attn_decode_noalloc.cu).
#pragma once
#include <type_traits>
#include "common.cuh"

namespace mb {

constexpr int kWarps = 4;

template <int D, int G>
__global__ void __launch_bounds__(kWarps * 32)
    attn_decode_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ kc,
                       const __nv_bfloat16* __restrict__ vc, const int* __restrict__ block_tables,
                       const int* __restrict__ ctx_lens, __nv_bfloat16* __restrict__ out, float* __restrict__ part_o,
                       float* __restrict__ part_lse, int Hkv, int max_blocks, int splits, float scale_log2) {
  pdl_wait();
  pdl_trigger();
  constexpr int BS = 16;
  constexpr int E = D / 32;      // P.V dims per lane
  constexpr int HD = D / 2;      // Q.K dims per lane
  __shared__ float qs[G][D];
  __shared__ float red_m[kWarps][G], red_l[kWarps][G];
  __shared__ float red_o[kWarps][G][D];
  const int b = blockIdx.x, hk = blockIdx.y, sp = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int Hq = Hkv * G;
  // The block table row holds max_blocks entries: a context longer than
  // 16 * max_blocks is clamped to what the row can address (never read past it).
  const int ctx = min(ctx_lens[b], max_blocks * BS);
  const int nblk = (ctx + BS - 1) / BS;
  const int bps = (nblk + splits - 1) / splits;
  const int blo = sp * bps, bhi = min(nblk, blo + bps);

  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    qs[g][d] = __bfloat162float(q[((size_t)b * Hq + hk * G + g) * D + d]) * scale_log2;
  }
  __syncthreads();

  float m[G], l[G], acc[G][E];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) acc[g][e] = 0.f;
  }
  const int tok = lane & 15, half = lane >> 4;
  for (int blk = blo + warp; blk < bhi; blk += kWarps) {
    const int phys = block_tables[(size_t)b * max_blocks + blk];
    const size_t base = ((size_t)phys * Hkv + hk) * BS * D;
    // issue K (this lane's token/half) and V (this lane's dims, all tokens)
    uint4 kr[HD / 8];
    const uint4* kp = reinterpret_cast<const uint4*>(kc + base + tok * D + half * HD);
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) kr[i] = kp[i];
    // V block is [D, BS]: this lane's E dims are E rows of 16 tokens (32 B each)
    uint4 vr[E][2];
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const uint4* vp = reinterpret_cast<const uint4*>(vc + base + (size_t)(lane * E + e) * BS);
      vr[e][0] = vp[0];
      vr[e][1] = vp[1];
    }

    float s[G];
#pragma unroll
    for (int g = 0; g < G; ++g) s[g] = 0.f;
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      const __nv_bfloat16* kh = reinterpret_cast<const __nv_bfloat16*>(&kr[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float kv = __bfloat162float(kh[j]);
#pragma unroll
        for (int g = 0; g < G; ++g) s[g] += kv * qs[g][half * HD + i * 8 + j];
      }
    }
    const bool valid = blk * BS + tok < ctx;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      s[g] += __shfl_xor_sync(0xffffffffu, s[g], 16);
      s[g] = valid ? s[g] : -INFINITY;
      float mb = s[g];
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, o));
      const float mn = fmaxf(m[g], mb);
      const float corr = exp2f(m[g] - mn);
      const float p = exp2f(s[g] - mn);
      float ps = p;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      l[g] = l[g] * corr + ps;
      m[g] = mn;
#pragma unroll
      for (int e = 0; e < E; ++e) acc[g][e] *= corr;
      s[g] = p;
    }
#pragma unroll
    for (int t = 0; t < BS; ++t) {
      float vf[E];
#pragma unroll
      for (int e = 0; e < E; ++e)
        vf[e] = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(&vr[e][t >> 3])[t & 7]);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pt = __shfl_sync(0xffffffffu, s[g], t);
#pragma unroll
        for (int e = 0; e < E; ++e) acc[g][e] += pt * vf[e];
      }
    }
  }
  // merge the warps
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      red_m[warp][g] = m[g];
      red_l[warp][g] = l[g];
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < E; ++e) red_o[warp][g][lane * E + e] = acc[g][e];
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) mx = fmaxf(mx, red_m[w][g]);
    float lsum = 0.f, o = 0.f;
    if (mx != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float c = exp2f(red_m[w][g] - mx);
        lsum += red_l[w][g] * c;
        o += red_o[w][g][d] * c;
      }
    }
    const int h = hk * G + g;
    if (splits == 1) {
      out[((size_t)b * Hq + h) * D + d] = __float2bfloat16(lsum > 0.f ? o / lsum : 0.f);
    } else {
      const size_t pi = ((size_t)b * Hq + h) * splits + sp;
      part_o[pi * D + d] = lsum > 0.f ? o / lsum : 0.f;
      if (d == 0) part_lse[pi] = lsum > 0.f ? mx + log2f(lsum) : -INFINITY;
    }
  }
}

template <int D>
__global__ void attn_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse,
                                    __nv_bfloat16* __restrict__ out, int splits) {
  pdl_wait();
  pdl_trigger();
  const size_t bh = blockIdx.x;
  float mx = -INFINITY;
  for (int s = 0; s < splits; ++s) mx = fmaxf(mx, part_lse[bh * splits + s]);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float o = 0.f, w = 0.f;
    if (mx != -INFINITY) {
      for (int s = 0; s < splits; ++s) {
        const float c = exp2f(part_lse[bh * splits + s] - mx);
        w += c;
        o += c * part_o[(bh * splits + s) * D + d];
      }
    }
    out[bh * D + d] = __float2bfloat16(w > 0.f ? o / w : 0.f);
  }
}

}  // namespace mb
