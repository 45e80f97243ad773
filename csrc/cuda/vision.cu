// Vision front end: image -> patch rows, and the bias / GELU step of the ViT MLP.
//
// patchify_kernel: one thread per output element of [B, N, C*p*p] (N = (S/p)^2
// patches in spatial-merge-group order: merge groups row-major over the grid,
// the m x m patches of a group consecutive).  Each element is a bilinear sample
// of the source image at the resized pixel (half-pixel centres, edge clamped:
// the align_corners = false convention), mean/std normalised, stored as bf16
// for the patch-embedding GEMM.  S equal to the input size makes the sample an
// exact copy.  Replaces the reference's host resize
// (pio/plugins/cpu/c_src/image_ops.c:8-39) and conv2d patch embedding
// (tensor_ops_cuda.cu:351-382).
//
// bias_act_kernel: y = act(y + bias) in place on bf16 rows (act = identity or
// tanh-approximated GELU), 8 columns per thread.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "launch.cuh"

namespace mb {

template <typename T>
__device__ __forceinline__ float ldf(const T* p, int64_t i);
template <>
__device__ __forceinline__ float ldf<float>(const float* p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float ldf<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}

struct PatchArgs {
  int B, C, H, W;   // source images [B, C, H, W]
  int S, p, m;      // target size, patch, merge
  float mean[4], inv_std[4];
};

template <typename T>
__global__ void patchify_kernel(const T* __restrict__ img, PatchArgs a, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int g = a.S / a.p, gm = g / a.m;
  const int per_patch = a.C * a.p * a.p;
  const int64_t total = (int64_t)a.B * g * g * per_patch;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  int64_t r = i;
  const int px = (int)(r % a.p); r /= a.p;
  const int py = (int)(r % a.p); r /= a.p;
  const int c = (int)(r % a.C); r /= a.C;
  const int n = (int)(r % (g * g));
  const int b = (int)(r / (g * g));
  // patch n in merge-group order -> grid (row, col)
  const int grp = n / (a.m * a.m), in = n % (a.m * a.m);
  const int row = (grp / gm) * a.m + in / a.m, col = (grp % gm) * a.m + in % a.m;
  const int y = row * a.p + py, x = col * a.p + px;   // pixel in the S x S image
  const T* src = img + ((int64_t)b * a.C + c) * a.H * a.W;
  float v;
  if (a.H == a.S && a.W == a.S) {
    v = ldf(src, (int64_t)y * a.W + x);
  } else {
    const float sy = fmaxf((y + 0.5f) * ((float)a.H / a.S) - 0.5f, 0.f);
    const float sx = fmaxf((x + 0.5f) * ((float)a.W / a.S) - 0.5f, 0.f);
    const int y0 = min((int)sy, a.H - 1), x0 = min((int)sx, a.W - 1);
    const int y1 = min(y0 + 1, a.H - 1), x1 = min(x0 + 1, a.W - 1);
    const float fy = sy - y0, fx = sx - x0;
    const float v00 = ldf(src, (int64_t)y0 * a.W + x0), v01 = ldf(src, (int64_t)y0 * a.W + x1);
    const float v10 = ldf(src, (int64_t)y1 * a.W + x0), v11 = ldf(src, (int64_t)y1 * a.W + x1);
    v = (v00 * (1.f - fx) + v01 * fx) * (1.f - fy) + (v10 * (1.f - fx) + v11 * fx) * fy;
  }
  out[i] = __float2bfloat16((v - a.mean[c]) * a.inv_std[c]);
}

void patchify(const at::Tensor& images, int64_t size, int64_t patch, int64_t merge, std::vector<double> mean,
              std::vector<double> stdv, at::Tensor& out) {
  TORCH_CHECK(images.is_cuda() && images.dim() == 4 && images.is_contiguous());
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous());
  const int B = (int)images.size(0), C = (int)images.size(1);
  TORCH_CHECK(C <= 4 && (int)mean.size() == C && (int)stdv.size() == C, "patchify: up to 4 channels with mean/std");
  TORCH_CHECK(size % (patch * merge) == 0, "patchify: size must be a multiple of patch * merge");
  const int64_t g = size / patch;
  TORCH_CHECK(out.numel() == (int64_t)B * g * g * C * patch * patch, "patchify: output shape");
  PatchArgs a{};
  a.B = B; a.C = C; a.H = (int)images.size(2); a.W = (int)images.size(3);
  a.S = (int)size; a.p = (int)patch; a.m = (int)merge;
  for (int c = 0; c < C; ++c) {
    a.mean[c] = (float)mean[c];
    a.inv_std[c] = (float)(1.0 / stdv[c]);
  }
  c10::cuda::CUDAGuard guard(images.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int64_t total = out.numel();
  const unsigned blocks = (unsigned)((total + 255) / 256);
  auto o = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  if (images.scalar_type() == at::kFloat) {
    launch_k(patchify_kernel<float>, blocks, 256, 0, st, images.data_ptr<float>(), a, o);
  } else {
    TORCH_CHECK(images.scalar_type() == at::kBFloat16, "patchify: f32 or bf16 images");
    launch_k(patchify_kernel<__nv_bfloat16>, blocks, 256, 0, st,
             reinterpret_cast<const __nv_bfloat16*>(images.data_ptr()), a, o);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f;  // sqrt(2 / pi)
  return 0.5f * x * (1.f + tanhf(k0 * (x + 0.044715f * x * x * x)));
}

template <bool GELU>
__global__ void bias_act_kernel(__nv_bfloat16* __restrict__ y, const __nv_bfloat16* __restrict__ bias, int64_t rows,
                                int cols) {
  pdl_wait();
  pdl_trigger();
  const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (i >= rows * cols) return;
  const int c = (int)(i % cols);
  uint4 raw = *reinterpret_cast<const uint4*>(y + i);
  const uint4 braw = bias ? *reinterpret_cast<const uint4*>(bias + c) : make_uint4(0, 0, 0, 0);
  __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(&raw);
  const __nv_bfloat16* bh = reinterpret_cast<const __nv_bfloat16*>(&braw);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    float v = __bfloat162float(h[q]) + (bias ? __bfloat162float(bh[q]) : 0.f);
    if (GELU) v = gelu_tanh(v);
    h[q] = __float2bfloat16(v);
  }
  *reinterpret_cast<uint4*>(y + i) = raw;
}

void bias_act(at::Tensor& y, const c10::optional<at::Tensor>& bias, bool gelu) {
  TORCH_CHECK(y.is_cuda() && y.scalar_type() == at::kBFloat16 && y.is_contiguous() && y.dim() == 2);
  const int64_t rows = y.size(0);
  const int cols = (int)y.size(1);
  TORCH_CHECK(cols % 8 == 0, "bias_act: columns must be a multiple of 8");
  const __nv_bfloat16* b = nullptr;
  if (bias && bias->defined()) {
    TORCH_CHECK(bias->scalar_type() == at::kBFloat16 && bias->is_contiguous() && bias->numel() == cols);
    b = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
  }
  if (rows == 0) return;
  c10::cuda::CUDAGuard guard(y.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int64_t n8 = rows * cols / 8;
  const unsigned blocks = (unsigned)((n8 + 255) / 256);
  auto p = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  if (gelu)
    launch_k(bias_act_kernel<true>, blocks, 256, 0, st, p, b, rows, cols);
  else
    launch_k(bias_act_kernel<false>, blocks, 256, 0, st, p, b, rows, cols);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ViT attention operands: 2-D rotary embedding of q and k (rotate-half; angle index i < D/4
// follows the patch row, D/4 <= i < D/2 the column; theta^(-i'/(D/4)) with i' = i mod D/4),
// q -> q_out [B*N, heads*D]; k and v of image b go to block b*nblk + t/16 of a paged cache
// (K [blocks, heads, 16, D], V [blocks, heads, D, 16]) so the bidirectional flash kernel can
// read every image as one sequence.  One CTA per patch row.
__global__ void vit_rope_kv_kernel(const __nv_bfloat16* __restrict__ qkv, const int* __restrict__ pos, int N,
                                  int heads, int D, int nblk, float theta, __nv_bfloat16* __restrict__ q_out,
                                  __nv_bfloat16* __restrict__ k_cache, __nv_bfloat16* __restrict__ v_cache) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x, b = row / N, t = row % N;
  const int half = D / 2, quarter = D / 4;
  const float pr = (float)pos[t * 2], pc = (float)pos[t * 2 + 1];
  const __nv_bfloat16* src = qkv + (size_t)row * 3 * heads * D;
  const size_t blk = (size_t)b * nblk + t / 16, off = t % 16;
  for (int i = threadIdx.x; i < heads * half; i += blockDim.x) {
    const int h = i / half, d = i % half;
    const int ii = d % quarter;
    const float inv = powf(theta, -(float)ii / (float)quarter);
    float sn, cs;
    sincosf((d < quarter ? pr : pc) * inv, &sn, &cs);
#pragma unroll
    for (int which = 0; which < 2; ++which) {  // q, k
      const __nv_bfloat16* x = src + (size_t)which * heads * D + h * D;
      const float x1 = __bfloat162float(x[d]), x2 = __bfloat162float(x[d + half]);
      const __nv_bfloat16 o1 = __float2bfloat16(x1 * cs - x2 * sn), o2 = __float2bfloat16(x2 * cs + x1 * sn);
      if (which == 0) {
        q_out[(size_t)row * heads * D + h * D + d] = o1;
        q_out[(size_t)row * heads * D + h * D + d + half] = o2;
      } else {
        __nv_bfloat16* kd = k_cache + ((blk * heads + h) * 16 + off) * D;
        kd[d] = o1;
        kd[d + half] = o2;
      }
    }
  }
  for (int i = threadIdx.x; i < heads * D; i += blockDim.x) {
    const int h = i / D, d = i % D;
    v_cache[((blk * heads + h) * D + d) * 16 + off] = src[(size_t)2 * heads * D + i];
  }
}

void vit_rope_kv(const at::Tensor& qkv, const at::Tensor& pos, int64_t N, int64_t heads, int64_t D, double theta,
                 at::Tensor& q_out, at::Tensor& k_cache, at::Tensor& v_cache) {
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.is_contiguous() && qkv.size(1) == 3 * heads * D);
  TORCH_CHECK(pos.scalar_type() == at::kInt && pos.is_contiguous() && pos.numel() == 2 * N && D % 4 == 0);
  const int64_t rows = qkv.size(0), nblk = (N + 15) / 16;
  TORCH_CHECK(rows % N == 0 && q_out.is_contiguous() && q_out.numel() == rows * heads * D);
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous() && k_cache.size(0) >= rows / N * nblk &&
              k_cache.size(1) == heads && k_cache.size(2) == 16 && k_cache.size(3) == D && v_cache.size(2) == D);
  if (rows == 0) return;
  c10::cuda::CUDAGuard guard(qkv.device());
  launch_k(vit_rope_kv_kernel, (unsigned)rows, 256, 0, at::cuda::getCurrentCUDAStream(),
           reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), (const int*)pos.data_ptr<int>(), (int)N,
           (int)heads, (int)D, (int)nblk, (float)theta, reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr()),
           reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr()), reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mb
