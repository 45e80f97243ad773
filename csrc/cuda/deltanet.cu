// Gated DeltaNet (Qwen3-Next linear attention) kernels.
//
// Math per value head h (state S in R^{dk x dv}, fp32):
//   x_c   = SiLU(sum_k conv_w[c,k] * hist_c[k])       causal depthwise conv over (history ++ input)
//   q, k  = L2-normalised (q also scaled by dk^-1/2); value heads share key heads (GQA-style)
//   beta  = sigmoid(b), decay = exp(-exp(A_log) * softplus(a + dt_bias))
//   S     = decay * S ;  delta = beta * (v - S^T k) ;  S += k delta^T ;  o = S^T q
//   out   = rmsnorm(o) * w_norm * silu(z)
//
// Work split: a value head's state columns belong to threads (column j, a
// band of rows each), so the rank-1 update needs no exchange and S^T k, S^T q
// only sum a few row-band partials; the state never leaves registers during a
// prefill scan and is streamed exactly once per decode step.
//
// deltanet_conv : prefill conv + SiLU + q/k L2 norm, CTA per token, fp32 out.
// deltanet_conv_decode : decode conv + SiLU, thread per (token, channel); advances
//                 the history (q/k are normalised by the step kernel).
// deltanet_step : decode state update + gated RMSNorm, CTA per (seq, value head).
// deltanet_scan : prefill recurrence, CTA per (sequence, value head); also
//                 advances the conv history to the sequence's last inputs.
// The sequential scan does O(L dk dv) work against O(L C (dk+dv)) + O(L dk dv)
// for the chunked (WY) form, so on CUDA cores it is the cheaper choice.
//
// Replaces the reference's decayed linear-attention recurrence
// (pio/plugins/cuda/c_src/tensor_ops_cuda.cu:420-452).
#include <cstdlib>
#include <type_traits>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "launch.cuh"

namespace mb {

namespace {

__device__ __forceinline__ float softplus_f(float x) { return x > 20.f ? x : log1pf(__expf(x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + __expf(-x)); }
__device__ __forceinline__ float bf(const __nv_bfloat16 v) { return __bfloat162float(v); }

}  // namespace

// Prefill conv + SiLU + q/k L2 norm, CTA per token.  mixed [T, C] raw; seq_of [T] / cu [nseq+1]
// place the token in its sequence, and positions before the sequence start read the slot's
// history (advanced later by the scan kernel).  Output xc [T, C] (fp32 for the token-serial scan,
// bf16 for the chunked scan, whose products take bf16 operands), q heads also scaled by DK^-1/2.
template <int DK, int KC, typename OutT>
__global__ void __launch_bounds__(256)
    deltanet_conv_kernel(const __nv_bfloat16* __restrict__ mixed, const __nv_bfloat16* __restrict__ conv_w,
                         float* __restrict__ conv_state, const int64_t* __restrict__ slots,
                         const int* __restrict__ seq_of, const int* __restrict__ cu, OutT* __restrict__ xc, int C,
                         int Hk) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float row[];  // C floats
  const int t = blockIdx.x;
  const int s = seq_of[t];
  const int start = cu[s], pos = t - start;
  float* hist = conv_state + slots[s] * (int64_t)C * (KC - 1);
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    float in[KC];
#pragma unroll
    for (int k = 0; k < KC; ++k) {
      const int p = pos - (KC - 1) + k;  // input position within the sequence
      in[k] = p >= 0 ? bf(mixed[(int64_t)(start + p) * C + c]) : hist[c * (KC - 1) + (KC - 1 + p)];
    }
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < KC; ++k) acc += bf(conv_w[c * KC + k]) * in[k];
    row[c] = silu(acc);
  }
  __syncthreads();
  // q/k heads: one warp per head, L2 norm
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int hh = w; hh < 2 * Hk; hh += nw) {
    float ss = 0.f;
    for (int i = l; i < DK; i += 32) ss += row[hh * DK + i] * row[hh * DK + i];
    ss = warp_sum(ss);
    const float sc = rsqrtf(ss + 1e-6f) * (hh < Hk ? rsqrtf((float)DK) : 1.f);
    for (int i = l; i < DK; i += 32) row[hh * DK + i] *= sc;
  }
  __syncthreads();
  OutT* dst = xc + (int64_t)t * C;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    if constexpr (std::is_same<OutT, float>::value) dst[c] = row[c];
    else dst[c] = __float2bfloat16(row[c]);
  }
}

// Decode conv: one thread per (token, channel), all channels in parallel.  Every token is its
// own sequence, so the thread also advances that channel's history in its slot.  Output xc
// [B, C] f32 = SiLU(conv), not normalised (the step kernel normalises q and k).
template <int KC>
__global__ void __launch_bounds__(256)
    deltanet_conv_decode_kernel(const __nv_bfloat16* __restrict__ mixed, const __nv_bfloat16* __restrict__ conv_w,
                                float* __restrict__ conv_state, const int64_t* __restrict__ slots,
                                float* __restrict__ xc, int B, int C) {
  pdl_wait();
  pdl_trigger();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)B * C) return;
  const int b = (int)(i / C), c = (int)(i - (int64_t)b * C);
  float* hist = conv_state + (slots[b] * (int64_t)C + c) * (KC - 1);
  float in[KC];
#pragma unroll
  for (int k = 0; k < KC - 1; ++k) in[k] = hist[k];
  in[KC - 1] = bf(mixed[i]);
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < KC; ++k) acc += bf(conv_w[c * KC + k]) * in[k];
#pragma unroll
  for (int k = 0; k < KC - 1; ++k) hist[k] = in[k + 1];
  xc[i] = silu(acc);
}

// Decode state update: CTA per (sequence, value head), R*DV threads; thread (g, j) holds rows
// [g*DK/R, (g+1)*DK/R) of column j.  Streams the state once (read + write); the two column dot
// products are summed over the R row groups through shared memory.
template <int DK, int DV, int R>
__global__ void __launch_bounds__(R* DV)
    deltanet_step_kernel(const float* __restrict__ xc, const __nv_bfloat16* __restrict__ z,
                         const __nv_bfloat16* __restrict__ ba, float* __restrict__ ssm,
                         const int64_t* __restrict__ slots, const float* __restrict__ A_log,
                         const float* __restrict__ dt_bias, const __nv_bfloat16* __restrict__ norm_w,
                         __nv_bfloat16* __restrict__ out, int Hk, int Hv, float eps) {
  static_assert(DK <= R * DV && DV % 32 == 0 && DK % R == 0, "layout");
  constexpr int RR = DK / R;
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int g = tid / DV, j = tid % DV;
  const int rep = Hv / Hk, hk = h / rep;
  const int C = 2 * Hk * DK + Hv * DV;
  const int64_t slot = slots[b];
  __shared__ float qs[DK], ks[DK], part[R][DV], red[DV / 32], qkred[2][DK / 32];
  const float* x = xc + (int64_t)b * C;
  float qv = 0.f, kv = 0.f;
  if (tid < DK) {  // q / k of this key head, L2-normalised here (q also scaled by DK^-1/2)
    qv = x[hk * DK + tid];
    kv = x[Hk * DK + hk * DK + tid];
    const float sq = warp_sum(qv * qv), sk = warp_sum(kv * kv);
    if ((tid & 31) == 0) {
      qkred[0][tid >> 5] = sq;
      qkred[1][tid >> 5] = sk;
    }
  }
  const float beta = sigmoid_f(bf(ba[(int64_t)b * 2 * Hv + h]));
  const float decay = __expf(-__expf(A_log[h]) * softplus_f(bf(ba[(int64_t)b * 2 * Hv + Hv + h]) + dt_bias[h]));
  float* S = ssm + ((slot * Hv + h) * (int64_t)DK + g * RR) * DV + j;
  float col[RR];
#pragma unroll
  for (int i = 0; i < RR; ++i) col[i] = S[(int64_t)i * DV] * decay;
  __syncthreads();
  if (tid < DK) {
    float sq = 0.f, sk = 0.f;
#pragma unroll
    for (int w = 0; w < DK / 32; ++w) {
      sq += qkred[0][w];
      sk += qkred[1][w];
    }
    qs[tid] = qv * rsqrtf(sq + 1e-6f) * rsqrtf((float)DK);
    ks[tid] = kv * rsqrtf(sk + 1e-6f);
  }
  __syncthreads();
  float p = 0.f;
#pragma unroll
  for (int i = 0; i < RR; ++i) p += col[i] * ks[g * RR + i];
  part[g][j] = p;
  __syncthreads();
  float kvj = 0.f;
#pragma unroll
  for (int r = 0; r < R; ++r) kvj += part[r][j];
  const float delta = (x[2 * Hk * DK + h * DV + j] - kvj) * beta;
  p = 0.f;
#pragma unroll
  for (int i = 0; i < RR; ++i) {
    col[i] += ks[g * RR + i] * delta;
    p += col[i] * qs[g * RR + i];
    S[(int64_t)i * DV] = col[i];
  }
  __syncthreads();  // every kvj read of part is done
  part[g][j] = p;
  __syncthreads();
  float o = 0.f, ss = 0.f;
  if (g == 0) {
#pragma unroll
    for (int r = 0; r < R; ++r) o += part[r][j];
    ss = warp_sum(o * o);
    if ((j & 31) == 0) red[j >> 5] = ss;
  }
  __syncthreads();
  if (g == 0) {
    float on = 0.f;
#pragma unroll
    for (int w = 0; w < DV / 32; ++w) on += red[w];
    const float zj = bf(z[(int64_t)b * Hv * DV + h * DV + j]);
    out[(int64_t)b * Hv * DV + h * DV + j] = __float2bfloat16(o * rsqrtf(on / DV + eps) * bf(norm_w[j]) * silu(zj));
  }
}

// Prefill recurrence: CTA per (sequence, value head), R*DV threads; thread (g, j) keeps rows
// [g*DK/R, (g+1)*DK/R) of column j in registers for the whole sequence.  Token t:
//   stage q_t/k_t (double-buffered) | B1 | partial S^T k -> kp ; sum(o_{t-1}) -> wred | B2 |
//   S^T k = sum kp, update, partial S^T q -> op ; write out_{t-1}
// so the output of a token is finished during the next one and each token costs two barriers.
// Finally advances the conv history to the last KC-1 inputs of (history ++ sequence).
template <int DK, int DV, int KC, int R>
__global__ void __launch_bounds__(R* DV)
    deltanet_scan_kernel(const float* __restrict__ xc, const __nv_bfloat16* __restrict__ mixed,
                         const __nv_bfloat16* __restrict__ z, const __nv_bfloat16* __restrict__ ba,
                         float* __restrict__ conv_state, float* __restrict__ ssm, const int64_t* __restrict__ slots,
                         const int* __restrict__ cu, const float* __restrict__ A_log,
                         const float* __restrict__ dt_bias, const __nv_bfloat16* __restrict__ norm_w,
                         __nv_bfloat16* __restrict__ out, int Hk, int Hv, float eps) {
  static_assert(DK <= DV && DV % 32 == 0 && DK % R == 0, "layout");
  constexpr int NW = DV / 32, RR = DK / R;
  pdl_wait();
  pdl_trigger();
  const int s = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int g = tid / DV, j = tid % DV;
  const int rep = Hv / Hk, hk = h / rep;
  const int C = 2 * Hk * DK + Hv * DV;
  const int start = cu[s], L = cu[s + 1] - start;
  const int64_t slot = slots[s];
  __shared__ float qs[2][DK], ks[2][DK], kp[R][DV], op[R][DV], wred[NW];
  const float A = __expf(A_log[h]), dtb = dt_bias[h], nwj = bf(norm_w[j]);
  float* S = ssm + ((slot * Hv + h) * (int64_t)DK + g * RR) * DV + j;
  float col[RR];
#pragma unroll
  for (int i = 0; i < RR; ++i) col[i] = S[(int64_t)i * DV];
  const int qc = hk * DK + j, kc = Hk * DK + hk * DK + j, vc = 2 * Hk * DK + h * DV + j;
  // operands of the next token, fetched one token ahead (group 0 stages q/k)
  float nq = 0.f, nk = 0.f, nv = 0.f, nb = 0.f, na = 0.f, nz = 0.f;
  auto fetch = [&](int t) {
    const int64_t r = start + t;
    if (g == 0 && j < DK) {
      nq = xc[r * C + qc];
      nk = xc[r * C + kc];
    }
    nv = xc[r * C + vc];
    nb = bf(ba[r * 2 * Hv + h]);
    na = bf(ba[r * 2 * Hv + Hv + h]);
    if (g == 0) nz = bf(z[r * Hv * DV + h * DV + j]);
  };
  float o_prev = 0.f, z_prev = 0.f;
  // group 0, between the barriers: o of the previous token and its warp sums of squares
  auto reduce_prev = [&]() {
    o_prev = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r) o_prev += op[r][j];
    const float ss = warp_sum(o_prev * o_prev);
    if ((j & 31) == 0) wred[j >> 5] = ss;
  };
  auto write_prev = [&](int t) {
    float on = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) on += wred[w];
    out[(int64_t)(start + t) * Hv * DV + h * DV + j] =
        __float2bfloat16(o_prev * rsqrtf(on / DV + eps) * nwj * silu(z_prev));
  };
  if (L > 0) fetch(0);
  float zc = 0.f;
  for (int t = 0; t < L; ++t) {
    const int buf = t & 1;
    if (g == 0 && j < DK) {
      qs[buf][j] = nq;
      ks[buf][j] = nk;
    }
    const float vj = nv;
    const float beta = sigmoid_f(nb);
    const float decay = __expf(-A * softplus_f(na + dtb));
    z_prev = zc;
    zc = nz;
    if (t + 1 < L) fetch(t + 1);
    __syncthreads();  // B1
    float p = 0.f;
#pragma unroll
    for (int i = 0; i < RR; ++i) {
      col[i] *= decay;
      p += col[i] * ks[buf][g * RR + i];
    }
    kp[g][j] = p;
    if (t > 0 && g == 0) reduce_prev();
    __syncthreads();  // B2
    if (t > 0 && g == 0) write_prev(t - 1);
    float kvj = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r) kvj += kp[r][j];
    const float delta = (vj - kvj) * beta;
    p = 0.f;
#pragma unroll
    for (int i = 0; i < RR; ++i) {
      col[i] += ks[buf][g * RR + i] * delta;
      p += col[i] * qs[buf][g * RR + i];
    }
    op[g][j] = p;
  }
  __syncthreads();
  if (L > 0 && g == 0) {
    z_prev = zc;
    reduce_prev();
  }
  __syncthreads();
  if (L > 0 && g == 0) write_prev(L - 1);
#pragma unroll
  for (int i = 0; i < RR; ++i) S[(int64_t)i * DV] = col[i];
  float* cs = conv_state + slot * (int64_t)C * (KC - 1);
  auto advance = [&](int c) {
#pragma unroll
    for (int k = 0; k < KC - 1; ++k) {
      const int idx = L + k;  // index into history ++ inputs; reads run ahead of writes
      cs[c * (KC - 1) + k] =
          idx < KC - 1 ? cs[c * (KC - 1) + idx] : bf(mixed[(int64_t)(start + idx - (KC - 1)) * C + c]);
    }
  };
  if (g == 0) {
    advance(vc);
    if (h % rep == 0 && j < DK) {
      advance(qc);
      advance(kc);
    }
  }
}

void deltanet_decode(const at::Tensor& mixed, const at::Tensor& z, const at::Tensor& ba, const at::Tensor& conv_w,
                     at::Tensor& conv_state, at::Tensor& ssm, const at::Tensor& slots, const at::Tensor& A_log,
                     const at::Tensor& dt_bias, const at::Tensor& norm_w, at::Tensor& out, int64_t Hk, int64_t Hv,
                     int64_t dk, int64_t dv, double eps) {
  TORCH_CHECK(mixed.scalar_type() == at::kBFloat16 && z.scalar_type() == at::kBFloat16 &&
              ba.scalar_type() == at::kBFloat16 && conv_w.scalar_type() == at::kBFloat16 &&
              norm_w.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16);
  TORCH_CHECK(conv_state.scalar_type() == at::kFloat && ssm.scalar_type() == at::kFloat &&
              A_log.scalar_type() == at::kFloat && dt_bias.scalar_type() == at::kFloat &&
              slots.scalar_type() == at::kLong);
  TORCH_CHECK(mixed.is_contiguous() && z.is_contiguous() && ba.is_contiguous() && conv_w.is_contiguous() &&
              conv_state.is_contiguous() && ssm.is_contiguous() && out.is_contiguous() && slots.is_contiguous());
  TORCH_CHECK(Hv % Hk == 0 && mixed.size(1) == 2 * Hk * dk + Hv * dv && z.size(1) == Hv * dv && ba.size(1) == 2 * Hv,
              "deltanet_decode: shape mismatch");
  const int B = (int)mixed.size(0), KC = (int)conv_w.size(1);
  if (B == 0) return;
  c10::cuda::CUDAGuard guard(mixed.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  auto bp = [](const at::Tensor& t) { return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()); };
  const int C = (int)mixed.size(1);
  auto xc = at::empty({B, C}, mixed.options().dtype(at::kFloat));
  const int64_t* sl = (const int64_t*)slots.data_ptr<int64_t>();
#define MB_DN(DK_, DV_, KC_, R_)                                                                                  \
  if (dk == DK_ && dv == DV_ && KC == KC_) {                                                                      \
    const int64_t n = (int64_t)B * C;                                                                             \
    launch_k(deltanet_conv_decode_kernel<KC_>, dim3((unsigned)((n + 255) / 256)), 256, 0, st, bp(mixed),        \
             bp(conv_w), conv_state.data_ptr<float>(), sl, xc.data_ptr<float>(), B, C);                           \
    C10_CUDA_KERNEL_LAUNCH_CHECK();                                                                               \
    launch_k(deltanet_step_kernel<DK_, DV_, R_>, dim3(B, (unsigned)Hv), R_ * DV_, 0, st,                         \
             (const float*)xc.data_ptr<float>(), bp(z), bp(ba), ssm.data_ptr<float>(), sl,                        \
             (const float*)A_log.data_ptr<float>(), (const float*)dt_bias.data_ptr<float>(), bp(norm_w),          \
             reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), (int)Hk, (int)Hv, (float)eps);                      \
    C10_CUDA_KERNEL_LAUNCH_CHECK();                                                                               \
    return;                                                                                                       \
  }
  MB_DN(128, 128, 4, 4)
  MB_DN(64, 64, 4, 2)
#undef MB_DN
  TORCH_CHECK(false, "deltanet_decode: unsupported head dims / conv kernel");
}

// Prefill of nseq sequences packed in mixed [T, C] (cu [nseq+1] int32 offsets, seq_of [T]).
void launch_deltanet_chunk(const __nv_bfloat16* xc, const __nv_bfloat16* mixed, float* conv_state, const __nv_bfloat16* z,
                           const __nv_bfloat16* ba, float* ssm, const int64_t* slots, const int* cu, const float* A_log,
                           const float* dt_bias, const __nv_bfloat16* norm_w, __nv_bfloat16* out, int nseq, int Hk,
                           int Hv, float eps, cudaStream_t st);

// Prefill recurrence: the chunked tensor-core form (deltanet_chunk.cu) for dk = dv = 128 and conv
// kernel 4, the token-serial scan otherwise (or with MB_DELTANET_CHUNK=0, kept for A/B timing).
static bool use_chunked() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("MB_DELTANET_CHUNK");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

void deltanet_prefill(const at::Tensor& mixed, const at::Tensor& z, const at::Tensor& ba, const at::Tensor& conv_w,
                      at::Tensor& conv_state, at::Tensor& ssm, const at::Tensor& slots, const at::Tensor& cu,
                      const at::Tensor& seq_of, const at::Tensor& A_log, const at::Tensor& dt_bias,
                      const at::Tensor& norm_w, at::Tensor& out, at::Tensor& xc, int64_t Hk, int64_t Hv, int64_t dk,
                      int64_t dv, double eps) {
  TORCH_CHECK(mixed.scalar_type() == at::kBFloat16 && mixed.is_contiguous() && z.is_contiguous() &&
              ba.is_contiguous() && out.is_contiguous());
  TORCH_CHECK(xc.scalar_type() == at::kFloat && xc.is_contiguous() && xc.numel() >= mixed.numel());
  TORCH_CHECK(cu.scalar_type() == at::kInt && seq_of.scalar_type() == at::kInt && slots.scalar_type() == at::kLong);
  TORCH_CHECK(conv_state.scalar_type() == at::kFloat && ssm.scalar_type() == at::kFloat &&
              conv_state.is_contiguous() && ssm.is_contiguous() && conv_w.is_contiguous());
  TORCH_CHECK(Hv % Hk == 0 && mixed.size(1) == 2 * Hk * dk + Hv * dv, "deltanet_prefill: shape mismatch");
  const int T = (int)mixed.size(0), C = (int)mixed.size(1), KC = (int)conv_w.size(1);
  const int nseq = (int)slots.size(0);
  if (T == 0 || nseq == 0) return;
  c10::cuda::CUDAGuard guard(mixed.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  auto bp = [](const at::Tensor& t) { return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()); };
  const size_t smem = (size_t)C * sizeof(float);
#define MB_DP(DK_, DV_, KC_)                                                                                      \
  if (dk == DK_ && dv == DV_ && KC == KC_) {                                                                      \
    const bool chunked = DK_ == 128 && DV_ == 128 && KC_ == 4 && use_chunked();                                   \
    if (chunked) {                                                                                                \
      /* bf16 conv output (written into the fp32 buffer's first half) for the chunked scan */                     \
      auto ck = deltanet_conv_kernel<DK_, KC_, __nv_bfloat16>;                                                    \
      if (smem > 48 * 1024)                                                                                       \
        C10_CUDA_CHECK(cudaFuncSetAttribute(ck, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));         \
      auto xb = reinterpret_cast<__nv_bfloat16*>(xc.data_ptr<float>());                                           \
      launch_k(ck, dim3(T), 256, smem, st, bp(mixed), bp(conv_w), conv_state.data_ptr<float>(),                   \
               (const int64_t*)slots.data_ptr<int64_t>(), (const int*)seq_of.data_ptr<int>(),                     \
               (const int*)cu.data_ptr<int>(), xb, C, (int)Hk);                                                   \
      C10_CUDA_KERNEL_LAUNCH_CHECK();                                                                             \
      launch_deltanet_chunk(xb, bp(mixed), conv_state.data_ptr<float>(), bp(z), bp(ba), ssm.data_ptr<float>(),    \
                            (const int64_t*)slots.data_ptr<int64_t>(), (const int*)cu.data_ptr<int>(),            \
                            (const float*)A_log.data_ptr<float>(), (const float*)dt_bias.data_ptr<float>(),       \
                            bp(norm_w), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), nseq, (int)Hk, (int)Hv, \
                            (float)eps, st);                                                                      \
      return;                                                                                                     \
    }                                                                                                             \
    auto ck = deltanet_conv_kernel<DK_, KC_, float>;                                                              \
    if (smem > 48 * 1024)                                                                                         \
      C10_CUDA_CHECK(cudaFuncSetAttribute(ck, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));           \
    launch_k(ck, dim3(T), 256, smem, st, bp(mixed), bp(conv_w), conv_state.data_ptr<float>(),                     \
             (const int64_t*)slots.data_ptr<int64_t>(), (const int*)seq_of.data_ptr<int>(),                       \
             (const int*)cu.data_ptr<int>(), xc.data_ptr<float>(), C, (int)Hk);                                    \
    C10_CUDA_KERNEL_LAUNCH_CHECK();                                                                               \
    launch_k(deltanet_scan_kernel<DK_, DV_, KC_, 2>, dim3(nseq, (unsigned)Hv), 2 * DV_, 0, st,                   \
             (const float*)xc.data_ptr<float>(), bp(mixed), bp(z), bp(ba), conv_state.data_ptr<float>(),           \
             ssm.data_ptr<float>(), (const int64_t*)slots.data_ptr<int64_t>(), (const int*)cu.data_ptr<int>(),    \
             (const float*)A_log.data_ptr<float>(), (const float*)dt_bias.data_ptr<float>(), bp(norm_w),          \
             reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), (int)Hk, (int)Hv, (float)eps);                      \
    C10_CUDA_KERNEL_LAUNCH_CHECK();                                                                               \
    return;                                                                                                       \
  }
  MB_DP(128, 128, 4)
  MB_DP(64, 64, 4)
#undef MB_DP
  TORCH_CHECK(false, "deltanet_prefill: unsupported head dims / conv kernel");
}

}  // namespace mb
