// Chunked gated-DeltaNet prefill on tensor cores (Qwen3-Next linear attention).
//
// The token-serial scan does two barriers per token, so a 32k-token sequence
// is a 65k-step dependent chain.  The chunked (WY / UT) form of the delta rule
// (Yang, Kautz, Hatamizadeh, "Gated Delta Networks", 2024) turns 64 tokens
// into a handful of small matrix products, so the chain is 512 chunk steps.
// Per chunk of C = 64 tokens (g = cumulative log-decay inside the chunk):
//   M   = strict_lower(diag(beta) K K^T * exp(g_i - g_j))
//   T   = (I + M)^{-1}                       (unit lower triangular)
//   u   = T (beta * V)        w = T (beta * exp(g) * K)
//   P   = lower(Q K^T * exp(g_i - g_j))
//   Vn  = u - w S                            (S: fp32 state [dk, dv])
//   O   = (exp(g) * Q) S + P Vn
//   S   = exp(g_last) S + (exp(g_last - g) * K)^T Vn
//   out = rmsnorm(O) * norm_w * silu(z)      (gated RMSNorm, per value head)
//
// One CTA of 8 warps per (sequence, value head); the state lives in registers
// (warp w owns state rows 16w .. 16w+15, all 128 columns) for the whole
// sequence, a bf16 copy of S^T in shared memory feeds the products that read
// it.  The products are warp-level tensor-core MMAs (mma.sync m16n8k16,
// bf16 operands, fp32 accumulation) on operands in padded shared memory: the
// chunk step is a dependent chain of small (64-row) products whose operands
// are produced by the previous product, so they are issued from registers and
// shared memory without a TMEM round trip.  T is built from 16x16 diagonal
// blocks (each inverted by forward substitution, one column per lane) and the
// block recurrence T_ij = -T_ii sum_k M_ik T_kj.
//
// Inputs are the outputs of deltanet_conv_kernel (conv + SiLU + q/k L2 norm,
// q scaled by dk^-1/2, bf16 [T, C]) plus the gate logits ba and z.  The next
// chunk's q / k / v rows are copied into a staging buffer with cp.async while
// the current chunk computes, so the chunk step never waits on global loads.
// Reference: pio/models/qwen3_coder_next/model.py:245-277 (a decayed linear
// attention in the reference, not the delta rule).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "launch.cuh"

namespace mb {

namespace {

constexpr int kC = 64;          // chunk length
constexpr int kD = 128;         // dk = dv
constexpr int kLdD = kD + 8;    // padded row (bf16 elements) of a [*, 128] operand
constexpr int kLdC = kC + 8;    // padded row of a [*, 64] operand
constexpr int kThreads = 256;

struct ChunkSmem {
  __nv_bfloat16 q[kC * kLdD];     // q, then exp(g) * q
  __nv_bfloat16 k[kC * kLdD];
  __nv_bfloat16 kT[kD * kLdC];    // (beta exp(g) k)^T, then (exp(g_last - g) k)^T
  __nv_bfloat16 vT[kD * kLdC];    // (beta v)^T, then Vn^T
  __nv_bfloat16 P[kC * kLdC];
  __nv_bfloat16 Tm[kC * kLdC];
  __nv_bfloat16 ST[kD * kLdD];    // S^T (bf16): row = value column, contiguous over key rows
  float Mf[kC * kLdD / 2];        // M ([64][65] fp32), then -w ([64][kLdD] bf16, aliased)
  float Tf[kC * (kC + 1)];        // T in fp32, and the block products
  float g[kC], gc[kC], beta[kC];
  float ss[2][kC];                // per-token sums of squares of O (two column halves)
  __nv_bfloat16 stg[3][kC * kLdD];  // next chunk's q, k, v rows, filled by cp.async during this chunk
};

// 16-byte asynchronous global -> shared copy; src_bytes = 0 fills the 16 bytes with zeros.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ void mma16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t lds32(const __nv_bfloat16* p) { return *reinterpret_cast<const uint32_t*>(p); }
// Two fp32 -> bf16 conversions in one packed instruction (the scalar form is a separate
// conversion per value, and the kernel is bound by that pipe otherwise).
__device__ __forceinline__ __nv_bfloat162 pk(float a, float b) { return __floats2bfloat162_rn(a, b); }
// A fragment (16x16) of a row-major [rows][ld] operand at (r0, k0).
__device__ __forceinline__ void lda(uint32_t* a, const __nv_bfloat16* A, int ld, int r0, int k0, int lane) {
  const int g = lane >> 2, t = lane & 3;
  a[0] = lds32(A + (r0 + g) * ld + k0 + 2 * t);
  a[1] = lds32(A + (r0 + g + 8) * ld + k0 + 2 * t);
  a[2] = lds32(A + (r0 + g) * ld + k0 + 2 * t + 8);
  a[3] = lds32(A + (r0 + g + 8) * ld + k0 + 2 * t + 8);
}
// C[r0:+16, n0:+8*NT] += A[r0:+16, 0:K] B[0:K, n0:+8*NT], A row-major [.][lda], B given as B^T row-major [n][ldb].
template <int NT>
__device__ __forceinline__ void warp_gemm(float (*c)[4], const __nv_bfloat16* A, int la, const __nv_bfloat16* Bt,
                                          int lb, int r0, int n0, int K, int lane) {
  const int g = lane >> 2, t = lane & 3;
  for (int k0 = 0; k0 < K; k0 += 16) {
    uint32_t a[4];
    lda(a, A, la, r0, k0, lane);
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const __nv_bfloat16* b = Bt + (n0 + n * 8 + g) * lb + k0 + 2 * t;
      mma16816(c[n], a, lds32(b), lds32(b + 8));
    }
  }
}

__device__ __forceinline__ float softplus_f(float x) { return x > 20.f ? x : log1pf(__expf(x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + __expf(-x)); }

__global__ void __launch_bounds__(kThreads, 1)
    deltanet_chunk_kernel(const __nv_bfloat16* __restrict__ xc, const __nv_bfloat16* __restrict__ mixed,
                          float* __restrict__ conv_state, const __nv_bfloat16* __restrict__ z,
                          const __nv_bfloat16* __restrict__ ba, float* __restrict__ ssm,
                          const int64_t* __restrict__ slots, const int* __restrict__ cu,
                          const float* __restrict__ A_log, const float* __restrict__ dt_bias,
                          const __nv_bfloat16* __restrict__ norm_w, __nv_bfloat16* __restrict__ out, int Hk, int Hv,
                          float eps) {
  extern __shared__ uint8_t smem_raw[];
  ChunkSmem& sm = *reinterpret_cast<ChunkSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  pdl_wait();
  pdl_trigger();
  const int s = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31, g4 = lane >> 2, t4 = lane & 3;
  const int hk = h / (Hv / Hk);
  const int Ctot = 2 * Hk * kD + Hv * kD;
  const int start = cu[s], L = cu[s + 1] - start;
  const int64_t slot = slots[s];
  float* S_g = ssm + (slot * Hv + h) * (int64_t)kD * kD;
  const float A = __expf(A_log[h]), dtb = dt_bias[h];
  // warp roles for the [64 x N] products: rows mt*16.., column half nh
  const int mt = warp & 3, nh = warp >> 2;

  // ---- state: registers (rows 16w.., all 128 columns: 16 fragments) + bf16 S^T in smem
  float S[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    const int r = warp * 16 + g4, c = n * 8 + 2 * t4;
    S[n][0] = S_g[(int64_t)r * kD + c];
    S[n][1] = S_g[(int64_t)r * kD + c + 1];
    S[n][2] = S_g[(int64_t)(r + 8) * kD + c];
    S[n][3] = S_g[(int64_t)(r + 8) * kD + c + 1];
  }
  auto store_ST = [&]() {
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      const int r = warp * 16 + g4, c = n * 8 + 2 * t4;
      const __nv_bfloat162 a = pk(S[n][0], S[n][1]), b = pk(S[n][2], S[n][3]);
      sm.ST[c * kLdD + r] = a.x;
      sm.ST[(c + 1) * kLdD + r] = a.y;
      sm.ST[c * kLdD + r + 8] = b.x;
      sm.ST[(c + 1) * kLdD + r + 8] = b.y;
    }
  };
  store_ST();

  const int nchunks = (L + kC - 1) / kC;
  // staging: chunk ch's q, k, v rows (16 x 16-byte pieces per 128-wide row); rows past the
  // sequence are zero-filled
  auto issue_stage = [&](int ch) {
    const int tb = start + ch * kC, nval = min(kC, L - ch * kC);
    for (int i = tid; i < 3 * kC * 16; i += kThreads) {
      const int a = i / (kC * 16), r = (i / 16) % kC, seg = i % 16;
      const int col = a == 0 ? hk * kD : a == 1 ? Hk * kD + hk * kD : 2 * Hk * kD + h * kD;
      const bool in = r < nval;
      const __nv_bfloat16* src = xc + (in ? (int64_t)(tb + r) * Ctot + col + seg * 8 : 0);
      cp_async16(sm.stg[a] + r * kLdD + seg * 8, src, in ? 16 : 0);
    }
    cp_async_commit();
  };
  if (nchunks > 0) issue_stage(0);
  for (int ch = 0; ch < nchunks; ++ch) {
    const int t0 = start + ch * kC;
    const int valid = min(kC, L - ch * kC);
    // ---------------- gates, then the cumulative log-decay
    if (tid < kC) {
      float gg = 0.f, bb = 0.f;
      if (tid < valid) {
        const int64_t r = t0 + tid;
        bb = sigmoid_f(__bfloat162float(ba[r * 2 * Hv + h]));
        gg = -A * softplus_f(__bfloat162float(ba[r * 2 * Hv + Hv + h]) + dtb);
      }
      sm.g[tid] = gg;
      sm.beta[tid] = bb;
    }
    __syncthreads();
    if (tid < kC) {
      float acc = 0.f;
      for (int i = 0; i <= tid; ++i) acc += sm.g[i];
      sm.gc[tid] = acc;
    }
    // ---------------- operands from the staging buffer: q, k rows (bf16), (beta v)^T
    cp_async_wait_all();
    __syncthreads();  // staged rows visible to every thread; gates of this chunk written
    // 8 channels per step: q, k rows copied; (beta v)^T and (beta exp(g) k)^T transposed
    for (int i = tid; i < kC * 16; i += kThreads) {
      const int r = i / 16, c0 = (i % 16) * 8;
      const uint4 q8 = *reinterpret_cast<const uint4*>(sm.stg[0] + r * kLdD + c0);
      const uint4 k8 = *reinterpret_cast<const uint4*>(sm.stg[1] + r * kLdD + c0);
      const uint4 v8 = *reinterpret_cast<const uint4*>(sm.stg[2] + r * kLdD + c0);
      *reinterpret_cast<uint4*>(sm.q + r * kLdD + c0) = q8;
      *reinterpret_cast<uint4*>(sm.k + r * kLdD + c0) = k8;
      const float b = sm.beta[r], bk = b * __expf(sm.gc[r]);
      const __nv_bfloat16* kh = reinterpret_cast<const __nv_bfloat16*>(&k8);
      const __nv_bfloat16* vh = reinterpret_cast<const __nv_bfloat16*>(&v8);
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const __nv_bfloat162 vv = pk(__bfloat162float(vh[e]) * b, __bfloat162float(vh[e + 1]) * b);
        const __nv_bfloat162 kv = pk(__bfloat162float(kh[e]) * bk, __bfloat162float(kh[e + 1]) * bk);
        sm.vT[(c0 + e) * kLdC + r] = vv.x;
        sm.vT[(c0 + e + 1) * kLdC + r] = vv.y;
        sm.kT[(c0 + e) * kLdC + r] = kv.x;
        sm.kT[(c0 + e + 1) * kLdC + r] = kv.y;
      }
    }
    __syncthreads();
    if (ch + 1 < nchunks) issue_stage(ch + 1);  // overlaps the rest of this chunk
    // ---------------- K K^T -> M (strict lower, decayed, beta rows);  Q K^T -> P (lower, decayed)
    {
      float kk[4][4], qk[4][4];
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) kk[n][e] = qk[n][e] = 0.f;
      warp_gemm<4>(kk, sm.k, kLdD, sm.k, kLdD, mt * 16, nh * 32, kD, lane);
      warp_gemm<4>(qk, sm.q, kLdD, sm.k, kLdD, mt * 16, nh * 32, kD, lane);
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int e2 = 0; e2 < 4; e2 += 2) {
          const int i = mt * 16 + g4 + (e2 >> 1) * 8, j = nh * 32 + n * 8 + 2 * t4;
          const float d0 = i >= j ? __expf(sm.gc[i] - sm.gc[j]) : 0.f;
          const float d1 = i >= j + 1 ? __expf(sm.gc[i] - sm.gc[j + 1]) : 0.f;
          sm.Mf[i * (kC + 1) + j] = i > j ? sm.beta[i] * kk[n][e2] * d0 : 0.f;
          sm.Mf[i * (kC + 1) + j + 1] = i > j + 1 ? sm.beta[i] * kk[n][e2 + 1] * d1 : 0.f;
          *reinterpret_cast<__nv_bfloat162*>(sm.P + i * kLdC + j) = pk(qk[n][e2] * d0, qk[n][e2 + 1] * d1);
        }
    }
    __syncthreads();
    // exp(g) q in place (used by O = (exp(g) q) S); diagonal 16x16 blocks of T by forward substitution
    for (int i = tid; i < kC * 16; i += kThreads) {
      const int r = i / 16, c0 = (i % 16) * 8;
      uint4 q8 = *reinterpret_cast<const uint4*>(sm.q + r * kLdD + c0);
      __nv_bfloat16* qh = reinterpret_cast<__nv_bfloat16*>(&q8);
      const float e = __expf(sm.gc[r]);
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        const __nv_bfloat162 v = pk(__bfloat162float(qh[j]) * e, __bfloat162float(qh[j + 1]) * e);
        qh[j] = v.x;
        qh[j + 1] = v.y;
      }
      *reinterpret_cast<uint4*>(sm.q + r * kLdD + c0) = q8;
    }
    if (warp < 4 && lane < 16) {  // warp b inverts diagonal block b; lane = column
      const int b0 = warp * 16, c = lane;
      float col[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float v = (i == c) ? 1.f : 0.f;
#pragma unroll
        for (int j = 0; j < i; ++j) v -= sm.Mf[(b0 + i) * (kC + 1) + b0 + j] * col[j];
        col[i] = v;
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) sm.Tf[(b0 + i) * (kC + 1) + b0 + c] = col[i];
    }
    __syncthreads();
    // off-diagonal blocks, one block row at a time: X_ij = sum_{k=j}^{i-1} M_ik T_kj ; T_ij = -T_ii X_ij
    for (int bi = 1; bi < 4; ++bi) {
      const int nent = bi * 256;  // entries of blocks (bi, 0 .. bi-1); up to 3 per thread
      float x[3] = {0.f, 0.f, 0.f};
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        const int e = tid + q * kThreads;
        if (e < nent) {
          const int bj = e / 256, row = bi * 16 + (e % 256) / 16, col = bj * 16 + e % 16;
          for (int kk2 = bj * 16; kk2 < bi * 16; ++kk2)
            x[q] += sm.Mf[row * (kC + 1) + kk2] * sm.Tf[kk2 * (kC + 1) + col];
        }
      }
      __syncthreads();
#pragma unroll
      for (int q = 0; q < 3; ++q) {  // X parked in T's own (still empty) block
        const int e = tid + q * kThreads;
        if (e < nent) sm.Tf[(bi * 16 + (e % 256) / 16) * (kC + 1) + (e / 256) * 16 + e % 16] = x[q];
      }
      __syncthreads();
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        const int e = tid + q * kThreads;
        x[q] = 0.f;
        if (e < nent) {
          const int bj = e / 256, row = bi * 16 + (e % 256) / 16, col = bj * 16 + e % 16;
#pragma unroll
          for (int kk2 = 0; kk2 < 16; ++kk2)
            x[q] -= sm.Tf[row * (kC + 1) + bi * 16 + kk2] * sm.Tf[(bi * 16 + kk2) * (kC + 1) + col];
        }
      }
      __syncthreads();
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        const int e = tid + q * kThreads;
        if (e < nent) sm.Tf[(bi * 16 + (e % 256) / 16) * (kC + 1) + (e / 256) * 16 + e % 16] = x[q];
      }
      __syncthreads();
    }
    // T (lower triangular, zero above the diagonal) as a bf16 operand
    for (int i = tid; i < kC * kC; i += kThreads) {
      const int r = i / kC, c = i % kC;
      sm.Tm[r * kLdC + c] = __float2bfloat16_rn(c <= r ? sm.Tf[r * (kC + 1) + c] : 0.f);
    }
    __syncthreads();
    // ---------------- u = T (beta v) [registers];  -w = -T (beta exp(g) k) -> smem (bf16, over Mf)
    float u[8][4], wv[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) u[n][e] = wv[n][e] = 0.f;
    warp_gemm<8>(u, sm.Tm, kLdC, sm.vT, kLdC, mt * 16, nh * 64, kC, lane);
    warp_gemm<8>(wv, sm.Tm, kLdC, sm.kT, kLdC, mt * 16, nh * 64, kC, lane);
    __nv_bfloat16* wneg = reinterpret_cast<__nv_bfloat16*>(sm.Mf);  // [64][kLdD] bf16 fits in Mf
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const int r = mt * 16 + g4, c = nh * 64 + n * 8 + 2 * t4;
      *reinterpret_cast<__nv_bfloat162*>(wneg + r * kLdD + c) = pk(-wv[n][0], -wv[n][1]);
      *reinterpret_cast<__nv_bfloat162*>(wneg + (r + 8) * kLdD + c) = pk(-wv[n][2], -wv[n][3]);
    }
    __syncthreads();
    // (exp(g_last - g) k)^T for the state update (kT is free: w is done)
    const float glast = sm.gc[kC - 1];
    for (int i = tid; i < kC * 16; i += kThreads) {
      const int r = i / 16, c0 = (i % 16) * 8;
      const uint4 k8 = *reinterpret_cast<const uint4*>(sm.k + r * kLdD + c0);
      const __nv_bfloat16* kh = reinterpret_cast<const __nv_bfloat16*>(&k8);
      const float e = __expf(glast - sm.gc[r]);
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        const __nv_bfloat162 v = pk(__bfloat162float(kh[j]) * e, __bfloat162float(kh[j + 1]) * e);
        sm.kT[(c0 + j) * kLdC + r] = v.x;
        sm.kT[(c0 + j + 1) * kLdC + r] = v.y;
      }
    }
    // ---------------- Vn = u - w S  (B^T = S^T)
    warp_gemm<8>(u, wneg, kLdD, sm.ST, kLdD, mt * 16, nh * 64, kD, lane);
    __syncthreads();  // every warp has read vT as (beta v)^T
#pragma unroll
    for (int n = 0; n < 8; ++n) {  // Vn^T into vT
      const int r = mt * 16 + g4, c = nh * 64 + n * 8 + 2 * t4;
      const __nv_bfloat162 a = pk(u[n][0], u[n][1]), b = pk(u[n][2], u[n][3]);
      sm.vT[c * kLdC + r] = a.x;
      sm.vT[(c + 1) * kLdC + r] = a.y;
      sm.vT[c * kLdC + r + 8] = b.x;
      sm.vT[(c + 1) * kLdC + r + 8] = b.y;
    }
    __syncthreads();
    // ---------------- O = (exp(g) q) S + P Vn   (reuse wv as the accumulator)
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) wv[n][e] = 0.f;
    warp_gemm<8>(wv, sm.q, kLdD, sm.ST, kLdD, mt * 16, nh * 64, kD, lane);
    warp_gemm<8>(wv, sm.P, kLdC, sm.vT, kLdC, mt * 16, nh * 64, kC, lane);
    // ---------------- S = exp(g_last) S + kd^T Vn   (rows 16w.. of the state, K = chunk tokens)
    const float dl = __expf(glast);
#pragma unroll
    for (int n = 0; n < 16; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) S[n][e] *= dl;
    warp_gemm<16>(S, sm.kT, kLdC, sm.vT, kLdC, warp * 16, 0, kC, lane);
    // ---------------- gated RMSNorm of O rows, output
    {
      float ssr[2] = {0.f, 0.f};
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        ssr[0] += wv[n][0] * wv[n][0] + wv[n][1] * wv[n][1];
        ssr[1] += wv[n][2] * wv[n][2] + wv[n][3] * wv[n][3];
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        ssr[e] += __shfl_xor_sync(0xffffffffu, ssr[e], 1);
        ssr[e] += __shfl_xor_sync(0xffffffffu, ssr[e], 2);
      }
      if (t4 == 0) {
        sm.ss[nh][mt * 16 + g4] = ssr[0];
        sm.ss[nh][mt * 16 + g4 + 8] = ssr[1];
      }
    }
    __syncthreads();  // sums of squares complete; every warp is past its reads of S^T
    store_ST();
    {
      // this thread's two rows: r0 = mt*16 + g4 and r0 + 8; columns in adjacent pairs
      const int r0 = mt * 16 + g4;
      const float inv0 = rsqrtf((sm.ss[0][r0] + sm.ss[1][r0]) / kD + eps);
      const float inv1 = rsqrtf((sm.ss[0][r0 + 8] + sm.ss[1][r0 + 8]) / kD + eps);
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const int c = nh * 64 + n * 8 + 2 * t4;
        const __nv_bfloat162 nw2 = *reinterpret_cast<const __nv_bfloat162*>(norm_w + c);
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          const int r = r0 + hr * 8;
          if (r < valid) {
            const int64_t off = (int64_t)(t0 + r) * Hv * kD + h * kD + c;
            const __nv_bfloat162 z2 = *reinterpret_cast<const __nv_bfloat162*>(z + off);
            const float inv = hr ? inv1 : inv0;
            *reinterpret_cast<__nv_bfloat162*>(out + off) =
                pk(wv[n][2 * hr] * inv * __bfloat162float(nw2.x) * silu(__bfloat162float(z2.x)),
                   wv[n][2 * hr + 1] * inv * __bfloat162float(nw2.y) * silu(__bfloat162float(z2.y)));
          }
        }
      }
    }
    __syncthreads();  // the next chunk overwrites every operand buffer
  }
  // ---- conv history: the last 3 inputs of (history ++ sequence) of this head's channels
  {
    constexpr int KC = 4;
    const int rep = Hv / Hk;
    float* cs = conv_state + slot * (int64_t)Ctot * (KC - 1);
    auto advance = [&](int c) {
      float nv[KC - 1];
#pragma unroll
      for (int k = 0; k < KC - 1; ++k) {
        const int idx = L + k;  // index into history ++ inputs
        nv[k] = idx < KC - 1 ? cs[c * (KC - 1) + idx] : __bfloat162float(mixed[(int64_t)(start + idx - (KC - 1)) * Ctot + c]);
      }
#pragma unroll
      for (int k = 0; k < KC - 1; ++k) cs[c * (KC - 1) + k] = nv[k];
    };
    if (tid < kD) {
      advance(2 * Hk * kD + h * kD + tid);
      if (h % rep == 0) {
        advance(hk * kD + tid);
        advance(Hk * kD + hk * kD + tid);
      }
    }
  }
  // ---- state back to memory
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    const int r = warp * 16 + g4, c = n * 8 + 2 * t4;
    S_g[(int64_t)r * kD + c] = S[n][0];
    S_g[(int64_t)r * kD + c + 1] = S[n][1];
    S_g[(int64_t)(r + 8) * kD + c] = S[n][2];
    S_g[(int64_t)(r + 8) * kD + c + 1] = S[n][3];
  }
}

}  // namespace

// Chunked prefill scan (dk = dv = 128, conv kernel 4), after deltanet_conv_kernel: xc [T, C] fp32;
// mixed [T, C] raw conv inputs (the conv history advances to the last three); z [T, Hv*128],
// ba [T, 2*Hv] bf16; ssm [slots, Hv, 128, 128] fp32 updated in place; out [T, Hv*128] bf16.
void launch_deltanet_chunk(const __nv_bfloat16* xc, const __nv_bfloat16* mixed, float* conv_state, const __nv_bfloat16* z,
                           const __nv_bfloat16* ba, float* ssm, const int64_t* slots, const int* cu, const float* A_log,
                           const float* dt_bias, const __nv_bfloat16* norm_w, __nv_bfloat16* out, int nseq, int Hk,
                           int Hv, float eps, cudaStream_t st) {
  const size_t smem = sizeof(ChunkSmem) + 128;
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(deltanet_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)smem));
    attr = true;
  }
  launch_k(deltanet_chunk_kernel, dim3(nseq, (unsigned)Hv), kThreads, smem, st, xc, mixed, conv_state, z, ba, ssm,
           slots, cu, A_log, dt_bias, norm_w, out, Hk, Hv, eps);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mb
