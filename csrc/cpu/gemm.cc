// GEMM  y[M, N] = x[M, K] * w[N, K]^T  (both operands K-contiguous), fp32
// activations and accumulation; weights fp32, bf16 or int8 (+ per-row scale).
//
// Register-blocked dot-product kernel: a 4 x 4 tile of outputs keeps 16
// accumulators along K (AVX-512 where the CPU has it, chosen at run time: 16
// lanes; else AVX2: 8 lanes); the 8 loads per k-step (4 rows of x, 4 rows of w)
// feed 16 FMAs.  OpenMP splits the tile grid; the single-row case (decode GEMV,
// weight-bandwidth bound) splits N.
//
// bf16 weights are widened to fp32 in registers (a bf16 value is the upper
// half of the fp32 with the same value, so the widening is a 16-bit shift):
// the result equals fp32 math on the bf16-rounded weights while the weight
// stream, which bounds decode, is halved.  int8 weights are widened the same
// way (sign-extend, convert) and the per-row scale multiplies each output once.
#include <immintrin.h>
#include <omp.h>
#include <algorithm>
#include <cstdint>
#include "cpu_ops.h"

namespace mbcpu {

static inline float hsum(__m256 v) {
  __m128 lo = _mm256_castps256_ps128(v), hi = _mm256_extractf128_ps(v, 1);
  lo = _mm_add_ps(lo, hi);
  lo = _mm_hadd_ps(lo, lo);
  lo = _mm_hadd_ps(lo, lo);
  return _mm_cvtss_f32(lo);
}

static inline float to_f32(float v) { return v; }
static inline float to_f32(int8_t v) { return (float)v; }
static inline float to_f32(uint16_t v) {
  const uint32_t u = (uint32_t)v << 16;
  float f;
  __builtin_memcpy(&f, &u, 4);
  return f;
}

// 8 weights as fp32 (AVX2)
static inline __m256 load8(const float* p) { return _mm256_loadu_ps(p); }
static inline __m256 load8(const uint16_t* p) {
  const __m128i h = _mm_loadu_si128(reinterpret_cast<const __m128i*>(p));
  return _mm256_castsi256_ps(_mm256_slli_epi32(_mm256_cvtepu16_epi32(h), 16));
}

static inline __m256 load8(const int8_t* p) {
  const __m128i b = _mm_loadl_epi64(reinterpret_cast<const __m128i*>(p));
  return _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(b));
}

// 16 weights as fp32 (AVX-512)
__attribute__((target("avx512f"))) static inline __m512 load16(const float* p) { return _mm512_loadu_ps(p); }
__attribute__((target("avx512f"))) static inline __m512 load16(const uint16_t* p) {
  const __m256i h = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(p));
  return _mm512_castsi512_ps(_mm512_slli_epi32(_mm512_cvtepu16_epi32(h), 16));
}

__attribute__((target("avx512f"))) static inline __m512 load16(const int8_t* p) {
  const __m128i b = _mm_loadu_si128(reinterpret_cast<const __m128i*>(p));
  return _mm512_cvtepi32_ps(_mm512_cvtepi8_epi32(b));
}

// rows [m0, m0+mr) x cols [n0, n0+nr), mr, nr <= 4
template <typename WT>
static void tile(const float* x, const WT* w, float* y, int64_t K, int64_t N, int64_t m0, int mr, int64_t n0,
                 int nr) {
  __m256 acc[4][4];
  for (int i = 0; i < 4; ++i)
    for (int j = 0; j < 4; ++j) acc[i][j] = _mm256_setzero_ps();
  const float* xr[4];
  const WT* wr[4];
  for (int i = 0; i < 4; ++i) xr[i] = x + (m0 + (i < mr ? i : 0)) * K;
  for (int j = 0; j < 4; ++j) wr[j] = w + (n0 + (j < nr ? j : 0)) * K;
  int64_t k = 0;
  for (; k + 8 <= K; k += 8) {
    __m256 xv[4], wv[4];
    for (int i = 0; i < 4; ++i) xv[i] = _mm256_loadu_ps(xr[i] + k);
    for (int j = 0; j < 4; ++j) wv[j] = load8(wr[j] + k);
    for (int i = 0; i < 4; ++i)
      for (int j = 0; j < 4; ++j) acc[i][j] = _mm256_fmadd_ps(xv[i], wv[j], acc[i][j]);
  }
  for (int i = 0; i < mr; ++i)
    for (int j = 0; j < nr; ++j) {
      float s = hsum(acc[i][j]);
      for (int64_t kk = k; kk < K; ++kk) s += xr[i][kk] * to_f32(wr[j][kk]);
      y[(m0 + i) * N + n0 + j] = s;
    }
}

// AVX-512 tile of MR x NR outputs.  Compiled for AVX-512 through the function's
// target attribute and chosen at run time, so the library still loads on hosts
// without AVX-512.
template <int MR, int NR, typename WT>
__attribute__((target("avx512f"))) static void tile512(const float* x, const WT* w, float* y, int64_t K,
                                                       int64_t N, int64_t m0, int mr, int64_t n0, int nr) {
  __m512 acc[MR][NR];
  for (int i = 0; i < MR; ++i)
    for (int j = 0; j < NR; ++j) acc[i][j] = _mm512_setzero_ps();
  const float* xr[MR];
  const WT* wr[NR];
  for (int i = 0; i < MR; ++i) xr[i] = x + (m0 + (i < mr ? i : 0)) * K;
  for (int j = 0; j < NR; ++j) wr[j] = w + (n0 + (j < nr ? j : 0)) * K;
  int64_t k = 0;
  for (; k + 16 <= K; k += 16) {
    __m512 xv[MR];
    for (int i = 0; i < MR; ++i) xv[i] = _mm512_loadu_ps(xr[i] + k);
    for (int j = 0; j < NR; ++j) {
      const __m512 wv = load16(wr[j] + k);
      for (int i = 0; i < MR; ++i) acc[i][j] = _mm512_fmadd_ps(xv[i], wv, acc[i][j]);
    }
  }
  for (int i = 0; i < mr; ++i)
    for (int j = 0; j < nr; ++j) {
      float s = _mm512_reduce_add_ps(acc[i][j]);
      for (int64_t kk = k; kk < K; ++kk) s += xr[i][kk] * to_f32(wr[j][kk]);
      y[(m0 + i) * N + n0 + j] = s;
    }
}

static bool has_avx512() {
  static const bool v = __builtin_cpu_supports("avx512f");
  return v;
}

template <typename WT>
static void gemv(const float* x, const WT* w, float* y, int64_t K, int64_t N) {
#pragma omp parallel for schedule(static)
  for (int64_t n0 = 0; n0 < N; n0 += 4) {
    const int nr = (int)std::min<int64_t>(4, N - n0);
    __m256 a0[4], a1[4];
    for (int j = 0; j < 4; ++j) a0[j] = a1[j] = _mm256_setzero_ps();
    const WT* wr[4];
    for (int j = 0; j < 4; ++j) wr[j] = w + (n0 + (j < nr ? j : 0)) * K;
    int64_t k = 0;
    for (; k + 16 <= K; k += 16) {
      const __m256 x0 = _mm256_loadu_ps(x + k), x1 = _mm256_loadu_ps(x + k + 8);
      for (int j = 0; j < 4; ++j) {
        a0[j] = _mm256_fmadd_ps(x0, load8(wr[j] + k), a0[j]);
        a1[j] = _mm256_fmadd_ps(x1, load8(wr[j] + k + 8), a1[j]);
      }
    }
    for (int j = 0; j < nr; ++j) {
      float s = hsum(_mm256_add_ps(a0[j], a1[j]));
      for (int64_t kk = k; kk < K; ++kk) s += x[kk] * to_f32(wr[j][kk]);
      y[n0 + j] = s;
    }
  }
}

template <typename WT>
static void gemm(const float* px, const WT* pw, float* py, int64_t M, int64_t K, int64_t N) {
  if (M == 1) {
    gemv(px, pw, py, K, N);
    return;
  }
  const int64_t MB = 64, NB = 64;
  const int64_t mt = (M + MB - 1) / MB, nt = (N + NB - 1) / NB;
  if (has_avx512()) {
    constexpr int TM = 4, TN = 4;  // 4 x 6 measured the same within noise; 4 x 4 held up better at K = 3072
    const int64_t NB5 = 16 * TN;   // column block: a multiple of the tile width
    const int64_t nt5 = (N + NB5 - 1) / NB5;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
    for (int64_t bi = 0; bi < mt; ++bi)
      for (int64_t bj = 0; bj < nt5; ++bj) {
        const int64_t m_end = std::min(M, (bi + 1) * MB), n_end = std::min(N, (bj + 1) * NB5);
        for (int64_t n0 = bj * NB5; n0 < n_end; n0 += TN)
          for (int64_t m0 = bi * MB; m0 < m_end; m0 += TM)
            tile512<TM, TN>(px, pw, py, K, N, m0, (int)std::min<int64_t>(TM, m_end - m0), n0,
                            (int)std::min<int64_t>(TN, n_end - n0));
      }
    return;
  }
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
  for (int64_t bi = 0; bi < mt; ++bi)
    for (int64_t bj = 0; bj < nt; ++bj) {
      const int64_t m_end = std::min(M, (bi + 1) * MB), n_end = std::min(N, (bj + 1) * NB);
      for (int64_t n0 = bj * NB; n0 < n_end; n0 += 4)
        for (int64_t m0 = bi * MB; m0 < m_end; m0 += 4)
          tile(px, pw, py, K, N, m0, (int)std::min<int64_t>(4, m_end - m0), n0, (int)std::min<int64_t>(4, n_end - n0));
    }
}

// int8 weight-only: y = (x . q^T) * scale[n], the per-channel scale applied once per output
void linear_w8(const at::Tensor& x, const at::Tensor& q, const at::Tensor& scale, at::Tensor& y) {
  TORCH_CHECK(x.scalar_type() == at::kFloat && y.scalar_type() == at::kFloat && scale.scalar_type() == at::kFloat);
  TORCH_CHECK(q.scalar_type() == at::kChar, "linear_w8: weights must be int8");
  TORCH_CHECK(x.is_contiguous() && q.is_contiguous() && y.is_contiguous() && scale.is_contiguous());
  const int64_t M = x.size(0), K = x.size(1), N = q.size(0);
  TORCH_CHECK(q.size(1) == K && y.size(0) == M && y.size(1) == N && scale.numel() == N);
  float* py = y.data_ptr<float>();
  gemm(x.data_ptr<float>(), reinterpret_cast<const int8_t*>(q.data_ptr()), py, M, K, N);
  const float* sc = scale.data_ptr<float>();
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < M; ++i)
    for (int64_t n = 0; n < N; ++n) py[i * N + n] *= sc[n];
}

void linear(const at::Tensor& x, const at::Tensor& w, at::Tensor& y) {
  TORCH_CHECK(x.scalar_type() == at::kFloat && y.scalar_type() == at::kFloat);
  TORCH_CHECK(w.scalar_type() == at::kFloat || w.scalar_type() == at::kBFloat16,
              "linear: weights must be fp32 or bf16");
  TORCH_CHECK(x.is_contiguous() && w.is_contiguous() && y.is_contiguous());
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K && y.size(0) == M && y.size(1) == N);
  const float* px = x.data_ptr<float>();
  float* py = y.data_ptr<float>();
  if (w.scalar_type() == at::kFloat)
    gemm(px, w.data_ptr<float>(), py, M, K, N);
  else
    gemm(px, reinterpret_cast<const uint16_t*>(w.data_ptr()), py, M, K, N);
}

}  // namespace mbcpu
