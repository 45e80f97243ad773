// CPU operators other than GEMM (fp32).
// KV cache layouts match the GPU: K [blocks, Hkv, BS, D], V [blocks, Hkv, D, BS]
// (V is stored transposed inside a block so the GPU P.V product reads it
// K-major).
#include <immintrin.h>
#include <omp.h>
#include <algorithm>
#include <cmath>
#include <numeric>
#include <vector>
#include "cpu_ops.h"

namespace mbcpu {

static const float* cf(const at::Tensor& t) { return t.data_ptr<float>(); }

// fp32 dot product with AVX2 FMAs (two 8-lane accumulators), scalar tail
static inline float dot(const float* a, const float* b, int64_t n) {
  __m256 s0 = _mm256_setzero_ps(), s1 = _mm256_setzero_ps();
  int64_t i = 0;
  for (; i + 16 <= n; i += 16) {
    s0 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), s0);
    s1 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i + 8), _mm256_loadu_ps(b + i + 8), s1);
  }
  for (; i + 8 <= n; i += 8) s0 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), s0);
  s0 = _mm256_add_ps(s0, s1);
  __m128 lo = _mm_add_ps(_mm256_castps256_ps128(s0), _mm256_extractf128_ps(s0, 1));
  lo = _mm_hadd_ps(lo, lo);
  lo = _mm_hadd_ps(lo, lo);
  float r = _mm_cvtss_f32(lo);
  for (; i < n; ++i) r += a[i] * b[i];
  return r;
}
static float* mf(at::Tensor& t) { return t.data_ptr<float>(); }

void rmsnorm(const at::Tensor& x, const c10::optional<at::Tensor>& residual, const at::Tensor& w, at::Tensor& out,
             double eps) {
  TORCH_CHECK(x.is_contiguous() && out.is_contiguous() && x.scalar_type() == at::kFloat);
  const int64_t H = x.size(-1), R = x.numel() / H;
  const bool add = residual && residual->defined();
  float* r = add ? residual->data_ptr<float>() : nullptr;
  const float *px = cf(x), *pw = cf(w);
  float* po = mf(out);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < R; ++i) {
    const float* src = px + i * H;
    if (add) {
      float* rr = r + i * H;
      for (int64_t j = 0; j < H; ++j) rr[j] += src[j];
      src = rr;
    }
    double ss = 0;
    for (int64_t j = 0; j < H; ++j) ss += (double)src[j] * src[j];
    const float inv = 1.f / std::sqrt((float)(ss / H) + (float)eps);
    for (int64_t j = 0; j < H; ++j) po[i * H + j] = src[j] * inv * pw[j];
  }
}

void rope_qknorm(const at::Tensor& qkv, const c10::optional<at::Tensor>& q_w, const c10::optional<at::Tensor>& k_w,
                 const at::Tensor& positions, const at::Tensor& inv_freq, const c10::optional<at::Tensor>& slots,
                 at::Tensor& q_out, at::Tensor& k_cache, at::Tensor& v_cache, int64_t Hq, int64_t Hkv, int64_t D,
                 int64_t rot, double eps) {
  const int64_t T = qkv.size(0), stride = qkv.stride(0);
  const float* src = cf(qkv);
  const int* pos = positions.data_ptr<int>();
  const float* invf = cf(inv_freq);
  const int* sl = (slots && slots->defined()) ? slots->data_ptr<int>() : nullptr;
  const float* qw = (q_w && q_w->defined()) ? q_w->data_ptr<float>() : nullptr;
  const float* kw = (k_w && k_w->defined()) ? k_w->data_ptr<float>() : nullptr;
  const int64_t bs = k_cache.size(2);
  float *pq = mf(q_out), *pk = mf(k_cache), *pv = mf(v_cache);
  const int64_t nh = Hq + 2 * Hkv;  // each head kind iterated with its own count (GQA-safe)
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t t = 0; t < T; ++t)
    for (int64_t h = 0; h < nh; ++h) {
      std::vector<float> v(src + t * stride + h * D, src + t * stride + h * D + D);
      const bool is_q = h < Hq, is_k = !is_q && h < Hq + Hkv;
      if (!is_q && (!sl || sl[t] < 0)) continue;
      if (is_q || is_k) {
        const float* nw = is_q ? qw : kw;
        if (nw) {
          double ss = 0;
          for (int64_t d = 0; d < D; ++d) ss += (double)v[d] * v[d];
          const float inv = 1.f / std::sqrt((float)(ss / D) + (float)eps);
          for (int64_t d = 0; d < D; ++d) v[d] = v[d] * inv * nw[d];
        }
        const int64_t half = rot / 2;
        for (int64_t i = 0; i < half; ++i) {
          const float a = (float)pos[t] * invf[i];
          const float c = std::cos(a), s = std::sin(a);
          const float x1 = v[i], x2 = v[i + half];
          v[i] = x1 * c - x2 * s;
          v[i + half] = x2 * c + x1 * s;
        }
      }
      if (is_q) {
        std::copy(v.begin(), v.end(), pq + (t * Hq + h) * D);
      } else {
        const int64_t blk = sl[t] / bs, off = sl[t] % bs;
        if (is_k) {
          std::copy(v.begin(), v.end(), pk + ((blk * Hkv + (h - Hq)) * bs + off) * D);
        } else {
          float* dst = pv + ((blk * Hkv + (h - Hq - Hkv)) * D) * bs + off;
          for (int64_t d = 0; d < D; ++d) dst[d * bs] = v[d];
        }
      }
    }
}

// Causal paged attention for a batch of sequences.  Sequence b has q_lens[b]
// new query rows (packed back to back in q) sitting at the END of its
// ctx_lens[b]-token context; decode is q_lens == 1.  GQA: query head h reads
// KV head h / (Hq/Hkv).
void attn_paged(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                const at::Tensor& block_tables, const at::Tensor& ctx_lens, const at::Tensor& q_lens,
                at::Tensor& out, double scale) {
  const int64_t Hq = q.size(1), D = q.size(2), Hkv = k_cache.size(1), bs = k_cache.size(2);
  const int64_t B = ctx_lens.size(0), MB = block_tables.size(1), G = Hq / Hkv;
  const int* bt = block_tables.data_ptr<int>();
  const int* cl = ctx_lens.data_ptr<int>();
  const int* ql = q_lens.data_ptr<int>();
  std::vector<int64_t> start(B + 1, 0);
  for (int64_t b = 0; b < B; ++b) start[b + 1] = start[b] + ql[b];
  const float *pq = cf(q), *pk = cf(k_cache), *pv = cf(v_cache);
  float* po = mf(out);
  const int64_t rows = start[B];
#pragma omp parallel for collapse(2) schedule(dynamic, 4)
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t h = 0; h < Hq; ++h) {
      const int64_t b = std::upper_bound(start.begin(), start.end(), r) - start.begin() - 1;
      const int64_t n = cl[b] - ql[b] + (r - start[b]) + 1;  // causal: keys [0, n)
      const int64_t hk = h / G;
      const float* qv = pq + (r * Hq + h) * D;
      std::vector<float> s(n);
      float mx = -INFINITY;
      for (int64_t j = 0; j < n; ++j) {  // K rows are contiguous: one vector dot product per key
        const int64_t blk = bt[b * MB + j / bs];
        s[j] = dot(qv, pk + ((blk * Hkv + hk) * bs + j % bs) * D, D) * (float)scale;
        mx = std::max(mx, s[j]);
      }
      float sum = 0.f;
      for (int64_t j = 0; j < n; ++j) sum += (s[j] = std::exp(s[j] - mx));
      const float inv = 1.f / sum;
      for (int64_t j = 0; j < n; ++j) s[j] *= inv;
      float* o = po + (r * Hq + h) * D;
      std::fill(o, o + D, 0.f);
      // V is stored [D, bs] inside a block: per block, each output element is one contiguous
      // dot product over the block's tokens
      for (int64_t j0 = 0; j0 < n; j0 += bs) {
        const int64_t blk = bt[b * MB + j0 / bs];
        const int64_t cnt = std::min<int64_t>(bs, n - j0);
        const float* vb = pv + ((blk * Hkv + hk) * D) * bs;
        for (int64_t d = 0; d < D; ++d) o[d] += dot(s.data() + j0, vb + d * bs, cnt);
      }
    }
}

void swiglu(const at::Tensor& gu, at::Tensor& out) {
  const int64_t I = gu.size(-1) / 2, R = gu.numel() / (2 * I);
  const float* p = cf(gu);
  float* o = mf(out);
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < R; ++r)
    for (int64_t i = 0; i < I; ++i) {
      const float g = p[r * 2 * I + i], u = p[r * 2 * I + I + i];
      o[r * I + i] = g / (1.f + std::exp(-g)) * u;
    }
}

void gelu_tanh(const at::Tensor& x, at::Tensor& out) {
  const int64_t n = x.numel();
  const float* p = cf(x);
  float* o = mf(out);
  const float c = std::sqrt(2.f / (float)M_PI);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) o[i] = 0.5f * p[i] * (1.f + std::tanh(c * (p[i] + 0.044715f * p[i] * p[i] * p[i])));
}

void embed(const at::Tensor& ids, const at::Tensor& table, at::Tensor& out) {
  const int64_t T = ids.numel(), H = table.size(1), V = table.size(0);
  const int64_t* pi = ids.data_ptr<int64_t>();
  const float* pt = cf(table);
  float* po = mf(out);
  for (int64_t t = 0; t < T; ++t) {
    const int64_t id = std::min<int64_t>(std::max<int64_t>(pi[t], 0), V - 1);
    std::copy(pt + id * H, pt + id * H + H, po + t * H);
  }
}

at::Tensor argmax(const at::Tensor& logits) {
  const int64_t R = logits.size(0), V = logits.size(1);
  auto out = at::empty({R}, at::kLong);
  const float* p = cf(logits);
  int64_t* o = out.data_ptr<int64_t>();
  for (int64_t r = 0; r < R; ++r) o[r] = std::max_element(p + r * V, p + r * V + V) - (p + r * V);
  return out;
}

void moe_route(const at::Tensor& logits, int64_t k, bool renorm, at::Tensor& ids, at::Tensor& wts) {
  const int64_t T = logits.size(0), E = logits.size(1);
  const float* p = cf(logits);
  int* pi = ids.data_ptr<int>();
  float* pw = mf(wts);
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < T; ++t) {
    std::vector<float> pr(p + t * E, p + t * E + E);
    const float mx = *std::max_element(pr.begin(), pr.end());
    float sum = 0.f;
    for (auto& v : pr) sum += (v = std::exp(v - mx));
    std::vector<int> idx(E);
    std::iota(idx.begin(), idx.end(), 0);
    std::partial_sort(idx.begin(), idx.begin() + k, idx.end(),
                      [&](int a, int b) { return pr[a] > pr[b] || (pr[a] == pr[b] && a < b); });
    float ps = 0.f;
    for (int64_t j = 0; j < k; ++j) ps += pr[idx[j]] / sum;
    for (int64_t j = 0; j < k; ++j) {
      pi[t * k + j] = idx[j];
      pw[t * k + j] = renorm ? (pr[idx[j]] / sum) / ps : pr[idx[j]] / sum;
    }
  }
}

// out[T,H] += sum over local experts [e_lo, e_lo+num_local) of the routed rows
void moe_experts(const at::Tensor& x, const at::Tensor& ids, const at::Tensor& wts, const at::Tensor& w13,
                 const at::Tensor& w2, int64_t e_lo, int64_t num_local, at::Tensor& out) {
  const int64_t T = x.size(0), H = x.size(1), K = ids.size(1), I = w2.size(1);
  const int* pi = ids.data_ptr<int>();
  const float* pw = cf(wts);
  std::vector<std::vector<std::pair<int64_t, float>>> rows(num_local);
  for (int64_t t = 0; t < T; ++t)
    for (int64_t j = 0; j < K; ++j) {
      const int64_t e = pi[t * K + j] - e_lo;
      if (e >= 0 && e < num_local) rows[e].emplace_back(t, pw[t * K + j]);
    }
  auto xc = x.contiguous();
  float* po = mf(out);
  for (int64_t e = 0; e < num_local; ++e) {
    if (rows[e].empty()) continue;
    const int64_t n = rows[e].size();
    auto xe = at::empty({n, H}, at::kFloat);
    for (int64_t i = 0; i < n; ++i) xe[i].copy_(xc[rows[e][i].first]);
    auto gu = at::empty({n, 2 * I}, at::kFloat);
    linear(xe, w13.narrow(0, e * 2 * I, 2 * I).contiguous(), gu);
    auto h = at::empty({n, I}, at::kFloat);
    swiglu(gu, h);
    auto ye = at::empty({n, H}, at::kFloat);
    linear(h, w2.narrow(0, e * H, H).contiguous(), ye);
    const float* py = cf(ye);
    for (int64_t i = 0; i < n; ++i) {
      const int64_t t = rows[e][i].first;
      const float wv = rows[e][i].second;
      for (int64_t d = 0; d < H; ++d) po[t * H + d] += wv * py[i * H + d];
    }
  }
}

// Gated delta rule, sequential in time, parallel over (batch, head).
// q,k [B,T,Hv,dk], v [B,T,Hv,dv], g,beta [B,T,Hv], state [B,Hv,dk,dv], out [B,T,Hv,dv]
void deltanet_recurrence(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& g,
                         const at::Tensor& beta, at::Tensor& state, at::Tensor& out) {
  const int64_t B = q.size(0), T = q.size(1), Hv = q.size(2), dk = q.size(3), dv = v.size(3);
  const float *pq = cf(q), *pk = cf(k), *pv = cf(v), *pg = cf(g), *pb = cf(beta);
  float *ps = mf(state), *po = mf(out);
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t b = 0; b < B; ++b)
    for (int64_t h = 0; h < Hv; ++h) {
      float* S = ps + ((b * Hv + h) * dk) * dv;
      std::vector<float> kv(dv);
      for (int64_t t = 0; t < T; ++t) {
        const int64_t r = (b * T + t) * Hv + h;
        const float* qt = pq + r * dk;
        const float* kt = pk + r * dk;
        const float* vt = pv + r * dv;
        const float decay = std::exp(pg[r]), bt = pb[r];
        std::fill(kv.begin(), kv.end(), 0.f);
        for (int64_t i = 0; i < dk; ++i) {
          float* Si = S + i * dv;
          for (int64_t j = 0; j < dv; ++j) {
            Si[j] *= decay;
            kv[j] += Si[j] * kt[i];
          }
        }
        for (int64_t j = 0; j < dv; ++j) kv[j] = (vt[j] - kv[j]) * bt;  // delta
        float* ot = po + r * dv;
        std::fill(ot, ot + dv, 0.f);
        for (int64_t i = 0; i < dk; ++i) {
          float* Si = S + i * dv;
          for (int64_t j = 0; j < dv; ++j) {
            Si[j] += kt[i] * kv[j];
            ot[j] += Si[j] * qt[i];
          }
        }
      }
    }
}

// Depthwise causal conv over time with a carried state of the last K-1 inputs.
// x [T, C], w [C, K], state [C, K-1] (updated), out [T, C] (before activation)
void conv1d_causal(const at::Tensor& x, const at::Tensor& w, at::Tensor& state, at::Tensor& out) {
  const int64_t T = x.size(0), C = x.size(1), K = w.size(1);
  const float *px = cf(x), *pw = cf(w);
  float *ps = mf(state), *po = mf(out);
#pragma omp parallel for schedule(static)
  for (int64_t c = 0; c < C; ++c) {
    std::vector<float> hist(ps + c * (K - 1), ps + c * (K - 1) + K - 1);
    for (int64_t t = 0; t < T; ++t) {
      float acc = pw[c * K + K - 1] * px[t * C + c];
      for (int64_t j = 0; j < K - 1; ++j) acc += pw[c * K + j] * hist[j];
      po[t * C + c] = acc;
      for (int64_t j = 0; j + 1 < K - 1; ++j) hist[j] = hist[j + 1];
      if (K > 1) hist[K - 2] = px[t * C + c];
    }
    std::copy(hist.begin(), hist.end(), ps + c * (K - 1));
  }
}

// Bilinear resize of a [C, H, W] image (half-pixel centres, edge clamp).
void resize_bilinear(const at::Tensor& img, at::Tensor& out) {
  const int64_t C = img.size(0), H = img.size(1), W = img.size(2), OH = out.size(1), OW = out.size(2);
  const float* pi = cf(img);
  float* po = mf(out);
  const float sy = (float)H / OH, sx = (float)W / OW;
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t c = 0; c < C; ++c)
    for (int64_t y = 0; y < OH; ++y) {
      const float fy = std::max(0.f, (y + 0.5f) * sy - 0.5f);
      const int64_t y0 = std::min<int64_t>((int64_t)fy, H - 1), y1 = std::min<int64_t>(y0 + 1, H - 1);
      const float wy = fy - y0;
      for (int64_t x = 0; x < OW; ++x) {
        const float fx = std::max(0.f, (x + 0.5f) * sx - 0.5f);
        const int64_t x0 = std::min<int64_t>((int64_t)fx, W - 1), x1 = std::min<int64_t>(x0 + 1, W - 1);
        const float wx = fx - x0;
        const float* p = pi + c * H * W;
        po[(c * OH + y) * OW + x] = (1 - wy) * ((1 - wx) * p[y0 * W + x0] + wx * p[y0 * W + x1]) +
                                    wy * ((1 - wx) * p[y1 * W + x0] + wx * p[y1 * W + x1]);
      }
    }
}

}  // namespace mbcpu
