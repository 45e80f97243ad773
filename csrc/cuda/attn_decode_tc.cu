// Paged decode attention on 5th-generation tensor cores (tcgen05 + TMEM).
//
// Persistent CTAs of 4 warps loop over (sequence, KV head, chunk) items; a
// chunk is ceil(max_blocks / splits) paged blocks.  The G query heads that
// share a KV head form the N = 16 side of both products (rows >= G are zero),
// so every K/V byte is read once per sequence.  Per 128-token tile:
//   1. one thread issues TMA loads of 8 paged 16-token blocks:
//        K block  [16 tok x 128 d]  -> two 128-byte-swizzled halves (d 0-63, 64-127)
//        V block  [128 d x 16 tok]  -> one 32-byte-swizzled [128 x 32 B] tile
//      (V is stored transposed inside a block, so it is K-major for P.V);
//   2. S^T[tok, h] = K . Q^T        8 MMAs, M=128 (tokens), N=16, K=16 (d)
//   3. thread t (= TMEM lane t = token t) reads its scores, the CTA reduces
//      per-head max and sum (online softmax, base 2), writes P[h, t] bf16 to
//      shared memory in the 32-byte-swizzled K-major layout;
//   4. O^T[d, h] = V^T . P^T        8 MMAs, M=128 (head dim), N=16, K=16: one
//      MMA per paged block;
//   5. thread d (= TMEM lane d) folds the tile into its fp32 accumulators with
//      the running-max correction.
// Shared memory is 74 KB, so three CTAs share an SM and overlap each other's
// loads and softmax.  Every wait is bounded (2 s); a timeout sets the status
// word and the CTA leaves the tile loop.
//
// Replaces fused_attention / paged_attention of the reference
// (pio/plugins/cuda/c_src/tensor_ops_cuda.cu:529-618,
//  pio/plugins/common/c_src/tensor_ops_opencl.c:526-565).
#include <cuda.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "attn_decode.cuh"
#include "common.cuh"
#include "launch.cuh"
#include "status.h"

namespace mb {

CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dt, int64_t rows, int64_t cols, int64_t ld_bytes,
                         int box_cols, int box_rows, CUtensorMapSwizzle sw);

namespace {

constexpr int kBS = 16;
// Head dim D = 128 or 256: K / Q are D/64 swizzle-width chunks; a V block is [D rows x 32 B];
// O^T (M = D) is D/128 MMAs of M = 128, each with its own 16 TMEM columns.
template <int D>
struct DecCfg {
  static constexpr int kChunks = D / 64;
  static constexpr int kKBytes = kChunks * 16384;   // chunks x [128 rows x 128 B]
  static constexpr int kVBlock = D * 32;
  static constexpr int kVBytes = 8 * kVBlock;        // eight blocks x [D rows x 32 B]
  static constexpr int kQBytes = kChunks * 2048;     // chunks x [16 rows x 128 B]
  static constexpr int kPBytes = 8 * 512;            // eight blocks x [16 rows x 32 B]
  static constexpr int kHalves = D / 128;
  static constexpr int kTmemCols = D > 128 ? 64 : 32;
  // One Q buffer: the next item's Q is written only after the last S MMA that reads the
  // current one has completed.  D = 128: 75,776 B per CTA, three CTAs per SM.
  static constexpr int kSmemBytes = 1024 + kKBytes + kVBytes + kQBytes + kPBytes + 1024;
};

// SW32 K-major descriptor: 8-row core groups of 32-byte rows (SBO = 256 B).
__device__ __forceinline__ uint64_t make_sdesc_k32(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFF) >> 4);
  d |= (uint64_t)1 << 16;               // LBO (unused: K of one MMA = one atom)
  d |= (uint64_t)(256 >> 4) << 32;      // SBO = 256 B
  d |= (uint64_t)1 << 46;               // version
  d |= (uint64_t)6 << 61;               // SWIZZLE_32B
  return d;
}

__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

struct TileRef {
  int b, hk, sp, t0, tok_hi, nblk, first, last;
};

// Walks this CTA's (item, tile) sequence: items blockIdx.x, +gridDim.x, ...
// Items whose chunk is empty get their (zero / -inf) output written here and
// are skipped.  Every thread runs the same walk.
template <int G, int D>
struct TileCursor {
  int item, t, nt;
  int B, Hkv, splits, chunk_blocks, items;
  const int* ctx_lens;
  int max_blocks;
  int* work;            // [2] device: next item ticket, finished CTAs (zero between launches)
  int* ticket;          // shared-memory slot that thread 0 publishes each ticket in
  int b, hk, sp, lo, hi, nblk;  // current item
  // Items are handed out one at a time from a device counter (longest-first
  // order: every sequence's first chunk, then every second chunk, ...), so a
  // CTA that finishes early takes more work instead of the grid waiting on the
  // CTAs that drew two long items.  All threads of the CTA call next() at the
  // same points, so the barriers inside are reached by every thread.
  // work == nullptr: static round-robin (item = blockIdx.x, + gridDim.x, ...).
  __device__ int fetch() {
    if (!work) return item < 0 ? (int)blockIdx.x : item + (int)gridDim.x;
    __syncthreads();
    if (threadIdx.x == 0) *ticket = atomicAdd(work, 1);
    __syncthreads();
    return *ticket;
  }
  __device__ bool next(TileRef& r, __nv_bfloat16* out, float* part_o, float* part_lse) {
    while (t + 1 >= nt) {
      item = fetch();
      if (item >= items) return false;
      const int bh = item % (B * Hkv);
      sp = item / (B * Hkv);
      hk = bh % Hkv;
      b = bh / Hkv;
      const int ctx = min(ctx_lens[b], max_blocks * 16);  // never past the block-table row
      nblk = (ctx + 15) / 16;
      const int blo = min(nblk, sp * chunk_blocks), bhi = min(nblk, blo + chunk_blocks);
      lo = blo * 16;
      hi = min(ctx, bhi * 16);
      nt = hi > lo ? (hi - lo + 127) / 128 : 0;
      t = -1;
      if (nt == 0) {  // empty chunk: write its output now and move on
        for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
          const int h = i / D, d = i % D;
          const size_t bh2 = (size_t)b * Hkv * G + hk * G + h;
          if (splits == 1) {
            out[bh2 * D + d] = __float2bfloat16(0.f);
          } else {
            part_o[(bh2 * splits + sp) * D + d] = 0.f;
            if (d == 0) part_lse[bh2 * splits + sp] = -INFINITY;
          }
        }
      }
    }
    ++t;
    r.b = b; r.hk = hk; r.sp = sp; r.nblk = nblk; r.tok_hi = hi;
    r.t0 = lo + t * 128;
    r.first = t == 0;
    r.last = t + 1 >= nt;
    return true;
  }
};

template <int G, int D>
__global__ void __launch_bounds__(128, 1)
    attn_decode_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                          const __nv_bfloat16* __restrict__ q, const int* __restrict__ block_tables,
                          const int* __restrict__ ctx_lens, __nv_bfloat16* __restrict__ out,
                          float* __restrict__ part_o, float* __restrict__ part_lse, int B, int Hkv, int max_blocks,
                          int splits, int chunk_blocks, float scale_log2, int* status, int* work) {
  using CF = DecCfg<D>;
  constexpr int kKBytes = CF::kKBytes, kVBytes = CF::kVBytes, kQBytes = CF::kQBytes, kPBytes = CF::kPBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = sm;
  uint8_t* sV = sK + kKBytes;
  uint8_t* sQ = sV + kVBytes;
  uint8_t* sP = sQ + kQBytes;
  float* red_max = reinterpret_cast<float*>(sP + kPBytes);   // [4][16]
  float* red_sum = red_max + 64;                              // [4][16]
  uint64_t* bars = reinterpret_cast<uint64_t*>(red_sum + 64); // K, V, S, O
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  int* ticket = abort_flag + 1;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int Hq = Hkv * G;
  const int items = B * Hkv * splits;

  if (tid == 0) {
    for (int i = 0; i < 4; ++i) mbar_init(&bars[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, CF::kTmemCols);
    tmem_relinquish();
  }
  if (tid == 0) {
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  // K/V tiles start zeroed (blocks past a sequence's end are never loaded and
  // must hold finite data); P rows >= G stay zero.
  for (int i = tid; i < (kKBytes + kVBytes + kQBytes + kPBytes) / 16; i += 128)
    reinterpret_cast<uint4*>(sK)[i] = make_uint4(0, 0, 0, 0);
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + 16;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  constexpr uint32_t idesc = make_idesc_bf16(128, 16);
  // everything below reads the cache, q and lengths written by earlier kernels
  pdl_wait();
  pdl_trigger();

  // tile descriptors: cur (being computed) and nxt (being loaded)
  TileCursor<G, D> cursor{-1, 0, 0, B, Hkv, splits, chunk_blocks, items, ctx_lens, max_blocks, work, ticket};
  TileRef cur, nxt;
  bool has_cur = cursor.next(cur, out, part_o, part_lse);
  bool has_nxt = false;
  auto advance = [&]() { has_nxt = cursor.next(nxt, out, part_o, part_lse); };
  if (has_cur) advance();

  auto issue_k = [&](const TileRef& r) {  // warp 0
    const int* bt = block_tables + (size_t)r.b * max_blocks;
    const int nv = max(0, min(8, r.nblk - r.t0 / 16));
    if (lane == 0) mbar_arrive_expect_tx(&bars[0], nv * D * 32);
    __syncwarp();
    if (lane < nv) {
      const int krow = (bt[r.t0 / 16 + lane] * Hkv + r.hk) * kBS;
#pragma unroll
      for (int c = 0; c < CF::kChunks; ++c) tma_load_2d(sK + c * 16384 + lane * 2048, &tmK, &bars[0], c * 64, krow);
    }
  };
  auto issue_v = [&](const TileRef& r) {  // warp 0
    const int* bt = block_tables + (size_t)r.b * max_blocks;
    const int nv = max(0, min(8, r.nblk - r.t0 / 16));
    if (lane == 0) mbar_arrive_expect_tx(&bars[1], nv * CF::kVBlock);
    __syncwarp();
    if (lane < nv)
      tma_load_2d(sV + lane * CF::kVBlock, &tmV, &bars[1], 0, (bt[r.t0 / 16 + lane] * Hkv + r.hk) * D);
  };
  auto load_q = [&](const TileRef& r) {  // all threads
    uint8_t* dst = sQ;
    for (int i = tid; i < G * D; i += 128) {
      const int h = i / D, d = i % D;
      uint32_t byte = h * 128 + (d % 64) * 2;
      byte ^= ((byte >> 7) & 7) << 4;
      *reinterpret_cast<__nv_bfloat16*>(dst + (d / 64) * 2048 + byte) = q[((size_t)r.b * Hq + r.hk * G + h) * D + d];
    }
  };

  if (has_cur) {
    if (warp == 0) {
      issue_k(cur);
      issue_v(cur);
    }
    load_q(cur);
    fence_async_smem();
    __syncthreads();
  }
  float m[G], l[G], acc[CF::kHalves][G];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.f;
#pragma unroll
    for (int hf = 0; hf < CF::kHalves; ++hf) acc[hf][h] = 0.f;
  }
  uint32_t it = 0;
  while (has_cur) {
    const uint32_t par = it & 1;
    // ---- S^T = K . Q^T
    bool ok = mbar_wait(&bars[0], par, status);
    tc_fence_after();
    if (tid == 32 && ok) {
      const uint32_t qb = smem_u32(sQ);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
        const uint32_t qoff = (kk >> 2) * 2048 + (kk & 3) * 32;
        tc_mma_bf16(tS, make_sdesc_k128(smem_u32(sK) + off), make_sdesc_k128(qb + qoff), idesc, kk > 0);
      }
      tc_commit(&bars[2]);
    }
    ok = mbar_wait(&bars[2], par, status) && ok;
    tc_fence_after();
    // K buffer is free: prefetch the next tile's K while this tile finishes
    if (warp == 0 && has_nxt && ok) issue_k(nxt);
    // ---- softmax: thread tid owns token cur.t0 + tid
    float s[16];
    tmem_ld16(tS + lane_off, s);
    const bool valid = cur.t0 + tid < cur.tok_hi;
    float p[G];
#pragma unroll
    for (int h = 0; h < G; ++h) {
      s[h] = valid ? s[h] * scale_log2 : -INFINITY;
      const float mx = warp_max(s[h]);
      if (lane == 0) red_max[warp * 16 + h] = mx;
    }
    __syncthreads();
    float corr[G];
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const float mt = fmaxf(fmaxf(red_max[h], red_max[16 + h]), fmaxf(red_max[32 + h], red_max[48 + h]));
      const float mn = fmaxf(m[h], mt);
      corr[h] = mn == -INFINITY ? 1.f : exp2f(m[h] - mn);
      p[h] = (mn == -INFINITY || s[h] == -INFINITY) ? 0.f : exp2f(s[h] - mn);
      m[h] = mn;
      const float ps = warp_sum(p[h]);
      if (lane == 0) red_sum[warp * 16 + h] = ps;
    }
    uint8_t* chunk = sP + (tid >> 4) * 512;
#pragma unroll
    for (int h = 0; h < G; ++h) {
      uint32_t byte = h * 32 + (tid & 15) * 2;
      byte ^= ((byte >> 7) & 1) << 4;
      *reinterpret_cast<__nv_bfloat16*>(chunk + byte) = __float2bfloat16(p[h]);
    }
    // next item's Q: every thread has waited on this tile's S MMA (bars[2]), the last reader of Q
    if (has_nxt && nxt.first) load_q(nxt);
    fence_async_smem();
    tc_fence_before();
    if (!ok) *abort_flag = 1;
    __syncthreads();
    tc_fence_after();
    // ---- O^T = V^T . P^T
    ok = !*abort_flag && mbar_wait(&bars[1], par, status);
    tc_fence_after();
    if (tid == 32 && ok) {
#pragma unroll
      for (int hf = 0; hf < CF::kHalves; ++hf)  // head-dim rows 128*hf.. of every V block
#pragma unroll
        for (int j = 0; j < 8; ++j)
          tc_mma_bf16(tO + hf * 16, make_sdesc_k32(smem_u32(sV) + j * CF::kVBlock + hf * 4096),
                      make_sdesc_k32(smem_u32(sP) + j * 512), idesc, j > 0);
      tc_commit(&bars[3]);
    }
    ok = ok && mbar_wait(&bars[3], par, status);
    tc_fence_after();
    if (warp == 0 && has_nxt && ok) issue_v(nxt);
#pragma unroll
    for (int hf = 0; hf < CF::kHalves; ++hf) {
      float o[16];
      tmem_ld16(tO + hf * 16 + lane_off, o);
#pragma unroll
      for (int h = 0; h < G; ++h) acc[hf][h] = acc[hf][h] * corr[h] + o[h];
    }
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const float lt = red_sum[h] + red_sum[16 + h] + red_sum[32 + h] + red_sum[48 + h];
      l[h] = l[h] * corr[h] + lt;
    }
    if (cur.last) {  // thread tid owns head-dim elements d = tid + 128 * hf
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const size_t bh = (size_t)cur.b * Hq + cur.hk * G + h;
#pragma unroll
        for (int hf = 0; hf < CF::kHalves; ++hf) {
          const int d = tid + 128 * hf;
          const float v = l[h] > 0.f ? acc[hf][h] / l[h] : 0.f;
          if (splits == 1) {
            out[bh * D + d] = __float2bfloat16(v);
          } else {
            part_o[(bh * splits + cur.sp) * D + d] = v;
            if (d == 0) part_lse[bh * splits + cur.sp] = l[h] > 0.f ? m[h] + log2f(l[h]) : -INFINITY;
          }
          acc[hf][h] = 0.f;
        }
        m[h] = -INFINITY;
        l[h] = 0.f;
      }
    }
    tc_fence_before();
    if (!ok) *abort_flag = 1;
    __syncthreads();
    if (*abort_flag) break;
    ++it;
    cur = nxt;
    has_cur = has_nxt;
    if (has_cur) advance();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, CF::kTmemCols);
  }
  // the last CTA to finish resets the work counter for the next launch (no CTA fetches any more)
  if (work && tid == 0 && atomicAdd(work + 1, 1) == (int)gridDim.x - 1) {
    work[0] = 0;
    work[1] = 0;
  }
}

}  // namespace

bool attn_decode_tc_supported(int64_t D, int64_t G) {
  return (D == 128 && (G == 1 || G == 2 || G == 4 || G == 8 || G == 16)) ||
         (D == 256 && (G == 1 || G == 2 || G == 4 || G == 8));
}

// Same contract as attn_decode (attn_decode.cu); head_dim 128 (group <= 16) or 256 (group <= 8).
void attn_decode_tc(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                    const at::Tensor& block_tables, const at::Tensor& ctx_lens, at::Tensor& out, int64_t splits,
                    const c10::optional<at::Tensor>& workspace, double scale, at::Tensor& work) {
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous() && out.is_contiguous());
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous() && k_cache.size(2) == 16 && v_cache.size(3) == 16);
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && ctx_lens.scalar_type() == at::kInt &&
              block_tables.is_contiguous());
  const int B = (int)q.size(0), Hq = (int)q.size(1), D = (int)q.size(2);
  const int Hkv = (int)k_cache.size(1), NB = (int)k_cache.size(0);
  TORCH_CHECK(Hq % Hkv == 0 && k_cache.size(3) == D && v_cache.size(2) == D);
  const int G = Hq / Hkv;
  TORCH_CHECK(attn_decode_tc_supported(D, G), "attn_decode_tc: needs head_dim 128 (group <= 16) or 256 (group <= 8)");
  TORCH_CHECK(work.scalar_type() == at::kInt && work.is_cuda() && (work.numel() == 0 || work.numel() >= 2),
              "attn_decode_tc: work must be empty (static schedule) or a zeroed int32 device tensor of 2 "
              "elements (dynamic schedule; kept zero by the kernel)");
  if (B == 0) return;
  splits = std::max<int64_t>(1, splits);
  float* po = nullptr;
  float* pl = nullptr;
  if (splits > 1) {
    TORCH_CHECK(workspace && workspace->defined() && workspace->scalar_type() == at::kFloat &&
                    workspace->numel() >= (int64_t)B * Hq * splits * (D + 1),
                "attn_decode_tc: split-KV needs an fp32 workspace of B*Hq*splits*(D+1)");
    po = workspace->data_ptr<float>();
    pl = po + (size_t)B * Hq * splits * D;
  }
  c10::cuda::CUDAGuard guard(q.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  auto tk = make_tmap_2d(k_cache.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (int64_t)NB * Hkv * 16, D, D * 2, 64,
                         16, CU_TENSOR_MAP_SWIZZLE_128B);
  auto tv = make_tmap_2d(v_cache.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (int64_t)NB * Hkv * D, 16, 32, 16, D,
                         CU_TENSOR_MAP_SWIZZLE_32B);
  const float sl2 = (float)(scale * 1.4426950408889634);
  // persistent grid: every resident CTA (three per SM at D = 128, one at D = 256)
  static int sms = 0;
  if (!sms) C10_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, q.device().index()));
  const int mbk = (int)block_tables.size(1);
  const int chunk_blocks = (mbk + (int)splits - 1) / (int)splits;
  const int items = B * Hkv * (int)splits;
  static bool attr[2][17] = {{false}};
  auto go = [&](auto kernel, int g, int smem) {
    const int di = D == 256;
    if (!attr[di][g]) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      attr[di][g] = true;
    }
    const int per_sm = std::max(1, std::min(3, (int)(228 * 1024 / (smem + 1024))));
    const int grid = std::min(items, per_sm * sms);
    launch_k(kernel, grid, 128, smem, st, tk, tv, reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()),
             block_tables.data_ptr<int>(), ctx_lens.data_ptr<int>(), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
             po, pl, B, Hkv, mbk, (int)splits, chunk_blocks, sl2, status_ptr(q.device().index()),
             work.numel() ? work.data_ptr<int>() : nullptr);
  };
  constexpr int s128 = DecCfg<128>::kSmemBytes, s256 = DecCfg<256>::kSmemBytes;
  if (D == 128) {
    switch (G) {
      case 1: go(attn_decode_tc_kernel<1, 128>, 1, s128); break;
      case 2: go(attn_decode_tc_kernel<2, 128>, 2, s128); break;
      case 4: go(attn_decode_tc_kernel<4, 128>, 4, s128); break;
      case 8: go(attn_decode_tc_kernel<8, 128>, 8, s128); break;
      default: go(attn_decode_tc_kernel<16, 128>, 16, s128); break;
    }
  } else {
    switch (G) {
      case 1: go(attn_decode_tc_kernel<1, 256>, 1, s256); break;
      case 2: go(attn_decode_tc_kernel<2, 256>, 2, s256); break;
      case 4: go(attn_decode_tc_kernel<4, 256>, 4, s256); break;
      default: go(attn_decode_tc_kernel<8, 256>, 8, s256); break;
    }
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  if (splits > 1) {
    if (D == 128)
      launch_k(attn_combine_kernel<128>, B * Hq, 128, 0, st, po, pl, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
               (int)splits);
    else
      launch_k(attn_combine_kernel<256>, B * Hq, 128, 0, st, po, pl, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
               (int)splits);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

}  // namespace mb
