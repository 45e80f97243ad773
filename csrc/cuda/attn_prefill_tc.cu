// Causal flash-attention prefill over the paged KV cache on tcgen05 tensor cores.
//
// q   [T, Hq*D] bf16 (packed rows of every sequence's new tokens; D = 64, 128 or 256)
// k/v cache as in decode: K [blocks, Hkv, 16, D], V [blocks, Hkv, D, 16]
// out [T, Hq*D] bf16
// Sequence b owns q rows [cu_q[b], cu_q[b+1]) whose absolute positions end
// at ctx_lens[b] - 1 (so prompts with a cached prefix work unchanged).
//
// CTA = one (sequence, query head, 128-row query tile); 5 warps:
//   warp 4      : TMA producer (Q once; K and V tiles of 8 paged blocks into a
//                 2-stage ring, block-table reads spread over 8 lanes)
//   warps 0-3   : thread t owns query row t.  Per 128-key tile:
//                 S = Q.K^T (M=128 queries, N=128 keys, 8 MMAs of K=16 over d,
//                 issued by thread 0, fp32 in TMEM) -> row max / exp2 / row sum
//                 entirely in the thread -> P (bf16) to shared memory ->
//                 O += P.V (M=128, N=128 (d), one K=16 MMA per paged V block).
//                 When a warp's running maxima move, its lanes rescale their O
//                 rows in TMEM (tcgen05.ld, scale, tcgen05.st) after the
//                 previous P.V has completed.
// Key tiles entirely above the causal diagonal are skipped.  Shared memory
// ~197 KB (one CTA per SM), TMEM 256 columns.  Every wait is bounded.
//
// Replaces the reference's S x S score materialisation without a causal mask
// (pio/plugins/cpu/c_src/tensor_ops.c:536-578, pio/core/engine/backend.py:771-790).
#include <cuda.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "launch.cuh"
#include "status.h"

namespace mb {

CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dt, int64_t rows, int64_t cols, int64_t ld_bytes,
                         int box_cols, int box_rows, CUtensorMapSwizzle sw);

namespace {

// Head dims 64 / 128 / 256: Q and K are D/64 swizzle-width chunks of [128 rows x 128 B]; a V
// block is [D x 32 B].  D = 256 fits one K/V stage in shared memory, smaller D two.
template <int D>
struct PrefillCfg {
  static constexpr int kChunks = D / 64;
  static constexpr int kQBytes = kChunks * 16384;
  static constexpr int kKBytes = kChunks * 16384;
  static constexpr int kVBlock = D * 32;
  static constexpr int kVBytes = 8 * kVBlock;
  static constexpr int kPBytes = 2 * 16384;    // two key-halves x [128 rows x 128 B]
  static constexpr int kStages = D > 128 ? 1 : 2;
  static constexpr int kSmem = 1024 + kQBytes + kStages * (kKBytes + kVBytes) + kPBytes + 512;
  static constexpr int kTmemCols = D > 128 ? 512 : 256;   // S (128 columns) + O (D columns)
};

__device__ __forceinline__ uint64_t sdesc_k32(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr & 0x3FFFF) >> 4);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(256 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)6 << 61;
  return d;
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

template <int D>
__global__ void __launch_bounds__(160, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, const int* __restrict__ block_tables,
                           const int* __restrict__ cu_q, const int* __restrict__ ctx_lens, __nv_bfloat16* __restrict__ out,
                           int Hq, int Hkv, int max_blocks, float scale_log2, int* status, int causal) {
  using CF = PrefillCfg<D>;
  constexpr int kQBytes = CF::kQBytes, kKBytes = CF::kKBytes, kVBytes = CF::kVBytes, kPBytes = CF::kPBytes;
  constexpr int kStages = CF::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = sm;
  uint8_t* sK = sQ + kQBytes;                       // [kStages][kKBytes]
  uint8_t* sV = sK + kStages * kKBytes;             // [kStages][kVBytes]
  uint8_t* sP = sV + kStages * kVBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + kPBytes);
  uint64_t* barQ = bars;                            // 1
  uint64_t* fullK = bars + 1;                       // kStages
  uint64_t* fullV = fullK + kStages;
  uint64_t* emptyK = fullV + kStages;
  uint64_t* emptyV = emptyK + kStages;
  uint64_t* barS = emptyV + kStages;
  uint64_t* barO = barS + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(barO + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (Hq / Hkv);

  if (tid == 0) {
    mbar_init(barQ, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&fullK[s], 1);
      mbar_init(&fullV[s], 1);
      mbar_init(&emptyK[s], 1);
      mbar_init(&emptyV[s], 1);
    }
    mbar_init(barS, 1);
    mbar_init(barO, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, CF::kTmemCols);
    tmem_relinquish();
  }
  if (tid == 128) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  pdl_wait();
  pdl_trigger();
  const int q0 = cu_q[b], ql = cu_q[b + 1] - q0;
  const int ctx = ctx_lens[b];
  // A tile past the sequence's last block leaves some block slots unloaded;
  // P is zero there, but 0 * (uninitialised NaN) would still poison O, so the
  // K/V stages start zeroed (later tiles only leave finite stale data).
  if (((ctx + 15) / 16) % 8 != 0) {
    for (int i = tid; i < kStages * (kKBytes + kVBytes) / 16; i += blockDim.x)
      reinterpret_cast<uint4*>(sK)[i] = make_uint4(0, 0, 0, 0);
    fence_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + 128;
  const int qrow0 = qt * 128;                        // first query row of this tile (within the sequence)
  if (qrow0 < ql) {
    const int pos0 = ctx - ql + qrow0;                 // absolute position of query row 0
    const int last_pos = causal ? min(ctx - 1, pos0 + 127) : ctx - 1;
    const int nkt = last_pos / 128 + 1;                // key tiles [0, nkt)
    const int nblk = (ctx + 15) / 16;
    const int* bt = block_tables + (size_t)b * max_blocks;

    if (warp == 4) {
      // ------------------------------------------------ producer
      if (lane == 0) {
        mbar_arrive_expect_tx(barQ, kQBytes);
#pragma unroll
        for (int c = 0; c < CF::kChunks; ++c) tma_load_2d(sQ + c * 16384, &tmQ, barQ, h * D + c * 64, q0 + qrow0);
      }
      for (int j = 0; j < nkt; ++j) {
        const int s = j % kStages;
        const uint32_t ph = (j / kStages) & 1;
        const int nv = max(0, min(8, nblk - j * 8));
        bool ok = true;
        if (lane == 0) ok = mbar_wait(&emptyK[s], ph ^ 1, status);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        if (lane == 0) mbar_arrive_expect_tx(&fullK[s], nv * D * 32);
        __syncwarp();
        int phys = 0;
        if (lane < nv) {
          phys = bt[j * 8 + lane];
          const int krow = (phys * Hkv + hk) * 16;
#pragma unroll
          for (int c = 0; c < CF::kChunks; ++c)
            tma_load_2d(sK + s * kKBytes + c * 16384 + lane * 2048, &tmK, &fullK[s], c * 64, krow);
        }
        if (lane == 0) ok = mbar_wait(&emptyV[s], ph ^ 1, status);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        if (lane == 0) mbar_arrive_expect_tx(&fullV[s], nv * CF::kVBlock);
        __syncwarp();
        if (lane < nv) tma_load_2d(sV + s * kVBytes + lane * CF::kVBlock, &tmV, &fullV[s], 0, (phys * Hkv + hk) * D);
      }
    } else {
      // ------------------------------------------------ softmax / MMA warps
      constexpr uint32_t idesc = make_idesc_bf16(128, 128);      // S = Q K^T: 128 queries x 128 keys
      constexpr uint32_t idesc_o = make_idesc_bf16(128, D);      // O += P V: 128 queries x D
      const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
      const int my_pos = pos0 + tid;                  // absolute position of this thread's query row
      float m = -INFINITY, l = 0.f;
      bool ok = mbar_wait(barQ, 0, status);
      for (int j = 0; j < nkt && ok; ++j) {
        const int s = j % kStages;
        const uint32_t ph = (j / kStages) & 1;
        ok = mbar_wait(&fullK[s], ph, status);
        tc_fence_after();
        if (tid == 0 && ok) {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
            tc_mma_bf16(tS, make_sdesc_k128(smem_u32(sQ) + off), make_sdesc_k128(smem_u32(sK + s * kKBytes) + off),
                        idesc, kk > 0);
          }
          tc_commit(barS);
          tc_commit(&emptyK[s]);
        }
        ok = ok && mbar_wait(barS, j & 1, status);
        // the previous P.V must be complete before P and O are touched
        if (j > 0) ok = ok && mbar_wait(barO, (j - 1) & 1, status);
        tc_fence_after();
        // ---- row softmax (this thread's row, 128 keys)
        float sc[128];
#pragma unroll
        for (int c = 0; c < 8; ++c) tmem_ld16(tS + lane_off + c * 16, sc + c * 16);
        float mt = -INFINITY;
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          const int kpos = j * 128 + c;
          sc[c] = ((!causal || kpos <= my_pos) && kpos < ctx) ? sc[c] * scale_log2 : -INFINITY;
          mt = fmaxf(mt, sc[c]);
        }
        const float mn = fmaxf(m, mt);
        const float corr = (mn == -INFINITY) ? 1.f : exp2f(m - mn);
        float rs = 0.f;
        // P row -> shared, 128-byte swizzle, two key-halves of 64
#pragma unroll
        for (int c = 0; c < 128; c += 8) {
          __align__(16) __nv_bfloat16 pv[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float p = (mn == -INFINITY || sc[c + e] == -INFINITY) ? 0.f : exp2f(sc[c + e] - mn);
            rs += p;
            pv[e] = __float2bfloat16(p);
          }
          uint32_t byte = tid * 128 + ((c % 64) * 2);
          byte ^= ((byte >> 7) & 7) << 4;
          *reinterpret_cast<uint4*>(sP + (c / 64) * 16384 + byte) = *reinterpret_cast<uint4*>(pv);
        }
        l = l * corr + rs;
        m = mn;
        // ---- rescale this warp's O rows when any running max moved
        if (j > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
#pragma unroll 1
          for (int c = 0; c < D; c += 16) {
            float o[16];
            tmem_ld16(tO + lane_off + c, o);
#pragma unroll
            for (int e = 0; e < 16; ++e) o[e] *= corr;
            tmem_st16(tO + lane_off + c, o);
          }
          tmem_wait_st();
        }
        fence_async_smem();
        tc_fence_before();
        if (!ok) *abort_flag = 1;
        asm volatile("bar.sync 1, 128;" ::: "memory");   // the four softmax warps only
        tc_fence_after();
        if (*abort_flag) { ok = false; break; }
        ok = mbar_wait(&fullV[s], ph, status);
        tc_fence_after();
        if (tid == 0 && ok) {
#pragma unroll
          for (int kb = 0; kb < 8; ++kb) {
            const uint32_t poff = (kb >> 2) * 16384 + (kb & 3) * 32;
            tc_mma_bf16(tO, make_sdesc_k128(smem_u32(sP) + poff),
                        sdesc_k32(smem_u32(sV + s * kVBytes) + kb * CF::kVBlock), idesc_o, (j > 0 || kb > 0));
          }
          tc_commit(barO);
          tc_commit(&emptyV[s]);
        }
      }
      // ---- epilogue: O / l -> out row
      if (ok && nkt > 0) ok = mbar_wait(barO, (nkt - 1) & 1, status);
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* dst = out + ((size_t)(q0 + qrow0 + tid) * Hq + h) * D;
      const bool store = ok && qrow0 + tid < ql;
#pragma unroll 1
      for (int c = 0; c < D; c += 16) {
        float o[16];
        tmem_ld16(tO + lane_off + c, o);
        if (store) {
          __align__(16) __nv_bfloat16 ob[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) ob[e] = __float2bfloat16(o[e] * inv);
          reinterpret_cast<uint4*>(dst + c)[0] = reinterpret_cast<uint4*>(ob)[0];
          reinterpret_cast<uint4*>(dst + c)[1] = reinterpret_cast<uint4*>(ob)[1];
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, CF::kTmemCols);
  }
}

}  // namespace

template <int D>
static void launch_prefill(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                           const at::Tensor& block_tables, const at::Tensor& cu_q, const at::Tensor& ctx_lens,
                           at::Tensor& out, int64_t max_q_len, double scale, bool causal) {
  using CF = PrefillCfg<D>;
  const int T = (int)q.size(0), Hkv = (int)k_cache.size(1), NB = (int)k_cache.size(0);
  const int Hq = (int)(q.size(1) / D);
  TORCH_CHECK(Hq * D == q.size(1) && Hq % Hkv == 0 && out.sizes() == q.sizes());
  const int B = (int)ctx_lens.numel();
  if (T == 0 || B == 0) return;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  auto tq = make_tmap_2d(q.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, T, (int64_t)Hq * D, (int64_t)Hq * D * 2, 64,
                         128, CU_TENSOR_MAP_SWIZZLE_128B);
  auto tk = make_tmap_2d(k_cache.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (int64_t)NB * Hkv * 16, D, D * 2, 64,
                         16, CU_TENSOR_MAP_SWIZZLE_128B);
  auto tv = make_tmap_2d(v_cache.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (int64_t)NB * Hkv * D, 16, 32, 16, D,
                         CU_TENSOR_MAP_SWIZZLE_32B);
  auto kern = attn_prefill_tc_kernel<D>;
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, CF::kSmem));
    attr = true;
  }
  const int qtiles = (int)((max_q_len + 127) / 128);
  launch_k(kern, dim3(qtiles, Hq, B), 160, CF::kSmem, st, tq, tk, tv, block_tables.data_ptr<int>(),
           cu_q.data_ptr<int>(), ctx_lens.data_ptr<int>(), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), Hq, Hkv,
           (int)block_tables.size(1), (float)(scale * 1.4426950408889634), status_ptr(q.device().index()),
           (int)causal);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// q [T, Hq*D] (contiguous rows), cu_q [B+1], ctx_lens [B], block_tables [B, max_blocks]; D in {64, 128, 256}.
// causal = false: every query row of sequence b sees all ctx_lens[b] keys (bidirectional, e.g. a ViT).
void attn_prefill_tc(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                     const at::Tensor& block_tables, const at::Tensor& cu_q, const at::Tensor& ctx_lens,
                     at::Tensor& out, int64_t max_q_len, double scale, bool causal) {
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous() && out.is_contiguous() && q.dim() == 2);
  const int64_t D = k_cache.size(3);
  TORCH_CHECK(v_cache.size(2) == D && k_cache.size(2) == 16 && v_cache.size(3) == 16);
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && cu_q.scalar_type() == at::kInt && ctx_lens.scalar_type() == at::kInt);
  c10::cuda::CUDAGuard guard(q.device());
  if (D == 128) launch_prefill<128>(q, k_cache, v_cache, block_tables, cu_q, ctx_lens, out, max_q_len, scale, causal);
  else if (D == 256) launch_prefill<256>(q, k_cache, v_cache, block_tables, cu_q, ctx_lens, out, max_q_len, scale, causal);
  else if (D == 64) launch_prefill<64>(q, k_cache, v_cache, block_tables, cu_q, ctx_lens, out, max_q_len, scale, causal);
  else TORCH_CHECK(false, "attn_prefill_tc: head_dim must be 64, 128 or 256");
}

}  // namespace mb
