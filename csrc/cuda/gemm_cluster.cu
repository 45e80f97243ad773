// Decode-shape dense GEMM: split-K across a thread-block cluster, partials
// reduced through distributed shared memory (DSMEM).
//
//   y[T, N] = x[T, K] @ w[N, K]^T        (T <= 128 tokens, N % 128 == 0)
//
// At decode the weight matrix is the only large operand, so the kernel is
// bound by how many SMs stream it and how little else they move.  One cluster
// of CS CTAs owns a 128-row slice of w (one "m tile"); CTA r of the cluster
// multiplies the K range [r*K/CS, (r+1)*K/CS) on the tensor cores (tcgen05,
// accumulator [128 features x BN tokens] in TMEM, swap-AB: the weights are the
// 128-row A operand, the tokens the N side).  The CS partial tiles are then
// summed without leaving the cluster: every CTA parks its tile in its own
// shared memory, a cluster barrier publishes them, and CTA r reads rows of
// all CS tiles through DSMEM for its share of the tokens.  No fp32 workspace
// in global memory and no second kernel, unlike a classic split-K.  Grids are
// m_tiles x CS CTAs, sized so that every SM streams weights (two CTAs per SM).
//
// Epilogues, applied by the CTA that finishes a token's 128 features:
//   kStore     y = bf16(acc) (+ residual)
//   kQkvRope   the tile is one attention head: q heads get RMSNorm * q_w and
//              rotate-half RoPE and go to q_out [T, Hq, 128]; k heads the same
//              with k_w, written into the paged K cache; v heads are written
//              into the paged V cache ([blocks, Hkv, D, 16]).  This replaces
//              the QKV GEMM + split-K reduction + RoPE/QK-norm kernels of a
//              decode step (three launches) with one.
//
// Warp roles (192 threads): warp 0 TMA producer, warp 1 MMA issuer, warps 2-5
// epilogue (TMEM lanes 0-127 = the tile's 128 features).  All waits are
// bounded; every thread of every CTA reaches both cluster barriers on every
// path, so an error never leaves a cluster waiting.
//
// Reference: the projections of the reference are linear_kernel_naive, one
// thread per output (pio/plugins/cuda/c_src/tensor_ops_cuda.cu:318-329).
#include <cuda.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "gemm_tc.cuh"  // i8x4_to_bf16x4
#include "launch.cuh"
#include "status.h"

namespace mb {

CUtensorMap make_tmap_bf16(const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows);
CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dt, int64_t rows, int64_t cols, int64_t ld_bytes,
                         int box_cols, int box_rows, CUtensorMapSwizzle sw);

namespace {

enum ClusterEpi : int { kCStore = 0, kCQkvRope = 1, kCSwiGLU = 2 };

struct ClusterArgs {
  int K, N, T;            // reduction length, output features, tokens
  int kb_per;             // 64-wide K blocks per CTA
  int mode;
  __nv_bfloat16* out;     // kCStore: [T, ldc]
  int ldc;
  const __nv_bfloat16* residual;  // kCStore, optional, same layout as out
  // kCQkvRope
  const __nv_bfloat16* q_w;
  const __nv_bfloat16* k_w;
  const int* pos;
  const float* inv_freq;
  const int* slots;
  __nv_bfloat16* q_out;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  int Hq, Hkv, rot_dim, block_size;
  float eps;
  int* status;
  const float* w_scale;   // int8 weights: per-row (output feature) scale, applied after the reduction
  // tensor parallelism: x is the gathered buffer that the shard owners push into; the producer
  // waits (bounded) until ag_flags[p] >= *ag_epoch for every rank p before it loads x
  const uint32_t* ag_flags;
  const uint32_t* ag_epoch;
  int ag_nranks;
  // kCSwiGLU: w = [gate; up] ([2I, K]); m tile i holds gate rows [64i, 64i+64) in its first 64 rows and
  // up rows [up_row0 + 64i, ...) in its last 64 (two TMA boxes of 64 rows), and produces outputs [64i, 64i+64)
  int up_row0;
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory location in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t map_rank(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_dsmem(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}

// Stage: A tile [128 x 64] bf16 SW128 | B tile [BN x 64] bf16 SW128 | (int8 weights) the raw
// int8 A tile [128 x 64] that the epilogue warps expand into the A slot.
template <int BN, int STAGES, bool W8>
struct CSmem {
  static constexpr int kABytes = 128 * 64 * 2;
  static constexpr int kBBytes = BN * 64 * 2;
  static constexpr int kRawBytes = W8 ? 128 * 64 : 0;
  static constexpr int kRawOff = kABytes + kBBytes;
  static constexpr int kStage = kABytes + kBBytes + kRawBytes;
  static constexpr int kTx = (W8 ? kRawBytes : kABytes) + kBBytes;   // bytes the TMA delivers per stage
  static constexpr int kPartial = BN * 128 * 4;   // fp32 tile parked for the cluster reduction
  static constexpr int kRing = STAGES * kStage > kPartial ? STAGES * kStage : kPartial;
  static constexpr int kBytes = 1024 + kRing + 2048;
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
};

template <int BN, int STAGES, bool W8>
__global__ void __launch_bounds__(192, 1)
    gemm_cluster_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        ClusterArgs args) {
  using L = CSmem<BN, STAGES, W8>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tail = smem + L::kRing;
  uint64_t* full = reinterpret_cast<uint64_t*>(tail);
  uint64_t* empty = full + STAGES;
  uint64_t* cfull = empty + STAGES;   // int8: the stage's A tile has been expanded (4 warp arrivals)
  uint64_t* tfull = cfull + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull + 1);
  float* red = reinterpret_cast<float*>(tmem_slot + 4);     // [4 warps] cross-warp sums
  float* rot = red + 8;                                      // [128] one head vector for RoPE
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  int csize;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(csize));
  const int m_tile = blockIdx.x / csize;
  const int kb_lo = (int)crank * args.kb_per;
  const int kb_total = (args.K + 63) / 64;
  const int kbs = max(0, min(kb_total, kb_lo + args.kb_per) - kb_lo);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&cfull[s], 4);
    }
    mbar_init(tfull, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    if (elect_one_sync()) {
      // weight tiles of the first stages go out before the dependency wait (weights are immutable)
      const int pre = min(STAGES, kbs);
      // the weight (A) tile of K block kb: one 128-row box, or (SwiGLU) 64 gate rows + the matching 64 up rows
      auto load_a = [&](uint8_t* dst, uint64_t* bar, int kb) {
        if (args.mode == kCSwiGLU) {
          tma_load_2d(dst, &tmA, bar, kb * 64, m_tile * 64);
          tma_load_2d(dst + (W8 ? 64 * 64 : 64 * 128), &tmA, bar, kb * 64, args.up_row0 + m_tile * 64);
        } else {
          tma_load_2d(dst, &tmA, bar, kb * 64, m_tile * 128);
        }
      };
      for (int s = 0; s < pre; ++s) {
        mbar_arrive_expect_tx(&full[s], L::kTx);
        load_a(smem + s * L::kStage + (W8 ? L::kRawOff : 0), &full[s], kb_lo + s);
      }
      pdl_wait();
      pdl_trigger();
      if (args.ag_flags) {  // every rank's shard of this boundary is in the gathered buffer
        const uint32_t want = *args.ag_epoch;
        for (int p = 0; p < args.ag_nranks; ++p) {
          const uint64_t t0 = globaltimer_ns();
          while (true) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(args.ag_flags + p) : "memory");
            if ((int32_t)(v - want) >= 0) break;
            // half the limit: the other warps' bounded mbarrier waits started with this one, so the
            // flag timeout is recorded first and the pipeline then drains normally
            if (globaltimer_ns() - t0 > kWaitLimitNs / 2) {
              set_status(args.status, kErrPeerTimeout);
              break;
            }
          }
        }
        // the peers' stores were observed through the generic proxy; the activation tiles are read by TMA
        asm volatile("fence.proxy.async.global;" ::: "memory");
      }
      for (int it = 0; it < kbs && ok; ++it) {
        const int s = it % STAGES;
        uint8_t* st = smem + s * L::kStage;
        if (it >= pre) {
          if (!mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1, args.status)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[s], L::kTx);
          load_a(st + (W8 ? L::kRawOff : 0), &full[s], kb_lo + it);
        }
        tma_load_2d(st + L::kABytes, &tmB, &full[s], (kb_lo + it) * 64, 0);
      }
    } else {
      pdl_wait();
      pdl_trigger();
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    pdl_wait();
    pdl_trigger();
    constexpr uint32_t idesc = make_idesc_bf16(128, BN);
    if (elect_one_sync()) {
      for (int it = 0; it < kbs && ok; ++it) {
        const int s = it % STAGES;
        if (!mbar_wait(&full[s], (it / STAGES) & 1, args.status)) { ok = false; break; }
        if (W8 && !mbar_wait(&cfull[s], (it / STAGES) & 1, args.status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem + s * L::kStage);
        const uint32_t b_addr = a_addr + L::kABytes;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma_bf16(tmem, make_sdesc_k128(a_addr + kk * 32), make_sdesc_k128(b_addr + kk * 32), idesc,
                      (it | kk) != 0);
        tc_commit(&empty[s]);
      }
      tc_commit(tfull);  // arrives once every MMA above has finished (also with kbs == 0)
    }
  } else {
    pdl_wait();
    pdl_trigger();
    if (W8) {
      // ------------------------------------------------ int8 -> bf16 expansion (epilogue warps)
      // thread c expands 16-byte chunks idx = c + 128 m of the [128 x 64] tile: row r = idx / 8,
      // chunk k = idx % 8 -> SW128 position r*128 + (k ^ (r % 8))*16
      const int c = threadIdx.x - 64;
      for (int it = 0; it < kbs; ++it) {
        const int s = it % STAGES;
        if (!mbar_wait(&full[s], (it / STAGES) & 1, args.status)) break;
        uint8_t* st = smem + s * L::kStage;
        const uint8_t* raw = st + L::kRawOff;
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const int idx = c + 128 * m, r = idx >> 3, k = idx & 7;
          const uint2 w = *reinterpret_cast<const uint2*>(raw + r * 64 + k * 8);
          uint4 o;
          i8x4_to_bf16x4(w.x, o.x, o.y);
          i8x4_to_bf16x4(w.y, o.z, o.w);
          *reinterpret_cast<uint4*>(st + r * 128 + ((k ^ (r & 7)) << 4)) = o;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor-core reads
        __syncwarp();
        if (lane == 0) mbar_arrive(&cfull[s]);
      }
    }
  }

  // ------------------------------------------------ park the partial tile in shared memory
  // P[j][i] (token j, feature i) in this CTA's ring, which every MMA has finished reading.
  float* P = reinterpret_cast<float*>(smem);
  if (warp >= 2) {
    const bool have = mbar_wait(tfull, 0, args.status);
    tc_fence_after();
    const uint32_t taddr = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const int lane_feat = (warp & 3) * 32 + lane;  // TMEM lane of this thread
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 16) {
      float v[16];
      tmem_ld16(taddr + c0, v);
#pragma unroll
      for (int q = 0; q < 16; ++q) P[(c0 + q) * 128 + lane_feat] = (have && kbs > 0) ? v[q] : 0.f;
    }
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync_all();  // every CTA's partial is in place

  // ------------------------------------------------ reduce this CTA's share of the tokens, epilogue
  if (warp >= 2) {
    const int f = (warp & 3) * 32 + lane;          // feature within the tile
    const int per = (BN + csize - 1) / csize;
    const int j0 = (int)crank * per, j1 = min(min(BN, args.T), j0 + per);
    const uint32_t p_addr = smem_u32(P);
    for (int j = j0; j < j1; ++j) {
      float part[8];  // all loads in flight before the sum (cluster size <= 8)
#pragma unroll
      for (int c = 0; c < 8; ++c)
        part[c] = c < csize ? ld_dsmem(map_rank(p_addr + (uint32_t)(j * 128 + f) * 4, (uint32_t)c)) : 0.f;
      float acc = 0.f;
#pragma unroll
      for (int c = 0; c < 8; ++c) acc += part[c];
      if (W8) acc *= args.w_scale[m_tile * 128 + f];
      if (args.mode == kCStore) {
        const size_t o = (size_t)j * args.ldc + (size_t)m_tile * 128 + f;
        if (args.residual) acc += __bfloat162float(args.residual[o]);
        args.out[o] = __float2bfloat16(acc);
        continue;
      }
      if (args.mode == kCSwiGLU) {  // feature f < 64 is a gate, f + 64 its up: out = silu(gate) * up
        rot[f] = acc;
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (f < 64) args.out[(size_t)j * args.ldc + (size_t)m_tile * 64 + f] = __float2bfloat16(silu(acc) * rot[f + 64]);
        asm volatile("bar.sync 1, 128;" ::: "memory");  // rot[] is reused by the next token
        continue;
      }
      // kCQkvRope: this tile is head h of the packed [q | k | v] projection
      const int h = m_tile;
      const bool is_q = h < args.Hq, is_k = !is_q && h < args.Hq + args.Hkv;
      float v = __bfloat162float(__float2bfloat16(acc));  // the projection output is bf16
      const int slot = args.slots ? args.slots[j] : -1;
      if (is_q || is_k) {
        const __nv_bfloat16* nw = is_q ? args.q_w : args.k_w;
        if (nw) {
          const float ss = warp_sum(v * v);
          if (lane == 0) red[warp & 3] = ss;
          asm volatile("bar.sync 1, 128;" ::: "memory");
          const float tot = red[0] + red[1] + red[2] + red[3];
          const float inv = rsqrtf(tot / 128.f + args.eps);
          v = __bfloat162float(__float2bfloat16(v * inv * __bfloat162float(nw[f])));
        }
        rot[f] = v;
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const int half = args.rot_dim / 2;
        if (f < args.rot_dim) {
          const int ii = f < half ? f : f - half;
          float s, c;
          sincosf((float)args.pos[j] * args.inv_freq[ii], &s, &c);
          const float other = f < half ? -rot[f + half] : rot[f - half];
          v = v * c + other * s;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");  // rot[] / red[] are reused by the next token
      }
      if (is_q) {
        args.q_out[((size_t)j * args.Hq + h) * 128 + f] = __float2bfloat16(v);
      } else if (slot >= 0) {
        const int hk = is_k ? h - args.Hq : h - args.Hq - args.Hkv;
        const size_t blk = slot / args.block_size, off = slot % args.block_size;
        if (is_k)
          args.k_cache[((blk * args.Hkv + hk) * args.block_size + off) * 128 + f] = __float2bfloat16(v);
        else  // V blocks are [Hkv, D, block_size]
          args.v_cache[((blk * args.Hkv + hk) * 128 + f) * args.block_size + off] = __float2bfloat16(v);
      }
    }
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync_all();  // no CTA leaves while another still reads its partial tile
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::kTmemCols);
  }
}

template <int BN, int STAGES, bool W8>
void launch_cluster(const CUtensorMap& ta, const CUtensorMap& tb, const ClusterArgs& a, int m_tiles, int cs,
                    cudaStream_t st) {
  using L = CSmem<BN, STAGES, W8>;
  auto k = gemm_cluster_kernel<BN, STAGES, W8>;
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes));
    attr = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(m_tiles * cs, 1, 1);
  cfg.blockDim = dim3(192, 1, 1);
  cfg.dynamicSmemBytes = L::kBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr2[2];
  attr2[0].id = cudaLaunchAttributeClusterDimension;
  attr2[0].val.clusterDim.x = cs;
  attr2[0].val.clusterDim.y = 1;
  attr2[0].val.clusterDim.z = 1;
  attr2[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr2[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr2;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k, ta, tb, a));
}

int sm_count(int dev) {
  static int n[64] = {0};
  if (!n[dev]) C10_CUDA_CHECK(cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev));
  return n[dev];
}

// Cluster size: the largest power of two <= 8 that keeps at least two 64-wide K
// blocks per CTA and the grid within two CTAs per SM.
int pick_cs(int m_tiles, int kb_total, int sms) {
  int cs = 1;
  while (cs * 2 <= 8 && kb_total / (cs * 2) >= 2 && m_tiles * cs * 2 <= 2 * sms) cs *= 2;
  return cs;
}

// w: bf16 [N, K], or int8 [N, K] with a.w_scale set (per-row scales).
void run(const at::Tensor& x, const at::Tensor& w, ClusterArgs a, int64_t cs_req) {
  const int64_t T = x.size(0), K = x.size(1), N = w.size(0);
  const bool w8 = w.scalar_type() == at::kChar;
  const int bn = T <= 16 ? 16 : T <= 32 ? 32 : T <= 64 ? 64 : 128;
  const bool sw = a.mode == kCSwiGLU;   // 64-row boxes, one m tile per 64 outputs
  const int box = sw ? 64 : 128;
  auto ta = w8 ? make_tmap_2d(w.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, N, K, w.stride(0), 64, box,
                              CU_TENSOR_MAP_SWIZZLE_NONE)
               : make_tmap_bf16(w.data_ptr(), N, K, w.stride(0), box);
  auto tb = make_tmap_bf16(x.data_ptr(), T, K, x.stride(0), bn);
  const int m_tiles = (int)(sw ? N / 2 / 64 : N / 128);
  const int kb_total = (int)((K + 63) / 64);
  int cs = cs_req > 0 ? (int)cs_req : pick_cs(m_tiles, kb_total, sm_count(x.device().index()));
  TORCH_CHECK(cs == 1 || cs == 2 || cs == 4 || cs == 8, "gemm_cluster: cluster size must be 1, 2, 4 or 8");
  a.kb_per = (kb_total + cs - 1) / cs;
  a.K = (int)K;
  a.N = (int)N;
  a.T = (int)T;
  a.status = status_ptr(x.device().index());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  // stage counts keep a CTA near 100-120 KB of shared memory
  if (w8) {
    switch (bn) {
      case 16: launch_cluster<16, 4, true>(ta, tb, a, m_tiles, cs, st); break;
      case 32: launch_cluster<32, 4, true>(ta, tb, a, m_tiles, cs, st); break;
      case 64: launch_cluster<64, 3, true>(ta, tb, a, m_tiles, cs, st); break;
      default: launch_cluster<128, 3, true>(ta, tb, a, m_tiles, cs, st); break;
    }
  } else {
    switch (bn) {
      case 16: launch_cluster<16, 5, false>(ta, tb, a, m_tiles, cs, st); break;
      case 32: launch_cluster<32, 5, false>(ta, tb, a, m_tiles, cs, st); break;
      case 64: launch_cluster<64, 4, false>(ta, tb, a, m_tiles, cs, st); break;
      default: launch_cluster<128, 3, false>(ta, tb, a, m_tiles, cs, st); break;
    }
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void set_wait(ClusterArgs& a, int64_t ag_flags, const c10::optional<at::Tensor>& state, int64_t nranks) {
  if (!ag_flags) return;
  TORCH_CHECK(state && state->defined() && state->scalar_type() == at::kInt && nranks >= 1,
              "gemm_cluster: waiting on shard flags needs the boundary state and the rank count");
  a.ag_flags = reinterpret_cast<const uint32_t*>(ag_flags);
  a.ag_epoch = reinterpret_cast<const uint32_t*>(state->data_ptr<int>());
  a.ag_nranks = (int)nranks;
}

void check_operands(const at::Tensor& x, const at::Tensor& w) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && x.scalar_type() == at::kBFloat16 &&
              (w.scalar_type() == at::kBFloat16 || w.scalar_type() == at::kChar));
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.stride(1) == 1 && w.stride(1) == 1 && w.size(1) == x.size(1));
  TORCH_CHECK(x.size(0) >= 1 && x.size(0) <= 128, "gemm_cluster: 1..128 tokens");
  TORCH_CHECK(w.size(0) % 128 == 0 && x.size(1) % 64 == 0, "gemm_cluster: N % 128 == 0 and K % 64 == 0");
}

}  // namespace

// y[T, N] = x @ w^T (+ residual) for decode-sized T (<= 128); cs = 0 picks the cluster size.
// ag_flags != 0 (tensor parallelism): x is the gathered buffer; the loads of x wait until every
// rank's flag reaches state[0] (bounded).
void linear_cluster(const at::Tensor& x, const at::Tensor& w, at::Tensor& y,
                    const c10::optional<at::Tensor>& residual, int64_t cs, int64_t ag_flags,
                    const c10::optional<at::Tensor>& state, int64_t nranks) {
  check_operands(x, w);
  TORCH_CHECK(w.scalar_type() == at::kBFloat16, "linear_cluster: bf16 weights (int8: linear_cluster_w8)");
  TORCH_CHECK(y.is_contiguous() && y.scalar_type() == at::kBFloat16 && y.size(0) == x.size(0) &&
              y.size(1) == w.size(0));
  c10::cuda::CUDAGuard guard(x.device());
  ClusterArgs a{};
  a.mode = kCStore;
  a.out = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  a.ldc = (int)y.size(1);
  if (residual && residual->defined()) {
    TORCH_CHECK(residual->is_contiguous() && residual->sizes() == y.sizes());
    a.residual = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
  }
  set_wait(a, ag_flags, state, nranks);
  run(x, w, a, cs);
}

// y[T, I] = silu(x @ gate^T) * (x @ up^T), w = [gate; up] ([2I, K], I % 64 == 0), decode-sized T;
// one launch (the split-K partials of gate and up are reduced through DSMEM, SwiGLU in the epilogue).
// ag_flags / state / nranks: as in linear_cluster.
void swiglu_cluster(const at::Tensor& x, const at::Tensor& w, at::Tensor& y, int64_t cs, int64_t ag_flags,
                    const c10::optional<at::Tensor>& state, int64_t nranks) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16,
              "swiglu_cluster: bf16 operands");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.stride(1) == 1 && w.is_contiguous() && w.size(1) == x.size(1));
  TORCH_CHECK(x.size(0) >= 1 && x.size(0) <= 128, "swiglu_cluster: 1..128 tokens");
  const int64_t I = w.size(0) / 2;
  TORCH_CHECK(w.size(0) % 128 == 0 && I % 64 == 0 && x.size(1) % 64 == 0,
              "swiglu_cluster: w must be [2I, K] with I % 64 == 0 and K % 64 == 0");
  TORCH_CHECK(y.is_contiguous() && y.scalar_type() == at::kBFloat16 && y.size(0) == x.size(0) && y.size(1) == I);
  c10::cuda::CUDAGuard guard(x.device());
  ClusterArgs a{};
  a.mode = kCSwiGLU;
  a.out = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  a.ldc = (int)I;
  a.up_row0 = (int)I;
  set_wait(a, ag_flags, state, nranks);
  run(x, w, a, cs);
}

// int8 weight-only: y = (x @ wq^T) * scale[n] (+ residual); wq int8 [N, K], scale fp32 [N].
void linear_cluster_w8(const at::Tensor& x, const at::Tensor& wq, const at::Tensor& scale, at::Tensor& y,
                       const c10::optional<at::Tensor>& residual, int64_t cs) {
  check_operands(x, wq);
  TORCH_CHECK(wq.scalar_type() == at::kChar && scale.scalar_type() == at::kFloat && scale.numel() == wq.size(0));
  TORCH_CHECK(y.is_contiguous() && y.scalar_type() == at::kBFloat16 && y.size(0) == x.size(0) &&
              y.size(1) == wq.size(0));
  c10::cuda::CUDAGuard guard(x.device());
  ClusterArgs a{};
  a.mode = kCStore;
  a.out = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  a.ldc = (int)y.size(1);
  a.w_scale = scale.data_ptr<float>();
  if (residual && residual->defined()) {
    TORCH_CHECK(residual->is_contiguous() && residual->sizes() == y.sizes());
    a.residual = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
  }
  run(x, wq, a, cs);
}

// Packed QKV projection (head_dim 128) with per-head QK-RMSNorm, RoPE and the
// paged KV write fused into the cluster reduction: same outputs as
// linear + rope_qknorm.
void qkv_rope_cluster(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& q_w,
                      const c10::optional<at::Tensor>& k_w, const at::Tensor& positions, const at::Tensor& inv_freq,
                      const c10::optional<at::Tensor>& slots, at::Tensor& q_out, at::Tensor& k_cache,
                      at::Tensor& v_cache, int64_t Hq, int64_t Hkv, int64_t rot_dim, double eps, int64_t cs,
                      int64_t ag_flags, const c10::optional<at::Tensor>& state, int64_t nranks) {
  check_operands(x, w);
  TORCH_CHECK(w.scalar_type() == at::kBFloat16, "qkv_rope_cluster: bf16 weights");
  const int64_t T = x.size(0);
  TORCH_CHECK(w.size(0) == (Hq + 2 * Hkv) * 128, "qkv_rope_cluster: w must be [(Hq + 2 Hkv) * 128, K]");
  TORCH_CHECK(positions.scalar_type() == at::kInt && positions.numel() == T && inv_freq.scalar_type() == at::kFloat);
  TORCH_CHECK(rot_dim % 2 == 0 && rot_dim <= 128 && inv_freq.numel() >= rot_dim / 2);
  TORCH_CHECK(q_out.is_contiguous() && q_out.numel() == T * Hq * 128);
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous() && k_cache.size(1) == Hkv && k_cache.size(3) == 128 &&
              v_cache.size(2) == 128 && v_cache.size(3) == k_cache.size(2));
  if (slots && slots->defined()) TORCH_CHECK(slots->scalar_type() == at::kInt && slots->numel() == T);
  c10::cuda::CUDAGuard guard(x.device());
  auto bf = [](const c10::optional<at::Tensor>& o) -> const __nv_bfloat16* {
    return (o && o->defined()) ? reinterpret_cast<const __nv_bfloat16*>(o->data_ptr()) : nullptr;
  };
  ClusterArgs a{};
  a.mode = kCQkvRope;
  a.q_w = bf(q_w);
  a.k_w = bf(k_w);
  a.pos = positions.data_ptr<int>();
  a.inv_freq = inv_freq.data_ptr<float>();
  a.slots = (slots && slots->defined()) ? slots->data_ptr<int>() : nullptr;
  a.q_out = reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr());
  a.k_cache = reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr());
  a.v_cache = reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr());
  a.Hq = (int)Hq;
  a.Hkv = (int)Hkv;
  a.rot_dim = (int)rot_dim;
  a.block_size = (int)k_cache.size(2);
  a.eps = (float)eps;
  set_wait(a, ag_flags, state, nranks);
  run(x, w, a, cs);
}

}  // namespace mb
