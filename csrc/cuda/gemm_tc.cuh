// bf16 GEMM on 5th-generation tensor cores (tcgen05 + TMEM), TMA-fed.
//
//   D[i, j] = sum_k A[i, k] * B[j, k]        (both operands K-major, bf16)
//
// A is the "M side" (128 rows per tile, one TMEM lane per row) and B the
// "N side" (BN rows per tile, one TMEM column per row).  Linear layers run in
// one of two orientations:
//   * swap   : A = weight [out, in], B = activations [tokens, in].  Decode and
//              MoE shapes have few tokens, so the 128-row MMA dimension is
//              filled by weight rows and the token count only sets BN.
//   * normal : A = activations, B = weight (large-M prefill).
// Grouped mode (MoE experts): group g uses A rows [g*a_group_rows, ...) and
// B rows [offs[g], offs[g+1]) where offs lives in device memory, so the
// schedule needs no host synchronisation and is CUDA-graph safe.
//
// CTA = 6 warps: warp 0 issues TMA loads, warp 1 allocates TMEM and issues
// tcgen05.mma from one elected lane, warps 2-5 drain TMEM accumulators
// (double-buffered, so the epilogue of tile t overlaps the MMAs of t+1).
// Replaces the reference's FP32 SIMT matmul/linear kernels
// (pio/plugins/cuda/c_src/tensor_ops_cuda.cu:290-329).
#pragma once
#include "common.cuh"

namespace mb {

enum EpiMode : int {
  kEpiStore = 0,      // bf16 store of D (optionally + bf16 residual)
  kEpiSwiGLU = 1,     // dual accumulator: silu(D_gate) * D_up
  kEpiPartialF32 = 2, // fp32 split-K partial to a workspace
  kEpiScatterRS = 3,  // tensor parallel: bf16 partial rows stored into the owning rank's slot (P2P)
  kEpiScatterRows = 4,  // (+ bias) each output row stored at row_map[row] of its owner's buffer (P2P)
};

// Tensor-parallel operands of a GEMM: a wait on the flags of the shards that
// the peers pushed into this rank's gathered buffer, and/or a reduce-scatter
// epilogue.  Peer memory is only written, by ordinary stores.
struct TpArgs {
  const uint32_t* ag_flags;       // [N] local: ag_flags[p] >= *epoch once rank p's shard is ready
  uint32_t* epoch;                // local boundary counter
  int peer_rows;                  // rows per shard (tokens per rank)
  int sub;                        // rows per TMA sub-load
  int nranks, rank;
  const uint64_t* rs_peers;       // [N] base of every rank's exchange buffer
  int64_t rs_off;                 // byte offset of the partial slots [N][peer_rows][ldc]
  int64_t rs_flag_off;            // byte offset of the RS flags [N]
  int* done;                      // local CTA-completion counter
  int epoch_add;                  // the producer waits for flags >= *epoch + epoch_add
  const int* row_map;             // kEpiScatterRows: destination of each output row, d * peer_rows + row
  int rank_row_stride;            // kEpiScatterRows: the row lands at rank * stride + row of rank d's buffer
};

struct GemmArgs {
  int K;                 // reduction length
  int a_rows;            // rows of A per group (multiple of 128)
  int a_up_offset;       // SwiGLU: row offset of the "up" half inside a group
  int b_rows;            // dense mode: rows of B; grouped mode: unused
  const int* b_offs;     // grouped mode: [groups+1] row offsets into B (device)
  int groups;
  int splits;            // split-K factor
  int swap;              // 1: out[j, i] ; 0: out[i, j]
  int mode;              // EpiMode
  void* out;             // bf16 [tokens, ldc] or f32 [splits, tokens, ldc]
  const __nv_bfloat16* residual;  // optional, same layout as out
  int ldc;
  int out_rows;          // tokens (rows of out) for the split-K workspace stride
  int* status;
  TpArgs tp;             // zero-initialised: not tensor parallel
  const float* w_scale;  // int8-weight variant: per-row scale of A (row g*a_rows + r), applied in the epilogue
  const __nv_bfloat16* bias;  // kEpiScatterRows: per output feature
  // Persistent schedule (items > 0): the grid is sized to the resident CTAs and
  // CTA b takes work items b, b + gridDim.x, ...; item i is (m_tile, y, z) with
  // m_tile = i % m_tiles, y = (i / m_tiles) % ny, z = i / (m_tiles * ny).  The
  // TMA/MMA stage ring and the TMEM double buffer carry over from one item to
  // the next, so a CTA streams weights without a pipeline drain per tile.
  // items == 0: one item per CTA, (blockIdx.x, blockIdx.y, blockIdx.z).
  int items, m_tiles, ny;
};

// One unit of CTA work: a 128-row A tile of group g, the N tiles
// y, y + ny, ... of that group, over one split's K-block range.
struct GemmItem {
  int g, split, m_tile, y, b0, cnt, my_tiles, kb_lo, kb_hi, kbs, a_row0;
};

__device__ __forceinline__ int gemm_num_items(const GemmArgs& a) { return a.items > 0 ? a.items : 1; }

__device__ __forceinline__ GemmItem gemm_item(const GemmArgs& a, int i) {
  GemmItem w;
  int y, z;
  if (a.items > 0) {
    const int idx = (int)blockIdx.x + i * (int)gridDim.x;
    w.m_tile = idx % a.m_tiles;
    y = (idx / a.m_tiles) % a.ny;
    z = idx / (a.m_tiles * a.ny);
  } else {
    w.m_tile = blockIdx.x;
    y = blockIdx.y;
    z = blockIdx.z;
  }
  w.y = y;
  w.g = z / a.splits;
  w.split = z % a.splits;
  if (a.b_offs != nullptr) {
    w.b0 = a.b_offs[w.g];
    w.cnt = a.b_offs[w.g + 1] - w.b0;
  } else {
    w.b0 = 0;
    w.cnt = a.b_rows;
  }
  w.my_tiles = 0;
  w.kb_lo = w.kb_hi = w.kbs = 0;
  w.a_row0 = w.g * a.a_rows + w.m_tile * 128;
  return w;
}

// Exact int8 -> bf16 for 4 packed values (byte i = element i).  Float
// magic-number method: placing the biased byte u = b + 128 in the low mantissa
// bits of 2^23 gives the float 2^23 + u; subtracting 2^23 + 128 leaves b
// exactly, and any integer in [-128, 127] is exact in bf16, so truncating to
// the upper half is exact too.  Full-rate PRMT/FADD only (no I2F).
__device__ __forceinline__ void i8x4_to_bf16x4(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t x = w ^ 0x80808080u;
  const float f0 = __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7650)) - 8388736.f;
  const float f1 = __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7651)) - 8388736.f;
  const float f2 = __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7652)) - 8388736.f;
  const float f3 = __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7653)) - 8388736.f;
  lo = __byte_perm(__float_as_uint(f0), __float_as_uint(f1), 0x7632);
  hi = __byte_perm(__float_as_uint(f2), __float_as_uint(f3), 0x7632);
}

// Loads `rows` activation rows starting at row `row0`, k-block kx.
__device__ __forceinline__ void load_act(const GemmArgs&, const CUtensorMap* local, void* dst, uint64_t* bar, int kx,
                                         int row0, int) {
  tma_load_2d(dst, local, bar, kx, row0);
}

// Stage layout: A tile(s) [128 x 64] bf16 SW128 | B tile [BN x 64] bf16 SW128 |
// (W8) raw int8 A tile(s) [128 x 64], unswizzled, that the converter warps expand
// into the A slots.
template <int BN, int STAGES, bool DUAL, bool W8 = false>
struct GemmSmem {
  static constexpr int kNA = DUAL ? 2 : 1;
  static constexpr int kABytes = 128 * 64 * 2;
  static constexpr int kBBytes = BN * 64 * 2;
  static constexpr int kRawBytes = W8 ? 128 * 64 : 0;
  static constexpr int kRawOff = kABytes * kNA + kBBytes;
  static constexpr int kStageBytes = kRawOff + kRawBytes * kNA;
  static constexpr int kTxBytes = kStageBytes - (W8 ? kABytes * kNA : 0);  // bytes TMA delivers per stage
  static constexpr int kBytes = STAGES * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
  static constexpr int kThreads = W8 ? 320 : 192;
};

// Warp roles: 0 TMA producer, 1 MMA issuer, 2-5 epilogue (TMEM lane quadrant
// warp % 4), 6-9 int8 -> bf16 converters (W8 only).
template <int BN, int STAGES, bool DUAL, bool W8 = false>
__global__ void __launch_bounds__(GemmSmem<BN, STAGES, DUAL, W8>::kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   GemmArgs args) {
  using L = GemmSmem<BN, STAGES, DUAL, W8>;
  constexpr int kAcc = DUAL ? 2 * BN : BN;          // TMEM columns per buffer
  constexpr int kTmemCols = (2 * kAcc <= 32) ? 32 : (2 * kAcc <= 64) ? 64 : (2 * kAcc <= 128) ? 128
                            : (2 * kAcc <= 256) ? 256 : 512;
  static_assert(2 * kAcc <= 512, "TMEM overflow");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * L::kStageBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;   // [2]
  uint64_t* tempty = tfull + 2;       // [2]
  uint64_t* cfull = tempty + 2;      // [STAGES] (W8) A tiles converted
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(cfull + STAGES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int ny = args.items > 0 ? args.ny : (int)gridDim.y;
  const int n_items = args.items > 0
                          ? ((int)blockIdx.x < args.items ? (args.items - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0)
                          : 1;

  // Dependent launch: every thread waits for the previous kernel before it
  // touches activations, group offsets or outputs.  The producer of a dense
  // GEMM (no device-side offsets) first prefetches weight tiles, which no
  // earlier kernel writes.
  const bool dense = args.b_offs == nullptr;
  if (!(warp == 0 && dense)) {
    pdl_wait();
    pdl_trigger();
  }
  // Work item i of this CTA: N tiles nt = y + r*ny of group g, over the
  // split's K-block range (see GemmItem).
  const int kb_total = (args.K + 63) / 64;
  const int kb_per = (kb_total + args.splits - 1) / args.splits;
  auto item = [&](int i) {
    GemmItem w = gemm_item(args, i);
    const int n_tiles = (w.cnt + BN - 1) / BN;
    w.my_tiles = n_tiles > w.y ? (n_tiles - 1 - w.y) / ny + 1 : 0;
    w.kb_lo = w.split * kb_per;
    w.kb_hi = min(kb_total, w.kb_lo + kb_per);
    w.kbs = max(0, w.kb_hi - w.kb_lo);
    if (w.kbs == 0) w.my_tiles = 0;
    return w;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      if (W8) mbar_init(&cfull[s], 4);  // one arrival per converter warp
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  {
    if (warp == 0) {
      // ------------------------------------------------ TMA producer
      const bool leader = elect_one_sync();
      // weight tiles of the first stages, issued before the dependency wait
      // (dense GEMMs only: their first item needs no device-side offsets)
      const GemmItem w0 = (dense && n_items > 0) ? item(0) : GemmItem{};
      const int pre = (dense && args.swap && n_items > 0 && w0.my_tiles > 0) ? min(STAGES, w0.kbs) : 0;
      if (leader) {
        for (int s = 0; s < pre; ++s) {
          uint8_t* st = smem + s * L::kStageBytes;
          uint8_t* wa = W8 ? st + L::kRawOff : st;
          mbar_arrive_expect_tx(&full[s], L::kTxBytes);
          tma_load_2d(wa, &tmA, &full[s], (w0.kb_lo + s) * 64, w0.a_row0);
          if (DUAL)
            tma_load_2d(wa + (W8 ? L::kRawBytes : L::kABytes), &tmA, &full[s], (w0.kb_lo + s) * 64,
                        w0.a_row0 + args.a_up_offset);
        }
      }
      if (dense) {
        pdl_wait();
        pdl_trigger();
      }
      if (args.tp.ag_flags && leader) {  // every peer's shard must be published for this boundary
        const uint32_t want = *args.tp.epoch + (uint32_t)args.tp.epoch_add;
        for (int p = 0; p < args.tp.nranks; ++p) {
          const uint64_t t0 = globaltimer_ns();
          while (true) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(args.tp.ag_flags + p) : "memory");
            if ((int32_t)(v - want) >= 0) break;
            // half the limit: the other warps' bounded mbarrier waits started with this one
            if (globaltimer_ns() - t0 > kWaitLimitNs / 2) {
              set_status(args.status, kErrPeerTimeout);
              break;
            }
          }
        }
      }
      if (leader) {
        int it = 0;
        bool ok = true;
        for (int wi = 0; wi < n_items && ok; ++wi) {
        const GemmItem w = item(wi);
        const int b0 = w.b0, a_row0 = w.a_row0;
        for (int t = 0; t < w.my_tiles && ok; ++t) {
          const int nt = w.y + t * ny;
          for (int kb = w.kb_lo; kb < w.kb_hi; ++kb, ++it) {
            const int s = it % STAGES;
            uint8_t* st = smem + s * L::kStageBytes;
            if (it < pre) {  // weights already in flight: add the activation tile
              load_act(args, &tmB, st + L::kABytes * (DUAL ? 2 : 1), &full[s], kb * 64, b0 + nt * BN, BN);
              continue;
            }
            const uint32_t ph = (it / STAGES) & 1;
            if (!mbar_wait(&empty[s], ph ^ 1, args.status)) { ok = false; break; }
            mbar_arrive_expect_tx(&full[s], L::kTxBytes);
            if (args.swap) {
              uint8_t* wa = W8 ? st + L::kRawOff : st;
              tma_load_2d(wa, &tmA, &full[s], kb * 64, a_row0);
              if (DUAL)
                tma_load_2d(wa + (W8 ? L::kRawBytes : L::kABytes), &tmA, &full[s], kb * 64,
                            a_row0 + args.a_up_offset);
              load_act(args, &tmB, st + L::kABytes * (DUAL ? 2 : 1), &full[s], kb * 64, b0 + nt * BN, BN);
            } else {  // normal orientation: activations are the 128-row A operand
              load_act(args, &tmA, st, &full[s], kb * 64, a_row0, 128);
              tma_load_2d(st + L::kABytes, &tmB, &full[s], kb * 64, b0 + nt * BN);
            }
          }
        }
        }
      }
    } else if (warp == 1) {
      // ------------------------------------------------ MMA issuer
      constexpr uint32_t idesc = make_idesc_bf16(128, BN);
      if (elect_one_sync()) {
        int it = 0, tt = 0;  // stage and TMEM-buffer counters run on across items
        bool ok = true;
        for (int wi = 0; wi < n_items && ok; ++wi) {
        const GemmItem w = item(wi);
        for (int t = 0; t < w.my_tiles && ok; ++t, ++tt) {
          const int buf = tt & 1;
          if (!mbar_wait(&tempty[buf], ((tt >> 1) & 1) ^ 1, args.status)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d0 = tmem_base + buf * kAcc;
          for (int kb = 0; kb < w.kbs; ++kb, ++it) {
            const int s = it % STAGES;
            const uint32_t ph = (it / STAGES) & 1;
            if (!mbar_wait(&full[s], ph, args.status)) { ok = false; break; }
            if (W8 && !mbar_wait(&cfull[s], ph, args.status)) { ok = false; break; }
            tc_fence_after();
            uint8_t* st = smem + s * L::kStageBytes;
            const uint32_t a_addr = smem_u32(st);
            const uint32_t b_addr = smem_u32(st + L::kABytes * (DUAL ? 2 : 1));
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t bd = make_sdesc_k128(b_addr + kk * 32);
              tc_mma_bf16(d0, make_sdesc_k128(a_addr + kk * 32), bd, idesc, (kb | kk) != 0);
              if (DUAL) tc_mma_bf16(d0 + BN, make_sdesc_k128(a_addr + L::kABytes + kk * 32), bd, idesc, (kb | kk) != 0);
            }
            tc_commit(&empty[s]);
          }
          tc_commit(&tfull[buf]);
        }
        }
      }
    } else if (W8 && warp >= 6) {
      // ------------------------------------------------ int8 -> bf16 converters (warps 6-9)
      // Thread c expands 16-byte chunks idx = c + 128 m of the [128 x 64] tile:
      // row r = idx / 8, chunk k = idx % 8 -> SW128 position r*128 + (k ^ (r % 8))*16.
      const int c = threadIdx.x - 192;
      int it = 0;
      bool ok = true;
      for (int wi = 0; wi < n_items && ok; ++wi) {
      const GemmItem w = item(wi);
      for (int t = 0; t < w.my_tiles && ok; ++t) {
        for (int kb = 0; kb < w.kbs; ++kb, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(&full[s], (it / STAGES) & 1, args.status)) { ok = false; break; }
          uint8_t* st = smem + s * L::kStageBytes;
#pragma unroll
          for (int a = 0; a < L::kNA; ++a) {
            const uint8_t* raw = st + L::kRawOff + a * L::kRawBytes;
            uint8_t* dst = st + a * L::kABytes;
#pragma unroll
            for (int m = 0; m < 8; ++m) {
              const int idx = c + 128 * m, r = idx >> 3, k = idx & 7;
              const uint2 w = *reinterpret_cast<const uint2*>(raw + r * 64 + k * 8);
              uint4 o;
              i8x4_to_bf16x4(w.x, o.x, o.y);
              i8x4_to_bf16x4(w.y, o.z, o.w);
              *reinterpret_cast<uint4*>(dst + r * 128 + ((k ^ (r & 7)) << 4)) = o;
            }
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor-core reads
          __syncwarp();
          if (lane == 0) mbar_arrive(&cfull[s]);
        }
      }
      }
    } else {
      // ------------------------------------------------ epilogue (warps 2-5)
      const int lane_base = (warp & 3) * 32;
      const int i = lane_base + lane;             // accumulator row (TMEM lane)
      int tt = 0;
      bool ok = true;
      for (int wi = 0; wi < n_items && ok; ++wi) {
      const GemmItem w = item(wi);
      const int g = w.g, split = w.split, b0 = w.b0, cnt = w.cnt;
      for (int t = 0; t < w.my_tiles; ++t, ++tt) {
        const int buf = tt & 1;
        const int nt = w.y + t * ny;
        if (!mbar_wait(&tfull[buf], (tt >> 1) & 1, args.status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t taddr = tmem_base + ((uint32_t)lane_base << 16) + buf * kAcc;
        const int arow = w.m_tile * 128 + i;      // row of A inside the group
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
          tmem_ld16(taddr + c0, v);
          if (W8) {
            const float sc = args.w_scale[g * args.a_rows + arow];
#pragma unroll
            for (int q = 0; q < 16; ++q) v[q] *= sc;
          }
          float u[16];
          if (DUAL) {
            tmem_ld16(taddr + BN + c0, u);
            if (W8) {
              const float sc = args.w_scale[g * args.a_rows + arow + args.a_up_offset];
#pragma unroll
              for (int q = 0; q < 16; ++q) u[q] *= sc;
            }
            if (args.mode != kEpiPartialF32) {
#pragma unroll
              for (int q = 0; q < 16; ++q) v[q] = silu(v[q]) * u[q];
            }
          }
          const int jbase = nt * BN + c0;         // B row inside the group
          if (args.swap) {
            // out[(b0 + j), arow]: lanes of a warp write consecutive columns.  The mode
            // switch sits outside the 16-column loop so each loop is straight-line code.
            const int nq = min(16, cnt - jbase);
            if (args.mode == kEpiPartialF32) {
              const size_t ld = DUAL ? 2 * (size_t)args.ldc : (size_t)args.ldc;
              float* p = reinterpret_cast<float*>(args.out) + (size_t)split * args.out_rows * ld +
                         (size_t)(b0 + jbase) * ld + arow;
#pragma unroll
              for (int q = 0; q < 16; ++q) {
                if (q < nq) {
                  p[q * ld] = v[q];
                  if (DUAL) p[q * ld + args.ldc] = u[q];  // raw gate | up partials; SwiGLU after the reduction
                }
              }
            } else if (args.mode == kEpiScatterRows) {
              const float bv = args.bias ? __bfloat162float(args.bias[arow]) : 0.f;
#pragma unroll
              for (int q = 0; q < 16; ++q) {
                if (q < nq) {  // row map may have been written by other GPUs: read it from L2
                  const int grow = __ldcg(args.tp.row_map + b0 + jbase + q);
                  const int d = grow / args.tp.peer_rows, jl = grow - d * args.tp.peer_rows;
                  if (d < 0 || d >= args.tp.nranks) continue;
                  __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(args.tp.rs_peers[d] + args.tp.rs_off);
                  dst[((size_t)args.tp.rank * args.tp.rank_row_stride + jl) * args.ldc + arow] =
                      __float2bfloat16(v[q] + bv);
                }
              }
            } else if (args.mode == kEpiScatterRS) {
#pragma unroll
              for (int q = 0; q < 16; ++q) {  // fully unrolled: v stays in registers
                if (q < nq) {
                  const int tok = b0 + jbase + q, d = tok / args.tp.peer_rows, jl = tok - d * args.tp.peer_rows;
                  __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(args.tp.rs_peers[d] + args.tp.rs_off);
                  dst[((size_t)args.tp.rank * args.tp.peer_rows + jl) * args.ldc + arow] = __float2bfloat16(v[q]);
                }
              }
            } else {
              const size_t off = (size_t)(b0 + jbase) * args.ldc + arow;
              __nv_bfloat16* p = reinterpret_cast<__nv_bfloat16*>(args.out) + off;
              if (args.residual) {
                const __nv_bfloat16* r = args.residual + off;
#pragma unroll
                for (int q = 0; q < 16; ++q)
                  if (q < nq) p[(size_t)q * args.ldc] = __float2bfloat16(v[q] + __bfloat162float(r[(size_t)q * args.ldc]));
              } else {
#pragma unroll
                for (int q = 0; q < 16; ++q)
                  if (q < nq) p[(size_t)q * args.ldc] = __float2bfloat16(v[q]);
              }
            }
          } else {
            // out[arow, j]: 16 consecutive columns per thread.
            const int grow = g * args.a_rows + arow;
            if (grow < args.out_rows && args.mode == kEpiScatterRS) {
              const int d = grow / args.tp.peer_rows, jl = grow - d * args.tp.peer_rows;
              __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(args.tp.rs_peers[d] + args.tp.rs_off) +
                                   ((size_t)args.tp.rank * args.tp.peer_rows + jl) * args.ldc + jbase;
              __align__(16) __nv_bfloat16 h[16];
#pragma unroll
              for (int q = 0; q < 16; ++q) h[q] = __float2bfloat16(v[q]);
              if (jbase + 16 <= cnt) {
                reinterpret_cast<uint4*>(dst)[0] = reinterpret_cast<uint4*>(h)[0];
                reinterpret_cast<uint4*>(dst)[1] = reinterpret_cast<uint4*>(h)[1];
              } else {
#pragma unroll
                for (int q = 0; q < 16; ++q)
                  if (jbase + q < cnt) dst[q] = h[q];
              }
            } else if (grow < args.out_rows) {
              const size_t o = (size_t)grow * args.ldc + jbase;
              if (args.mode == kEpiPartialF32) {
                float* dst = reinterpret_cast<float*>(args.out) + (size_t)split * args.out_rows * args.ldc + o;
#pragma unroll
                for (int q = 0; q < 16; ++q)
                  if (jbase + q < cnt) dst[q] = v[q];
              } else if (jbase + 16 <= cnt && (args.ldc & 7) == 0) {
                __align__(16) __nv_bfloat16 h[16];
#pragma unroll
                for (int q = 0; q < 16; ++q) {
                  float r = args.residual ? __bfloat162float(args.residual[o + q]) : 0.f;
                  h[q] = __float2bfloat16(v[q] + r);
                }
                uint4* d = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(args.out) + o);
                d[0] = reinterpret_cast<uint4*>(h)[0];
                d[1] = reinterpret_cast<uint4*>(h)[1];
              } else {
#pragma unroll
                for (int q = 0; q < 16; ++q)
                  if (jbase + q < cnt) {
                    float r = args.residual ? __bfloat162float(args.residual[o + q]) : 0.f;
                    reinterpret_cast<__nv_bfloat16*>(args.out)[o + q] = __float2bfloat16(v[q] + r);
                  }
              }
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty[buf]);
      }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (args.mode == kEpiScatterRS || args.mode == kEpiScatterRows) {
    // last CTA: every row of this rank is stored -> release the owners' flags
    __shared__ int last;
    __syncthreads();
    const int nct = gridDim.x * gridDim.y * gridDim.z;
    if (threadIdx.x == 0) {  // one system-scope fence per CTA, after the CTA barrier
      __threadfence_system();
      last = atomicAdd(args.tp.done, 1) == nct - 1;
    }
    __syncthreads();
    if (last) {
      __threadfence_system();
      const uint32_t e = *args.tp.epoch + (uint32_t)args.tp.epoch_add;
      for (int d = threadIdx.x; d < args.tp.nranks; d += blockDim.x) {
        uint32_t* f = reinterpret_cast<uint32_t*>(args.tp.rs_peers[d] + args.tp.rs_flag_off) + args.tp.rank;
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(e) : "memory");
      }
      if (threadIdx.x == 0) *args.tp.done = 0;
    }
  }
}

}  // namespace mb
