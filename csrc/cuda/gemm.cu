// Host side of the tcgen05 GEMM: tensor maps, tile/split selection, split-K
// reduction.  Exposed to Python through ops.cpp.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <mutex>

#include "gemm_tc.cuh"
#include "launch.cuh"
#include "status.h"

namespace mb {

static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    TORCH_CHECK(p != nullptr && q == cudaDriverEntryPointSuccess, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D bf16 map over a row-major [rows, cols] matrix with leading dimension ld
// (elements); box = 64 columns (128 B, the swizzle span) x box_rows rows.
CUtensorMap make_tmap_bf16(const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return m;
}

// General 2-D map: [rows, cols] of `dt` with row pitch ld_bytes; box = box_cols x box_rows.
CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dt, int64_t rows, int64_t cols, int64_t ld_bytes,
                         int box_cols, int box_rows, CUtensorMapSwizzle sw) {
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK(ld_bytes % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld_bytes};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode()(&m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return m;
}

template <int BN, int STAGES, bool DUAL, bool W8 = false>
static void launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, dim3 grid, cudaStream_t st) {
  using L = GemmSmem<BN, STAGES, DUAL, W8>;
  auto k = gemm_tc_kernel<BN, STAGES, DUAL, W8>;
  static bool attr = false;  // per instantiation
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes));
    attr = true;
  }
  GemmArgs args = a;
  if (args.items > 0) {  // persistent schedule: one wave of resident CTAs loops over the items
    static int resident = 0;  // per instantiation
    if (!resident) {
      int occ = 0, sms = 0;
      C10_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, L::kThreads, L::kBytes));
      C10_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, c10::cuda::current_device()));
      resident = std::max(1, occ) * sms;
    }
    // With few items per resident CTA a static stride balances worse than the hardware's
    // block scheduler (measured: MoE gate/up at 2.6 items per CTA ran 4% slower, the MoE
    // down GEMM at 6.9 items per CTA 7% faster), so persistence needs >= 4 items per CTA.
    if (args.items >= 4 * resident)
      grid = dim3((unsigned)resident, 1, 1);
    else
      args.items = 0;
  }
  launch_k(k, grid, L::kThreads, L::kBytes, st, ta, tb, args);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Grouped GEMMs run persistently unless MB_GEMM_PERSIST=0 (kept for A/B timing).
static bool persist_grouped() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("MB_GEMM_PERSIST");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

// Dispatch on the N tile.  DUAL keeps 4 accumulators of BN columns in TMEM,
// so it stops at BN = 128.
static void dispatch(int bn, bool dual, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, dim3 grid,
                     cudaStream_t st) {
  // Stage counts keep shared memory near 110 KB where possible, so two CTAs
  // share an SM and one CTA's prologue/epilogue overlaps the other's loads.
  if (dual) {
    switch (bn) {
      case 16: return launch<16, 3, true>(ta, tb, a, grid, st);
      case 32: return launch<32, 3, true>(ta, tb, a, grid, st);
      case 64: return launch<64, 4, true>(ta, tb, a, grid, st);
      default: return launch<128, 4, true>(ta, tb, a, grid, st);
    }
  }
  switch (bn) {
    case 16: return launch<16, 6, false>(ta, tb, a, grid, st);
    case 32: return launch<32, 5, false>(ta, tb, a, grid, st);
    case 64: return launch<64, 4, false>(ta, tb, a, grid, st);
    case 128: return launch<128, 3, false>(ta, tb, a, grid, st);
    default: return launch<256, 4, false>(ta, tb, a, grid, st);
  }
}

// int8-weight variant: each stage also holds the raw int8 A tile(s) (8 KB each).
// Stage counts keep two CTAs per SM up to BN = 128 (single accumulator) / 64 (dual).
static void dispatch_w8(int bn, bool dual, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a,
                        dim3 grid, cudaStream_t st) {
  if (dual) {
    switch (bn) {
      case 16: return launch<16, 2, true, true>(ta, tb, a, grid, st);
      case 32: return launch<32, 2, true, true>(ta, tb, a, grid, st);
      case 64: return launch<64, 2, true, true>(ta, tb, a, grid, st);
      default: return launch<128, 3, true, true>(ta, tb, a, grid, st);
    }
  }
  switch (bn) {
    case 16: return launch<16, 4, false, true>(ta, tb, a, grid, st);
    case 32: return launch<32, 3, false, true>(ta, tb, a, grid, st);
    case 64: return launch<64, 3, false, true>(ta, tb, a, grid, st);
    case 128: return launch<128, 2, false, true>(ta, tb, a, grid, st);
    default: return launch<256, 3, false, true>(ta, tb, a, grid, st);
  }
}

static int pick_bn(int64_t rows, bool dual) {
  int cap = dual ? 128 : 256;
  int bn = 16;
  while (bn < rows && bn < cap) bn *= 2;
  return bn;
}

static int num_sms() {
  static int n = 0;
  if (!n) C10_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, c10::cuda::current_device()));
  return n;
}

// split-K reduction: out = bf16(sum_s ws[s] (+ residual))
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits, int64_t n,
                                     const __nv_bfloat16* __restrict__ residual, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (i >= n) return;
  float4 acc = *reinterpret_cast<const float4*>(ws + i);
  for (int s = 1; s < splits; ++s) {
    float4 v = *reinterpret_cast<const float4*>(ws + (int64_t)s * n + i);
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
  }
  if (residual) {
    acc.x += __bfloat162float(residual[i]);
    acc.y += __bfloat162float(residual[i + 1]);
    acc.z += __bfloat162float(residual[i + 2]);
    acc.w += __bfloat162float(residual[i + 3]);
  }
  __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
  reinterpret_cast<__nv_bfloat162*>(out + i)[0] = lo;
  reinterpret_cast<__nv_bfloat162*>(out + i)[1] = hi;
}

// SwiGLU split-K reduction: ws [splits][T][2*I] (gate | up) -> out [T, I]
__global__ void splitk_swiglu_kernel(const float* __restrict__ ws, int splits, int T, int I,
                                     __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)T * I) return;
  const int64_t t = i / I, c = i % I;
  float g = 0.f, u = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float* p = ws + ((int64_t)s * T + t) * 2 * I;
    g += p[c];
    u += p[I + c];
  }
  out[i] = __float2bfloat16(silu(g) * u);
}

// y[T, I] = silu(x @ gate^T) * (x @ up^T) with w = [gate; up] ([2I, K]), dual-accumulator
// tcgen05 GEMM; decode shapes (T <= 256) use split-K with the SwiGLU applied after the reduction.
void swiglu_linear(const at::Tensor& x, const at::Tensor& w, at::Tensor& y, const c10::optional<at::Tensor>& workspace,
                   int64_t wait_flags, const c10::optional<at::Tensor>& state, int64_t nranks) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && w.is_contiguous());
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && y.is_contiguous());
  const int64_t T = x.size(0), K = x.size(1), I = w.size(0) / 2;
  TORCH_CHECK(w.size(1) == K && y.size(0) == T && y.size(1) == I && I % 128 == 0 && T <= 256,
              "swiglu_linear: needs T <= 256 and I % 128 == 0");
  if (T == 0) return;
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  GemmArgs a{};
  a.K = (int)K;
  a.groups = 1;
  a.ldc = (int)I;
  a.out_rows = (int)T;
  a.status = status_ptr(x.device().index());
  if (wait_flags && state && state->defined()) {  // wait for every rank's published shard
    TORCH_CHECK(nranks >= 1, "swiglu_linear: waiting on shard flags needs the rank count");
    a.tp.ag_flags = reinterpret_cast<const uint32_t*>(wait_flags);
    a.tp.epoch = reinterpret_cast<uint32_t*>(state->data_ptr<int>());
    a.tp.nranks = (int)nranks;
  }
  const int bn = pick_bn(T, true);
  auto ta = make_tmap_bf16(w.data_ptr(), w.size(0), K, K, 128);
  auto tb = make_tmap_bf16(x.data_ptr(), T, K, x.stride(0), bn);
  a.a_rows = (int)w.size(0);
  a.a_up_offset = (int)I;
  a.b_rows = (int)T;
  a.swap = 1;
  const int m_tiles = (int)(I / 128);
  const int kb = (int)((K + 63) / 64);
  int splits = 1;
  while (m_tiles * splits * 2 <= 2 * num_sms() && splits * 2 <= kb / 4 && splits * 2 <= (T >= 64 ? 4 : 8)) splits *= 2;
  if (!(workspace && workspace->defined() && workspace->numel() >= (int64_t)splits * T * 2 * I)) splits = 1;
  a.splits = splits;
  a.mode = splits > 1 ? kEpiPartialF32 : kEpiSwiGLU;
  a.out = splits > 1 ? workspace->data_ptr() : y.data_ptr();
  dispatch(bn, true, ta, tb, a, dim3(m_tiles, 1, splits), st);
  if (splits > 1) {
    const int64_t n = T * I;
    launch_k(splitk_swiglu_kernel, (unsigned)((n + 255) / 256), 256, 0, st, (const float*)workspace->data_ptr<float>(),
             splits, (int)T, (int)I, reinterpret_cast<__nv_bfloat16*>(y.data_ptr()));
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// y[T, N] = x[T, K] @ w[N, K]^T (+ residual).  `workspace` (fp32, may be
// empty) enables split-K for decode shapes that would otherwise leave SMs idle.
void linear(const at::Tensor& x, const at::Tensor& w, at::Tensor& y, const c10::optional<at::Tensor>& residual,
            const c10::optional<at::Tensor>& workspace, int64_t splits_req, int64_t orient) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && y.is_cuda());
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && y.scalar_type() == at::kBFloat16);
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.stride(1) == 1 && w.stride(1) == 1 && y.is_contiguous());
  const int64_t T = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K && y.size(0) == T && y.size(1) == N);
  TORCH_CHECK(K % 8 == 0, "K must be a multiple of 8");
  if (T == 0) return;
  const __nv_bfloat16* res = nullptr;
  if (residual && residual->defined()) {
    TORCH_CHECK(residual->is_contiguous() && residual->sizes() == y.sizes());
    res = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
  }
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  GemmArgs a{};
  a.K = (int)K;
  a.groups = 1;
  a.ldc = (int)N;
  a.out_rows = (int)T;
  a.status = status_ptr(x.device().index());
  a.residual = res;
  // orient: -1 automatic, 0 normal (activations on the 128-row side), 1 swap
  const bool swap = orient == 1 || (orient < 0 && T <= 256 && N % 128 == 0);
  TORCH_CHECK(!swap || (T <= 256 && N % 128 == 0), "swap orientation needs T <= 256 and N % 128 == 0");
  if (swap) {
    const int bn = pick_bn(T, false);
    auto ta = make_tmap_bf16(w.data_ptr(), N, K, w.stride(0), 128);
    auto tb = make_tmap_bf16(x.data_ptr(), T, K, x.stride(0), bn);
    a.a_rows = (int)N;
    a.b_rows = (int)T;
    a.swap = 1;
    const int m_tiles = (int)(N / 128);
    const int kb = (int)((K + 63) / 64);
    int splits = (int)splits_req;
    if (splits <= 0) {
      splits = 1;
      // two CTAs fit per SM: fill up to 2 x SMs so more weight bytes are in flight; past 4
      // splits (T >= 64) the fp32 partial traffic outweighs the extra parallelism
      // A GEMM of a few weight tiles (router-like) is pure latency: split it down to 2 K-blocks
      // per CTA; its partials stay small (m_tiles x 128 x T floats per split).
      const int cap = m_tiles <= 8 ? 16 : (T >= 64 ? 4 : 8);
      const int min_kb = m_tiles <= 8 ? 2 : 4;
      while (m_tiles * splits * 2 <= 2 * num_sms() && splits * 2 <= kb / min_kb && splits * 2 <= cap) splits *= 2;
    }
    bool use_ws = splits > 1 && workspace && workspace->defined() &&
                  workspace->numel() >= (int64_t)splits * T * N && (T * N) % 4 == 0;
    if (!use_ws) splits = 1;
    a.splits = splits;
    if (splits > 1) {
      a.mode = kEpiPartialF32;
      a.out = workspace->data_ptr();
      a.residual = nullptr;
    } else {
      a.mode = kEpiStore;
      a.out = y.data_ptr();
    }
    dispatch(bn, false, ta, tb, a, dim3(m_tiles, 1, splits), st);
    if (splits > 1) {
      int64_t n = T * N;
      int threads = 256;
      int64_t blocks = (n / 4 + threads - 1) / threads;
      launch_k(splitk_reduce_kernel, blocks, threads, 0, st, workspace->data_ptr<float>(), splits, n, res,
                                                     reinterpret_cast<__nv_bfloat16*>(y.data_ptr()));
      C10_CUDA_KERNEL_LAUNCH_CHECK();
    }
  } else {
    // Normal orientation: 128 activation rows x BN weight rows per tile.
    const int bn = N >= 256 ? 256 : pick_bn(N, false);
    auto ta = make_tmap_bf16(x.data_ptr(), T, K, x.stride(0), 128);
    auto tb = make_tmap_bf16(w.data_ptr(), N, K, w.stride(0), bn);
    a.a_rows = (int)((T + 127) / 128 * 128);
    a.b_rows = (int)N;
    a.swap = 0;
    a.splits = 1;
    a.mode = kEpiStore;
    a.out = y.data_ptr();
    const int m_tiles = (int)((T + 127) / 128);
    const int n_tiles = (int)((N + bn - 1) / bn);
    // Each CTA walks N tiles with stride gridDim.y; cap the grid near a few
    // waves so TMEM double-buffering overlaps epilogue and MMA.
    int ny = n_tiles;
    const int target = num_sms() * 2;
    while ((int64_t)m_tiles * ny > target && ny > 1) ny = (ny + 1) / 2;
    dispatch(bn, false, ta, tb, a, dim3(m_tiles, ny, 1), st);
  }
}

// Grouped (MoE) GEMM, swap orientation.  w: [G * rows_per_group, K] (experts
// stacked), x: [R, K] tokens sorted by group, offs: [G+1] int32 on device.
// SwiGLU mode: each group holds [gate; up] rows (2*I) and y gets I columns.
static void grouped_impl(const at::Tensor& x, const at::Tensor& w, const at::Tensor& offs, at::Tensor& y,
                         int64_t groups, bool swiglu, int64_t max_rows_per_group, int64_t wait_flags, int* epoch,
                         int nranks, int epoch_add) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && y.scalar_type() == at::kBFloat16);
  TORCH_CHECK(offs.scalar_type() == at::kInt && offs.numel() == groups + 1);
  TORCH_CHECK(x.is_contiguous() && w.is_contiguous() && y.is_contiguous());
  const int64_t R = x.size(0), K = x.size(1);
  const int64_t rows_pg = w.size(0) / groups;
  TORCH_CHECK(rows_pg * groups == w.size(0) && w.size(1) == K);
  const int64_t n_out = swiglu ? rows_pg / 2 : rows_pg;
  TORCH_CHECK(n_out % 128 == 0, "grouped GEMM needs output features % 128 == 0");
  TORCH_CHECK(y.size(0) == R && y.size(1) == n_out);
  if (R == 0) return;
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int bn = pick_bn(std::max<int64_t>(1, max_rows_per_group), swiglu);
  auto ta = make_tmap_bf16(w.data_ptr(), w.size(0), K, K, 128);
  auto tb = make_tmap_bf16(x.data_ptr(), R, K, K, bn);
  GemmArgs a{};
  a.K = (int)K;
  a.a_rows = (int)rows_pg;
  a.a_up_offset = swiglu ? (int)n_out : 0;
  a.b_offs = offs.data_ptr<int>();
  a.groups = (int)groups;
  a.splits = 1;
  a.swap = 1;
  a.mode = swiglu ? kEpiSwiGLU : kEpiStore;
  a.out = y.data_ptr();
  a.ldc = (int)n_out;
  a.out_rows = (int)R;
  a.status = status_ptr(x.device().index());
  if (wait_flags) {  // activations written by other GPUs: the producer waits on their flags first
    a.tp.ag_flags = reinterpret_cast<const uint32_t*>(wait_flags);
    a.tp.epoch = reinterpret_cast<uint32_t*>(epoch);
    a.tp.nranks = nranks;
    a.tp.epoch_add = epoch_add;
  }
  const int m_tiles = (int)(n_out / 128);
  // gridDim.y splits a group's token tiles across CTAs when groups are large.
  int ny = (int)std::max<int64_t>(1, std::min<int64_t>((max_rows_per_group + bn - 1) / bn, 8));
  if (persist_grouped()) {
    a.items = m_tiles * ny * (int)groups;
    a.m_tiles = m_tiles;
    a.ny = ny;
  }
  dispatch(bn, swiglu, ta, tb, a, dim3(m_tiles, ny, groups), st);
}

void grouped_linear(const at::Tensor& x, const at::Tensor& w, const at::Tensor& offs, at::Tensor& y,
                    int64_t groups, bool swiglu, int64_t max_rows_per_group) {
  grouped_impl(x, w, offs, y, groups, swiglu, max_rows_per_group, 0, nullptr, 0, 0);
}

// Grouped GEMM whose activation rows arrive from other GPUs: the TMA producer
// waits (bounded) until flags[p] >= state[0] + epoch_add for every p < nranks.
void grouped_linear_wait(const at::Tensor& x, const at::Tensor& w, const at::Tensor& offs, at::Tensor& y,
                         int64_t groups, bool swiglu, int64_t max_rows_per_group, int64_t flags, at::Tensor& state,
                         int64_t nranks, int64_t epoch_add) {
  TORCH_CHECK(state.scalar_type() == at::kInt && state.is_cuda());
  grouped_impl(x, w, offs, y, groups, swiglu, max_rows_per_group, flags, state.data_ptr<int>(), (int)nranks,
               (int)epoch_add);
}

}  // namespace mb

namespace mb {

// Tensor-parallel GEMM.
//   wait    : the activations x are this rank's gathered buffer, filled by the
//             peers' P2P pushes; the TMA producer waits (bounded) until every
//             rank's shard of the current epoch has arrived.
//   scatter : partial output rows go to their owners' reduce-scatter slots
//             (directly from the epilogue, or after a split-K reduction).
void tp_splitk_scatter(const at::Tensor& ws, int64_t splits, int64_t T, int64_t H, int64_t peer_rows,
                       const at::Tensor& peers, int64_t rank, int64_t rs_off, int64_t rs_flag_off, at::Tensor& state);

void tp_gemm(const at::Tensor& x, const at::Tensor& w, at::Tensor& out, bool wait, bool scatter, bool swiglu,
             int64_t ag_flags, at::Tensor& state, int64_t rank, int64_t nranks, int64_t peer_rows,
             const at::Tensor& rs_peers, int64_t rs_off, int64_t rs_flag_off, const c10::optional<at::Tensor>& workspace) {
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && w.is_contiguous() && x.scalar_type() == at::kBFloat16);
  const int64_t T = x.size(0), K = w.size(1);
  TORCH_CHECK(x.size(1) == K && x.stride(1) == 1);
  const int64_t n_out = swiglu ? w.size(0) / 2 : w.size(0);
  TORCH_CHECK(!(scatter && swiglu), "tp_gemm: scatter with swiglu is not supported");
  TORCH_CHECK(!scatter || T == peer_rows * nranks, "tp_gemm: scatter needs T == peer_rows * ranks");
  c10::cuda::CUDAGuard guard(w.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  GemmArgs a{};
  a.K = (int)K;
  a.groups = 1;
  a.ldc = (int)n_out;
  a.out_rows = (int)T;
  a.status = status_ptr(w.device().index());
  int* s = state.data_ptr<int>();
  a.tp.ag_flags = wait ? reinterpret_cast<const uint32_t*>(ag_flags) : nullptr;
  a.tp.epoch = reinterpret_cast<uint32_t*>(s);
  a.tp.done = s + 4;
  a.tp.peer_rows = (int)peer_rows;
  a.tp.nranks = (int)nranks;
  a.tp.rank = (int)rank;
  a.tp.rs_peers = rs_peers.numel() ? reinterpret_cast<const uint64_t*>(rs_peers.data_ptr<int64_t>()) : nullptr;
  a.tp.rs_off = rs_off;
  a.tp.rs_flag_off = rs_flag_off;
  const bool swap = T <= 256 && n_out % 128 == 0;
  if (swap) {
    const int bn = pick_bn(T, swiglu);
    auto ta = make_tmap_bf16(w.data_ptr(), w.size(0), K, K, 128);
    auto tb = make_tmap_bf16(x.data_ptr(), T, K, x.stride(0), bn);
    a.a_rows = (int)w.size(0);
    a.a_up_offset = swiglu ? (int)n_out : 0;
    a.b_rows = (int)T;
    a.swap = 1;
    const int m_tiles = (int)(n_out / 128);
    const int kb = (int)((K + 63) / 64);
    int splits = 1;
    if (!swiglu) {
      while (m_tiles * splits * 2 <= 2 * num_sms() && splits * 2 <= kb / 4 && splits * 2 <= (T >= 64 ? 4 : 8)) splits *= 2;
      if (!(workspace && workspace->defined() && workspace->numel() >= (int64_t)splits * T * n_out)) splits = 1;
    }
    a.splits = splits;
    if (splits > 1) {
      a.mode = kEpiPartialF32;
      a.out = workspace->data_ptr();
    } else if (scatter) {
      a.mode = kEpiScatterRS;
    } else {
      a.mode = swiglu ? kEpiSwiGLU : kEpiStore;
      a.out = out.data_ptr();
    }
    dispatch(bn, swiglu, ta, tb, a, dim3(m_tiles, 1, splits), st);
    if (splits > 1) {
      if (scatter) {
        tp_splitk_scatter(*workspace, splits, T, n_out, peer_rows, rs_peers, rank, rs_off, rs_flag_off, state);
      } else {
        const int64_t n = T * n_out;
        launch_k(splitk_reduce_kernel, (unsigned)((n / 4 + 255) / 256), 256, 0, st, (const float*)workspace->data_ptr<float>(),
                 splits, n, (const __nv_bfloat16*)nullptr, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
      }
    }
  } else {
    TORCH_CHECK(!swiglu, "tp_gemm: fused SwiGLU needs T <= 256");
    const int bn = n_out >= 256 ? 256 : pick_bn(n_out, false);
    auto ta = make_tmap_bf16(x.data_ptr(), T, K, x.stride(0), 128);
    auto tb = make_tmap_bf16(w.data_ptr(), w.size(0), K, K, bn);
    a.a_rows = (int)((T + 127) / 128 * 128);
    a.b_rows = (int)n_out;
    a.swap = 0;
    a.splits = 1;
    a.mode = scatter ? kEpiScatterRS : kEpiStore;
    a.out = scatter ? nullptr : out.data_ptr();
    const int m_tiles = (int)((T + 127) / 128);
    const int n_tiles = (int)((n_out + bn - 1) / bn);
    int ny = n_tiles;
    while ((int64_t)m_tiles * ny > num_sms() * 2 && ny > 1) ny = (ny + 1) / 2;
    dispatch(bn, false, ta, tb, a, dim3(m_tiles, ny, 1), st);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Non-owning bf16 [rows, cols] view of device memory (exchange buffers).
// int8 weight-only GEMM with per-row (output channel) scales:
//   y[t, n] = scale[n] * sum_k x[t, k] * wq[n, k]  (+ residual)
// Weights are the 128-row A operand (swap orientation) at every T; converter
// warps expand each int8 tile to bf16 in shared memory, so weight traffic is
// half of the bf16 GEMM's.  offs (int32 [groups+1]) selects grouped (MoE)
// mode; swiglu takes [2I, K] gate|up weights per group and writes silu(g)*u.
void linear_w8(const at::Tensor& x, const at::Tensor& wq, const at::Tensor& scale, at::Tensor& y,
               const c10::optional<at::Tensor>& residual, const c10::optional<at::Tensor>& workspace,
               const c10::optional<at::Tensor>& offs, int64_t groups, bool swiglu, int64_t max_rows_per_group) {
  TORCH_CHECK(x.is_cuda() && wq.is_cuda() && scale.is_cuda() && y.is_cuda());
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && wq.scalar_type() == at::kChar && scale.scalar_type() == at::kFloat &&
              y.scalar_type() == at::kBFloat16);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && wq.is_contiguous() && scale.is_contiguous() && y.is_contiguous());
  const bool grouped = offs && offs->defined();
  const int64_t T = x.size(0), K = x.size(1);
  TORCH_CHECK(wq.size(1) == K && K % 64 == 0, "linear_w8: K must be a multiple of 64");
  TORCH_CHECK(scale.numel() == wq.size(0), "linear_w8: one scale per weight row");
  if (!grouped) groups = 1;
  const int64_t rows_pg = wq.size(0) / groups;
  TORCH_CHECK(rows_pg * groups == wq.size(0));
  const int64_t n_out = swiglu ? rows_pg / 2 : rows_pg;
  TORCH_CHECK(n_out % 128 == 0, "linear_w8: output features must be a multiple of 128");
  TORCH_CHECK(y.size(0) == T && y.size(1) == n_out);
  if (T == 0) return;
  const __nv_bfloat16* res = nullptr;
  if (residual && residual->defined()) {
    TORCH_CHECK(!swiglu && residual->is_contiguous() && residual->sizes() == y.sizes());
    res = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
  }
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int64_t rows_hint = grouped ? std::max<int64_t>(1, max_rows_per_group) : T;
  const int bn = pick_bn(std::min<int64_t>(rows_hint, 256), swiglu);
  auto ta = make_tmap_2d(wq.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, wq.size(0), K, K, 64, 128,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
  auto tb = make_tmap_bf16(x.data_ptr(), T, K, x.stride(0), bn);
  GemmArgs a{};
  a.K = (int)K;
  a.a_rows = (int)rows_pg;
  a.a_up_offset = swiglu ? (int)n_out : 0;
  a.b_rows = (int)T;
  a.b_offs = grouped ? offs->data_ptr<int>() : nullptr;
  a.groups = (int)groups;
  a.swap = 1;
  a.ldc = (int)n_out;
  a.out_rows = (int)T;
  a.status = status_ptr(x.device().index());
  a.w_scale = scale.data_ptr<float>();
  a.residual = res;
  const int m_tiles = (int)(n_out / 128);
  const int n_tiles = (int)((rows_hint + bn - 1) / bn);
  int splits = 1;
  if (!grouped && T <= 256) {
    const int kb = (int)(K / 64);
    while (m_tiles * splits * 2 <= 2 * num_sms() && splits * 2 <= kb / 4 && splits * 2 <= (T >= 64 ? 4 : 8)) splits *= 2;
    const int64_t need = (int64_t)splits * T * n_out * (swiglu ? 2 : 1);
    if (!(workspace && workspace->defined() && workspace->numel() >= need && (T * n_out) % 4 == 0)) splits = 1;
  }
  a.splits = splits;
  if (splits > 1) {
    a.mode = kEpiPartialF32;
    a.out = workspace->data_ptr();
    a.residual = nullptr;
  } else {
    a.mode = swiglu ? kEpiSwiGLU : kEpiStore;
    a.out = y.data_ptr();
  }
  int ny;
  if (grouped) {
    ny = std::max(1, std::min(n_tiles, 8));
  } else {  // token tiles spread over CTAs, a couple of waves at most
    ny = n_tiles;
    while ((int64_t)m_tiles * ny > 2 * num_sms() && ny > 1) ny = (ny + 1) / 2;
  }
  dispatch_w8(bn, swiglu, ta, tb, a, dim3(m_tiles, ny, grouped ? groups : splits), st);
  if (splits > 1) {
    const int64_t n = T * n_out;
    if (swiglu) {
      launch_k(splitk_swiglu_kernel, (unsigned)((n + 255) / 256), 256, 0, st,
               (const float*)workspace->data_ptr<float>(), splits, (int)T, (int)n_out,
               reinterpret_cast<__nv_bfloat16*>(y.data_ptr()));
    } else {
      launch_k(splitk_reduce_kernel, (unsigned)((n / 4 + 255) / 256), 256, 0, st, workspace->data_ptr<float>(), splits,
               n, res, reinterpret_cast<__nv_bfloat16*>(y.data_ptr()));
    }
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

// Vision -> LLM exchange fused into the merger's last linear: out[r] = x[r] @ w^T + bias
// is stored straight into row row_map[r] % peer_rows of rank row_map[r] / peer_rows's
// buffer (peers[d] + off), P2P; the last CTA releases flags (peers[d] + flag_off)[rank] =
// state[0] + 1 at every rank.  Weights are the 128-row side, R visual rows the N side.
void vis_scatter_gemm(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& bias,
                      const at::Tensor& row_map, const at::Tensor& peers, int64_t rank, int64_t peer_rows,
                      int64_t off, int64_t flag_off, at::Tensor& state) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && x.is_contiguous() &&
              w.is_contiguous() && x.size(1) == w.size(1));
  TORCH_CHECK(row_map.scalar_type() == at::kInt && row_map.numel() == x.size(0));
  const int64_t R = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(N % 128 == 0 && K % 8 == 0 && R > 0, "vis_scatter_gemm: N % 128, K % 8, at least one row");
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int bn = pick_bn(std::min<int64_t>(R, 128), false);
  auto ta = make_tmap_bf16(w.data_ptr(), N, K, K, 128);
  auto tb = make_tmap_bf16(x.data_ptr(), R, K, K, bn);
  GemmArgs a{};
  a.K = (int)K;
  a.a_rows = (int)N;
  a.b_rows = (int)R;
  a.groups = 1;
  a.splits = 1;
  a.swap = 1;
  a.mode = kEpiScatterRows;
  a.ldc = (int)N;
  a.out_rows = (int)R;
  a.status = status_ptr(x.device().index());
  a.bias = (bias && bias->defined()) ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr;
  int* s = state.data_ptr<int>();
  a.tp.rs_peers = reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>());
  a.tp.rs_off = off;
  a.tp.rs_flag_off = flag_off;
  a.tp.peer_rows = (int)peer_rows;
  a.tp.nranks = (int)peers.numel();
  a.tp.rank = (int)rank;
  a.tp.epoch = reinterpret_cast<uint32_t*>(s);
  a.tp.epoch_add = 1;
  a.tp.done = s + 7;
  a.tp.row_map = row_map.data_ptr<int>();
  const int m_tiles = (int)(N / 128);
  int ny = (int)((R + bn - 1) / bn);
  while ((int64_t)m_tiles * ny > 2 * num_sms() && ny > 1) ny = (ny + 1) / 2;
  dispatch(bn, false, ta, tb, a, dim3(m_tiles, ny, 1), st);
}

at::Tensor wrap_bf16(int64_t addr, int64_t rows, int64_t cols) {
  return at::from_blob(reinterpret_cast<void*>(addr), {rows, cols},
                       at::TensorOptions().dtype(at::kBFloat16).device(at::kCUDA, c10::cuda::current_device()));
}

}  // namespace mb
