// NVLS flavour of the tensor-parallel layer boundary: the reduce-scatter is
// done by the NVSwitch (multimem.ld_reduce) and the all-gather by multicast
// stores (multimem.st), both issued from inside one kernel.
//
// Every rank owns one symmetric buffer (same layout on every rank) that is
// also bound to an NVLink multicast object; `mc` is the multicast address of
// its base, `self` the unicast address of this rank's copy:
//   gathered [N*rows, H] bf16   every rank's normed shard (written by multicast stores)
//   part     [N*rows, H] bf16   this rank's full row-parallel GEMM output (a local GEMM writes it)
//   ag_flags [N] u32            ag_flags[p] = epoch once rank p's shard is in every replica
//   rs_flags [N] u32            rs_flags[p] = epoch once rank p's `part` is complete
// A boundary with partials, on rank r (CTA per owned row t):
//   1. CTA 0 announces that this rank's GEMM output is complete: one
//      multimem.st.release of rs_flags[r] reaches every rank.
//   2. bounded wait until every rank's rs flag carries this boundary's epoch.
//   3. multimem.ld_reduce of row r*rows + t of `part`: the switch returns the
//      sum over the ranks (fp32 accumulation of bf16 pairs), 16 bytes a thread.
//   4. + residual (+ x_add), RMSNorm, residual stored locally.
//   5. multimem.st of the normed row into `gathered` row r*rows + t: one store
//      reaches every replica, so each byte leaves the GPU once.
//   6. the last CTA publishes ag_flags[r] = epoch with one multicast release.
// The column-parallel GEMMs that follow read `gathered` locally after the
// same flag wait as the P2P flavour (tp.cu), so they need no change.
//
// `part` can be overwritten by the next boundary's GEMM only after this rank
// passed the next all-gather wait, which needs every owner's ag flag, which
// each owner releases after its CTAs finished reading `part`.
//
// No TMA or bulk copy touches the multicast range: the multicast object is
// reached only by multimem.* instructions issued by threads.
#include <cuda.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "launch.cuh"
#include "multimem.cuh"
#include "status.h"

namespace mb {

// row_stride: rows between two ranks' blocks in part / gathered (the TP layout packs them, stride = rows; the
// expert-parallel layout keeps a fixed per-rank capacity).  publish = 0: the normed row stays local (local_out)
// and no all-gather flag is released.  rows == 0 launches one CTA that only announces and waits, so the peers'
// waits are met.
__global__ void __launch_bounds__(1024)
    tp_nvls_reduce_kernel(uint64_t self, uint64_t mc, int rank, int nranks, int with_partials, int rows,
                          int row_stride, int publish, int H, int64_t ag_off, int64_t part_off, int64_t ag_flag_off, int64_t rs_flag_off, uint32_t* epoch,
                          int* done, const __nv_bfloat16* __restrict__ x_add, __nv_bfloat16* __restrict__ residual,
                          const __nv_bfloat16* __restrict__ w, float eps, __nv_bfloat16* __restrict__ local_out,
                          int* status) {
  pdl_wait();  // this rank's GEMM output (part) and the residual are complete
  pdl_trigger();
  const uint32_t e = *epoch, ne = e + 1;
  const int t = blockIdx.x, tid = threadIdx.x;
  const int col = tid * 8;
  __shared__ float red[32];
  __shared__ int ok_all, last;
  if (tid == 0) ok_all = 1;
  if (with_partials) {
    if (t == 0 && tid == 0) {
      __threadfence_system();
      mc_store_release_u32(mc + rs_flag_off + 4ull * rank, ne);
    }
    __syncthreads();
    const uint32_t* rf = reinterpret_cast<const uint32_t*>(self + rs_flag_off);
    for (int p = tid; p < nranks; p += blockDim.x) {
      const uint64_t t0 = globaltimer_ns();
      while ((int32_t)(ld_acquire_sys_u32(rf + p) - ne) < 0) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          set_status(status, kErrPeerTimeout);
          ok_all = 0;
          break;
        }
      }
    }
    __syncthreads();
    __threadfence_system();
  } else {
    __syncthreads();
  }
  if (t < rows) {
  const size_t off = (size_t)t * H + col;
  const size_t grow = (size_t)rank * row_stride + t;  // this row's index in part / gathered
  uint4 sum = make_uint4(0, 0, 0, 0);
  if (with_partials && ok_all) sum = mc_ld_reduce_bf16x8(mc + part_off + (grow * H + col) * 2);
  const uint4 rr = *reinterpret_cast<const uint4*>(residual + off);
  const uint4 xa = x_add ? *reinterpret_cast<const uint4*>(x_add + off) : make_uint4(0, 0, 0, 0);
  const uint4 wr = *reinterpret_cast<const uint4*>(w + col);
  __align__(16) __nv_bfloat16 hb[8];
  float v[8], ss = 0.f;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    float a = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(&rr)[q]);
    if (x_add) a += __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(&xa)[q]);
    a += __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(&sum)[q]);
    hb[q] = __float2bfloat16(a);
    v[q] = __bfloat162float(hb[q]);
    ss += v[q] * v[q];
  }
  *reinterpret_cast<uint4*>(residual + off) = *reinterpret_cast<const uint4*>(hb);
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
  const float inv = rsqrtf(tot / H + eps);
  __align__(16) __nv_bfloat16 o[8];
#pragma unroll
  for (int q = 0; q < 8; ++q)
    o[q] = __float2bfloat16(v[q] * inv * __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(&wr)[q]));
  if (publish) mc_store_16(mc + ag_off + (grow * H + col) * 2, *reinterpret_cast<const uint4*>(o));
  if (local_out) *reinterpret_cast<uint4*>(local_out + off) = *reinterpret_cast<const uint4*>(o);
  }
  // CTA barrier, one system-scope fence + arrive per CTA; the last CTA publishes
  __syncthreads();
  if (tid == 0) {
    __threadfence_system();
    last = atomicAdd(done, 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  if (tid == 0) {
    __threadfence_system();
    if (publish) mc_store_release_u32(mc + ag_flag_off + 4ull * rank, ne);
    *epoch = ne;
    *done = 0;
  }
}

void tp_nvls_reduce(int64_t self, int64_t mc, int64_t rank, int64_t nranks, bool with_partials, int64_t rows,
                    int64_t row_stride, bool publish, int64_t H, int64_t ag_off, int64_t part_off, int64_t ag_flag_off, int64_t rs_flag_off,
                    at::Tensor& state, const c10::optional<at::Tensor>& x_add, at::Tensor& residual,
                    const at::Tensor& w, double eps, const c10::optional<at::Tensor>& local_out) {
  TORCH_CHECK(H % 256 == 0 && H / 8 <= 1024, "tp_nvls_reduce: hidden size must be a multiple of 256 (<= 8192)");
  TORCH_CHECK(residual.scalar_type() == at::kBFloat16 && residual.is_contiguous() && residual.size(0) == rows &&
              residual.size(1) == H);
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && w.is_contiguous() && w.numel() == H);
  TORCH_CHECK(mc != 0 && self != 0, "tp_nvls_reduce: no multicast mapping");
  TORCH_CHECK(ag_off % 16 == 0 && part_off % 16 == 0 && ag_flag_off % 4 == 0 && rs_flag_off % 4 == 0,
              "tp_nvls_reduce: misaligned offsets");
  TORCH_CHECK(state.scalar_type() == at::kInt && state.numel() >= 8);
  c10::cuda::CUDAGuard guard(residual.device());
  auto bf = [](const c10::optional<at::Tensor>& t) -> __nv_bfloat16* {
    if (!(t && t->defined())) return nullptr;
    TORCH_CHECK(t->scalar_type() == at::kBFloat16 && t->is_contiguous());
    return reinterpret_cast<__nv_bfloat16*>(t->data_ptr());
  };
  if (row_stride <= 0) row_stride = rows;
  TORCH_CHECK(rows <= row_stride, "tp_nvls_reduce: ", rows, " rows exceed the per-rank stride ", row_stride);
  TORCH_CHECK((local_out && local_out->defined()) || publish, "tp_nvls_reduce: the normed rows must go somewhere");
  if (rows == 0 && !with_partials) return;  // nothing to publish and nothing to announce
  int* s = state.data_ptr<int>();
  launch_k(tp_nvls_reduce_kernel, (int)std::max<int64_t>(rows, 1), (int)(H / 8), 0, at::cuda::getCurrentCUDAStream(),
           (uint64_t)self, (uint64_t)mc, (int)rank, (int)nranks, with_partials ? 1 : 0, (int)rows, (int)row_stride,
           publish ? 1 : 0, (int)H, ag_off, part_off,
           ag_flag_off, rs_flag_off, reinterpret_cast<uint32_t*>(s), s + 5, (const __nv_bfloat16*)bf(x_add),
           reinterpret_cast<__nv_bfloat16*>(residual.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
           (float)eps, bf(local_out), status_ptr(residual.device().index()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED of a device (switch multicast and
// in-switch reduction), read through the driver entry point.
bool multicast_supported(int64_t device) {
  using GetAttr = CUresult (*)(int*, CUdevice_attribute, CUdevice);
  static GetAttr fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuDeviceGetAttribute", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !p)
      return false;
    fn = reinterpret_cast<GetAttr>(p);
  }
  int v = 0;
  if (fn(&v, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, (CUdevice)device) != CUDA_SUCCESS) return false;
  return v != 0;
}

}  // namespace mb
