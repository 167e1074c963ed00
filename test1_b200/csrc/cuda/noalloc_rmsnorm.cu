// t1_rmsnorm_bwd_noalloc -- an RMSNorm backward that allocates nothing.
//
// This entry point has no counterpart in the reference.  It exists for
// callers that cannot allocate device memory: code running inside a custom
// memory arena or a framework that owns every device allocation (where a
// stray cudaMalloc would bypass its accounting or fail outright), real-time
// or embedded loops that forbid allocation after start-up, and plain C/C++
// programs that link this library without PyTorch's caching allocator.  The
// regular `rmsnorm_bwd` binding asks PyTorch for its dx/dw outputs and for a
// partial-sum workspace on every call; this variant takes the outputs from
// the caller and keeps its workspace in a fixed file-scope device array.
//
// The prototype, return codes and limits are declared in t1_noalloc.h (the
// compiler checks this definition against it).
//
// Limits: H must be a positive multiple of 8 and at most 8192; T >= 0.
// The scratch array holds kScratchFloats = 524288 floats (2 MiB).  It is part
// of the module image, so every GPU that loads this library keeps those 2 MiB
// until the process exits.  The number of row groups is chosen so that
// groups * H always fits the array; larger H is rejected.
//
// Return value: 0 on success; 1 if an argument is invalid (null pointer,
// T < 0, H not a multiple of 8, or H <= 0); 2 if H exceeds 8192 (the
// scratch maximum); 3 if the scratch array's device address could not be
// obtained; 4 if a CUDA error from earlier, unrelated work was already
// pending on entry (nothing is launched and that error is left for its owner
// to see); otherwise 1000 + the cudaError_t of the failed launch.
//
// Set-up: the first call on each device looks up the scratch array's device
// address with cudaGetSymbolAddress (with that device current) and caches
// it.  Make that first call before any stream capture begins.
//
// Sharing: every call on a device uses the same scratch array, and the array
// keeps whatever the last call wrote.  Nothing in it needs to start at zero:
// each call writes every scratch entry it later reads.  Calls whose GPU work
// overlaps (different streams, or different host threads without ordering)
// race on the scratch array and can produce wrong dw; serialise them.
//
// The function calls no cudaMalloc, no cudaFree and no allocating library
// routine.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "bounds.cuh"
#include "t1_noalloc.h"

namespace t1 {
namespace noalloc {

using bf16 = __nv_bfloat16;

constexpr int kScratchFloats = 1 << 19;  // 2 MiB
constexpr int kMaxH = T1_NOALLOC_MAX_H;
constexpr int kThreads = 256;
constexpr int kMaxDevices = 64;

// File-scope scratch: per-row-group partial sums of dw, [groups, H] fp32.
static __device__ __align__(256) float g_scratch[kScratchFloats];

struct __align__(16) Vec8 {
  __nv_bfloat162 h[4];
};

__device__ __forceinline__ void ld8(const bf16* p, float (&f)[8]) {
  Vec8 v = *reinterpret_cast<const Vec8*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(v.h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ void st8(bf16* p, const float (&f)[8]) {
  Vec8 v;
#pragma unroll
  for (int i = 0; i < 4; ++i) v.h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  *reinterpret_cast<Vec8*>(p) = v;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = lane < (kThreads >> 5) ? red[lane] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return t;
}

// One CTA per group of `rows` consecutive rows; column partials of dw go to
// part[group, :] (every column of the group's row is written).
template <int VPT>
__global__ void __launch_bounds__(kThreads) rows_kernel(const bf16* __restrict__ dy,
                                                        const bf16* __restrict__ x,
                                                        const bf16* __restrict__ w,
                                                        const float* __restrict__ rstd,
                                                        const bf16* __restrict__ resid,
                                                        bf16* __restrict__ dx,
                                                        float* __restrict__ part, int T, int H,
                                                        int rows) {
  __shared__ float red[32];
  const int nvec = H >> 3;
  float wv[VPT][8], acc[VPT][8];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int i = threadIdx.x + k * kThreads;
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[k][j] = 0.f;
    if (i < nvec) ld8(w + 8 * i, wv[k]);
  }
  const int r0 = blockIdx.x * rows;
  const int r1 = min(T, r0 + rows);
  for (int row = r0; row < r1; ++row) {
    const float r = rstd[row];
    float xh[VPT][8], dxh[VPT][8];
    float dot = 0.f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int i = threadIdx.x + k * kThreads;
      if (i < nvec) {
        float xv[8], dv[8];
        ld8(x + static_cast<size_t>(row) * H + 8 * i, xv);
        ld8(dy + static_cast<size_t>(row) * H + 8 * i, dv);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          xh[k][j] = xv[j] * r;
          dxh[k][j] = dv[j] * wv[k][j];
          dot += dxh[k][j] * xh[k][j];
          acc[k][j] += dv[j] * xh[k][j];
        }
      }
    }
    dot = block_sum(dot, red);
    const float c = dot / static_cast<float>(H);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int i = threadIdx.x + k * kThreads;
      if (i < nvec) {
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = r * (dxh[k][j] - xh[k][j] * c);
        if (resid != nullptr) {
          float rv[8];
          ld8(resid + static_cast<size_t>(row) * H + 8 * i, rv);
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] += rv[j];
        }
        st8(dx + static_cast<size_t>(row) * H + 8 * i, o);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int i = threadIdx.x + k * kThreads;
    if (i < nvec && !T1_OOB(static_cast<long long>(blockIdx.x) * H + 8 * i + 7, kScratchFloats)) {
      float* dst = part + static_cast<size_t>(blockIdx.x) * H + 8 * i;
#pragma unroll
      for (int j = 0; j < 8; ++j) dst[j] = acc[k][j];
    }
  }
}

// dw[c] = sum over groups of part[g, c], fixed order.
__global__ void reduce_kernel(const float* __restrict__ part, int groups, int H,
                              bf16* __restrict__ dw) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= H) return;
  float s = 0.f;
  for (int g = 0; g < groups; ++g) s += part[static_cast<size_t>(g) * H + c];
  dw[c] = __float2bfloat16_rn(s);
}

static std::mutex g_mu;
static float* g_scratch_addr[kMaxDevices] = {nullptr};

// Device address of g_scratch for the current device (looked up once).
static float* scratch_for_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_scratch) != cudaSuccess || p == nullptr) return nullptr;
    g_scratch_addr[dev] = static_cast<float*>(p);
  }
  return g_scratch_addr[dev];
}

}  // namespace noalloc

T1_BOUNDS_READER(noalloc_rmsnorm)

}  // namespace t1

extern "C" int t1_rmsnorm_bwd_noalloc(const __nv_bfloat16* dy, const __nv_bfloat16* x,
                                      const __nv_bfloat16* w, const float* rstd,
                                      const __nv_bfloat16* residual_grad, __nv_bfloat16* dx,
                                      __nv_bfloat16* dw, int T, int H, cudaStream_t stream) {
  using namespace t1::noalloc;
  if (dy == nullptr || x == nullptr || w == nullptr || rstd == nullptr || dx == nullptr ||
      dw == nullptr || T < 0 || H <= 0 || H % 8 != 0)
    return T1_NOALLOC_BAD_ARGUMENT;
  if (H > kMaxH) return T1_NOALLOC_TOO_LARGE;
  // an error left by earlier work would otherwise be reported (and cleared)
  // as a failure of these launches
  if (cudaPeekAtLastError() != cudaSuccess) return T1_NOALLOC_PENDING_ERROR;
  float* scratch = scratch_for_current_device();
  if (scratch == nullptr) return T1_NOALLOC_NO_SCRATCH;
  const int max_groups = kScratchFloats / H;  // >= 64 since H <= 8192
  int groups = 0;
  if (T > 0) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    groups = 2 * sms;
    if (groups > max_groups) groups = max_groups;
    if (groups > T) groups = T;
    const int rows = (T + groups - 1) / groups;
    groups = (T + rows - 1) / rows;
    const int vpt = (H / 8 + kThreads - 1) / kThreads;
    switch (vpt) {
      case 1: rows_kernel<1><<<groups, kThreads, 0, stream>>>(dy, x, w, rstd, residual_grad, dx, scratch, T, H, rows); break;
      case 2: rows_kernel<2><<<groups, kThreads, 0, stream>>>(dy, x, w, rstd, residual_grad, dx, scratch, T, H, rows); break;
      default: rows_kernel<4><<<groups, kThreads, 0, stream>>>(dy, x, w, rstd, residual_grad, dx, scratch, T, H, rows); break;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return T1_NOALLOC_LAUNCH_ERROR + static_cast<int>(e);
    reduce_kernel<<<(H + 255) / 256, 256, 0, stream>>>(scratch, groups, H, dw);
  } else {
    // no rows: dw is the empty sum
    reduce_kernel<<<(H + 255) / 256, 256, 0, stream>>>(scratch, 0, H, dw);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? T1_NOALLOC_OK : T1_NOALLOC_LAUNCH_ERROR + static_cast<int>(e);
}
