// Multi-tensor Adam / AdamW on the GPU: the counterpart of the reference's
// FusedAdam extension (optimizer/layer_adam/csrc/multi_tensor_adam.cu:33-203,
// fused_adam_frontend.cpp:8-25), which the reference builds but never calls.
//
// Same entry point and semantics: multi_tensor_adam(chunk_size, noop_flag,
// [grads, params, exp_avgs, exp_avg_sqs], lr, beta1, beta2, eps, step, mode,
// bias_correction, weight_decay); mode 0 = L2 (g += wd * p), mode 1 = AdamW
// (decoupled: p -= lr * (m_hat / (sqrt(v_hat) + eps) + wd * p)); all four
// tensors of one entry have one dtype (fp32, fp16, bf16 or fp64); fp32 math.
//
// Design (not the apex metadata scheme): one launch covers up to
// kMaxTensors tensors whose pointers, sizes and chunk prefix sums travel in
// the kernel's parameter space (CUDA 12 allows 32 KB of parameters, so no
// device-side table or per-launch host copy is needed).  The grid is
// persistent (a multiple of the SM count); each CTA takes chunks in
// grid-stride order and finds the owning tensor by binary search over the
// chunk prefix sums.  Tensors whose four pointers are 16-byte aligned use
// 16-byte vector loads and stores; others take a scalar path.  Indices are
// 64-bit throughout.
#include "common.cuh"

#include <cmath>
#include <vector>

namespace t1 {
namespace {

constexpr int kMaxTensors = 192;
constexpr int kThreads = 256;

struct AdamTable {
  void* g[kMaxTensors];
  void* p[kMaxTensors];
  void* m[kMaxTensors];
  void* v[kMaxTensors];
  int64_t n[kMaxTensors];
  int64_t chunk_start[kMaxTensors + 1];  // prefix sums of chunks per tensor
  uint8_t aligned[kMaxTensors];
  int count;
};
static_assert(sizeof(AdamTable) < 32000, "kernel parameter space is 32 KB");

struct AdamHyper {
  float lr, beta1, beta2, eps, wd, bc1, bc2;
  int mode;
  int64_t chunk;
};

template <typename T>
__device__ __forceinline__ float to_f(T x) {
  return static_cast<float>(x);
}
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}
template <>
__device__ __forceinline__ float to_f<__half>(__half x) {
  return __half2float(x);
}
template <typename T>
__device__ __forceinline__ T from_f(float x) {
  return static_cast<T>(x);
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <>
__device__ __forceinline__ __half from_f<__half>(float x) {
  return __float2half_rn(x);
}

__device__ __forceinline__ void adam_elem(float& p, float& m, float& v, float g, const AdamHyper& h) {
  if (h.mode == 0) {
    g = g + h.wd * p;
    m = h.beta1 * m + (1.f - h.beta1) * g;
    v = h.beta2 * v + (1.f - h.beta2) * g * g;
    float denom = sqrtf(v / h.bc2) + h.eps;
    p = p - h.lr * ((m / h.bc1) / denom);
  } else {
    m = h.beta1 * m + (1.f - h.beta1) * g;
    v = h.beta2 * v + (1.f - h.beta2) * g * g;
    float denom = sqrtf(v / h.bc2) + h.eps;
    p = p - h.lr * ((m / h.bc1) / denom + h.wd * p);
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) multi_tensor_adam_kernel(const __grid_constant__ AdamTable tab,
                                                                     const __grid_constant__ AdamHyper h) {
  constexpr int VEC = 16 / sizeof(T);
  const int64_t total = tab.chunk_start[tab.count];
  for (int64_t c = blockIdx.x; c < total; c += gridDim.x) {
    // tensor owning chunk c: last t with chunk_start[t] <= c
    int lo = 0, hi = tab.count - 1;
    while (lo < hi) {
      int mid = (lo + hi + 1) >> 1;
      if (tab.chunk_start[mid] <= c) lo = mid; else hi = mid - 1;
    }
    const int t = lo;
    const int64_t base = (c - tab.chunk_start[t]) * h.chunk;
    if (T1_OOB(base, tab.n[t])) continue;  // a chunk starts inside its tensor
    const int64_t end = min(tab.n[t], base + h.chunk);
    T* g = static_cast<T*>(tab.g[t]);
    T* p = static_cast<T*>(tab.p[t]);
    T* m = static_cast<T*>(tab.m[t]);
    T* v = static_cast<T*>(tab.v[t]);
    if (tab.aligned[t]) {
      // chunk sizes are multiples of VEC, so base is vector aligned
      const int64_t vend = base + (end - base) / VEC * VEC;
      for (int64_t i = base + (int64_t)threadIdx.x * VEC; i < vend; i += (int64_t)kThreads * VEC) {
        uint4 rg = *reinterpret_cast<const uint4*>(g + i);
        uint4 rp = *reinterpret_cast<const uint4*>(p + i);
        uint4 rm = *reinterpret_cast<const uint4*>(m + i);
        uint4 rv = *reinterpret_cast<const uint4*>(v + i);
        const T* eg = reinterpret_cast<const T*>(&rg);
        T* ep = reinterpret_cast<T*>(&rp);
        T* em = reinterpret_cast<T*>(&rm);
        T* ev = reinterpret_cast<T*>(&rv);
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
          float fp = to_f(ep[k]), fm = to_f(em[k]), fv = to_f(ev[k]);
          adam_elem(fp, fm, fv, to_f(eg[k]), h);
          ep[k] = from_f<T>(fp);
          em[k] = from_f<T>(fm);
          ev[k] = from_f<T>(fv);
        }
        *reinterpret_cast<uint4*>(p + i) = rp;
        *reinterpret_cast<uint4*>(m + i) = rm;
        *reinterpret_cast<uint4*>(v + i) = rv;
      }
      for (int64_t i = vend + threadIdx.x; i < end; i += kThreads) {
        float fp = to_f(p[i]), fm = to_f(m[i]), fv = to_f(v[i]);
        adam_elem(fp, fm, fv, to_f(g[i]), h);
        p[i] = from_f<T>(fp);
        m[i] = from_f<T>(fm);
        v[i] = from_f<T>(fv);
      }
    } else {
      for (int64_t i = base + threadIdx.x; i < end; i += kThreads) {
        float fp = to_f(p[i]), fm = to_f(m[i]), fv = to_f(v[i]);
        adam_elem(fp, fm, fv, to_f(g[i]), h);
        p[i] = from_f<T>(fp);
        m[i] = from_f<T>(fm);
        v[i] = from_f<T>(fv);
      }
    }
  }
}

template <typename T>
void launch_batch(const std::vector<std::vector<torch::Tensor>>& lists, size_t b0, size_t b1,
                  const AdamHyper& h) {
  AdamTable tab;
  tab.count = static_cast<int>(b1 - b0);
  int64_t chunks = 0;
  for (size_t k = b0; k < b1; ++k) {
    const int j = static_cast<int>(k - b0);
    tab.g[j] = lists[0][k].data_ptr();
    tab.p[j] = lists[1][k].data_ptr();
    tab.m[j] = lists[2][k].data_ptr();
    tab.v[j] = lists[3][k].data_ptr();
    tab.n[j] = lists[1][k].numel();
    tab.chunk_start[j] = chunks;
    chunks += (tab.n[j] + h.chunk - 1) / h.chunk;
    uintptr_t a = reinterpret_cast<uintptr_t>(tab.g[j]) | reinterpret_cast<uintptr_t>(tab.p[j]) |
                  reinterpret_cast<uintptr_t>(tab.m[j]) | reinterpret_cast<uintptr_t>(tab.v[j]);
    tab.aligned[j] = (a % 16) == 0;
  }
  tab.chunk_start[tab.count] = chunks;
  if (chunks == 0) return;
  const int64_t grid = std::min<int64_t>(chunks, (int64_t)num_sms() * 8);
  multi_tensor_adam_kernel<T><<<(unsigned)grid, kThreads, 0, stream()>>>(tab, h);
  count_launch();
  check_launch("multi_tensor_adam");
}

}  // namespace

T1_BOUNDS_READER(fused_adam)

void multi_tensor_adam(int64_t chunk_size, torch::Tensor noop_flag,
                       std::vector<std::vector<torch::Tensor>> tensor_lists, double lr, double beta1,
                       double beta2, double eps, int64_t step, int64_t mode, int64_t bias_correction,
                       double weight_decay) {
  (void)noop_flag;  // as in the reference, inf/nan propagate (no early exit)
  TORCH_CHECK(tensor_lists.size() == 4, "tensor_lists must be [grads, params, exp_avgs, exp_avg_sqs]");
  const size_t n = tensor_lists[0].size();
  for (auto& l : tensor_lists) TORCH_CHECK(l.size() == n, "tensor lists differ in length");
  if (n == 0) return;
  TORCH_CHECK(mode == 0 || mode == 1, "mode must be 0 (L2) or 1 (AdamW)");
  const auto dt = tensor_lists[1][0].scalar_type();
  for (size_t k = 0; k < n; ++k) {
    for (int l = 0; l < 4; ++l) {
      const auto& t = tensor_lists[l][k];
      TORCH_CHECK(t.is_cuda() && t.is_contiguous(), "tensors must be contiguous CUDA tensors");
      TORCH_CHECK(t.scalar_type() == dt, "all tensors must share one dtype");
      TORCH_CHECK(t.numel() == tensor_lists[1][k].numel(), "grad/param/state sizes differ");
    }
  }
  const at::cuda::CUDAGuard guard(tensor_lists[1][0].device());
  AdamHyper h;
  h.lr = (float)lr;
  h.beta1 = (float)beta1;
  h.beta2 = (float)beta2;
  h.eps = (float)eps;
  h.wd = (float)weight_decay;
  h.mode = (int)mode;
  float bc1 = 1.f, bc2 = 1.f;
  if (bias_correction == 1) {
    bc1 = 1.f - (float)std::pow(beta1, (double)step);
    bc2 = 1.f - (float)std::pow(beta2, (double)step);
  }
  h.bc1 = bc1;
  h.bc2 = bc2;
  // chunks are a multiple of one 16-byte vector of the narrowest type
  h.chunk = std::max<int64_t>(8, (chunk_size + 7) / 8 * 8);
  for (size_t b0 = 0; b0 < n; b0 += kMaxTensors) {
    const size_t b1 = std::min(n, b0 + kMaxTensors);
    switch (dt) {
      case at::kFloat: launch_batch<float>(tensor_lists, b0, b1, h); break;
      case at::kBFloat16: launch_batch<__nv_bfloat16>(tensor_lists, b0, b1, h); break;
      case at::kHalf: launch_batch<__half>(tensor_lists, b0, b1, h); break;
      case at::kDouble: launch_batch<double>(tensor_lists, b0, b1, h); break;
      default: TORCH_CHECK(false, "multi_tensor_adam: unsupported dtype ", dt);
    }
  }
}

}  // namespace t1
