// Fused NVLink collectives of the sliding engine (sm_100a, one process per
// GPU, buffers in symmetric memory mapped into every peer).
//
//  * fused_rs_d2h: the gpu_reduce path.  Rank r reads its shard
//    [offset, offset + n) of the layer gradient from every peer's pool unit
//    (P2P loads over NVLink), sums in fp32, multiplies by `scale` (1/N),
//    rounds to bf16 and stores straight into its page-locked host gradient
//    shard (zero-copy, mapped memory).  One kernel replaces NCCL
//    reduce_scatter + a device-to-host copy.
//
//  * fused_shard_gather: the shard path.  Rank r reads its shard of the
//    layer and stores it into every peer's pool unit at the shard offset
//    (P2P stores over NVLink).  The source is either page-locked host memory
//    read zero-copy (fp32 master, cast to bf16 here, or the bf16 shadow) --
//    one kernel instead of a host-to-device copy + NCCL all_gather (+ the
//    cast) -- or, in the staged form, the shard already copied into this
//    rank's own unit by the copy engine: the kernel is then the NVLink
//    broadcast alone, runs on a few CTAs next to the compute kernels, and
//    skips the store onto itself.
//
// Cross-GPU ordering uses per-buffer signal pads (uint32 slots in each
// rank's pad, written by peers with release stores at system scope, read
// with acquire loads).  Slot layout: [0, W) "ready/free" from peer p,
// [W, 2W) "done" from peer p.  Values are monotonically increasing epochs
// (one per launch on that buffer, identical on all ranks), so pads never
// need resetting.  Every wait is bounded (%globaltimer, 4 s); on expiry the
// kernel writes an error code and returns without touching more data.
#include "common.cuh"
#include "sm100.cuh"

namespace t1 {
namespace fused {

using bf16 = __nv_bfloat16;
constexpr int kMaxRanks = 8;

struct Peers {
  uint64_t ptr[kMaxRanks];  // base address of the symmetric buffer on each rank
  uint64_t sig[kMaxRanks];  // signal pad base on each rank
  uint64_t wait_ns;         // limit of every wait on a peer
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Wait until pad[slot0 + p] >= epoch for every p < world.  Thread-local.
__device__ __forceinline__ bool wait_all(const uint32_t* pad, int slot0, int world, uint32_t epoch,
                                         uint64_t wait_ns) {
  const uint64_t t0 = sm100::globaltimer_ns();
  for (int p = 0; p < world; ++p) {
    uint32_t n = 0;
    while (ld_acquire_sys(pad + slot0 + p) < epoch) {
      if ((++n & 255u) == 0 && sm100::globaltimer_ns() - t0 > wait_ns) return false;
    }
  }
  return true;
}

__device__ __forceinline__ void signal_all(const Peers& pe, int slot, int world, uint32_t epoch) {
  for (int p = 0; p < world; ++p)
    st_release_sys(reinterpret_cast<uint32_t*>(pe.sig[p]) + slot, epoch);
}

// Block-wide "all peers reached slot0 phase" barrier entry; returns false
// (for every thread) when the wait expired.
__device__ __forceinline__ bool block_wait(const uint32_t* my_pad, int slot0, int world,
                                           uint32_t epoch, uint64_t wait_ns, int* err, int code) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = wait_all(my_pad, slot0, world, epoch, wait_ns) ? 1 : 0;
    if (!ok && err) atomicCAS(err, 0, code);
    __threadfence_system();
  }
  __syncthreads();
  return ok != 0;
}

// The last CTA to finish signals `slot` (done) to every peer and waits for
// theirs; `counter` is a device-local int reset by that CTA.
__device__ __forceinline__ void finish(const Peers& pe, int rank, int world, uint32_t epoch,
                                       int* counter, int* err, int code) {
  __threadfence_system();  // every thread's peer / host stores are visible system-wide
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(counter, 1);
    if (prev == static_cast<int>(gridDim.x) - 1) {
      signal_all(pe, world + rank, world, epoch);
      const uint32_t* my_pad = reinterpret_cast<const uint32_t*>(pe.sig[rank]);
      if (!wait_all(my_pad, world, world, epoch, pe.wait_ns) && err) atomicCAS(err, 0, code);
      atomicExch(counter, 0);
    }
  }
}

// ---------------------------------------------------------- reduce-scatter
__global__ void __launch_bounds__(256) rs_d2h_kernel(Peers pe, int rank, int world, long offset,
                                                     long n, bf16* __restrict__ host_out,
                                                     float scale, uint32_t epoch, int* counter,
                                                     int* err) {
  if (blockIdx.x == 0 && threadIdx.x == 0) signal_all(pe, rank, world, epoch);  // my grads ready
  const uint32_t* my_pad = reinterpret_cast<const uint32_t*>(pe.sig[rank]);
  if (!block_wait(my_pad, 0, world, epoch, pe.wait_ns, err, 201)) return;
  const long n8 = n >> 3;
  const long stride = static_cast<long>(gridDim.x) * blockDim.x;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8; i += stride) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll 1
    for (int p = 0; p < world; ++p) {
      const bf16* src = reinterpret_cast<const bf16*>(pe.ptr[p]) + offset + 8 * i;
      int4 raw = __ldcg(reinterpret_cast<const int4*>(src));
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float2 f = __bfloat1622float2(h[k]);
        acc[2 * k] += f.x;
        acc[2 * k + 1] += f.y;
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] *= scale;
    store8(host_out + 8 * i, acc);
  }
  // tail (n % 8) by block 0
  if (blockIdx.x == 0) {
    for (long j = (n8 << 3) + threadIdx.x; j < n; j += blockDim.x) {
      float s = 0.f;
      for (int p = 0; p < world; ++p)
        s += __bfloat162float(reinterpret_cast<const bf16*>(pe.ptr[p])[offset + j]);
      host_out[j] = __float2bfloat16_rn(s * scale);
    }
  }
  finish(pe, rank, world, epoch, counter, err, 202);
}

// ------------------------------------------------------------ shard gather
// Source kinds: 0 = bf16 copy, 1 = fp32 master, 2 = split fp32 master (a
// bf16-rounded high plane and a 16-bit low plane, value =
// ((hi << 16) | lo) - 0x8000).  Kinds 1 and 2 are cast to bf16 (nearest
// even) here.
enum SrcKind : int { kSrcBf16 = 0, kSrcF32 = 1, kSrcSplit = 2 };

__device__ __forceinline__ int4 load8_as_bf16(int kind, const void* src, const void* src_lo, long e) {
  int4 out;
  if (kind == kSrcBf16) {
    out = *reinterpret_cast<const int4*>(static_cast<const bf16*>(src) + e);
    return out;
  }
  float f[8];
  if (kind == kSrcF32) {
    const float4* s = reinterpret_cast<const float4*>(static_cast<const float*>(src) + e);
    float4 a = s[0], b = s[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
    int4 hv = *reinterpret_cast<const int4*>(static_cast<const uint16_t*>(src) + e);
    int4 lv = *reinterpret_cast<const int4*>(static_cast<const uint16_t*>(src_lo) + e);
    const uint16_t* h = reinterpret_cast<const uint16_t*>(&hv);
    const uint16_t* l = reinterpret_cast<const uint16_t*>(&lv);
#pragma unroll
    for (int k = 0; k < 8; ++k)
      f[k] = __uint_as_float(((static_cast<uint32_t>(h[k]) << 16) | l[k]) - 0x8000u);
  }
  __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
  for (int k = 0; k < 4; ++k) o[k] = __floats2bfloat162_rn(f[2 * k], f[2 * k + 1]);
  return out;
}

__device__ __forceinline__ bf16 load1_as_bf16(int kind, const void* src, const void* src_lo, long e) {
  if (kind == kSrcBf16) return static_cast<const bf16*>(src)[e];
  if (kind == kSrcF32) return __float2bfloat16_rn(static_cast<const float*>(src)[e]);
  const uint32_t b = ((static_cast<uint32_t>(static_cast<const uint16_t*>(src)[e]) << 16) |
                      static_cast<const uint16_t*>(src_lo)[e]) - 0x8000u;
  return __float2bfloat16_rn(__uint_as_float(b));
}

__global__ void __launch_bounds__(256) shard_gather_kernel(Peers pe, int rank, int world, long offset,
                                                           long n, int kind, const void* __restrict__ host_src,
                                                           const void* __restrict__ host_src_lo,
                                                           int skip_self, uint32_t epoch, int* counter,
                                                           int* err) {
  // my unit is free (stream order): announce it, wait until every peer's is
  if (blockIdx.x == 0 && threadIdx.x == 0) signal_all(pe, rank, world, epoch);
  const uint32_t* my_pad = reinterpret_cast<const uint32_t*>(pe.sig[rank]);
  if (!block_wait(my_pad, 0, world, epoch, pe.wait_ns, err, 211)) return;
  const long n8 = n >> 3;
  const long stride = static_cast<long>(gridDim.x) * blockDim.x;
  // kU vectors per thread in flight: the loads (local HBM or PCIe) are
  // issued together before the peer stores, so latency overlaps
  constexpr int kU = 4;
  for (long i0 = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i0 < n8; i0 += kU * stride) {
    int4 out[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u)
      if (i0 + u * stride < n8) out[u] = load8_as_bf16(kind, host_src, host_src_lo, 8 * (i0 + u * stride));
#pragma unroll 1
    for (int p = 0; p < world; ++p) {
      if (skip_self && p == rank) continue;  // the source already is this rank's unit
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const long i = i0 + u * stride;
        if (i < n8) *reinterpret_cast<int4*>(reinterpret_cast<bf16*>(pe.ptr[p]) + offset + 8 * i) = out[u];
      }
    }
  }
  if (blockIdx.x == 0) {
    for (long j = (n8 << 3) + threadIdx.x; j < n; j += blockDim.x) {
      const bf16 v = load1_as_bf16(kind, host_src, host_src_lo, j);
      for (int p = 0; p < world; ++p)
        if (!(skip_self && p == rank)) reinterpret_cast<bf16*>(pe.ptr[p])[offset + j] = v;
    }
  }
  finish(pe, rank, world, epoch, counter, err, 212);
}

}  // namespace fused

// ================================================================ host side
T1_BOUNDS_READER(fused_comm)

// Limit of the fused kernels' waits on peer GPUs (T1_PEER_WAIT_S or
// fused_set_peer_wait; default 60 s).
static uint64_t& peer_wait_ns() {
  static uint64_t v = [] {
    const char* e = std::getenv("T1_PEER_WAIT_S");
    const double s = e != nullptr ? std::atof(e) : 0.0;
    return s > 0.0 ? static_cast<uint64_t>(s * 1e9) : sm100::kPeerWaitDefaultNs;
  }();
  return v;
}

void fused_set_peer_wait(double seconds) {
  TORCH_CHECK(seconds > 0.0 && seconds <= 3600.0, "peer wait limit must be in (0, 3600] seconds");
  peer_wait_ns() = static_cast<uint64_t>(seconds * 1e9);
}

uint64_t fused_peer_wait_ns() { return peer_wait_ns(); }

static fused::Peers make_peers(torch::Tensor ptrs, torch::Tensor sigs, int world) {
  TORCH_CHECK(world >= 1 && world <= fused::kMaxRanks, "world size must be 1..8");
  TORCH_CHECK(ptrs.device().is_cpu() && ptrs.scalar_type() == torch::kInt64 && ptrs.numel() == world,
              "peer pointers must be a CPU int64 tensor of world entries");
  TORCH_CHECK(sigs.device().is_cpu() && sigs.scalar_type() == torch::kInt64 && sigs.numel() == world,
              "signal pads must be a CPU int64 tensor of world entries");
  fused::Peers pe;
  auto pa = ptrs.accessor<int64_t, 1>();
  auto sa = sigs.accessor<int64_t, 1>();
  for (int i = 0; i < fused::kMaxRanks; ++i) {
    pe.ptr[i] = i < world ? static_cast<uint64_t>(pa[i]) : 0;
    pe.sig[i] = i < world ? static_cast<uint64_t>(sa[i]) : 0;
    if (i < world) TORCH_CHECK(pe.ptr[i] % 16 == 0, "peer buffer ", i, " is not 16-byte aligned");
  }
  pe.wait_ns = peer_wait_ns();
  return pe;
}

// max_ctas > 0 caps the grid (a gather that overlaps compute kernels takes
// only a few SMs); otherwise up to two CTAs per SM.
static int comm_grid(long n8, long max_ctas = 0) {
  long want = (n8 + 255) / 256;
  long cap = max_ctas > 0 ? max_ctas : 2L * num_sms();
  return static_cast<int>(std::max<long>(1, std::min(want, cap)));
}

void fused_rs_d2h(torch::Tensor ptrs, torch::Tensor sigs, int64_t rank, int64_t world,
                  int64_t offset, int64_t n, torch::Tensor host_out, double scale, int64_t epoch,
                  torch::Tensor counter, torch::Tensor err) {
  auto pe = make_peers(ptrs, sigs, world);
  TORCH_CHECK(counter.is_cuda() && err.is_cuda(), "counter/err must live on the GPU");
  // A rank whose share of the range is empty still launches (one CTA): the
  // launch is its half of the per-epoch handshake with the peers.
  if (n < 0) n = 0;
  void* out_dev = nullptr;
  if (n > 0) {
    TORCH_CHECK(host_out.scalar_type() == torch::kBFloat16 && host_out.is_contiguous() &&
                    host_out.numel() >= n, "host_out must be a contiguous bf16 tensor of >= n elements");
    TORCH_CHECK(offset % 8 == 0, "shard offset must be a multiple of 8 elements");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(host_out.data_ptr()) % 16 == 0, "host_out misaligned");
    out_dev = host_out.data_ptr();
    if (host_out.device().is_cpu()) {
      T1_CHECK_CUDA(cudaHostGetDevicePointer(&out_dev, host_out.data_ptr(), 0));
    }
  }
  fused::rs_d2h_kernel<<<n > 0 ? comm_grid(n / 8) : 1, 256, 0, stream()>>>(
      pe, rank, world, offset, n, reinterpret_cast<__nv_bfloat16*>(out_dev), (float)scale,
      static_cast<uint32_t>(epoch), counter.data_ptr<int>(), err.data_ptr<int>());
  check_launch("fused_rs_d2h");
  count_launch();
}

// Device view of a page-locked host tensor (UVA: the host address itself).
static const void* device_view(const torch::Tensor& t) {
  if (!t.device().is_cpu()) return t.data_ptr();
  void* d = nullptr;
  T1_CHECK_CUDA(cudaHostGetDevicePointer(&d, t.data_ptr(), 0));
  return d;
}

// host_src: this rank's shard: fp32 master, bf16 copy, or (with host_src_lo)
// the high plane of a split master.
// host_src on the GPU must be this rank's own unit at [offset, offset + n)
// (the staged form): the kernel then only broadcasts it to the peers.
void fused_shard_gather(torch::Tensor ptrs, torch::Tensor sigs, int64_t rank, int64_t world,
                        int64_t offset, int64_t n, torch::Tensor host_src,
                        c10::optional<torch::Tensor> host_src_lo, int64_t epoch,
                        torch::Tensor counter, torch::Tensor err, int64_t max_ctas) {
  auto pe = make_peers(ptrs, sigs, world);
  if (n <= 0) {
    // empty share: still take part in the per-epoch handshake (one CTA)
    fused::shard_gather_kernel<<<1, 256, 0, stream()>>>(pe, rank, world, offset, 0, fused::kSrcBf16,
                                                        nullptr, nullptr, 0, static_cast<uint32_t>(epoch),
                                                        counter.data_ptr<int>(), err.data_ptr<int>());
    check_launch("fused_shard_gather");
    count_launch();
    return;
  }
  TORCH_CHECK(host_src.is_contiguous() && host_src.numel() >= n, "host_src too small");
  TORCH_CHECK(offset % 8 == 0, "shard offset must be a multiple of 8 elements");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(host_src.data_ptr()) % 16 == 0, "host_src misaligned");
  int kind;
  const void* lo = nullptr;
  if (host_src_lo.has_value() && host_src_lo->defined()) {
    TORCH_CHECK(host_src.element_size() == 2 && host_src_lo->element_size() == 2 &&
                    host_src_lo->is_contiguous() && host_src_lo->numel() >= n,
                "split master planes must be 16-bit tensors of >= n elements");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(host_src_lo->data_ptr()) % 16 == 0, "low plane misaligned");
    kind = fused::kSrcSplit;
    lo = device_view(*host_src_lo);
  } else if (host_src.scalar_type() == torch::kFloat32) {
    kind = fused::kSrcF32;
  } else {
    TORCH_CHECK(host_src.scalar_type() == torch::kBFloat16, "host_src must be fp32 or bf16");
    kind = fused::kSrcBf16;
  }
  int skip_self = 0;
  if (host_src.is_cuda()) {
    TORCH_CHECK(kind == fused::kSrcBf16, "a device-resident shard source must be bf16");
    TORCH_CHECK(reinterpret_cast<uint64_t>(host_src.data_ptr()) == pe.ptr[rank] + 2 * static_cast<uint64_t>(offset),
                "a device-resident shard source must be this rank's own unit at the shard offset");
    skip_self = 1;
  }
  fused::shard_gather_kernel<<<comm_grid(n / 8, max_ctas), 256, 0, stream()>>>(
      pe, rank, world, offset, n, kind, device_view(host_src), lo, skip_self,
      static_cast<uint32_t>(epoch), counter.data_ptr<int>(), err.data_ptr<int>());
  check_launch("fused_shard_gather");
  count_launch();
}

}  // namespace t1
