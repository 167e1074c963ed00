// C ABI shared by the host SIMD kernels (LayerAdam step, casts, slot
// reductions, sum of squares).  Each ISA variant lives in its own translation
// unit (host_kernels_{scalar,avx2,avx512}.cpp) compiled with `#pragma GCC
// target`, includes no torch/STL headers (so no inline function compiled for
// a wider ISA can leak into the rest of the binary through the linker), and
// exports only the functions declared here.  dispatch.cpp picks the widest
// variant the running CPU supports.
#pragma once

#include <cstdint>

namespace t1h {

enum HostDType : int { kF32 = 0, kBF16 = 1, kF16 = 2, kSplit = 3 };

// kSplit: an fp32 value stored as two 16-bit planes.  With b = bits(x) +
// 0x8000 (mod 2^32), hi = b >> 16 and lo = b & 0xffff; hi alone is x rounded
// to bf16 (nearest, ties away from zero), and ((hi << 16) | lo) - 0x8000
// restores x exactly.  A master kept this way carries its own bf16 copy, so
// the optimizer writes no separate shadow.

struct AdamHyper {
  float beta1;
  float beta2;
  float one_minus_beta1;
  float one_minus_beta2;
  float eps;
  float bc2_rsqrt;   // 1/sqrt(1 - beta2^t), or 1 without bias correction
  float step_size;   // -lr / (1 - beta1^t), or -lr without bias correction
  float wd;          // weight decay coefficient
  float wd_step;     // -lr * wd (decoupled AdamW decay factor)
  float grad_scale;  // multiplies every gradient element before use
  int adamw;         // 1: decoupled decay (AdamW), 0: L2 added to the gradient
  int has_wd;        // wd > 0
  int stream_shadow; // 1: non-temporal stores for the shadow when aligned
};

struct AdamArgs {
  void* param;       // kSplit: the hi plane
  void* param_lo;    // kSplit only: the lo plane
  int param_dt;
  const void* grad;  // may be null: the gradient is treated as all zeros
  int grad_dt;
  void* exp_avg;
  void* exp_avg_sq;
  int state_dt;
  void* shadow;      // optional low-precision copy of the updated param
  int shadow_dt;
  AdamHyper h;
};

// Every kernel processes elements [begin, end) of its operands.
#define T1H_DECLARE_ISA(ISA)                                                   \
  void adam_range_##ISA(const AdamArgs& a, int64_t begin, int64_t end);        \
  void cast_range_##ISA(const void* src, int src_dt, void* dst, int dst_dt,    \
                        float scale, int64_t begin, int64_t end);              \
  void sum_slots_range_##ISA(const void* const* srcs, int nsrc, int src_dt,    \
                             void* dst, int dst_dt, float scale,               \
                             int64_t begin, int64_t end);                      \
  double sumsq_range_##ISA(const void* src, int dt, int64_t begin, int64_t end);             \
  void split_range_##ISA(const float* src, uint16_t* hi, uint16_t* lo, int64_t begin,        \
                         int64_t end);                                                       \
  void unsplit_range_##ISA(const uint16_t* hi, const uint16_t* lo, float* dst, int64_t begin, \
                           int64_t end);

T1H_DECLARE_ISA(scalar)
T1H_DECLARE_ISA(avx2)
T1H_DECLARE_ISA(avx512)

}  // namespace t1h
