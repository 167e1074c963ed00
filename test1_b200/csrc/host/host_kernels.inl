// Kernel bodies shared by the three ISA translation units.  The including TU
// defines a vector-traits struct `V` and the macro T1H_ISA before including
// this file.  Nothing here may include torch or STL headers (see
// host_kernels.h).
//
// LayerAdam element update (same operation order as the reference CPU Adam,
// optimizer/layer_adam/csrc/cpu_adam.h:152-193, so fp32 results agree to the
// last ulp of each fused multiply-add):
//   g  = grad * grad_scale            (+ wd * p first, in L2 mode)
//   m  = beta1 * m + (1 - beta1) * g
//   v  = beta2 * v + (1 - beta2) * g^2
//   u  = m / (sqrt(v) * (1/sqrt(1 - beta2^t)) + eps)
//   p  = p + (-lr * wd) * p           (AdamW mode only)
//   p  = p + (-lr / (1 - beta1^t)) * u
// An optional shadow (bf16/fp16 copy of the new p) is written in the same
// pass, which removes the separate per-step cast of every layer.

#include <math.h>
#include <stdint.h>
#include <string.h>

#include "host_kernels.h"

namespace t1h {
namespace T1H_ISA {

// ---------------------------------------------------------------- scalar cvt
static inline float s_bf16_to_f32(uint16_t h) {
  uint32_t u = static_cast<uint32_t>(h) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

// Round-to-nearest-even; every NaN becomes the canonical quiet NaN 0x7FC0
// (torch's bfloat16 conversion does the same).
static inline uint16_t s_f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0;
  u += 0x7fffu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

static inline float s_f16_to_f32(uint16_t h) {
  uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1fu;
  uint32_t m = h & 0x3ffu;
  uint32_t out;
  if (e == 0) {
    float f = static_cast<float>(m) * 5.9604644775390625e-8f;  // m * 2^-24
    memcpy(&out, &f, 4);
    out |= sign;
  } else if (e == 31) {
    out = sign | 0x7f800000u | (m << 13);
  } else {
    out = sign | ((e + 112u) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &out, 4);
  return f;
}

static inline uint16_t s_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7fffffffu;
  if (ax > 0x7f800000u) return static_cast<uint16_t>(sign | 0x7e00u);
  if (ax >= 0x477ff000u) return static_cast<uint16_t>(sign | 0x7c00u);
  if (ax < 0x38800000u) {
    float af;
    memcpy(&af, &ax, 4);
    uint32_t m = static_cast<uint32_t>(nearbyintf(af * 16777216.0f));
    return static_cast<uint16_t>(sign | m);
  }
  uint32_t r = ax - 0x38000000u;
  r += 0xfffu + ((r >> 13) & 1u);
  return static_cast<uint16_t>(sign | (r >> 13));
}

template <int DT> struct Elem;
template <> struct Elem<kF32> {
  using type = float;
  static inline float ld(const float* p) { return *p; }
  static inline void st(float* p, float x) { *p = x; }
};
template <> struct Elem<kBF16> {
  using type = uint16_t;
  static inline float ld(const uint16_t* p) { return s_bf16_to_f32(*p); }
  static inline void st(uint16_t* p, float x) { *p = s_f32_to_bf16(x); }
};
template <> struct Elem<kF16> {
  using type = uint16_t;
  static inline float ld(const uint16_t* p) { return s_f16_to_f32(*p); }
  static inline void st(uint16_t* p, float x) { *p = s_f32_to_f16(x); }
};

// ------------------------------------------------------------- split planes
static inline float s_split_ld(const uint16_t* hi, const uint16_t* lo, int64_t i) {
  uint32_t b = ((static_cast<uint32_t>(hi[i]) << 16) | lo[i]) - 0x8000u;
  float f;
  memcpy(&f, &b, 4);
  return f;
}
static inline void s_split_st(uint16_t* hi, uint16_t* lo, int64_t i, float x) {
  uint32_t b;
  memcpy(&b, &x, 4);
  b += 0x8000u;
  hi[i] = static_cast<uint16_t>(b >> 16);
  lo[i] = static_cast<uint16_t>(b & 0xffffu);
}

// ------------------------------------------------------------------- adam
constexpr int kNoShadow = -1;

// The param access of the Adam kernel: a plain pointer, or two planes.
template <int PDT>
struct ParamIO {
  using PT = typename Elem<PDT>::type;
  PT* p;
  ParamIO(const AdamArgs& a) : p(static_cast<PT*>(a.param)) {}
  inline typename V::R vload(int64_t j) const { return V::template ld<PDT>(p + j); }
  inline void vstore(int64_t j, typename V::R x) const { V::template st<PDT>(p + j, x); }
  inline float sload(int64_t j) const { return Elem<PDT>::ld(p + j); }
  inline void sstore(int64_t j, float x) const { Elem<PDT>::st(p + j, x); }
};
template <>
struct ParamIO<kSplit> {
  uint16_t* hi;
  uint16_t* lo;
  ParamIO(const AdamArgs& a)
      : hi(static_cast<uint16_t*>(a.param)), lo(static_cast<uint16_t*>(a.param_lo)) {}
  inline typename V::R vload(int64_t j) const { return V::split_ld(hi + j, lo + j); }
  inline void vstore(int64_t j, typename V::R x) const { V::split_st(hi + j, lo + j, x); }
  inline float sload(int64_t j) const { return s_split_ld(hi, lo, j); }
  inline void sstore(int64_t j, float x) const { s_split_st(hi, lo, j, x); }
};

template <int PDT, int GDT, int SDT, int HDT>
static void adam_kernel(const AdamArgs& a, int64_t begin, int64_t end) {
  using GT = typename Elem<GDT>::type;
  using ST = typename Elem<SDT>::type;
  using HT = typename Elem<(HDT < 0 ? kBF16 : HDT)>::type;
  const ParamIO<PDT> p(a);
  const GT* g = static_cast<const GT*>(a.grad);
  ST* m = static_cast<ST*>(a.exp_avg);
  ST* v = static_cast<ST*>(a.exp_avg_sq);
  HT* sh = static_cast<HT*>(a.shadow);
  const AdamHyper& h = a.h;
  const bool l2 = h.has_wd && !h.adamw;
  const bool decoupled = h.has_wd && h.adamw;

  using R = typename V::R;
  const R b1 = V::set1(h.beta1), b2 = V::set1(h.beta2);
  const R omb1 = V::set1(h.one_minus_beta1), omb2 = V::set1(h.one_minus_beta2);
  const R eps = V::set1(h.eps), bc2 = V::set1(h.bc2_rsqrt);
  const R step = V::set1(h.step_size), wd = V::set1(h.wd), wdstep = V::set1(h.wd_step);
  const R gscale = V::set1(h.grad_scale);
  // The shadow is write-only: stream it past the caches when its vectors
  // are aligned (saves the read-for-ownership of every shadow line).
  const bool nt = HDT >= 0 && h.stream_shadow &&
                  V::template can_stream<(HDT < 0 ? kBF16 : HDT)>(sh + begin);

  auto body = [&](int64_t j) __attribute__((always_inline)) {
    R gr = g ? V::mul(V::template ld<GDT>(g + j), gscale) : V::zero();
    R pr = p.vload(j);
    R mr = V::template ld<SDT>(m + j);
    R vr = V::template ld<SDT>(v + j);
    if (l2) gr = V::fmadd(pr, wd, gr);
    mr = V::mul(mr, b1);
    mr = V::fmadd(gr, omb1, mr);
    vr = V::mul(vr, b2);
    R g2 = V::mul(gr, gr);
    vr = V::fmadd(g2, omb2, vr);
    R d = V::sqrt(vr);
    d = V::fmadd(d, bc2, eps);
    R u = V::div(mr, d);
    if (decoupled) pr = V::fmadd(pr, wdstep, pr);
    pr = V::fmadd(u, step, pr);
    p.vstore(j, pr);
    V::template st<SDT>(m + j, mr);
    V::template st<SDT>(v + j, vr);
    if (HDT >= 0) {
      if (nt) V::template st_stream<(HDT < 0 ? kBF16 : HDT)>(sh + j, pr);
      else V::template st<(HDT < 0 ? kBF16 : HDT)>(sh + j, pr);
    }
  };

  int64_t i = begin;
  constexpr int W = V::W;
  for (; i + 4 * W <= end; i += 4 * W) {
    body(i);
    body(i + W);
    body(i + 2 * W);
    body(i + 3 * W);
  }
  for (; i + W <= end; i += W) body(i);
  for (; i < end; ++i) {
    float gv = g ? Elem<GDT>::ld(g + i) * h.grad_scale : 0.0f;
    float pv = p.sload(i);
    float mv = Elem<SDT>::ld(m + i);
    float vv = Elem<SDT>::ld(v + i);
    if (l2) gv = fmaf(pv, h.wd, gv);
    mv = mv * h.beta1;
    mv = fmaf(gv, h.one_minus_beta1, mv);
    vv = vv * h.beta2;
    float g2 = gv * gv;
    vv = fmaf(g2, h.one_minus_beta2, vv);
    float d = sqrtf(vv);
    d = fmaf(d, h.bc2_rsqrt, h.eps);
    float u = mv / d;
    if (decoupled) pv = fmaf(pv, h.wd_step, pv);
    pv = fmaf(u, h.step_size, pv);
    p.sstore(i, pv);
    Elem<SDT>::st(m + i, mv);
    Elem<SDT>::st(v + i, vv);
    if (HDT >= 0) Elem<(HDT < 0 ? kBF16 : HDT)>::st(sh + i, pv);
  }
  if (nt) V::fence();
}

template <int PDT, int GDT, int SDT>
static void adam_dispatch_shadow(const AdamArgs& a, int64_t b, int64_t e) {
  if (a.shadow == nullptr) return adam_kernel<PDT, GDT, SDT, kNoShadow>(a, b, e);
  switch (a.shadow_dt) {
    case kBF16: return adam_kernel<PDT, GDT, SDT, kBF16>(a, b, e);
    case kF16: return adam_kernel<PDT, GDT, SDT, kF16>(a, b, e);
    default: return adam_kernel<PDT, GDT, SDT, kF32>(a, b, e);
  }
}

template <int PDT, int GDT>
static void adam_dispatch_state(const AdamArgs& a, int64_t b, int64_t e) {
  switch (a.state_dt) {
    case kBF16: return adam_dispatch_shadow<PDT, GDT, kBF16>(a, b, e);
    case kF16: return adam_dispatch_shadow<PDT, GDT, kF16>(a, b, e);
    default: return adam_dispatch_shadow<PDT, GDT, kF32>(a, b, e);
  }
}

template <int PDT>
static void adam_dispatch_grad(const AdamArgs& a, int64_t b, int64_t e) {
  switch (a.grad_dt) {
    case kBF16: return adam_dispatch_state<PDT, kBF16>(a, b, e);
    case kF16: return adam_dispatch_state<PDT, kF16>(a, b, e);
    default: return adam_dispatch_state<PDT, kF32>(a, b, e);
  }
}

// ------------------------------------------------------------------- cast
template <int SDT, int DDT>
static void cast_kernel(const void* src, void* dst, float scale, int64_t b, int64_t e) {
  using STy = typename Elem<SDT>::type;
  using DTy = typename Elem<DDT>::type;
  const STy* s = static_cast<const STy*>(src);
  DTy* d = static_cast<DTy*>(dst);
  const typename V::R sc = V::set1(scale);
  constexpr int W = V::W;
  int64_t i = b;
  for (; i + W <= e; i += W) V::template st<DDT>(d + i, V::mul(V::template ld<SDT>(s + i), sc));
  for (; i < e; ++i) Elem<DDT>::st(d + i, Elem<SDT>::ld(s + i) * scale);
}

template <int SDT>
static void cast_dispatch_dst(const void* src, void* dst, int ddt, float scale, int64_t b, int64_t e) {
  switch (ddt) {
    case kBF16: return cast_kernel<SDT, kBF16>(src, dst, scale, b, e);
    case kF16: return cast_kernel<SDT, kF16>(src, dst, scale, b, e);
    default: return cast_kernel<SDT, kF32>(src, dst, scale, b, e);
  }
}

// ------------------------------------------------------------- slot reduce
template <int SDT, int DDT>
static void sum_slots_kernel(const void* const* srcs, int nsrc, void* dst, float scale,
                             int64_t b, int64_t e) {
  using STy = typename Elem<SDT>::type;
  using DTy = typename Elem<DDT>::type;
  DTy* d = static_cast<DTy*>(dst);
  const typename V::R sc = V::set1(scale);
  constexpr int W = V::W;
  int64_t i = b;
  // The destination is only written: streaming stores skip the
  // read-for-ownership that a cached store costs (a quarter of the traffic
  // with two sources).  Elements up to the first vector-aligned one go
  // through the scalar path.
  while (i < e && !V::template can_stream<DDT>(d + i) && i - b < W) {
    float acc = 0.0f;
    for (int k = 0; k < nsrc; ++k) acc += Elem<SDT>::ld(static_cast<const STy*>(srcs[k]) + i);
    Elem<DDT>::st(d + i, acc * scale);
    ++i;
  }
  const bool nt = i < e && V::template can_stream<DDT>(d + i);
  for (; i + W <= e; i += W) {
    typename V::R acc = V::zero();
    for (int k = 0; k < nsrc; ++k)
      acc = V::add(acc, V::template ld<SDT>(static_cast<const STy*>(srcs[k]) + i));
    if (nt)
      V::template st_stream<DDT>(d + i, V::mul(acc, sc));
    else
      V::template st<DDT>(d + i, V::mul(acc, sc));
  }
  if (nt) V::fence();
  for (; i < e; ++i) {
    float acc = 0.0f;
    for (int k = 0; k < nsrc; ++k) acc += Elem<SDT>::ld(static_cast<const STy*>(srcs[k]) + i);
    Elem<DDT>::st(d + i, acc * scale);
  }
}

template <int SDT>
static void sum_slots_dispatch_dst(const void* const* srcs, int nsrc, void* dst, int ddt,
                                   float scale, int64_t b, int64_t e) {
  switch (ddt) {
    case kBF16: return sum_slots_kernel<SDT, kBF16>(srcs, nsrc, dst, scale, b, e);
    case kF16: return sum_slots_kernel<SDT, kF16>(srcs, nsrc, dst, scale, b, e);
    default: return sum_slots_kernel<SDT, kF32>(srcs, nsrc, dst, scale, b, e);
  }
}

// ------------------------------------------------------------------ sumsq
template <int DT>
static double sumsq_kernel(const void* src, int64_t b, int64_t e) {
  using Ty = typename Elem<DT>::type;
  const Ty* s = static_cast<const Ty*>(src);
  constexpr int W = V::W;
  double total = 0.0;
  int64_t i = b;
  // Accumulate in fp32 vectors over short blocks, then fold into double.
  while (i + W <= e) {
    typename V::R acc = V::zero();
    int64_t stop = i + 4096 * W;
    if (stop > e) stop = e - ((e - i) % W);
    for (; i < stop; i += W) {
      typename V::R x = V::template ld<DT>(s + i);
      acc = V::fmadd(x, x, acc);
    }
    total += V::hsum(acc);
  }
  for (; i < e; ++i) {
    double x = Elem<DT>::ld(s + i);
    total += x * x;
  }
  return total;
}

}  // namespace T1H_ISA

#define T1H_CAT2(a, b) a##_##b
#define T1H_CAT(a, b) T1H_CAT2(a, b)

void T1H_CAT(adam_range, T1H_ISA)(const AdamArgs& a, int64_t begin, int64_t end) {
  using namespace T1H_ISA;
  switch (a.param_dt) {
    case kSplit: return adam_dispatch_grad<kSplit>(a, begin, end);
    case kBF16: return adam_dispatch_grad<kBF16>(a, begin, end);
    case kF16: return adam_dispatch_grad<kF16>(a, begin, end);
    default: return adam_dispatch_grad<kF32>(a, begin, end);
  }
}

void T1H_CAT(cast_range, T1H_ISA)(const void* src, int src_dt, void* dst, int dst_dt,
                                  float scale, int64_t begin, int64_t end) {
  using namespace T1H_ISA;
  switch (src_dt) {
    case kBF16: return cast_dispatch_dst<kBF16>(src, dst, dst_dt, scale, begin, end);
    case kF16: return cast_dispatch_dst<kF16>(src, dst, dst_dt, scale, begin, end);
    default: return cast_dispatch_dst<kF32>(src, dst, dst_dt, scale, begin, end);
  }
}

void T1H_CAT(sum_slots_range, T1H_ISA)(const void* const* srcs, int nsrc, int src_dt, void* dst,
                                       int dst_dt, float scale, int64_t begin, int64_t end) {
  using namespace T1H_ISA;
  switch (src_dt) {
    case kBF16: return sum_slots_dispatch_dst<kBF16>(srcs, nsrc, dst, dst_dt, scale, begin, end);
    case kF16: return sum_slots_dispatch_dst<kF16>(srcs, nsrc, dst, dst_dt, scale, begin, end);
    default: return sum_slots_dispatch_dst<kF32>(srcs, nsrc, dst, dst_dt, scale, begin, end);
  }
}

void T1H_CAT(split_range, T1H_ISA)(const float* src, uint16_t* hi, uint16_t* lo, int64_t begin,
                                   int64_t end) {
  using namespace T1H_ISA;
  constexpr int W = V::W;
  int64_t i = begin;
  for (; i + W <= end; i += W) V::split_st(hi + i, lo + i, V::template ld<kF32>(src + i));
  for (; i < end; ++i) s_split_st(hi, lo, i, src[i]);
}

void T1H_CAT(unsplit_range, T1H_ISA)(const uint16_t* hi, const uint16_t* lo, float* dst,
                                     int64_t begin, int64_t end) {
  using namespace T1H_ISA;
  constexpr int W = V::W;
  int64_t i = begin;
  for (; i + W <= end; i += W) V::template st<kF32>(dst + i, V::split_ld(hi + i, lo + i));
  for (; i < end; ++i) dst[i] = s_split_ld(hi, lo, i);
}

double T1H_CAT(sumsq_range, T1H_ISA)(const void* src, int dt, int64_t begin, int64_t end) {
  using namespace T1H_ISA;
  switch (dt) {
    case kBF16: return sumsq_kernel<kBF16>(src, begin, end);
    case kF16: return sumsq_kernel<kF16>(src, begin, end);
    default: return sumsq_kernel<kF32>(src, begin, end);
  }
}

}  // namespace t1h
