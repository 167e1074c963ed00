// Portable fallback of the host kernels (one float per "vector").
#define T1H_ISA scalar
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "host_kernels.h"

namespace t1h {
namespace scalar {
struct V {
  static constexpr int W = 1;
  using R = float;
  static inline R zero() { return 0.0f; }
  static inline R set1(float x) { return x; }
  static inline R add(R a, R b) { return a + b; }
  static inline R mul(R a, R b) { return a * b; }
  static inline R fmadd(R a, R b, R c) { return fmaf(a, b, c); }
  static inline R sqrt(R a) { return sqrtf(a); }
  static inline R div(R a, R b) { return a / b; }
  static inline double hsum(R a) { return a; }
  template <int DT, class T> static inline R ld(const T* p);
  template <int DT, class T> static inline void st(T* p, R x);
  template <int DT, class T> static inline bool can_stream(const T*) { return false; }
  template <int DT, class T> static inline void st_stream(T* p, R x) { st<DT>(p, x); }
  static inline void fence() {}
  static inline R split_ld(const uint16_t* hi, const uint16_t* lo);
  static inline void split_st(uint16_t* hi, uint16_t* lo, R x);
};
}  // namespace scalar
}  // namespace t1h

#include "host_kernels.inl"

namespace t1h {
namespace scalar {
template <int DT, class T> inline float V::ld(const T* p) { return Elem<DT>::ld(p); }
template <int DT, class T> inline void V::st(T* p, float x) { Elem<DT>::st(p, x); }
inline float V::split_ld(const uint16_t* hi, const uint16_t* lo) { return s_split_ld(hi, lo, 0); }
inline void V::split_st(uint16_t* hi, uint16_t* lo, float x) { s_split_st(hi, lo, 0, x); }
}  // namespace scalar
}  // namespace t1h
