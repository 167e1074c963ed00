// AVX2 + FMA + F16C variant of the host kernels (8 floats per vector).
// bf16 is handled with integer shifts, so unlike the reference's AVX2 build
// (optimizer/layer_adam/csrc/simd.h:110-146) bf16 params/state work here too.
#pragma GCC target("avx2,fma,f16c")
#define T1H_ISA avx2
#include <immintrin.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "host_kernels.h"

namespace t1h {
namespace avx2 {
struct V {
  static constexpr int W = 8;
  using R = __m256;
  static inline R zero() { return _mm256_setzero_ps(); }
  static inline R set1(float x) { return _mm256_set1_ps(x); }
  static inline R add(R a, R b) { return _mm256_add_ps(a, b); }
  static inline R mul(R a, R b) { return _mm256_mul_ps(a, b); }
  static inline R fmadd(R a, R b, R c) { return _mm256_fmadd_ps(a, b, c); }
  static inline R sqrt(R a) { return _mm256_sqrt_ps(a); }
  static inline R div(R a, R b) { return _mm256_div_ps(a, b); }
  static inline double hsum(R a) {
    __m128 lo = _mm256_castps256_ps128(a), hi = _mm256_extractf128_ps(a, 1);
    __m128 s = _mm_add_ps(lo, hi);
    s = _mm_hadd_ps(s, s);
    s = _mm_hadd_ps(s, s);
    return _mm_cvtss_f32(s);
  }
  template <int DT, class T> static inline R ld(const T* p);
  template <int DT, class T> static inline void st(T* p, R x);
  template <int DT, class T> static inline void st_stream(T* p, R x);
  // streaming stores need the vector's natural alignment
  template <int DT, class T> static inline bool can_stream(const T* p) {
    return (reinterpret_cast<uintptr_t>(p) % (sizeof(T) * W)) == 0;
  }
  static inline void fence() { _mm_sfence(); }
  static inline R split_ld(const uint16_t* hi, const uint16_t* lo) {
    __m256i h = _mm256_slli_epi32(_mm256_cvtepu16_epi32(_mm_loadu_si128(reinterpret_cast<const __m128i*>(hi))), 16);
    __m256i l = _mm256_cvtepu16_epi32(_mm_loadu_si128(reinterpret_cast<const __m128i*>(lo)));
    return _mm256_castsi256_ps(_mm256_sub_epi32(_mm256_or_si256(h, l), _mm256_set1_epi32(0x8000)));
  }
  static inline void split_st(uint16_t* hi, uint16_t* lo, R x) {
    __m256i b = _mm256_add_epi32(_mm256_castps_si256(x), _mm256_set1_epi32(0x8000));
    __m256i h = _mm256_srli_epi32(b, 16);
    __m256i l = _mm256_and_si256(b, _mm256_set1_epi32(0xffff));
    _mm_storeu_si128(reinterpret_cast<__m128i*>(hi),
                     _mm_packus_epi32(_mm256_castsi256_si128(h), _mm256_extracti128_si256(h, 1)));
    _mm_storeu_si128(reinterpret_cast<__m128i*>(lo),
                     _mm_packus_epi32(_mm256_castsi256_si128(l), _mm256_extracti128_si256(l, 1)));
  }
};

template <> inline __m256 V::ld<kF32, float>(const float* p) { return _mm256_loadu_ps(p); }
template <> inline __m256 V::ld<kBF16, uint16_t>(const uint16_t* p) {
  __m256i w = _mm256_cvtepu16_epi32(_mm_loadu_si128(reinterpret_cast<const __m128i*>(p)));
  return _mm256_castsi256_ps(_mm256_slli_epi32(w, 16));
}
template <> inline __m256 V::ld<kF16, uint16_t>(const uint16_t* p) {
  return _mm256_cvtph_ps(_mm_loadu_si128(reinterpret_cast<const __m128i*>(p)));
}
template <> inline void V::st<kF32, float>(float* p, __m256 x) { _mm256_storeu_ps(p, x); }
template <> inline void V::st<kBF16, uint16_t>(uint16_t* p, __m256 x) {
  __m256i u = _mm256_castps_si256(x);
  __m256i lsb = _mm256_and_si256(_mm256_srli_epi32(u, 16), _mm256_set1_epi32(1));
  __m256i r = _mm256_srli_epi32(_mm256_add_epi32(u, _mm256_add_epi32(lsb, _mm256_set1_epi32(0x7fff))), 16);
  __m256 nan = _mm256_cmp_ps(x, x, _CMP_UNORD_Q);
  r = _mm256_castps_si256(_mm256_blendv_ps(_mm256_castsi256_ps(r),
                                           _mm256_castsi256_ps(_mm256_set1_epi32(0x7fc0)), nan));
  __m128i packed = _mm_packus_epi32(_mm256_castsi256_si128(r), _mm256_extracti128_si256(r, 1));
  _mm_storeu_si128(reinterpret_cast<__m128i*>(p), packed);
}
template <> inline void V::st<kF16, uint16_t>(uint16_t* p, __m256 x) {
  _mm_storeu_si128(reinterpret_cast<__m128i*>(p), _mm256_cvtps_ph(x, _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC));
}
template <> inline void V::st_stream<kBF16, uint16_t>(uint16_t* p, __m256 x) {
  __m256i u = _mm256_castps_si256(x);
  __m256i lsb = _mm256_and_si256(_mm256_srli_epi32(u, 16), _mm256_set1_epi32(1));
  __m256i r = _mm256_srli_epi32(_mm256_add_epi32(u, _mm256_add_epi32(lsb, _mm256_set1_epi32(0x7fff))), 16);
  __m256 nan = _mm256_cmp_ps(x, x, _CMP_UNORD_Q);
  r = _mm256_castps_si256(_mm256_blendv_ps(_mm256_castsi256_ps(r),
                                           _mm256_castsi256_ps(_mm256_set1_epi32(0x7fc0)), nan));
  __m128i packed = _mm_packus_epi32(_mm256_castsi256_si128(r), _mm256_extracti128_si256(r, 1));
  _mm_stream_si128(reinterpret_cast<__m128i*>(p), packed);
}
template <> inline void V::st_stream<kF16, uint16_t>(uint16_t* p, __m256 x) {
  _mm_stream_si128(reinterpret_cast<__m128i*>(p), _mm256_cvtps_ph(x, _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC));
}
template <> inline void V::st_stream<kF32, float>(float* p, __m256 x) { _mm256_stream_ps(p, x); }
}  // namespace avx2
}  // namespace t1h

#include "host_kernels.inl"
