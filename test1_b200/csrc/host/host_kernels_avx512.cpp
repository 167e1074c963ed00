// AVX-512 (F/BW/VL) + FMA + F16C variant of the host kernels (16 floats per
// vector).
#pragma GCC target("avx512f,avx512bw,avx512vl,avx2,fma,f16c")
#define T1H_ISA avx512
#include <immintrin.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "host_kernels.h"

namespace t1h {
namespace avx512 {
struct V {
  static constexpr int W = 16;
  using R = __m512;
  static inline R zero() { return _mm512_setzero_ps(); }
  static inline R set1(float x) { return _mm512_set1_ps(x); }
  static inline R add(R a, R b) { return _mm512_add_ps(a, b); }
  static inline R mul(R a, R b) { return _mm512_mul_ps(a, b); }
  static inline R fmadd(R a, R b, R c) { return _mm512_fmadd_ps(a, b, c); }
  static inline R sqrt(R a) { return _mm512_sqrt_ps(a); }
  static inline R div(R a, R b) { return _mm512_div_ps(a, b); }
  static inline double hsum(R a) { return _mm512_reduce_add_ps(a); }
  template <int DT, class T> static inline R ld(const T* p);
  template <int DT, class T> static inline void st(T* p, R x);
  template <int DT, class T> static inline void st_stream(T* p, R x);
  // streaming stores need the vector's natural alignment
  template <int DT, class T> static inline bool can_stream(const T* p) {
    return (reinterpret_cast<uintptr_t>(p) % (sizeof(T) * W)) == 0;
  }
  static inline void fence() { _mm_sfence(); }
  static inline R split_ld(const uint16_t* hi, const uint16_t* lo) {
    __m512i h = _mm512_slli_epi32(_mm512_cvtepu16_epi32(_mm256_loadu_si256(reinterpret_cast<const __m256i*>(hi))), 16);
    __m512i l = _mm512_cvtepu16_epi32(_mm256_loadu_si256(reinterpret_cast<const __m256i*>(lo)));
    return _mm512_castsi512_ps(_mm512_sub_epi32(_mm512_or_si512(h, l), _mm512_set1_epi32(0x8000)));
  }
  static inline void split_st(uint16_t* hi, uint16_t* lo, R x) {
    __m512i b = _mm512_add_epi32(_mm512_castps_si512(x), _mm512_set1_epi32(0x8000));
    _mm256_storeu_si256(reinterpret_cast<__m256i*>(hi), _mm512_cvtepi32_epi16(_mm512_srli_epi32(b, 16)));
    _mm256_storeu_si256(reinterpret_cast<__m256i*>(lo), _mm512_cvtepi32_epi16(b));
  }
};

template <> inline __m512 V::ld<kF32, float>(const float* p) { return _mm512_loadu_ps(p); }
template <> inline __m512 V::ld<kBF16, uint16_t>(const uint16_t* p) {
  __m512i w = _mm512_cvtepu16_epi32(_mm256_loadu_si256(reinterpret_cast<const __m256i*>(p)));
  return _mm512_castsi512_ps(_mm512_slli_epi32(w, 16));
}
template <> inline __m512 V::ld<kF16, uint16_t>(const uint16_t* p) {
  return _mm512_cvtph_ps(_mm256_loadu_si256(reinterpret_cast<const __m256i*>(p)));
}
template <> inline void V::st<kF32, float>(float* p, __m512 x) { _mm512_storeu_ps(p, x); }
template <> inline void V::st<kBF16, uint16_t>(uint16_t* p, __m512 x) {
  __m512i u = _mm512_castps_si512(x);
  __m512i lsb = _mm512_and_si512(_mm512_srli_epi32(u, 16), _mm512_set1_epi32(1));
  __m512i r = _mm512_srli_epi32(_mm512_add_epi32(u, _mm512_add_epi32(lsb, _mm512_set1_epi32(0x7fff))), 16);
  __mmask16 nan = _mm512_cmp_ps_mask(x, x, _CMP_UNORD_Q);
  r = _mm512_mask_mov_epi32(r, nan, _mm512_set1_epi32(0x7fc0));
  _mm256_storeu_si256(reinterpret_cast<__m256i*>(p), _mm512_cvtepi32_epi16(r));
}
template <> inline void V::st<kF16, uint16_t>(uint16_t* p, __m512 x) {
  _mm256_storeu_si256(reinterpret_cast<__m256i*>(p), _mm512_cvtps_ph(x, _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC));
}
template <> inline void V::st_stream<kBF16, uint16_t>(uint16_t* p, __m512 x) {
  __m512i u = _mm512_castps_si512(x);
  __m512i lsb = _mm512_and_si512(_mm512_srli_epi32(u, 16), _mm512_set1_epi32(1));
  __m512i r = _mm512_srli_epi32(_mm512_add_epi32(u, _mm512_add_epi32(lsb, _mm512_set1_epi32(0x7fff))), 16);
  __mmask16 nan = _mm512_cmp_ps_mask(x, x, _CMP_UNORD_Q);
  r = _mm512_mask_mov_epi32(r, nan, _mm512_set1_epi32(0x7fc0));
  _mm256_stream_si256(reinterpret_cast<__m256i*>(p), _mm512_cvtepi32_epi16(r));
}
template <> inline void V::st_stream<kF16, uint16_t>(uint16_t* p, __m512 x) {
  _mm256_stream_si256(reinterpret_cast<__m256i*>(p), _mm512_cvtps_ph(x, _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC));
}
template <> inline void V::st_stream<kF32, float>(float* p, __m512 x) { _mm512_stream_ps(p, x); }
}  // namespace avx512
}  // namespace t1h

#include "host_kernels.inl"
