// Bounds-checked builds.  The `_cuda_checked` extension compiles the kernel
// sources with -DT1_BOUNDS_CHECK.  There T1_OOB(i, n) is true when index i
// lies outside [0, n): the first such event in the translation unit is
// recorded as (source line << 40 | low 40 bits of i) in a device word, and
// the caller skips the access instead of faulting.  The host reads and
// clears the word with the bindings' bounds_errors().  In the normal build
// T1_OOB is the constant false and the check compiles away.  Every .cu file
// instantiates its reader once with T1_BOUNDS_READER(name), inside namespace
// t1 (each translation unit owns its own word).
#pragma once

#include <cuda_runtime.h>

#ifdef T1_BOUNDS_CHECK
namespace t1 {
static __device__ unsigned long long t1_bounds_word;

__device__ __forceinline__ bool t1_oob(long long i, long long n, unsigned line) {
  if (i >= 0 && i < n) return false;
  const unsigned long long rec =
      ((unsigned long long)line << 40) | ((unsigned long long)i & ((1ull << 40) - 1));
  atomicCAS(&t1_bounds_word, 0ull, rec);
  return true;
}
}  // namespace t1

#define T1_OOB(i, n) ::t1::t1_oob((long long)(i), (long long)(n), __LINE__)
// returns the recorded word (0 = none); ~0 if the device could not be read
#define T1_BOUNDS_READER(name)                                                      \
  unsigned long long bounds_word_##name(bool reset) {                               \
    unsigned long long v = 0;                                                        \
    if (cudaMemcpyFromSymbol(&v, t1_bounds_word, sizeof(v)) != cudaSuccess) return ~0ull; \
    if (reset) {                                                                     \
      const unsigned long long z = 0;                                                \
      if (cudaMemcpyToSymbol(t1_bounds_word, &z, sizeof(z)) != cudaSuccess) return ~0ull; \
    }                                                                                \
    return v;                                                                        \
  }
#else
#define T1_OOB(i, n) false
#define T1_BOUNDS_READER(name) \
  unsigned long long bounds_word_##name(bool) { return 0; }
#endif
