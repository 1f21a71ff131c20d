// Shared host/device helpers of libspeckv: status reporting, the device error
// word, fast integer division and vector-width selection for row copies.
#pragma once

#include <cuda_runtime.h>
#include <initializer_list>
#include <stdint.h>
#include <stdarg.h>
#include <stdio.h>

#include "../../include/speckv.h"

namespace speckv {

// ---- status reporting (host) ------------------------------------------------

// Records a formatted message for speckv_last_error() and returns `code`.
int fail(int code, const char* fmt, ...);

// Returns SPECKV_OK or SPECKV_ECUDA (with message) for the last launch.
int check_launch(const char* what);

// Device address of the library's error word on the current device.
unsigned long long* device_error_word();

// Kernels launch on the current GPU: returns SPECKV_EINVAL (with message) when one of
// `ptrs` is device memory of another GPU or plain (unregistered) host memory. Null
// entries, pinned host memory and managed memory pass. One driver query per pointer.
int check_current_device(const char* fn, std::initializer_list<const void*> ptrs);

// ---- device error word --------------------------------------------------------

__device__ __forceinline__ void record_error(unsigned long long* err, unsigned kind,
                                             long long value) {
  unsigned long long v = (unsigned long long)value & 0xFFFFFFFFFFFFull;
  atomicCAS(err, 0ull, ((unsigned long long)kind << 48) | v);
}

// ---- fast division of non-negative 31-bit integers by a runtime divisor -----
// q = (umulhi(n, m) + n) >> s, with s = ceil(log2 d), m = floor(2^32 (2^s - d) / d) + 1.
struct FastDiv {
  uint32_t d, m, s;
  FastDiv() : d(1), m(1), s(0) {}
  explicit FastDiv(uint32_t divisor) {
    d = divisor < 1 ? 1 : divisor;
    s = 0;
    while ((1ull << s) < d) ++s;
    m = (uint32_t)(((1ull << 32) * ((1ull << s) - d)) / d + 1);
  }
  __host__ __device__ __forceinline__ uint32_t div(uint32_t n) const {
#ifdef __CUDA_ARCH__
    return (__umulhi(n, m) + n) >> s;
#else
    return (uint32_t)((((uint64_t)n * m >> 32) + n) >> s);
#endif
  }
  __host__ __device__ __forceinline__ void divmod(uint32_t n, uint32_t& q, uint32_t& r) const {
    q = div(n);
    r = n - q * d;
  }
};

// ---- vector types for row copies ---------------------------------------------
template <int V> struct Vec;
template <> struct Vec<16> { typedef uint4 T; };
template <> struct Vec<8> { typedef uint2 T; };
template <> struct Vec<4> { typedef unsigned int T; };
template <> struct Vec<2> { typedef unsigned short T; };
template <> struct Vec<1> { typedef unsigned char T; };

// Largest power of two <= 16 dividing every value (byte sizes, strides, addresses).
inline int pick_vec(const long long* vals, int n) {
  int g = 16;
  for (int i = 0; i < n; ++i) {
    while (g > 1 && (vals[i] % g) != 0) g >>= 1;
  }
  return g;
}

inline bool fits_u31(long long x) { return x >= 0 && x < (1ll << 31); }

}  // namespace speckv

// Dispatches a templated launch on vector width `vec` (16/8/4/2/1).
#define SPECKV_DISPATCH_VEC(vec, ...)               \
  switch (vec) {                                    \
    case 16: { constexpr int V = 16; __VA_ARGS__; } break; \
    case 8: { constexpr int V = 8; __VA_ARGS__; } break;   \
    case 4: { constexpr int V = 4; __VA_ARGS__; } break;   \
    case 2: { constexpr int V = 2; __VA_ARGS__; } break;   \
    default: { constexpr int V = 1; __VA_ARGS__; } break;  \
  }
