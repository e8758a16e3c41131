// Shared definitions of the isotonic-regression kernels: bit tricks that also compile on the
// host (so that the kernels' phase logic can be run by the CPU emulator in tests/emu), the pool
// predicate, element conversions, and a division by an invariant divisor.
#pragma once

#include <stdint.h>

#ifdef TISO_HOST_EMU
#include <cmath>
#define TISO_HD inline
#define TISO_DEV inline
#else
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#define TISO_HD __host__ __device__ __forceinline__
#define TISO_DEV __device__ __forceinline__
#endif

namespace tiso {

// ---------------------------------------------------------------------------------------------
// Bit helpers (device intrinsics, or the compiler's builtins in the emulator).

TISO_HD int clz32(uint32_t x) {
#if defined(__CUDA_ARCH__)
  return __clz(static_cast<int>(x));
#else
  return x ? __builtin_clz(x) : 32;
#endif
}

TISO_HD int ffs32(uint32_t x) {  // 1 + index of the lowest set bit, 0 if none
#if defined(__CUDA_ARCH__)
  return __ffs(static_cast<int>(x));
#else
  return __builtin_ffs(static_cast<int>(x));
#endif
}

TISO_HD int popc32(uint32_t x) {
#if defined(__CUDA_ARCH__)
  return __popc(x);
#else
  return __builtin_popcount(x);
#endif
}

TISO_HD int high_bit(uint32_t x) { return 31 - clz32(x); }  // x != 0
TISO_HD int low_bit(uint32_t x) { return ffs32(x) - 1; }    // x != 0
TISO_HD uint32_t bits_upto(int p) {  // bits 0..p (p in 0..31)
  return p >= 31 ? 0xffffffffu : ((2u << p) - 1u);
}
TISO_HD uint32_t bits_below(int p) {  // bits 0..p-1 (p in 0..32)
  return p >= 32 ? 0xffffffffu : ((1u << p) - 1u);
}

TISO_HD double fma_(double a, double b, double c) {
#if defined(__CUDA_ARCH__)
  return fma(a, b, c);
#else
  return std::fma(a, b, c);
#endif
}

TISO_HD float fma_(float a, float b, float c) {
#if defined(__CUDA_ARCH__)
  return fmaf(a, b, c);
#else
  return std::fma(a, b, c);
#endif
}

// -infinity (the stacks' sentinel), without a division
TISO_HD double neg_inf() {
#if defined(__CUDA_ARCH__)
  return __longlong_as_double(static_cast<long long>(0xfff0000000000000ULL));
#else
  return -HUGE_VAL;
#endif
}

TISO_HD double fabs_(double x) {
#if defined(__CUDA_ARCH__)
  return fabs(x);
#else
  return x < 0 ? -x : x;
#endif
}

// v (0 <= v < 2^31) as a double without an int-to-double conversion instruction (those issue
// on the slow conversion pipe): the bits of 2^52 + v, minus 2^52.
TISO_HD double small_double(int v) {
#if defined(__CUDA_ARCH__)
  return __longlong_as_double(0x4330000000000000LL | static_cast<long long>(v)) -
         4503599627370496.0;
#else
  return static_cast<double>(v);
#endif
}
TISO_HD float small_float(int v) {  // 0 <= v < 2^23
#if defined(__CUDA_ARCH__)
  return __int_as_float(0x4B000000 | v) - 8388608.0f;
#else
  return static_cast<float>(v);
#endif
}
// The reverse: an exact integer-valued w (0 <= w < 2^31, resp. 2^23) back to an int, by the
// same offset: the low bits of w + 2^52 (2^23) are w.
TISO_HD int small_int(double w) {
#if defined(__CUDA_ARCH__)
  return static_cast<int>(__double_as_longlong(w + 4503599627370496.0) & 0x7fffffffLL);
#else
  return static_cast<int>(w);
#endif
}
TISO_HD int small_int(float w) {
#if defined(__CUDA_ARCH__)
  return __float_as_int(w + 8388608.0f) & 0x7fffff;
#else
  return static_cast<int>(w);
#endif
}

template <typename S>
TISO_HD S count_as(int v);
template <>
TISO_HD double count_as<double>(int v) { return small_double(v); }
template <>
TISO_HD float count_as<float>(int v) { return small_float(v); }

// The offset y0 that a row's values are fitted relative to (y - y0; the fit is y0 plus the fit
// of those). Pooling decisions do not depend on it; the exactness of the sums does. From the
// row's first element v: if |v| >= 1, v cut to 8 significant bits, else 0. Cutting keeps the
// last bit of y0 coarse (>= 2^-7), so that y - y0 has no lower bits than y itself unless y is
// 2^16 times larger than v; and data close to a large value (1e6 + small) become small numbers
// whose products with float32 weights and their sums stay exact in double. NaN and infinity give
// 0 (such rows are NaN, or not meaningful, either way).
TISO_HD double offset_of(double v) {
  if (!(fabs_(v) >= 1.0) || fabs_(v) > 1.7976931348623157e308) return 0.0;
#if defined(__CUDA_ARCH__)
  return __longlong_as_double(__double_as_longlong(v) & ~((1LL << 45) - 1));
#else
  long long b;
  __builtin_memcpy(&b, &v, 8);
  b &= ~((1LL << 45) - 1);
  double r;
  __builtin_memcpy(&r, &b, 8);
  return r;
#endif
}
TISO_HD float offset_of(float v) {
  if (!(v >= 1.0f || v <= -1.0f) || v > 3.4028234e38f || v < -3.4028234e38f) return 0.0f;
#if defined(__CUDA_ARCH__)
  return __int_as_float(__float_as_int(v) & ~((1 << 16) - 1));
#else
  int b;
  __builtin_memcpy(&b, &v, 4);
  b &= ~((1 << 16) - 1);
  float r;
  __builtin_memcpy(&r, &b, 4);
  return r;
#endif
}

// ---------------------------------------------------------------------------------------------
// The pool predicate of PAVA: block a (left) and block b (right), with weighted sums T and
// total weights W > 0, pool when mean(a) >= mean(b), i.e. Ta Wb >= Tb Wa - so equal means pool
// (the reference's merge test, src/torchisotonic/csrc/pava.h:46-55).
//
// In double: q = Tb Wa rounded, d = Ta Wb - q with one rounding (fma). The exact difference is
// d_exact - e with e = Tb Wa - q, |e| <= 2^-53 |q|; so |d| > 2^-52 |q| settles the sign. Else
// e is computed exactly (fma) and the sign taken from d - e: exact but for ties closer than
// about 2^-104 of the products - far closer than the data's own resolution. Equal products
// give d = e exactly, hence pooling. A NaN anywhere gives false (no pooling).
TISO_HD bool pool(double ta, double wa, double tb, double wb) {
  const double q = tb * wa;
  const double d = fma_(ta, wb, -q);
  if (fabs_(d) > 2.220446049250313e-16 * fabs_(q)) {
    return d > 0;
  }
  const double e = fma_(tb, wa, -q);
  return d >= e;
}

// The same decision without a branch, for loops whose threads must stay in step. With q as
// above, e = tb wa - q exactly (the rounding error of a product is a double) and d is
// ta wb - q rounded once, so D = ta wb - tb wa = (ta wb - q) - e. Rounding is monotone and e
// is a double: D >= 0 gives d >= e; D < 0 gives d <= e, with equality only when rounding
// ta wb - q moved it across e, i.e. |D| <= 2^-53 |ta wb - q| <= ~2^-106 |q|.
TISO_HD bool pool_nb(double ta, double wa, double tb, double wb) {
  const double q = tb * wa;
  const double d = fma_(ta, wb, -q);
  const double e = fma_(tb, wa, -q);
  return d >= e;
}

// exact=False on float32: single-precision sums and a plain comparison.
TISO_HD bool pool(float ta, float wa, float tb, float wb) { return ta * wb >= tb * wa; }
TISO_HD bool pool_nb(float ta, float wa, float tb, float wb) { return ta * wb >= tb * wa; }

// ---------------------------------------------------------------------------------------------
// q = n / d for 0 <= n < 2^31 and a divisor d fixed for a launch (Granlund & Montgomery's
// multiply-high method, "Division by invariant integers using multiplication", 1994, with a
// 33-bit magic number m + 2^32): q = (umulhi(n, m) + n) >> s.
struct FastDiv {
  uint32_t d, m, s;
};

inline FastDiv make_fastdiv(uint32_t d) {
  FastDiv f{d, 0, 0};
  uint32_t s = 0;
  while ((uint64_t{1} << s) < d) ++s;
  f.s = s;
  // m = floor(2^32 (2^s - d) / d) + 1
  f.m = static_cast<uint32_t>(((uint64_t{1} << 32) * ((uint64_t{1} << s) - d)) / d + 1);
  return f;
}

TISO_HD uint32_t fastdiv(uint32_t n, const FastDiv& f) {
#if defined(__CUDA_ARCH__)
  const uint32_t hi = __umulhi(n, f.m);
#else
  const uint32_t hi = static_cast<uint32_t>((static_cast<uint64_t>(n) * f.m) >> 32);
#endif
  return static_cast<uint32_t>((static_cast<uint64_t>(hi) + n) >> f.s);
}

}  // namespace tiso
