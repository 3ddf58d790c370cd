// Semiring definitions shared by every kernel of the engine.
//
// Each semiring S provides, for a scalar type T:
//   zero()          the semiring zero, which is also the accumulator start
//   mul(a, b)       the semiring product (the reference's MUL_OP)
//   better(p, acc)  strict improvement test used by the argmax kernels
//   reduce(acc, p)  the value-only accumulation used by the plain kernels
//
// Float semantics follow crates/tropical-gemm-cuda/kernels/tropical_gemm.cu
// (instantiations :1043-1060): MaxPlus uses +, fmaxf, -inf; MinPlus uses +,
// fminf, +inf; MaxMul uses *, fmaxf, 0.  Integer semantics follow the
// reference GPU sentinels (:15-21) and saturating adds (:33-50): a product
// whose operand equals the sentinel is the sentinel; MaxMul multiplies with
// wrap-around.  The CPU crate's own ring definitions
// (crates/tropical-gemm/src/types/{max_plus,min_plus,max_mul}.rs) agree for
// floats, including the strict tie rule.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace tg {

constexpr int32_t kInfI32 = 46340;
constexpr int64_t kInfI64 = 3037000499LL;

enum SemiringId { kMaxPlus = 0, kMinPlus = 1, kMaxMul = 2 };

template <int S, typename T> struct Ring;

// ---------------------------------------------------------------- floats
template <typename T> __device__ __forceinline__ T pos_inf();
template <> __device__ __forceinline__ float pos_inf<float>() { return __int_as_float(0x7f800000); }
template <> __device__ __forceinline__ double pos_inf<double>() { return __longlong_as_double(0x7ff0000000000000LL); }

template <typename T> struct Ring<kMaxPlus, T> {
  static __device__ __forceinline__ T zero() { return -pos_inf<T>(); }
  static __device__ __forceinline__ T mul(T a, T b) { return a + b; }
  static __device__ __forceinline__ bool better(T p, T acc) { return p > acc; }
  static __device__ __forceinline__ T reduce(T acc, T p) { return fmax(acc, p); }
};
template <typename T> struct Ring<kMinPlus, T> {
  static __device__ __forceinline__ T zero() { return pos_inf<T>(); }
  static __device__ __forceinline__ T mul(T a, T b) { return a + b; }
  static __device__ __forceinline__ bool better(T p, T acc) { return p < acc; }
  static __device__ __forceinline__ T reduce(T acc, T p) { return fmin(acc, p); }
};
template <typename T> struct Ring<kMaxMul, T> {
  static __device__ __forceinline__ T zero() { return T(0); }
  static __device__ __forceinline__ T mul(T a, T b) { return a * b; }
  static __device__ __forceinline__ bool better(T p, T acc) { return p > acc; }
  static __device__ __forceinline__ T reduce(T acc, T p) { return fmax(acc, p); }
};

// ---------------------------------------------------------------- integers
#define TG_INT_RINGS(T, INF)                                                         \
  template <> struct Ring<kMaxPlus, T> {                                             \
    static __device__ __forceinline__ T zero() { return -(INF); }                    \
    static __device__ __forceinline__ T mul(T a, T b) {                              \
      return (a == -(INF) || b == -(INF)) ? T(-(INF)) : T((unsigned long long)a + (unsigned long long)b);                    \
    }                                                                                \
    static __device__ __forceinline__ bool better(T p, T acc) { return p > acc; }   \
    static __device__ __forceinline__ T reduce(T acc, T p) { return acc > p ? acc : p; } \
  };                                                                                 \
  template <> struct Ring<kMinPlus, T> {                                             \
    static __device__ __forceinline__ T zero() { return (INF); }                     \
    static __device__ __forceinline__ T mul(T a, T b) {                              \
      return (a == (INF) || b == (INF)) ? T(INF) : T((unsigned long long)a + (unsigned long long)b);                         \
    }                                                                                \
    static __device__ __forceinline__ bool better(T p, T acc) { return p < acc; }   \
    static __device__ __forceinline__ T reduce(T acc, T p) { return acc < p ? acc : p; } \
  };                                                                                 \
  template <> struct Ring<kMaxMul, T> {                                              \
    static __device__ __forceinline__ T zero() { return T(0); }                      \
    static __device__ __forceinline__ T mul(T a, T b) {                              \
      return T((unsigned long long)a * (unsigned long long)b);                       \
    }                                                                                \
    static __device__ __forceinline__ bool better(T p, T acc) { return p > acc; }   \
    static __device__ __forceinline__ T reduce(T acc, T p) { return acc > p ? acc : p; } \
  };

TG_INT_RINGS(int32_t, kInfI32)
TG_INT_RINGS(int64_t, kInfI64)
#undef TG_INT_RINGS

}  // namespace tg
