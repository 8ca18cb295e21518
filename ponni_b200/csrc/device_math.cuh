// Per-dtype arithmetic of the tile kernel.
//
// Storage type T is the model's `real` (float, double, half_t, bhalf_t in the
// reference, src/ponni_create_model.h:70-98).  Compute type C is float for the
// 16-bit types and T otherwise.  Every reference operation on `real` rounds to
// `real`, so the 16-bit paths round after each operation (rnd()), which is the
// behaviour of Kokkos half_t/bhalf_t arithmetic; the transcendental functions
// are evaluated in float and rounded once, as PONNI's TwoHalf does for every
// non-linear function (reference src/utils/ponni_TwoHalf.h:138-370).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "activation.cuh"
#include "program.h"

namespace ponni_b200 {

template <class T> struct Num;
template <> struct Num<float> {
  using C = float;
  static __device__ __forceinline__ float to_c(float x) { return x; }
  static __device__ __forceinline__ float from_c(float x) { return x; }
};
template <> struct Num<double> {
  using C = double;
  static __device__ __forceinline__ double to_c(double x) { return x; }
  static __device__ __forceinline__ double from_c(double x) { return x; }
};
template <> struct Num<__half> {
  using C = float;
  static __device__ __forceinline__ float to_c(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_c(float x) { return __float2half_rn(x); }
};
template <> struct Num<__nv_bfloat16> {
  using C = float;
  static __device__ __forceinline__ float to_c(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_c(float x) { return __float2bfloat16_rn(x); }
};

// Round a compute-type value to the storage type and back.
template <class T>
__device__ __forceinline__ typename Num<T>::C rnd(typename Num<T>::C x) {
  return Num<T>::to_c(Num<T>::from_c(x));
}

}  // namespace ponni_b200
