// Packed fp32 pair arithmetic for sm_100a (add/sub/mul/fma .rn.f32x2): one
// instruction rounds two independent IEEE fp32 operations, each exactly as
// its scalar form (no contraction unless fma is asked for), so results are
// bit-identical to the scalar code they replace while the epilogues issue
// half as many FP32 instructions.
#pragma once

namespace ponni_b200 {
namespace f2 {

#define PONNI_B200_F32X2_BIN(name, op)                                                                  \
  __device__ __forceinline__ void name(float& d0, float& d1, float a0, float a1, float b0, float b1) { \
    asm("{\n\t.reg .b64 x, y, z;\n\t"                                                                   \
        "mov.b64 x, {%2, %3};\n\t"                                                                      \
        "mov.b64 y, {%4, %5};\n\t" op                                                                   \
        " z, x, y;\n\t"                                                                                 \
        "mov.b64 {%0, %1}, z;\n\t}\n"                                                                   \
        : "=f"(d0), "=f"(d1)                                                                            \
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1));                                                          \
  }

PONNI_B200_F32X2_BIN(add, "add.rn.f32x2")
PONNI_B200_F32X2_BIN(sub, "sub.rn.f32x2")
PONNI_B200_F32X2_BIN(mul, "mul.rn.f32x2")
#undef PONNI_B200_F32X2_BIN

// d = a * b + c, one rounding per lane.
__device__ __forceinline__ void fma(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0, float c1) {
  asm("{\n\t.reg .b64 x, y, z, w;\n\t"
      "mov.b64 x, {%2, %3};\n\t"
      "mov.b64 y, {%4, %5};\n\t"
      "mov.b64 z, {%6, %7};\n\t"
      "fma.rn.f32x2 w, x, y, z;\n\t"
      "mov.b64 {%0, %1}, w;\n\t}\n"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}

// v[i] += w[i] over an even-length array.
template <int N>
__device__ __forceinline__ void add_n(float (&v)[N], const float (&w)[N]) {
  static_assert(N % 2 == 0, "even length");
#pragma unroll
  for (int j = 0; j < N; j += 2) add(v[j], v[j + 1], v[j], v[j + 1], w[j], w[j + 1]);
}

}  // namespace f2
}  // namespace ponni_b200
