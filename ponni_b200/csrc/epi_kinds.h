// Pointwise operation kinds (values match ponni_b200_layer_kind).  No
// includes: this header is also compiled at run time (NVRTC) into the
// model-specialised narrow kernel.
#pragma once

namespace ponni_b200 {

enum EpiKind : int {
  EPI_NONE = 0,
  EPI_BIAS = 1, EPI_RELU = 2, EPI_LEAKY_RELU = 3, EPI_ELU = 4, EPI_SELU = 5, EPI_GELU = 6,
  EPI_SILU = 7, EPI_SIGMOID = 8, EPI_TANH = 9, EPI_SOFTPLUS = 10, EPI_HARD_SIGMOID = 11,
  EPI_HARD_SWISH = 12, EPI_MISH = 13,
};

// Epilogue-entry flag: a 16-bit model evaluates this activation with the
// reference's own rounding points (activation16), not in float with one
// rounding (the generated model's half2 arithmetic).
constexpr int EPI_FLAG_REF16 = 0x100;

}  // namespace ponni_b200
