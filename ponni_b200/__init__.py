"""ponni_b200 -- B200-native batched inference for PONNI models.

Host-side mirror of PONNI's template API (layers + create_inference_model +
Inference) over the C ABI of libponni_b200 (include/ponni_b200.h), whose
fused sm_100a kernel runs the whole layer chain per batch tile on chip.
"""
from . import _abi
from ._abi import PonniError, F32, F64, F16, BF16
from .layers import (Layer, Matvec, Bias, Relu, ReLU, LeakyRelu, LeakyReLU, Elu, ELU, Selu, SELU, Gelu,
                     GELU, Silu, SiLU, Sigmoid, Tanh, Softplus, HardSigmoid, HardSwish, Mish, LayerNorm,
                     MinMaxNorm, Softmax, LogSoftmax, Save_State, Binop_Add, Binop_Concatenate,
                     Binop_Projection_Add)
from .generated import Dense, GeneratedModel
from .generated import LayerNorm as GeneratedLayerNorm
from .inference import (Inference, create_inference_model, create_inference_model_single_precision,
                        create_inference_model_double_precision, create_inference_model_half_precision,
                        create_inference_model_bhalf_precision, build_descriptors, to_dtype_bytes,
                        from_dtype_bytes, bf16_bits, bf16_to_f32, dtype_code, torch_stream_handle)


def device_count() -> int:
    import ctypes
    n = ctypes.c_int(0)
    _abi.lib().ponni_b200_device_count(ctypes.byref(n))
    return n.value


def fill_synthetic(tensor, seed: int, col0: int = 0, dist: str = "normal", lo: float = -1.0, hi: float = 1.0):
    """Fill a CUDA tensor [rows, cols] with the counter-based synthetic inputs
    keyed by (seed, row, col0 + col), on the current torch stream."""
    code = dtype_code(tensor.dtype)
    rows, cols = tensor.shape
    st = _abi.lib().ponni_b200_fill_synthetic(code, tensor.data_ptr(), rows, cols, tensor.stride(0), col0,
                                              seed & 0xFFFFFFFFFFFFFFFF, 0 if dist == "normal" else 1,
                                              lo, hi, torch_stream_handle(tensor.device))
    if st != 0:
        raise PonniError(st, "fill_synthetic failed")
    return tensor
