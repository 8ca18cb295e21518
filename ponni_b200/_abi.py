"""ctypes binding of libponni_b200 (include/ponni_b200.h).

The shared library is built in-tree (``ponni_b200/libponni_b200.so``) by
``__graft_entry__.build()`` / ``make -C ponni_b200/csrc``.  There is no
fallback: when the library is missing every model call raises.
"""
from __future__ import annotations

import ctypes
import os

# PONNI_B200_LIB selects another build of the library (e.g. an instrumented one).
LIB_PATH = os.environ.get("PONNI_B200_LIB") or os.path.join(os.path.dirname(os.path.abspath(__file__)),
                                                             "libponni_b200.so")

# ponni_b200_status
OK = 0
STATUS_NAMES = {
    0: "OK", 1: "INVALID_ARGUMENT", 2: "VALIDATION", 3: "UNSUPPORTED", 4: "CUDA",
    5: "IO", 6: "MISMATCH", 7: "DEVICE",
}

# ponni_b200_dtype
F32, F64, F16, BF16 = 0, 1, 2, 3

# ponni_b200_layer_kind
(MATVEC, BIAS, RELU, LEAKY_RELU, ELU, SELU, GELU, SILU, SIGMOID, TANH, SOFTPLUS, HARD_SIGMOID,
 HARD_SWISH, MISH, LAYER_NORM, MIN_MAX_NORM, SOFTMAX, LOG_SOFTMAX, SAVE_STATE, BINOP_ADD,
 BINOP_CONCATENATE, BINOP_PROJECTION_ADD) = range(22)

ARITH_AUTO, ARITH_REFERENCE, ARITH_TENSOR, ARITH_GENERATED = 0, 1, 2, 3
KERNEL_TILE, KERNEL_TENSOR, KERNEL_NARROW, KERNEL_NARROW_JIT, KERNEL_TENSOR_STREAM, KERNEL_TENSOR_RESID = 1, 2, 3, 4, 5, 6

FLAG_TRAINABLE = 0x1
FLAG_APPROXIMATE = 0x2
FLAG_AFTER = 0x4


class LayerDesc(ctypes.Structure):
    _fields_ = [
        ("kind", ctypes.c_int32),
        ("num_inputs", ctypes.c_int32),
        ("num_outputs", ctypes.c_int32),
        ("save_index", ctypes.c_int32),
        ("aux", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("scalar", ctypes.c_double * 3),
        ("params", ctypes.c_void_p),
    ]


# Every function include/ponni_b200.h declares: name -> (restype, argtypes).
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_STATUS = ctypes.c_int
SIGNATURES = {
    "ponni_b200_abi_version": (_I, []),
    "ponni_b200_device_count": (_STATUS, [ctypes.POINTER(_I)]),
    "ponni_b200_model_create": (_STATUS, [ctypes.POINTER(LayerDesc), _I, _I, _I, ctypes.POINTER(_P)]),
    "ponni_b200_model_destroy": (None, [_P]),
    "ponni_b200_last_error": (ctypes.c_char_p, [_P]),
    "ponni_b200_create_error": (ctypes.c_char_p, []),
    "ponni_b200_model_validate": (_STATUS, [_P]),
    "ponni_b200_num_inputs": (_I, [_P]),
    "ponni_b200_num_outputs": (_I, [_P]),
    "ponni_b200_num_layers": (_I, [_P]),
    "ponni_b200_model_dtype": (_I, [_P]),
    "ponni_b200_model_stream": (_P, [_P]),
    "ponni_b200_model_set_stream": (_STATUS, [_P, _P]),
    "ponni_b200_model_synchronize": (_STATUS, [_P]),
    "ponni_b200_model_set_arithmetic": (_STATUS, [_P, _I]),
    "ponni_b200_model_kernel": (_I, [_P]),
    "ponni_b200_model_specialised": (_I, [_P, ctypes.POINTER(ctypes.c_char_p)]),
    "ponni_b200_model_device_program": (_I, [_P, ctypes.POINTER(_P), ctypes.POINTER(_P), ctypes.POINTER(_I),
                                            ctypes.POINTER(_I)]),
    "ponni_b200_model_diagnostics": (_STATUS, [_P, ctypes.POINTER(ctypes.c_uint64), _I]),
    "ponni_b200_forward": (_STATUS, [_P, _P, _I64, _P, _I64, _I64, _P]),
    "ponni_b200_forward_host": (_STATUS, [_P, _P, _I64, _P, _I64, _I64]),
    "ponni_b200_forward_host_static": (_STATUS, [_P, _P, _I64, _P, _I64, _I64]),
    "ponni_b200_reallocate_internal_state": (_STATUS, [_P, _I64]),
    "ponni_b200_internal_state_capacity": (_I64, [_P]),
    "ponni_b200_planned_temporary_size": (_I, [_P, _I]),
    "ponni_b200_saved_state_size": (_I, [_P, _I]),
    "ponni_b200_num_saved_states": (_I, [_P]),
    "ponni_b200_scratch_bytes": (_I64, [_P]),
    "ponni_b200_num_trainable_parameters": (_I64, [_P]),
    "ponni_b200_set_trainable_parameters": (_STATUS, [_P, _P, _I64]),
    "ponni_b200_get_trainable_parameters": (_STATUS, [_P, _P, _I64]),
    "ponni_b200_set_trainable_parameters_device": (_STATUS, [_P, _P, ctypes.c_int, _I64, _P]),
    "ponni_b200_get_trainable_parameters_device": (_STATUS, [_P, _P, ctypes.c_int, _I64, _P]),
    "ponni_b200_check_parameters": (_STATUS, [_P, ctypes.POINTER(_I64), ctypes.POINTER(_I64)]),
    "ponni_b200_weight_schema_fingerprint": (_STATUS, [_P, ctypes.c_char_p, ctypes.c_size_t]),
    "ponni_b200_model_save_weights": (_STATUS, [_P, ctypes.c_char_p]),
    "ponni_b200_model_load_weights": (_STATUS, [_P, ctypes.c_char_p]),
    "ponni_b200_read_ponni_tensor": (_STATUS, [ctypes.c_char_p, ctypes.c_char_p, _P, ctypes.c_size_t,
                                               ctypes.POINTER(_I64), ctypes.POINTER(_I), ctypes.c_char_p,
                                               ctypes.c_size_t]),
    "ponni_b200_model_summary": (_STATUS, [_P, ctypes.c_char_p, ctypes.c_size_t]),
    "ponni_b200_fill_synthetic": (_STATUS, [_I, _P, _I64, _I64, _I64, _I64, ctypes.c_uint64, _I,
                                            ctypes.c_double, ctypes.c_double, _P]),
}

_lib = None


def lib():
    """Load libponni_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"libponni_b200.so not found at {LIB_PATH}: build it with "
                "`python -c 'import __graft_entry__ as g; g.build()'` (no CPU fallback exists)")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


class PonniError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"ponni_b200 {STATUS_NAMES.get(status, status)}: {message}")
        self.status = status
        self.message = message
