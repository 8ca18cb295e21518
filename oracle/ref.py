"""ctypes wrapper of oracle/_ref/libponni_ref.so (test infrastructure only).

That library is the reference's own template inference code (its unmodified
headers) compiled against the host Kokkos shim in oracle/kokkos_shim/, for
the network structures oracle/ref_driver.cpp instantiates.  `available()` is
False where it was not built (no reference checkout).

`forward(layers, dtype, x)` runs Inference::forward_batch_parallel of the
reference on host arrays, with the weights of `layers` loaded through the
reference's set_trainable_parameters.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_ref", "libponni_ref.so")
_lib = None


def available() -> bool:
    return os.path.exists(LIB)


def lib():
    global _lib
    if _lib is None:
        h = ctypes.CDLL(LIB)
        h.ponni_ref_forward.restype = ctypes.c_int
        h.ponni_ref_forward.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                        ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
                                        ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int]
        _lib = h
    return _lib


def network_of(layers):
    """(network name, Matvec widths) of a layer list that ref_driver.cpp
    instantiates, or None."""
    names = [type(l).__name__ for l in layers]
    mv = [l for l in layers if type(l).__name__ == "Matvec"]
    dims = [mv[0].num_inputs] + [m.num_outputs for m in mv]
    for act, net in (("Relu", "mlp_relu"), ("Silu", "mlp_silu")):
        n = len(mv)
        if 2 <= n <= 8 and names == ["Matvec", "Bias", act] * (n - 1) + ["Matvec", "Bias"]:
            return net, dims
    block = ["Save_State", "LayerNorm", "Matvec", "Bias", "Gelu", "Matvec", "Bias", "Binop_Add"]
    if names == ["Matvec", "Bias"] + block * 4 + ["Matvec", "Bias"]:
        w = mv[0].num_outputs
        if all(m.num_inputs == w for m in mv[1:]) and all(m.num_outputs == w for m in mv[:-1]):
            ln = [l for l in layers if type(l).__name__ == "LayerNorm"]
            gelu = [l for l in layers if type(l).__name__ == "Gelu"]
            if all(abs(l.scalar[0] - 1e-5) < 1e-12 for l in ln) and all(not (g.flags & 0x2) for g in gelu):
                return "resmlp", [mv[0].num_inputs, w, mv[-1].num_outputs]
    if names == ["Matvec", "Bias", "LeakyRelu"] and abs(layers[2].scalar[0] - 0.1) < 1e-12:
        return "ones", dims
    head = ["Matvec", "Bias", "Elu", "Save_State", "Selu"]
    rest = ["Softplus", "Matvec", "Gelu", "Gelu", "Mish", "LayerNorm", "HardSigmoid", "HardSwish", "Binop_Add",
            "Save_State", "Sigmoid", "Tanh", "Silu", "MinMaxNorm", "Binop_Concatenate", "Relu", "LeakyRelu",
            "Save_State", "Softmax", "Binop_Projection_Add", "LogSoftmax", "Matvec", "Bias"]
    for h in (head, ["Matvec", "Bias", "Save_State"]):  # the 16-bit instantiation has no ELU / SELU
        if names != h + rest:
            continue
        s = [tuple(l.scalar) for l in layers]
        o = len(h)  # index of Softplus
        want = {o: (1.5,), o + 6: (0.2, 0.5), o + 13: (-1.0, 2.0, 1e-12), o + 16: (0.05,)}
        if h is head:
            want[2] = (0.7,)
        ok = all(all(abs(s[i][k] - v) < 1e-15 for k, v in enumerate(w)) for i, w in want.items())
        ok = ok and not (layers[o + 2].flags & 0x2) and bool(layers[o + 3].flags & 0x2) and abs(s[o + 5][0] - 1e-5) < 1e-15
        ok = ok and bool(layers[o + 14].flags & 0x4) and [l.save_index for l in layers
                                                          if l.save_index >= 0] == [0, 0, 1, 1, 2, 2]
        if ok:
            return "all_kinds", [mv[0].num_inputs, mv[0].num_outputs, mv[-1].num_outputs]
    return None


def forward(layers, dtype: int, x: np.ndarray, nthreads: int = 0) -> np.ndarray:
    """x: host array in the model dtype's storage ([nin, batch]; 16-bit types
    as uint16 bits).  Raises ValueError for a structure the driver does not
    instantiate."""
    net = network_of(layers)
    if net is None:
        raise ValueError("network structure not instantiated by oracle/ref_driver.cpp")
    name, dims = net
    # trainable parameters in tuple order (Inference::set_trainable_parameters)
    params = np.concatenate([np.zeros(0)] + [np.asarray(l.parameters(), np.float64).reshape(-1) for l in layers
                                             if getattr(l, "flags", 0) & 1])
    # the model-dtype values (the reference model holds `real` parameters)
    from ponni_b200.inference import from_dtype_bytes, to_dtype_bytes
    params = np.ascontiguousarray(from_dtype_bytes(to_dtype_bytes(params, dtype), dtype), np.float64)
    d = np.ascontiguousarray(dims, np.int32)
    x = np.ascontiguousarray(x)
    out = np.empty((layers[-1].num_outputs, x.shape[1]), dtype=x.dtype)
    rc = lib().ponni_ref_forward(name.encode(), dtype, d.size, d.ctypes.data, params.ctypes.data, params.size,
                                 x.ctypes.data, x.shape[1], out.ctypes.data, out.shape[1], x.shape[1], nthreads)
    if rc != 0:
        raise RuntimeError(f"reference forward failed ({rc})")
    return out
