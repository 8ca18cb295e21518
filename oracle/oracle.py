"""ctypes wrapper of oracle/_build/libponni_oracle.so (test infrastructure only).

`forward(layers, dtype, x)` runs the plain-C restatement of the reference's
per-sample traversal (oracle/ponni_oracle.c) on host arrays.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_build", "libponni_oracle.so")
_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        h = ctypes.CDLL(LIB)
        h.ponni_oracle_forward.restype = ctypes.c_int
        h.ponni_oracle_forward.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                           ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                           ctypes.c_int]
        h.ponni_oracle_forward_ex.restype = ctypes.c_int
        h.ponni_oracle_forward_ex.argtypes = h.ponni_oracle_forward.argtypes + [ctypes.c_int]
        for name in ("ponni_oracle_round_f16", "ponni_oracle_round_bf16"):
            getattr(h, name).restype = ctypes.c_float
            getattr(h, name).argtypes = [ctypes.c_float]
        _lib = h
    return _lib


def forward(layers, dtype: int, x: np.ndarray, nthreads: int = 0, acc32: bool = False,
            generated: bool = False) -> np.ndarray:
    """x: host array in the model dtype's storage ([nin, batch]; bf16 as uint16 bits).
    acc32: fp32-accumulation semantics (tensor-core path of 16-bit models).
    generated: the generated-model arithmetic (bias-first sums, fused 16-bit
    multiply-adds; src/generator/kokkos_nn/emitter.py:704-708, :975-983)."""
    from ponni_b200.inference import build_descriptors

    descs, keep = build_descriptors(layers, dtype)
    x = np.ascontiguousarray(x)
    out = np.empty((layers[-1].num_outputs, x.shape[1]), dtype=x.dtype)
    rc = lib().ponni_oracle_forward_ex(ctypes.cast(descs, ctypes.c_void_p), len(layers), dtype, x.ctypes.data,
                                       x.shape[1], out.ctypes.data, x.shape[1], x.shape[1], nthreads,
                                       int(acc32) | (int(generated) << 1))
    if rc != 0:
        raise RuntimeError(f"oracle failed ({rc})")
    del keep
    return out
