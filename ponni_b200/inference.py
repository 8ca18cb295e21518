"""Python host mirror of ponni::Inference and the create_inference_model factories.

Reference: src/ponni_Inference.h (Inference), src/ponni_create_model.h
(factories).  Names, argument meaning and error behaviour follow the
reference: where the reference calls Kokkos::abort this raises PonniError with
the reference's message; `load_weights`/`save_weights` return (ok, error)
like the reference's `bool f(path, std::string* error)`.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _abi
from .layers import Layer

_DTYPE_NAMES = {"float32": _abi.F32, "float": _abi.F32, "f32": _abi.F32, "float64": _abi.F64,
                "double": _abi.F64, "f64": _abi.F64, "float16": _abi.F16, "half": _abi.F16, "f16": _abi.F16,
                "bfloat16": _abi.BF16, "bhalf": _abi.BF16, "bf16": _abi.BF16}
_NP_STORAGE = {_abi.F32: np.float32, _abi.F64: np.float64, _abi.F16: np.float16, _abi.BF16: np.uint16}


def dtype_code(dtype) -> int:
    if isinstance(dtype, int):
        return dtype
    s = str(dtype).replace("torch.", "")
    if s in _DTYPE_NAMES:
        return _DTYPE_NAMES[s]
    raise ValueError(f"unsupported dtype {dtype!r}")


def bf16_bits(f32: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns (uint16), round to nearest even.
    32-bit arithmetic: u + 0x7FFF + lsb cannot wrap below the NaN patterns,
    which are replaced afterwards (quiet NaN, payload kept)."""
    u = np.ascontiguousarray(f32, dtype=np.float32).view(np.uint32)
    r = u >> 16
    r &= 1
    r += 0x7FFF
    r += u
    r >>= 16
    out = r.astype(np.uint16)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    if nan.any():
        out[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return out


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def to_dtype_bytes(values, code: int) -> np.ndarray:
    """Round float64 values to the model dtype; returns the storage array (bf16 as uint16 bits)."""
    v = np.asarray(values, dtype=np.float64)
    shape = v.shape
    v = v.reshape(-1)
    if code == _abi.F32:
        out = v.astype(np.float32)
    elif code == _abi.F64:
        out = v.copy()
    elif code == _abi.F16:
        out = v.astype(np.float16)
    elif code == _abi.BF16:
        out = bf16_bits(v.astype(np.float32))
    else:
        raise ValueError(code)
    return out.reshape(shape)


def from_dtype_bytes(raw, code: int) -> np.ndarray:
    """Storage array -> float64 values (same shape)."""
    if code == _abi.BF16:
        a = np.asarray(raw)
        return bf16_to_f32(a.reshape(-1)).astype(np.float64).reshape(a.shape)
    return np.asarray(raw).astype(np.float64)


def torch_stream_handle(device) -> int:
    """The current torch stream as a cudaStream_t for the C ABI.  torch's
    default stream is the legacy NULL stream; the C ABI reads NULL as "the
    model's own stream", so the legacy stream is passed as cudaStreamLegacy."""
    import torch
    index = device.index if isinstance(device, torch.device) else int(device)
    try:  # the raw handle without building a Stream object (per-call cost)
        h = torch._C._cuda_getCurrentRawStream(index)
    except AttributeError:
        h = torch.cuda.current_stream(index).cuda_stream
    return h if h else 0x1


def _check(status: int, model_ptr=None):
    if status != _abi.OK:
        L = _abi.lib()
        message = L.ponni_b200_last_error(model_ptr) if model_ptr else L.ponni_b200_create_error()
        raise _abi.PonniError(status, message.decode() if message else "")


def build_descriptors(layers, code: int):
    """Lower a layer list to (LayerDesc array, keep-alive buffers)."""
    descs = (_abi.LayerDesc * len(layers))()
    keep = []
    for i, L in enumerate(layers):
        if not isinstance(L, Layer):
            raise TypeError(f"layer {i} is not a ponni_b200 layer")
        d = descs[i]
        d.kind, d.num_inputs, d.num_outputs = L.kind, L.num_inputs, L.num_outputs
        d.save_index, d.aux, d.flags = L.save_index, L.aux, L.flags
        for k in range(3):
            d.scalar[k] = L.scalar[k]
        p = L.parameters()
        if p.size:
            raw = np.ascontiguousarray(to_dtype_bytes(p, code))
            keep.append(raw)
            d.params = raw.ctypes.data
        else:
            d.params = None
    return descs, keep


class Inference:
    """A model on one GPU; mirrors ponni::Inference (src/ponni_Inference.h:13-740)."""

    def __init__(self, layers, dtype=_abi.F32, device: int = 0, arithmetic: int | None = None):
        self.layers = list(layers)
        self.dtype = dtype_code(dtype)
        self.device = int(device)
        self._tdtype = None
        self._fwd = _abi.lib().ponni_b200_forward
        descs, keep = build_descriptors(self.layers, self.dtype)
        ptr = ctypes.c_void_p()
        _check(_abi.lib().ponni_b200_model_create(descs, len(self.layers), self.dtype, self.device,
                                                  ctypes.byref(ptr)))
        self._m = ptr
        if arithmetic is not None:
            self.set_arithmetic(arithmetic)

    def __del__(self):
        m = getattr(self, "_m", None)
        if m:
            try:
                _abi.lib().ponni_b200_model_destroy(m)
            except Exception:
                pass
            self._m = None

    # -- structure -----------------------------------------------------------
    @property
    def num_layers(self) -> int:
        return len(self.layers)

    def get_num_inputs(self) -> int:
        return self.layers[0].num_inputs

    def get_num_outputs(self) -> int:
        return self.layers[-1].num_outputs

    def validate(self) -> None:
        """Raise PonniError(VALIDATION) on a size mismatch (reference aborts)."""
        _check(_abi.lib().ponni_b200_model_validate(self._m), self._m)

    def summary(self) -> str:
        buf = ctypes.create_string_buffer(1 << 16)
        _check(_abi.lib().ponni_b200_model_summary(self._m, buf, len(buf)), self._m)
        return buf.value.decode()

    def print(self) -> None:
        print(self.summary(), end="")

    # -- forward -------------------------------------------------------------
    def forward_batch_parallel(self, input, output=None):
        """Run the model over the batch columns of `input` [num_inputs, batch].

        A CUDA torch tensor runs device-resident on the current torch stream
        (asynchronous, like the reference).  A numpy array or CPU torch tensor
        runs through the host pipeline and returns when the output is filled.
        """
        try:
            import torch
            if isinstance(input, torch.Tensor) and input.is_cuda:
                return self._forward_device(input, output)
        except ImportError:
            pass
        return self._forward_host(input, output)

    def _layout(self, t, rows, what):
        if t.dim() != 2 or t.shape[0] != rows:
            msg = ("Error: Provided # inputs differs from model's # inputs" if what == "input"
                   else "Error: Provided output dimensions do not match the model and input batch")
            raise _abi.PonniError(2, msg)
        if t.shape[1] > 1 and t.stride(1) != 1:
            raise _abi.PonniError(1, f"{what} must be LayoutRight (batch index contiguous)")

    def torch_dtype(self):
        import torch
        if self._tdtype is None:
            self._tdtype = {_abi.F32: torch.float32, _abi.F64: torch.float64, _abi.F16: torch.float16,
                            _abi.BF16: torch.bfloat16}[self.dtype]
        return self._tdtype

    def _forward_device(self, input, output):
        import torch

        nin, nout = self.get_num_inputs(), self.get_num_outputs()
        self._layout(input, nin, "input")
        if input.dtype != self.torch_dtype():
            raise _abi.PonniError(1, f"input dtype {input.dtype} does not match the model dtype")
        dev = input.device
        if dev.index != self.device:
            raise _abi.PonniError(1, f"input is on {dev}, the model on cuda:{self.device}")
        batch = input.shape[1]
        if batch == 0:
            raise _abi.PonniError(1, "Inference requires a nonzero batch size")
        if output is None:
            output = torch.empty((nout, batch), dtype=input.dtype, device=dev)
        else:
            self._layout(output, nout, "output")
            if output.shape[1] != batch or output.dtype != input.dtype:
                raise _abi.PonniError(2, "Error: Provided output dimensions do not match the model and input batch")
            if output.device != dev:
                raise _abi.PonniError(1, f"output is on {output.device}, the input on {dev}")
        _check(self._fwd(self._m, input.data_ptr(), input.stride(0), output.data_ptr(), output.stride(0), batch,
                         torch_stream_handle(self.device)), self._m)
        return output

    def _forward_host(self, input, output):
        try:
            import torch
            is_torch = isinstance(input, torch.Tensor)
        except ImportError:
            is_torch = False
        if is_torch:
            src = input
            if src.dtype != self.torch_dtype():
                raise _abi.PonniError(1, f"input dtype {src.dtype} does not match the model dtype")
            self._layout(src, self.get_num_inputs(), "input")
            batch = src.shape[1]
            if output is None:
                output = torch.empty((self.get_num_outputs(), batch), dtype=src.dtype, pin_memory=src.is_pinned())
            in_ptr, in_ld, out_ptr, out_ld = src.data_ptr(), src.stride(0), output.data_ptr(), output.stride(0)
        else:
            src = np.asarray(input)
            if src.ndim != 2 or src.shape[0] != self.get_num_inputs():
                raise _abi.PonniError(2, "Error: Provided # inputs differs from model's # inputs")
            want = _NP_STORAGE[self.dtype]
            if src.dtype != want:
                raise _abi.PonniError(1, f"input dtype {src.dtype} does not match the model dtype")
            src = np.ascontiguousarray(src)
            batch = src.shape[1]
            if output is None:
                output = np.empty((self.get_num_outputs(), batch), dtype=want)
            in_ptr, in_ld = src.ctypes.data, src.shape[1]
            out_ptr, out_ld = output.ctypes.data, output.strides[0] // output.itemsize
        if batch == 0:
            raise _abi.PonniError(1, "Inference requires a nonzero batch size")
        _check(_abi.lib().ponni_b200_forward_host(self._m, in_ptr, in_ld, out_ptr, out_ld, batch), self._m)
        return output

    def set_arithmetic(self, mode: int) -> None:
        """ARITH_AUTO (tensor cores where supported), ARITH_REFERENCE (tile
        kernel, the reference's operation order), ARITH_TENSOR (require the
        tensor-core kernel)."""
        _check(_abi.lib().ponni_b200_model_set_arithmetic(self._m, int(mode)), self._m)

    def specialised(self):
        """(True, "") when the next forward runs a kernel compiled for this model's
        structure at plan time (NVRTC), else (False, reason)."""
        why = ctypes.c_char_p()
        r = int(_abi.lib().ponni_b200_model_specialised(self._m, ctypes.byref(why)))
        return bool(r), (why.value or b"").decode()

    def kernel(self) -> int:
        """Kernel the next forward uses: 1 tile kernel, 2 tensor-core kernel (plans the model)."""
        k = int(_abi.lib().ponni_b200_model_kernel(self._m))
        if k == 0:
            raise _abi.PonniError(3, _abi.lib().ponni_b200_last_error(self._m).decode())
        return k

    def synchronize(self) -> None:
        _check(_abi.lib().ponni_b200_model_synchronize(self._m), self._m)

    # -- scratch -------------------------------------------------------------
    def reallocate_internal_state(self, batch_size: int) -> None:
        _check(_abi.lib().ponni_b200_reallocate_internal_state(self._m, int(batch_size)), self._m)

    def internal_state_capacity(self) -> int:
        return int(_abi.lib().ponni_b200_internal_state_capacity(self._m))

    def get_planned_temporary_size(self, which: int) -> int:
        return int(_abi.lib().ponni_b200_planned_temporary_size(self._m, int(which)))

    def get_saved_state_size(self, index: int) -> int:
        return int(_abi.lib().ponni_b200_saved_state_size(self._m, int(index)))

    def get_num_saved_states(self) -> int:
        return int(_abi.lib().ponni_b200_num_saved_states(self._m))

    def scratch_bytes(self) -> int:
        return int(_abi.lib().ponni_b200_scratch_bytes(self._m))

    # -- parameters ----------------------------------------------------------
    def get_num_trainable_parameters(self) -> int:
        return int(_abi.lib().ponni_b200_num_trainable_parameters(self._m))

    def get_trainable_parameters(self) -> np.ndarray:
        n = self.get_num_trainable_parameters()
        raw = np.empty(n, dtype=_NP_STORAGE[self.dtype])
        _check(_abi.lib().ponni_b200_get_trainable_parameters(self._m, raw.ctypes.data, n), self._m)
        return from_dtype_bytes(raw, self.dtype)

    def _sync_layers(self, values):
        off = 0
        for L in self.layers:
            k = L.get_num_trainable_parameters()
            if k:
                L.set_parameters(values[off:off + k])
                off += k

    def set_trainable_parameters(self, values) -> None:
        v = np.asarray(values, dtype=np.float64).reshape(-1)
        raw = np.ascontiguousarray(to_dtype_bytes(v, self.dtype))
        _check(_abi.lib().ponni_b200_set_trainable_parameters(self._m, raw.ctypes.data, v.size), self._m)
        self._sync_layers(v)

    # -- parameters in device memory (no re-plan) -----------------------------
    def _torch_code(self, t) -> int:
        import torch
        codes = {torch.float32: _abi.F32, torch.float64: _abi.F64, torch.float16: _abi.F16,
                 torch.bfloat16: _abi.BF16}
        if t.dtype not in codes:
            raise _abi.PonniError(1, f"parameter dtype {t.dtype} is not fp32, fp64, fp16 or bf16")
        return codes[t.dtype]

    def parameter_device(self):
        """The torch device of this model's parameters."""
        import torch
        return torch.device(f"cuda:{self.device}")

    def set_trainable_parameters_device(self, values) -> None:
        """Trainable parameters (tuple order) from a CUDA tensor of fp32, fp64,
        fp16 or bf16 on this model's device, converted to the model dtype and
        written into the planned device images on the current torch stream
        (generated set_parameters, emitter.py:1826-1866).  The Python layer
        objects keep their earlier values; get_trainable_parameters() reads
        the model."""
        if not (hasattr(values, "is_cuda") and values.is_cuda):
            raise _abi.PonniError(1, "set_trainable_parameters_device needs a CUDA tensor")
        if values.device.index != self.device:
            raise _abi.PonniError(1, f"parameters are on {values.device}, the model on cuda:{self.device}")
        v = values.reshape(-1)
        if not v.is_contiguous():
            v = v.contiguous()
        _check(_abi.lib().ponni_b200_set_trainable_parameters_device(
            self._m, v.data_ptr(), self._torch_code(v), v.numel(), torch_stream_handle(self.device)), self._m)

    def get_trainable_parameters_device(self, dtype=None):
        """Trainable parameters (tuple order) as a CUDA tensor of `dtype`
        (default: the model dtype), on the current torch stream."""
        import torch
        dt = self.torch_dtype() if dtype is None else dtype
        out = torch.empty(self.get_num_trainable_parameters(), dtype=dt, device=f"cuda:{self.device}")
        _check(_abi.lib().ponni_b200_get_trainable_parameters_device(
            self._m, out.data_ptr(), self._torch_code(out), out.numel(), torch_stream_handle(self.device)), self._m)
        return out

    def check_parameters(self) -> tuple[int, int]:
        """(device image locations that disagree with the parameters,
        trainable values that are not finite)."""
        mism, nonfinite = ctypes.c_int64(), ctypes.c_int64()
        _check(_abi.lib().ponni_b200_check_parameters(self._m, ctypes.byref(mism), ctypes.byref(nonfinite)), self._m)
        return int(mism.value), int(nonfinite.value)

    def parameters_synchronized(self) -> bool:
        return self.check_parameters()[0] == 0

    def parameters_are_finite(self) -> bool:
        return self.check_parameters()[1] == 0

    def weight_schema_fingerprint(self) -> str:
        buf = ctypes.create_string_buffer(64)
        _check(_abi.lib().ponni_b200_weight_schema_fingerprint(self._m, buf, len(buf)), self._m)
        return buf.value.decode()

    def save_weights(self, path: str):
        s = _abi.lib().ponni_b200_model_save_weights(self._m, str(path).encode())
        if s != _abi.OK:
            return False, _abi.lib().ponni_b200_last_error(self._m).decode()
        return True, ""

    def load_weights(self, path: str):
        s = _abi.lib().ponni_b200_model_load_weights(self._m, str(path).encode())
        if s != _abi.OK:
            return False, _abi.lib().ponni_b200_last_error(self._m).decode()
        self._sync_layers(self.get_trainable_parameters())
        return True, ""


def create_inference_model(*layers, dtype=_abi.F32, device: int = 0) -> Inference:
    """ponni::create_inference_model (src/ponni_create_model.h:41-66): float model."""
    return Inference(layers, dtype=dtype, device=device)


def create_inference_model_single_precision(*layers, device: int = 0) -> Inference:
    return Inference(layers, dtype=_abi.F32, device=device)


def create_inference_model_double_precision(*layers, device: int = 0) -> Inference:
    return Inference(layers, dtype=_abi.F64, device=device)


def create_inference_model_half_precision(*layers, device: int = 0) -> Inference:
    return Inference(layers, dtype=_abi.F16, device=device)


def create_inference_model_bhalf_precision(*layers, device: int = 0) -> Inference:
    return Inference(layers, dtype=_abi.BF16, device=device)
