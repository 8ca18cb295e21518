"""The reference's generated (AOT) model struct on libponni_b200.

PONNI's generator (src/generator/kokkos_nn/emitter.py) emits a C++ struct per
model with load_weights / infer_batch / infer_batch_half2 / infer_one /
get_parameters / set_parameters (emitter.py:1724-1955).  Its arithmetic
differs from the template path in two ways, both reproduced here through
ARITH_GENERATED:

* dense layers store W as [out, in] (the PyTorch / ONNX convention) and start
  each sum at the bias (emitter.py:704-708: ``Scalar sum = bias(i); sum +=
  W(i, j) * x(j)``);
* infer_batch_half2 takes and returns fp32 values but keeps fp16 parameters
  and accumulates with one fused multiply-add per product
  (TwoHalf::fma, emitter.py:975-983).

* LayerNormalization nodes run one Welford pass for the mean and second
  moment (emitter.py:867-889; the half2 path in float, :1161-1191) and
  output ((x - mean) * inv_stddev) * scale + bias.

The ONNX import and graph compiler of the generator are not rebuilt: a model
is given as the list of nodes the generator's passes produce for MLPs and
residual MLPs: ``Dense`` (Dense / DenseBiasActivation, and
DenseResidualActivation when it names a ``residual`` tensor: activation(W x +
b + residual), emitter.py:726-729) and ``LayerNorm`` (LayerNormalization).
A residual names an earlier node's output, or "input".  Named weights load
from a .ponni file as ``<name>.weight`` [out, in] and ``<name>.bias`` [out]
(LayerNorm: ``<name>.scale`` and ``<name>.bias``).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _abi
from . import layers as L
from .inference import Inference, from_dtype_bytes, to_dtype_bytes

_ACT = {
    None: None,
    "relu": lambda n, a: L.Relu(n),
    "leaky_relu": lambda n, a: L.LeakyRelu(n, a),
    "elu": lambda n, a: L.Elu(n, a),
    "selu": lambda n, a: L.Selu(n),
    "gelu": lambda n, a: L.Gelu(n),
    "gelu_tanh": lambda n, a: L.Gelu(n, True),
    "silu": lambda n, a: L.Silu(n),
    "sigmoid": lambda n, a: L.Sigmoid(n),
    "tanh": lambda n, a: L.Tanh(n),
    "softplus": lambda n, a: L.Softplus(n, 1.0),
    "hard_swish": lambda n, a: L.HardSwish(n),
    "mish": lambda n, a: L.Mish(n),
}


@dataclass
class Dense:
    """One fused dense node: y = activation(bias + W x [+ residual]), W[out, in]."""
    name: str
    weight: np.ndarray
    bias: np.ndarray | None = None
    activation: str | None = None
    alpha: float = 0.01  # LeakyReLU slope / ELU alpha
    residual: str | None = None  # DenseResidualActivation: name of an earlier node, or "input"

    @property
    def width_in(self) -> int:
        return self.weight.shape[1]

    @property
    def width_out(self) -> int:
        return self.weight.shape[0]

    def tensors(self):
        out = [("weight", self.weight)]
        if self.bias is not None:
            out.append(("bias", self.bias))
        return out

    def __post_init__(self):
        self.weight = np.asarray(self.weight, dtype=np.float64)
        if self.weight.ndim != 2:
            raise ValueError(f"{self.name}: weight must be [out, in]")
        if self.bias is not None:
            self.bias = np.asarray(self.bias, dtype=np.float64).reshape(-1)
            if self.bias.size != self.weight.shape[0]:
                raise ValueError(f"{self.name}: bias size differs from the output width")
        if self.activation not in _ACT:
            raise ValueError(f"{self.name}: unsupported activation {self.activation!r}")


@dataclass
class LayerNorm:
    """One LayerNormalization node over the feature vector: scale and bias [n]."""
    name: str
    scale: np.ndarray
    bias: np.ndarray
    epsilon: float = 1e-5

    def __post_init__(self):
        self.scale = np.asarray(self.scale, dtype=np.float64).reshape(-1)
        self.bias = np.asarray(self.bias, dtype=np.float64).reshape(-1)
        if self.scale.size != self.bias.size:
            raise ValueError(f"{self.name}: scale and bias sizes differ")

    @property
    def width_in(self) -> int:
        return self.scale.size

    @property
    def width_out(self) -> int:
        return self.scale.size

    def tensors(self):
        return [("scale", self.scale), ("bias", self.bias)]


def _read_tensor(path: str, name: str) -> np.ndarray:
    lib = _abi.lib()
    shape = (ctypes.c_int64 * 4)()
    rank = ctypes.c_int()
    err = ctypes.create_string_buffer(512)
    st = lib.ponni_b200_read_ponni_tensor(path.encode(), name.encode(), None, 0, shape, ctypes.byref(rank), err, 512)
    if st != 0:
        raise _abi.PonniError(st, err.value.decode())
    dims = [shape[i] for i in range(rank.value)]
    out = np.empty(int(np.prod(dims)) if dims else 1, dtype=np.float32)
    st = lib.ponni_b200_read_ponni_tensor(path.encode(), name.encode(), out.ctypes.data, out.size, shape,
                                          ctypes.byref(rank), err, 512)
    if st != 0:
        raise _abi.PonniError(st, err.value.decode())
    return out.reshape(dims)


class GeneratedModel:
    """Mirror of the generated model struct (``Scalar`` = float or double)."""

    def __init__(self, dense: list, scalar=np.float32, device: int = 0):
        if not dense:
            raise ValueError("a generated model needs at least one node")
        names = {"input"}
        for a, b in zip(dense, dense[1:]):
            if a.width_out != b.width_in:
                raise ValueError(f"{a.name} -> {b.name}: width mismatch")
        widths = {"input": dense[0].width_in}
        for n in dense:
            if n.name in names:
                raise ValueError(f"node name {n.name!r} used twice")
            if isinstance(n, Dense) and n.residual is not None:
                if n.residual not in names:
                    raise ValueError(f"{n.name}: residual {n.residual!r} is not an earlier node or the input")
                if widths[n.residual] != n.width_out:
                    raise ValueError(f"{n.name}: residual {n.residual!r} has width {widths[n.residual]}, "
                                     f"the node {n.width_out}")
            names.add(n.name)
            widths[n.name] = n.width_out
        self.dense = list(dense)  # the nodes, in order (Dense and LayerNorm)
        self.scalar = np.dtype(scalar)
        if self.scalar not in (np.dtype(np.float32), np.dtype(np.float64)):
            raise ValueError("GeneratedModel Scalar must be float or double")
        self.device = device
        self.num_inputs = self.dense[0].width_in
        self.num_outputs = self.dense[-1].width_out
        self._models: dict[int, Inference] = {}

    # -- parameters (emitter.py:1724-1895) --
    @staticmethod
    def _layer_list(dense, rnd=lambda a: a):
        """Lower the nodes to the template layer tuple: residual sources are
        saved (Save_State) where they are produced and added (Binop_Add)
        after the bias, before the activation."""
        sources = [n.residual for n in dense if isinstance(n, Dense) and n.residual is not None]
        slot = {name: i for i, name in enumerate(dict.fromkeys(sources))}
        out = []
        if "input" in slot:
            out.append(L.Save_State(dense[0].width_in, slot["input"]))
        for d in dense:
            if isinstance(d, LayerNorm):
                out.append(L.LayerNorm(rnd(d.scale), rnd(d.bias), d.epsilon))
            else:
                out.append(L.Matvec(rnd(d.weight).T))
                if d.bias is not None:
                    out.append(L.Bias(rnd(d.bias)))
                if d.residual is not None:
                    out.append(L.Binop_Add(d.width_out, slot[d.residual]))
                if d.activation is not None:
                    out.append(_ACT[d.activation](d.weight.shape[0], d.alpha))
            if d.name in slot:
                out.append(L.Save_State(d.width_out, slot[d.name]))
        return out

    def _trainable_order(self) -> np.ndarray:
        """Index of each trainable value (Inference tuple order: Matvec W[in][out],
        then the bias; LayerNorm gamma then beta) in the generated order
        (W[out, in], then the bias; scale then bias)."""
        if getattr(self, "_perm", None) is None:
            parts, g = [], 0
            for d in self.dense:
                if isinstance(d, LayerNorm):
                    parts.append(g + np.arange(2 * d.scale.size, dtype=np.int64))
                    g += 2 * d.scale.size
                    continue
                o, i = d.weight.shape
                parts.append(g + np.arange(o * i, dtype=np.int64).reshape(o, i).T.reshape(-1))
                g += o * i
                if d.bias is not None:
                    parts.append(g + np.arange(o, dtype=np.int64))
                    g += o
            self._perm = np.concatenate(parts)
        return self._perm

    def get_num_parameters(self) -> int:
        return int(sum(t.size for d in self.dense for _, t in d.tensors()))

    def get_parameters(self) -> np.ndarray:
        """Learned parameters in node order: W[out, in] row-major, then the
        bias (LayerNorm: scale, then bias)."""
        self._pull_dense()
        return np.concatenate([t.reshape(-1) for d in self.dense for _, t in d.tensors()]).astype(self.scalar)

    def set_parameters(self, values) -> None:
        v = np.asarray(values, dtype=np.float64).reshape(-1)
        if v.size != self.get_num_parameters():
            raise _abi.PonniError(2, "GeneratedModel::set_parameters source extent is incorrect")
        if not np.all(np.isfinite(v)):
            raise _abi.PonniError(2, "GeneratedModel::set_parameters received non-finite values")
        self._set_dense(v)
        # Planned models take the values into their device images (pinned
        # staging + device scatter, no re-plan); the fp16 mirror follows.
        self._dense_stale = False
        self._push_host()

    def _mirror_values(self, a):
        """The fp16 mirror is fp16(float(Scalar value)) (emitter.py:1742-1743, 1779-1783):
        round to Scalar and to float first, so that the final rounding to fp16
        is the only one left."""
        return np.asarray(a).astype(self.scalar).astype(np.float32).astype(np.float64)

    def _push_host(self):
        t = self.get_parameters().astype(np.float64)[self._trainable_order()]
        for dt, m in self._models.items():
            m.set_trainable_parameters(self._mirror_values(t) if dt == _abi.F16 else t)

    def _set_dense(self, v):
        off = 0
        for d in self.dense:
            for attr, t in d.tensors():
                setattr(d, attr, v[off:off + t.size].reshape(t.shape).copy())
                off += t.size

    def _scalar_dtype(self) -> int:
        return _abi.F32 if self.scalar == np.float32 else _abi.F64

    def _pull_dense(self):
        """After a device update the scalar model holds the parameters."""
        if getattr(self, "_dense_stale", False):
            t = self._models[self._scalar_dtype()].get_trainable_parameters()
            v = np.empty_like(t)
            v[self._trainable_order()] = t
            self._set_dense(v)
            self._dense_stale = False

    # -- device-resident parameters (emitter.py:1769-1895) --
    def set_parameters_device(self, values) -> None:
        """Learned parameters (generated order) from a CUDA tensor of fp32 or
        fp64: converted to Scalar and scattered into the scalar model's device
        images, then into the fp16 mirror (refresh_half_parameters), all on
        the device and the current torch stream."""
        import torch
        if not (isinstance(values, torch.Tensor) and values.is_cuda):
            raise _abi.PonniError(1, "set_parameters_device needs a CUDA tensor")
        if values.numel() != self.get_num_parameters():
            raise _abi.PonniError(2, "GeneratedModel::set_parameters source extent is incorrect")
        if getattr(self, "_perm_dev", None) is None or self._perm_dev.device != values.device:
            self._perm_dev = torch.from_numpy(self._trainable_order()).to(values.device)
        t = values.reshape(-1).index_select(0, self._perm_dev)
        self._model(self._scalar_dtype()).set_trainable_parameters_device(t)
        self._dense_stale = True
        self.refresh_half_parameters()

    def get_parameters_device(self, dtype=None):
        """Learned parameters (generated order) as a CUDA tensor."""
        import torch
        t = self._model(self._scalar_dtype()).get_trainable_parameters_device(dtype)
        if getattr(self, "_perm_dev", None) is None or self._perm_dev.device != t.device:
            self._perm_dev = torch.from_numpy(self._trainable_order()).to(t.device)
        out = torch.empty_like(t)
        out[self._perm_dev] = t
        return out

    def refresh_half_parameters(self) -> None:
        """fp16 mirror <- fp16(float(parameters)), device to device."""
        half = self._models.get(_abi.F16)
        if half is None:
            return
        scalar = self._model(self._scalar_dtype())
        half.set_trainable_parameters_device(scalar.get_trainable_parameters_device())

    def parameters_are_finite(self) -> bool:
        return self._model(self._scalar_dtype()).parameters_are_finite()

    def parameters_synchronized(self) -> bool:
        """Every device image agrees with the parameters, and the fp16 mirror
        holds fp16(float(parameters)) (emitter.py:1882-1895)."""
        import torch
        scalar = self._model(self._scalar_dtype())
        if not scalar.parameters_synchronized():
            return False
        half = self._models.get(_abi.F16)
        if half is None:
            return True
        if not half.parameters_synchronized():
            return False
        return bool(torch.equal(half.get_trainable_parameters_device(torch.float16),
                                scalar.get_trainable_parameters_device(torch.float16)))

    def load_weights(self, path: str) -> None:
        """Named tensors <name>.weight [out, in] and <name>.bias (LayerNorm:
        <name>.scale and <name>.bias) of a .ponni file."""
        for d in self.dense:
            for attr, t in d.tensors():
                v = _read_tensor(path, f"{d.name}.{attr}").astype(np.float64)
                if v.size != t.size or (attr == "weight" and v.shape != t.shape):
                    raise _abi.PonniError(2, f"{d.name}.{attr} has shape {v.shape}, expected {t.shape}")
                setattr(d, attr, v.reshape(t.shape))
        self._dense_stale = False
        self._push_host()

    # -- inference --
    def _model(self, dtype: int) -> Inference:
        m = self._models.get(dtype)
        if m is None:
            self._pull_dense()
            rnd = self._mirror_values if dtype == _abi.F16 else (lambda a: a)
            m = Inference(self._layer_list(self.dense, rnd), dtype=dtype, device=self.device,
                          arithmetic=_abi.ARITH_GENERATED)
            self._models[dtype] = m
        return m

    def infer_batch(self, inputs):
        """inputs [num_inputs, batch] in Scalar (numpy, or a CUDA torch tensor) -> outputs."""
        dt = _abi.F32 if self.scalar == np.float32 else _abi.F64
        return self._model(dt).forward_batch_parallel(inputs)

    def infer_batch_half2(self, inputs):
        """fp32 inputs -> fp32 outputs with fp16 parameters and fused fp16
        accumulation (the generated infer_batch_half2)."""
        m = self._model(_abi.F16)
        try:
            import torch
            if isinstance(inputs, torch.Tensor) and inputs.is_cuda:
                return m.forward_batch_parallel(inputs.to(torch.float16)).to(torch.float32)
        except ImportError:
            pass
        x = to_dtype_bytes(np.asarray(inputs, dtype=np.float64), _abi.F16)
        return from_dtype_bytes(m.forward_batch_parallel(x), _abi.F16).astype(np.float32)

    def infer_one(self, inputs) -> np.ndarray:
        x = np.asarray(inputs, dtype=self.scalar).reshape(self.num_inputs, 1)
        return np.asarray(self.infer_batch(x)).reshape(-1)
