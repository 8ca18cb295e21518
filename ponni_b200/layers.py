"""Layer descriptors mirroring PONNI's template layer structs (src/layers/*.h).

Each class takes the reference constructor's arguments (the weights that the
reference passes as Kokkos Views are numpy arrays here, same shapes, same
row-major order) and lowers itself to one ``LayerDesc`` of the C ABI.
Parameters are kept in float64 and rounded to the model dtype when a model is
created, as the reference stores them in its `real` type.
"""
from __future__ import annotations

import numpy as np

from . import _abi


class Layer:
    kind: int = -1
    label: str = ""
    save = False   # Save_State
    binop = False  # Binop_*

    def __init__(self, num_inputs: int, num_outputs: int | None = None):
        self.num_inputs = int(num_inputs)
        self.num_outputs = int(num_inputs if num_outputs is None else num_outputs)
        self.save_index = -1
        self.aux = 0
        self.flags = 0
        self.scalar = [0.0, 0.0, 0.0]

    def parameters(self) -> np.ndarray:
        """All parameters in the reference's flattened order (float64)."""
        return np.zeros(0, dtype=np.float64)

    def set_parameters(self, flat: np.ndarray) -> None:
        pass

    @property
    def trainable(self) -> bool:
        return bool(self.flags & _abi.FLAG_TRAINABLE)

    def get_num_inputs(self) -> int:
        return self.num_inputs

    def get_num_outputs(self) -> int:
        return self.num_outputs

    def get_num_trainable_parameters(self) -> int:
        return int(self.parameters().size) if self.trainable else 0

    def get_label(self) -> str:
        return self.label


def _as2d(w) -> np.ndarray:
    a = np.array(w, dtype=np.float64, copy=True)
    if a.ndim != 2:
        raise ValueError("weights must be two-dimensional")
    return a


def _as1d(w) -> np.ndarray:
    return np.array(w, dtype=np.float64, copy=True).reshape(-1)


class Matvec(Layer):
    """Dense layer, weights W[num_inputs, num_outputs] (src/layers/ponni_Matvec.h)."""
    kind, label = _abi.MATVEC, "Matvec"

    def __init__(self, weights, trainable: bool = True):
        w = _as2d(weights)
        super().__init__(w.shape[0], w.shape[1])
        self.weights = w
        self.flags = _abi.FLAG_TRAINABLE if trainable else 0

    def parameters(self):
        return self.weights.reshape(-1)

    def set_parameters(self, flat):
        self.weights = np.asarray(flat, dtype=np.float64).reshape(self.weights.shape).copy()


class Bias(Layer):
    """Per-feature bias b[n] (src/layers/ponni_Bias.h)."""
    kind, label = _abi.BIAS, "Bias"

    def __init__(self, weights, trainable: bool = True):
        b = _as1d(weights)
        super().__init__(b.size)
        self.weights = b
        self.flags = _abi.FLAG_TRAINABLE if trainable else 0

    def parameters(self):
        return self.weights

    def set_parameters(self, flat):
        self.weights = np.asarray(flat, dtype=np.float64).reshape(-1).copy()


class Relu(Layer):
    kind, label = _abi.RELU, "ReLU"


ReLU = Relu


class LeakyRelu(Layer):
    kind, label = _abi.LEAKY_RELU, "LeakyReLU"

    def __init__(self, num_inputs: int, negative_slope: float = 0.01):
        super().__init__(num_inputs)
        self.scalar[0] = float(negative_slope)


LeakyReLU = LeakyRelu


class Elu(Layer):
    kind, label = _abi.ELU, "ELU"

    def __init__(self, num_inputs: int, alpha: float = 1.0):
        super().__init__(num_inputs)
        self.scalar[0] = float(alpha)


ELU = Elu


class Selu(Layer):
    kind, label = _abi.SELU, "SELU"


SELU = Selu


class Gelu(Layer):
    kind, label = _abi.GELU, "GELU"

    def __init__(self, num_inputs: int, approximate: bool = False):
        super().__init__(num_inputs)
        if approximate:
            self.flags |= _abi.FLAG_APPROXIMATE


GELU = Gelu


class Silu(Layer):
    kind, label = _abi.SILU, "SiLU"


SiLU = Silu


class Sigmoid(Layer):
    kind, label = _abi.SIGMOID, "Sigmoid"


class Tanh(Layer):
    kind, label = _abi.TANH, "Tanh"


class Softplus(Layer):
    kind, label = _abi.SOFTPLUS, "Softplus"

    def __init__(self, num_inputs: int, beta: float = 1.0):
        super().__init__(num_inputs)
        self.scalar[0] = float(beta)


class HardSigmoid(Layer):
    kind, label = _abi.HARD_SIGMOID, "HardSigmoid"

    def __init__(self, num_inputs: int, alpha: float = 0.2, beta: float = 0.5):
        super().__init__(num_inputs)
        self.scalar[0] = float(alpha)
        self.scalar[1] = float(beta)


class HardSwish(Layer):
    kind, label = _abi.HARD_SWISH, "HardSwish"


class Mish(Layer):
    kind, label = _abi.MISH, "Mish"


class LayerNorm(Layer):
    """LayerNorm(num_inputs | gamma, beta, epsilon=1e-5, trainable) (src/layers/ponni_LayerNorm.h)."""
    kind, label = _abi.LAYER_NORM, "LayerNorm"

    def __init__(self, num_inputs_or_gamma, beta=None, epsilon: float = 1e-5, trainable: bool = True):
        if beta is None and np.ndim(num_inputs_or_gamma) == 0:
            n = int(num_inputs_or_gamma)
            gamma, beta = np.ones(n), np.zeros(n)
        else:
            gamma, beta = _as1d(num_inputs_or_gamma), _as1d(beta)
            if gamma.size != beta.size:
                raise ValueError("ERROR: LayerNorm gamma and beta size mismatch")
        super().__init__(gamma.size)
        self.gamma, self.beta = np.asarray(gamma, np.float64), np.asarray(beta, np.float64)
        self.scalar[0] = float(epsilon)
        self.flags = _abi.FLAG_TRAINABLE if trainable else 0

    def parameters(self):
        return np.concatenate([self.gamma, self.beta])

    def set_parameters(self, flat):
        n = self.gamma.size
        flat = np.asarray(flat, dtype=np.float64).reshape(-1)
        self.gamma, self.beta = flat[:n].copy(), flat[n:2 * n].copy()


class MinMaxNorm(Layer):
    kind, label = _abi.MIN_MAX_NORM, "MinMaxNorm"

    def __init__(self, num_inputs: int, out_min: float = 0.0, out_max: float = 1.0, epsilon: float = 1e-12):
        super().__init__(num_inputs)
        self.scalar = [float(out_min), float(out_max), float(epsilon)]


class Softmax(Layer):
    kind, label = _abi.SOFTMAX, "Softmax"


class LogSoftmax(Layer):
    kind, label = _abi.LOG_SOFTMAX, "LogSoftmax"


class Save_State(Layer):
    """Save_State<ISAVE>(n): identity that stores the state in slot ISAVE."""
    kind, label, save = _abi.SAVE_STATE, "Save_State", True

    def __init__(self, num_inputs: int, index: int = 0):
        super().__init__(num_inputs)
        self.save_index = int(index)


class Binop_Add(Layer):
    kind, label, binop = _abi.BINOP_ADD, "Binop_Add", True

    def __init__(self, num_inputs: int, index: int = 0):
        super().__init__(num_inputs)
        self.save_index = int(index)


class Binop_Concatenate(Layer):
    kind, label, binop = _abi.BINOP_CONCATENATE, "Binop_Concatenate", True

    def __init__(self, num_inputs: int, num_outputs: int, after: bool = True, index: int = 0):
        super().__init__(num_inputs, num_outputs)
        self.save_index = int(index)
        if after:
            self.flags |= _abi.FLAG_AFTER


class Binop_Projection_Add(Layer):
    """out = in + bias + W^T saved; W[num_saved, num_inputs] (src/layers/ponni_Binop_Projection_Add.h)."""
    kind, label, binop = _abi.BINOP_PROJECTION_ADD, "Binop_Projection_Add", True

    def __init__(self, weights, bias, trainable: bool = True, index: int = 0):
        w, b = _as2d(weights), _as1d(bias)
        if w.shape[1] != b.size:
            raise ValueError("ERROR: Binop_Projection_Add incompatible weights/bias shapes")
        super().__init__(w.shape[1])
        self.weights, self.bias = w, b
        self.aux = w.shape[0]
        self.save_index = int(index)
        self.flags = _abi.FLAG_TRAINABLE if trainable else 0

    def parameters(self):
        return np.concatenate([self.weights.reshape(-1), self.bias])

    def set_parameters(self, flat):
        flat = np.asarray(flat, dtype=np.float64).reshape(-1)
        nw = self.weights.size
        self.weights = flat[:nw].reshape(self.weights.shape).copy()
        self.bias = flat[nw:nw + self.bias.size].copy()
