"""A CPU stand-in for the part of ``mlx.core`` that the reference package uses.

Test infrastructure only.  The reference (mace-mlx) is written against MLX,
which is not installed in this image.  This module re-implements the subset of
the MLX array API that ``mace_mlx`` calls on its CPU path (about 45 functions
plus the array methods and operators) on top of torch CPU tensors, so that the
UNMODIFIED reference package can be imported and executed here to produce
golden energies, forces and stresses.  Nothing in the product imports it.

Precision: the environment variable ``REFSHIM_FLOAT`` selects the storage of
MLX's ``float32`` dtype: ``float64`` (default) runs the reference's arithmetic
in double precision -- every ``mx.float32`` array, cast and constant is held as
a torch float64 tensor -- which gives the reference's algorithm without fp32
rounding noise; ``float32`` runs it in single precision like MLX itself.

Semantics follow the MLX documentation:
* ``array`` wraps one torch tensor; operators broadcast like numpy; indexing
  accepts ints, slices, None, Ellipsis and integer/boolean arrays;
* ``x.at[idx].add(v)`` is an out-of-place scatter-add that accumulates
  repeated indices (``torch.index_put(..., accumulate=True)``);
* ``value_and_grad(f, argnums)`` differentiates the first output of ``f``
  (the rest rides along as auxiliary data) with torch autograd;
* ``compile`` is the identity, ``eval`` a no-op (torch is eager);
* the device is always the CPU, so the reference's Metal kernels
  (``mx.fast.metal_kernel``) are never launched: it checks the default device
  before taking those paths.
"""

from __future__ import annotations

import os
import types

import numpy as np
import torch

_FLOAT_MODE = os.environ.get("REFSHIM_FLOAT", "float64")
if _FLOAT_MODE not in ("float64", "float32"):
    raise ValueError(f"REFSHIM_FLOAT must be float64 or float32, not {_FLOAT_MODE!r}")
_F = torch.float64 if _FLOAT_MODE == "float64" else torch.float32
torch.set_default_dtype(_F)


# --------------------------------------------------------------------------
# dtypes
# --------------------------------------------------------------------------
class Dtype:
    def __init__(self, name: str, torch_dtype: torch.dtype, category: str):
        self.name = name
        self.torch = torch_dtype
        self.category = category
        self.size = torch.empty((), dtype=torch_dtype).element_size()

    def __repr__(self):
        return f"mlx.core.{self.name}"


class _Category:
    def __init__(self, name):
        self.name = name

    def __repr__(self):
        return f"mlx.core.{self.name}"


floating = _Category("floating")
integer = _Category("integer")
signedinteger = _Category("signedinteger")
number = _Category("number")
generic = _Category("generic")

float32 = Dtype("float32", _F, "floating")
float64 = Dtype("float64", torch.float64, "floating")
float16 = Dtype("float16", torch.float16, "floating")
bfloat16 = Dtype("bfloat16", torch.bfloat16, "floating")
int8 = Dtype("int8", torch.int8, "integer")
int16 = Dtype("int16", torch.int16, "integer")
int32 = Dtype("int32", torch.int32, "integer")
int64 = Dtype("int64", torch.int64, "integer")
uint8 = Dtype("uint8", torch.uint8, "integer")
uint32 = Dtype("uint32", torch.int64, "integer")
bool_ = Dtype("bool", torch.bool, "bool")

_FROM_TORCH = {
    _F: float32,
    torch.float16: float16,
    torch.bfloat16: bfloat16,
    torch.int8: int8,
    torch.int16: int16,
    torch.int32: int32,
    torch.int64: int64,
    torch.uint8: uint8,
    torch.bool: bool_,
}
if _F is not torch.float64:
    _FROM_TORCH[torch.float64] = float64


def issubdtype(a, b) -> bool:
    if isinstance(a, Dtype) and isinstance(b, _Category):
        if b is floating:
            return a.category == "floating"
        if b in (integer, signedinteger):
            return a.category == "integer"
        return b in (number, generic)
    return a is b


def _torch_dtype(d):
    if d is None:
        return None
    if isinstance(d, Dtype):
        return d.torch
    raise TypeError(f"not an mlx dtype: {d!r}")


# --------------------------------------------------------------------------
# conversion helpers
# --------------------------------------------------------------------------
def _contig(a: np.ndarray) -> np.ndarray:
    # a C-ordered copy that keeps 0-d arrays 0-d (np.ascontiguousarray makes them 1-d)
    return a if a.flags.c_contiguous else a.copy(order="C")


def _np_to_torch(a: np.ndarray) -> torch.Tensor:
    if a.dtype.kind == "f":
        return torch.from_numpy(_contig(a)).to(_F)
    if a.dtype.kind == "b":
        return torch.from_numpy(_contig(a))
    if a.dtype.kind in "iu":
        if a.dtype == np.uint32 or a.dtype == np.uint64:
            a = a.astype(np.int64)
        return torch.from_numpy(_contig(a))
    raise TypeError(f"unsupported numpy dtype {a.dtype}")


def _to_tensor(x) -> torch.Tensor:
    """Anything array-like -> torch tensor with MLX's default dtypes."""
    if isinstance(x, array):
        return x._t
    if isinstance(x, torch.Tensor):
        return x
    if isinstance(x, np.ndarray):
        return _np_to_torch(x)
    if isinstance(x, (bool, np.bool_)):
        return torch.tensor(bool(x))
    if isinstance(x, (int, np.integer)):
        return torch.tensor(int(x), dtype=torch.int32)
    if isinstance(x, (float, np.floating)):
        return torch.tensor(float(x), dtype=_F)
    if isinstance(x, (list, tuple)):
        if len(x) and any(isinstance(v, array) for v in x):
            return torch.stack([_to_tensor(v) for v in x])
        a = np.asarray(x)
        if a.dtype.kind == "i":
            a = a.astype(np.int32)
        return _np_to_torch(a)
    raise TypeError(f"cannot convert {type(x)} to an mlx array")


def _operand(x):
    """Operand of a binary op: arrays unwrap, Python scalars stay weak scalars."""
    if isinstance(x, array):
        return x._t
    if isinstance(x, (bool, int, float)):
        return x
    if isinstance(x, np.floating):
        return float(x)
    if isinstance(x, np.integer):
        return int(x)
    return _to_tensor(x)


def _index(idx):
    if isinstance(idx, tuple):
        return tuple(_index(i) for i in idx)
    if isinstance(idx, array):
        t = idx._t
        return t if t.dtype == torch.bool else t.long()
    if isinstance(idx, np.ndarray):
        t = torch.from_numpy(np.ascontiguousarray(idx))
        return t if t.dtype == torch.bool else t.long()
    if isinstance(idx, list):
        return torch.tensor(idx, dtype=torch.long)
    return idx


def _is_advanced(idx) -> bool:
    items = idx if isinstance(idx, tuple) else (idx,)
    return any(isinstance(i, torch.Tensor) for i in items)


# --------------------------------------------------------------------------
# the array type
# --------------------------------------------------------------------------
class _AtOp:
    def __init__(self, arr: "array", idx):
        self._arr = arr
        self._idx = idx

    def _apply(self, v, op):
        t = self._arr._t
        idx = _index(self._idx)
        val = _operand(v)
        if not isinstance(val, torch.Tensor):
            val = torch.tensor(val, dtype=t.dtype)
        val = val.to(t.dtype)
        if op == "add" and _is_advanced(idx):
            idx_t = idx if isinstance(idx, tuple) else (idx,)
            target_shape = t[idx_t].shape
            return array(torch.index_put(t, idx_t, val.expand(target_shape), accumulate=True))
        out = t.clone()
        cur = out[idx]
        if op == "add":
            out[idx] = cur + val
        elif op == "subtract":
            out[idx] = cur - val
        elif op == "multiply":
            out[idx] = cur * val
        else:
            raise NotImplementedError(op)
        return array(out)

    def add(self, v):
        return self._apply(v, "add")

    def subtract(self, v):
        return self._apply(v, "subtract")

    def multiply(self, v):
        return self._apply(v, "multiply")


class _At:
    def __init__(self, arr):
        self._arr = arr

    def __getitem__(self, idx):
        return _AtOp(self._arr, idx)


class array:
    """MLX-style array over a torch tensor (see the module docstring)."""

    __slots__ = ("_t",)

    def __init__(self, val=None, dtype: Dtype | None = None):
        t = _to_tensor(val)
        if dtype is not None:
            t = t.to(_torch_dtype(dtype))
        self._t = t

    # --- metadata ---------------------------------------------------------
    @property
    def shape(self):
        return tuple(self._t.shape)

    @property
    def ndim(self):
        return self._t.dim()

    @property
    def size(self):
        return self._t.numel()

    @property
    def dtype(self):
        return _FROM_TORCH.get(self._t.dtype, float64)

    @property
    def itemsize(self):
        return self._t.element_size()

    @property
    def nbytes(self):
        return self._t.numel() * self._t.element_size()

    @property
    def at(self):
        return _At(self)

    @property
    def T(self):
        return array(self._t.permute(*reversed(range(self._t.dim()))))

    def __len__(self):
        return self._t.shape[0]

    def __iter__(self):
        for i in range(self._t.shape[0]):
            yield array(self._t[i])

    def __repr__(self):
        return f"array({self._t.detach().numpy()!r}, dtype={self.dtype.name})"

    def __array__(self, dtype=None, copy=None):
        a = self._t.detach().cpu().numpy()
        return a.astype(dtype) if dtype is not None else a

    def __bool__(self):
        return bool(self._t)

    def __float__(self):
        return float(self._t)

    def __int__(self):
        return int(self._t)

    def __hash__(self):
        return id(self)

    # --- conversions ------------------------------------------------------
    def item(self):
        return self._t.item()

    def tolist(self):
        return self._t.tolist()

    def astype(self, dtype, stream=None):
        return array(self._t.to(_torch_dtype(dtype)))

    # --- shape ops --------------------------------------------------------
    def reshape(self, *shape, stream=None):
        if len(shape) == 1 and isinstance(shape[0], (tuple, list)):
            shape = tuple(shape[0])
        return array(self._t.reshape(shape))

    def squeeze(self, axis=None):
        if axis is None:
            return array(self._t.squeeze())
        axes = axis if isinstance(axis, (tuple, list)) else (axis,)
        t = self._t
        for a in sorted((a % t.dim() for a in axes), reverse=True):
            if t.shape[a] != 1:
                raise ValueError("cannot squeeze an axis of size != 1")
            t = t.squeeze(a)
        return array(t)

    def transpose(self, *axes):
        if len(axes) == 1 and isinstance(axes[0], (tuple, list)):
            axes = tuple(axes[0])
        if not axes:
            axes = tuple(reversed(range(self._t.dim())))
        return array(self._t.permute(*axes))

    def swapaxes(self, a, b):
        return array(self._t.transpose(a, b))

    def flatten(self, start_axis=0, end_axis=-1):
        return array(self._t.flatten(start_axis, end_axis))

    # --- reductions -------------------------------------------------------
    def _reduce(self, fn, axis, keepdims):
        if axis is None:
            r = fn(self._t)
            return array(r.reshape([1] * self._t.dim()) if keepdims else r)
        return array(fn(self._t, dim=axis, keepdim=keepdims))

    def sum(self, axis=None, keepdims=False, stream=None):
        return self._reduce(torch.sum, axis, keepdims)

    def mean(self, axis=None, keepdims=False, stream=None):
        return self._reduce(torch.mean, axis, keepdims)

    def max(self, axis=None, keepdims=False, stream=None):
        return self._reduce(torch.amax, axis, keepdims)

    def min(self, axis=None, keepdims=False, stream=None):
        return self._reduce(torch.amin, axis, keepdims)

    def abs(self):
        return array(self._t.abs())

    def square(self):
        return array(self._t * self._t)

    def sqrt(self):
        return array(self._t.sqrt())

    def exp(self):
        return array(self._t.exp())

    # --- indexing ---------------------------------------------------------
    def __getitem__(self, idx):
        return array(self._t[_index(idx)])

    def __setitem__(self, idx, val):
        raise TypeError("mlx arrays are immutable; use x.at[idx]")

    # --- operators --------------------------------------------------------
    def __add__(self, o):
        return array(self._t + _operand(o))

    def __radd__(self, o):
        return array(_operand(o) + self._t)

    def __sub__(self, o):
        return array(self._t - _operand(o))

    def __rsub__(self, o):
        return array(_operand(o) - self._t)

    def __mul__(self, o):
        return array(self._t * _operand(o))

    def __rmul__(self, o):
        return array(_operand(o) * self._t)

    def __truediv__(self, o):
        return array(torch.true_divide(self._t, _operand(o)))

    def __rtruediv__(self, o):
        o = _operand(o)
        if not isinstance(o, torch.Tensor):
            o = torch.tensor(o, dtype=self._t.dtype if self._t.is_floating_point() else _F)
        return array(torch.true_divide(o, self._t))

    def __floordiv__(self, o):
        return array(torch.floor_divide(self._t, _operand(o)))

    def __mod__(self, o):
        return array(torch.remainder(self._t, _operand(o)))

    def __pow__(self, o):
        return array(torch.pow(self._t, _operand(o)))

    def __rpow__(self, o):
        return array(torch.pow(_operand(o), self._t))

    def __matmul__(self, o):
        return array(self._t @ _operand(o))

    def __rmatmul__(self, o):
        return array(_operand(o) @ self._t)

    def __neg__(self):
        return array(-self._t)

    def __abs__(self):
        return array(self._t.abs())

    def __lt__(self, o):
        return array(self._t < _operand(o))

    def __le__(self, o):
        return array(self._t <= _operand(o))

    def __gt__(self, o):
        return array(self._t > _operand(o))

    def __ge__(self, o):
        return array(self._t >= _operand(o))

    def __eq__(self, o):
        return array(self._t == _operand(o))

    def __ne__(self, o):
        return array(self._t != _operand(o))

    def __and__(self, o):
        return array(self._t & _operand(o))

    def __or__(self, o):
        return array(self._t | _operand(o))

    def __invert__(self):
        return array(~self._t)


# --------------------------------------------------------------------------
# free functions
# --------------------------------------------------------------------------
def _t(x):
    return x._t if isinstance(x, array) else _to_tensor(x)


def _shape(shape):
    return (shape,) if isinstance(shape, int) else tuple(shape)


def zeros(shape, dtype=float32, stream=None):
    return array(torch.zeros(_shape(shape), dtype=_torch_dtype(dtype)))


def ones(shape, dtype=float32, stream=None):
    return array(torch.ones(_shape(shape), dtype=_torch_dtype(dtype)))


def full(shape, vals, dtype=None, stream=None):
    v = _t(vals)
    if dtype is not None:
        v = v.to(_torch_dtype(dtype))
    return array(torch.broadcast_to(v, _shape(shape)).clone())


def zeros_like(a, stream=None):
    return array(torch.zeros_like(_t(a)))


def ones_like(a, stream=None):
    return array(torch.ones_like(_t(a)))


def arange(*args, dtype=None, stream=None):
    t = torch.arange(*args)
    if dtype is not None:
        t = t.to(_torch_dtype(dtype))
    elif not t.is_floating_point():
        t = t.to(torch.int32)
    return array(t)


def linspace(start, stop, num=50, dtype=float32, stream=None):
    return array(torch.linspace(float(start), float(stop), int(num), dtype=_torch_dtype(dtype)))


def eye(n, m=None, k=0, dtype=float32, stream=None):
    return array(torch.eye(n, m if m is not None else n, dtype=_torch_dtype(dtype)))


def einsum(subscripts, *operands, stream=None):
    return array(torch.einsum(subscripts, *[_t(o) for o in operands]))


def concatenate(arrays, axis=0, stream=None):
    return array(torch.cat([_t(a) for a in arrays], dim=axis))


def stack(arrays, axis=0, stream=None):
    return array(torch.stack([_t(a) for a in arrays], dim=axis))


def take(a, indices, axis=None, stream=None):
    a = _t(a)
    idx = _t(indices).long()
    if axis is None:
        return array(a.reshape(-1)[idx])
    axis = axis % a.dim()
    flat = torch.index_select(a, axis, idx.reshape(-1))
    return array(flat.reshape(a.shape[:axis] + idx.shape + a.shape[axis + 1:]))


def take_along_axis(a, indices, axis=None, stream=None):
    return array(torch.take_along_dim(_t(a), _t(indices).long(), dim=axis))


def where(cond, x, y, stream=None):
    c = _t(cond).bool()
    xo, yo = _operand(x), _operand(y)
    if not isinstance(xo, torch.Tensor) and not isinstance(yo, torch.Tensor):
        xo = torch.tensor(xo, dtype=_F)
    return array(torch.where(c, xo, yo))


def _reduce_fn(fn, a, axis, keepdims):
    t = _t(a)
    if axis is None:
        r = fn(t)
        return array(r.reshape([1] * t.dim()) if keepdims else r)
    return array(fn(t, dim=axis, keepdim=keepdims))


def sum(a, axis=None, keepdims=False, stream=None):  # noqa: A001 - MLX name
    return _reduce_fn(torch.sum, a, axis, keepdims)


def mean(a, axis=None, keepdims=False, stream=None):
    return _reduce_fn(torch.mean, a, axis, keepdims)


def max(a, axis=None, keepdims=False, stream=None):  # noqa: A001
    return _reduce_fn(torch.amax, a, axis, keepdims)


def min(a, axis=None, keepdims=False, stream=None):  # noqa: A001
    return _reduce_fn(torch.amin, a, axis, keepdims)


def argmax(a, axis=None, keepdims=False, stream=None):
    t = _t(a)
    if axis is None:
        return array(torch.argmax(t).to(torch.int64))
    return array(torch.argmax(t, dim=axis, keepdim=keepdims).to(torch.int64))


def _unary(fn):
    def f(a, stream=None):
        return array(fn(_t(a)))
    return f


sqrt = _unary(torch.sqrt)
rsqrt = _unary(torch.rsqrt)
exp = _unary(torch.exp)
log = _unary(torch.log)
tanh = _unary(torch.tanh)
sin = _unary(torch.sin)
cos = _unary(torch.cos)
sigmoid = _unary(torch.sigmoid)
abs = _unary(torch.abs)  # noqa: A001
square = _unary(torch.square)
negative = _unary(torch.neg)
erf = _unary(torch.erf)


def _binary_tensors(a, b):
    ao, bo = _operand(a), _operand(b)
    if not isinstance(ao, torch.Tensor):
        ao = torch.tensor(ao, dtype=bo.dtype if isinstance(bo, torch.Tensor) else _F)
    if not isinstance(bo, torch.Tensor):
        bo = torch.tensor(bo, dtype=ao.dtype)
    return ao, bo


def maximum(a, b, stream=None):
    return array(torch.maximum(*_binary_tensors(a, b)))


def minimum(a, b, stream=None):
    return array(torch.minimum(*_binary_tensors(a, b)))


def power(a, b, stream=None):
    return array(torch.pow(_operand(a), _operand(b)))


def matmul(a, b, stream=None):
    return array(_t(a) @ _t(b))


def broadcast_to(a, shape, stream=None):
    return array(torch.broadcast_to(_t(a), tuple(shape)))


def moveaxis(a, source, destination, stream=None):
    return array(torch.movedim(_t(a), source, destination))


def swapaxes(a, a1, a2, stream=None):
    return array(_t(a).transpose(a1, a2))


def transpose(a, axes=None, stream=None):
    t = _t(a)
    if axes is None:
        axes = tuple(reversed(range(t.dim())))
    return array(t.permute(*axes))


def reshape(a, shape, stream=None):
    return array(_t(a).reshape(tuple(shape)))


def expand_dims(a, axis, stream=None):
    t = _t(a)
    axes = axis if isinstance(axis, (tuple, list)) else (axis,)
    nd = t.dim() + len(axes)
    for ax in sorted(x % nd for x in axes):
        t = t.unsqueeze(ax)
    return array(t)


def squeeze(a, axis=None, stream=None):
    return array(_t(a)).squeeze(axis)


def atleast_1d(a, stream=None):
    return array(torch.atleast_1d(_t(a)))


def atleast_2d(a, stream=None):
    return array(torch.atleast_2d(_t(a)))


def atleast_3d(a, stream=None):
    return array(torch.atleast_3d(_t(a)))


def outer(a, b, stream=None):
    return array(torch.outer(_t(a), _t(b)))


def split(a, indices_or_sections, axis=0, stream=None):
    t = _t(a)
    if isinstance(indices_or_sections, int):
        parts = torch.tensor_split(t, indices_or_sections, dim=axis)
    else:
        parts = torch.tensor_split(t, list(indices_or_sections), dim=axis)
    return [array(p) for p in parts]


def stop_gradient(a, stream=None):
    return array(_t(a).detach())


def eval(*args):  # noqa: A001 - MLX name
    return None


def async_eval(*args):
    return None


def compile(fun, inputs=None, outputs=None, shapeless=False):  # noqa: A001
    return fun


def _tree_map(fn, tree):
    if isinstance(tree, array):
        return fn(tree)
    if isinstance(tree, (list, tuple)):
        return type(tree)(_tree_map(fn, v) for v in tree)
    if isinstance(tree, dict):
        return {k: _tree_map(fn, v) for k, v in tree.items()}
    return tree


def value_and_grad(fun, argnums=0, argnames=()):
    """``(value, grads)`` of ``fun``; the gradient is of its first output."""

    def wrapped(*args, **kwargs):
        nums = (argnums,) if isinstance(argnums, int) else tuple(argnums)
        args = list(args)
        leaves = []
        for i in nums:
            leaf = _t(args[i]).detach().clone().requires_grad_(True)
            args[i] = array(leaf)
            leaves.append(leaf)
        with torch.enable_grad():
            out = fun(*args, **kwargs)
            loss = out[0] if isinstance(out, (tuple, list)) else out
            grads = torch.autograd.grad(_t(loss), leaves, allow_unused=True)
        grads = [array(g.detach() if g is not None else torch.zeros_like(leaf)) for g, leaf in zip(grads, leaves)]
        out = _tree_map(lambda a: array(a._t.detach()), out)
        return out, (grads[0] if isinstance(argnums, int) else tuple(grads))

    return wrapped


def grad(fun, argnums=0, argnames=()):
    vg = value_and_grad(fun, argnums, argnames)

    def wrapped(*args, **kwargs):
        return vg(*args, **kwargs)[1]

    return wrapped


class custom_function:  # noqa: N801 - MLX name
    """Decorator stand-in: the forward runs as written (torch autograd gives the
    VJP); ``.vjp`` / ``.jvp`` / ``.vmap`` registrations are accepted and unused.
    The reference only defines custom functions around its Metal kernels, which
    never run on the CPU device."""

    def __init__(self, fun):
        self._fun = fun

    def __call__(self, *args, **kwargs):
        return self._fun(*args, **kwargs)

    def vjp(self, f):
        return f

    def jvp(self, f):
        return f

    def vmap(self, f):
        return f


# --------------------------------------------------------------------------
# devices, random, IO, fast
# --------------------------------------------------------------------------
class DeviceType:
    cpu = "cpu"
    gpu = "gpu"


class Device:
    def __init__(self, type_):
        self.type = type_

    def __eq__(self, other):
        return isinstance(other, Device) and other.type == self.type

    def __hash__(self):
        return hash(self.type)

    def __repr__(self):
        return f"Device({self.type}, 0)"


cpu = Device(DeviceType.cpu)
gpu = Device(DeviceType.gpu)


def default_device():
    return cpu


def set_default_device(device):
    """The stand-in only has a CPU; selecting the GPU is accepted and ignored."""
    return None


class _Random:
    def __init__(self):
        self._gen = torch.Generator().manual_seed(0)

    def seed(self, s):
        self._gen.manual_seed(int(s))

    def normal(self, shape=(), dtype=float32, loc=0.0, scale=1.0, key=None, stream=None):
        return array(torch.randn(_shape(shape), generator=self._gen, dtype=_torch_dtype(dtype)) * scale + loc)

    def uniform(self, low=0.0, high=1.0, shape=(), dtype=float32, key=None, stream=None):
        u = torch.rand(_shape(shape), generator=self._gen, dtype=_torch_dtype(dtype))
        return array(u * (float(high) - float(low)) + float(low))


random = _Random()


def load(path, format=None, return_metadata=False):  # noqa: A002
    with np.load(path) as z:
        return {k: array(z[k]) for k in z.files}


def savez(path, *args, **kwargs):
    np.savez(path, *[np.asarray(a) for a in args], **{k: np.asarray(v) for k, v in kwargs.items()})


def _metal_kernel(*args, **kwargs):
    def _never(*a, **k):
        raise RuntimeError("Metal kernels do not run on the CPU stand-in of mlx")
    return _never


fast = types.SimpleNamespace(metal_kernel=_metal_kernel)
metal = types.SimpleNamespace(is_available=lambda: False)
