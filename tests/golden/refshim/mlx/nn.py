"""CPU stand-in for the part of ``mlx.nn`` that the reference package uses.

Test infrastructure only (see ``mlx/core.py``).  ``Module`` follows MLX's
documented container semantics: a module is a ``dict`` whose array, list,
dict and sub-module attributes are stored as items; ``parameters()`` returns
the nested items whose keys do not start with ``_`` (non-array members of
lists and dicts flatten to nothing); ``load_weights`` takes flat
``"a.b.0.c"`` keys, checks them against the parameters (strict) and updates
the tree.  ``Linear`` computes ``x @ W.T + b`` with ``W`` of shape
(out, in); ``LayerNorm`` normalises the last axis with eps 1e-5.
"""

from __future__ import annotations

import math

import torch

from . import core as mx
from .utils import tree_flatten, tree_unflatten


class Module(dict):
    def __init__(self):
        super().__init__()
        object.__setattr__(self, "_training", True)

    # attribute <-> item mapping --------------------------------------------
    def __setattr__(self, key, val):
        if isinstance(val, (mx.array, dict, list, tuple)):
            if key in self.__dict__:
                object.__delattr__(self, key)
            self[key] = val
        else:
            if key in self:
                del self[key]
            object.__setattr__(self, key, val)

    def __getattr__(self, key):
        if key in self:
            return self[key]
        raise AttributeError(f"{type(self).__name__!r} object has no attribute {key!r}")

    def __delattr__(self, key):
        if key in self:
            del self[key]
        else:
            object.__delattr__(self, key)

    def __hash__(self):
        return id(self)

    def __eq__(self, other):
        return self is other

    @property
    def training(self):
        return self._training

    def train(self, mode: bool = True):
        for _, m in self.named_modules():
            object.__setattr__(m, "_training", mode)
        return self

    def eval(self):  # noqa: A003 - MLX name
        return self.train(False)

    # trees -------------------------------------------------------------------
    @staticmethod
    def _valid(key, value):
        # MLX's valid_parameter_filter: arrays, dicts and lists under public keys
        return isinstance(value, (dict, list, mx.array)) and not str(key).startswith("_")

    def _filter(self, value):
        if isinstance(value, mx.array):
            return value
        if isinstance(value, Module):
            return value.parameters()
        if isinstance(value, dict):
            return {k: (self._filter(v) if self._valid(k, v) else {}) for k, v in value.items()}
        if isinstance(value, list):
            return [(self._filter(v) if self._valid(i, v) else {}) for i, v in enumerate(value)]
        raise RuntimeError("unexpected leaf in the module tree")

    def parameters(self):
        return {k: self._filter(v) for k, v in self.items() if self._valid(k, v)}

    def trainable_parameters(self):
        return self.parameters()

    def children(self):
        out = {}
        for k, v in self.items():
            if isinstance(v, Module):
                out[k] = v
            elif isinstance(v, (list, tuple)) and any(isinstance(x, Module) for x in v):
                out[k] = [x for x in v if isinstance(x, Module)]
            elif isinstance(v, dict) and any(isinstance(x, Module) for x in v.values()):
                out[k] = {kk: x for kk, x in v.items() if isinstance(x, Module)}
        return out

    def named_modules(self):
        result = []

        def visit(prefix, m):
            result.append((prefix, m))
            for k, v in m.items():
                name = f"{prefix}.{k}" if prefix else k
                if isinstance(v, Module):
                    visit(name, v)
                elif isinstance(v, (list, tuple)):
                    for i, x in enumerate(v):
                        if isinstance(x, Module):
                            visit(f"{name}.{i}", x)
                elif isinstance(v, dict):
                    for kk, x in v.items():
                        if isinstance(x, Module):
                            visit(f"{name}.{kk}", x)

        visit("", self)
        return result[::-1]

    def modules(self):
        return [m for _, m in self.named_modules()]

    def leaf_modules(self):
        return {k: m for k, m in self.named_modules() if not m.children()}

    def update(self, parameters, strict: bool = True):
        def apply(dst, src):
            if isinstance(src, dict):
                for k, v in src.items():
                    if isinstance(v, mx.array):
                        dst[k] = v
                    else:
                        apply(dst[k], v)
            elif isinstance(src, list):
                for i, v in enumerate(src):
                    if isinstance(v, mx.array):
                        dst[i] = v
                    else:
                        apply(dst[i], v)
        apply(self, parameters)
        return self

    def load_weights(self, file_or_weights, strict: bool = True):
        if isinstance(file_or_weights, str):
            weights = list(mx.load(file_or_weights).items())
        else:
            weights = list(file_or_weights)
        if strict:
            new = dict(weights)
            curr = dict(tree_flatten(self.parameters()))
            extras = sorted(set(new) - set(curr))
            missing = sorted(set(curr) - set(new))
            if extras:
                raise ValueError(f"Received parameters not in model: {', '.join(extras)}.")
            if missing:
                raise ValueError(f"Missing parameters: {', '.join(missing)}.")
            for k, v in curr.items():
                if tuple(v.shape) != tuple(new[k].shape):
                    raise ValueError(f"Expected shape {v.shape} but received shape {new[k].shape} for parameter {k}")
        self.update(tree_unflatten(weights))
        return self

    def freeze(self, recurse=True, keys=None, strict=False):
        return self

    def unfreeze(self, recurse=True, keys=None, strict=False):
        return self

    def set_dtype(self, dtype, predicate=None):
        for _, m in self.named_modules():
            for k in list(m.keys()):
                v = m[k]
                if not k.startswith("_") and isinstance(v, mx.array) and mx.issubdtype(v.dtype, mx.floating):
                    m[k] = v.astype(dtype)


class Linear(Module):
    def __init__(self, input_dims: int, output_dims: int, bias: bool = True):
        super().__init__()
        scale = math.sqrt(1.0 / input_dims)
        self.weight = mx.random.uniform(-scale, scale, (output_dims, input_dims))
        if bias:
            self.bias = mx.random.uniform(-scale, scale, (output_dims,))

    def __call__(self, x):
        y = x @ self.weight.T
        if "bias" in self:
            y = y + self.bias
        return y


class Sequential(Module):
    def __init__(self, *modules):
        super().__init__()
        self.layers = list(modules)

    def __call__(self, x):
        for m in self.layers:
            x = m(x)
        return x


def silu(x):
    return x * mx.sigmoid(x)


def sigmoid(x):
    return mx.sigmoid(x)


class SiLU(Module):
    def __call__(self, x):
        return silu(x)


class LayerNorm(Module):
    def __init__(self, dims: int, eps: float = 1e-5, affine: bool = True, bias: bool = True):
        super().__init__()
        self.dims = dims
        self.eps = eps
        if affine:
            self.weight = mx.ones((dims,))
            if bias:
                self.bias = mx.zeros((dims,))

    def __call__(self, x):
        t = x._t
        mean = t.mean(dim=-1, keepdim=True)
        var = ((t - mean) ** 2).mean(dim=-1, keepdim=True)
        y = (t - mean) * torch.rsqrt(var + self.eps)
        if "weight" in self:
            y = y * self.weight._t
        if "bias" in self:
            y = y + self.bias._t
        return mx.array(y)
