"""A small NumPy-backed stand-in for ``mlx.core`` -- fixture generation only.

MLX is not installable here, so ``make_golden.py`` runs the reference's own
Python (codec, cache, attention dispatch, unpack, its test helpers) on top of
this module.  It implements only the array API those files use, with MLX's
numeric conventions made explicit:

* elementwise float ops are evaluated exactly (float64) and rounded once to
  the result dtype (fp16 / bf16 / fp32) -- IEEE correctly rounded results;
* Python scalars are weakly typed (they take the array's dtype);
* fp16 op bf16 promotes to fp32; int op float promotes to the float type;
* matmul accumulates wider than its inputs and rounds the result once;
* ``round`` is round-half-to-even; float->int casts truncate, and NaN casts
  to 0 (the ARM64 conversion result);
* ``softmax(precise=True)`` is evaluated in float64 and rounded once.

``fast.metal_kernel`` cannot run Metal.  It returns restatements of the two
reference kernels by name (the INT4 pack and the fused decode SDPA); they are
marked as restatements in the fixtures that use them.
"""

from __future__ import annotations

import math as _math
import numpy as _np


class Dtype:
    def __init__(self, name, np_storage, itemsize, kind):
        self.name = name
        self.np = _np.dtype(np_storage)
        self.size = itemsize
        self.kind = kind  # 'f', 'i', 'u', 'b'

    def __repr__(self):
        return f"mlx.core.{self.name}"

    def __eq__(self, other):
        return isinstance(other, Dtype) and other.name == self.name

    def __hash__(self):
        return hash(self.name)


float16 = Dtype("float16", _np.float16, 2, "f")
bfloat16 = Dtype("bfloat16", _np.float32, 2, "f")  # stored as float32, rounded to bf16
float32 = Dtype("float32", _np.float32, 4, "f")
float64 = Dtype("float64", _np.float64, 8, "f")
int8 = Dtype("int8", _np.int8, 1, "i")
int16 = Dtype("int16", _np.int16, 2, "i")
int32 = Dtype("int32", _np.int32, 4, "i")
int64 = Dtype("int64", _np.int64, 8, "i")
uint8 = Dtype("uint8", _np.uint8, 1, "u")
uint16 = Dtype("uint16", _np.uint16, 2, "u")
uint32 = Dtype("uint32", _np.uint32, 4, "u")
uint64 = Dtype("uint64", _np.uint64, 8, "u")
bool_ = Dtype("bool", _np.bool_, 1, "b")

_BY_NP = {
    _np.dtype(_np.float16): float16, _np.dtype(_np.float32): float32, _np.dtype(_np.float64): float32,
    _np.dtype(_np.int8): int8, _np.dtype(_np.int16): int16, _np.dtype(_np.int32): int32,
    _np.dtype(_np.int64): int64, _np.dtype(_np.uint8): uint8, _np.dtype(_np.uint16): uint16,
    _np.dtype(_np.uint32): uint32, _np.dtype(_np.uint64): uint64, _np.dtype(_np.bool_): bool_,
}


def _round_bf16(a64):
    a = _np.asarray(a64, dtype=_np.float64).astype(_np.float32)
    bits = a.view(_np.uint32).astype(_np.uint64)
    lsb = (bits >> _np.uint64(16)) & _np.uint64(1)
    r = ((bits + _np.uint64(0x7FFF) + lsb) & _np.uint64(0xFFFF0000)).astype(_np.uint32).view(_np.float32)
    return _np.where(_np.isnan(a), a, r)


NAN_CASTS = [0]


def _cast(values, dt: Dtype):
    """Convert a NumPy array to the storage of ``dt`` with MLX rounding."""
    v = _np.asarray(values)
    if dt.kind == "f":
        if dt == bfloat16:
            return _round_bf16(v).astype(_np.float32)
        return v.astype(_np.float64).astype(dt.np) if v.dtype.kind == "f" else v.astype(dt.np)
    if dt.kind == "b":
        return v.astype(_np.bool_)
    if v.dtype.kind == "f":
        nan = _np.isnan(v)
        if nan.any():
            NAN_CASTS[0] += int(nan.sum())
        v = _np.where(nan, 0.0, v)
        v = _np.trunc(v)
        if dt.kind == "u":
            return v.astype(_np.int64).astype(dt.np)
        return v.astype(_np.int64).astype(dt.np)
    return v.astype(dt.np)


def _promote(a: Dtype, b: Dtype) -> Dtype:
    if a == b:
        return a
    if a.kind == "b":
        return b
    if b.kind == "b":
        return a
    if a.kind == "f" and b.kind == "f":
        if {a.name, b.name} == {"float16", "bfloat16"}:
            return float32
        return a if a.size > b.size else b
    if a.kind == "f":
        return a
    if b.kind == "f":
        return b
    # integers
    if a.kind == b.kind:
        return a if a.size >= b.size else b
    s, u = (a, b) if a.kind == "i" else (b, a)
    if s.size > u.size:
        return s
    return {1: int16, 2: int32, 4: int64}.get(u.size, float32)


def _weak(scalar, other: Dtype) -> Dtype:
    if isinstance(scalar, bool):
        return other
    if isinstance(scalar, int):
        return other if other.kind != "b" else int32
    if isinstance(scalar, float):
        return other if other.kind == "f" else float32
    raise TypeError(type(scalar))


class array:
    def __init__(self, value, dtype: Dtype | None = None):
        if isinstance(value, array):
            self._a, self.dtype = value._a, value.dtype
            if dtype is not None and dtype != value.dtype:
                self._a, self.dtype = _cast(value._a, dtype), dtype
            return
        v = _np.asarray(value)
        if dtype is None:
            if v.dtype.kind == "f":
                dtype = float32
            elif v.dtype.kind == "b":
                dtype = bool_
            elif v.dtype == _np.int64 and not isinstance(value, _np.ndarray):
                dtype = int32
            else:
                dtype = _BY_NP[v.dtype]
        self.dtype = dtype
        self._a = _cast(v, dtype)

    # --- construction helpers -------------------------------------------------
    @classmethod
    def _wrap(cls, a, dtype):
        o = cls.__new__(cls)
        o._a = _cast(a, dtype)
        o.dtype = dtype
        return o

    # --- properties -----------------------------------------------------------
    @property
    def shape(self):
        return tuple(self._a.shape)

    @property
    def ndim(self):
        return self._a.ndim

    @property
    def size(self):
        return int(self._a.size)

    @property
    def nbytes(self):
        return int(self._a.size) * self.dtype.size

    @property
    def T(self):
        return array._wrap(self._a.T, self.dtype)

    def item(self):
        return self._a.item()

    def tolist(self):
        return self._a.tolist()

    def __array__(self, dtype=None, copy=None):
        return self._a if dtype is None else self._a.astype(dtype)

    def __len__(self):
        return self._a.shape[0]

    def __repr__(self):
        return f"array({self._a!r}, dtype={self.dtype.name})"

    # --- shape ops ------------------------------------------------------------
    def astype(self, dtype):
        return array._wrap(self._a, dtype)

    def reshape(self, *shape):
        if len(shape) == 1 and isinstance(shape[0], (tuple, list)):
            shape = tuple(shape[0])
        return array._wrap(self._a.reshape(shape), self.dtype)

    def squeeze(self, axis=None):
        return array._wrap(_np.squeeze(self._a, axis=axis), self.dtype)

    def transpose(self, *axes):
        if len(axes) == 1 and isinstance(axes[0], (tuple, list)):
            axes = tuple(axes[0])
        return array._wrap(_np.transpose(self._a, axes or None), self.dtype)

    def __getitem__(self, idx):
        if isinstance(idx, array):
            idx = idx._a
        elif isinstance(idx, tuple):
            idx = tuple(i._a if isinstance(i, array) else i for i in idx)
        return array._wrap(self._a[idx], self.dtype)

    # --- reductions -----------------------------------------------------------
    def max(self, axis=None, keepdims=False):
        return array._wrap(self._a.max(axis=axis, keepdims=keepdims), self.dtype)

    def min(self, axis=None, keepdims=False):
        return array._wrap(self._a.min(axis=axis, keepdims=keepdims), self.dtype)

    def sum(self, axis=None, keepdims=False):
        return sum(self, axis=axis, keepdims=keepdims)

    # --- arithmetic -------------------------------------------------------------
    def _bin(self, other, fn, reverse=False, kind="arith"):
        if isinstance(other, array):
            odt, ov = other.dtype, other._a
        else:
            odt, ov = _weak(other, self.dtype), _np.asarray(other)
            ov = _cast(ov, odt) if not isinstance(other, bool) else ov
        rdt = _promote(self.dtype, odt)
        a, b = (ov, self._a) if reverse else (self._a, ov)
        if kind == "cmp":
            if rdt.kind == "f":
                return array._wrap(fn(a.astype(_np.float64), b.astype(_np.float64)), bool_)
            return array._wrap(fn(a.astype(rdt.np), b.astype(rdt.np)), bool_)
        if rdt.kind == "f":
            with _np.errstate(all="ignore"):
                r = fn(a.astype(_np.float64), b.astype(_np.float64))
            return array._wrap(r, rdt)
        with _np.errstate(all="ignore"):
            r = fn(a.astype(rdt.np), b.astype(rdt.np))
        return array._wrap(r, rdt)

    def __add__(self, o): return self._bin(o, _np.add)
    def __radd__(self, o): return self._bin(o, _np.add, True)
    def __sub__(self, o): return self._bin(o, _np.subtract)
    def __rsub__(self, o): return self._bin(o, _np.subtract, True)
    def __mul__(self, o): return self._bin(o, _np.multiply)
    def __rmul__(self, o): return self._bin(o, _np.multiply, True)

    def __truediv__(self, o):
        if not isinstance(o, array) and self.dtype.kind != "f":
            return self.astype(float32)._bin(o, _np.divide)
        return self._bin(o, _np.divide)

    def __rtruediv__(self, o): return self._bin(o, _np.divide, True)
    def __floordiv__(self, o): return self._bin(o, _np.floor_divide)
    def __mod__(self, o): return self._bin(o, _np.mod)
    def __rshift__(self, o): return self._bin(o, _np.right_shift)
    def __lshift__(self, o): return self._bin(o, _np.left_shift)
    def __and__(self, o): return self._bin(o, _np.bitwise_and)
    def __or__(self, o): return self._bin(o, _np.bitwise_or)
    def __lt__(self, o): return self._bin(o, _np.less, kind="cmp")
    def __le__(self, o): return self._bin(o, _np.less_equal, kind="cmp")
    def __gt__(self, o): return self._bin(o, _np.greater, kind="cmp")
    def __ge__(self, o): return self._bin(o, _np.greater_equal, kind="cmp")
    def __eq__(self, o): return self._bin(o, _np.equal, kind="cmp")
    def __ne__(self, o): return self._bin(o, _np.not_equal, kind="cmp")
    def __neg__(self): return array._wrap(-self._a, self.dtype)
    __hash__ = object.__hash__

    def __matmul__(self, o):
        return matmul(self, o)


# ---------------------------------------------------------------------------
# free functions
# ---------------------------------------------------------------------------

def _arr(x):
    return x if isinstance(x, array) else array(x)


def abs(x):  # noqa: A001
    x = _arr(x)
    return array._wrap(_np.abs(x._a), x.dtype)


def round(x, decimals=0):  # noqa: A001
    x = _arr(x)
    return array._wrap(_np.rint(x._a.astype(_np.float64)), x.dtype)


def maximum(a, b):
    a = _arr(a)
    return a._bin(b, _np.maximum)


def minimum(a, b):
    a = _arr(a)
    return a._bin(b, _np.minimum)


def clip(x, a_min, a_max):
    x = _arr(x)
    r = x
    if a_min is not None:
        r = maximum(r, a_min)
    if a_max is not None:
        r = minimum(r, a_max)
    return r


def where(cond, a, b):
    cond = _arr(cond)
    if isinstance(a, array) and isinstance(b, array):
        dt = _promote(a.dtype, b.dtype)
    elif isinstance(a, array):
        dt = _promote(a.dtype, _weak(b, a.dtype))
    elif isinstance(b, array):
        dt = _promote(b.dtype, _weak(a, b.dtype))
    else:
        dt = array(a).dtype
    av = a._a if isinstance(a, array) else _cast(_np.asarray(a), dt)
    bv = b._a if isinstance(b, array) else _cast(_np.asarray(b), dt)
    return array._wrap(_np.where(cond._a.astype(bool), av.astype(_np.float64) if dt.kind == "f" else av,
                                 bv.astype(_np.float64) if dt.kind == "f" else bv), dt)


def concatenate(arrays, axis=0):
    dt = arrays[0].dtype
    for a in arrays[1:]:
        dt = _promote(dt, a.dtype)
    return array._wrap(_np.concatenate([_cast(a._a, dt) for a in arrays], axis=axis), dt)


def take(a, indices, axis=None):
    idx = indices._a if isinstance(indices, array) else _np.asarray(indices)
    return array._wrap(_np.take(a._a, idx, axis=axis), a.dtype)


def arange(start, stop=None, step=None, dtype=None):
    if stop is None:
        start, stop = 0, start
    v = _np.arange(start, stop, step if step is not None else 1)
    if dtype is None:
        dtype = float32 if any(isinstance(x, float) for x in (start, stop, step)) else int32
    return array._wrap(v, dtype)


def zeros(shape, dtype=float32):
    return array._wrap(_np.zeros(shape, dtype=dtype.np), dtype)


def ones(shape, dtype=float32):
    return array._wrap(_np.ones(shape, dtype=dtype.np), dtype)


def zeros_like(x):
    return array._wrap(_np.zeros_like(x._a), x.dtype)


def pad(x, pad_width, constant_values=0):
    return array._wrap(_np.pad(x._a, pad_width, constant_values=constant_values), x.dtype)


def sum(x, axis=None, keepdims=False):  # noqa: A001
    x = _arr(x)
    dt = int32 if x.dtype.kind == "b" else x.dtype
    r = _np.sum(x._a.astype(_np.float64) if dt.kind == "f" else x._a.astype(_np.int64), axis=axis, keepdims=keepdims)
    return array._wrap(r, dt)


def matmul(a, b):
    a, b = _arr(a), _arr(b)
    dt = _promote(a.dtype, b.dtype)
    r = _np.matmul(a._a.astype(_np.float64), b._a.astype(_np.float64))
    return array._wrap(r, dt)


def softmax(x, axis=-1, precise=False):
    x = _arr(x)
    v = x._a.astype(_np.float64)
    v = v - v.max(axis=axis, keepdims=True)
    e = _np.exp(v)
    return array._wrap(e / e.sum(axis=axis, keepdims=True), x.dtype)


def eval(*args):  # noqa: A001
    return None


class finfo:
    def __init__(self, dtype):
        self.min = {"float16": -65504.0, "bfloat16": -3.3895313892515355e38,
                    "float32": float(_np.finfo(_np.float32).min)}[dtype.name]
        self.max = -self.min


# ---------------------------------------------------------------------------
# mx.random (seeded, for running the reference's own tests)
# ---------------------------------------------------------------------------

class _Random:
    def __init__(self):
        self._g = _np.random.default_rng(0)

    def seed(self, s):
        self._g = _np.random.default_rng(s)

    def normal(self, shape=(), dtype=float32, loc=0.0, scale=1.0, key=None):
        return array._wrap(self._g.standard_normal(shape) * scale + loc, dtype)

    def randint(self, low, high, shape=(), dtype=int32, key=None):
        return array._wrap(self._g.integers(low, high, size=shape), dtype)


random = _Random()


# ---------------------------------------------------------------------------
# mx.fast.metal_kernel -- restatements of the reference's two Metal kernels
# ---------------------------------------------------------------------------

class _PackKernel:
    """Restates kernels.py:9-22: word w = OR_i (codes[8w+i] & 0xF) << 4i."""

    def __call__(self, inputs, grid, threadgroup, output_shapes, output_dtypes, **kw):
        flat = inputs[0]._a.astype(_np.uint32)
        nw = output_shapes[0][0]
        out = _np.zeros(nw, _np.uint32)
        for i in range(8):
            idx = _np.arange(nw) * 8 + i
            ok = idx < flat.size
            vals = _np.zeros(nw, _np.uint32)
            vals[ok] = flat[idx[ok]] & _np.uint32(0xF)
            out |= vals << _np.uint32(4 * i)
        return [array._wrap(out, output_dtypes[0])]


class _SdpaKernel:
    """Restates the fused decode kernel kernels.py:79-228 (exact softmax,
    fp32 ``anchor + code*scale`` dequant, output fp32 [Hq*D])."""

    def __call__(self, inputs, grid, threadgroup, output_shapes, output_dtypes, **kw):
        q, kfk, pk, sk, kfv, pv, sv, params = [x._a for x in inputs]
        T, sk_, sv_ = (int(x) for x in params)
        Hq, D = q.shape
        Hkv = kfk.shape[0]
        rep = Hq // Hkv

        def dq(kf, packed, scales, stride):
            pos = _np.arange(T)
            a = pos // stride
            is_kf = pos % stride == 0
            pf = _np.where(is_kf, 0, pos - a - 1)
            val = kf[:, a, :].astype(_np.float64)
            words = packed[:, pf, :].astype(_np.uint32)
            dims = _np.arange(D)
            nib = ((words[:, :, dims >> 3] >> ((dims & 7) << 2).astype(_np.uint32)) & 0xF).astype(_np.int64) - 8
            sc = scales[:, pf].astype(_np.float32).astype(_np.float64)
            add = nib.astype(_np.float64) * sc[..., None]
            return val + _np.where(is_kf[None, :, None], 0.0, add)

        k = dq(kfk, pk, sk, sk_)
        v = dq(kfv, pv, sv, sv_)
        out = _np.zeros((Hq, D))
        for h in range(Hq):
            s = k[h // rep] @ q[h].astype(_np.float64)
            p = _np.exp(s - s.max())
            out[h] = (p @ v[h // rep]) / p.sum()
        return [array._wrap(out.reshape(-1), output_dtypes[0])]


class _Fast:
    def metal_kernel(self, name, input_names, output_names, source, header="", **kw):
        if name == "chronoquant_pack_int4":
            return _PackKernel()
        if name == "chronoquant_sdpa":
            return _SdpaKernel()
        raise NotImplementedError(f"no restatement for Metal kernel {name!r}")


fast = _Fast()
