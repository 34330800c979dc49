"""mlx.core stand-in on torch CPU tensors (test infrastructure; ../README.md).

Semantics follow MLX's documentation for the operations the reference's MoE
block calls:
  * an array has a dtype; results of binary operations take the promoted
    dtype (a floating type wins over integer types, float32 over the half
    types, and bfloat16 with float16 gives float32); Python scalars are
    weakly typed and never promote an array;
  * elementwise results are computed in float32 and rounded once to the
    result dtype;
  * reductions accumulate in float32 and round to the input dtype;
  * softmax(precise=True) accumulates in float32 and returns the input dtype;
  * argpartition returns indices of a valid partition (here: a stable
    ascending sort, so equal keys keep ascending index order);
  * quantized products dequantise w = scale * q + bias per group (q in bits
    4 (k % 8) of word k / 8), accumulate in float32 and round the result once
    to the promoted dtype of x, scales and biases.
"""
from __future__ import annotations

import numpy as np
import torch


class Dtype:
    def __init__(self, name: str, t: torch.dtype):
        self.name = name
        self.torch = t

    def __repr__(self):
        return f"mlx.core.{self.name}"

    def __eq__(self, other):
        return isinstance(other, Dtype) and other.torch == self.torch

    def __hash__(self):
        return hash(self.torch)


bfloat16 = Dtype("bfloat16", torch.bfloat16)
float16 = Dtype("float16", torch.float16)
float32 = Dtype("float32", torch.float32)
int32 = Dtype("int32", torch.int32)
int64 = Dtype("int64", torch.int64)
uint32 = Dtype("uint32", torch.int64)   # held widened; only used for indices
bool_ = Dtype("bool", torch.bool)
_BY_TORCH = {d.torch: d for d in (bfloat16, float16, float32, int32, int64, bool_)}

_HALF = (torch.float16, torch.bfloat16)


def _promote(a: torch.dtype, b: torch.dtype) -> torch.dtype:
    if a == b:
        return a
    fa, fb = a.is_floating_point, b.is_floating_point
    if fa and not fb:
        return a
    if fb and not fa:
        return b
    if fa and fb:
        return torch.float32   # float32 with anything, or bfloat16 with float16
    return torch.promote_types(a, b)


def _tensor(v) -> torch.Tensor:
    if isinstance(v, array):
        return v._t
    if isinstance(v, torch.Tensor):
        return v
    a = np.asarray(v)
    if a.dtype == np.float64:
        a = a.astype(np.float32)
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32).copy())  # bit pattern kept
    if a.dtype == np.uint16:
        return torch.from_numpy(a.astype(np.int32))
    return torch.from_numpy(np.ascontiguousarray(a).copy())


def _round(t32: torch.Tensor, dt: torch.dtype) -> torch.Tensor:
    return t32 if dt == torch.float32 else t32.to(dt)


class array:
    """An MLX-like array: a torch CPU tensor plus its MLX dtype."""

    __array_priority__ = 1000

    def __init__(self, val, dtype: Dtype = None):
        t = _tensor(val)
        if dtype is not None:
            t = t.to(dtype.torch)
        self._t = t

    # -- metadata ------------------------------------------------------------
    @property
    def dtype(self) -> Dtype:
        return _BY_TORCH.get(self._t.dtype, Dtype(str(self._t.dtype), self._t.dtype))

    @property
    def shape(self):
        return tuple(self._t.shape)

    @property
    def ndim(self):
        return self._t.dim()

    @property
    def size(self):
        return self._t.numel()

    def __len__(self):
        return self._t.shape[0]

    def __array__(self, dtype=None, copy=None):
        t = self._t
        if t.dtype in _HALF:
            t = t.float()
        a = t.numpy()
        return a.astype(dtype) if dtype is not None else a

    def __repr__(self):
        return f"array({self._t}, dtype={self.dtype})"

    def item(self):
        return self._t.item()

    def tolist(self):
        return self._t.tolist()

    # -- shape ---------------------------------------------------------------
    def reshape(self, *shape):
        if len(shape) == 1 and isinstance(shape[0], (tuple, list)):
            shape = tuple(shape[0])
        return array(self._t.reshape(shape))

    def squeeze(self, axis=None):
        return array(self._t.squeeze() if axis is None else self._t.squeeze(axis))

    def flatten(self):
        return array(self._t.flatten())

    def astype(self, dtype: Dtype):
        return array(self._t.to(dtype.torch))

    def __getitem__(self, idx):
        if isinstance(idx, tuple):
            idx = tuple(i._t if isinstance(i, array) else i for i in idx)
        elif isinstance(idx, array):
            idx = idx._t
        return array(self._t[idx])

    # -- reductions ----------------------------------------------------------
    def sum(self, axis=None, keepdims=False):
        t = self._t
        dt = t.dtype
        acc = t.float() if dt.is_floating_point else t
        r = acc.sum() if axis is None else acc.sum(dim=axis, keepdim=keepdims)
        return array(_round(r, dt) if dt.is_floating_point else r)

    def max(self, axis=None, keepdims=False):
        t = self._t
        r = t.max() if axis is None else t.amax(dim=axis, keepdim=keepdims)
        return array(r)

    # -- arithmetic ----------------------------------------------------------
    def _binary(self, other, fn, reverse=False):
        a = self._t
        if isinstance(other, (array, torch.Tensor, np.ndarray)):
            b = _tensor(other)
            dt = _promote(a.dtype, b.dtype)
        else:  # Python scalar: weakly typed
            b = torch.tensor(other)
            dt = a.dtype if (a.dtype.is_floating_point or not isinstance(other, float)) \
                else torch.float32
        if dt.is_floating_point:
            x, y = a.float(), b.float()
            r = fn(y, x) if reverse else fn(x, y)
            return array(_round(r, dt))
        x, y = a.to(dt), b.to(dt)
        return array(fn(y, x) if reverse else fn(x, y))

    def __add__(self, o):
        return self._binary(o, torch.add)

    def __radd__(self, o):
        return self._binary(o, torch.add, True)

    def __sub__(self, o):
        return self._binary(o, torch.sub)

    def __rsub__(self, o):
        return self._binary(o, torch.sub, True)

    def __mul__(self, o):
        return self._binary(o, torch.mul)

    def __rmul__(self, o):
        return self._binary(o, torch.mul, True)

    def __truediv__(self, o):
        return self._binary(o, torch.div)

    def __rtruediv__(self, o):
        return self._binary(o, torch.div, True)

    def __neg__(self):
        return array(-self._t)

    def __matmul__(self, o):
        return matmul(self, o)


# --------------------------------------------------------------------------- #
# module-level operations
# --------------------------------------------------------------------------- #

def eval(*args):  # noqa: A001 - MLX's name; arrays here are always evaluated
    return None


def clear_cache():
    return None


def zeros(shape, dtype: Dtype = float32):
    return array(torch.zeros(shape, dtype=dtype.torch))


def stack(arrays, axis=0):
    return array(torch.stack([_tensor(a) for a in arrays], dim=axis))


def concatenate(arrays, axis=0):
    return array(torch.cat([_tensor(a) for a in arrays], dim=axis))


def expand_dims(a, axis):
    t = _tensor(a)
    axes = (axis,) if isinstance(axis, int) else tuple(axis)
    nd = t.dim() + len(axes)
    for ax in sorted(x % nd for x in axes):
        t = t.unsqueeze(ax)
    return array(t)


def matmul(a, b):
    """a @ b, accumulated in float32, rounded once to the promoted dtype."""
    x, y = _tensor(a), _tensor(b)
    dt = _promote(x.dtype, y.dtype)
    return array(_round(x.float() @ y.float(), dt))


def _unary_f32(a, fn):
    t = _tensor(a)
    dt = t.dtype if t.dtype.is_floating_point else torch.float32
    return array(_round(fn(t.float()), dt))


def sigmoid(a):
    return _unary_f32(a, torch.sigmoid)


def exp(a):
    return _unary_f32(a, torch.exp)


def softmax(a, axis=-1, precise=False):
    t = _tensor(a)
    dt = t.dtype
    if precise or dt == torch.float32:
        r = torch.softmax(t.float(), dim=axis)
    else:  # the exponentials and the sum in the input dtype
        m = t.amax(dim=axis, keepdim=True)
        e = torch.exp((t - m).float()).to(dt)
        s = e.float().sum(dim=axis, keepdim=True).to(dt)
        r = e.float() / s.float()
    return array(_round(r, dt))


def argpartition(a, kth, axis=-1):
    t = _tensor(a)
    order = torch.sort(t.float(), dim=axis, stable=True).indices
    return array(order.to(torch.int32))


def argsort(a, axis=-1):
    return argpartition(a, 0, axis)


def take_along_axis(a, indices, axis=-1):
    return array(torch.take_along_dim(_tensor(a), _tensor(indices).long(), dim=axis))


def _dequant(w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
             group_size: int, bits: int) -> torch.Tensor:
    """[..., N, K/8] int32 words + [..., N, K/group] scales/biases ->
    float32 [..., N, K] = scale * q + bias."""
    if bits != 4:
        raise NotImplementedError("the stand-in implements 4-bit quantisation")
    words = w.to(torch.int64) & 0xFFFFFFFF
    shifts = torch.arange(8, dtype=torch.int64) * 4
    q = ((words[..., None] >> shifts) & 0xF).float()
    q = q.reshape(*words.shape[:-1], words.shape[-1] * 8)
    *lead, n, k = q.shape
    qg = q.reshape(*lead, n, k // group_size, group_size)
    s = scales.float()[..., None]
    b = biases.float()[..., None]
    return (qg * s + b).reshape(*lead, n, k)


def quantized_matmul(x, w, scales, biases, transpose=True, group_size=64, bits=4):
    if not transpose:
        raise NotImplementedError("the stand-in implements transpose=True")
    xt, st, bt = _tensor(x), _tensor(scales), _tensor(biases)
    dt = _promote(_promote(xt.dtype, st.dtype), bt.dtype)
    W = _dequant(_tensor(w), st, bt, group_size, bits)
    return array(_round(xt.to(dt).float() @ W.transpose(-1, -2), dt))


def gather_qmm(x, w, scales, biases, lhs_indices=None, rhs_indices=None, transpose=True,
               group_size=64, bits=4, sorted_indices=False):
    """out[b] = x[b] @ dequant(w[rhs[b]]).T over the broadcast batch of x's
    leading dims and the index array."""
    if not transpose:
        raise NotImplementedError("the stand-in implements transpose=True")
    if lhs_indices is not None:
        raise NotImplementedError("the stand-in implements rhs gathers only")
    xt, wt, st, bt = _tensor(x), _tensor(w), _tensor(scales), _tensor(biases)
    dt = _promote(_promote(xt.dtype, st.dtype), bt.dtype)
    idx = _tensor(rhs_indices).long()
    batch = torch.broadcast_shapes(xt.shape[:-2], idx.shape)
    M, K = xt.shape[-2:]
    xb = xt.to(dt).float().expand(*batch, M, K).reshape(-1, M, K)
    ib = idx.expand(batch).reshape(-1)
    N = wt.shape[-2]
    out = torch.empty((ib.numel(), M, N), dtype=torch.float32)
    for e in torch.unique(ib).tolist():
        sel = (ib == e).nonzero().flatten()
        W = _dequant(wt[e], st[e], bt[e], group_size, bits)     # [N, K]
        out[sel] = xb[sel] @ W.t()
    return array(_round(out.reshape(*batch, M, N), dt))
