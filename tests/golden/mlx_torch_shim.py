"""A minimal PyTorch (CPU) stand-in for the parts of the ``mlx`` API the reference MoE uses.

MLX cannot be installed in this environment, so golden vectors are produced by executing
the reference's own, unmodified ``dspark_mlx/model/moe.py`` (and the dequant helpers in
``dspark_mlx/loading.py``) over this stand-in. The stand-in restates MLX's documented
semantics: dtype promotion (bf16 op fp32 -> fp32, Python scalars are weak), fp32
accumulation inside ``matmul`` / ``gather_mm`` / ``gather_qmm`` with the result in the
promoted (resp. activation) dtype, numpy-style broadcasting for ``take_along_axis`` and
the ``gather_mm`` batch/index shapes, ``nn.Module`` as a dict of parameters, and the affine
``quantize``. Summation order inside MLX kernels and ``argsort`` tie order are not
reproducible here; ``argsort`` is a stable ascending sort.

Test infrastructure only: used by ``make_golden.py`` and by the tests that replay the
reference's own unit tests through it.
"""

from __future__ import annotations

import sys
import types
from typing import Optional

import numpy as np
import torch

float32 = torch.float32
float16 = torch.float16
bfloat16 = torch.bfloat16
int32 = torch.int32
int64 = torch.int64
uint32 = torch.int64  # unsigned 32-bit results are carried as int64
uint8 = torch.uint8
bool_ = torch.bool


def _t(v, like: Optional[torch.Tensor] = None) -> torch.Tensor:
    if isinstance(v, array):
        return v.t
    if isinstance(v, torch.Tensor):
        return v
    if isinstance(v, (int, float, bool)) and like is not None:
        return torch.tensor(v, dtype=like.dtype if not isinstance(v, float) or like.is_floating_point() else torch.float32)
    a = np.asarray(v)
    if a.dtype == np.float64:
        a = a.astype(np.float32)
    if a.dtype == np.int64:
        a = a.astype(np.int32)
    return torch.from_numpy(np.ascontiguousarray(a))


class array:
    """A tensor wrapper with the mlx.core.array surface the reference touches."""

    __slots__ = ("t",)

    def __init__(self, v, dtype=None):
        t = _t(v)
        if dtype is not None:
            t = t.to(dtype)
        self.t = t

    # -- metadata -------------------------------------------------------------------------
    @property
    def shape(self):
        return tuple(self.t.shape)

    @property
    def dtype(self):
        return self.t.dtype

    @property
    def ndim(self):
        return self.t.ndim

    @property
    def size(self):
        return self.t.numel()

    @property
    def nbytes(self):
        return self.t.numel() * self.t.element_size()

    # -- conversion -----------------------------------------------------------------------
    def astype(self, dtype):
        return array(self.t.to(dtype))

    def __array__(self, dtype=None, copy=None):
        t = self.t
        if t.dtype == torch.bfloat16:
            t = t.to(torch.float32)
        a = t.detach().numpy()
        return a.astype(dtype) if dtype is not None else a

    def item(self):
        return self.t.item()

    def tolist(self):
        return self.t.tolist()

    def __float__(self):
        return float(self.t)

    def __int__(self):
        return int(self.t)

    # -- shape ops ------------------------------------------------------------------------
    def reshape(self, *shape):
        if len(shape) == 1 and isinstance(shape[0], (tuple, list)):
            shape = tuple(shape[0])
        return array(self.t.reshape(shape))

    @property
    def T(self):
        return array(self.t.permute(*reversed(range(self.t.ndim))))

    def swapaxes(self, a, b):
        return array(self.t.transpose(a, b))

    def transpose(self, *axes):
        return array(self.t.permute(*axes))

    def squeeze(self, axis=None):
        return array(self.t.squeeze() if axis is None else self.t.squeeze(axis))

    def __getitem__(self, key):
        def conv(k):
            if isinstance(k, array):
                k = k.t
            if isinstance(k, torch.Tensor) and not k.dtype == torch.bool:
                return k.to(torch.int64)
            return k

        key = tuple(conv(k) for k in key) if isinstance(key, tuple) else conv(key)
        return array(self.t[key])

    def __len__(self):
        return self.t.shape[0]

    # -- arithmetic -----------------------------------------------------------------------
    def _bin(self, other, fn):
        return array(fn(self.t, other.t if isinstance(other, array) else other))

    def __add__(self, o):
        return self._bin(o, torch.add)

    def __radd__(self, o):
        return self._bin(o, lambda a, b: b + a)

    def __sub__(self, o):
        return self._bin(o, torch.sub)

    def __rsub__(self, o):
        return self._bin(o, lambda a, b: b - a)

    def __mul__(self, o):
        return self._bin(o, torch.mul)

    def __rmul__(self, o):
        return self._bin(o, lambda a, b: b * a)

    def __truediv__(self, o):
        return self._bin(o, torch.true_divide)

    def __rtruediv__(self, o):
        return self._bin(o, lambda a, b: b / a)

    def __pow__(self, o):
        return self._bin(o, torch.pow)

    def __rpow__(self, o):
        return array(torch.pow(torch.tensor(o, dtype=self.t.dtype), self.t))

    def __matmul__(self, o):
        return matmul(self, o)

    def __neg__(self):
        return array(-self.t)

    def __eq__(self, o):
        return self._bin(o, torch.eq)

    def __ne__(self, o):
        return self._bin(o, torch.ne)

    def __lt__(self, o):
        return self._bin(o, torch.lt)

    def __le__(self, o):
        return self._bin(o, torch.le)

    def __gt__(self, o):
        return self._bin(o, torch.gt)

    def __ge__(self, o):
        return self._bin(o, torch.ge)

    __hash__ = object.__hash__


def _promote(a: torch.Tensor, b: torch.Tensor) -> torch.dtype:
    return torch.promote_types(a.dtype, b.dtype)


def zeros(shape, dtype=float32):
    return array(torch.zeros(shape, dtype=dtype))


def ones(shape, dtype=float32):
    return array(torch.ones(shape, dtype=dtype))


def full(shape, value, dtype=None):
    return array(torch.full(shape if isinstance(shape, (tuple, list)) else (shape,), value, dtype=dtype))


def eval(*args):  # noqa: A001 - mirrors mx.eval
    return None


def matmul(a, b):
    a, b = _t(a), _t(b)
    return array((a.to(torch.float32) @ b.to(torch.float32)).to(_promote(a, b)))


def _unary(fn):
    def f(x):
        x = _t(x)
        return array(fn(x.to(torch.float32)).to(x.dtype) if x.is_floating_point() else fn(x))

    return f


exp = _unary(torch.exp)
log1p = _unary(torch.log1p)
sqrt = _unary(torch.sqrt)
rsqrt = _unary(torch.rsqrt)
sigmoid = _unary(torch.sigmoid)
abs = _unary(torch.abs)  # noqa: A001
log = _unary(torch.log)
cos = _unary(torch.cos)
sin = _unary(torch.sin)
round = _unary(torch.round)  # noqa: A001


def softmax(x, axis=-1):
    x = _t(x)
    return array(torch.softmax(x.to(torch.float32), dim=axis).to(x.dtype))


def maximum(a, b):
    ta = _t(a)
    tb = _t(b, like=ta)
    return array(torch.maximum(ta, tb.to(ta.dtype) if tb.ndim == 0 else tb))


def minimum(a, b):
    ta = _t(a)
    tb = _t(b, like=ta)
    return array(torch.minimum(ta, tb.to(ta.dtype) if tb.ndim == 0 else tb))


def clip(x, lo, hi):
    return array(torch.clamp(_t(x), lo, hi))


def where(cond, a, b):
    c = _t(cond)
    ta = _t(a) if isinstance(a, (array, torch.Tensor)) else None
    tb = _t(b) if isinstance(b, (array, torch.Tensor)) else None
    ref = ta if ta is not None else tb
    ta = ta if ta is not None else torch.tensor(a, dtype=ref.dtype)
    tb = tb if tb is not None else torch.tensor(b, dtype=ref.dtype)
    return array(torch.where(c, ta, tb))


def sum(x, axis=None, keepdims=False):  # noqa: A001
    x = _t(x)
    if axis is None:
        return array(x.sum())
    return array(x.sum(dim=axis, keepdim=keepdims))


def mean(x, axis=None, keepdims=False):
    x = _t(x)
    if axis is None:
        return array(x.mean())
    return array(x.mean(dim=axis, keepdim=keepdims))


def max(x, axis=None, keepdims=False):  # noqa: A001
    x = _t(x)
    if axis is None:
        return array(x.max())
    return array(x.amax(dim=axis, keepdim=keepdims))


def argmax(x, axis=-1):
    return array(_t(x).argmax(dim=axis).to(torch.int32))


def argsort(x, axis=-1):
    return array(torch.sort(_t(x), dim=axis, stable=True).indices.to(torch.int32))


def take_along_axis(a, idx, axis):
    ta, ti = _t(a), _t(idx).to(torch.int64)
    nd = builtins_max(ta.ndim, ti.ndim)
    ta = ta.reshape((1,) * (nd - ta.ndim) + tuple(ta.shape))
    ti = ti.reshape((1,) * (nd - ti.ndim) + tuple(ti.shape))
    ax = axis % nd
    bshape = []
    for d in range(nd):
        if d == ax:
            bshape.append(None)
        else:
            sa, si = ta.shape[d], ti.shape[d]
            if sa != si and sa != 1 and si != 1:
                raise ValueError(f"take_along_axis: cannot broadcast {tuple(ta.shape)} with {tuple(ti.shape)}")
            bshape.append(builtins_max(sa, si))
    ea = [ta.shape[d] if d == ax else bshape[d] for d in range(nd)]
    ei = [ti.shape[d] if d == ax else bshape[d] for d in range(nd)]
    return array(torch.gather(ta.expand(*ea), ax, ti.expand(*ei)))


def expand_dims(x, axes):
    t = _t(x)
    if isinstance(axes, int):
        axes = (axes,)
    out_nd = t.ndim + len(axes)
    norm = sorted(a % out_nd for a in axes)
    for a in norm:
        t = t.unsqueeze(a)
    return array(t)


def concatenate(xs, axis=0):
    return array(torch.cat([_t(x) for x in xs], dim=axis))


def stack(xs, axis=0):
    return array(torch.stack([_t(x) for x in xs], dim=axis))


def broadcast_to(x, shape):
    return array(_t(x).expand(*shape))


def swapaxes(x, a, b):
    return array(_t(x).transpose(a, b))


def outer(a, b):
    return array(torch.outer(_t(a), _t(b)))


def arange(*args, dtype=None):
    return array(torch.arange(*args, dtype=dtype))


def _gathered(b: torch.Tensor, lhs_batch, rhs_indices):
    """Broadcast ``lhs_batch`` (a shape) with ``rhs_indices`` and select rhs matrices."""
    idx = _t(rhs_indices).to(torch.int64)
    bshape = torch.broadcast_shapes(tuple(lhs_batch), tuple(idx.shape))
    return bshape, b[idx.expand(*bshape)]


def gather_mm(a, b, lhs_indices=None, rhs_indices=None, sorted_indices=False):
    ta, tb = _t(a), _t(b)
    if lhs_indices is not None:
        raise NotImplementedError("lhs_indices")
    bshape, rsel = _gathered(tb, ta.shape[:-2], rhs_indices)
    lhs = ta.expand(*bshape, *ta.shape[-2:])
    out = lhs.to(torch.float32) @ rsel.to(torch.float32)
    return array(out.to(_promote(ta, tb)))


def _unpack(wq: torch.Tensor, bits: int) -> torch.Tensor:
    c = wq.to(torch.int32)
    if bits == 8:
        return c
    lo, hi = c & 0xF, (c >> 4) & 0xF
    return torch.stack([lo, hi], dim=-1).reshape(*c.shape[:-1], c.shape[-1] * 2)


def dequantize(wq, scales, biases, group_size=64, bits=4):
    q = _unpack(_t(wq), bits).to(torch.float32)
    s = _t(scales).to(torch.float32).repeat_interleave(group_size, dim=-1)
    b = _t(biases).to(torch.float32).repeat_interleave(group_size, dim=-1)
    return array((q * s + b).to(_t(scales).dtype))


def gather_qmm(x, w, scales, biases, lhs_indices=None, rhs_indices=None, transpose=True,
               group_size=64, bits=4, sorted_indices=False):
    tx = _t(x)
    q = _unpack(_t(w), bits).to(torch.float32)
    s = _t(scales).to(torch.float32).repeat_interleave(group_size, dim=-1)
    bb = _t(biases).to(torch.float32).repeat_interleave(group_size, dim=-1)
    wd = q * s + bb  # [E, out, in], fp32
    if transpose:
        wd = wd.transpose(-1, -2)
    if lhs_indices is not None:
        raise NotImplementedError("lhs_indices")
    bshape, rsel = _gathered(wd, tx.shape[:-2], rhs_indices)
    lhs = tx.expand(*bshape, *tx.shape[-2:])
    return array((lhs.to(torch.float32) @ rsel).to(tx.dtype))


def quantize(w, group_size=64, bits=4):
    """MLX affine quantize (fp32 arithmetic; scales/biases stored in the weight dtype)."""
    tw = _t(w)
    shape = tw.shape
    K = shape[-1]
    wf = tw.to(torch.float32).reshape(-1, K // group_size, group_size)
    n_bins = float((1 << bits) - 1)
    w_max = wf.amax(dim=-1, keepdim=True)
    w_min = wf.amin(dim=-1, keepdim=True)
    mask = w_min.abs() > w_max.abs()
    scale = torch.clamp((w_max - w_min) / n_bins, min=1e-7)
    scale = torch.where(mask, scale, -scale)
    edge = torch.where(mask, w_min, w_max)
    q0 = torch.round(edge / scale)
    scale = torch.where(q0 != 0, edge / q0, scale)
    bias = torch.where(q0 == 0, torch.zeros_like(edge), edge)
    q = torch.clamp(torch.round((wf - bias) / scale), 0, n_bins).to(torch.uint8).reshape(*shape[:-1], K)
    codes = q if bits == 8 else (q[..., 0::2] | (q[..., 1::2] << 4)).to(torch.uint8)
    return (array(codes), array(scale.reshape(*shape[:-1], K // group_size).to(tw.dtype)),
            array(bias.reshape(*shape[:-1], K // group_size).to(tw.dtype)))


builtins_max = __builtins__["max"] if isinstance(__builtins__, dict) else __builtins__.max


# ---------------------------------------------------------------------------------------
# mlx.nn
# ---------------------------------------------------------------------------------------
class Module(dict):
    """Parameters and sub-modules live in the dict; other attributes are plain attributes."""

    def __init__(self):
        super().__init__()

    def __getattr__(self, key):
        try:
            return self[key]
        except KeyError:
            raise AttributeError(key) from None

    def __setattr__(self, key, value):
        if isinstance(value, (array, Module, list, dict)):
            self[key] = value
            if key in self.__dict__:
                del self.__dict__[key]
        else:
            if key in self:
                del self[key]
            object.__setattr__(self, key, value)

    def __delattr__(self, key):
        if key in self:
            del self[key]
        else:
            object.__delattr__(self, key)

    def parameters(self):
        """The arrays of this module and its children as a nested dict (lists stay lists), as
        ``mlx.nn.Module.parameters`` returns them."""

        def conv(v):
            if isinstance(v, Module):
                return v.parameters()
            if isinstance(v, (list, tuple)):
                return [conv(x) for x in v]
            return v

        return {k: conv(v) for k, v in self.items() if isinstance(v, (array, Module, list, tuple))}

    def update(self, tree):
        """Replace arrays from a nested dict as ``mlx.nn.Module.update`` does."""

        def put(cur, new):
            if isinstance(cur, Module):
                for k, v in new.items():
                    if isinstance(cur.get(k), (Module, list)):
                        put(cur[k], v)
                    else:
                        cur[k] = v
            elif isinstance(cur, list):
                items = new.items() if isinstance(new, dict) else enumerate(new)
                for i, v in items:
                    put(cur[int(i)], v)

        put(self, tree)
        return self

    def named_modules(self):
        out = [("", self)]

        def walk(prefix, m):
            for k, v in m.items():
                if isinstance(v, Module):
                    out.append((prefix + k, v))
                    walk(prefix + k + ".", v)

        walk("", self)
        return out


class Linear(Module):
    def __init__(self, input_dims: int, output_dims: int, bias: bool = True):
        super().__init__()
        scale = 1.0 / np.sqrt(input_dims)
        self.weight = array(torch.empty(output_dims, input_dims).uniform_(-scale, scale))
        if bias:
            self.bias = array(torch.zeros(output_dims))

    def __call__(self, x):
        y = matmul(x, self.weight.T)
        if "bias" in self:
            y = y + self.bias
        return y


def silu(x):
    return x * sigmoid(x)


class Embedding(Module):
    def __init__(self, num_embeddings: int, dims: int):
        super().__init__()
        self.weight = array(torch.randn(num_embeddings, dims) * (1.0 / np.sqrt(dims)))

    def __call__(self, x):
        return array(self.weight.t[_t(x).to(torch.int64)])


# mlx.core.random.uniform served from a seeded torch generator; every draw is recorded so a
# golden case can store the uniforms the reference's sampler consumed
_random_gen = torch.Generator().manual_seed(0)
random_draws: list = []


def _uniform(low=0.0, high=1.0, shape=(), dtype=float32, key=None):
    u = torch.rand(tuple(shape), generator=_random_gen) * (high - low) + low
    random_draws.append(u.clone())
    return array(u.to(dtype))


def _sdpa(q, k, v, scale, mask=None):
    """``mx.fast.scaled_dot_product_attention``: softmax(q k^T * scale) v with fp32
    accumulation and q's dtype out; grouped-query heads share their KV head."""
    tq, tk, tv = _t(q), _t(k), _t(v)
    rep = tq.shape[1] // tk.shape[1]
    kf = tk.to(torch.float32).repeat_interleave(rep, dim=1)
    vf = tv.to(torch.float32).repeat_interleave(rep, dim=1)
    s = (tq.to(torch.float32) @ kf.transpose(-1, -2)) * scale
    if mask is not None:
        s = s + _t(mask).to(torch.float32)
    return array((torch.softmax(s, dim=-1) @ vf).to(tq.dtype))


def random_seed(seed: int) -> None:
    _random_gen.manual_seed(seed)
    random_draws.clear()


def _tree_unflatten(items):
    out = {}
    for path, v in items:
        node = out
        parts = path.split(".")
        for p in parts[:-1]:
            node = node.setdefault(p, {})
        node[parts[-1]] = v
    return out


def _tree_flatten(tree, prefix=""):
    out = []
    if isinstance(tree, dict):
        for k, v in tree.items():
            out.extend(_tree_flatten(v, f"{prefix}{k}."))
    elif isinstance(tree, (list, tuple)):
        for i, v in enumerate(tree):
            out.extend(_tree_flatten(v, f"{prefix}{i}."))
    else:
        out.append((prefix[:-1], tree))
    return out


def install() -> None:
    """Register ``mlx``, ``mlx.core``, ``mlx.nn`` and ``mlx.utils`` in ``sys.modules``."""
    core = sys.modules[__name__]
    mlx = types.ModuleType("mlx")
    nn = types.ModuleType("mlx.nn")
    nn.Module = Module
    nn.Linear = Linear
    nn.silu = silu
    nn.Embedding = Embedding
    fast = types.ModuleType("mlx.core.fast")
    fast.scaled_dot_product_attention = _sdpa
    core.fast = fast
    rnd = types.ModuleType("mlx.core.random")
    rnd.uniform = _uniform
    rnd.seed = random_seed
    core.random = rnd
    utils = types.ModuleType("mlx.utils")
    utils.tree_unflatten = _tree_unflatten
    utils.tree_flatten = _tree_flatten
    mlx.core = core
    mlx.nn = nn
    mlx.utils = utils
    sys.modules["mlx"] = mlx
    sys.modules["mlx.core"] = core
    sys.modules["mlx.nn"] = nn
    sys.modules["mlx.utils"] = utils
