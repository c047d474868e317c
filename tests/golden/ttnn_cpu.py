"""A CPU stand-in for the ``ttnn`` operations the reference's Orb model code calls, so that
``make_golden.py`` can run the reference's own Orb forward and reverse pass
(tt_atom/orb_model.py:92-338, tt_atom/orb_forces.py:27-372, tt_atom/scatter.py:47-110) on
seeded inputs and commit the results as golden vectors.

Test infrastructure only: nothing in the package imports it. Every operation is the plain
fp32 torch meaning of the ttnn call (dtype, layout, memory and compute-kernel arguments are
accepted and ignored, so all values stay fp32: the reference's algorithm at fp32, not its
bf16 device arithmetic). The experimental fused ops are absent, so the reference takes its
stock-op paths. ``install()`` registers the module as ``ttnn``.
"""
from __future__ import annotations

import builtins
import sys
import types

import torch

TILE_LAYOUT, ROW_MAJOR_LAYOUT = "tile", "row_major"
bfloat16, bfloat8_b, float32, uint32 = "bfloat16", "bfloat8_b", "float32", "uint32"
DRAM_MEMORY_CONFIG, L1_MEMORY_CONFIG = "dram", "l1"


class MathFidelity:
    HiFi4 = "hifi4"
    HiFi2 = "hifi2"
    LoFi = "lofi"


def WormholeComputeKernelConfig(**kw):
    return dict(kw)


def from_torch(t, dtype=None, layout=None, device=None, **kw):
    t = torch.as_tensor(t)
    if t.is_floating_point():
        return t.detach().to(torch.float32).clone()
    return t.detach().to(torch.int64).clone()


def to_torch(t, **kw):
    return t


def to_layout(t, layout, **kw):
    return t


def linear(x, w, bias=None, **kw):
    y = x @ w
    return y + bias.reshape(-1) if bias is not None else y


def matmul(a, b, transpose_a=False, transpose_b=False, **kw):
    return (a.transpose(-1, -2) if transpose_a else a) @ (b.transpose(-1, -2) if transpose_b else b)


def silu(x, **kw):
    return torch.nn.functional.silu(x)


def sigmoid(x, **kw):
    return torch.sigmoid(x)


def rsqrt(x, **kw):
    return torch.rsqrt(x)


def multiply(a, b, **kw):
    return a * b


def add(a, b, **kw):
    return a + b


def subtract(a, b, **kw):
    return a - b


def mean(x, dim, keepdim=False, **kw):
    return x.mean(dim=dim, keepdim=keepdim)


def sum(x, dim, keepdim=False, **kw):  # noqa: A001 - the ttnn name
    return x.sum(dim=dim, keepdim=keepdim)


def embedding(idx, table, **kw):
    return table[idx.long().reshape(-1)]


def concat(ts, dim=0, **kw):
    return torch.cat(list(ts), dim=dim)


def slice(t, start, end, **kw):  # noqa: A001 - the ttnn name
    return t[tuple(builtins.slice(a, b) for a, b in zip(start, end))]


def reshape(t, shape, **kw):
    return t.reshape(tuple(shape))


def ones(shape, dtype=None, layout=None, device=None, **kw):
    return torch.ones(tuple(shape), dtype=torch.float32)


def zeros(shape, dtype=None, layout=None, device=None, **kw):
    return torch.zeros(tuple(shape), dtype=torch.float32)


def silu_bw(grad, x, **kw):
    s = torch.sigmoid(x)
    return [grad * (s * (1.0 + x * (1.0 - s)))]


def sigmoid_bw(grad, x, **kw):
    s = torch.sigmoid(x)
    return [grad * s * (1.0 - s)]


experimental = types.SimpleNamespace()     # no minimal_matmul: the reference's stock matmuls


def install():
    """Register this module as ``ttnn`` (with an empty experimental-ops package)."""
    me = sys.modules[__name__]
    sys.modules["ttnn"] = me
    pk = types.ModuleType("ttnn._ttnn")
    ops = types.ModuleType("ttnn._ttnn.operations")
    exp = types.ModuleType("ttnn._ttnn.operations.experimental")
    pk.operations, ops.experimental = ops, exp
    me._ttnn = pk
    sys.modules.update({"ttnn._ttnn": pk, "ttnn._ttnn.operations": ops,
                        "ttnn._ttnn.operations.experimental": exp})
    return me
