"""Einsum contraction engine: canonicalise to batched GEMM, run the native kernel.

A two-operand equation ``X,Y->Z`` is classified per letter:

* batch ``B``  - in X, Y and Z
* row   ``M``  - in X and Z only
* col   ``N``  - in Y and Z only
* red.  ``K``  - in X and Y, not Z
* letters of only one operand and not Z are summed out first.

X is viewed as ``[B, M, K]`` and Y as ``[B, K, N]`` (a permute plus reshape,
which is free whenever the grouped dimensions are adjacent in memory), the
product ``[B, M, N]`` is computed by :func:`..ops.gemm.matmul` and the result is
reshaped/permuted to Z's order.  The native GEMM reads either operand in
K-major or MN-major order, so transposed views need no copy.

Equations with repeated letters inside one operand (diagonals), ellipses that
cannot be aligned, a single operand, or dtypes/devices the native kernel does
not cover go to ``torch.einsum``.

Replaces the reference's local ``torch.einsum`` call
(``src/torch_einshard/einsum.py:132``) for bf16/fp16 CUDA operands.
"""

import math

import torch

from . import gemm

__all__ = ["contract", "canonical_gemm"]


def _split_eq(equation):
    lhs, rhs = equation.split("->")
    return lhs.split(","), rhs


def canonical_gemm(equation, x_shape, y_shape):
    """Return the batched-GEMM decomposition of ``equation`` or ``None``."""
    (ex, ey), ez = _split_eq(equation)
    if "..." in equation:
        return None
    if len(set(ex)) != len(ex) or len(set(ey)) != len(ey) or len(set(ez)) != len(ez):
        return None
    if len(ex) != len(x_shape) or len(ey) != len(y_shape):
        return None
    sx, sy, sz = set(ex), set(ey), set(ez)
    if not sz <= (sx | sy):
        return None
    size = {}
    for letters, shape in ((ex, x_shape), (ey, y_shape)):
        for letter, extent in zip(letters, shape):
            if letter in size and size[letter] != extent:
                if size[letter] != 1 and extent != 1:
                    return None
                return None  # broadcasting over size-1 dims: leave to torch
            size[letter] = extent
    batch = [c for c in ez if c in sx and c in sy]
    rows = [c for c in ez if c in sx and c not in sy]
    cols = [c for c in ez if c in sy and c not in sx]
    red = [c for c in ex if c in sy and c not in sz]
    x_only = [c for c in ex if c not in sy and c not in sz]
    y_only = [c for c in ey if c not in sx and c not in sz]
    return dict(batch=batch, rows=rows, cols=cols, red=red, x_only=x_only, y_only=y_only,
                size=size, ex=ex, ey=ey, ez=ez)


def _prod(letters, size):
    return math.prod(size[c] for c in letters) if letters else 1


def _activate(z, activation):
    if activation is None:
        return z
    if activation != "silu":
        raise ValueError(f"unsupported activation {activation!r} (supported: 'silu')")
    return gemm.silu(z)


def contract(equation, *operands, activation=None):
    """``torch.einsum(equation, *operands)``, optionally followed by an
    elementwise ``activation`` ("silu"), which the native GEMM applies in its
    epilogue."""
    if len(operands) != 2:
        return _activate(torch.einsum(equation, *operands), activation)
    x, y = operands
    if not gemm.eligible(x, y):
        return _activate(torch.einsum(equation, x, y), activation)
    plan = canonical_gemm(equation, tuple(x.shape), tuple(y.shape))
    if plan is None:
        return _activate(torch.einsum(equation, x, y), activation)
    size = plan["size"]
    ex, ey, ez = plan["ex"], plan["ey"], plan["ez"]
    if plan["x_only"]:
        x = x.sum(dim=[ex.index(c) for c in plan["x_only"]])
        ex = "".join(c for c in ex if c not in plan["x_only"])
    if plan["y_only"]:
        y = y.sum(dim=[ey.index(c) for c in plan["y_only"]])
        ey = "".join(c for c in ey if c not in plan["y_only"])
    batch, rows, cols, red = plan["batch"], plan["rows"], plan["cols"], plan["red"]
    B, M, N, K = (_prod(batch, size), _prod(rows, size), _prod(cols, size), _prod(red, size))
    if K == 0 or M == 0 or N == 0 or B == 0:
        return _activate(torch.einsum(equation, operands[0], operands[1]), activation)
    xv = x.permute([ex.index(c) for c in batch + rows + red]).reshape(B, M, K)
    yv = y.permute([ey.index(c) for c in batch + red + cols]).reshape(B, K, N)
    z = gemm.matmul(xv, yv, activation=activation)
    z = z.reshape([size[c] for c in batch + rows + cols])
    order = batch + rows + cols
    return z.permute([order.index(c) for c in ez])
