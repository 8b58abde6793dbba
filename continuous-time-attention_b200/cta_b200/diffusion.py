"""Diffusion stencil kernel API on [B, D, L] tensors, B200-native.

Drop-in for the public functions of the reference's kernels/diffusion_triton.py:

================================  =============================================
reference (kernels/diffusion_triton.py)   here
================================  =============================================
``diffusion_step_triton``  :812   ``diffusion_step_triton``   (1 launch)
``diffusion_triton``       :817   ``diffusion_triton``        (steps launches,
                                  rounds to the input dtype after every step,
                                  exactly like the reference loop)
``diffusion_triton_fused`` :891   ``diffusion_triton_fused``  (1 launch, fp32
                                  between steps; steps 1..8 instead of
                                  {1, 2, 4, 8}); backward is ONE fused launch
``diffusion_step_triton_backward`` :765  same name (1 launch)
================================  =============================================

Same argument meaning, same aliasing of the identity cases (steps == 0 and
L < 3) and the same exceptions (ValueError for device / rank / steps,
RuntimeError when the native library is unavailable).  Every value the
reference computes in fp32 is computed here with the same rounding sequence,
so fp32 results are bit-identical to the reference's PyTorch path.
"""
from __future__ import annotations

import torch

from . import _lib, ops

__all__ = [
    "diffusion_step_triton",
    "diffusion_triton",
    "diffusion_triton_fused",
    "diffusion_step_triton_backward",
]


def _require_backend() -> None:
    # kernels/diffusion_triton.py:35-40 raises RuntimeError when its backend is missing
    _lib.load()


def _step_forward(x: torch.Tensor, alpha: float = 0.10) -> torch.Tensor:
    """One step (kernels/diffusion_triton.py:732-762)."""
    _require_backend()
    if x.device.type != "cuda":
        raise ValueError("x must be on CUDA")
    if x.ndim != 3:
        raise ValueError("x must have shape (B, D, L)")
    if not x.is_contiguous():
        x = x.contiguous()
    if x.shape[2] < 3:
        return x.clone()
    if x.numel() == 0:
        return torch.empty_like(x)
    return ops.bdl_simple(x, float(alpha), 1)


def diffusion_step_triton_backward(grad_out: torch.Tensor, alpha: float = 0.10) -> torch.Tensor:
    """Adjoint of one step (kernels/diffusion_triton.py:765-794)."""
    _require_backend()
    if grad_out.device.type != "cuda":
        raise ValueError("grad_out must be on CUDA")
    if grad_out.ndim != 3:
        raise ValueError("grad_out must have shape (B, D, L)")
    if grad_out.shape[2] < 3:
        return grad_out
    if not grad_out.is_contiguous():
        grad_out = grad_out.contiguous()
    if grad_out.numel() == 0:
        return torch.empty_like(grad_out)
    return ops.bdl_simple(grad_out, float(alpha), 1, backward=True)


def _fused_backward(grad_out: torch.Tensor, alpha: float, steps: int) -> torch.Tensor:
    if not grad_out.is_contiguous():
        grad_out = grad_out.contiguous()
    if grad_out.numel() == 0:
        return torch.empty_like(grad_out)
    return ops.bdl_simple(grad_out, float(alpha), int(steps), backward=True)


class _DiffusionStep(torch.autograd.Function):
    """kernels/diffusion_triton.py:797-809."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, alpha: float) -> torch.Tensor:
        ctx.alpha = float(alpha)
        ctx.l = x.shape[-1]
        return _step_forward(x, alpha=alpha)

    @staticmethod
    def backward(ctx, grad_out: torch.Tensor):
        if ctx.l < 3:
            return grad_out, None
        return diffusion_step_triton_backward(grad_out, alpha=ctx.alpha), None


def diffusion_step_triton(x: torch.Tensor, alpha: float = 0.10) -> torch.Tensor:
    """Autograd-enabled single diffusion step on CUDA [B, D, L]."""
    return _DiffusionStep.apply(x, float(alpha))


def diffusion_triton(x: torch.Tensor, alpha: float = 0.10, steps: int = 1) -> torch.Tensor:
    """Multi-step diffusion as a loop of single steps (kernels/diffusion_triton.py:817-826).

    Rounds to ``x.dtype`` after every step, like the reference loop; use
    ``diffusion_triton_fused`` for the single-launch fp32-between-steps form.
    """
    y = x
    for _ in range(steps):
        y = diffusion_step_triton(y, alpha=alpha)
    return y


def _fused_forward(x: torch.Tensor, alpha: float = 0.10, steps: int = 1) -> torch.Tensor:
    """kernels/diffusion_triton.py:829-868, one launch for any steps in 1..8."""
    _require_backend()
    if steps < 0:
        raise ValueError(f"steps must be >= 0, got {steps}")
    if steps == 0:
        return x
    if x.device.type != "cuda":
        raise ValueError("x must be on CUDA")
    if x.ndim != 3:
        raise ValueError("x must have shape (B, D, L)")
    if not x.is_contiguous():
        x = x.contiguous()
    if x.shape[2] < 3:
        return x
    if steps > _lib.MAX_STEPS:
        raise ValueError(f"fused kernel supports steps in 1..{_lib.MAX_STEPS}, got {steps}")
    if x.numel() == 0:
        return torch.empty_like(x)
    return ops.bdl_simple(x, float(alpha), int(steps))


class _DiffusionFused(torch.autograd.Function):
    """kernels/diffusion_triton.py:871-888; the backward is one fused launch."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, alpha: float, steps: int) -> torch.Tensor:
        ctx.alpha = float(alpha)
        ctx.steps = int(steps)
        ctx.l = x.shape[-1]
        return _fused_forward(x, alpha=alpha, steps=steps)

    @staticmethod
    def backward(ctx, grad_out: torch.Tensor):
        if ctx.steps == 0 or ctx.l < 3:
            return grad_out, None, None
        return _fused_backward(grad_out, ctx.alpha, ctx.steps), None, None


def diffusion_triton_fused(x: torch.Tensor, alpha: float = 0.10, steps: int = 1) -> torch.Tensor:
    """Multi-step diffusion in ONE launch (kernels/diffusion_triton.py:891-910).

    x: CUDA tensor (B, D, L); non-contiguous input is made contiguous.
    Arithmetic in fp32, rounded to x.dtype once at the end.
    """
    if steps == 0:
        return x
    if x.requires_grad:
        return _DiffusionFused.apply(x, float(alpha), int(steps))
    return _fused_forward(x, alpha=alpha, steps=steps)
