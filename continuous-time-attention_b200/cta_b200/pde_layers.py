"""PDE refinement layers backed by the fused sm_100a stencil kernels.

Drop-in for the diffusion family of the reference's src/models/pde_layers.py:

* ``DiffusionPDELayer(hidden_size, alpha_init=0.10, layout="bdl", causal=False)``
  -- one refinement step, ``forward(x, attention_mask=None)``; same parameter
  (``alpha``, shape [1]), same layouts, causal stencil and mask rule
  (pde_layers.py:39-64,113-188,195-219), one kernel launch forward and one
  backward (which also returns d(alpha)).
* ``WavePDELayer`` -- the reference's wave layer updates by alpha**2 * lap
  (pde_layers.py:244-246), i.e. a diffusion step with coefficient alpha**2.
* ``create_pde_layer`` -- the reference factory (pde_layers.py:325-357).
* ``diffusion_pde_stack(x, layers, attention_mask)`` -- runs a list of
  consecutive layers (each with its own alpha) as ONE fused launch, keeping
  fp32 between the layers; the reference applies the layers one by one and
  rounds to the input dtype after each (identical in fp32; within 2e-2 in
  bf16).

* ``AdvectionDiffusionPDELayer`` / ``ReactionDiffusionPDELayer`` -- the
  reference's other two layers (pde_layers.py:249-318, parameters ``alpha``
  and ``beta``): one launch per step forward and one backward (dx, d(alpha),
  d(beta)), as the reference runs them layer by layer.

Arithmetic follows the reference op by op (fp32, no fused multiply-add), so a
single fp32 or bf16 diffusion, wave or advection layer step is bit-identical to
the reference layer; the reaction layer's sigmoid uses the fast intrinsics
``__expf`` and ``__fdividef``, so it matches to fp32 rounding rather than bit
for bit.
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch
import torch.nn as nn

from . import _lib, ops

__all__ = [
    "DiffusionPDELayer",
    "WavePDELayer",
    "create_pde_layer",
    "diffusion_pde_stack",
    "diffusion_stack_function",
    "diffusion_stack_pool",
    "pde_stack_forward",
]


class _StackBLD(torch.autograd.Function):
    """Fused forward/backward of `len(alphas)` layers on [B, L, D]."""

    @staticmethod
    def forward(ctx, x, mask, causal, *alphas):
        steps = len(alphas)
        y = ops.bld_forward(x, list(alphas), steps, causal=causal, mask=mask, arith="exact")
        ctx.causal = causal
        ctx.steps = steps
        ctx.save_for_backward(x, mask, *alphas)
        return y

    @staticmethod
    def backward(ctx, g):
        x, mask, *alphas = ctx.saved_tensors
        need_da = any(ctx.needs_input_grad[3:])
        dx, da = ops.bld_backward(g, alphas, ctx.steps, x=x, causal=ctx.causal, mask=mask, need_dalpha=need_da)
        dalphas = []
        for k, a in enumerate(alphas):
            if ctx.needs_input_grad[3 + k]:
                dalphas.append(da[k : k + 1].reshape(a.shape).to(a.dtype))
            else:
                dalphas.append(None)
        return (dx if ctx.needs_input_grad[0] else None), None, None, *dalphas


class _StackBDL(torch.autograd.Function):
    """Fused forward/backward of `len(alphas)` layers on [B, D, L].

    The backward uses the [B, D, L] adjoint kernel; when d(alpha) is needed the
    gradient and input are viewed in [B, L, D] order and sent through the
    [B, L, D] adjoint kernel, which carries the d(alpha) reduction.
    """

    @staticmethod
    def forward(ctx, x, mask, causal, *alphas):
        steps = len(alphas)
        y = ops.bdl(x, list(alphas), steps, causal=causal, mask=mask, arith="exact")
        ctx.causal = causal
        ctx.steps = steps
        ctx.save_for_backward(x, mask, *alphas)
        return y

    @staticmethod
    def backward(ctx, g):
        x, mask, *alphas = ctx.saved_tensors
        need_da = any(ctx.needs_input_grad[3:])
        if need_da:
            dx_bld, da = ops.bld_backward(
                g.transpose(1, 2).contiguous(), alphas, ctx.steps, x=x.transpose(1, 2).contiguous(),
                causal=ctx.causal, mask=mask, need_dalpha=True,
            )
            dx = dx_bld.transpose(1, 2).contiguous()
        else:
            dx = ops.bdl(g, alphas, ctx.steps, causal=ctx.causal, mask=mask, backward=True)
            da = None
        dalphas = []
        for k, a in enumerate(alphas):
            if ctx.needs_input_grad[3 + k]:
                dalphas.append(da[k : k + 1].reshape(a.shape).to(a.dtype))
            else:
                dalphas.append(None)
        return (dx if ctx.needs_input_grad[0] else None), None, None, *dalphas


class _StackPoolBLD(torch.autograd.Function):
    """The last refinement of the classifier and its masked mean pool
    (src/models/transformers.py:120-139) in one forward pass over [B, L, D]."""

    @staticmethod
    def forward(ctx, x, mask, *alphas):
        steps = len(alphas)
        pooled = ops.bld_forward_pool(x, list(alphas), steps, mask)
        ctx.steps = steps
        ctx.save_for_backward(x, mask, *alphas)
        return pooled

    @staticmethod
    def backward(ctx, gp):
        x, mask, *alphas = ctx.saved_tensors
        # the pool's gradient, in x's dtype as the reference's autograd forms it:
        # d(sum) = gp / count, then d(y) = d(sum) * mask
        count = torch.clamp(mask.sum(dim=1, keepdim=True), min=1)
        g = ((gp.to(x.dtype) / count).unsqueeze(1) * mask.unsqueeze(-1)).to(x.dtype)
        need_da = any(ctx.needs_input_grad[2:])
        dx, da = ops.bld_backward(g, alphas, ctx.steps, x=x, causal=False, mask=mask, need_dalpha=need_da)
        dalphas = [da[k : k + 1].reshape(a.shape).to(a.dtype) if ctx.needs_input_grad[2 + k] else None
                   for k, a in enumerate(alphas)]
        return (dx if ctx.needs_input_grad[0] else None), None, *dalphas


def diffusion_stack_pool(x: torch.Tensor, layers: Sequence[nn.Module], attention_mask: torch.Tensor) -> torch.Tensor:
    """``diffusion_pde_stack`` on [B, L, D] followed by the classifier's masked mean
    pool, with the last up-to-8 steps and the pool fused into one pass (the
    stepped tensor of those steps is never written).  Returns [B, D]."""
    layers = list(layers)
    mask = attention_mask.to(x.device) if attention_mask.device != x.device else attention_mask
    alphas = [l.effective_alpha() for l in layers]
    head = len(alphas) - ((len(alphas) - 1) % _lib.MAX_STEPS + 1)
    if head > 0:
        x = diffusion_stack_function(x, alphas[:head], layout="bld", causal=False, attention_mask=mask)
    return _StackPoolBLD.apply(x, mask, *alphas[head:])


def diffusion_stack_function(
    x: torch.Tensor,
    alphas: Sequence[torch.Tensor],
    *,
    layout: str = "bld",
    causal: bool = False,
    attention_mask: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Apply len(alphas) diffusion steps (alpha_k a device scalar each) fused.

    Groups of up to 8 steps run per launch; fp32 is kept within a group.
    """
    if layout not in {"bdl", "bld"}:
        raise ValueError("layout must be 'bdl' or 'bld'")
    seq_dim = 2 if layout == "bdl" else 1
    if x.dim() != 3:
        raise ValueError(f"expected a 3-D input, got {x.dim()}-D")
    if x.size(seq_dim) < 3 or len(alphas) == 0:
        return x
    if x.device.type != "cuda":
        raise ValueError("x must be on CUDA (the stencil runs only on the sm_100a kernels)")
    fn = _StackBDL if layout == "bdl" else _StackBLD
    mask = attention_mask
    if mask is not None and mask.device != x.device:
        mask = mask.to(x.device)
    y = x
    for i in range(0, len(alphas), _lib.MAX_STEPS):
        y = fn.apply(y, mask, bool(causal), *alphas[i : i + _lib.MAX_STEPS])
    return y


class _DiffusionFamilyLayer(nn.Module):
    """Shared layout/causal handling (src/models/pde_layers.py:71-88)."""

    def __init__(self, hidden_size: int, layout: str = "bdl", causal: bool = False):
        super().__init__()
        if layout not in {"bdl", "bld"}:
            raise ValueError("layout must be 'bdl' or 'bld'")
        self.layout = layout
        self.causal = causal

    def effective_alpha(self) -> torch.Tensor:
        """The coefficient multiplying the Laplacian, as an fp32 [1] tensor."""
        raise NotImplementedError

    def forward(self, x: torch.Tensor, attention_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One refinement step (src/models/pde_layers.py:113-188)."""
        return diffusion_stack_function(
            x, [self.effective_alpha()], layout=self.layout, causal=self.causal, attention_mask=attention_mask
        )


class DiffusionPDELayer(_DiffusionFamilyLayer):
    """Diffusion PDE ``du/dt = alpha * d2u/dx2`` (src/models/pde_layers.py:195-219)."""

    def __init__(self, hidden_size: int, alpha_init: float = 0.10, layout: str = "bdl", causal: bool = False):
        super().__init__(hidden_size, layout=layout, causal=causal)
        self.alpha = nn.Parameter(torch.tensor([alpha_init]))

    def effective_alpha(self) -> torch.Tensor:
        # pde_layers.py:219 multiplies by alpha.to(float32); the kernel reads
        # the parameter as stored and widens it to fp32 the same way
        return self.alpha


class WavePDELayer(_DiffusionFamilyLayer):
    """Wave PDE, reference update ``alpha**2 * lap`` (src/models/pde_layers.py:222-246)."""

    def __init__(self, hidden_size: int, alpha_init: float = 0.15, layout: str = "bdl", causal: bool = False):
        super().__init__(hidden_size, layout=layout, causal=causal)
        self.alpha = nn.Parameter(torch.tensor([alpha_init]))

    def effective_alpha(self) -> torch.Tensor:
        return self.alpha.to(dtype=torch.float32) ** 2


class _PDEStep(torch.autograd.Function):
    """One advection- / reaction-diffusion step on [B, L, D]: forward and
    backward are one launch each (the backward needs x: reaction is nonlinear)."""

    @staticmethod
    def forward(ctx, x, mask, kind, causal, alpha, beta):
        y = ops.pde_step(x, kind, alpha, beta, causal=causal, mask=mask)
        ctx.save_for_backward(x, alpha, beta)
        ctx.mask, ctx.kind, ctx.causal = mask, kind, causal
        return y

    @staticmethod
    def backward(ctx, g):
        x, alpha, beta = ctx.saved_tensors
        dx, dcoef = ops.pde_step(x, ctx.kind, alpha, beta, causal=ctx.causal, mask=ctx.mask,
                                 grad_out=g.to(x.dtype).contiguous())
        da = dcoef[0:1].to(alpha.dtype).view_as(alpha) if ctx.needs_input_grad[4] else None
        db = dcoef[1:2].to(beta.dtype).view_as(beta) if ctx.needs_input_grad[5] else None
        return dx, None, None, None, da, db


class _TwoCoefficientLayer(nn.Module):
    """Layout/causal handling of the reference base layer (pde_layers.py:71-188)
    for the layers with an extra ``beta`` term."""

    KIND = -1

    def __init__(self, hidden_size: int, alpha_init: float, beta_init: float, layout: str = "bdl",
                 causal: bool = False):
        super().__init__()
        if layout not in {"bdl", "bld"}:
            raise ValueError("layout must be 'bdl' or 'bld'")
        self.layout = layout
        self.causal = causal
        self.alpha = nn.Parameter(torch.tensor([alpha_init]))
        self.beta = nn.Parameter(torch.tensor([beta_init]))

    def forward(self, x: torch.Tensor, attention_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One refinement step (src/models/pde_layers.py:113-188)."""
        seq_dim = 2 if self.layout == "bdl" else 1
        if x.size(seq_dim) < 3:
            return x
        if x.device.type != "cuda":
            raise ValueError("x must be on CUDA")
        mask = attention_mask
        if mask is not None:
            if mask.device != x.device:
                mask = mask.to(x.device)
            if mask.dtype == torch.bool:
                mask = mask.to(torch.uint8)
        xb = x.transpose(1, 2) if self.layout == "bdl" else x
        y = _PDEStep.apply(xb.contiguous(), mask, self.KIND, bool(self.causal), self.alpha, self.beta)
        return y.transpose(1, 2) if self.layout == "bdl" else y


class ReactionDiffusionPDELayer(_TwoCoefficientLayer):
    """Reaction-diffusion ``du/dt = alpha*lap + beta*u*(1 - sigmoid(u))``
    (src/models/pde_layers.py:249-281)."""

    KIND = _lib.PDE_REACTION

    def __init__(self, hidden_size: int, alpha_init: float = 0.10, beta_init: float = 0.02, layout: str = "bdl",
                 causal: bool = False):
        super().__init__(hidden_size, alpha_init, beta_init, layout=layout, causal=causal)


class AdvectionDiffusionPDELayer(_TwoCoefficientLayer):
    """Advection-diffusion ``du/dt = alpha*lap + beta*du/dx`` with a central
    (causal: backward) difference (src/models/pde_layers.py:284-318)."""

    KIND = _lib.PDE_ADVECTION

    def __init__(self, hidden_size: int, alpha_init: float = 0.10, beta_init: float = 0.03, layout: str = "bdl",
                 causal: bool = False):
        super().__init__(hidden_size, alpha_init, beta_init, layout=layout, causal=causal)


def pde_stack_forward(
    x: torch.Tensor,
    layers: Sequence[nn.Module],
    attention_mask: Optional[torch.Tensor] = None,
    layout: Optional[str] = None,
) -> torch.Tensor:
    """Inference forward of consecutive advection- or reaction-diffusion layers
    (one kind, one causality): one launch per 4 layers instead of one per layer,
    fp32 kept between all layers (identical to the layer chain in fp32 rounded
    once; within one rounding per layer of the 16-bit layer chain).  ``layout`` is x's
    layout (default: the layers'); the kernel runs on [B, L, D].  No autograd
    graph is recorded: training takes the per-layer path, whose backward needs
    every layer's input."""
    layers = list(layers)
    if not layers:
        return x
    kind, causal = layers[0].KIND, layers[0].causal
    for l in layers:
        if not isinstance(l, _TwoCoefficientLayer) or l.KIND != kind or l.causal != causal:
            raise ValueError("a fused stack needs advection- or reaction-diffusion layers of one kind and causality")
    layout = layers[0].layout if layout is None else layout
    seq_dim = 2 if layout == "bdl" else 1
    if x.size(seq_dim) < 3:
        return x
    if x.device.type != "cuda":
        raise ValueError("x must be on CUDA")
    mask = attention_mask
    if mask is not None:
        if mask.device != x.device:
            mask = mask.to(x.device)
        if mask.dtype == torch.bool:
            mask = mask.to(torch.uint8)
    y = x.transpose(1, 2) if layout == "bdl" else x
    n = _lib.PDE_STACK_MAX_STEPS
    # more layers than one launch holds: 16-bit input runs the launches in fp32
    # and is rounded once at the end, so fp32 is kept between every two layers
    widen = len(layers) > n and y.dtype != torch.float32
    with torch.no_grad():
        if widen:
            y = y.float()
        for i in range(0, len(layers), n):
            chunk = layers[i : i + n]
            y = ops.pde_stack(y.contiguous(), kind, [l.alpha for l in chunk], [l.beta for l in chunk], causal=causal,
                              mask=mask)
        if widen:
            y = y.to(x.dtype)
    return y.transpose(1, 2).contiguous() if layout == "bdl" else y


_PDE_REGISTRY = {
    "diffusion": DiffusionPDELayer,
    "wave": WavePDELayer,
    "reaction-diffusion": ReactionDiffusionPDELayer,
    "advection-diffusion": AdvectionDiffusionPDELayer,
}


def create_pde_layer(pde_type: str, hidden_size: int, causal: bool = False, **kwargs) -> nn.Module:
    """Factory with the reference's signature (src/models/pde_layers.py:333-357)."""
    if pde_type not in _PDE_REGISTRY:
        raise ValueError(f"Unknown PDE type: {pde_type}. Available types: {list(_PDE_REGISTRY.keys())}")
    kwargs["causal"] = causal
    return _PDE_REGISTRY[pde_type](hidden_size, **kwargs)


def diffusion_pde_stack(
    x: torch.Tensor, layers: Sequence[nn.Module], attention_mask: Optional[torch.Tensor] = None
) -> torch.Tensor:
    """Run consecutive diffusion-family layers as one fused launch.

    Equivalent to ``for l in layers: x = l(x, attention_mask=attention_mask)``
    except that fp32 is kept between the layers.  All layers must share layout
    and causality.
    """
    layers = list(layers)
    if not layers:
        return x
    layout, causal = layers[0].layout, layers[0].causal
    for l in layers:
        if not isinstance(l, _DiffusionFamilyLayer):
            raise TypeError(f"{type(l).__name__} is not a diffusion-family layer")
        if l.layout != layout or l.causal != causal:
            raise ValueError("all layers of a fused stack must share layout and causality")
    return diffusion_stack_function(
        x, [l.effective_alpha() for l in layers], layout=layout, causal=causal, attention_mask=attention_mask
    )
