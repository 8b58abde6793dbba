"""CPU oracle for the fused diffusion stencil -- TEST INFRASTRUCTURE ONLY.

A restatement, in plain PyTorch on the CPU, of the reference's own algorithm
for the hot path.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it, and
only as the checker or the timed CPU baseline; the product path
(``cta_b200``) never calls it and has no CPU fallback.

Pinning: ``tests/golden/make_golden.py`` runs the reference itself (imported
from its source tree in the build container) on seeded inputs and commits the
results under ``tests/golden/``; ``tests/test_oracle_golden.py`` checks that
every function below reproduces them bit for bit (forward) or to 1e-6
(gradients).

Every function follows the reference op by op -- separately rounded fp32 ops
in the reference's order -- so its fp32 results are the reference's results.
Citations are to files of the reference project.
"""
from __future__ import annotations

from typing import Optional, Sequence, Union

import torch

Alpha = Union[float, torch.Tensor]


# ---------------------------------------------------------------------------
# the update u + alpha * lap in two arithmetics
# ---------------------------------------------------------------------------
def _update(u: torch.Tensor, a, lap: torch.Tensor, contracted: bool) -> torch.Tensor:
    """u + alpha * lap, fp32.

    contracted=False: the reference's PyTorch ops -- the product rounded to fp32,
    then the sum rounded (src/cta/ops/diffusion.py:52-53).
    contracted=True: the product and the sum rounded ONCE, a fused multiply-add:
    the op order the reference's Triton kernels compile to
    (kernels/diffusion_triton.py:89-90, :252-259; Triton contracts a multiply
    feeding an add into one fma by default).  Emulated in fp64: the product of
    two fp32 values is exact there, the sum rounds to fp64 and then to fp32,
    which equals the single fp32 rounding except in double-rounding ties of
    probability about 2**-29 per element (absorbed by any 16-bit output rounding).
    """
    if not contracted:
        return u + a * lap
    a64 = a.double() if isinstance(a, torch.Tensor) else float(torch.tensor(float(a), dtype=torch.float32))
    return (u.double() + a64 * lap.double()).to(torch.float32)


# ---------------------------------------------------------------------------
# core stencil along the last axis, fp32
# ---------------------------------------------------------------------------
def _lap_last(u: torch.Tensor) -> torch.Tensor:
    # src/cta/ops/diffusion.py:48-52 : right - 2.0 * mid + left
    return u[..., 2:] - 2.0 * u[..., 1:-1] + u[..., :-2]


def step_bdl(x_bdl: torch.Tensor, *, alpha: float, out_dtype: Optional[torch.dtype] = None,
             contracted: bool = False) -> torch.Tensor:
    """One non-causal step on [B, D, L], copy boundary (src/cta/ops/diffusion.py:17-56)."""
    if x_bdl.ndim != 3:
        raise ValueError(f"expected x_bdl.ndim == 3, got {x_bdl.ndim}")
    out_dtype = x_bdl.dtype if out_dtype is None else out_dtype
    if x_bdl.shape[2] < 3:
        return x_bdl.to(dtype=out_dtype)
    u = x_bdl.to(dtype=torch.float32)
    mid = u[:, :, 1:-1]
    new_mid = _update(mid, float(alpha), _lap_last(u), contracted)
    return torch.cat([u[:, :, :1], new_mid, u[:, :, -1:]], dim=2).to(dtype=out_dtype)


def steps_bdl(x_bdl: torch.Tensor, *, alpha: float, steps: int, out_dtype: Optional[torch.dtype] = None,
              contracted: bool = False):
    """`steps` steps, fp32 in between, rounded once (src/cta/ops/diffusion.py:59-77)."""
    if steps < 0:
        raise ValueError(f"expected steps >= 0, got {steps}")
    out_dtype = x_bdl.dtype if out_dtype is None else out_dtype
    if steps == 0:
        return x_bdl.to(dtype=out_dtype)
    u = x_bdl
    for _ in range(steps):
        u = step_bdl(u, alpha=alpha, out_dtype=torch.float32, contracted=contracted)
    return u.to(dtype=out_dtype)


def steps_bld(x_bld: torch.Tensor, *, alpha: float, steps: int, contracted: bool = False) -> torch.Tensor:
    """[B, L, D] form, fp32 in between (src/cta/serving_vllm.py:29-46)."""
    if steps <= 0:
        return x_bld
    if x_bld.ndim != 3:
        raise ValueError(f"expected x_bld.ndim == 3, got {x_bld.ndim}")
    if x_bld.shape[1] < 3:
        return x_bld
    u = x_bld.to(dtype=torch.float32)
    for _ in range(steps):
        lap = u[:, 2:, :] - 2.0 * u[:, 1:-1, :] + u[:, :-2, :]
        u = torch.cat([u[:, :1, :], _update(u[:, 1:-1, :], float(alpha), lap, contracted), u[:, -1:, :]], dim=1)
    return u.to(dtype=x_bld.dtype)


# ---------------------------------------------------------------------------
# PDE layer (diffusion), src/models/pde_layers.py
# ---------------------------------------------------------------------------
def _alpha_f32(alpha: Alpha) -> Union[float, torch.Tensor]:
    if isinstance(alpha, torch.Tensor):
        return alpha.to(dtype=torch.float32)  # pde_layers.py:219
    return float(alpha)


def _valid3(mask: torch.Tensor, n_out: int) -> torch.Tensor:
    # pde_layers.py:39-64 -- all three stencil rows valid, last n_out windows, as (B, 1, n_out)
    full = mask[:, :-2] * mask[:, 1:-1] * mask[:, 2:]
    return full[:, -n_out:].unsqueeze(1).bool()


def layer_step(
    x: torch.Tensor,
    alpha: Alpha,
    *,
    layout: str = "bdl",
    causal: bool = False,
    attention_mask: Optional[torch.Tensor] = None,
    keep_fp32: bool = False,
    contracted: bool = False,
) -> torch.Tensor:
    """One DiffusionPDELayer step (src/models/pde_layers.py:113-188, :218-219).

    keep_fp32=True returns the fp32 result instead of casting back to x.dtype
    (the fused stack keeps fp32 between steps).
    """
    seq_dim = 2 if layout == "bdl" else 1
    if x.size(seq_dim) < 3:
        return x
    u = x.to(dtype=torch.float32)
    if layout == "bld":
        u = u.transpose(1, 2)
    lap = u[:, :, 2:] - 2.0 * u[:, :, 1:-1] + u[:, :, :-2]
    a = _alpha_f32(alpha)
    if causal:
        interior = u[:, :, 2:]
        upd = _update(interior, a, lap, contracted)
        if attention_mask is not None:
            upd = torch.where(_valid3(attention_mask, upd.size(2)), upd, interior)
        y = torch.cat([u[:, :, :2], upd], dim=2)
    else:
        interior = u[:, :, 1:-1]
        upd = _update(interior, a, lap, contracted)
        if attention_mask is not None:
            upd = torch.where(_valid3(attention_mask, upd.size(2)), upd, interior)
        y = torch.cat([u[:, :, :1], upd, u[:, :, -1:]], dim=2)
    if attention_mask is not None:
        m = attention_mask.bool().to(dtype=y.dtype).unsqueeze(1)  # pde_layers.py:26-36
        y = y * m + u * (1 - m)
    if layout == "bld":
        y = y.transpose(1, 2)
    return y if keep_fp32 else y.to(dtype=x.dtype)


def pde_layer_step(
    x: torch.Tensor,
    kind: str,
    alpha: Alpha,
    beta: Alpha,
    *,
    layout: str = "bdl",
    causal: bool = False,
    attention_mask: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """One AdvectionDiffusionPDELayer (kind "advection") or ReactionDiffusionPDELayer
    (kind "reaction") step: the base forward of src/models/pde_layers.py:113-188 with
    the updates of :309-318 and :276-281."""
    seq_dim = 2 if layout == "bdl" else 1
    if x.size(seq_dim) < 3:
        return x
    u = x.to(dtype=torch.float32)
    if layout == "bld":
        u = u.transpose(1, 2)
    lap = u[:, :, 2:] - 2.0 * u[:, :, 1:-1] + u[:, :, :-2]
    a, b = _alpha_f32(alpha), _alpha_f32(beta)
    interior = u[:, :, 2:] if causal else u[:, :, 1:-1]
    diffusion = a * lap
    if kind == "advection":
        gradient = (u[:, :, 2:] - u[:, :, 1:-1]) if causal else (u[:, :, 2:] - u[:, :, :-2]) / 2.0
        dx = diffusion + b * gradient
    elif kind == "reaction":
        dx = diffusion + b * interior * (1.0 - torch.sigmoid(interior))
    else:
        raise ValueError(f"unknown kind {kind!r}")
    upd = interior + dx
    if attention_mask is not None:
        upd = torch.where(_valid3(attention_mask, upd.size(2)), upd, interior)
    if causal:
        y = torch.cat([u[:, :, :2], upd], dim=2)
    else:
        y = torch.cat([u[:, :, :1], upd, u[:, :, -1:]], dim=2)
    if attention_mask is not None:
        m = attention_mask.bool().to(dtype=y.dtype).unsqueeze(1)
        y = y * m + u * (1 - m)
    if layout == "bld":
        y = y.transpose(1, 2)
    return y.to(dtype=x.dtype)


def layer_chain(
    x: torch.Tensor,
    alphas: Sequence[Alpha],
    *,
    layout: str = "bdl",
    causal: bool = False,
    attention_mask: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Consecutive layers, each rounding to x.dtype (transformers.py:127-133 loop)."""
    y = x
    for a in alphas:
        y = layer_step(y, a, layout=layout, causal=causal, attention_mask=attention_mask)
    return y


def fused_stack(
    x: torch.Tensor,
    alphas: Sequence[Alpha],
    *,
    layout: str = "bdl",
    causal: bool = False,
    attention_mask: Optional[torch.Tensor] = None,
    contracted: bool = False,
) -> torch.Tensor:
    """The same layers with fp32 kept between them and one final rounding."""
    seq_dim = 2 if layout == "bdl" else 1
    if x.size(seq_dim) < 3 or len(alphas) == 0:
        return x
    y = x.to(torch.float32)
    for a in alphas:
        y = layer_step(y, a, layout=layout, causal=causal, attention_mask=attention_mask, keep_fp32=True,
                       contracted=contracted)
    return y.to(dtype=x.dtype)


# ---------------------------------------------------------------------------
# adjoint of one step (kernels/diffusion_triton.py:96-133)
# ---------------------------------------------------------------------------
def step_adjoint_bdl(g: torch.Tensor, *, alpha: float) -> torch.Tensor:
    """dx for one non-causal step: interior (1-2a) dy + a (dy[i-1][i-1>=1] + dy[i+1][i+1<=L-2]),
    ends dy[0] + a dy[1] and dy[L-1] + a dy[L-2]; L < 3 returns g."""
    L = g.shape[-1]
    if L < 3:
        return g
    dy = g.to(torch.float32)
    a = float(alpha)
    prev = torch.zeros_like(dy)
    nxt = torch.zeros_like(dy)
    prev[..., 2:] = dy[..., 1:-1]   # dy[i-1] where i-1 >= 1
    nxt[..., :-2] = dy[..., 1:-1]   # dy[i+1] where i+1 <= L-2
    dx = (1.0 - 2.0 * a) * dy + a * (prev + nxt)
    dx[..., 0] = dy[..., 0] + a * dy[..., 1]
    dx[..., -1] = dy[..., -1] + a * dy[..., -2]
    return dx.to(g.dtype)


def grads(fn, x: torch.Tensor, grad_out: torch.Tensor, params: Sequence[torch.Tensor] = ()):
    """(dx, [dparam...]) of sum(fn(x) * grad_out) by autograd through the oracle."""
    xr = x.detach().clone().requires_grad_(True)
    ps = [p.detach().clone().requires_grad_(True) for p in params]
    y = fn(xr, *ps)
    (y.float() * grad_out.float()).sum().backward()
    return xr.grad.detach(), [p.grad.detach() for p in ps]


# ---------------------------------------------------------------------------
# packed variable-length prefill
# ---------------------------------------------------------------------------
def mixer_packed(x_flat: torch.Tensor, qsl: Sequence[int], max_len: int, *, alpha: float, steps: int,
                 contracted: bool = False):
    """Reference packed path: zero-pad every request to max_len, run the [B, L, D]
    stencil, unpack (src/cta/serving_vllm.py:72-111, :292-303)."""
    qsl = [int(v) for v in qsl]
    if max_len < 3 or steps <= 0:
        return x_flat.clone()
    R = len(qsl) - 1
    padded = torch.zeros((R, max_len, x_flat.shape[-1]), dtype=x_flat.dtype)
    for i in range(R):
        s, e = qsl[i], qsl[i + 1]
        if e > s:
            padded[i, : e - s] = x_flat[s:e]
    y = steps_bld(padded, alpha=alpha, steps=steps, contracted=contracted)
    out = torch.empty_like(x_flat)
    for i in range(R):
        s, e = qsl[i], qsl[i + 1]
        if e > s:
            out[s:e] = y[i, : e - s]
    return out


def varlen_per_sequence(x_flat: torch.Tensor, qsl: Sequence[int], *, alpha: float, steps: int,
                        contracted: bool = False):
    """Every sequence refined on its own, with its own copy boundary."""
    qsl = [int(v) for v in qsl]
    out = x_flat.clone()
    for i in range(len(qsl) - 1):
        s, e = qsl[i], qsl[i + 1]
        if e > s:
            out[s:e] = steps_bld(x_flat[s:e].unsqueeze(0), alpha=alpha, steps=steps, contracted=contracted)[0]
    return out


# ---------------------------------------------------------------------------
# L-sharded view: output rows [a, b) need input rows [a - h, b + h) only
# ---------------------------------------------------------------------------
def window_bld(
    x_window: torch.Tensor, *, win_start: int, global_len: int, out_start: int, out_stop: int, alpha: float,
    steps: int, contracted: bool = False,
) -> torch.Tensor:
    """Rows [out_start, out_stop) of steps_bld over a global sequence, given only the rows
    x_window = global rows [win_start, win_start + len) (which must cover the halo)."""
    n = x_window.shape[1]
    u = x_window.to(torch.float32)
    pos = torch.arange(win_start, win_start + n)
    fixed = ((pos <= 0) | (pos >= global_len - 1)).view(1, n, 1)
    for _ in range(steps):
        lap = u[:, 2:, :] - 2.0 * u[:, 1:-1, :] + u[:, :-2, :]
        mid = _update(u[:, 1:-1, :], float(alpha), lap, contracted)
        mid = torch.where(fixed[:, 1:-1, :], u[:, 1:-1, :], mid)
        u = torch.cat([u[:, :1, :], mid, u[:, -1:, :]], dim=1)
    return u[:, out_start - win_start : out_stop - win_start, :].to(x_window.dtype)


def window_bld_grads(
    g_window: torch.Tensor, x_window: torch.Tensor, *, win_start: int, global_len: int, out_start: int,
    out_stop: int, alphas: Sequence[float], causal: bool = False,
):
    """(dx rows [out_start, out_stop), d(alpha_k) summed over those rows only) of
    the fused stack of layers (src/models/pde_layers.py:113-188, :218-219, fp32
    between steps, no mask) over a global sequence of global_len rows, given only
    global rows [win_start, win_start + n) of the forward input and of the output
    gradient.  The window must reach `steps` rows beyond the output rows on each
    side (2*steps before them and 2*steps after them for the causal stencil);
    rows outside it read as zero and cannot reach the output rows.  d(alpha) is
    taken per row through a per-row copy of each alpha, so that a shard sums
    only its own rows."""
    n = x_window.shape[1]
    pos = torch.arange(win_start, win_start + n)
    upd = ((pos >= 2) & (pos <= global_len - 1)) if causal else ((pos >= 1) & (pos <= global_len - 2))
    upd = upd.view(1, n, 1)
    xr = x_window.to(torch.float32).detach().clone().requires_grad_(True)
    per_row = [torch.full((1, n, 1), float(a)).requires_grad_(True) for a in alphas]
    u = xr
    for a in per_row:
        z = torch.zeros_like(u[:, :1])
        up = torch.cat([z, z, u], dim=1) if causal else torch.cat([z, u, z], dim=1)
        # pde_layers.py:143-175 : (x[i+1] - 2x[i]) + x[i-1], causal (x[i] - 2x[i-1]) + x[i-2]
        lap = up[:, 2:] - 2.0 * up[:, 1:-1] + up[:, :-2]
        u = torch.where(upd, u + a * lap, u)
    (u * g_window.to(torch.float32)).sum().backward()
    o0, o1 = out_start - win_start, out_stop - win_start
    dalpha = torch.stack([a.grad[:, o0:o1].double().sum() for a in per_row])
    return xr.grad[:, o0:o1].detach(), dalpha
