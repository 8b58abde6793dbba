"""Functional wrappers over the C ABI: torch tensors in, torch tensors out.

These are the single-launch building blocks used by the reference-compatible
modules (``diffusion_triton``, ``pde_layers``, ``transformers``,
``serving_vllm``, ``sharded``).  They validate shapes, allocate outputs with
torch (the library itself never allocates) and enqueue one kernel on the
current CUDA stream.  Callers handle the identity cases (``steps == 0``,
sequence length < 3) with the reference's aliasing rules before calling here.
"""
from __future__ import annotations

from typing import Optional, Sequence, Union

import torch

from . import _lib

AlphaLike = Union[float, torch.Tensor]


def _require_cuda(t: torch.Tensor, name: str) -> None:
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be on CUDA")


def _alpha_args(alphas: Sequence[AlphaLike], steps: int, device: torch.device):
    """Host floats -> (float array, NULL); device scalars -> (NULL, pointer array)."""
    if len(alphas) != steps:
        raise ValueError(f"expected {steps} alpha values, got {len(alphas)}")
    if all(not isinstance(a, torch.Tensor) for a in alphas):
        return _lib.float_array(alphas), None, 0, []
    tens = []
    for a in alphas:
        if not isinstance(a, torch.Tensor):
            a = torch.tensor([float(a)], dtype=torch.float32, device=device)
        if a.device != device:
            raise ValueError(f"alpha on {a.device}, expected {device}")
        if a.dtype not in (torch.float32, torch.bfloat16, torch.float16):
            a = a.float()
        if a.numel() < 1:
            raise ValueError("alpha tensor is empty")
        a = a.detach()
        if not a.is_contiguous():
            a = a.contiguous()
        tens.append(a)
    code = _lib.dtype_code(tens[0].dtype)
    if any(t.dtype != tens[0].dtype for t in tens):
        tens = [t.float() for t in tens]
        code = 0
    return None, _lib.ptr_array(tens), code, tens  # keep tensors alive for the call


def _mask_args(mask: Optional[torch.Tensor], B: int, L: int, device: torch.device):
    if mask is None:
        return None, 0, 0, 0
    if mask.dim() != 2 or mask.shape[0] != B or mask.shape[1] != L:
        raise ValueError(f"attention_mask must be ({B}, {L}), got {tuple(mask.shape)}")
    if mask.device != device:
        raise ValueError(f"attention_mask on {mask.device}, expected {device}")
    if mask.dtype == torch.bool:
        mask = mask.view(torch.uint8)
    return mask, _lib.mask_code(mask.dtype), mask.stride(0), mask.stride(1)


def _out(out: Optional[torch.Tensor], shape, like: torch.Tensor, contiguous: bool = False) -> torch.Tensor:
    """The caller's output buffer after checking it, or a new one."""
    if out is None:
        return torch.empty(shape, dtype=like.dtype, device=like.device)
    if tuple(out.shape) != tuple(shape) or out.dtype != like.dtype or out.device != like.device:
        raise ValueError(f"out must be {tuple(shape)} {like.dtype} on {like.device}")
    if out.stride(-1) != 1 or (contiguous and not out.is_contiguous()):
        raise ValueError("out must have a contiguous last axis" + (" and be contiguous" if contiguous else ""))
    return out


def _residual_view(residual: torch.Tensor, shape, like: torch.Tensor) -> torch.Tensor:
    if tuple(residual.shape) != tuple(shape) or residual.dtype != like.dtype or residual.device != like.device:
        raise ValueError(f"residual must be {tuple(shape)} {like.dtype} on {like.device}")
    return residual if residual.stride(-1) == 1 else residual.contiguous()


# ---------------------------------------------------------------------------
# [B, D, L]
# ---------------------------------------------------------------------------
def bdl(
    x: torch.Tensor,
    alphas: Sequence[AlphaLike],
    steps: int,
    *,
    causal: bool = False,
    backward: bool = False,
    mask: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
    arith: Optional[str] = None,
) -> torch.Tensor:
    """`steps` fused steps (or their adjoint) on a contiguous [B, D, L] tensor.

    `arith` ("exact" / "contracted", None = the process default) selects the
    forward update's arithmetic for 16-bit tensors (cta_b200.set_arithmetic)."""
    _require_cuda(x, "x")
    if x.dim() != 3:
        raise ValueError("x must have shape (B, D, L)")
    if x.stride(2) != 1 or x.stride(0) != x.shape[1] * x.stride(1):
        x = x.contiguous()
    B, D, L = x.shape
    y = _out(out, x.shape, x, contiguous=True)
    fa, pa, pcode, keep = _alpha_args(alphas, steps, x.device)
    m, mcode, msb, msl = _mask_args(mask, B, L, x.device)
    lib = _lib.load()
    with _lib.on_device(x), _lib.thread_arithmetic(arith):
        rc = lib.cta_diffusion_bdl_ex(
            _lib.ptr(x), _lib.ptr(y), B, D, L, x.stride(1), y.stride(1), _lib.dtype_code(x.dtype), steps,
            int(causal), int(backward), fa, pa, pcode, _lib.ptr(m), mcode, msb, msl, _lib.stream_ptr(x),
        )
    del keep
    _lib.check(rc)
    return y


def bdl_simple(x: torch.Tensor, alpha: float, steps: int, backward: bool = False,
               out: Optional[torch.Tensor] = None, arith: Optional[str] = None) -> torch.Tensor:
    """Reference kernel API path: one host alpha, no mask, non-causal."""
    _require_cuda(x, "x")
    if not x.is_contiguous():
        x = x.contiguous()
    B, D, L = x.shape
    y = _out(out, x.shape, x, contiguous=True)
    lib = _lib.load()
    fn = lib.cta_diffusion_bwd_bdl if backward else lib.cta_diffusion_fwd_bdl
    with _lib.on_device(x), _lib.thread_arithmetic(arith):
        rc = fn(_lib.ptr(x), _lib.ptr(y), B, D, L, L, _lib.dtype_code(x.dtype), steps, float(alpha),
                _lib.stream_ptr(x))
    _lib.check(rc)
    return y


# ---------------------------------------------------------------------------
# [B, L, D]
# ---------------------------------------------------------------------------
def _bld_view(x: torch.Tensor) -> torch.Tensor:
    if x.stride(2) != 1:
        x = x.contiguous()
    return x


def bld_forward(
    x: torch.Tensor,
    alphas: Sequence[AlphaLike],
    steps: int,
    *,
    causal: bool = False,
    mask: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
    residual: Optional[torch.Tensor] = None,
    arith: Optional[str] = None,
) -> torch.Tensor:
    """`steps` fused steps on [B, L, D] (feature axis contiguous), one launch.

    With `residual` (non-causal, host alphas) the same launch returns
    residual + stencil(x), equal bit for bit to the two-pass result.  `arith`
    ("exact" / "contracted", None = the process default) selects the update's
    arithmetic for 16-bit tensors (cta_b200.set_arithmetic)."""
    _require_cuda(x, "x")
    if x.dim() != 3:
        raise ValueError("x must have shape (B, L, D)")
    x = _bld_view(x)
    B, L, D = x.shape
    y = _out(out, (B, L, D), x)
    fa, pa, pcode, keep = _alpha_args(alphas, steps, x.device)
    m, mcode, msb, msl = _mask_args(mask, B, L, x.device)
    lib = _lib.load()
    if residual is not None:
        r = _residual_view(residual, (B, L, D), x)
        if causal or pa is not None:
            raise ValueError("the fused residual add takes the non-causal stencil with host alphas")
        with _lib.on_device(x), _lib.thread_arithmetic(arith):
            rc = lib.cta_diffusion_fwd_bld_residual(
                _lib.ptr(x), _lib.ptr(r), _lib.ptr(y), B, L, D, x.stride(0), x.stride(1), r.stride(0), r.stride(1),
                y.stride(0), y.stride(1), _lib.dtype_code(x.dtype), steps, fa, _lib.ptr(m), mcode, msb, msl,
                _lib.stream_ptr(x),
            )
        del keep
        _lib.check(rc)
        return y
    with _lib.on_device(x), _lib.thread_arithmetic(arith):
        rc = lib.cta_diffusion_fwd_bld(
            _lib.ptr(x), _lib.ptr(y), B, L, D, x.stride(0), x.stride(1), y.stride(0), y.stride(1),
            _lib.dtype_code(x.dtype), steps, int(causal), fa, pa, pcode, _lib.ptr(m), mcode, msb, msl,
            _lib.stream_ptr(x),
        )
    del keep
    _lib.check(rc)
    return y


_WS: "OrderedDict" = None  # (device, stream, tag) -> buffer, most recently used last
_WS_PER_DEVICE = 8


def _workspace(device: torch.device, nbytes: int, tag: str = "dalpha") -> torch.Tensor:
    """Zero-initialised scratch, one per (device, stream, tag), at most
    _WS_PER_DEVICE per device (least recently used dropped first).

    "dalpha": the d(alpha) reductions; their kernels leave the completion
    counters at zero, so the buffer stays reusable without clearing between
    calls on the same stream.  Other users take their own tag, so that nothing
    else ever writes into those counters.  A buffer is only ever used on the
    stream it was allocated on, so dropping it hands its memory back to torch's
    stream-ordered caching allocator without a race against kernels in flight.
    """
    global _WS
    if _WS is None:
        from collections import OrderedDict

        _WS = OrderedDict()
    key = (device, torch.cuda.current_stream(device).cuda_stream, tag)
    buf = _WS.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 4096), dtype=torch.uint8, device=device)
        _WS[key] = buf
        same = [k for k in _WS if k[0] == device]
        for k in same[: max(0, len(same) - _WS_PER_DEVICE)]:
            del _WS[k]
    _WS.move_to_end(key)
    return buf


def bld_backward(
    grad_out: torch.Tensor,
    alphas: Sequence[AlphaLike],
    steps: int,
    *,
    x: Optional[torch.Tensor] = None,
    causal: bool = False,
    mask: Optional[torch.Tensor] = None,
    need_dalpha: bool = False,
    out: Optional[torch.Tensor] = None,
    arith: Optional[str] = None,
):
    """grad_in = A_1^T .. A_S^T grad_out; with need_dalpha also d(alpha_k) (fp32 [steps]).
    `arith` as for bld_forward (16-bit tensors; None = the process default)."""
    _require_cuda(grad_out, "grad_out")
    g = _bld_view(grad_out)
    B, L, D = g.shape
    dx = _out(out, (B, L, D), g)
    fa, pa, pcode, keep = _alpha_args(alphas, steps, g.device)
    m, mcode, msb, msl = _mask_args(mask, B, L, g.device)
    lib = _lib.load()
    dalpha = None
    ws = None
    ws_bytes = 0
    xs = None
    if need_dalpha:
        if x is None:
            raise ValueError("need_dalpha requires the forward input x")
        xs = _bld_view(x)
        if xs.dtype != g.dtype or tuple(xs.shape) != (B, L, D):
            raise ValueError("x must match grad_out in shape and dtype")
        dalpha = torch.empty(steps, dtype=torch.float32, device=g.device)
        ws_bytes = int(lib.cta_diffusion_bwd_bld_workspace_bytes(B, L, D, _lib.dtype_code(g.dtype), steps,
                                                                 int(causal)))
        ws = _workspace(g.device, ws_bytes)
    with _lib.on_device(g), _lib.thread_arithmetic(arith):
        rc = lib.cta_diffusion_bwd_bld(
            _lib.ptr(g), _lib.ptr(dx), _lib.ptr(xs), _lib.ptr(dalpha), _lib.ptr(ws), ws_bytes, B, L, D,
            g.stride(0), g.stride(1), xs.stride(0) if xs is not None else 0, xs.stride(1) if xs is not None else 0,
            dx.stride(0), dx.stride(1), _lib.dtype_code(g.dtype), steps, int(causal), fa, pa, pcode, _lib.ptr(m),
            mcode, msb, msl, _lib.stream_ptr(g),
        )
    del keep
    _lib.check(rc)
    return dx, dalpha


def varlen_forward(
    x: torch.Tensor,
    cu_seqlens: torch.Tensor,
    max_len: int,
    alpha: float,
    steps: int,
    *,
    pad_to_max: bool,
    out: Optional[torch.Tensor] = None,
    residual: Optional[torch.Tensor] = None,
    arith: Optional[str] = None,
) -> torch.Tensor:
    """Packed [T, D] prefill with device cu_seqlens (int32, nseq+1); one launch."""
    _require_cuda(x, "x")
    if x.dim() != 2:
        raise ValueError("x must have shape (T, D)")
    if x.stride(1) != 1:
        x = x.contiguous()
    if cu_seqlens.device != x.device:
        raise ValueError("cu_seqlens must be on the same device as x")
    if cu_seqlens.dtype != torch.int32:
        cu_seqlens = cu_seqlens.to(torch.int32)
    if not cu_seqlens.is_contiguous():
        cu_seqlens = cu_seqlens.contiguous()
    T, D = x.shape
    y = _out(out, (T, D), x, contiguous=True)
    nseq = cu_seqlens.numel() - 1
    lib = _lib.load()
    if residual is not None:
        r = _residual_view(residual, (T, D), x)
        with _lib.on_device(x), _lib.thread_arithmetic(arith):
            rc = lib.cta_diffusion_fwd_varlen_residual(
                _lib.ptr(x), _lib.ptr(r), _lib.ptr(y), T, D, x.stride(0), r.stride(0), y.stride(0),
                _lib.ptr(cu_seqlens), nseq, int(max_len), int(pad_to_max), _lib.dtype_code(x.dtype), steps,
                float(alpha), _lib.stream_ptr(x),
            )
        _lib.check(rc)
        return y
    with _lib.on_device(x), _lib.thread_arithmetic(arith):
        rc = lib.cta_diffusion_fwd_varlen(
            _lib.ptr(x), _lib.ptr(y), T, D, x.stride(0), y.stride(0), _lib.ptr(cu_seqlens), nseq, int(max_len),
            int(pad_to_max), _lib.dtype_code(x.dtype), steps, float(alpha), _lib.stream_ptr(x),
        )
    _lib.check(rc)
    return y


def shard_part(
    x_local: torch.Tensor,
    out: torch.Tensor,
    part: int,
    *,
    pos_offset: int,
    global_len: int,
    alpha: float,
    steps: int,
    causal: bool = False,
    backward: bool = False,
    lo_halo: Optional[torch.Tensor] = None,
    hi_halo: Optional[torch.Tensor] = None,
    stream: Optional[torch.cuda.Stream] = None,
    arith: Optional[str] = None,
) -> None:
    """One launch over a part (interior / lo edge / hi edge) of an L-shard."""
    B, Lloc, D = x_local.shape
    for h in (lo_halo, hi_halo):
        if h is not None and (not h.is_contiguous() or h.shape[0] != B or h.shape[2] != D or h.dtype != x_local.dtype):
            raise ValueError("halo must be a contiguous (B, rows, D) tensor of the shard's dtype")
    lo_rows = lo_halo.shape[1] if lo_halo is not None else 0
    hi_rows = hi_halo.shape[1] if hi_halo is not None else 0
    st = stream if stream is not None else torch.cuda.current_stream(x_local.device)
    lib = _lib.load()
    with _lib.on_device(x_local), _lib.thread_arithmetic(arith):
        rc = lib.cta_diffusion_shard_bld(
            _lib.ptr(x_local), _lib.ptr(out), B, Lloc, D, int(pos_offset), int(global_len), _lib.ptr(lo_halo),
            lo_rows, _lib.ptr(hi_halo), hi_rows, int(part), _lib.dtype_code(x_local.dtype), steps, int(causal),
            int(backward), float(alpha), st.cuda_stream,
        )
    _lib.check(rc)


def shard_part_dalpha(
    g_local: torch.Tensor,
    x_local: torch.Tensor,
    dx_out: torch.Tensor,
    dalpha: torch.Tensor,
    part: int,
    *,
    pos_offset: int,
    global_len: int,
    alphas: Sequence[float],
    steps: int,
    causal: bool = False,
    g_lo: Optional[torch.Tensor] = None,
    g_hi: Optional[torch.Tensor] = None,
    x_lo: Optional[torch.Tensor] = None,
    x_hi: Optional[torch.Tensor] = None,
    stream: Optional[torch.cuda.Stream] = None,
    arith: Optional[str] = None,
) -> None:
    """One launch over a part of an L-shard's backward with d(alpha): writes the
    part's rows of dx_out and ADDS the part's d(alpha) sum to `dalpha` (fp32 [steps])."""
    B, Lloc, D = g_local.shape
    if tuple(x_local.shape) != (B, Lloc, D) or x_local.dtype != g_local.dtype:
        raise ValueError("x_local must match g_local in shape and dtype")
    if dalpha.dtype != torch.float32 or dalpha.numel() < steps or not dalpha.is_contiguous():
        raise ValueError("dalpha must be a contiguous fp32 tensor of at least `steps` entries")
    for h in (g_lo, g_hi, x_lo, x_hi):
        if h is not None and (not h.is_contiguous() or h.shape[0] != B or h.shape[2] != D or h.dtype != g_local.dtype):
            raise ValueError("halo must be a contiguous (B, rows, D) tensor of the shard's dtype")
    rows = [h.shape[1] if h is not None else 0 for h in (g_lo, g_hi, x_lo, x_hi)]
    if len(alphas) != steps:
        raise ValueError("need one alpha per step")
    st = stream if stream is not None else torch.cuda.current_stream(g_local.device)
    lib = _lib.load()
    code = _lib.dtype_code(g_local.dtype)
    ws_bytes = int(lib.cta_diffusion_bwd_bld_workspace_bytes(B, Lloc, D, code, steps, int(causal)))
    with torch.cuda.stream(st):
        ws = _workspace(g_local.device, ws_bytes)
    with _lib.on_device(g_local), _lib.thread_arithmetic(arith):
        rc = lib.cta_diffusion_shard_bld_dalpha(
            _lib.ptr(g_local), _lib.ptr(x_local), _lib.ptr(dx_out), _lib.ptr(dalpha), _lib.ptr(ws), ws_bytes, B, Lloc,
            D, int(pos_offset), int(global_len), _lib.ptr(g_lo), rows[0], _lib.ptr(g_hi), rows[1], _lib.ptr(x_lo),
            rows[2], _lib.ptr(x_hi), rows[3], int(part), code, steps, int(causal),
            _lib.float_array([float(a) for a in alphas]), st.cuda_stream,
        )
    _lib.check(rc)


def pde_step(
    x: torch.Tensor,
    kind: int,
    alpha: torch.Tensor,
    beta: torch.Tensor,
    *,
    causal: bool = False,
    mask: Optional[torch.Tensor] = None,
    grad_out: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
):
    """One advection- / reaction-diffusion step on [B, L, D] (kind _lib.PDE_*).

    Forward (grad_out None): returns y.  Backward: returns (dx, dcoef) with
    dcoef = fp32 [d(alpha), d(beta)].  alpha, beta: the layer's [1] parameters,
    read on the device."""
    _require_cuda(x, "x")
    if x.dim() != 3:
        raise ValueError("x must have shape (B, L, D)")
    x = _bld_view(x)
    B, L, D = x.shape
    coefs = []
    for c in (alpha, beta):
        c = c.detach()
        if c.device != x.device:
            raise ValueError(f"coefficient on {c.device}, expected {x.device}")
        if c.dtype not in (torch.float32, torch.bfloat16, torch.float16):
            c = c.float()
        coefs.append(c.contiguous())
    if coefs[0].dtype != coefs[1].dtype:
        coefs = [c.float() for c in coefs]
    m, mcode, msb, msl = _mask_args(mask, B, L, x.device)
    lib = _lib.load()
    code = _lib.dtype_code(x.dtype)
    y = _out(out, (B, L, D), x)
    g = None
    dcoef = ws = None
    ws_bytes = 0
    if grad_out is not None:
        g = _bld_view(grad_out)
        if tuple(g.shape) != (B, L, D) or g.dtype != x.dtype:
            raise ValueError("grad_out must match x in shape and dtype")
        dcoef = torch.empty(2, dtype=torch.float32, device=x.device)
        ws_bytes = int(lib.cta_pde_step_workspace_bytes(B, L, D))
        ws = _workspace(x.device, ws_bytes, tag="pde_step")
    with _lib.on_device(x):
        rc = lib.cta_pde_step_bld(
            _lib.ptr(x), _lib.ptr(g), _lib.ptr(y), _lib.ptr(dcoef), _lib.ptr(ws), ws_bytes, B, L, D, x.stride(0),
            x.stride(1), g.stride(0) if g is not None else 0, g.stride(1) if g is not None else 0, y.stride(0),
            y.stride(1), code, int(kind), int(causal), int(grad_out is not None), _lib.ptr(coefs[0]),
            _lib.ptr(coefs[1]), _lib.dtype_code(coefs[0].dtype), _lib.ptr(m), mcode, msb, msl, _lib.stream_ptr(x),
        )
    _lib.check(rc)
    return y if grad_out is None else (y, dcoef)


def pde_stack(
    x: torch.Tensor,
    kind: int,
    alphas: Sequence[torch.Tensor],
    betas: Sequence[torch.Tensor],
    *,
    causal: bool = False,
    mask: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Forward of up to 4 consecutive advection- / reaction-diffusion layers of
    one kind (_lib.PDE_*) on [B, L, D] in one launch, fp32 kept between them.
    alphas[k], betas[k]: layer k's [1] parameters, read on the device."""
    _require_cuda(x, "x")
    if x.dim() != 3:
        raise ValueError("x must have shape (B, L, D)")
    steps = len(alphas)
    if steps != len(betas) or not 1 <= steps <= _lib.PDE_STACK_MAX_STEPS:
        raise ValueError(f"need 1..{_lib.PDE_STACK_MAX_STEPS} alpha / beta pairs")
    x = _bld_view(x)
    B, L, D = x.shape
    coefs = []
    for c in list(alphas) + list(betas):
        c = c.detach()
        if c.device != x.device:
            raise ValueError(f"coefficient on {c.device}, expected {x.device}")
        coefs.append(c.float().contiguous() if c.dtype != torch.float32 else c.contiguous())
    m, mcode, msb, msl = _mask_args(mask, B, L, x.device)
    y = _out(out, (B, L, D), x)
    lib = _lib.load()
    with _lib.on_device(x):
        rc = lib.cta_pde_stack_bld(
            _lib.ptr(x), _lib.ptr(y), B, L, D, x.stride(0), x.stride(1), y.stride(0), y.stride(1),
            _lib.dtype_code(x.dtype), int(kind), steps, int(causal), _lib.ptr_array(coefs[:steps]),
            _lib.ptr_array(coefs[steps:]), 0, _lib.ptr(m), mcode, msb, msl, _lib.stream_ptr(x),
        )
    del coefs
    _lib.check(rc)
    return y


def bld_forward_pool(
    x: torch.Tensor, alphas: Sequence[AlphaLike], steps: int, mask: torch.Tensor
) -> torch.Tensor:
    """`steps` fused non-causal steps on [B, L, D] under `mask`, followed by the
    masked mean pool over L, without writing the stepped tensor: [B, D]."""
    _require_cuda(x, "x")
    if x.dim() != 3:
        raise ValueError("x must have shape (B, L, D)")
    x = _bld_view(x)
    B, L, D = x.shape
    fa, pa, pcode, keep = _alpha_args(alphas, steps, x.device)
    m, mcode, msb, msl = _mask_args(mask, B, L, x.device)
    if m is None:
        raise ValueError("the masked pool needs an attention mask")
    lib = _lib.load()
    pooled = torch.empty((B, D), dtype=x.dtype, device=x.device)
    ws_bytes = int(lib.cta_diffusion_fwd_bld_pool_workspace_bytes(B, L, D))
    ws = _workspace(x.device, ws_bytes, tag="pool")
    with _lib.on_device(x):
        rc = lib.cta_diffusion_fwd_bld_pool(
            _lib.ptr(x), _lib.ptr(pooled), _lib.ptr(ws), ws_bytes, B, L, D, x.stride(0), x.stride(1),
            _lib.dtype_code(x.dtype), steps, fa, pa, pcode, _lib.ptr(m), mcode, msb, msl, _lib.stream_ptr(x),
        )
    del keep
    _lib.check(rc)
    return pooled
