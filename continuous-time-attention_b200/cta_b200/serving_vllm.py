"""CTA post-attention mixer for vLLM, served by the fused sm_100a kernels.

Drop-in for src/cta/serving_vllm.py of the reference: ``CtaConfig`` (same
fields, plus ``varlen_mode`` and ``fuse_any_steps``) and
``CtaPostAttnMixer(config).forward(x, *, attn_metadata=None, is_prefill=None)``
with the same gating (prefill inference :49-61, step policies :177-189).

What changes:
  * [B, L, D] inputs run the [B, L, D] kernel directly -- no BLD<->BDL
    transposes or staging buffers (:234-266);
  * packed 2-D inputs ([T, H] + ``query_start_loc``) run ONE varlen launch that
    reads the offsets on the device: no host sync, no pad / unpack copies and no
    Python loop over requests (:72-111, :275-303).  ``varlen_mode="reference"``
    (default) reproduces the reference's zero-padding-to-``max_query_len`` rule
    exactly; ``"sequence"`` gives every sequence its own copy boundary;
  * every step count 1..8 is fused (the reference fuses only {1, 2, 4, 8} and
    loops single steps, rounding each, otherwise); ``fuse_any_steps=False``
    restores the reference's per-step rounding for the other counts.
The kernels are the only compute path: ``use_triton`` is kept for config
compatibility and a CPU tensor raises ``ValueError``.
"""
from __future__ import annotations

import math
from contextlib import nullcontext
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn

from . import _lib, ops
from .diffusion import diffusion_triton

try:
    from torch.profiler import record_function
except Exception:  # noqa: BLE001

    def record_function(_name: str):  # type: ignore
        return nullcontext()


__all__ = ["CtaConfig", "CtaPostAttnMixer"]


def _infer_prefill(attn_metadata: Optional[object]) -> bool:
    """src/cta/serving_vllm.py:49-61."""
    if attn_metadata is None:
        return True
    for attr in ("is_prefill", "prefill"):
        val = getattr(attn_metadata, attr, None)
        if isinstance(val, bool):
            return val
    num_prefill = getattr(attn_metadata, "num_prefill_tokens", None)
    if isinstance(num_prefill, int):
        return num_prefill > 0
    if getattr(attn_metadata, "prefill_metadata", None) is not None:
        return True
    return True


def _to_int(value: object) -> Optional[int]:
    """src/cta/serving_vllm.py:64-69."""
    if isinstance(value, int):
        return value
    if isinstance(value, torch.Tensor) and value.numel() == 1:
        return int(value.item())
    return None


def _max_query_len(attn_metadata: object) -> Optional[int]:
    """max_query_len of the batch as a host int, without a device sync where the
    metadata allows it.

    vLLM 0.22's v1 metadata (``FlashAttentionMetadata``,
    ``CommonAttentionMetadata``) carries it as a Python int.  A device tensor is
    read through the metadata's host copy of the offsets (``query_start_loc_cpu``)
    when there is one; only otherwise does it cost a ``.item()`` sync, as in the
    reference (src/cta/serving_vllm.py:64-69, :292)."""
    value = getattr(attn_metadata, "max_query_len", None)
    if isinstance(value, torch.Tensor) and value.numel() == 1 and value.device.type != "cpu":
        host = getattr(attn_metadata, "query_start_loc_cpu", None)
        if isinstance(host, torch.Tensor) and host.numel() >= 2:
            return int((host[1:] - host[:-1]).max())
    return _to_int(value)


@dataclass
class CtaConfig:
    """src/cta/serving_vllm.py:135-150, plus two fields of this build."""

    enabled: bool = True
    prefill_only: bool = True
    steps: int = 4
    alpha: float = 0.10
    layout: str = "bld"
    use_triton: bool = True
    fused: bool = True
    allow_transpose: bool = True
    min_seq_len: int = 0
    steps_policy: str = "fixed"
    steps_scale: int = 2048
    max_steps: int = 8
    use_buffer_pool: bool = False
    trace: bool = True
    # packed prefill rule: "reference" = zero padding to max_query_len, "sequence" = per-sequence boundary
    varlen_mode: str = "reference"
    # fuse step counts outside {1, 2, 4, 8} too (fp32 between steps)
    fuse_any_steps: bool = True


class CtaPostAttnMixer(nn.Module):
    """Apply CTA diffusion after the attention output (prefill-only by default)."""

    def __init__(self, config: CtaConfig):
        super().__init__()
        if config.layout not in {"bld", "bdl"}:
            raise ValueError("layout must be 'bld' or 'bdl'")
        if config.varlen_mode not in {"reference", "sequence"}:
            raise ValueError("varlen_mode must be 'reference' or 'sequence'")
        self.config = config
        self._qsl_cache: dict = {}

    def _resolve_steps(self, seq_len: int) -> int:
        """src/cta/serving_vllm.py:177-189."""
        if seq_len < self.config.min_seq_len:
            return 0
        policy = self.config.steps_policy
        if policy == "fixed":
            steps = self.config.steps
        elif policy == "linear":
            steps = max(1, seq_len // max(1, self.config.steps_scale))
        elif policy == "log2":
            steps = max(1, int(math.log2(max(2, seq_len))))
        else:
            steps = self.config.steps
        return min(self.config.max_steps, int(steps))

    def _arith(self):
        """The arithmetic of the reference path this call replaces: its Triton
        kernels (use_triton, with allow_transpose for the [B, L, D] layout)
        contract c + alpha * lap into one fma, its PyTorch fallback
        (src/cta/serving_vllm.py:268-273) rounds the product and the sum
        separately.  None: the process default."""
        cfg = self.config
        if not cfg.use_triton or (cfg.layout == "bld" and not cfg.allow_transpose):
            return "exact"
        return None

    def _fused_ok(self, steps: int) -> bool:
        if not self.config.fused:
            return False
        if steps in (1, 2, 4, 8):
            return True
        return self.config.fuse_any_steps and 1 <= steps <= _lib.MAX_STEPS

    def forward(  # type: ignore[override]
        self,
        x: torch.Tensor,
        *,
        attn_metadata: Optional[object] = None,
        is_prefill: Optional[bool] = None,
        residual: Optional[torch.Tensor] = None,
    ) -> torch.Tensor:
        """The mixer of src/cta/serving_vllm.py:225-273.  With `residual` it
        returns residual + mixer(x), the decoder layer's next line
        (serving/vllm/patches/vllm_0_13_0_cta_post_attn.patch:66-68), with the add
        fused into the stencil's last launch where there is one."""
        out, fused = self._mix(x, attn_metadata=attn_metadata, is_prefill=is_prefill, residual=residual)
        if residual is not None and not fused:
            out = residual + out
        return out

    def _mix(self, x, *, attn_metadata, is_prefill, residual):
        """(output, residual already added)."""
        if x.ndim == 2:
            return self._mix_packed(x, attn_metadata=attn_metadata, is_prefill=is_prefill, residual=residual)
        if not self.config.enabled:
            return x, False
        if self.config.prefill_only:
            if is_prefill is None:
                is_prefill = _infer_prefill(attn_metadata)
            if not is_prefill:
                return x, False
        seq_dim = 2 if self.config.layout == "bdl" else 1
        steps = self._resolve_steps(x.size(seq_dim))
        if steps <= 0:
            return x, False
        if x.device.type != "cuda":
            raise ValueError("x must be on CUDA")
        if x.ndim != 3:
            raise ValueError(f"expected x.ndim == 3, got {x.ndim}")
        if x.size(seq_dim) < 3:
            return x, False
        ctx = record_function("cta_post_attn_mixer") if self.config.trace else nullcontext()
        alpha = float(self.config.alpha)
        with ctx, _lib.thread_arithmetic(self._arith()):
            if self._fused_ok(steps):
                out = x
                for i in range(0, steps, _lib.MAX_STEPS):
                    s = min(_lib.MAX_STEPS, steps - i)
                    if self.config.layout == "bdl":
                        out = ops.bdl_simple(out, alpha, s)
                    elif residual is not None and i + s == steps:
                        return ops.bld_forward(out, [alpha] * s, s, residual=residual), True
                    else:
                        out = ops.bld_forward(out, [alpha] * s, s)
                return out, False
            # reference's non-fused path: one step at a time, rounded each step
            if self.config.layout == "bdl":
                return diffusion_triton(x, alpha=alpha, steps=steps), False
            out = x
            for _ in range(steps):
                out = ops.bld_forward(out, [alpha], 1)
            return out, False

    def _device_qsl(self, qsl: object, device: torch.device) -> torch.Tensor:
        if isinstance(qsl, torch.Tensor):
            if qsl.device == device and qsl.dtype == torch.int32:
                return qsl
            return qsl.to(device=device, dtype=torch.int32, non_blocking=True)
        return torch.tensor(list(qsl), dtype=torch.int32).to(device, non_blocking=True)

    def _forward_packed(
        self,
        x: torch.Tensor,
        *,
        attn_metadata: Optional[object],
        is_prefill: Optional[bool],
    ) -> torch.Tensor:
        """Packed [T, H] prefill (src/cta/serving_vllm.py:275-303), one launch."""
        return self._mix_packed(x, attn_metadata=attn_metadata, is_prefill=is_prefill, residual=None)[0]

    def _packed_plan(self, attn_metadata: Optional[object], is_prefill: Optional[bool]):
        """The gate of src/cta/serving_vllm.py:281-298 on the metadata alone:
        None (x passes through unchanged) or (query_start_loc as given,
        max_query_len as a host int, steps)."""
        if not self.config.enabled:
            return None
        if attn_metadata is None:
            return None
        if self.config.prefill_only:
            if is_prefill is None:
                is_prefill = _infer_prefill(attn_metadata)
            if not is_prefill:
                return None
        max_query_len = _max_query_len(attn_metadata)
        query_start_loc = getattr(attn_metadata, "query_start_loc", None)
        if max_query_len is None or query_start_loc is None:
            return None
        if max_query_len < 3:
            return None
        steps = self._resolve_steps(max_query_len)
        if steps <= 0:
            return None
        return query_start_loc, max_query_len, steps

    def _mix_packed(
        self,
        x: torch.Tensor,
        *,
        attn_metadata: Optional[object],
        is_prefill: Optional[bool],
        residual: Optional[torch.Tensor] = None,
    ):
        """_forward_packed, optionally with the residual add fused into the last
        launch.  Returns (output, residual already added).

        vLLM 0.22 (v1 engine) metadata has no prefill flag, so, as in the
        reference's ``_infer_prefill``, a packed batch counts as prefill and every
        sequence of it goes through the stencil, decodes included.  A decode row
        (query length 1) is unchanged under both rules: a one-row sequence is its
        own boundary row.  A speculative-decode sequence of two rows changes
        under the reference rule (zero padding to max_query_len makes its last
        row interior) exactly as in the reference, and is unchanged under
        ``varlen_mode="sequence"`` (sequences shorter than 3 rows are the
        identity).  Rows after the last sequence (padding tokens of a CUDA-graph
        batch) are not written, as the reference's unpack leaves them."""
        plan = self._packed_plan(attn_metadata, is_prefill)
        if plan is None:
            return x, False
        query_start_loc, max_query_len, steps = plan
        if x.device.type != "cuda":
            raise ValueError("x must be on CUDA")
        cu = self._device_qsl(query_start_loc, x.device)
        pad = self.config.varlen_mode == "reference"
        alpha = float(self.config.alpha)
        ctx = record_function("cta_post_attn_mixer") if self.config.trace else nullcontext()
        with ctx, _lib.thread_arithmetic(self._arith()):
            out = x
            for i in range(0, steps, _lib.MAX_STEPS):
                s = min(_lib.MAX_STEPS, steps - i)
                last = i + s == steps
                out = ops.varlen_forward(out, cu, max_query_len, alpha, s, pad_to_max=pad,
                                         residual=residual if last else None)
            return out, residual is not None
