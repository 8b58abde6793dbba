"""cta_b200 -- B200-native (sm_100a) fused diffusion stencil of Continuous-Time
Attention, behind the reference's Python operator surface.

Modules
  diffusion / diffusion_triton : [B, D, L] kernel API (kernels/diffusion_triton.py)
  pde_layers                   : DiffusionPDELayer & co. (src/models/pde_layers.py)
  transformers                 : PDE Transformer models (src/models/transformers.py)
  serving_vllm                 : CtaConfig / CtaPostAttnMixer (src/cta/serving_vllm.py)
  sharded                      : L-sharded stencil over NCCL for very long sequences
  ops                          : single-launch functional wrappers over the C ABI
  build                        : nvcc build of libcta_stencil.so
"""
from . import _lib  # noqa: F401
from .diffusion import (  # noqa: F401
    diffusion_step_triton,
    diffusion_step_triton_backward,
    diffusion_triton,
    diffusion_triton_fused,
)

__version__ = "0.2.0"


def set_arithmetic(mode: str) -> str:
    """Process default of the forward update's arithmetic for bf16 / fp16
    tensors, returning the previous one:

    * ``"contracted"`` (initial): ``c + alpha * lap`` as one fused multiply-add,
      the op order the reference's Triton kernels compile to
      (kernels/diffusion_triton.py); within one bf16 / fp16 rounding of the
      exact result;
    * ``"exact"``: the product and the sum rounded separately, the reference's
      PyTorch ops (src/cta/ops/diffusion.py, src/models/pde_layers.py), bit for
      bit.

    fp32 tensors, the backward kernels and the PDE layers always use the exact
    arithmetic (the layers replace the reference's PyTorch layers)."""
    prev = _lib.load().cta_set_arithmetic(_lib.arith_code(mode))
    return "exact" if prev == _lib.ARITH_EXACT else "contracted"
