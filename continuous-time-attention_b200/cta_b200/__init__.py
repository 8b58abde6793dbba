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

__version__ = "0.1.0"
