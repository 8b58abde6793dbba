"""Import-path alias for code written against the reference's
``kernels.diffusion_triton`` module: the same four public functions, served by
the sm_100a kernels of :mod:`cta_b200.diffusion` (no Triton involved)."""
from .diffusion import (  # noqa: F401
    diffusion_step_triton,
    diffusion_step_triton_backward,
    diffusion_triton,
    diffusion_triton_fused,
)

__all__ = [
    "diffusion_step_triton",
    "diffusion_triton",
    "diffusion_triton_fused",
    "diffusion_step_triton_backward",
]
