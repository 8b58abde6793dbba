"""CPU-only checks: the C ABI library loads and exports every declared symbol,
argument validation fails cleanly without touching a device, and the host-side
logic of the Python surface (gating, step policies, errors) matches the reference."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch

REPO = Path(__file__).resolve().parents[1]


def _declared_symbols():
    text = (REPO / "include" / "cta_stencil.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(cta_\w+)\s*\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    from cta_b200 import _lib

    lib = _lib.load()
    names = _declared_symbols()
    assert len(names) >= 12, names
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/cta_stencil.h but not exported"
    assert set(names) == set(_lib._SIGNATURES), "ctypes signatures out of sync with the header"
    assert lib.cta_abi_version() == 1


def test_invalid_arguments_fail_before_launch():
    from cta_b200 import _lib

    lib = _lib.load()
    one = _lib.float_array([0.1])
    null = ctypes.c_void_p(0)
    # bad dtype
    rc = lib.cta_diffusion_fwd_bld(null, null, 1, 10, 8, 80, 8, 80, 8, 7, 1, 0, one, None, 0, null, 0, 0, 0, null)
    assert rc == _lib.CTA_EINVAL and b"dtype" in lib.cta_last_error()
    # steps out of range
    rc = lib.cta_diffusion_fwd_bdl(null, null, 1, 1, 10, 10, 0, 9, ctypes.c_float(0.1), null)
    assert rc == _lib.CTA_EINVAL and b"steps" in lib.cta_last_error()
    # L < 3 is the caller's identity case
    rc = lib.cta_diffusion_fwd_bdl(ctypes.c_void_p(16), ctypes.c_void_p(16), 1, 1, 2, 2, 0, 1, ctypes.c_float(0.1),
                                   null)
    assert rc == _lib.CTA_EINVAL
    # alpha missing
    rc = lib.cta_diffusion_fwd_bld(null, null, 1, 10, 8, 80, 8, 80, 8, 0, 1, 0, None, None, 0, null, 0, 0, 0, null)
    assert rc == _lib.CTA_EINVAL and b"alpha" in lib.cta_last_error()
    # empty tensors are a no-op
    rc = lib.cta_diffusion_fwd_bld(null, null, 0, 10, 8, 80, 8, 80, 8, 0, 1, 0, one, None, 0, null, 0, 0, 0, null)
    assert rc == _lib.CTA_OK
    # bad shard part
    rc = lib.cta_diffusion_shard_bld(ctypes.c_void_p(16), ctypes.c_void_p(16), 1, 100, 8, 0, 100, null, 0, null, 0,
                                     7, 0, 2, 0, 0, ctypes.c_float(0.1), null)
    assert rc == _lib.CTA_EINVAL
    assert lib.cta_diffusion_bwd_bld_workspace_bytes(1, 16384, 512, 1, 4, 0) >= 256 + 4 * 4 * 512
    # the pooled classifier form: per row tile (>= 32 rows) D column sums + one count
    assert lib.cta_diffusion_fwd_bld_pool_workspace_bytes(2, 1000, 64) >= 4 * 32 * 2 * 65
    assert lib.cta_diffusion_fwd_bld_pool_workspace_bytes(0, 1000, 64) == 256
    x16 = ctypes.c_void_p(16)
    # no mask: the pooled form is the masked mean
    rc = lib.cta_diffusion_fwd_bld_pool(x16, x16, x16, 1 << 20, 1, 100, 8, 800, 8, 1, 2, one, None, 0, null, 0,
                                        0, 0, null)
    assert rc == _lib.CTA_EINVAL and b"mask" in lib.cta_last_error()
    # workspace below the size query
    rc = lib.cta_diffusion_fwd_bld_pool(x16, x16, x16, 64, 1, 100, 8, 800, 8, 1, 2, one, None, 0, x16, 2, 100, 1,
                                        null)
    assert rc == _lib.CTA_EINVAL and b"workspace" in lib.cta_last_error()


def test_python_errors_without_gpu():
    from cta_b200 import diffusion as D
    from cta_b200.pde_layers import DiffusionPDELayer, create_pde_layer

    with pytest.raises(ValueError):
        D.diffusion_triton_fused(torch.randn(1, 2, 10), steps=2)  # CPU tensor
    with pytest.raises(ValueError):
        D.diffusion_triton_fused(torch.randn(1, 2, 10), steps=-1)
    x = torch.randn(1, 2, 10)
    assert D.diffusion_triton_fused(x, steps=0) is x
    with pytest.raises(ValueError):
        DiffusionPDELayer(4, layout="lbd")
    with pytest.raises(ValueError):
        create_pde_layer("heat", 4)
    # the reference's four types, its parameter names and defaults (pde_layers.py:195-318)
    rd = create_pde_layer("reaction-diffusion", 4, causal=True, layout="bld")
    ad = create_pde_layer("advection-diffusion", 4)
    assert sorted(n for n, _ in rd.named_parameters()) == ["alpha", "beta"] and rd.causal and rd.layout == "bld"
    assert abs(rd.beta.item() - 0.02) < 1e-7 and abs(ad.beta.item() - 0.03) < 1e-7 and ad.layout == "bdl"
    assert rd(torch.randn(1, 2, 4)).shape == (1, 2, 4)  # L < 3 identity before any device work
    with pytest.raises(ValueError):
        ad(torch.randn(1, 4, 10))  # no CPU path
    layer = DiffusionPDELayer(4, layout="bdl")
    short = torch.randn(1, 4, 2)
    assert layer(short) is short  # pde_layers.py:130-131
    with pytest.raises(ValueError):
        layer(torch.randn(1, 4, 10))  # no CPU path


def test_mixer_host_logic():
    from cta_b200.serving_vllm import CtaConfig, CtaPostAttnMixer, _infer_prefill, _to_int

    assert _infer_prefill(None) is True
    assert _infer_prefill(SimpleNamespace(is_prefill=False)) is False
    assert _infer_prefill(SimpleNamespace(num_prefill_tokens=0)) is False
    assert _infer_prefill(SimpleNamespace(prefill_metadata=object())) is True
    assert _to_int(torch.tensor([7])) == 7 and _to_int("7") is None
    m = CtaPostAttnMixer(CtaConfig(steps_policy="linear", steps_scale=1024, max_steps=8))
    assert [m._resolve_steps(n) for n in (10, 1024, 5000, 10**6)] == [1, 1, 4, 8]
    m = CtaPostAttnMixer(CtaConfig(steps_policy="log2", max_steps=8, min_seq_len=16))
    assert [m._resolve_steps(n) for n in (8, 16, 100, 10**6)] == [0, 4, 6, 8]
    with pytest.raises(ValueError):
        CtaPostAttnMixer(CtaConfig(layout="xyz"))
    with pytest.raises(ValueError):
        CtaPostAttnMixer(CtaConfig(varlen_mode="xyz"))
    x = torch.randn(2, 10, 4)
    assert CtaPostAttnMixer(CtaConfig(enabled=False))(x) is x
    assert CtaPostAttnMixer(CtaConfig())(x, is_prefill=False) is x
    flat = torch.randn(10, 4)
    assert CtaPostAttnMixer(CtaConfig())(flat) is flat  # no metadata -> passthrough (:284-285)
    md = SimpleNamespace(max_query_len=2, query_start_loc=[0, 2, 4])
    assert CtaPostAttnMixer(CtaConfig())(flat, attn_metadata=md) is flat  # max_query_len < 3


def test_arithmetic_mode_codes():
    """Mode names map to the C ABI codes; unknown modes are rejected on the host
    and by the library."""
    from cta_b200 import _lib

    assert _lib.arith_code("exact") == _lib.ARITH_EXACT == 0
    assert _lib.arith_code("contracted") == _lib.ARITH_CONTRACTED == 1
    with pytest.raises(ValueError):
        _lib.arith_code("fast")
    lib = _lib.load()
    assert lib.cta_set_arithmetic(7) == -1
    assert lib.cta_set_thread_arithmetic(7) == -2
    prev = lib.cta_set_thread_arithmetic(0)
    assert lib.cta_set_thread_arithmetic(prev) == 0


def test_build_rejects_kernel_stack_frames():
    """The build parses ptxas -v and fails on a kernel whose stack frame shows a
    helper that was not inlined (its register state in local memory)."""
    from cta_b200 import build as B

    log = "\n".join([
        "ptxas info    : Compiling entry function '_Z6kernelILi5EEvv' for 'sm_100a'",
        "ptxas info    : Function properties for _Z6kernelILi5EEvv",
        "    1432 bytes stack frame, 0 bytes spill stores, 0 bytes spill loads",
        "ptxas info    : Used 126 registers, used 1 barriers, 1432 bytes cumulative stack size",
        "ptxas info    : Compiling entry function '_Z6kernelILi4EEvv' for 'sm_100a'",
        "ptxas info    : Function properties for _Z6kernelILi4EEvv",
        "    16 bytes stack frame, 16 bytes spill stores, 16 bytes spill loads",
    ])
    assert B.stack_frames(log) == [("_Z6kernelILi5EEvv", 1432)]
