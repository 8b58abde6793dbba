"""The packed-prefill mixer driven by vLLM 0.22's own attention metadata.

vLLM's v1 engine hands the attention layer ``FlashAttentionMetadata`` (built
from ``CommonAttentionMetadata``): ``query_start_loc`` on the device,
``max_query_len`` as a host int, and no prefill flag.  The reference's gate
(src/cta/serving_vllm.py:49-61) therefore treats every packed batch as prefill,
and so does the drop-in.  CPU tests cover the gate and the host-side reading of
the metadata; the GPU tests run the mixer on a mixed prefill + decode batch and
compare with the oracle under both packing rules.
"""
from __future__ import annotations

import pytest
import torch

from oracle import diffusion_oracle as O

vllm_fa = pytest.importorskip("vllm.v1.attention.backends.flash_attn")
vllm_utils = pytest.importorskip("vllm.v1.attention.backends.utils")

# prefill 700, two decodes, prefill 300, a two-row speculative decode, prefill 41
LENS = [700, 1, 1, 300, 2, 41]


def _qsl(lens, device="cpu"):
    q = torch.zeros(len(lens) + 1, dtype=torch.int32)
    q[1:] = torch.cumsum(torch.tensor(lens), 0)
    return q.to(device)


def _flash_md(lens, device="cpu", max_query_len=None):
    q = _qsl(lens, device)
    n = len(lens)
    return vllm_fa.FlashAttentionMetadata(
        num_actual_tokens=int(sum(lens)),
        max_query_len=max(lens) if max_query_len is None else max_query_len,
        query_start_loc=q,
        max_seq_len=max(lens),
        seq_lens=torch.tensor(lens, dtype=torch.int32, device=device),
        block_table=torch.zeros(n, 1, dtype=torch.int32, device=device),
        slot_mapping=torch.zeros(int(sum(lens)), dtype=torch.int64, device=device),
        use_cascade=False,
        common_prefix_len=0,
        cu_prefix_query_lens=None,
        prefix_kv_lens=None,
        suffix_kv_lens=None,
    )


def _common_md(lens, device="cpu", max_query_len=None):
    n = len(lens)
    return vllm_utils.CommonAttentionMetadata(
        query_start_loc=_qsl(lens, device),
        query_start_loc_cpu=_qsl(lens),
        seq_lens=torch.tensor(lens, dtype=torch.int32, device=device),
        num_reqs=n,
        num_actual_tokens=int(sum(lens)),
        max_query_len=max(lens) if max_query_len is None else max_query_len,
        max_seq_len=max(lens),
        block_table_tensor=torch.zeros(n, 1, dtype=torch.int32, device=device),
        slot_mapping=torch.zeros(int(sum(lens)), dtype=torch.int64, device=device),
    )


def test_v1_metadata_counts_as_prefill():
    """No is_prefill / prefill / num_prefill_tokens / prefill_metadata in v1:
    the reference's gate falls through to True, and so does ours."""
    from cta_b200.serving_vllm import _infer_prefill

    for md in (_flash_md(LENS), _common_md(LENS)):
        for attr in ("is_prefill", "prefill", "num_prefill_tokens", "prefill_metadata"):
            assert not hasattr(md, attr)
        assert _infer_prefill(md) is True


def test_max_query_len_host_int_and_host_offsets():
    from cta_b200.serving_vllm import _max_query_len

    assert _max_query_len(_flash_md(LENS)) == 700
    assert _max_query_len(_common_md(LENS)) == 700
    # a one-element CPU tensor reads without any device sync
    assert _max_query_len(_flash_md(LENS, max_query_len=torch.tensor(700))) == 700


def test_pure_decode_batch_is_untouched_before_any_launch(monkeypatch):
    """max_query_len < 3 returns x itself (src/cta/serving_vllm.py:297-298): no
    launch, so a CPU tensor passes through too."""
    from cta_b200 import ops
    from cta_b200.serving_vllm import CtaConfig, CtaPostAttnMixer

    def boom(*a, **k):
        raise AssertionError("no launch expected")

    monkeypatch.setattr(ops, "varlen_forward", boom)
    x = torch.randn(4, 16)
    mixer = CtaPostAttnMixer(CtaConfig())
    assert mixer(x, attn_metadata=_flash_md([1, 1, 1, 1])) is x
    assert mixer(x, attn_metadata=_common_md([2, 1, 1])) is x


def test_packed_plan_keeps_the_metadata_offsets():
    """The launch gets the metadata's own offsets tensor (no host copy of it) and
    max_query_len as the padding length of the reference rule."""
    from cta_b200.serving_vllm import CtaConfig, CtaPostAttnMixer

    mixer = CtaPostAttnMixer(CtaConfig(steps=4))
    for md in (_flash_md(LENS), _common_md(LENS)):
        qsl, max_len, steps = mixer._packed_plan(md, None)
        assert qsl is md.query_start_loc and max_len == 700 and steps == 4
    # the step policies see max_query_len (src/cta/serving_vllm.py:177-189)
    lin = CtaPostAttnMixer(CtaConfig(steps_policy="linear", steps_scale=128))
    assert lin._packed_plan(_flash_md(LENS), None)[2] == 700 // 128
    assert CtaPostAttnMixer(CtaConfig(prefill_only=True))._packed_plan(_flash_md(LENS), False) is None


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["reference", "sequence"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_mixer_on_v1_metadata_mixed_batch(mode, dtype):
    """A mixed prefill + decode batch through FlashAttentionMetadata and
    CommonAttentionMetadata on the device, bit for bit against the oracle:
    the reference's zero-pad rule, or the per-sequence rule."""
    from cta_b200.serving_vllm import CtaConfig, CtaPostAttnMixer

    torch.manual_seed(5)
    T, D = sum(LENS), 256
    x = torch.randn(T, D, dtype=dtype)
    qsl = _qsl(LENS).tolist()
    if mode == "reference":
        ref = O.mixer_packed(x, qsl, max(LENS), alpha=0.1, steps=4, contracted=dtype != torch.float32)
    else:
        ref = O.varlen_per_sequence(x, qsl, alpha=0.1, steps=4, contracted=dtype != torch.float32)
    mixer = CtaPostAttnMixer(CtaConfig(steps=4, alpha=0.1, varlen_mode=mode, trace=False))
    for md in (_flash_md(LENS, "cuda"), _common_md(LENS, "cuda")):
        y = mixer(x.cuda(), attn_metadata=md).cpu()
        assert torch.equal(y, ref), mode
        # decode rows (query length 1) are unchanged under both rules
        for i, n in enumerate(LENS):
            if n == 1:
                assert torch.equal(y[qsl[i]], x[qsl[i]])
