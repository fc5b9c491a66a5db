"""CPU: the drop-in Python surface — validation and error messages of the
reference wrapper (python/modeling_attention.py:21-192), mask/score merging as
handed to the op, the HF adapter's defaults, and no CPU fallback."""

from __future__ import annotations

import pytest
import torch

import tilelang_fa2_4d_mask as api
import python as py_alias
import python.fa2 as py_fa2
import python.modeling_attention as py_ma
from oracle.eager import merge_wrapper_inputs

impl_ma = __import__("fa2_with_4d_mask_b200.modeling_attention", fromlist=["x"])


def qkv(B=1, Hq=4, Hk=2, Tq=16, Tk=24, D=64, dtype=torch.bfloat16, layout="bhsd"):
    q = torch.randn(B, Hq, Tq, D).to(dtype)
    k = torch.randn(B, Hk, Tk, D).to(dtype)
    v = torch.randn(B, Hk, Tk, D).to(dtype)
    if layout == "bshd":
        q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    return q, k, v


@pytest.fixture
def captured(monkeypatch):
    """Replaces the op the wrapper calls and records its positional arguments."""
    calls = []

    def fake(*args):
        calls.append(args)
        return args[0]

    monkeypatch.setattr(impl_ma, "flash_attention_with_4d_mask", fake)
    return calls


def test_import_paths_expose_the_reference_names():
    for mod in (api, py_alias):
        for name in ("flash_attention_with_4d_mask", "tilelang_attention_forward", "tilelang_flash_attention"):
            assert callable(getattr(mod, name))
    assert py_fa2.flash_attention_with_4d_mask is api.flash_attention_with_4d_mask
    assert py_ma.tilelang_flash_attention is api.tilelang_flash_attention


@pytest.mark.parametrize(
    "mutate,msg",
    [
        (lambda q, k, v: (q[0], k, v), "query, key, and value must be rank-4 tensors"),
        (lambda q, k, v: (q, k[:, :, :20], v), "key and value must have the same sequence length"),
        (lambda q, k, v: (q, k[:, :1], v), "key and value must have the same number of heads"),
        (lambda q, k, v: (q, k[..., :32], v), "query, key, and value must have the same head dimension"),
        (lambda q, k, v: (q[:, :3], k, v), "query heads (3) must be divisible by key/value heads (2)"),
        (lambda q, k, v: (q, torch.cat([k, k]), v), "query, key, and value must have the same batch size"),
        (lambda q, k, v: (q.float(), k.float(), v.float()), "TileLang attention expects fp16 or bf16 inputs, got torch.float32"),
        (lambda q, k, v: (q, k.half(), v), "query, key, and value must have the same dtype"),
    ],
)
def test_validation_messages_match_reference(mutate, msg):
    q, k, v = mutate(*qkv())
    with pytest.raises(ValueError) as ei:
        api.tilelang_flash_attention(q, k, v)
    assert str(ei.value) == msg


def test_layout_and_mask_errors():
    q, k, v = qkv()
    with pytest.raises(ValueError, match="unsupported layout: bsdh"):
        api.tilelang_flash_attention(q, k, v, layout="bsdh")
    with pytest.raises(ValueError, match="mask must be a bool tensor with True for valid entries"):
        api.tilelang_flash_attention(q, k, v, mask=torch.ones(1, 1, 16, 24))
    with pytest.raises(ValueError, match="score must be a floating-point tensor"):
        api.tilelang_flash_attention(q, k, v, score=torch.ones(1, 1, 16, 24, dtype=torch.int32))
    with pytest.raises(ValueError, match=r"mask has trailing shape \(16, 23\), expected \(16, 24\)"):
        api.tilelang_flash_attention(q, k, v, mask=torch.ones(1, 1, 16, 23, dtype=torch.bool))
    with pytest.raises(ValueError, match="mask head dimension must be 1 or 4"):
        api.tilelang_flash_attention(q, k, v, mask=torch.ones(1, 2, 16, 24, dtype=torch.bool))
    with pytest.raises(ValueError, match="mask batch dimension must be 1 or 1"):
        api.tilelang_flash_attention(q, k, v, mask=torch.ones(2, 1, 16, 24, dtype=torch.bool))
    with pytest.raises(ValueError, match=r"score must have shape \[B, H or 1, Tq, Tk\]"):
        api.tilelang_flash_attention(q, k, v, score=torch.ones(16, 24))
    with pytest.raises(ValueError, match="attention_mask must be bool or floating point"):
        api.tilelang_flash_attention(q, k, v, attention_mask=torch.ones(1, 1, 16, 24, dtype=torch.int64))


def test_merges_as_the_reference_wrapper(captured):
    q, k, v = qkv()
    scale = 0.125
    mask = torch.rand(1, 1, 16, 24) > 0.3
    score = torch.randn(1, 4, 16, 24)
    am_f = torch.randn(1, 1, 16, 24)
    am_b = torch.rand(1, 4, 16, 24) > 0.2
    for am, scaled in ((am_f, True), (am_f, False), (am_b, True)):
        captured.clear()
        api.tilelang_flash_attention(q, k, v, mask=mask, score=score, attention_mask=am, scale=scale,
                                     attention_mask_is_scaled=scaled)
        args = captured[0]
        m_ref, s_ref = merge_wrapper_inputs(batch=1, heads=4, seqlen_q=16, seqlen_k=24, scale=scale, mask=mask,
                                            score=score, attention_mask=am, attention_mask_is_scaled=scaled)
        assert torch.equal(args[3].expand(1, 4, 16, 24), m_ref)
        torch.testing.assert_close(args[4].expand(1, 4, 16, 24), s_ref)
        assert args[5] == scale and args[6] is False and args[7] is True and args[8] is True


def test_broadcast_mask_is_not_materialised(captured):
    q, k, v = qkv()
    mask = torch.rand(1, 1, 16, 24) > 0.3
    api.tilelang_flash_attention(q, k, v, mask=mask)
    m = captured[0][3]
    assert m.shape == (1, 4, 16, 24) and m.stride(1) == 0 and m.data_ptr() == mask.data_ptr()


def test_defaults_and_bshd(captured):
    q, k, v = qkv(layout="bshd")
    api.tilelang_flash_attention(q, k, v, layout="bshd", is_causal=True, use_atomic_backward=False)
    args = captured[0]
    assert args[3] is None and args[4] is None
    assert args[5] == pytest.approx(64 ** -0.5)
    assert args[6] is True and args[7] is False and args[8] is False and args[9] == "top_left"


class _Module:
    is_causal = True


def test_hf_adapter(captured):
    q, k, v = qkv()
    out, w = api.tilelang_attention_forward(_Module(), q, k, v, None, scaling=0.2)
    assert w is None and out is q
    assert captured[-1][6] is True  # attention_mask None and module.is_causal
    api.tilelang_attention_forward(_Module(), q, k, v, torch.ones(1, 1, 16, 24, dtype=torch.bool), scaling=0.2)
    assert captured[-1][6] is False  # a mask was given
    api.tilelang_attention_forward(object(), q, k, v, None, scaling=0.2)
    assert captured[-1][6] is True  # default module.is_causal = True
    api.tilelang_attention_forward(_Module(), q, k, v, None, scaling=0.2, is_causal=False, layout="bhsd",
                                   causal_align="bottom_right")
    assert captured[-1][6] is False and captured[-1][9] == "bottom_right"
    with pytest.raises(ValueError, match="TileLang FA2 wrapper does not implement attention dropout"):
        api.tilelang_attention_forward(_Module(), q, k, v, None, scaling=0.2, dropout=0.1)


def test_no_cpu_fallback():
    q, k, v = qkv()
    with pytest.raises(RuntimeError, match="CUDA"):
        api.tilelang_flash_attention(q, k, v)


def test_unknown_causal_align():
    causal_mode = __import__("fa2_with_4d_mask_b200.fa2", fromlist=["x"]).causal_mode
    assert causal_mode(False, "middle") == 0
    assert causal_mode(True) == 1 and causal_mode(True, "bottom_right") == 2
    with pytest.raises(ValueError, match="unsupported causal_align"):
        causal_mode(True, "middle")


def test_doc_ids_are_validated_and_forwarded(captured):
    q, k, v = qkv(B=2, Tq=16, Tk=16)
    ids = torch.zeros(2, 16, dtype=torch.int32)
    api.tilelang_flash_attention(q, k, v, doc_ids=ids)
    assert captured[-1][10] is ids


def test_doc_id_parsing():
    impl_fa2 = __import__("fa2_with_4d_mask_b200.fa2", fromlist=["x"])
    dq, dk = impl_fa2._doc_ids(torch.arange(8).view(1, 8), 2, 8, 8, "cpu")
    assert dq.dtype == torch.int32 and dq.shape == (1, 8) and dk is not None
    with pytest.raises(ValueError, match="Tq == Tk"):
        impl_fa2._doc_ids(torch.zeros(1, 8, dtype=torch.int64), 1, 8, 9, "cpu")
    with pytest.raises(ValueError, match="doc_k must be"):
        impl_fa2._doc_ids((torch.zeros(1, 8, dtype=torch.int64), torch.zeros(1, 7, dtype=torch.int64)), 1, 8, 9, "cpu")
    with pytest.raises(ValueError, match="integer"):
        impl_fa2._doc_ids(torch.zeros(1, 8), 1, 8, 8, "cpu")


def _op_inputs(bhsd=True):
    """Q [1, 4, 16, 64], K/V [1, 2, 24, 64] (BHSD) or their BSHD transposes."""
    q, k, v = qkv(B=1, Hq=4, Hk=2, Tq=16, Tk=24, D=64)
    if not bhsd:
        q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    return q, k, v


@pytest.mark.parametrize(
    "case,msg",
    [
        ("v_seq", "K and V must have the same shape"),
        ("v_heads", "K and V must have the same shape"),
        ("k_batch", "same batch size"),
        ("k_dim", "same head dimension"),
        ("gqa", r"query heads \(3\) must be divisible by key/value heads \(2\)"),
        ("mask_rank", r"Mask must have shape \[B or 1, Hq or 1, Tq, Tk\]"),
        ("mask_tq", r"Mask has trailing shape \(15, 24\), expected \(16, 24\)"),
        ("mask_tk", r"Mask has trailing shape \(16, 23\), expected \(16, 24\)"),
        ("mask_heads_hk", "Mask head dimension must be 1 or 4"),
        ("mask_batch", "Mask batch dimension must be 1 or 1"),
        ("mask_float", "Mask must be a bool tensor"),
        ("score_tk", r"Score has trailing shape \(16, 25\), expected \(16, 24\)"),
        ("score_heads", "Score head dimension must be 1 or 4"),
        ("score_int", "Score must be a floating-point tensor"),
        ("dtype", "must have the same dtype"),
        ("fp32", "Q must be fp16 or bf16"),
    ],
)
@pytest.mark.parametrize("bhsd", [True, False])
def test_op_rejects_shapes_the_kernels_would_read_out_of_bounds(case, msg, bhsd):
    """The autograd op (not only the wrapper) refuses mask / score / V shapes that do
    not match Q and K, before anything reaches the C ABI."""
    q, k, v = _op_inputs(bhsd)
    mask = score = None
    seq = 2 if bhsd else 1  # sequence axis of Q/K/V in this layout
    head = 1 if bhsd else 2
    if case == "v_seq":
        v = v.narrow(seq, 0, 20)
    elif case == "v_heads":
        v = v.narrow(head, 0, 1)
    elif case == "k_batch":
        k, v = torch.cat([k, k]), torch.cat([v, v])
    elif case == "k_dim":
        k, v = k[..., :32], v[..., :32]
    elif case == "gqa":
        q = q.narrow(head, 0, 3)
    elif case == "mask_rank":
        mask = torch.ones(16, 24, dtype=torch.bool)
    elif case == "mask_tq":
        mask = torch.ones(1, 1, 15, 24, dtype=torch.bool)
    elif case == "mask_tk":
        mask = torch.ones(1, 1, 16, 23, dtype=torch.bool)
    elif case == "mask_heads_hk":
        mask = torch.ones(1, 2, 16, 24, dtype=torch.bool)
    elif case == "mask_batch":
        mask = torch.ones(2, 1, 16, 24, dtype=torch.bool)
    elif case == "mask_float":
        mask = torch.ones(1, 1, 16, 24)
    elif case == "score_tk":
        score = torch.zeros(1, 4, 16, 25)
    elif case == "score_heads":
        score = torch.zeros(1, 2, 16, 24)
    elif case == "score_int":
        score = torch.zeros(1, 4, 16, 24, dtype=torch.int32)
    elif case == "dtype":
        v = v.half()
    elif case == "fp32":
        q, k, v = q.float(), k.float(), v.float()
    with pytest.raises(ValueError, match=msg):
        api.flash_attention_with_4d_mask(q, k, v, mask, score, None, False, True, bhsd)


def test_op_accepts_broadcast_mask_and_score_then_needs_cuda():
    """Well-formed inputs pass the checks and reach the (absent) device path."""
    q, k, v = _op_inputs()
    mask = torch.ones(1, 1, 16, 24, dtype=torch.bool)
    score = torch.zeros(1, 4, 16, 24)
    with pytest.raises(RuntimeError, match="CUDA"):
        api.flash_attention_with_4d_mask(q, k, v, mask, score, None, False, True, True)
