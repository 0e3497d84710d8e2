"""Host-side API behaviour that needs no GPU: exported names, registration,
error messages, CPU tensors rejected (no CPU fallback), index helpers."""

import pytest
import torch

import hf_attention_normalizers_b200 as H
from hf_attention_normalizers_b200 import backends, kernels, paged, varlen

REFERENCE_ALL = [
    "AttentionReplacementPolicy", "Qwen3AttentionExtra", "Qwen3AttentionExtrea", "apply_softmax1_attention",
    "apply_softmax_attention", "from_pretrained_with_registered_softmax_attention",
    "from_pretrained_with_softmax_attention", "register_attention_replacement_policy",
    "register_entmax15_attention_backends", "register_softmax1_attention_backends",
    "register_softmax_attention_backends", "register_sparsemax_attention_backends", "replace_attention_modules",
    "replace_qwen3_attention_modules", "set_softmax_attention_backend", "softmax_attention_backend_name",
    "supported_attention_policies", "triton_entmax15_attention_forward", "triton_sparsemax_attention_forward",
    "paged_attention", "paged_cache_indices", "paged_triton_attention", "DifferentiablePagedCache",
    "DifferentiablePagedCacheLayer", "varlen_hopper_attention",
]


def test_public_names_match_reference():
    assert sorted(H.__all__) == sorted(REFERENCE_ALL)
    for name in REFERENCE_ALL:
        assert hasattr(H, name)
    for name in kernels.__all__:
        assert callable(getattr(kernels, name))


def test_registration_names():
    names = H.register_entmax15_attention_backends()
    assert names[0] == "entmax15_eager" and names[-1] == "entmax15_triton" and len(names) == 11
    assert len(H.register_softmax1_attention_backends()) == 10
    assert H.softmax_attention_backend_name("triton", "sparsemax") == "sparsemax_triton"
    assert H.softmax_attention_backend_name("flash_attention_3", "softmax1") == "softmax1_flash_attention_3"
    with pytest.raises(ValueError, match="mode must be"):
        H.register_softmax_attention_backends("softmax1", mode="bogus")
    with pytest.raises(ValueError, match="fallback_backend must be one of"):
        H.register_softmax_attention_backends("softmax1", fallback_backend="nope")


def test_strict_mode_unsupported_backend_raises_on_call():
    fwd = backends._make_softmax_attention_forward("flash_attention_3", softmax_fn="softmax", mode="strict")
    with pytest.raises(NotImplementedError, match="does not have a custom-softmax kernel"):
        fwd(None, None, None, None, None)
    fb = backends._make_softmax_attention_forward("flash_attention_3", softmax_fn="softmax", mode="fallback")
    assert callable(fb)


def test_resolve_softmax_fn():
    assert backends.resolve_softmax_fn("softmax1") is backends.softmax_1
    with pytest.raises(ValueError, match="Invalid softmax function"):
        backends.resolve_softmax_fn("nope")


def test_cpu_tensors_are_rejected_not_computed():
    q = torch.randn(1, 2, 8, 32)
    for fn in (kernels.hopper_softmax1_attention, kernels.hopper_sparsemax_attention,
               kernels.hopper_entmax15_attention):
        with pytest.raises(ValueError, match="requires CUDA tensors"):
            fn(q, q, q, is_causal=True)
    with pytest.raises(ValueError, match="requires CUDA tensors"):
        varlen.varlen_hopper_attention(q[0], q[0], q[0], torch.tensor([0, 8]), torch.tensor([0, 8]), "entmax15")
    with pytest.raises(ValueError, match="CUDA"):
        kc = torch.randn(16, 2, 32)
        H.paged_attention(q, kc, kc, torch.tensor([[0, 1]]), torch.tensor([8]), 4)
    with pytest.raises(ValueError, match="CUDA"):
        from hf_attention_normalizers_b200.vutils import sparsemax
        sparsemax(torch.randn(3, 4))


def test_varlen_shape_validation_messages():
    q = torch.randn(8, 4, 32)
    with pytest.raises(ValueError, match=r"Packed Q/K/V must have shape"):
        varlen.varlen_hopper_attention(q[None], q, q, torch.tensor([0, 8]), torch.tensor([0, 8]), "sparsemax")
    with pytest.raises(ValueError, match="divisible by KV heads"):
        varlen.varlen_hopper_attention(q, q[:, :3], q[:, :3], torch.tensor([0, 8]), torch.tensor([0, 8]), "sparsemax")
    with pytest.raises(ValueError, match="must start at zero"):
        varlen._validate_cumulative_lengths(torch.tensor([1, 8]), 8, "cu_seqlens_q")
    with pytest.raises(ValueError, match="must end at the total token count"):
        varlen._validate_cumulative_lengths(torch.tensor([0, 7]), 8, "cu_seqlens_q")
    with pytest.raises(ValueError, match="nondecreasing"):
        varlen._validate_cumulative_lengths(torch.tensor([0, 5, 3, 8]), 8, "cu_seqlens_q")
    with pytest.raises(ValueError, match="int32 or int64"):
        varlen._validate_cumulative_lengths(torch.tensor([0.0, 8.0]), 8, "cu_seqlens_q")


def test_paged_cache_indices_matches_golden_layout(golden):
    g = golden("paged")
    bt = torch.tensor(g["paged_shared_block_table"])
    sl = torch.tensor(g["paged_shared_seq_lens"])
    phys, valid = H.paged_cache_indices(bt, sl, int(g["paged_shared_block_size"]))
    assert phys.tolist() == [[8, 9, 10, 11, 0, 1, 2], [8, 9, 10, 11, 12, 13, 14]]
    assert valid.tolist() == [[True] * 5 + [False] * 2, [True] * 7]
    with pytest.raises(ValueError, match="enough blocks"):
        H.paged_cache_indices(bt, torch.tensor([5, 9]), 4)
    with pytest.raises(ValueError, match="positive"):
        H.paged_cache_indices(bt, torch.tensor([0, 3]), 4)


def test_paged_entry_validation_messages():
    q = torch.randn(2, 4, 1, 8)
    kc = torch.randn(16, 2, 8)
    with pytest.raises(ValueError, match="supports 'softmax1', 'sparsemax', or 'entmax15'"):
        H.paged_triton_attention(q, kc, kc, torch.zeros(2, 2, dtype=torch.long), torch.tensor([3, 3]), 4, "softmax")
    with pytest.raises(ValueError, match="key_cache and value_cache shapes must match"):
        H.paged_attention(q, kc, kc[:8], torch.zeros(2, 2, dtype=torch.long), torch.tensor([3, 3]), 4)
