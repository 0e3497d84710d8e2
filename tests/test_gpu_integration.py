"""Model-level GPU tests: the fused kernels inside HuggingFace Qwen3 models.

* A bf16 Qwen3 with head_dim 128 (the tensor-core kernels): every fused
  attention call of a forward is recorded (its q, k, v and output) and the
  output is checked against the numpy oracle on those very inputs; a backward
  through the whole model gives finite gradients.
* Incremental training through DifferentiablePagedCache, as the reference's
  tests/test_paged_attention.py:197-248 does: two cached forward steps, and
  the loss gradient reaches the cache pages and the parameters.  Run at the
  reference's shape (fp16, head_dim 16) and at a tensor-core shape (bf16,
  head_dim 128).
"""

import pytest
import torch

import oracle
import hf_attention_normalizers_b200 as H
from hf_attention_normalizers_b200 import ops

from test_gpu_parity import _np, assert_close

pytestmark = pytest.mark.gpu

NORMS = ("softmax1", "sparsemax", "entmax15")


@pytest.mark.parametrize("norm", NORMS)
def test_qwen3_bf16_head_dim_128_layers_match_oracle(norm, monkeypatch):
    from transformers.models.qwen3 import Qwen3Config, Qwen3ForCausalLM

    config = Qwen3Config(vocab_size=256, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                         num_attention_heads=4, num_key_value_heads=2, head_dim=128, max_position_embeddings=512)
    torch.manual_seed(0)
    model = Qwen3ForCausalLM(config).to(device="cuda", dtype=torch.bfloat16).train()
    H.set_softmax_attention_backend(model, base_backend="sdpa", softmax_fn=norm, mode="strict")
    calls = []
    real = ops.attn_fwd

    def recording(q, k, v, *args, **kwargs):
        out = real(q, k, v, *args, **kwargs)
        calls.append((q.detach().clone(), k.detach().clone(), v.detach().clone(), out[0].detach().clone(), args))
        return out

    monkeypatch.setattr(ops, "attn_fwd", recording)
    ids = torch.randint(0, config.vocab_size, (2, 200), device="cuda")
    logits = model(ids).logits
    logits.float().square().mean().backward()
    assert len(calls) == config.num_hidden_layers
    assert all(p.grad is None or torch.isfinite(p.grad).all() for p in model.parameters())
    for layer, (q, k, v, o, args) in enumerate(calls):
        scale, causal, window, out_bshd = args[1], args[2], args[3], args[4]
        assert causal and out_bshd and window == -1
        ref = oracle.attention_forward(_np(q), _np(k), _np(v), norm, scale=scale, causal=True)
        assert_close(o.transpose(1, 2), ref, torch.bfloat16, f"qwen3/{norm}/layer {layer}")


@pytest.mark.parametrize("dtype,head_dim", [(torch.float16, 16), (torch.bfloat16, 128)])
@pytest.mark.parametrize("norm", ("sparsemax", "entmax15"))
def test_qwen3_incremental_training_with_differentiable_paged_cache(norm, dtype, head_dim):
    from transformers.models.qwen3 import Qwen3Config, Qwen3ForCausalLM

    config = Qwen3Config(vocab_size=128, hidden_size=64, intermediate_size=128, num_hidden_layers=1,
                         num_attention_heads=4, num_key_value_heads=2, head_dim=head_dim,
                         max_position_embeddings=64)
    torch.manual_seed(0)
    model = Qwen3ForCausalLM(config).to(device="cuda", dtype=dtype).train()
    H.set_softmax_attention_backend(model, base_backend="triton", softmax_fn=norm)
    cache = H.DifferentiablePagedCache(num_hidden_layers=1, block_table=torch.tensor([[0, 1], [2, 3]], device="cuda"),
                                       block_size=4, num_key_value_heads=2, head_dim=head_dim, dtype=dtype,
                                       device=torch.device("cuda"))
    model(torch.randint(0, config.vocab_size, (2, 4), device="cuda"), past_key_values=cache, use_cache=True,
          cache_position=torch.arange(4, device="cuda"))
    output = model(torch.randint(0, config.vocab_size, (2, 4), device="cuda"), past_key_values=cache,
                   use_cache=True, cache_position=torch.arange(4, 8, device="cuda")).logits
    cache.layers[0].keys.retain_grad()
    cache.layers[0].values.retain_grad()
    output.float().square().mean().backward()
    assert cache.get_seq_length() == 8
    assert torch.isfinite(output).all()
    for grad in (cache.layers[0].keys.grad, cache.layers[0].values.grad):
        assert grad is not None and torch.isfinite(grad).all()
        assert float(grad.abs().sum()) > 0.0  # the loss reaches the pages
    grads = [p.grad for p in model.parameters() if p.grad is not None]
    assert grads and all(torch.isfinite(g).all() for g in grads)
