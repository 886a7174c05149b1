"""The transformers quantizer plugin: a small random Llama saved with
save_pretrained and loaded with `quantization_config=TensorShrinkConfig`
streams its projections through the GPU quantizer as the checkpoint loads;
the result equals `quantize_module` applied to the same model loaded dense
(same layers replaced, bit-identical buffers and logits)."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_from_pretrained_matches_quantize_module(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from transformers import LlamaConfig, LlamaForCausalLM
    import tensorshrink_b200 as ts
    from tensorshrink_b200.hf_integration import TensorShrinkConfig
    torch.manual_seed(0)
    cfg = LlamaConfig(hidden_size=256, intermediate_size=768, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, vocab_size=1000, max_position_embeddings=128, attention_bias=True)
    LlamaForCausalLM(cfg).to(torch.float16).save_pretrained(tmp_path)

    # (no device_map: that path needs `accelerate`; the quantized layers are
    # built on the current CUDA device as the weights stream in)
    q = LlamaForCausalLM.from_pretrained(tmp_path, dtype=torch.float16,
                                         quantization_config=TensorShrinkConfig(bits=4, min_numel=1, verbose=False))
    q = q.cuda()
    dense = LlamaForCausalLM.from_pretrained(tmp_path, dtype=torch.float16).cuda()
    ts.quantize_module(dense, bits=4, min_numel=1, verbose=False)

    qa = {n: m for n, m in q.named_modules() if isinstance(m, ts.QuantLinear)}
    qb = {n: m for n, m in dense.named_modules() if isinstance(m, ts.QuantLinear)}
    assert set(qa) == set(qb) and len(qa) == 14     # 7 projections x 2 layers
    for n in qa:
        for b in ("packed", "dq_scale_codes", "dq_gmin_meta", "outlier_col", "bias"):
            x, y = getattr(qa[n], b), getattr(qb[n], b)
            assert (x is None and y is None) or torch.equal(x, y), (n, b)
    assert q.is_tensorshrink_quantized and q.tensorshrink_stats["n_replaced"] == 14
    ids = torch.randint(0, 1000, (2, 16), device="cuda")
    with torch.no_grad():
        assert torch.equal(q(ids).logits, dense(ids).logits)
