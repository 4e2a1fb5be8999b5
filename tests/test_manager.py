"""MultiLoRAManager on the CPU: wrapping a model's target linears, PEFT-style keys,
routing of a forward (routing-only pool; the CUDA kernels are exercised in the
-m gpu tests)."""

from __future__ import annotations

import pytest
import torch

from multi_lora_b200.layers import LinearWithLoRA
from multi_lora_b200.manager import MultiLoRAManager


def test_from_model_wraps_target_suffixes():
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(hidden_size=32, intermediate_size=64, num_hidden_layers=2, num_attention_heads=2,
                      num_key_value_heads=1, vocab_size=64)
    model = LlamaForCausalLM(cfg)
    mgr = MultiLoRAManager.from_model(model, target_suffixes=("q_proj", "down_proj"), device=torch.device("cpu"),
                                      dtype=torch.float32, max_loras_per_batch=2, max_lora_rank=4)
    assert sorted(mgr.lora_wrappers) == ["layers.0.mlp.down_proj", "layers.0.self_attn.q_proj",
                                         "layers.1.mlp.down_proj", "layers.1.self_attn.q_proj"]
    assert isinstance(model.model.layers[0].self_attn.q_proj, LinearWithLoRA)
    assert isinstance(model.model.layers[0].self_attn.k_proj, torch.nn.Linear)
    assert mgr.inference_model is model


def test_manager_without_model_refuses_model_calls():
    mgr = MultiLoRAManager({}, device=torch.device("cpu"), dtype=torch.float32)
    with pytest.raises(RuntimeError):
        _ = mgr.inference_model
