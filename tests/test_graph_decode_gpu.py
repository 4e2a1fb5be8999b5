"""A decode step of a transformers model with the LoRA ops inside, captured in a
CUDA graph: replay equals direct execution, and capture moves no resident tensor
(multi_lora/tests/test_graph_decode.py:62-106 of the reference).

The model is a randomly initialised tiny Llama (no checkpoints here) in bf16
on cuda:0, every q/k/v/o/gate/up/down linear wrapped with LinearWithLoRA, the
RMSNorms routed through the fused kernel; two rank-4 adapters alternate over a
batch of four rows.
"""

from __future__ import annotations

import pytest
import torch

from multi_lora_b200.graph_decode import DecodeStep, capture_graph
from multi_lora_b200.manager import MultiLoRAManager
from multi_lora_b200.rmsnorm import fuse_rmsnorm
from multi_lora_b200.weights import AdapterWeights

pytestmark = pytest.mark.gpu

LOGIT_ATOL = 1e-2  # bf16 logits
CHECK_STEPS = 5
BATCH = 4
PROMPT = 6
TARGETS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


@pytest.fixture(scope="module")
def graph_mgr(cuda_dev):
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    cfg = LlamaConfig(hidden_size=128, intermediate_size=256, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, vocab_size=256, max_position_embeddings=128, rms_norm_eps=1e-6)
    model = LlamaForCausalLM(cfg).to(cuda_dev, torch.bfloat16).eval()
    mgr = MultiLoRAManager.from_model(model, target_suffixes=TARGETS, device=cuda_dev, dtype=torch.bfloat16,
                                      max_loras_per_batch=2, max_lora_rank=4)
    assert fuse_rmsnorm(model) == 2 * cfg.num_hidden_layers + 1
    for name, seed in (("a", 11), ("b", 22)):
        g = torch.Generator().manual_seed(seed)
        mods = {}
        for key, wrapper in mgr.lora_wrappers.items():
            lin = wrapper.base_layer
            mods[key] = ((torch.randn(4, lin.in_features, generator=g) * 0.2).bfloat16(),
                         (torch.randn(lin.out_features, 4, generator=g) * 0.2).bfloat16())
        mgr.register_adapter(name, AdapterWeights(rank=4, scaling=2.0, modules=mods))
    return mgr


def _prefill(mgr, ids, names, start, max_len):
    step = DecodeStep.new(mgr, BATCH, start, max_len)
    first = step.prefill(mgr, ids, torch.ones_like(ids), names)
    step.input_ids.copy_(first)
    mgr._setup_forward_batch(names, seq_lens=[1] * BATCH)
    return step, first


def _prompt(dev):
    return torch.randint(0, 256, (BATCH, PROMPT), generator=torch.Generator().manual_seed(5)).to(dev)


@torch.inference_mode()
def test_replay_matches_direct_run(graph_mgr, cuda_dev):
    mgr = graph_mgr
    ids = _prompt(cuda_dev)
    names = ["a", "b", "a", "b"]
    max_len = PROMPT + 3 + 1 + CHECK_STEPS + 2  # warm-up 3 + capture 1 + checked steps, one position each
    recorded = _prefill(mgr, ids, names, PROMPT, max_len)[0]
    graph, out = capture_graph(mgr, recorded)
    direct = _prefill(mgr, ids, names, PROMPT, max_len)[0]
    for step in range(CHECK_STEPS):
        graph.replay()
        mine = out.logits[:, -1]
        theirs = direct.run(mgr).logits[:, -1]
        gap = (mine.float() - theirs.float()).abs().max().item()
        assert gap <= LOGIT_ATOL, f"step {step}: max |diff| {gap:.4f}"
        nxt = mine.argmax(dim=-1, keepdim=True)
        recorded.input_ids.copy_(nxt)
        direct.input_ids.copy_(nxt)
    del graph


@torch.inference_mode()
def test_lora_changes_the_decode_step(graph_mgr, cuda_dev):
    """The adapters are live inside the captured step: base-only routing differs."""
    mgr = graph_mgr
    ids = _prompt(cuda_dev)
    step, _ = _prefill(mgr, ids, ["a", "b", "a", "b"], PROMPT, PROMPT + 4)
    with_lora = step.run(mgr).logits[:, -1].float().clone()
    base, _ = _prefill(mgr, ids, [None] * BATCH, PROMPT, PROMPT + 4)
    base.input_ids.copy_(step.input_ids)
    base_logits = base.run(mgr).logits[:, -1].float()
    assert (with_lora - base_logits).abs().max().item() > 1e-2


@torch.inference_mode()
def test_capture_reuses_same_tensors(graph_mgr, cuda_dev):
    mgr = graph_mgr
    ids = _prompt(cuda_dev)
    step, _ = _prefill(mgr, ids, ["a", "b", "a", "b"], PROMPT, PROMPT + 8)
    tensors = lambda: (step.kv.layers[0].keys, step.input_ids, step.position_ids, step.kv_pos,  # noqa: E731
                       step.attn_mask, mgr._resident_meta.seg_indptr, mgr._resident_meta.weight_indices)
    before = [t.data_ptr() for t in tensors()]
    graph, _ = capture_graph(mgr, step)
    assert before == [t.data_ptr() for t in tensors()]
    del graph
