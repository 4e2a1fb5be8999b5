"""A model decode step with the LoRA ops inside it, captured once into a CUDA graph.

Drop-in for ``multi_lora/graph_decode.py:24-111``. A decode step can be
captured only if every tensor it touches keeps its address and shape from
step to step, so the KV cache is a ``StaticCache`` allocated once, and the
attention mask, positions and KV write index are resident tensors advanced in
place inside the graph; only their contents change between replays. The
LoRA side meets the same rule by construction: the routing tables are
rewritten in place (``write_kernel_input_metadata``), the backend's ``mid``
buffer is resident, and no ``torch.ops.mlora`` op allocates or synchronises.

    step = DecodeStep.new(mgr, batch, start, max_len)
    first = step.prefill(mgr, input_ids, attention_mask, lora_names)
    step.input_ids.copy_(first)
    graph, out = capture_graph(mgr, step)      # then graph.replay() per step
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from transformers import StaticCache

WARMUP_ROUNDS = 3  # eager steps before the capture: one-time setup (library handles, workspaces) happens there


@dataclass
class DecodeStep:
    """Every tensor one decode step touches; addresses fixed once built."""

    kv: StaticCache             # KV cache of max_len positions
    input_ids: torch.Tensor     # (batch, 1) the token fed this step
    position_ids: torch.Tensor  # (batch, 1) rotary positions
    kv_pos: torch.Tensor        # (1,) KV position written this step
    attn_mask: torch.Tensor     # (batch, 1, 1, max_len) visible KV positions
    grid: torch.Tensor          # (max_len,) 0..max_len-1, for the mask
    batch: int
    start: int                  # first position after the prefill; rewind target
    max_len: int

    @classmethod
    def new(cls, mgr, batch: int, start: int, max_len: int) -> "DecodeStep":
        """An empty cache, positions at ``start``; the caller fills ``input_ids``."""
        dev = mgr.pool.device
        return cls(
            kv=StaticCache(config=mgr.inference_model.config, max_cache_len=max_len),
            input_ids=torch.zeros((batch, 1), device=dev, dtype=torch.long),
            position_ids=torch.full((batch, 1), start, device=dev, dtype=torch.long),
            kv_pos=torch.tensor([start], device=dev, dtype=torch.long),
            attn_mask=torch.zeros((batch, 1, 1, max_len), device=dev, dtype=torch.bool),
            grid=torch.arange(max_len, device=dev, dtype=torch.long),
            batch=batch,
            start=start,
            max_len=max_len,
        )

    def like_new(self, mgr) -> "DecodeStep":
        """Another set of the same shape: empty cache, positions at ``start``."""
        return DecodeStep.new(mgr, self.batch, self.start, self.max_len)

    def rewind(self) -> None:
        """Write index and positions back to ``start``. Stale KV entries past it
        need no clearing: each step overwrites the position it attends up to."""
        for layer in self.kv.layers:
            layer.cumulative_length.fill_(self.start)
        self.position_ids.fill_(self.start)
        self.kv_pos.fill_(self.start)

    def prefill(self, mgr, input_ids, attention_mask, lora_names) -> torch.Tensor:
        """Run the prompt through the model (filling KV positions [0, start)) and
        return the next token per row, (batch, 1)."""
        out = mgr.forward_with_lora(input_ids=input_ids, attention_mask=attention_mask, lora_names=lora_names,
                                    seq_lens=[int(input_ids.shape[1])] * self.batch, past_key_values=self.kv,
                                    use_cache=True)
        return out.logits[:, -1].argmax(dim=-1, keepdim=True)

    def run(self, mgr):
        """One decode step: refresh the mask, forward (writing KV), advance positions."""
        self.attn_mask.copy_((self.grid <= self.kv_pos).view(1, 1, 1, -1))
        out = mgr.inference_model(input_ids=self.input_ids, attention_mask=self.attn_mask,
                                  position_ids=self.position_ids, past_key_values=self.kv,
                                  cache_position=self.kv_pos, use_cache=True)
        self.position_ids.add_(1)
        self.kv_pos.add_(1)
        return out


def capture_graph(mgr, step: DecodeStep):
    """Warm up on a side stream with a second cache, capture one step, return
    ``(graph, captured output)``. The capture runs the step once, so ``step``
    is rewound before returning."""
    warm = step.like_new(mgr)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(WARMUP_ROUNDS):
            warm.run(mgr)
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = step.run(mgr)
    step.rewind()
    return graph, out
