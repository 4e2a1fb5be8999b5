"""PEFT adapter directories (adapter_config.json + adapter_model.safetensors) read
without ``peft``: module keys, scaling and the reference's one-rank rule
(multi_lora/weights.py:36-68). The directories are written in the format
``save_pretrained`` produces (tensor names ``<module>.lora_A.weight`` /
``.lora_B.weight`` under ``base_model.model.``). CPU only."""

from __future__ import annotations

import json
import math

import pytest
import torch
from safetensors.torch import save_file

from multi_lora_b200.layers import LinearWithLoRA
from multi_lora_b200.manager import MultiLoRAManager
from multi_lora_b200.peft_io import load_adapter_dir, save_adapter_dir
from multi_lora_b200.weights import AdapterWeights

MODS = {"model.layers.0.self_attn.q_proj": (32, 48), "model.layers.0.mlp.down_proj": (64, 32)}  # (in, out)


def _write(tmp, r=8, alpha=16, rslora=False, extra_cfg=None, drop_b=False, bad_rank=False):
    g = torch.Generator().manual_seed(r)
    state, want = {}, {}
    for key, (n_in, n_out) in MODS.items():
        ra = r + 1 if bad_rank and "down" in key else r
        a, b = torch.randn(ra, n_in, generator=g), torch.randn(n_out, ra, generator=g)
        state[f"base_model.model.{key}.lora_A.weight"] = a
        if not (drop_b and "down" in key):
            state[f"base_model.model.{key}.lora_B.weight"] = b
        want[key] = (a, b)
    save_file(state, str(tmp / "adapter_model.safetensors"))
    cfg = {"peft_type": "LORA", "r": r, "lora_alpha": alpha, "use_rslora": rslora,
           "target_modules": ["q_proj", "down_proj"], **(extra_cfg or {})}
    (tmp / "adapter_config.json").write_text(json.dumps(cfg))
    return want


def test_load_keys_shapes_and_scaling(tmp_path):
    want = _write(tmp_path, r=8, alpha=16)
    w = load_adapter_dir(tmp_path)
    assert w.rank == 8 and w.scaling == 2.0 and not w.flattened
    assert set(w.modules) == set(MODS)  # "base_model.model." stripped, as normalize_module_key does
    for key, (a, b) in want.items():
        assert torch.equal(w.modules[key][0], a) and torch.equal(w.modules[key][1], b)
    w16 = load_adapter_dir(tmp_path, dtype=torch.bfloat16)
    assert w16.modules[next(iter(MODS))][0].dtype == torch.bfloat16


def test_rslora_scaling(tmp_path):
    _write(tmp_path, r=16, alpha=32, rslora=True)
    assert load_adapter_dir(tmp_path).scaling == pytest.approx(32 / math.sqrt(16))


def test_one_rank_per_adapter_and_pairing(tmp_path):
    (tmp_path / "a").mkdir()
    _write(tmp_path / "a", bad_rank=True)
    with pytest.raises(ValueError, match="rank mismatch"):
        load_adapter_dir(tmp_path / "a")
    (tmp_path / "b").mkdir()
    _write(tmp_path / "b", drop_b=True)
    with pytest.raises(ValueError, match="no matching"):
        load_adapter_dir(tmp_path / "b")
    (tmp_path / "c").mkdir()
    _write(tmp_path / "c", extra_cfg={"rank_pattern": {"down_proj": 4}})
    with pytest.raises(ValueError, match="rank_pattern"):
        load_adapter_dir(tmp_path / "c")
    with pytest.raises(FileNotFoundError):
        load_adapter_dir(tmp_path / "missing")


def test_save_load_round_trip(tmp_path):
    g = torch.Generator().manual_seed(4)
    mods = {k: (torch.randn(4, i, generator=g), torch.randn(o, 4, generator=g)) for k, (i, o) in MODS.items()}
    w = AdapterWeights(rank=4, scaling=0.5, modules=mods)
    back = load_adapter_dir(save_adapter_dir(w, tmp_path / "rt"))
    assert back.rank == 4 and back.scaling == 0.5
    for k in mods:
        assert torch.equal(back.modules[k][0], mods[k][0]) and torch.equal(back.modules[k][1], mods[k][1])


def test_manager_load_adapter(tmp_path):
    _write(tmp_path, r=8, alpha=8)
    lin = torch.nn.Linear(32, 48, bias=False)
    mgr = MultiLoRAManager({"model.layers.0.self_attn.q_proj": LinearWithLoRA(lin)}, device=torch.device("cpu"),
                           dtype=torch.float32, max_loras_per_batch=2, max_lora_rank=8)
    w = mgr.load_adapter("tuned", tmp_path)
    assert w.scaling == 1.0
    info = mgr.prepare_lora_batch(["tuned", None])
    assert info.lora_ranks[info.weight_indices[0]] == 8
