"""Checkpoint converter (megakernel_b200.convert, replacing
host/weight_loader.py:63-206): an HF Qwen3 checkpoint written to disk in both
serialisations converts to the same flat binary as the seeded weights it was
built from, and mismatches are rejected."""
import json
import os

import numpy as np
import pytest
import torch

from megakernel_b200 import convert
from megakernel_b200 import weights as W
from megakernel_b200.shapes import QWEN3_0_6B_D128, TINY
from oracle.hf_reference import build_hf_model


def _checkpoint(tmp_path, fmt):
    w = W.random_weights(TINY, 3)
    model = build_hf_model(TINY, w, dtype=torch.bfloat16)
    d = tmp_path / fmt
    d.mkdir()
    cfg = model.config.to_dict()
    with open(d / "config.json", "w") as f:
        json.dump(cfg, f, default=str)
    sd = {k: v.contiguous() for k, v in model.state_dict().items() if k != "lm_head.weight"}
    if fmt == "safetensors":
        from safetensors.torch import save_file
        save_file(sd, str(d / "model.safetensors"))
    else:
        torch.save(sd, str(d / "pytorch_model.bin"))
    return w, str(d)


@pytest.mark.parametrize("fmt", ["safetensors", "bin"])
def test_checkpoint_dir_round_trip(tmp_path, fmt):
    w, d = _checkpoint(tmp_path, fmt)
    out = str(tmp_path / "weights.bin")
    shape, offs = convert.convert(d, out)
    assert shape is TINY
    buf, offs2 = W.load_flat_binary(out)
    assert offs2 == offs
    want, want_offs = W.flat_bytes(TINY, w)
    assert offs == want_offs and np.array_equal(buf, want)


def test_model_object_and_rejections(tmp_path):
    w = W.random_weights(TINY, 4)
    model = build_hf_model(TINY, w, dtype=torch.bfloat16)
    shape, _ = convert.convert(model, str(tmp_path / "m.bin"))
    assert shape is TINY
    sd = dict(model.state_dict())
    sd["lm_head.weight"] = sd["lm_head.weight"].clone() + 1.0
    with pytest.raises(ValueError, match="tied"):
        convert.from_state_dict(TINY, sd)
    sd = dict(model.state_dict())
    sd["model.layers.0.mlp.down_proj.weight"] = sd["model.layers.0.mlp.down_proj.weight"].t()
    with pytest.raises(ValueError, match="w_down"):
        convert.from_state_dict(TINY, sd)
    cfg = dict(model.config.to_dict())
    cfg["num_attention_heads"] = 8       # no compiled shape
    with pytest.raises(ValueError, match="no compiled shape"):
        convert.shape_from_config(cfg)


def test_real_qwen3_config_maps_to_head_dim_128_shape():
    # Qwen/Qwen3-0.6B's config.json values (the shape src/config.cuh compiles)
    cfg = dict(hidden_size=1024, num_hidden_layers=28, num_attention_heads=16, num_key_value_heads=8,
               head_dim=128, intermediate_size=3072, vocab_size=151936)
    assert convert.shape_from_config(cfg) is QWEN3_0_6B_D128
