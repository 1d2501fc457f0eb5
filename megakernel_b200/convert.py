"""Convert a Hugging Face Qwen3 checkpoint into the flat-binary weight format.

Replaces the reference's converter (host/weight_loader.py:63-206:
``extract_weights``, ``validate_shapes``, ``save_flat_binary``) and writes the
same two files: ``weights.bin`` (bf16 tensors concatenated in flat-binary
order) and ``weights_offsets.json``.  Differences: it reads a local checkpoint
directory (``config.json`` plus ``*.safetensors`` or ``pytorch_model*.bin``),
an in-memory state_dict or a model object, with no download; the model shape
comes from the checkpoint's config and must be one the kernel compiles; and
``o_proj`` is checked as [hidden, q_dim], as HF stores it (the reference's
``validate_shapes`` expects the transpose, host/weight_loader.py:128, which
only passes when the two are equal).

    python -m megakernel_b200.convert <checkpoint_dir> <out/weights.bin>
"""
from __future__ import annotations

import glob
import json
import os
import sys

import torch

from .shapes import SHAPES, Shape
from .weights import save_flat_binary

# flat-binary layer key -> HF Qwen3 parameter name (per layer)
HF_LAYER = {
    "attn_norm": "input_layernorm.weight",
    "w_q": "self_attn.q_proj.weight",
    "w_k": "self_attn.k_proj.weight",
    "w_v": "self_attn.v_proj.weight",
    "q_norm": "self_attn.q_norm.weight",
    "k_norm": "self_attn.k_norm.weight",
    "w_o": "self_attn.o_proj.weight",
    "ffn_norm": "post_attention_layernorm.weight",
    "w_gate": "mlp.gate_proj.weight",
    "w_up": "mlp.up_proj.weight",
    "w_down": "mlp.down_proj.weight",
}


def shape_from_config(cfg: dict) -> Shape:
    """The compiled model shape matching an HF Qwen3 config dict."""
    hd = cfg.get("head_dim") or cfg["hidden_size"] // cfg["num_attention_heads"]
    want = (cfg["hidden_size"], cfg["num_hidden_layers"], cfg["num_attention_heads"],
            cfg["num_key_value_heads"], hd, cfg["intermediate_size"], cfg["vocab_size"])
    for s in SHAPES.values():
        if (s.hidden, s.layers, s.q_heads, s.kv_heads, s.head_dim, s.intermediate, s.vocab) == want:
            return s
    raise ValueError(f"no compiled shape matches (hidden, layers, heads, kv_heads, head_dim, "
                     f"intermediate, vocab) = {want}")


def from_state_dict(shape: Shape, sd: dict) -> dict:
    """HF Qwen3ForCausalLM state_dict -> flat-binary name -> bf16 tensor,
    every tensor shape-checked.  The LM head must be tied to the embedding
    (absent, or equal to it), as in the kernel and the reference."""
    def get(k):
        for name in (k, k.replace("model.", "", 1)):
            if name in sd:
                return sd[name]
        raise KeyError(f"checkpoint has no {k}")

    src = {"embedding": get("model.embed_tokens.weight"), "final_norm": get("model.norm.weight")}
    for i in range(shape.layers):
        for k, hf in HF_LAYER.items():
            src[f"layer.{i}.{k}"] = get(f"model.layers.{i}.{hf}")
    lm = sd.get("lm_head.weight")
    if lm is not None and lm.data_ptr() != src["embedding"].data_ptr() and not torch.equal(
            lm.to(torch.float32), src["embedding"].to(torch.float32)):
        raise ValueError("lm_head is not tied to the embedding: the kernel computes the LM head "
                         "from the embedding matrix")
    out = {}
    for name, s in shape.tensor_shapes():
        t = src[name]
        if tuple(t.shape) != tuple(s):
            raise ValueError(f"{name}: checkpoint shape {tuple(t.shape)}, expected {tuple(s)}")
        out[name] = t.detach().to(torch.bfloat16).contiguous()
    return out


def load_checkpoint_dir(path: str) -> tuple[dict, dict]:
    """(config dict, state_dict) of a local HF checkpoint directory."""
    with open(os.path.join(path, "config.json")) as f:
        cfg = json.load(f)
    sd = {}
    files = sorted(glob.glob(os.path.join(path, "*.safetensors")))
    if files:
        from safetensors.torch import load_file
        for fn in files:
            sd.update(load_file(fn))
    else:
        files = sorted(glob.glob(os.path.join(path, "pytorch_model*.bin")))
        if not files:
            raise FileNotFoundError(f"{path}: no *.safetensors or pytorch_model*.bin")
        for fn in files:
            sd.update(torch.load(fn, map_location="cpu", weights_only=True))
    return cfg, sd


def convert(src, output_path: str):
    """Write weights.bin + weights_offsets.json from `src`: a checkpoint
    directory, an HF model object, or a (config dict, state_dict) pair.
    Returns (shape, offsets)."""
    if isinstance(src, str):
        cfg, sd = load_checkpoint_dir(src)
    elif isinstance(src, tuple):
        cfg, sd = src
    else:
        cfg, sd = src.config.to_dict(), src.state_dict()
    shape = shape_from_config(cfg)
    offsets = save_flat_binary(shape, from_state_dict(shape, sd), output_path)
    return shape, offsets


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    if len(argv) != 2:
        print(__doc__.strip().splitlines()[-1].strip(), file=sys.stderr)
        return 2
    shape, offsets = convert(argv[0], argv[1])
    print(f"{argv[1]}: {shape.name}, {len(offsets)} tensors, {shape.weight_bytes} bytes")
    return 0


if __name__ == "__main__":
    sys.exit(main())
