"""The reference's PyTorch path on our flat-binary weights: TEST/BASELINE ONLY.

The reference validates and benchmarks against HF ``Qwen3ForCausalLM``
(host/validate.py:20-52, host/benchmark.py:59-77).  Its ``get_reference_model``
downloads a checkpoint, which cannot work offline, so this module builds the
same HF model class from a random-init ``Qwen3Config`` and loads the flat-binary
weights into it by inverting the name map of ``extract_weights``
(host/weight_loader.py:63-110).

Used by tests/golden/make_golden.py (golden vectors), the CPU parity pin tests
and ``bench.py --impl reference`` / the ``cpu_baseline`` leg (greedy
``model.generate`` on the host cores, as host/validate.py:40-52 runs it).
Never imported by the product.
"""
from __future__ import annotations

import torch

HF_NAME = {
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


def hf_state_dict(shape, weights: dict, dtype=torch.float32) -> dict:
    """Flat-binary tensor dict -> HF Qwen3ForCausalLM state_dict (inverse of
    host/weight_loader.py:63-110)."""
    sd = {"model.embed_tokens.weight": weights["embedding"].to(dtype),
          "model.norm.weight": weights["final_norm"].to(dtype),
          "lm_head.weight": weights["embedding"].to(dtype)}
    for i in range(shape.layers):
        for k, hf in HF_NAME.items():
            sd[f"model.layers.{i}.{hf}"] = weights[f"layer.{i}.{k}"].to(dtype)
    return sd


def build_hf_model(shape, weights: dict, dtype=torch.float32):
    """HF Qwen3ForCausalLM with the flat-binary weights, eval mode, eager attention."""
    from transformers import Qwen3Config, Qwen3ForCausalLM

    cfg = Qwen3Config(**shape.hf_config_kwargs())
    cfg._attn_implementation = "eager"
    with torch.device("meta"):
        model = Qwen3ForCausalLM(cfg)
    model = model.to_empty(device="cpu")
    missing, unexpected = model.load_state_dict(hf_state_dict(shape, weights, dtype),
                                                strict=False, assign=True)
    missing = [m for m in missing if "rotary_emb" not in m]
    if missing or unexpected:
        raise RuntimeError(f"state_dict mismatch: missing={missing} unexpected={unexpected}")
    model.tie_weights()
    # Rotary inv_freq buffers were created on meta; recompute them for real.
    rot = model.model.rotary_emb
    inv, _ = rot.compute_default_rope_parameters(cfg, device="cpu")
    model.to(dtype)
    rot.inv_freq = inv
    rot.original_inv_freq = inv.clone()
    model.eval()
    return model


@torch.no_grad()
def hf_generate(model, ids: list[int], max_new_tokens: int) -> list[int]:
    """Greedy generation as host/validate.py:40-52 runs it (do_sample=False)."""
    inp = torch.tensor([ids])
    out = model.generate(inp, attention_mask=torch.ones_like(inp),
                         max_new_tokens=max_new_tokens, min_new_tokens=max_new_tokens,
                         do_sample=False, pad_token_id=0, eos_token_id=None)
    return out[0].tolist()


@torch.no_grad()
def hf_forward_logits(model, ids: list[int]) -> torch.Tensor:
    """All-position logits [T, vocab] in fp32, as host/validate.py:33-37 returns them."""
    return model(torch.tensor([ids])).logits[0].float()
