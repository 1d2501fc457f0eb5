"""Model shapes served by the decode megakernel.

The reference hard-codes one shape in ``src/config.cuh:13-22`` (head_dim 128,
intermediate 3072) while its host code and headline numbers use head_dim 64 /
intermediate 2816 (``host/benchmark.py:29-37``, ``src/gemv.cuh:19-24``).  Both
are compiled here as template instantiations of the same kernel, plus a tiny
shape used by fast parity tests.  The CUDA side mirrors this table in
``csrc/shapes.cuh``; the shape ids below must match it.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Shape:
    name: str
    hidden: int
    layers: int
    q_heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    rope_theta: float = 1.0e6
    rms_eps: float = 1.0e-6

    @property
    def q_dim(self) -> int:
        return self.q_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim

    # --- flat-binary layout (host/weight_loader.py:141-206) -----------------
    LAYER_KEYS = ("attn_norm", "w_q", "w_k", "w_v", "q_norm", "k_norm",
                  "w_o", "ffn_norm", "w_gate", "w_up", "w_down")

    def tensor_shapes(self):
        """Ordered (name, shape) list in flat-binary order.

        Order and names follow ``save_flat_binary`` (host/weight_loader.py:141-206)
        and the offsets layout documented at src/megakernel.cu:518-532.
        ``w_o`` is [hidden, q_dim] as HF stores ``o_proj`` (the reference's
        ``validate_shapes`` check at host/weight_loader.py:128 has it transposed).
        """
        H, Q, KV, D, I, V = (self.hidden, self.q_dim, self.kv_dim, self.head_dim,
                             self.intermediate, self.vocab)
        out = [("embedding", (V, H)), ("final_norm", (H,))]
        per = {
            "attn_norm": (H,), "w_q": (Q, H), "w_k": (KV, H), "w_v": (KV, H),
            "q_norm": (D,), "k_norm": (D,), "w_o": (H, Q), "ffn_norm": (H,),
            "w_gate": (I, H), "w_up": (I, H), "w_down": (H, I),
        }
        for i in range(self.layers):
            for k in self.LAYER_KEYS:
                out.append((f"layer.{i}.{k}", per[k]))
        return out

    @property
    def num_offsets(self) -> int:
        return 2 + 11 * self.layers

    @property
    def weight_bytes(self) -> int:
        n = 0
        for _, s in self.tensor_shapes():
            c = 1
            for d in s:
                c *= d
            n += 2 * c
        return n

    def tp_weight_bytes(self, tp: int) -> int:
        """Weight bytes one GPU streams per token under tensor parallelism over
        `tp` GPUs: attention (norms, QKV, O) and the final norm replicated,
        the MLP matrices and the LM head (tied embedding) split `tp` ways."""
        mlp = 3 * 2 * self.intermediate * self.hidden * self.layers
        lm = 2 * self.vocab * self.hidden
        return self.weight_bytes - mlp - lm + (mlp + lm) // tp

    @property
    def kv_bytes_per_position(self) -> int:
        """bf16 K and V bytes for one position across all layers."""
        return 2 * self.kv_dim * 2 * self.layers

    def algorithmic_bytes(self, pos: int, batch: int = 1) -> int:
        """HBM bytes one decode step at 0-based position ``pos`` must move.

        Weights once (the embedding row gather is inside the LM-head read), plus
        per sequence the K/V of ``pos`` cached positions plus the current one
        read and the current one written: kv_bytes_per_position * (pos + 2).
        """
        return self.weight_bytes + batch * self.kv_bytes_per_position * (pos + 2)

    def hf_config_kwargs(self) -> dict:
        return dict(vocab_size=self.vocab, hidden_size=self.hidden,
                    intermediate_size=self.intermediate,
                    num_hidden_layers=self.layers,
                    num_attention_heads=self.q_heads,
                    num_key_value_heads=self.kv_heads, head_dim=self.head_dim,
                    rms_norm_eps=self.rms_eps, tie_word_embeddings=True,
                    rope_theta=self.rope_theta, max_position_embeddings=40960,
                    attention_bias=False, hidden_act="silu")


# Graded shape: BASELINE configs[0] (head_dim 64, intermediate 2816).
QWEN3_0_6B_D64 = Shape("qwen3-0.6b-d64", 1024, 28, 16, 8, 64, 2816, 151936)
# Shape that the reference's src/config.cuh:13-22 actually compiles.
QWEN3_0_6B_D128 = Shape("qwen3-0.6b-d128", 1024, 28, 16, 8, 128, 3072, 151936)
# Small shape for fast parity tests (same kernel template, same code paths).
TINY = Shape("tiny", 256, 2, 4, 2, 64, 512, 2048)

SHAPES = {s.name: s for s in (QWEN3_0_6B_D64, QWEN3_0_6B_D128, TINY)}
# Must match the shape ids in csrc/shapes.cuh.
SHAPE_IDS = {QWEN3_0_6B_D64.name: 0, QWEN3_0_6B_D128.name: 1, TINY.name: 2}
