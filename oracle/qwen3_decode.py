"""CPU/fp32 restatement of the decode forward: TEST INFRASTRUCTURE ONLY.

This module is the parity oracle.  Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline leg may import it, and only to check or time
against the CUDA path; the product never routes through it.

What it restates.  The reference's oracle is its PyTorch path,
``host/validate.py:33-37`` (``reference_forward``), which runs HF
``Qwen3ForCausalLM`` (transformers 5.5.0, ``models/qwen3/modeling_qwen3.py``;
the version is unpinned in the reference, whose notebook runs
``pip install transformers`` at ``megakernel_colab.ipynb:37``).  The decode
step below follows that module for one new token with an explicit KV cache:

* RMSNorm in fp32: w * (x * rsqrt(mean(x^2) + eps)) (modeling_qwen3.py:59-64);
* q/k/v projections, per-head q_norm/k_norm before RoPE (modeling_qwen3.py:263-264,
  same order as the reference kernel, src/megakernel.cu:172-188);
* RoPE with inv_freq = 1 / theta^(arange(0, d, 2)/d) in fp32, angle = inv_freq *
  pos in fp32, cos/sin of cat(freqs, freqs), rotate_half
  (modeling_rope_utils.py:178, modeling_qwen3.py:140-151);
* GQA softmax(q k^T * d^-0.5) v in fp32 (modeling_qwen3.py:196-218);
* SwiGLU MLP down(silu(gate(x)) * up(x)) (modeling_qwen3.py:82);
* tied LM head logits = h E^T (modeling_qwen3.py:505), greedy argmax that
  returns the lowest index among equal maxima (torch.argmax).

``kv_bf16=True`` rounds K (after RoPE) and V to bf16 before they are cached and
used, which is what the kernel does: its KV cache is bf16
(src/kv_cache.cuh:9-32 layout ``[layer, 2, kv_head, max_seq, head_dim]``).  With
``kv_bf16=False`` it is the plain HF fp32 forward.  ``kv_fp8=True`` rounds
them to float8 e4m3 instead (round to nearest, saturating at +-448), the
batched decoder's optional fp8 cache.  ``w_fp8=True`` runs the matrix
products on e4m3 weights with one scale per row (max |w| / 448), as the
batched decoder's optional e4m3 weights do; the embedding lookup and the
norms keep the bf16 weights.

Parity pin: tests/test_oracle_pin.py checks this module against golden logits
that tests/golden/make_golden.py produced by running the reference's own
``reference_forward`` (host/validate.py:33-37) on HF Qwen3 in the build
container.
"""
from __future__ import annotations

import numpy as np
import torch


def rope_tables(head_dim: int, theta: float, positions: int):
    """fp32 cos/sin tables [positions, head_dim/2] computed as HF does."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64)
                                .to(dtype=torch.float) / head_dim))
    pos = torch.arange(positions, dtype=torch.float32)
    freqs = pos[:, None] * inv_freq[None, :]
    return freqs.cos(), freqs.sin()


def quant_rows_e4m3(w: torch.Tensor) -> torch.Tensor:
    """w with each row rounded to e4m3 at its own scale (max |row| / 448), dequantised to fp32."""
    amax = w.abs().amax(dim=1, keepdim=True)
    sc = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    inv = 1.0 / sc            # the kernel scales by the fp32 reciprocal, then rounds
    return (w * inv).clamp(-448, 448).to(torch.float8_e4m3fn).float() * sc


class Qwen3DecodeOracle:
    """Token-serial fp32 decode over bf16-valued weights with an explicit KV cache."""

    def __init__(self, shape, weights: dict, kv_bf16: bool = True,
                 max_seq: int = 2048, device: str = "cpu", kv_fp8: bool = False, w_fp8: bool = False):
        self.s = shape
        self.kv_bf16 = kv_bf16
        self.kv_fp8 = kv_fp8
        self.dev = torch.device(device)
        f = lambda n: weights[n].to(self.dev).float()  # noqa: E731
        # e4m3 rounding is done on the CPU (torch's CUDA cast rounded some
        # values differently from the CPU cast and the kernel's cvt.rn).
        q = lambda n: quant_rows_e4m3(weights[n].float()).to(self.dev)  # noqa: E731
        self.emb = f("embedding")
        self.lm = q("embedding") if w_fp8 else self.emb
        self.final_norm = f("final_norm")
        self.layers = []
        gemm_keys = {"w_q", "w_k", "w_v", "w_o", "w_gate", "w_up", "w_down"}
        for i in range(shape.layers):
            self.layers.append({k: (q(f"layer.{i}.{k}") if w_fp8 and k in gemm_keys else f(f"layer.{i}.{k}"))
                                for k in shape.LAYER_KEYS})
        self.max_seq = max_seq
        self.cos, self.sin = rope_tables(shape.head_dim, shape.rope_theta, max_seq)
        self.cos, self.sin = self.cos.to(self.dev), self.sin.to(self.dev)
        L, KVH, D = shape.layers, shape.kv_heads, shape.head_dim
        self.k = torch.zeros(L, KVH, max_seq, D, device=self.dev)
        self.v = torch.zeros(L, KVH, max_seq, D, device=self.dev)
        self.pos = 0

    def reset(self):
        self.k.zero_()
        self.v.zero_()
        self.pos = 0

    def set_kv(self, layer: int, k: torch.Tensor, v: torch.Tensor, start: int = 0):
        """Inject cached K (post-RoPE) / V [kv_heads, n, head_dim] at positions start.."""
        n = k.shape[1]
        self.k[layer, :, start:start + n] = k.to(self.dev).float()
        self.v[layer, :, start:start + n] = v.to(self.dev).float()

    def _rms(self, x, w):
        var = x.pow(2).mean(-1, keepdim=True)
        return w * (x * torch.rsqrt(var + self.s.rms_eps))

    def _rope(self, x, pos):
        # x [heads, D]; rotate_half pairs (i, i + D/2).
        half = x.shape[-1] // 2
        c = torch.cat([self.cos[pos], self.cos[pos]])
        sn = torch.cat([self.sin[pos], self.sin[pos]])
        rot = torch.cat([-x[:, half:], x[:, :half]], dim=-1)
        return x * c + rot * sn

    @torch.no_grad()
    def step(self, token: int) -> torch.Tensor:
        """One decode step at ``self.pos``; returns fp32 logits [vocab]."""
        s = self.s
        p = self.pos
        if p >= self.max_seq:
            raise ValueError("KV capacity exceeded")
        D, NQ, NKV = s.head_dim, s.q_heads, s.kv_heads
        grp = NQ // NKV
        x = self.emb[token].clone()
        for li, w in enumerate(self.layers):
            xn = self._rms(x, w["attn_norm"])
            q = (w["w_q"] @ xn).view(NQ, D)
            k = (w["w_k"] @ xn).view(NKV, D)
            v = (w["w_v"] @ xn).view(NKV, D)
            q = self._rms(q, w["q_norm"])
            k = self._rms(k, w["k_norm"])
            q = self._rope(q, p)
            k = self._rope(k, p)
            if self.kv_fp8:
                # rounded on the CPU, like the weights (see __init__)
                k = k.cpu().clamp(-448, 448).to(torch.float8_e4m3fn).float().to(self.dev)
                v = v.cpu().clamp(-448, 448).to(torch.float8_e4m3fn).float().to(self.dev)
            elif self.kv_bf16:
                k = k.to(torch.bfloat16).float()
                v = v.to(torch.bfloat16).float()
            self.k[li, :, p] = k
            self.v[li, :, p] = v
            K = self.k[li, :, :p + 1]                 # [NKV, p+1, D]
            V = self.v[li, :, :p + 1]
            Kq = K.repeat_interleave(grp, dim=0)      # [NQ, p+1, D]
            Vq = V.repeat_interleave(grp, dim=0)
            sc = torch.einsum("hd,hpd->hp", q, Kq) * (D ** -0.5)
            pr = torch.softmax(sc, dim=-1)
            att = torch.einsum("hp,hpd->hd", pr, Vq).reshape(-1)
            x = x + w["w_o"] @ att
            xn = self._rms(x, w["ffn_norm"])
            g = w["w_gate"] @ xn
            u = w["w_up"] @ xn
            x = x + w["w_down"] @ (torch.nn.functional.silu(g) * u)
        h = self._rms(x, self.final_norm)
        self.pos += 1
        return self.lm @ h

    def run(self, forced: list[int], n_steps: int, want_logits: bool = True):
        """Teacher-forced for len(forced) steps then greedy; mirrors megakernel_decode_n.

        Returns (argmax per step [n_steps], logits [n_steps, vocab] or None,
        top-2 margin per step).
        """
        toks, logits, margins = [], [], []
        cur = forced[0]
        for i in range(n_steps):
            inp = forced[i] if i < len(forced) else cur
            lg = self.step(inp)
            cur = int(torch.argmax(lg))
            toks.append(cur)
            t2 = torch.topk(lg, 2).values
            margins.append(float(t2[0] - t2[1]))
            if want_logits:
                logits.append(lg.cpu().numpy())
        return (np.array(toks, dtype=np.int64),
                np.stack(logits) if want_logits else None,
                np.array(margins, dtype=np.float64))
