"""Small, bounded launches of the decode kernels for profilers (ncu).

    python -m megakernel_b200.profile_case b1 --tokens 2 [--pos 0]
        batch-1 decode megakernel: one launch decoding `tokens` tokens from
        position `pos` (d64 shape, seeded random weights); ~1 GB on the device.
    python -m megakernel_b200.profile_case batch --batch 64 --pos 1024 --steps 1
        batched decode: `steps` steps of `batch` sequences at position `pos`
        (KV capacity pos + 16, so 64 x 1040 positions hold ~3.8 GB of cache).

Weights are the benchmark's (bf16 N(0, 0.02), seed 0).  Exits 0 on success.
"""
from __future__ import annotations

import argparse

import torch

from . import weights as W
from .shapes import QWEN3_0_6B_D64


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["b1", "batch"])
    ap.add_argument("--tokens", type=int, default=2)
    ap.add_argument("--pos", type=int, default=0)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--steps", type=int, default=1)
    a = ap.parse_args()
    shape = QWEN3_0_6B_D64
    flat, offs = W.flat_bytes(shape, W.random_weights(shape, 0))
    dev = torch.device("cuda", 0)
    if a.case == "b1":
        from .bridge import MegakernelEngine
        eng = MegakernelEngine(flat=flat, offsets=offs, shape=shape, max_seq=a.pos + a.tokens + 8)
        eng.set_pos(a.pos)
        toks = torch.ones(1, dtype=torch.int32, device=dev)
        out = torch.zeros(a.tokens, dtype=torch.int32, device=dev)
        eng.decode_n(toks, 1, out, n_steps=a.tokens)
        eng.close()
    else:
        from .batch import BatchDecoder
        bd = BatchDecoder(flat, offs, batch=a.batch, max_seq=a.pos + a.steps + 16)
        bd.set_pos([a.pos] * a.batch)
        f = torch.randint(0, shape.vocab, (1, a.batch), generator=torch.Generator().manual_seed(1))
        bd.decode_n(f.to(dev, torch.int32), a.steps)
        bd.close()
    torch.cuda.synchronize()
    print("ok")


if __name__ == "__main__":
    main()
