"""Generate the golden parity fixtures in this directory.

Run in a container where the reference tree is available (its path in the
MK_REFERENCE_ROOT environment variable, required) and ``transformers`` is
installed:

    MK_REFERENCE_ROOT=<reference checkout> python tests/golden/make_golden.py [name ...]

With names, only those fixtures are regenerated.

For each shape it builds the seeded random-init model (weights seed 0, prompt
seed 1, as BASELINE configs[0] specifies), runs the reference's greedy
generation path (``model.generate(do_sample=False)``, host/validate.py:40-52)
in fp32 to get a token sequence, then the reference's own
``reference_forward`` (host/validate.py:33-37, imported from the reference
tree) over the whole sequence to get teacher-forced logits for every
position.  Stored per position: argmax, top-2 margin, the 8 largest logits
with their ids, and the logits at a fixed random subset of vocab ids (all of
them for the tiny shape).  The bf16 HF model's greedy tokens are stored too
(information only: the parity gate is the fp32 model).

The fixtures are committed; the tests never import the reference.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from megakernel_b200 import weights as W  # noqa: E402
from megakernel_b200.shapes import QWEN3_0_6B_D64, QWEN3_0_6B_D128, TINY  # noqa: E402
from oracle.hf_reference import build_hf_model, hf_generate  # noqa: E402

CASES = [
    # fixture name, shape, prompt length, greedy tokens, stored vocab subset
    # (None = all), also record the bf16 model's greedy tokens
    ("tiny", TINY, 8, 24, None, True),
    ("qwen3-0.6b-d64", QWEN3_0_6B_D64, 16, 64, 512, True),
    ("qwen3-0.6b-d128", QWEN3_0_6B_D128, 16, 16, 512, True),
    # BASELINE configs[1] itself: 128-token prompt, 512 greedy tokens, so the
    # benchmarked positions 128..639 (1 to 5 split-KV chunks per head) are
    # pinned.  The bf16 run is skipped (information only, and slow on CPU).
    ("qwen3-0.6b-d64-c1", QWEN3_0_6B_D64, 128, 512, 256, False),
]


def main():
    ref_root = os.environ.get("MK_REFERENCE_ROOT")
    if not ref_root:
        sys.exit("set MK_REFERENCE_ROOT to the reference checkout (it holds host/validate.py)")
    sys.path.insert(0, ref_root)
    from host.validate import reference_forward  # the reference's own oracle call

    only = set(sys.argv[1:])
    torch.set_num_threads(os.cpu_count() or 1)
    for name, shape, n_prompt, n_gen, n_sub, with_bf16 in CASES:
        if only and name not in only:
            continue
        w = W.random_weights(shape, seed=0)
        prompt = W.prompt_ids(shape, n_prompt, seed=1)
        m32 = build_hf_model(shape, w, torch.float32)
        seq = hf_generate(m32, prompt, n_gen)
        with torch.no_grad():
            logits = reference_forward(m32, torch.tensor([seq]))[0].float().numpy()
        if with_bf16:
            m16 = build_hf_model(shape, w, torch.bfloat16)
            seq16 = hf_generate(m16, prompt, n_gen)
            del m16
        else:
            seq16 = []
        top = np.argsort(-logits, axis=1)[:, :8]
        topv = np.take_along_axis(logits, top, axis=1)
        if n_sub is None:
            sub = np.arange(shape.vocab)
        else:
            sub = np.sort(np.random.default_rng(3).choice(shape.vocab, n_sub, replace=False))
        out = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(
            out, seq=np.array(seq, np.int64), n_prompt=n_prompt,
            argmax=logits.argmax(1).astype(np.int64), margin=(topv[:, 0] - topv[:, 1]).astype(np.float32),
            top_ids=top.astype(np.int64), top_vals=topv.astype(np.float32),
            sub_ids=sub.astype(np.int64), sub_logits=logits[:, sub].astype(np.float32),
            seq_bf16=np.array(seq16, np.int64))
        div = next((i for i, (a, b) in enumerate(zip(seq, seq16)) if a != b), None)
        print(f"{name}: {len(seq)} positions, bf16 greedy diverges at {div}, "
              f"min margin {float((topv[:, 0] - topv[:, 1]).min()):.2e} -> {out}")


if __name__ == "__main__":
    main()
