"""Flat-binary weight format and the seeded synthetic weights.

File format (unchanged from the reference so existing ``weights.bin`` files
load as they are):

* ``weights.bin``: every tensor as raw little-endian bf16, concatenated in the
  order of ``Shape.tensor_shapes()`` with no padding
  (host/weight_loader.py:141-206, ``save_flat_binary``).
* ``weights_offsets.json``: ``{name: byte offset}`` for every tensor, same key
  names as the reference (``embedding``, ``final_norm``, ``layer.{i}.{key}``).
* The C ABI takes the offsets as a ``long long[2 + 11 * layers]`` array in the
  order built by host/bridge.py:89-96.

Synthetic weights (no checkpoint is available offline): every matrix and the
embedding are bf16(N(0, 0.02)) drawn from one ``torch.Generator`` seeded with
``seed`` in flat-binary order; all norm gains are 1.0 and draw nothing.
"""
from __future__ import annotations

import json
import os

import numpy as np
import torch

from .shapes import Shape

NORM_KEYS = ("final_norm", "attn_norm", "ffn_norm", "q_norm", "k_norm")


def _is_norm(name: str) -> bool:
    return name.split(".")[-1] in NORM_KEYS


def random_weights(shape: Shape, seed: int = 0, std: float = 0.02) -> dict:
    """Seeded bf16 weights as a name -> CPU bf16 tensor dict (flat-binary order)."""
    g = torch.Generator().manual_seed(seed)
    out = {}
    for name, s in shape.tensor_shapes():
        if _is_norm(name):
            out[name] = torch.ones(s, dtype=torch.bfloat16)
        else:
            t = torch.empty(s, dtype=torch.float32)
            t.normal_(0.0, std, generator=g)
            out[name] = t.to(torch.bfloat16)
    return out


def flat_bytes(shape: Shape, weights: dict) -> tuple[np.ndarray, dict]:
    """Pack ``weights`` into one uint8 array plus the ``{name: offset}`` dict."""
    total = shape.weight_bytes
    buf = np.empty(total, dtype=np.uint8)
    offsets = {}
    cur = 0
    for name, s in shape.tensor_shapes():
        t = weights[name]
        if tuple(t.shape) != tuple(s):
            raise ValueError(f"{name}: shape {tuple(t.shape)} != {s}")
        raw = t.contiguous().view(torch.uint16).numpy().view(np.uint8).reshape(-1)
        offsets[name] = cur
        buf[cur:cur + raw.size] = raw
        cur += raw.size
    assert cur == total
    return buf, offsets


def save_flat_binary(shape: Shape, weights: dict, output_path: str) -> dict:
    """Write ``weights.bin`` + ``*_offsets.json`` exactly like the reference."""
    buf, offsets = flat_bytes(shape, weights)
    buf.tofile(output_path)
    offsets_path = output_path.replace(".bin", "_offsets.json")
    with open(offsets_path, "w") as f:
        json.dump(offsets, f, indent=2)
    return offsets


def offsets_list(shape: Shape, offsets: dict) -> list[int]:
    """Ordered offsets for the C ABI (host/bridge.py:89-96)."""
    out = [offsets["embedding"], offsets["final_norm"]]
    for i in range(shape.layers):
        for k in Shape.LAYER_KEYS:
            out.append(offsets[f"layer.{i}.{k}"])
    return out


def load_flat_binary(weights_path: str, offsets_path: str | None = None):
    """Read a flat binary + offsets JSON from disk: (uint8 array, offsets dict)."""
    if offsets_path is None:
        offsets_path = weights_path.replace(".bin", "_offsets.json")
    with open(offsets_path) as f:
        offsets = json.load(f)
    data = np.fromfile(weights_path, dtype=np.uint8)
    return data, offsets


def unpack(shape: Shape, buf: np.ndarray, offsets: dict) -> dict:
    """Inverse of ``flat_bytes``: name -> bf16 tensors copied out of ``buf``."""
    out = {}
    for name, s in shape.tensor_shapes():
        n = 1
        for d in s:
            n *= d
        o = offsets[name]
        raw = np.ascontiguousarray(buf[o:o + 2 * n]).view(np.int16).copy()
        out[name] = torch.from_numpy(raw).view(torch.bfloat16).reshape(s)
    return out


def synthetic_flat(shape: Shape, seed: int = 0, cache_dir: str | None = None):
    """Seeded weights as (uint8 flat array, offsets dict), optionally cached on disk."""
    if cache_dir:
        os.makedirs(cache_dir, exist_ok=True)
        path = os.path.join(cache_dir, f"{shape.name}_seed{seed}.bin")
        if os.path.exists(path) and os.path.getsize(path) == shape.weight_bytes:
            return load_flat_binary(path)
        w = random_weights(shape, seed)
        save_flat_binary(shape, w, path)
        return load_flat_binary(path)
    w = random_weights(shape, seed)
    return flat_bytes(shape, w)


def prompt_ids(shape: Shape, n: int, seed: int = 1) -> list[int]:
    """Uniform-random prompt token ids from ``torch.Generator`` seeded ``seed``."""
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, shape.vocab, (n,), generator=g).tolist()
