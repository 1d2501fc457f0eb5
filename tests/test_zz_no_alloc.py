"""megakernel_decode_noalloc: decode for callers that cannot allocate device memory.

Such callers (a runtime that owns every device allocation, an allocator-free
loader, a plugin that must keep its memory footprint fixed) hand the library
only their own buffers; the entry point's scratch is a fixed array in the
library's device image.  This test calls it through the C ABI twice in a row
(prefill + greedy, then continuing from the returned position) and checks
tokens and logits against the allocating entry point, megakernel_decode_n,
within the suite's logit tolerance.  The file is named so that pytest
collects it last; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from megakernel_b200 import _lib
from megakernel_b200.bridge import MegakernelEngine
from megakernel_b200.weights import offsets_list

from ._common import LOGIT_TOL, golden, weights

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
NAME = "qwen3-0.6b-d64"


def test_noalloc_matches_allocating_entry_point_twice():
    shape, _, flat, offs = weights(NAME)
    g = golden(NAME)
    prompt = g["seq"][:int(g["n_prompt"])].tolist()
    n1, n2 = len(prompt) + 8, 6
    max_seq = 64

    # Allocating path (reference for this test): one engine, two launches.
    eng = MegakernelEngine(flat=flat, offsets=offs, shape=shape, max_seq=max_seq)
    toks = torch.tensor(prompt, dtype=torch.int32, device=DEV)
    out_a = torch.zeros(n1 + n2, dtype=torch.int32, device=DEV)
    lg_a = torch.zeros(n1 + n2, shape.vocab, device=DEV)
    eng.decode_n(toks, len(prompt), out_a[:n1], logits=lg_a[:n1])
    nxt = out_a[n1 - 1:n1].clone()
    eng.decode_n(nxt, 1, out_a[n1:], logits=lg_a[n1:])
    weights_dev = eng._gpu_buffer

    # No-allocation path: caller-owned weights, KV cache, tokens and outputs.
    L = _lib.load()
    ol = offsets_list(shape, offs)
    arr = (ctypes.c_longlong * len(ol))(*ol)
    kv = torch.zeros(shape.layers, 2, shape.kv_heads, max_seq, shape.head_dim, dtype=torch.bfloat16,
                     device=DEV)
    out_b = torch.zeros(n1 + n2, dtype=torch.int32, device=DEV)
    lg_b = torch.zeros(n1 + n2, shape.vocab, device=DEV)
    stream = torch.cuda.current_stream(DEV).cuda_stream
    rc = L.megakernel_decode_noalloc(ctypes.c_void_p(weights_dev.data_ptr()), arr, len(ol),
                                     ctypes.c_void_p(kv.data_ptr()), max_seq, 0,
                                     ctypes.c_void_p(toks.data_ptr()), len(prompt), n1,
                                     ctypes.c_void_p(out_b.data_ptr()), ctypes.c_void_p(lg_b.data_ptr()),
                                     ctypes.c_void_p(stream))
    assert rc == 0, _lib.ERRORS.get(rc, rc)
    nxt_b = out_b[n1 - 1:n1].clone()
    rc = L.megakernel_decode_noalloc(ctypes.c_void_p(weights_dev.data_ptr()), arr, len(ol),
                                     ctypes.c_void_p(kv.data_ptr()), max_seq, n1,
                                     ctypes.c_void_p(nxt_b.data_ptr()), 1, n2,
                                     ctypes.c_void_p(out_b[n1:].data_ptr()),
                                     ctypes.c_void_p(lg_b[n1:].data_ptr()), ctypes.c_void_p(stream))
    assert rc == 0, _lib.ERRORS.get(rc, rc)
    torch.cuda.synchronize()

    assert torch.equal(out_a, out_b)
    err = (lg_a - lg_b).abs().max().item()
    assert err < LOGIT_TOL, err
    # and the KV cache it wrote matches the engine's
    assert torch.equal(kv[:, :, :, :n1 + n2], eng.kv_cache()[:, :, :, :n1 + n2])

    # positions beyond the static limit are refused with a clear status
    rc = L.megakernel_decode_noalloc(ctypes.c_void_p(weights_dev.data_ptr()), arr, len(ol),
                                     ctypes.c_void_p(kv.data_ptr()), 1 << 20, 2047,
                                     ctypes.c_void_p(nxt_b.data_ptr()), 1, 2,
                                     ctypes.c_void_p(out_b.data_ptr()), None, ctypes.c_void_p(stream))
    assert rc == -4
    eng.close()
