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


def _call(L, w, arr, n_off, kv, kv_max, pos, toks, n_forced, n_steps, out, lg, stream):
    return L.megakernel_decode_noalloc(ctypes.c_void_p(w), arr, n_off, ctypes.c_void_p(kv), kv_max, pos,
                                       ctypes.c_void_p(toks), n_forced, n_steps, ctypes.c_void_p(out),
                                       ctypes.c_void_p(lg) if lg else None, ctypes.c_void_p(stream))


def test_noalloc_long_context_allocates_nothing():
    """From position 1,900 (15 split-KV chunks per head, the two-level merge)
    on a cache prefix both paths share, twice in a row, against the
    allocating path run with the direct merge (so the direct merge's
    multi-group loop is compared too).  Device memory in use is unchanged
    across the calls, and refused calls (misaligned KV, capacity) leave no
    state behind."""
    shape, _, flat, offs = weights(NAME)
    P0, n = 1900, 6
    max_seq = 2048
    eng = MegakernelEngine(flat=flat, offsets=offs, shape=shape, max_seq=max_seq, timeout_ns=2_000_000_000)
    gen = torch.Generator().manual_seed(5)
    prefix = torch.randn(shape.layers, 2, shape.kv_heads, P0, shape.head_dim, generator=gen).to(torch.bfloat16)
    eng.kv_cache()[:, :, :, :P0] = prefix.to(DEV)
    kv = torch.zeros(shape.layers, 2, shape.kv_heads, max_seq, shape.head_dim, dtype=torch.bfloat16, device=DEV)
    kv[:, :, :, :P0] = prefix.to(DEV)
    torch.cuda.synchronize()
    seq = golden(NAME)["seq"][:2 * n].tolist()
    toks = torch.tensor(seq, dtype=torch.int32, device=DEV)

    eng.set_merge_mode(1)
    eng.set_pos(P0)
    out_a = torch.zeros(2 * n, dtype=torch.int32, device=DEV)
    lg_a = torch.zeros(2 * n, shape.vocab, device=DEV)
    eng.decode_n(toks[:n], n, out_a[:n], logits=lg_a[:n])
    eng.decode_n(toks[n:], n, out_a[n:], logits=lg_a[n:])
    eng.set_merge_mode(0)

    L = _lib.load()
    ol = offsets_list(shape, offs)
    arr = (ctypes.c_longlong * len(ol))(*ol)
    w = eng._gpu_buffer.data_ptr()
    out_b = torch.zeros(2 * n, dtype=torch.int32, device=DEV)
    lg_b = torch.zeros(2 * n, shape.vocab, device=DEV)
    stream = torch.cuda.current_stream(DEV).cuda_stream
    # The first call sets the device up (symbol address, kernel attributes,
    # RoPE tables); memory in use is measured after it.
    rc = _call(L, w, arr, len(ol), kv.data_ptr(), max_seq, P0, toks.data_ptr(), n, n,
               out_b.data_ptr(), lg_b.data_ptr(), stream)
    assert rc == 0, _lib.ERRORS.get(rc, rc)
    torch.cuda.synchronize()
    used0 = torch.cuda.memory_allocated(DEV)
    free0, _ = torch.cuda.mem_get_info(DEV)
    # misaligned KV pointer: refused before any launch
    assert _call(L, w, arr, len(ol), kv.data_ptr() + 2, max_seq, P0 + n, toks[n:].data_ptr(), n, n,
                 out_b[n:].data_ptr(), None, stream) == -1
    rc = _call(L, w, arr, len(ol), kv.data_ptr(), max_seq, P0 + n, toks[n:].data_ptr(), n, n,
               out_b[n:].data_ptr(), lg_b[n:].data_ptr(), stream)
    assert rc == 0, _lib.ERRORS.get(rc, rc)
    # capacity refusal, then a call without logits still runs clean
    assert _call(L, w, arr, len(ol), kv.data_ptr(), max_seq, 2047, toks.data_ptr(), 1, 2,
                 out_b.data_ptr(), None, stream) == -4
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated(DEV) == used0
    free1, _ = torch.cuda.mem_get_info(DEV)
    assert free1 == free0

    assert torch.equal(out_a, out_b)
    err = (lg_a - lg_b).abs().max().item()
    assert err < LOGIT_TOL, err
    # The prefix is untouched; the appended K/V agree to bf16 rounding (the
    # two merges sum the chunks in different orders).
    ref_kv = eng.kv_cache()
    assert torch.equal(kv[:, :, :, :P0], ref_kv[:, :, :, :P0])
    d = (kv[:, :, :, P0:P0 + 2 * n].float() - ref_kv[:, :, :, P0:P0 + 2 * n].float()).abs().max().item()
    assert d < 0.1, d
    tail = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc = _call(L, w, arr, len(ol), kv.data_ptr(), max_seq, P0 + 2 * n, out_b[-1:].data_ptr(), 1, 1,
               tail.data_ptr(), None, stream)
    assert rc == 0
    eng.close()
