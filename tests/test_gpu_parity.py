"""GPU parity: the CUDA megakernel (through the C ABI) against the golden
vectors of the reference's fp32 forward and against the fp32 oracle.

Gates: logits within 2e-2 max-abs of the fp32
reference; argmax equal wherever the reference's top-2 margin exceeds 1e-2;
free-running greedy tokens equal up to the first low-margin step.
"""
import ctypes

import numpy as np
import pytest
import torch

from megakernel_b200 import _lib
from megakernel_b200.bridge import MegakernelEngine
from oracle.qwen3_decode import Qwen3DecodeOracle

from ._common import LOGIT_TOL, MARGIN, golden, weights

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
_ENGINES = {}


def engine(name):
    if name not in _ENGINES:
        shape, _, flat, offs = weights(name)
        _ENGINES[name] = MegakernelEngine(flat=flat, offsets=offs, shape=shape, max_seq=1024,
                                          timeout_ns=2_000_000_000)
    eng = _ENGINES[name]
    eng.reset()
    return eng


def teacher_forced(eng, seq):
    n = len(seq)
    toks = torch.tensor(seq, dtype=torch.int32, device=DEV)
    out = torch.zeros(n, dtype=torch.int32, device=DEV)
    lg = torch.zeros(n, eng.vocab, dtype=torch.float32, device=DEV)
    eng.decode_n(toks, n, out, logits=lg)
    return out.cpu().numpy(), lg.cpu().numpy()


@pytest.mark.parametrize("name", ["tiny", "qwen3-0.6b-d64", "qwen3-0.6b-d128"])
def test_teacher_forced_logits_vs_reference(name):
    g = golden(name)
    eng = engine(name)
    toks, lg = teacher_forced(eng, g["seq"].tolist())
    err_sub = np.abs(lg[:, g["sub_ids"]] - g["sub_logits"]).max()
    top = np.take_along_axis(lg, g["top_ids"], axis=1)
    err_top = np.abs(top - g["top_vals"]).max()
    assert err_sub < LOGIT_TOL and err_top < LOGIT_TOL, (err_sub, err_top)
    ok = g["margin"] > MARGIN
    assert np.array_equal(toks[ok], g["argmax"][ok])


@pytest.mark.parametrize("name", ["tiny", "qwen3-0.6b-d64"])
def test_free_running_greedy_vs_reference(name):
    g = golden(name)
    eng = engine(name)
    n_prompt = int(g["n_prompt"])
    seq = g["seq"]
    n = len(seq) - 1
    toks = torch.tensor(seq[:n_prompt].tolist(), dtype=torch.int32, device=DEV)
    out = torch.zeros(n, dtype=torch.int32, device=DEV)
    eng.decode_n(toks, n_prompt, out, n_steps=n)
    got = out.cpu().numpy()[n_prompt - 1:]
    want = seq[n_prompt:]
    # equal up to the first step whose reference margin is <= 1e-2
    low = np.nonzero(g["margin"][n_prompt - 1:-1] <= MARGIN)[0]
    upto = int(low[0]) if low.size else len(want)
    assert np.array_equal(got[:upto], want[:upto]), (got[:upto], want[:upto])


def test_tiny_vs_oracle_with_bf16_kv():
    """Same arithmetic as the oracle with bf16 K/V: only fp32 summation order differs."""
    shape, w, _, _ = weights("tiny")
    g = golden("tiny")
    seq = g["seq"].tolist()
    eng = engine("tiny")
    toks, lg = teacher_forced(eng, seq)
    o = Qwen3DecodeOracle(shape, w, kv_bf16=True, max_seq=64)
    otoks, olg, _ = o.run(seq, len(seq))
    assert np.abs(lg - olg).max() < 1e-4
    assert np.array_equal(toks, otoks)


def test_deterministic_and_split_launches():
    """Bit-identical logits across runs; n steps in one launch == in pieces."""
    g = golden("tiny")
    seq = g["seq"].tolist()
    eng = engine("tiny")
    t1, l1 = teacher_forced(eng, seq)
    eng.reset()
    t2, l2 = teacher_forced(eng, seq)
    assert np.array_equal(l1, l2) and np.array_equal(t1, t2)
    eng.reset()
    parts = []
    for a in range(0, len(seq), 5):
        chunk = seq[a:a + 5]
        toks = torch.tensor(chunk, dtype=torch.int32, device=DEV)
        out = torch.zeros(len(chunk), dtype=torch.int32, device=DEV)
        lg = torch.zeros(len(chunk), eng.vocab, device=DEV)
        eng.decode_n(toks, len(chunk), out, logits=lg)
        parts.append(lg.cpu().numpy())
    assert np.abs(np.concatenate(parts) - l1).max() < 1e-5
    assert eng.pos == len(seq)


def test_reference_abi_decode_loop():
    """megakernel_init/decode/reset/get_pos/free exactly as host/bridge.py drives them."""
    shape, _, flat, offs = weights("tiny")
    from megakernel_b200.weights import offsets_list
    L = _lib.load()
    buf = torch.from_numpy(flat).to(DEV)
    ol = offsets_list(shape, offs)
    arr = (ctypes.c_longlong * len(ol))(*ol)
    h = L.megakernel_init(ctypes.c_void_p(buf.data_ptr()), arr, len(ol))
    assert h
    g = golden("tiny")
    seq = g["seq"].tolist()
    outs = []
    for t in seq[:12]:
        outs.append(L.megakernel_decode(h, t))
    assert L.megakernel_get_pos(h) == 12
    ok = g["margin"][:12] > MARGIN
    assert np.array_equal(np.array(outs)[ok], g["argmax"][:12][ok])
    L.megakernel_reset(h)
    assert L.megakernel_get_pos(h) == 0
    assert L.megakernel_decode(h, seq[0]) == outs[0]
    assert L.megakernel_decode(h, shape.vocab) == -1          # out-of-range token
    assert L.megakernel_last_error(h) == -1
    L.megakernel_sync()
    L.megakernel_free(h)


def test_generate_host_buffers_and_logits_capture():
    g = golden("tiny")
    eng = engine("tiny")
    n_prompt = int(g["n_prompt"])
    prompt = g["seq"][:n_prompt].tolist()
    out = eng.generate_ids(prompt, 10)
    eng.reset()
    toks = torch.tensor(prompt, dtype=torch.int32, device=DEV)
    dev_out = torch.zeros(n_prompt + 9, dtype=torch.int32, device=DEV)
    eng.decode_n(toks, n_prompt, dev_out)
    assert out == dev_out.cpu().tolist()[n_prompt - 1:]
    eng.reset()
    eng.set_logits_capture(True)
    t = eng.decode_token(prompt[0])
    lg = eng.logits()
    eng.set_logits_capture(False)
    assert int(np.argmax(lg)) == t
    assert abs(lg[g["sub_ids"]] - g["sub_logits"][0]).max() < LOGIT_TOL


def test_capacity_and_argument_errors():
    eng = engine("tiny")
    eng.set_pos(1020)
    toks = torch.ones(8, dtype=torch.int32, device=DEV)
    out = torch.zeros(8, dtype=torch.int32, device=DEV)
    with pytest.raises(RuntimeError, match="capacity"):
        eng.decode_n(toks, 8, out)
    assert eng.pos == 1020
    with pytest.raises(RuntimeError):
        eng.set_pos(1024)
    eng.reset()
    with pytest.raises(RuntimeError, match="invalid"):
        eng.decode_n(toks, 9, out, n_steps=8)


def test_kv_cache_layout_and_injection():
    """K/V land at [layer, 0/1, kv_head, pos, :] (src/kv_cache.cuh:26-32 layout);
    a cache injected through kv_cache() + set_pos continues like a decoded one."""
    shape, w, _, _ = weights("tiny")
    g = golden("tiny")
    seq = g["seq"].tolist()
    eng = engine("tiny")
    _, lg_ref = teacher_forced(eng, seq[:12])
    kv = eng.kv_cache()
    saved = kv[:, :, :, :11].clone()
    assert torch.count_nonzero(kv[:, :, :, 12:]) == 0
    o = Qwen3DecodeOracle(shape, w, kv_bf16=True, max_seq=64)
    o.run(seq[:12], 12)
    assert torch.allclose(kv[:, 0, :, :12].float().cpu(), o.k[:, :, :12], atol=2e-2)
    assert torch.allclose(kv[:, 1, :, :12].float().cpu(), o.v[:, :, :12], atol=2e-2)
    eng.reset()
    kv = eng.kv_cache()
    kv[:, :, :, :11] = saved
    torch.cuda.synchronize()
    eng.set_pos(11)
    toks = torch.tensor(seq[11:12], dtype=torch.int32, device=DEV)
    out = torch.zeros(1, dtype=torch.int32, device=DEV)
    lg = torch.zeros(1, eng.vocab, device=DEV)
    eng.decode_n(toks, 1, out, logits=lg)
    assert np.abs(lg.cpu().numpy()[0] - lg_ref[11]).max() < 1e-4


def test_timeout_reports_error_and_handle_recovers():
    """A CTA that never publishes its layer-0 output (test hook): every other
    CTA's bounded wait expires, the call returns MK_ERR_TIMEOUT, no hang."""
    shape, _, flat, offs = weights("tiny")
    eng = MegakernelEngine(flat=flat, offsets=offs, shape=shape, max_seq=64,
                           timeout_ns=50_000_000, debug_skip_cta=3)
    toks = torch.ones(2, dtype=torch.int32, device=DEV)
    out = torch.zeros(2, dtype=torch.int32, device=DEV)
    with pytest.raises(RuntimeError, match="timed out"):
        eng.decode_n(toks, 2, out)
    assert eng.lib.megakernel_last_error(eng._handle) == -3
    assert eng.pos == 0
    eng.close()
    # the device context is intact: a normal engine still matches the reference
    g = golden("tiny")
    toks, lg = teacher_forced(engine("tiny"), g["seq"].tolist()[:4])
    assert np.abs(lg[:, g["sub_ids"]] - g["sub_logits"][:4]).max() < LOGIT_TOL


def test_long_context_prefilled_kv_vs_oracle():
    """K/V of positions 0..8191 in every layer set to
    bf16(N(0,1)) (seed 2), then decode from position 8192 (split-KV across
    CTAs).  Compared with the fp32 oracle given the same cache."""
    shape, w, flat, offs = weights("qwen3-0.6b-d64")
    P0, steps = 8192, 4
    eng = MegakernelEngine(flat=flat, offsets=offs, shape=shape, max_seq=P0 + 64,
                           timeout_ns=2_000_000_000)
    g = torch.Generator().manual_seed(2)
    kv_host = torch.randn(shape.layers, 2, shape.kv_heads, P0, shape.head_dim, generator=g)
    kv_host = kv_host.to(torch.bfloat16)
    kv = eng.kv_cache()
    kv[:, :, :, :P0] = kv_host.to(DEV)
    torch.cuda.synchronize()
    eng.set_pos(P0)
    seq = golden("qwen3-0.6b-d64")["seq"][:steps].tolist()
    toks = torch.tensor(seq, dtype=torch.int32, device=DEV)
    out = torch.zeros(steps, dtype=torch.int32, device=DEV)
    lg = torch.zeros(steps, shape.vocab, device=DEV)
    eng.decode_n(toks, steps, out, logits=lg)
    o = Qwen3DecodeOracle(shape, w, kv_bf16=True, max_seq=P0 + 8, device="cuda")
    for layer in range(shape.layers):
        o.set_kv(layer, kv_host[layer, 0], kv_host[layer, 1])
    o.pos = P0
    otoks, olg, omargin = o.run(seq, steps)
    err = np.abs(lg.cpu().numpy() - olg).max()
    assert err < LOGIT_TOL, err
    ok = omargin > MARGIN
    assert np.array_equal(out.cpu().numpy()[ok], otoks[ok])
    eng.close()


def test_parallel_prefill_vs_reference():
    """megakernel_prefill (64 positions per batched tcgen05 step) fills the
    engine's cache so that the next token and every later step match the
    reference forward (BASELINE §8f: parallel prefill)."""
    g = golden("qwen3-0.6b-d64")
    eng = engine("qwen3-0.6b-d64")
    seq = g["seq"].tolist()
    k = 70                                   # one full chunk of 64 + a partial one
    nxt = eng.prefill(torch.tensor(seq[:k], dtype=torch.int32, device=DEV))
    assert eng.pos == k
    if g["margin"][k - 1] > MARGIN:
        assert int(nxt.item()) == int(g["argmax"][k - 1])
    n = len(seq) - k
    toks = torch.tensor(seq[k:], dtype=torch.int32, device=DEV)
    out = torch.zeros(n, dtype=torch.int32, device=DEV)
    lg = torch.zeros(n, eng.vocab, dtype=torch.float32, device=DEV)
    eng.decode_n(toks, n, out, logits=lg)
    lg = lg.cpu().numpy()
    err = np.abs(lg[:, g["sub_ids"]] - g["sub_logits"][k:]).max()
    assert err < LOGIT_TOL, err
    ok = g["margin"][k:] > MARGIN
    assert np.array_equal(out.cpu().numpy()[ok], g["argmax"][k:][ok])
