"""Batched decode (megakernel_batch_*: up to 64 sequences per step, tcgen05
GEMMs) against the fp32 oracle, per sequence.

Gates as for the single-stream path: logits within
2e-2 max-abs of the fp32 reference, argmax equal wherever the reference's
top-2 margin exceeds 1e-2.  The oracle runs each sequence alone (same
weights, same tokens, bf16 K/V), which is what a batched decode must
reproduce.
"""
import numpy as np
import pytest
import torch

from megakernel_b200.batch import BatchDecoder
from oracle.qwen3_decode import Qwen3DecodeOracle

from ._common import LOGIT_TOL, MARGIN, weights

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _tokens(batch, steps, seed=1):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 151936, (batch, steps), generator=g)


def _run_forced(bd, toks):
    lgs, outs = [], []
    for t in range(toks.shape[1]):
        out, lg = bd.step(toks[:, t].to(DEV), logits=True)
        lgs.append(lg.cpu().numpy())
        outs.append(out.cpu().numpy())
    return np.stack(lgs, 1), np.stack(outs, 1)


def _check_seq(shape, w, seq, lg, out):
    o = Qwen3DecodeOracle(shape, w, kv_bf16=True, max_seq=64, device="cuda")
    ot, ol, om = o.run(seq, len(seq))
    assert np.abs(lg - ol).max() < LOGIT_TOL, np.abs(lg - ol).max()
    ok = om > MARGIN
    assert np.array_equal(out[ok], ot[ok])


def test_batch_teacher_forced_vs_oracle():
    shape, w, flat, offs = weights("qwen3-0.6b-d64")
    toks = _tokens(4, 6)
    bd = BatchDecoder(flat, offs, batch=4, max_seq=128)
    lg, out = _run_forced(bd, toks)
    assert bd.pos == [6] * 4
    for b in range(4):
        _check_seq(shape, w, toks[b].tolist(), lg[b], out[b])
    bd.close()


def test_batch_full_64_vs_oracle():
    shape, w, flat, offs = weights("qwen3-0.6b-d64")
    toks = _tokens(64, 3, seed=5)
    bd = BatchDecoder(flat, offs, batch=64, max_seq=96)
    lg, out = _run_forced(bd, toks)
    for b in (0, 31, 63):
        _check_seq(shape, w, toks[b].tolist(), lg[b], out[b])
    bd.close()


def test_batch_decode_n_equals_steps():
    """One decode_n call (forced prefix, then greedy) == step-by-step calls; bit-exact."""
    shape, w, flat, offs = weights("qwen3-0.6b-d64")
    toks = _tokens(8, 3, seed=7).to(DEV, torch.int32)
    bd = BatchDecoder(flat, offs, batch=8, max_seq=64)
    out_n = bd.decode_n(toks.t().contiguous(), 7).cpu().numpy()
    bd.reset()
    ref, cur = [], None
    for t in range(7):
        cur = bd.step(toks[:, t] if t < 3 else cur)
        ref.append(cur.cpu().numpy())
    assert np.array_equal(out_n, np.stack(ref, 0))
    assert bd.pos == [7] * 8
    bd.close()


def test_batch_long_context_configs3_vs_oracle():
    """BASELINE configs[3]'s own regime: 64 sequences prefilled to 1,024
    positions through the batched step (teacher-forced decode_n), then three
    steps at positions 1024-1026 -- 16 and 17 chunks of 64 positions per
    (sequence, KV head) through battn_kernel's merge -- compared per
    sequence with the fp32 oracle run alone on that sequence."""
    shape, w, flat, offs = weights("qwen3-0.6b-d64")
    B, P, S = 64, 1024, 3
    toks = _tokens(B, P + S, seed=11)
    bd = BatchDecoder(flat, offs, batch=B, max_seq=P + S + 16)
    bd.decode_n(toks[:, :P].t().contiguous().to(DEV, torch.int32), P)
    assert bd.pos == [P] * B
    lgs, outs = [], []
    for t in range(P, P + S):
        out, lg = bd.step(toks[:, t].to(DEV), logits=True)
        lgs.append(lg.cpu().numpy())
        outs.append(out.cpu().numpy())
    lg, out = np.stack(lgs, 1), np.stack(outs, 1)
    bd.close()
    for b in (0, 37, 63):
        o = Qwen3DecodeOracle(shape, w, kv_bf16=True, max_seq=P + S + 8, device="cuda")
        ot, ol, om = o.run(toks[b].tolist(), P + S)
        err = np.abs(lg[b] - ol[P:]).max()
        assert err < LOGIT_TOL, (b, err)
        ok = om[P:] > MARGIN
        assert np.array_equal(out[b][ok], ot[P:][ok])


def test_batch_fp8_kv_cache_vs_oracle():
    """The batched decoder with an e4m3 KV cache (megakernel_batch_init_ex):
    against the fp32 oracle that rounds K/V to e4m3 the same way -- the
    north-star logit gate and argmax where the margin > 1e-2 -- and, for the
    record, the error against the bf16-cache oracle (the reference's cache
    precision), which must stay below the documented 0.5 bound."""
    shape, w, flat, offs = weights("qwen3-0.6b-d64")
    B, P, S = 8, 200, 3
    toks = _tokens(B, P + S, seed=13)
    bd = BatchDecoder(flat, offs, batch=B, max_seq=P + S + 16, kv_dtype="fp8")
    assert bd.kv_cache().dtype == torch.float8_e4m3fn
    bd.decode_n(toks[:, :P].t().contiguous().to(DEV, torch.int32), P)
    lgs, outs = [], []
    for t in range(P, P + S):
        out, lg = bd.step(toks[:, t].to(DEV), logits=True)
        lgs.append(lg.cpu().numpy())
        outs.append(out.cpu().numpy())
    lg, out = np.stack(lgs, 1), np.stack(outs, 1)
    bd.close()
    for b in (0, 5):
        o8 = Qwen3DecodeOracle(shape, w, kv_fp8=True, max_seq=P + S + 8, device="cuda")
        ot, ol, om = o8.run(toks[b].tolist(), P + S)
        err = np.abs(lg[b] - ol[P:]).max()
        assert err < LOGIT_TOL, (b, err)
        ok = om[P:] > MARGIN
        assert np.array_equal(out[b][ok], ot[P:][ok])
        o16 = Qwen3DecodeOracle(shape, w, kv_bf16=True, max_seq=P + S + 8, device="cuda")
        _, ol16, _ = o16.run(toks[b].tolist(), P + S)
        err16 = np.abs(lg[b] - ol16[P:]).max()
        print(f"fp8 KV, sequence {b}: max |logit - e4m3 oracle| {err:.2e}, vs bf16-cache oracle {err16:.2e}")
        assert err16 < 0.5, err16


def test_batch_fp8_weights_vs_oracle():
    """The batched decoder on e4m3 weights (per-row scales; the tcgen05 GEMMs
    expand each e4m3 W block to bf16 in shared memory): against the fp32
    oracle with the same weight rounding -- the north-star logit gate and
    argmax where the margin > 1e-2 -- and, for the record, against the bf16
    model (documented bound 1.0)."""
    shape, w, flat, offs = weights("qwen3-0.6b-d64")
    B, P, S = 4, 40, 3
    toks = _tokens(B, P + S, seed=17)
    bd = BatchDecoder(flat, offs, batch=B, max_seq=P + S + 16, w_dtype="fp8")
    bd.decode_n(toks[:, :P].t().contiguous().to(DEV, torch.int32), P)
    lgs, outs = [], []
    for t in range(P, P + S):
        out, lg = bd.step(toks[:, t].to(DEV), logits=True)
        lgs.append(lg.cpu().numpy())
        outs.append(out.cpu().numpy())
    lg, out = np.stack(lgs, 1), np.stack(outs, 1)
    bd.close()
    for b in (0, 3):
        o8 = Qwen3DecodeOracle(shape, w, kv_bf16=True, max_seq=P + S + 8, device="cuda", w_fp8=True)
        ot, ol, om = o8.run(toks[b].tolist(), P + S)
        err = np.abs(lg[b] - ol[P:]).max()
        assert err < LOGIT_TOL, (b, err)
        ok = om[P:] > MARGIN
        assert np.array_equal(out[b][ok], ot[P:][ok])
        o16 = Qwen3DecodeOracle(shape, w, kv_bf16=True, max_seq=P + S + 8, device="cuda")
        _, ol16, _ = o16.run(toks[b].tolist(), P + S)
        err16 = np.abs(lg[b] - ol16[P:]).max()
        print(f"fp8 weights, sequence {b}: max |logit - e4m3-weight oracle| {err:.2e}, vs bf16 model {err16:.2e}")
        assert err16 < 1.0, err16
