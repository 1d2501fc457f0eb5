"""Pin the oracle to the reference: oracle/qwen3_decode.py vs golden logits that
the reference's reference_forward (host/validate.py:33-37) produced."""
import numpy as np
import pytest
import torch

from oracle.qwen3_decode import Qwen3DecodeOracle, rope_tables

from ._common import LOGIT_TOL, MARGIN, golden, weights


def _teacher_forced(shape_name, n, kv_bf16, golden_name=None):
    shape, w, _, _ = weights(shape_name)
    g = golden(golden_name or shape_name)
    seq = g["seq"].tolist()[:n]
    o = Qwen3DecodeOracle(shape, w, kv_bf16=kv_bf16, max_seq=max(64, n + 1))
    toks, logits, margins = o.run(seq, n)
    return g, toks, logits


def test_tiny_fp32_matches_reference_exactly():
    g, toks, logits = _teacher_forced("tiny", 32, kv_bf16=False)
    assert np.abs(logits[:, g["sub_ids"]] - g["sub_logits"]).max() < 1e-5
    assert np.array_equal(toks, g["argmax"])


@pytest.mark.parametrize("name,n,gname", [("qwen3-0.6b-d64", 12, None), ("qwen3-0.6b-d128", 6, None),
                                          ("qwen3-0.6b-d64", 8, "qwen3-0.6b-d64-c1")])
def test_full_shape_fp32_matches_reference(name, n, gname):
    g, toks, logits = _teacher_forced(name, n, kv_bf16=False, golden_name=gname)
    err = np.abs(logits[:, g["sub_ids"]] - g["sub_logits"][:n]).max()
    # Same math in fp32 on the same CPU; only summation order differs.
    assert err < 2e-3, err
    top = np.take_along_axis(logits, g["top_ids"][:n], axis=1)
    assert np.abs(top - g["top_vals"][:n]).max() < 2e-3
    ok = g["margin"][:n] > MARGIN
    assert np.array_equal(toks[ok], g["argmax"][:n][ok])


def test_bf16_kv_within_gate():
    """The kernel keeps K/V in bf16 (the reference's cache layout); the oracle
    run with the same rounding stays inside the north-star logit tolerance."""
    g, toks, logits = _teacher_forced("tiny", 32, kv_bf16=True)
    assert np.abs(logits[:, g["sub_ids"]] - g["sub_logits"]).max() < LOGIT_TOL


def test_greedy_sequence_is_oracle_greedy():
    """The golden sequence is the fp32 model's own greedy continuation."""
    g = golden("tiny")
    seq, n_prompt = g["seq"], int(g["n_prompt"])
    assert np.array_equal(g["argmax"][n_prompt - 1:-1], seq[n_prompt:])


def test_rope_tables_match_hf():
    c, s = rope_tables(64, 1e6, 8)
    assert torch.allclose(c[0], torch.ones(32)) and torch.allclose(s[0], torch.zeros(32))


def test_e4m3_weight_rounding():
    """quant_rows_e4m3 (the oracle's model of the batched decoder's e4m3
    weights): each row's largest magnitude maps to 448 x its scale, every
    value is an e4m3 number times the row scale, and the relative rounding
    error stays within e4m3's 2^-4."""
    from oracle.qwen3_decode import quant_rows_e4m3
    g = torch.Generator().manual_seed(0)
    w = (torch.randn(64, 256, generator=g) * 0.02).to(torch.bfloat16).float()
    q = quant_rows_e4m3(w)
    sc = w.abs().amax(dim=1, keepdim=True) / 448.0
    assert torch.allclose(q.abs().amax(dim=1, keepdim=True), w.abs().amax(dim=1, keepdim=True), rtol=1e-6)
    e = (q / sc)
    assert torch.allclose(e.to(torch.float8_e4m3fn).float(), e, rtol=1e-5, atol=0)
    big = w.abs() > 1e-2 * w.abs().amax(dim=1, keepdim=True)
    assert ((q - w).abs()[big] / w.abs()[big]).max() <= 2.0 ** -4
