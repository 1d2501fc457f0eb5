"""MegakernelEngine's reference methods (host/bridge.py:118-261): generate
with a tokenizer (text in, text out, EOS stop) and with id lists, benchmark,
and benchmark_sweep, whose tokens are checked against the fp32 oracle at one
position per attention-merge regime."""
import numpy as np
import pytest
import torch

from megakernel_b200.bridge import MegakernelEngine
from oracle.qwen3_decode import Qwen3DecodeOracle

from ._common import MARGIN, golden, weights

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


class StubTokenizer:
    """encode: one id per character (ord % vocab); decode: ids back to text."""

    def __init__(self, vocab, eos):
        self.vocab, self.eos_token_id = vocab, eos

    def encode(self, text):
        return [ord(c) % self.vocab for c in text]

    def decode(self, ids, skip_special_tokens=False):
        return "".join(f"<{i}>" for i in ids if not (skip_special_tokens and i == self.eos_token_id))


@pytest.fixture(scope="module")
def tiny():
    shape, w, flat, offs = weights("tiny")
    eng = MegakernelEngine(flat=flat, offsets=offs, shape=shape, max_seq=256, timeout_ns=2_000_000_000)
    yield shape, w, eng
    eng.close()


def test_generate_ids_matches_golden(tiny):
    shape, _, eng = tiny
    g = golden("tiny")
    n_prompt = int(g["n_prompt"])
    out, tps = eng.generate(g["seq"][:n_prompt].tolist(), max_tokens=8)
    assert tps > 0 and len(out) == 8
    want = g["seq"][n_prompt:n_prompt + 8]
    low = np.nonzero(g["margin"][n_prompt - 1:n_prompt + 7] <= MARGIN)[0]
    upto = int(low[0]) if low.size else 8
    assert out[:upto] == want[:upto].tolist()


def test_generate_text_with_tokenizer_and_eos(tiny):
    shape, _, eng = tiny
    prompt = "hello megakernel"
    ids = [ord(c) % shape.vocab for c in prompt]
    full, _ = eng.generate(ids, max_tokens=12)
    # EOS = the 4th generated token: generation stops right after it
    tok = StubTokenizer(shape.vocab, full[3])
    eng.tokenizer = tok
    try:
        text, tps = eng.generate(prompt, max_tokens=12)
    finally:
        eng.tokenizer = None
    stop = full.index(full[3]) + 1
    assert text == tok.decode(ids + full[:stop], skip_special_tokens=True)
    assert tps > 0


def test_benchmark_runs(tiny):
    _, _, eng = tiny
    assert eng.benchmark(num_tokens=10) > 0
    assert eng.pos == 10


def test_benchmark_sweep_tokens_vs_oracle():
    """Sweep positions 1, 100 (one chunk per head), 300 (3 chunks, direct
    merge) and 700 (6 chunks, two-level merge) on the graded shape; the
    generated greedy tokens equal the oracle's until its first low-margin step."""
    shape, w, flat, offs = weights("qwen3-0.6b-d64")
    eng = MegakernelEngine(flat=flat, offsets=offs, shape=shape, max_seq=1024, timeout_ns=2_000_000_000)
    res = eng.benchmark_sweep(positions=[1, 100, 300, 700], bench_tokens=6)
    eng.close()
    assert [r["position"] for r in res] == [1, 100, 300, 700]
    for r in res:
        assert r["tok_per_sec"] > 0 and r["bw_gbps"] > 0
        pos = r["position"]
        o = Qwen3DecodeOracle(shape, w, kv_bf16=True, max_seq=pos + 16, device="cuda")
        toks, _, margins = o.run([1] * pos, pos + 6, want_logits=False)
        # tokens[k] is the argmax at step pos + k; it depends on the argmaxes
        # of steps pos-1 .. pos+k, so it is gated on their margins.
        m = margins[pos - 1:pos + 6]
        low = np.nonzero(m <= MARGIN)[0]
        upto = int(low[0]) if low.size else len(m)
        n_ok = max(upto - 1, 0)
        assert r["tokens"][:n_ok] == toks[pos:pos + n_ok].tolist(), (pos, r["tokens"], toks[pos:])
