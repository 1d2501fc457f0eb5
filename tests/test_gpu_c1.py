"""GPU parity on BASELINE configs[1] itself: 128-token prompt, 512 greedy
tokens, positions 0..639 -- the positions the benchmark decodes.

Golden vectors: tests/golden/qwen3-0.6b-d64-c1.npz, made by the reference's
own reference_forward (host/validate.py:33-37) on the fp32 HF model.  At
these positions every KV head is split into 1..5 chunks of 128 cached
positions, so both attention merges run: the direct merge (forced for the
whole launch) and the two-level merge (forced from position 0; picked
automatically only past 5 chunks, i.e. positions > 640).
"""
import numpy as np
import pytest
import torch

from megakernel_b200.bridge import MegakernelEngine

from ._common import LOGIT_TOL, MARGIN, golden, weights

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
NAME = "qwen3-0.6b-d64-c1"


@pytest.fixture(scope="module")
def eng():
    shape, _, flat, offs = weights("qwen3-0.6b-d64")
    e = MegakernelEngine(flat=flat, offsets=offs, shape=shape, max_seq=2048, timeout_ns=2_000_000_000)
    yield e
    e.close()


def check_logits(g, toks, lg, lo=0):
    err_sub = np.abs(lg[:, g["sub_ids"]] - g["sub_logits"][lo:lo + len(lg)]).max()
    top = np.take_along_axis(lg, g["top_ids"][lo:lo + len(lg)], axis=1)
    err_top = np.abs(top - g["top_vals"][lo:lo + len(lg)]).max()
    assert err_sub < LOGIT_TOL and err_top < LOGIT_TOL, (err_sub, err_top)
    ok = g["margin"][lo:lo + len(lg)] > MARGIN
    assert np.array_equal(toks[ok], g["argmax"][lo:lo + len(lg)][ok])
    return max(err_sub, err_top)


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_teacher_forced_640_positions(eng, mode):
    """All 640 positions teacher-forced in one launch, each merge kernel."""
    g = golden(NAME)
    seq = g["seq"].tolist()
    eng.reset()
    eng.set_merge_mode(mode)
    try:
        n = len(seq)
        toks = torch.tensor(seq, dtype=torch.int32, device=DEV)
        out = torch.zeros(n, dtype=torch.int32, device=DEV)
        lg = torch.zeros(n, eng.vocab, dtype=torch.float32, device=DEV)
        eng.decode_n(toks, n, out, logits=lg)
        check_logits(g, out.cpu().numpy(), lg.cpu().numpy())
    finally:
        eng.set_merge_mode(0)


def test_free_running_greedy_as_benchmarked(eng):
    """The benchmark's own call sequence: parallel prefill of the 128-token
    prompt, then one launch of 512 greedy steps; tokens equal to the
    reference's greedy continuation up to its first low-margin step."""
    g = golden(NAME)
    seq, n_prompt = g["seq"], int(g["n_prompt"])
    eng.reset()
    first = eng.prefill(torch.tensor(seq[:n_prompt].tolist(), dtype=torch.int32, device=DEV))
    n_gen = len(seq) - n_prompt
    out = torch.zeros(n_gen, dtype=torch.int32, device=DEV)
    eng.decode_n(first, 1, out, n_steps=n_gen)
    got = np.concatenate([[int(first.item())], out.cpu().numpy()[:n_gen - 1]])
    want = seq[n_prompt:]
    low = np.nonzero(g["margin"][n_prompt - 1:-1] <= MARGIN)[0]
    upto = int(low[0]) if low.size else len(want)
    assert upto >= 16, upto
    assert np.array_equal(got[:upto], want[:upto]), (got[:upto], want[:upto])


def test_out_of_range_forced_token_is_rejected_on_device(eng):
    """A device token id >= vocab ends the launch with MK_ERR_INVALID_ARG
    before any embedding read; the engine stays usable."""
    eng.reset()
    toks = torch.tensor([1, 2, eng.vocab, 3], dtype=torch.int32, device=DEV)
    out = torch.zeros(4, dtype=torch.int32, device=DEV)
    with pytest.raises(RuntimeError, match="invalid"):
        eng.decode_n(toks, 4, out)
    assert eng.lib.megakernel_last_error(eng._handle) == -1
    assert eng.pos == 0
    toks = torch.tensor([-5], dtype=torch.int32, device=DEV)
    with pytest.raises(RuntimeError, match="invalid"):
        eng.decode_n(toks, 1, out[:1])
    g = golden(NAME)
    seq = g["seq"].tolist()[:8]
    toks = torch.tensor(seq, dtype=torch.int32, device=DEV)
    out = torch.zeros(8, dtype=torch.int32, device=DEV)
    lg = torch.zeros(8, eng.vocab, dtype=torch.float32, device=DEV)
    eng.decode_n(toks, 8, out, logits=lg)
    check_logits(g, out.cpu().numpy(), lg.cpu().numpy())
