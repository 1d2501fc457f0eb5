"""Flat-binary format: layout, offsets order and round trip (host/weight_loader.py:141-206)."""
import json
import os

import numpy as np
import pytest
import torch

from megakernel_b200 import weights as W
from megakernel_b200.shapes import QWEN3_0_6B_D64, QWEN3_0_6B_D128, TINY


@pytest.mark.parametrize("shape", [TINY, QWEN3_0_6B_D64, QWEN3_0_6B_D128])
def test_sizes(shape):
    # 971,891,712 B for the graded shape, 1,192,099,840 B for d128.
    want = {"tiny": None, "qwen3-0.6b-d64": 971891712, "qwen3-0.6b-d128": 1192099840}[shape.name]
    if want:
        assert shape.weight_bytes == want
    assert shape.num_offsets == 2 + 11 * shape.layers


def test_roundtrip_and_order(tmp_path):
    w = W.random_weights(TINY, 0)
    path = str(tmp_path / "weights.bin")
    offs = W.save_flat_binary(TINY, w, path)
    with open(path.replace(".bin", "_offsets.json")) as f:
        assert json.load(f) == offs
    names = [n for n, _ in TINY.tensor_shapes()]
    assert list(offs.keys()) == names
    ol = W.offsets_list(TINY, offs)
    # host/bridge.py:89-96 order: embedding, final_norm, 11 keys per layer.
    assert ol[0] == offs["embedding"] and ol[1] == offs["final_norm"]
    assert ol[2 + 11 * 1 + 6] == offs["layer.1.w_o"]
    assert all(b > a for a, b in zip(ol, ol[1:]))
    assert all(o % 16 == 0 for o in ol)
    data, offs2 = W.load_flat_binary(path)
    back = W.unpack(TINY, data, offs2)
    for n in names:
        assert torch.equal(back[n].view(torch.int16), w[n].view(torch.int16)), n


def test_seeded_init_deterministic():
    a = W.random_weights(TINY, 0)
    b = W.random_weights(TINY, 0)
    c = W.random_weights(TINY, 1)
    assert all(torch.equal(a[k], b[k]) for k in a)
    assert not torch.equal(a["layer.0.w_q"], c["layer.0.w_q"])
    assert torch.all(a["layer.1.q_norm"] == 1)
    s = a["embedding"].float().std().item()
    assert 0.018 < s < 0.022


# The reference checkout, when available, is named by MK_REFERENCE_ROOT.
REF = os.environ.get("MK_REFERENCE_ROOT", "")


@pytest.mark.skipif(not REF or not os.path.exists(os.path.join(REF, "host", "weight_loader.py")),
                    reason="MK_REFERENCE_ROOT does not name a reference checkout")
def test_bytes_match_reference_writer(tmp_path):
    """Our writer produces the same bytes and offsets as the reference's
    save_flat_binary (which hard-codes the head_dim-128 shape)."""
    import sys
    sys.path.insert(0, REF)
    from host.weight_loader import save_flat_binary as ref_save
    w = W.random_weights(QWEN3_0_6B_D128, 0)
    ours = str(tmp_path / "ours.bin")
    theirs = str(tmp_path / "theirs.bin")
    o1 = W.save_flat_binary(QWEN3_0_6B_D128, w, ours)
    o2 = ref_save(w, theirs)
    assert o1 == o2
    a = np.fromfile(ours, dtype=np.uint8)
    b = np.fromfile(theirs, dtype=np.uint8)
    assert a.size == b.size and np.array_equal(a, b)
