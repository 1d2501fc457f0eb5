"""The C-ABI library loads and exports every symbol include/megakernel.h
declares; host-only helpers (no GPU) behave."""
import ctypes
import os
import re

import numpy as np
import pytest

from megakernel_b200 import _lib
from megakernel_b200 import weights as W
from megakernel_b200.shapes import SHAPE_IDS, SHAPES
from oracle.qwen3_decode import rope_tables

from ._common import lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "megakernel.h")


def header_functions():
    txt = open(HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(megakernel_\w+)\s*\(", txt)))


def test_exports_every_declared_symbol():
    L = lib()
    names = header_functions()
    assert len(names) >= 25
    for n in names:
        assert hasattr(L, n), n
    # the ctypes declarations cover the header exactly
    assert set(_lib.signatures()) == set(names)


def test_reference_surface_present():
    for n in ["megakernel_init", "megakernel_decode", "megakernel_reset", "megakernel_get_pos",
              "megakernel_free", "megakernel_sync"]:
        assert n in header_functions()


def _offsets(shape):
    offs, cur = {}, 0
    for n, s in shape.tensor_shapes():
        offs[n] = cur
        cur += 2 * int(np.prod(s))
    return W.offsets_list(shape, offs)


@pytest.mark.parametrize("name", list(SHAPES))
def test_infer_shape(name):
    L = lib()
    ol = _offsets(SHAPES[name])
    arr = (ctypes.c_longlong * len(ol))(*ol)
    assert L.megakernel_infer_shape(arr, len(ol)) == SHAPE_IDS[name]
    bad = list(ol)
    bad[4] += 32  # w_k size no longer matches
    arr = (ctypes.c_longlong * len(bad))(*bad)
    assert L.megakernel_infer_shape(arr, len(bad)) == -5
    assert L.megakernel_infer_shape(arr, 7) == -5


def test_null_handle_paths():
    L = lib()
    assert L.megakernel_get_pos(None) == -1
    assert L.megakernel_decode(None, 1) == -1
    assert L.megakernel_last_error(None) == -1
    L.megakernel_reset(None)
    L.megakernel_free(None)
    assert L.megakernel_error_string(-3) == b"in-kernel wait timed out"
    opts = _lib.MkOptions()
    L.megakernel_default_options(ctypes.byref(opts))
    assert opts.device == -1 and opts.shape_id == -1 and opts.debug_skip_cta == -1


@pytest.mark.parametrize("D", [64, 128])
def test_rope_table_matches_hf(D):
    L = lib()
    n = 8448
    c = np.zeros((n, D // 2), np.float32)
    s = np.zeros_like(c)
    fp = ctypes.POINTER(ctypes.c_float)
    assert L.megakernel_rope_table(D, 1e6, n, c.ctypes.data_as(fp), s.ctypes.data_as(fp)) == 0
    tc, ts = rope_tables(D, 1e6, n)
    # Same fp32 formula; torch's vectorised pow differs from a correctly
    # rounded one by 1 ulp in one inv_freq entry for head_dim 128, which moves
    # the angle at position 8447 by < 1e-6 rad.
    assert np.abs(c - tc.numpy()).max() <= 1e-6
    assert np.abs(s - ts.numpy()).max() <= 1e-6


@pytest.mark.parametrize("name", ["qwen3-0.6b-d64", "qwen3-0.6b-d128"])
@pytest.mark.parametrize("pos", [0, 1, 2, 384, 8192])
def test_plan_covers_every_byte_once(name, pos):
    """Per-CTA streams add up to every weight matrix plus the cached K/V that
    travels through the rings (all positions but the previous one)."""
    L = lib()
    shape = SHAPES[name]
    n = 148
    b = (ctypes.c_longlong * n)()
    assert L.megakernel_plan_bytes(SHAPE_IDS[name], n, pos, b) == 0
    b = np.array(b)
    norms = 2 * (shape.hidden + shape.layers * (2 * shape.hidden + 2 * shape.head_dim))
    kv = shape.kv_bytes_per_position * max(pos - 1, 0)
    assert b.sum() == shape.weight_bytes - norms + kv
    # Long contexts are capped at 8 split-KV chunks per head, which leaves
    # the CTAs holding attention items ~7% heavier at 8k positions.
    assert b.max() / b.mean() < (1.06 if pos <= 1024 else 1.10)


def test_extension_argument_checks_without_a_device():
    """Argument checks that return before any CUDA call."""
    L = lib()
    assert L.megakernel_set_merge_mode(None, 1) == -1
    arr = (ctypes.c_longlong * 310)()
    # unknown storage flags: refused before the weights are touched
    assert L.megakernel_batch_init_ex(ctypes.c_void_p(16), arr, 310, 4, 64, 4) is None
    assert L.megakernel_batch_init_ex(ctypes.c_void_p(16), arr, 310, 4, 64, -1) is None
    assert L.megakernel_tp_exchange_slots(None, None) == -1
    assert L.megakernel_tc_gemm_test_e4m3(None, 64, None, None, 1024, 1024, None, None) == -1
    # split factor outside 1..4, or a split left without a K block
    x, w, o = ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16)
    assert L.megakernel_tc_gemm_test_split(x, 64, w, 1024, 1024, 5, o, None) == -1
    assert L.megakernel_tc_gemm_test_split(x, 64, w, 1024, 1024, 0, o, None) == -1
    assert L.megakernel_tc_gemm_test_split(x, 64, w, 128, 64, 3, o, None) == -1
