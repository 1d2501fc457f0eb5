"""``BatchDecoder``: batched greedy decode of up to 64 sequences per step.

The reference runs one sequence per launch (host/bridge.py:110-162); this is
the concurrent-sequence extension (``megakernel_batch_*`` in
include/megakernel.h).  Each step feeds one token per sequence at that
sequence's own position and returns the next greedy token of each; the
matrix products run on tcgen05 tensor cores with the 64 sequences as the M
dimension.  Same weights format (flat binary + offsets) as the single-stream
engine; d64 shape only.  There is no CPU path.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from .shapes import QWEN3_0_6B_D64
from .weights import offsets_list


class BatchDecoder:
    KV_DTYPES = {"bf16": 0, "fp8": 1}
    W_DTYPES = {"bf16": 0, "fp8": 2}

    def __init__(self, flat, offsets, batch, max_seq, shape=QWEN3_0_6B_D64, device=0, lib_path=None,
                 kv_dtype="bf16", w_dtype="bf16"):
        """kv_dtype: "bf16" (the reference's cache format) or "fp8" (e4m3,
        half the cache bytes); w_dtype: "bf16" or "fp8" (the GEMMs on an
        e4m3 copy of the weights with per-row scales).  See
        megakernel_batch_init_ex."""
        if shape.name != QWEN3_0_6B_D64.name:
            raise ValueError("the batched path supports the head_dim-64 / intermediate-2816 shape only")
        self.lib = _lib.load(lib_path)
        self.shape = shape
        self.batch = int(batch)
        self.max_seq = int(max_seq)
        self.device = torch.device("cuda", device)
        torch.cuda.set_device(self.device)
        if isinstance(flat, torch.Tensor):
            self._weights = flat.to(self.device, torch.uint8)
        else:
            self._weights = torch.from_numpy(np.asarray(flat, dtype=np.uint8)).to(self.device)
        ol = offsets_list(shape, offsets)
        arr = (ctypes.c_longlong * len(ol))(*ol)
        self.kv_dtype, self.w_dtype = kv_dtype, w_dtype
        flags = self.KV_DTYPES[kv_dtype] | self.W_DTYPES[w_dtype]
        self._handle = self.lib.megakernel_batch_init_ex(ctypes.c_void_p(self._weights.data_ptr()), arr, len(ol),
                                                         self.batch, self.max_seq, flags)
        if not self._handle:
            raise RuntimeError("megakernel_batch_init failed (shape, alignment, batch <= 64 or memory)")
        self.vocab = shape.vocab

    def close(self):
        if self._handle:
            self.lib.megakernel_batch_free(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- positions / cache ------------------------------------------------
    def set_pos(self, pos):
        pos = [int(p) for p in pos]
        if len(pos) != self.batch:
            raise ValueError("one position per sequence")
        arr = (ctypes.c_int * self.batch)(*pos)
        _lib.check(self.lib.megakernel_batch_set_pos(self._handle, arr), "megakernel_batch_set_pos")

    def reset(self):
        self.set_pos([0] * self.batch)

    @property
    def pos(self):
        arr = (ctypes.c_int * self.batch)()
        _lib.check(self.lib.megakernel_batch_get_pos(self._handle, arr), "megakernel_batch_get_pos")
        return list(arr)

    def kv_cache(self):
        """View [batch, layers, 2, kv_heads, max_seq, head_dim] of the cache
        (zero copy): bf16, or float8_e4m3fn with an fp8 cache."""
        s = self.shape
        shape = (self.batch, s.layers, 2, s.kv_heads, self.max_seq, s.head_dim)
        ptr = self.lib.megakernel_batch_kv_ptr(self._handle)
        n = int(np.prod(shape))
        fp8 = self.kv_dtype == "fp8"

        class _Holder:
            __cuda_array_interface__ = {"shape": (n,), "typestr": "|u1" if fp8 else "<i2", "data": (ptr, False),
                                        "version": 3}

        t = torch.as_tensor(_Holder(), device=self.device)
        return t.view(torch.float8_e4m3fn if fp8 else torch.bfloat16).view(*shape)

    # ---- decoding -----------------------------------------------------------
    def step(self, tokens, logits=False, stream=None):
        """One token per sequence (device int32 [batch]) -> next tokens (device int32 [batch])."""
        tok = torch.as_tensor(tokens, dtype=torch.int32, device=self.device).contiguous()
        out = torch.empty(self.batch, dtype=torch.int32, device=self.device)
        lg = torch.empty(self.batch, self.vocab, device=self.device) if logits else None
        st = stream.cuda_stream if stream is not None else torch.cuda.current_stream(self.device).cuda_stream
        rc = self.lib.megakernel_batch_step(self._handle, ctypes.c_void_p(tok.data_ptr()),
                                            ctypes.c_void_p(out.data_ptr()),
                                            ctypes.c_void_p(lg.data_ptr()) if lg is not None else None,
                                            ctypes.c_void_p(st))
        _lib.check(rc, "megakernel_batch_step")
        return (out, lg) if logits else out

    def decode_n(self, forced, n_steps, out=None, stream=None):
        """forced: device int32 [n_forced, batch]; steps < n_forced consume them,
        later steps consume the previous step's greedy tokens.  Returns [n_steps, batch]."""
        forced = torch.as_tensor(forced, dtype=torch.int32, device=self.device).contiguous()
        n_forced = forced.shape[0]
        if out is None:
            out = torch.empty(n_steps, self.batch, dtype=torch.int32, device=self.device)
        st = stream.cuda_stream if stream is not None else torch.cuda.current_stream(self.device).cuda_stream
        rc = self.lib.megakernel_batch_decode_n(self._handle, ctypes.c_void_p(forced.data_ptr()), n_forced, n_steps,
                                                ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(st))
        _lib.check(rc, "megakernel_batch_decode_n")
        return out
