"""``MegakernelEngine``: the reference's Python host surface over libmegakernel.

Mirrors ``host/bridge.py:29-270`` -- same constructor arguments, same methods
(``reset``, ``decode_token``, ``generate``, ``benchmark``, ``benchmark_sweep``,
``close``) and the same weight-loading path (flat binary + offsets JSON into
one CUDA uint8 buffer).  Differences, all additive: the engine can also be
built from an in-memory flat buffer, the tokenizer is optional (token-id
prompts work without one), ``generate`` runs prefill and the greedy loop in
one kernel launch instead of one launch per token (and prefills once, not
twice as host/bridge.py:137-159 does), and extra methods expose the
extension ABI (``decode_n``, ``logits``, ``set_pos``, ``kv_cache``).

There is no CPU path: every method goes through the CUDA library.
"""
from __future__ import annotations

import ctypes
import json
import time

import numpy as np
import torch

from . import _lib
from .shapes import SHAPES, SHAPE_IDS
from .weights import offsets_list


class MegakernelEngine:
    """Python wrapper around libmegakernel (host/bridge.py:29)."""

    def __init__(self, weights_path=None, offsets_path=None, lib_path=None, tokenizer=None, *,
                 flat=None, offsets=None, shape=None, device=0, max_seq=0, num_ctas=0,
                 timeout_ns=0, debug_skip_cta=-1, tp_rank=0, tp_size=1):
        self.tokenizer = tokenizer
        self.lib = _lib.load(lib_path)
        self._handle = None
        if flat is None:
            with open(offsets_path) as f:
                offsets = json.load(f)
            flat = np.fromfile(weights_path, dtype=np.uint8)
        self.shape = shape or self._shape_from_offsets(offsets)
        self.device = torch.device("cuda", device)
        # host/bridge.py:69-97: one uint8 device buffer holding the flat binary.
        if isinstance(flat, torch.Tensor):
            self._gpu_buffer = flat.to(self.device)
        else:
            self._gpu_buffer = torch.from_numpy(np.ascontiguousarray(flat)).to(self.device)
        offs = offsets_list(self.shape, offsets)
        self._num_offsets = len(offs)
        self._offsets_arr = (ctypes.c_longlong * len(offs))(*offs)
        opts = _lib.MkOptions()
        self.lib.megakernel_default_options(ctypes.byref(opts))
        opts.device = device
        opts.shape_id = SHAPE_IDS[self.shape.name]
        opts.max_seq = max_seq
        opts.num_ctas = num_ctas
        opts.timeout_ns = timeout_ns
        opts.debug_skip_cta = debug_skip_cta
        h = ctypes.c_void_p()
        self.tp_rank, self.tp_size = tp_rank, tp_size
        if tp_size > 1:
            # Tensor-parallel rank: call tp_connect (megakernel_b200.tp.connect)
            # on every rank before decoding.
            rc = self.lib.megakernel_tp_init(ctypes.c_void_p(self._gpu_buffer.data_ptr()),
                                             self._offsets_arr, self._num_offsets, ctypes.byref(opts),
                                             int(tp_rank), int(tp_size), ctypes.byref(h))
            _lib.check(rc, "megakernel_tp_init")
        else:
            rc = self.lib.megakernel_init_ex(ctypes.c_void_p(self._gpu_buffer.data_ptr()),
                                             self._offsets_arr, self._num_offsets,
                                             ctypes.byref(opts), ctypes.byref(h))
            _lib.check(rc, "megakernel_init_ex")
        self._handle = h.value
        self.vocab = self.shape.vocab
        self.max_seq = self.lib.megakernel_max_seq(self._handle)
        self.num_ctas = self.lib.megakernel_num_ctas(self._handle)

    @staticmethod
    def _shape_from_offsets(offsets: dict):
        for s in SHAPES.values():
            names = [n for n, _ in s.tensor_shapes()]
            if set(names) == set(offsets.keys()) and \
               offsets["final_norm"] - offsets["embedding"] == 2 * s.vocab * s.hidden and \
               offsets["layer.0.k_norm"] - offsets["layer.0.q_norm"] == 2 * s.head_dim and \
               offsets["layer.0.w_up"] - offsets["layer.0.w_gate"] == 2 * s.intermediate * s.hidden:
                return s
        raise ValueError("offsets match no compiled model shape")

    # ---- reference surface -------------------------------------------------
    def reset(self):
        """Reset KV cache and position (host/bridge.py:110)."""
        self.lib.megakernel_reset(self._handle)

    def decode_token(self, token_id):
        """One launch: input token -> next token (host/bridge.py:114-116)."""
        t = self.lib.megakernel_decode(self._handle, int(token_id))
        if t < 0:
            _lib.check(self.lib.megakernel_last_error(self._handle), "megakernel_decode")
        return t

    def generate(self, prompt, max_tokens=100, print_stream=False):
        """Prefill + greedy decode (host/bridge.py:118-192).

        ``prompt`` is a string (needs a tokenizer) or a list of token ids.
        Returns (text or token list, tokens_per_second); generation stops at
        EOS when a tokenizer is present, like the reference loop.
        """
        ids = self.tokenizer.encode(prompt) if isinstance(prompt, str) else list(prompt)
        self.reset()
        torch.cuda.synchronize(self.device)
        start = time.perf_counter()
        out = self.generate_ids(ids, max_tokens)
        elapsed = time.perf_counter() - start
        eos = getattr(self.tokenizer, "eos_token_id", None) if self.tokenizer else None
        if eos is not None and eos in out:
            out = out[:out.index(eos) + 1]
        if print_stream and self.tokenizer:
            print(self.tokenizer.decode(out))
        tps = len(out) / elapsed if elapsed > 0 else 0.0
        if self.tokenizer:
            return self.tokenizer.decode(ids + out, skip_special_tokens=True), tps
        return out, tps

    def generate_ids(self, ids, n_gen):
        """Host-buffer C-ABI call: prompt ids in, n_gen greedy ids out."""
        arr = (ctypes.c_int * len(ids))(*ids)
        out = (ctypes.c_int * n_gen)()
        _lib.check(self.lib.megakernel_generate(self._handle, arr, len(ids), n_gen, out),
                   "megakernel_generate")
        return list(out)

    def benchmark(self, num_tokens=50, prompt_token=1):
        """Raw per-token decode throughput through megakernel_decode (host/bridge.py:194-218)."""
        self.reset()
        token = prompt_token
        for _ in range(5):
            token = self.decode_token(token)
        self.reset()
        self.lib.megakernel_sync()
        token = prompt_token
        start = time.perf_counter()
        for _ in range(num_tokens):
            token = self.decode_token(token)
        self.lib.megakernel_sync()
        return num_tokens / (time.perf_counter() - start)

    def benchmark_sweep(self, positions=None, bench_tokens=20):
        """Throughput at several context positions (host/bridge.py:220-261).

        Bandwidth counts weights plus K/V bytes (the reference counts a fixed
        926 MB of weights only, host/bridge.py:229).  Each entry also carries
        the greedy tokens generated after the all-ones prefix of `position`
        tokens (an addition, for checking)."""
        if positions is None:
            positions = [1, 10, 50, 100, 500, 1000, 2000]
        res = []
        for pos in positions:
            self.reset()
            toks = torch.ones(pos + bench_tokens, dtype=torch.int32, device=self.device)
            outs = torch.empty_like(toks)
            if pos > 0:
                self.decode_n(toks[:pos], pos, outs[:pos])
            torch.cuda.synchronize(self.device)
            start = time.perf_counter()
            first = outs[pos - 1:pos].clone() if pos > 0 else toks[:1]
            self.decode_n(first, 1, outs[pos:], n_steps=bench_tokens)
            elapsed = time.perf_counter() - start
            tps = bench_tokens / elapsed
            nbytes = np.mean([self.shape.algorithmic_bytes(pos + i) for i in range(bench_tokens)])
            res.append({"position": pos, "tok_per_sec": tps, "latency_us": elapsed * 1e6 / bench_tokens,
                        "bw_gbps": nbytes * tps / 1e9,
                        "tokens": outs[pos:pos + bench_tokens].cpu().tolist()})
        return res

    def close(self):
        """Free device state (host/bridge.py:263-267)."""
        if self._handle:
            self.lib.megakernel_free(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- extensions --------------------------------------------------------
    @property
    def pos(self):
        return self.lib.megakernel_get_pos(self._handle)

    def set_pos(self, pos):
        _lib.check(self.lib.megakernel_set_pos(self._handle, int(pos)), "megakernel_set_pos")

    def kv_cache(self) -> torch.Tensor:
        """The engine's KV cache as a [L, 2, KVH, max_seq, D] bf16 view (no copy)."""
        s = self.shape
        ptr = self.lib.megakernel_kv_ptr(self._handle)
        shape = (s.layers, 2, s.kv_heads, self.max_seq, s.head_dim)
        return _device_view(ptr, shape, torch.bfloat16, self.device)

    def decode_n(self, tokens: torch.Tensor, n_forced: int, out: torch.Tensor,
                 n_steps: int | None = None, logits: torch.Tensor | None = None, stream=None):
        """One launch of n_steps steps on device tensors (megakernel_decode_n)."""
        n_steps = n_steps or out.numel()
        assert tokens.dtype == torch.int32 and out.dtype == torch.int32 and out.numel() >= n_steps
        assert tokens.is_contiguous() and out.is_contiguous()
        lp = logits.data_ptr() if logits is not None else None
        # Default: torch's current stream, so the launch is ordered after the
        # work that produced `tokens` and initialised the output tensors.
        st = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        rc = self.lib.megakernel_decode_n(self._handle, tokens.data_ptr(), int(n_forced), int(n_steps),
                                          out.data_ptr(), lp, st)
        _lib.check(rc, "megakernel_decode_n")
        return out

    def prefill(self, tokens: torch.Tensor, stream=None) -> torch.Tensor:
        """Parallel prefill (megakernel_prefill): feed the int32 device tensor
        `tokens` at the current position, 64 positions per batched tcgen05
        step; returns the greedy next token as a 1-element device tensor."""
        assert tokens.dtype == torch.int32 and tokens.is_contiguous()
        nxt = torch.empty(1, dtype=torch.int32, device=tokens.device)
        # Default: torch's current stream, so the launch is ordered after the
        # work that produced `tokens` and initialised the output tensors.
        st = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        rc = self.lib.megakernel_prefill(self._handle, tokens.data_ptr(), int(tokens.numel()), nxt.data_ptr(), st)
        _lib.check(rc, "megakernel_prefill")
        return nxt

    def tp_ipc_handle(self) -> bytes:
        """64-byte CUDA IPC handle of this rank's exchange buffer."""
        buf = ctypes.create_string_buffer(64)
        _lib.check(self.lib.megakernel_tp_ipc_handle(self._handle, buf), "megakernel_tp_ipc_handle")
        return buf.raw

    def tp_connect(self, handles):
        """Map every rank's exchange buffer (handles in rank order)."""
        assert len(handles) == self.tp_size and all(len(h) == 64 for h in handles)
        buf = ctypes.create_string_buffer(b"".join(handles), 64 * self.tp_size)
        _lib.check(self.lib.megakernel_tp_connect(self._handle, buf), "megakernel_tp_connect")

    def set_merge_mode(self, mode: int):
        """0 auto (default), 1 direct attention merge, 2 two-level merge instance."""
        _lib.check(self.lib.megakernel_set_merge_mode(self._handle, int(mode)), "megakernel_set_merge_mode")

    def set_logits_capture(self, enable=True):
        _lib.check(self.lib.megakernel_set_logits_capture(self._handle, int(enable)))

    def logits(self) -> np.ndarray:
        out = np.empty(self.vocab, dtype=np.float32)
        _lib.check(self.lib.megakernel_get_logits(
            self._handle, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float))))
        return out


def _device_view(ptr: int, shape, dtype, device) -> torch.Tensor:
    """Wrap externally owned device memory as a tensor (via __cuda_array_interface__)."""
    typestr = {torch.bfloat16: "<i2", torch.float32: "<f4", torch.int32: "<i4"}[dtype]

    class _Holder:
        __cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                    "data": (ptr, False), "version": 3, "strides": None}

    t = torch.as_tensor(_Holder(), device=device)
    return t.view(dtype) if dtype == torch.bfloat16 else t
