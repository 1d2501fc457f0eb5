"""Build and load ``libmegakernel.so`` (the C ABI declared in include/megakernel.h).

The library is built in-tree with nvcc for sm_100a only.  Loading never falls
back to anything: if the shared library is missing or lacks a symbol, the
caller gets an exception.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_PATH = os.path.join(PKG_DIR, "libmegakernel.so")
HEADER = os.path.join(ROOT, "include", "megakernel.h")
SOURCES = [os.path.join(CSRC, f) for f in ("megakernel.cu", "noalloc.cu", "decode_kernel.cuh", "ptx.cuh",
                                                  "shapes.cuh", "batch.cu", "tc_gemm.cuh", "tc_ptx.cuh",
                                                  "tp.cu")]
# Translation units, compiled in parallel and linked into one library.
UNITS = ["megakernel.cu", "tp.cu"]

NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
              "-Xcompiler", "-fPIC"]

MK_OK = 0
ERRORS = {0: "ok", -1: "invalid argument", -2: "CUDA runtime error", -3: "in-kernel wait timed out",
          -4: "KV capacity exceeded", -5: "offsets match no compiled model shape",
          -6: "cooperative launch not possible", -7: "device allocation failed"}


def nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile libmegakernel.so in-tree if it is missing or older than its sources."""
    if not force and os.path.exists(LIB_PATH):
        lib_m = os.path.getmtime(LIB_PATH)
        if all(os.path.getmtime(s) <= lib_m for s in SOURCES + [HEADER]):
            return LIB_PATH
    objs, procs = [], []
    for u in UNITS:
        obj = os.path.join(PKG_DIR, u.replace(".cu", ".o"))
        cmd = [nvcc()] + NVCC_FLAGS + (["-Xptxas=-v"] if verbose else []) + \
            ["-c", os.path.join(CSRC, u), "-o", obj]
        objs.append(obj)
        procs.append(subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True))
    errs = []
    for p in procs:
        _, err = p.communicate()
        if p.returncode != 0:
            errs.append(err)
        elif verbose:
            print(err)
    if errs:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errs))
    r = subprocess.run([nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared"] + objs +
                       ["-o", LIB_PATH + ".tmp"], capture_output=True, text=True)
    for o in objs:
        os.remove(o)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{r.stderr}")
    os.replace(LIB_PATH + ".tmp", LIB_PATH)
    return LIB_PATH


class MkOptions(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("shape_id", ctypes.c_int), ("max_seq", ctypes.c_int),
                ("num_ctas", ctypes.c_int), ("timeout_ns", ctypes.c_longlong),
                ("debug_skip_cta", ctypes.c_int)]


def signatures() -> dict:
    """name -> (argtypes, restype) for every function include/megakernel.h declares."""
    c_int, c_ll, vp = ctypes.c_int, ctypes.c_longlong, ctypes.c_void_p
    ip = ctypes.POINTER(ctypes.c_int)
    llp = ctypes.POINTER(ctypes.c_longlong)
    fp = ctypes.POINTER(ctypes.c_float)
    return {
        # reference surface (host/bridge.py:39-67)
        "megakernel_init": ([vp, llp, c_int], vp),
        "megakernel_decode": ([vp, c_int], c_int),
        "megakernel_reset": ([vp], None),
        "megakernel_get_pos": ([vp], c_int),
        "megakernel_free": ([vp], None),
        "megakernel_sync": ([], None),
        # extensions
        "megakernel_default_options": ([ctypes.POINTER(MkOptions)], None),
        "megakernel_init_ex": ([vp, llp, c_int, ctypes.POINTER(MkOptions), ctypes.POINTER(vp)], c_int),
        "megakernel_decode_n": ([vp, vp, c_int, c_int, vp, vp, vp], c_int),
        "megakernel_generate": ([vp, ip, c_int, c_int, ip], c_int),
        "megakernel_set_logits_capture": ([vp, c_int], c_int),
        "megakernel_get_logits": ([vp, fp], c_int),
        "megakernel_set_pos": ([vp, c_int], c_int),
        "megakernel_kv_ptr": ([vp], vp),
        "megakernel_kv_bytes": ([vp], c_ll),
        "megakernel_max_seq": ([vp], c_int),
        "megakernel_shape_id": ([vp], c_int),
        "megakernel_num_ctas": ([vp], c_int),
        "megakernel_set_merge_mode": ([vp, c_int], c_int),
        "megakernel_last_error": ([vp], c_int),
        "megakernel_error_string": ([c_int], ctypes.c_char_p),
        "megakernel_set_trace": ([vp, vp, c_int], c_int),
        "megakernel_trace_points": ([vp], c_int),
        "megakernel_set_trace_detail": ([vp, vp], c_int),
        "megakernel_decode_noalloc": ([vp, llp, c_int, vp, c_int, c_int, vp, c_int, c_int, vp, vp, vp],
                                      c_int),
        "megakernel_tc_gemm_test": ([vp, c_int, vp, c_int, c_int, vp, vp], c_int),
        "megakernel_tc_gemm_test_split": ([vp, c_int, vp, c_int, c_int, c_int, vp, vp], c_int),
        "megakernel_tc_gemm_test_e4m3": ([vp, c_int, vp, vp, c_int, c_int, vp, vp], c_int),
        "megakernel_prefill": ([vp, vp, c_int, vp, vp], c_int),
        "megakernel_batch_init": ([vp, llp, c_int, c_int, c_int], vp),
        "megakernel_batch_init_ex": ([vp, llp, c_int, c_int, c_int, c_int], vp),
        "megakernel_batch_free": ([vp], None),
        "megakernel_batch_size": ([vp], c_int),
        "megakernel_batch_step": ([vp, vp, vp, vp, vp], c_int),
        "megakernel_batch_decode_n": ([vp, vp, c_int, c_int, vp, vp], c_int),
        "megakernel_batch_set_pos": ([vp, ip], c_int),
        "megakernel_batch_get_pos": ([vp, ip], c_int),
        "megakernel_batch_kv_ptr": ([vp], vp),
        "megakernel_batch_kv_bytes": ([vp], c_ll),
        "megakernel_batch_last_error": ([vp], c_int),
        "megakernel_tp_init": ([vp, llp, c_int, ctypes.POINTER(MkOptions), c_int, c_int, ctypes.POINTER(vp)],
                               c_int),
        "megakernel_tp_ipc_handle": ([vp, vp], c_int),
        "megakernel_tp_connect": ([vp, vp], c_int),
        "megakernel_tp_info": ([vp, ip, ip], c_int),
        "megakernel_tp_exchange_slots": ([vp, vp], c_int),
        "megakernel_infer_shape": ([llp, c_int], c_int),
        "megakernel_rope_table": ([c_int, ctypes.c_double, c_int, fp, fp], c_int),
        "megakernel_plan_bytes": ([c_int, c_int, c_int, llp], c_int),
    }


def _declare(lib: ctypes.CDLL) -> ctypes.CDLL:
    for name, (args, res) in signatures().items():
        f = getattr(lib, name)
        f.argtypes = args
        f.restype = res
    return lib


_LIB = None


def load(path: str | None = None) -> ctypes.CDLL:
    """Load the in-tree library (raises if it has not been built)."""
    global _LIB
    if path is None and _LIB is not None:
        return _LIB
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise RuntimeError(f"{p} is missing: run megakernel_b200._lib.build() (needs nvcc)")
    lib = _declare(ctypes.CDLL(p))
    if path is None:
        _LIB = lib
    return lib


def check(rc: int, what: str = "megakernel") -> None:
    if rc != MK_OK:
        raise RuntimeError(f"{what}: {ERRORS.get(rc, rc)} ({rc})")
