"""Build helpers with the reference's launcher names (host/launcher.py).

``compile_shared_library`` replaces host/launcher.py:103-132: it builds
``megakernel.so`` -- the library a reference caller loads through ctypes --
by running this repository's ``make lib`` (sm_100a only; no GPU needed to
compile).  ``detect_gpu`` reports the current device the way the reference's
helper does, for callers that print it.
"""
from __future__ import annotations

import os
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def detect_gpu() -> dict:
    """Name and arch flag of device 0 (the library itself targets sm_100a only)."""
    import torch
    if not torch.cuda.is_available():
        return {"name": None, "arch_flag": "sm_100a", "class": "B200 (no device visible)"}
    p = torch.cuda.get_device_properties(0)
    return {"name": p.name, "arch_flag": f"sm_{p.major}{p.minor}a", "class": p.name}


def compile_shared_library(src_dir=None, output="megakernel.so", gpu_info=None) -> str:
    """Build the C-ABI library at `output` (relative paths: the repository
    root) with `make lib`; returns its absolute path.  `src_dir` and
    `gpu_info` are accepted for call compatibility and ignored: the sources
    are this package's csrc/ and the target is always sm_100a."""
    out = output if os.path.isabs(output) else os.path.join(ROOT, output)
    r = subprocess.run(["make", "-s", "-C", ROOT, "lib", f"LIB_OUT={out}"], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"make lib failed:\n{r.stderr[-2000:]}")
    return out
