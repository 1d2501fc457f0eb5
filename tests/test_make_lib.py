"""`make lib` builds megakernel.so for sm_100a (cross-compiled, no GPU) and it
exports the reference's six C symbols (src/megakernel.cu:544-622) and every
extension include/megakernel.h declares."""
import os
import shutil
import subprocess

import pytest

from megakernel_b200 import launcher

from .test_abi import header_functions

REFERENCE_SYMBOLS = ["megakernel_init", "megakernel_decode", "megakernel_reset", "megakernel_get_pos",
                     "megakernel_free", "megakernel_sync"]


@pytest.mark.skipif(shutil.which("nvcc") is None and not os.path.exists("/usr/local/cuda/bin/nvcc"),
                    reason="nvcc not available")
def test_make_lib_exports(tmp_path):
    out = launcher.compile_shared_library(output=str(tmp_path / "megakernel.so"))
    assert os.path.exists(out)
    nm = subprocess.run(["nm", "-D", "--defined-only", out], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in nm.splitlines() if " T " in line}
    for name in REFERENCE_SYMBOLS + header_functions():
        assert name in exported, name
