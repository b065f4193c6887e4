"""Build the CUDA library in-tree (``make -C fa4-cp_b200/csrc``) for sm_100a."""

import os
import subprocess

CSRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "csrc")


def build(jobs: int = 8, quiet: bool = True) -> str:
    """Compile every kernel of ``csrc/`` into ``fa4_ring/libfa4cp_b200.so``; return its path."""
    from ._lib import LIB_PATH

    res = subprocess.run(["make", "-C", CSRC, f"-j{jobs}"], capture_output=quiet, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"building libfa4cp_b200.so failed:\n{res.stdout}\n{res.stderr}")
    return LIB_PATH
