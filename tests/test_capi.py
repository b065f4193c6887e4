"""The C-ABI library loads and exports exactly what include/fa4cp_b200.h declares.

Host-side argument validation of the boundary is exercised too; every call here
returns before any CUDA API call, so no GPU is needed.
"""

import ctypes
import os
import re
import subprocess

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "fa4cp_b200.h")


def _declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"FA4CP_API\s+[\w\s\*]+?\b(fa4cp_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from fa4_ring import _build, _lib
    _build.build()
    return _lib.load()


def test_header_declares_the_boundary():
    names = _declared()
    for n in ("fa4cp_attn_fwd", "fa4cp_merge_state_inplace", "fa4cp_merge_states",
              "fa4cp_zigzag_shard", "fa4cp_zigzag_unshard", "fa4cp_half_index"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    from fa4_ring import _lib
    for name in _declared():
        assert hasattr(lib, name), name
    assert set(_declared()) == set(_lib.EXPORTED)
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True).stdout
    exported = sorted(set(re.findall(r" T (fa4cp_\w+)", out)))
    assert exported == _declared()


def test_version_and_error_text(lib):
    assert lib.fa4cp_version() >= 100
    rc = lib.fa4cp_merge_states(None, None, 0, None, None, 1, 1, 8, 1, None)
    assert rc == -1
    assert b"num_states" in lib.fa4cp_last_error()


@pytest.mark.parametrize("args,needle", [
    # bad head ratio
    (dict(hq=6, hkv=4), b"multiple"),
    # unknown pattern
    (dict(pattern=7), b"pattern"),
    # unsupported dtype combination
    (dict(in_dtype=2), b"dtype"),
])
def test_attn_argument_validation(lib, args, needle):
    a = dict(hq=8, hkv=2, pattern=0, in_dtype=1)
    a.update(args)
    dummy = ctypes.c_void_p(16)
    rc = lib.fa4cp_attn_fwd(dummy, dummy, dummy, dummy, dummy, dummy, dummy, 1, 128, 128, 128,
                            a["hq"], a["hkv"], 128, a["in_dtype"], 1, a["pattern"], 1, 0.1,
                            None, None, None, 0, None)
    assert rc == -1
    assert needle in lib.fa4cp_last_error()


def test_kv8_sizes_that_would_overflow_are_rejected(lib):
    """A K/V row count whose bf16 byte count overflows int64 (2^56 rows x 1 head x 64 dims
    x 4 bytes = 2^64) gives -1 from the workspace-size helper, and both kv8 entry points
    reject it before any device work (the no-alloc one by its division bound)."""
    big = 1 << 56
    assert lib.fa4cp_attn_kv8_workspace_bytes(big, 1, 64) == -1
    assert lib.fa4cp_attn_kv8_workspace_bytes((1 << 20), 8, 128) == (1 << 20) * 8 * 128 * 4
    assert lib.fa4cp_attn_kv8_workspace_bytes(-1, 8, 128) == -1
    dummy = ctypes.c_void_p(256)
    common = [dummy] * 7 + [1, 128, 128, big, 8, 1, 64, 1, 0, 1, 0.125, None, None, 0]
    rc = lib.fa4cp_attn_fwd_kv8(*common, dummy, 1 << 40, None)
    assert rc == -1 and b"overflow" in lib.fa4cp_last_error()
    rc = lib.fa4cp_attn_fwd_kv8_noalloc(*common, None)
    assert rc == -1 and b"scratch" in lib.fa4cp_last_error()
    # one element past the 32 MiB scratch: K and V of 8,388,608 + 1 elements each
    common[10] = (1 << 23) // 64 + 1
    rc = lib.fa4cp_attn_fwd_kv8_noalloc(*common, None)
    assert rc == -1 and b"scratch" in lib.fa4cp_last_error()


def test_backward_argument_validation(lib):
    dummy = ctypes.c_void_p(16)

    def bwd(dtype=1, pattern=0, hq=8, hkv=2, d=128):
        return lib.fa4cp_attn_bwd(dummy, dummy, dummy, dummy, dummy, dummy, dummy, dummy, dummy,
                                  dummy, dummy, 1, 128, 128, 128, hq, hkv, d, dtype, pattern, 1,
                                  0.1, None)

    assert bwd(dtype=3) == -1 and b"f16 or bf16" in lib.fa4cp_last_error()  # no e4m3 backward
    assert bwd(pattern=5) == -1 and b"pattern" in lib.fa4cp_last_error()
    assert bwd(hq=6, hkv=4) == -1 and b"multiple" in lib.fa4cp_last_error()
    assert bwd(d=256) == -2 and b"head_dim" in lib.fa4cp_last_error()        # unsupported
    assert lib.fa4cp_attn_bwd_preprocess(dummy, dummy, dummy, 4, 2, 128, 2, None) == -1
    assert lib.fa4cp_add_f32(dummy, dummy, 6, None) == -1                     # 6 % 4 != 0
    assert lib.fa4cp_convert_f32(dummy, dummy, 4, 3, None) == -1              # no e4m3 target


def test_ring_handles_are_checked(lib):
    """A handle the library did not hand out (or already destroyed) is an argument error,
    never dereferenced."""
    bogus = 0x7F00DEADBEE0
    for call in (lambda: lib.fa4cp_ring_set_fused(bogus, 1),
                 lambda: lib.fa4cp_ring_set_sm_reserve(bogus, 4),
                 lambda: lib.fa4cp_ring_ipc_close(bogus),
                 lambda: lib.fa4cp_ring_timing(bogus, 4),
                 lambda: lib.fa4cp_ring_comm_destroy(bogus)):
        assert call() == -1
        assert b"unknown ring handle" in lib.fa4cp_last_error()


def test_zigzag_argument_validation(lib):
    dummy = ctypes.c_void_p(16)
    assert lib.fa4cp_zigzag_shard(dummy, dummy, None, 1, 10, 0, 2, 4, None) == -1  # 10 % 4 != 0
    assert b"divisible" in lib.fa4cp_last_error()
    assert lib.fa4cp_zigzag_shard(dummy, dummy, None, 1, 8, 2, 2, 4, None) == -1   # rank >= cp
    assert lib.fa4cp_half_index(dummy, 1, 7, 1, dummy, None) == -1                  # odd total


def test_header_is_c_and_library_links_from_c(lib, tmp_path):
    """include/fa4cp_b200.h compiles as C; a C program links the library and calls the
    host-only entry points (tests/c_abi/c_abi_check.c)."""
    from fa4_ring import _lib
    src = os.path.join(ROOT, "tests", "c_abi", "c_abi_check.c")
    exe = str(tmp_path / "c_abi_check")
    libdir = os.path.dirname(_lib.LIB_PATH)
    cc = subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                         src, "-o", exe, "-L", libdir, "-l:" + os.path.basename(_lib.LIB_PATH),
                         "-Wl,-rpath," + libdir], capture_output=True, text=True)
    assert cc.returncode == 0, cc.stderr
    run = subprocess.run([exe], capture_output=True, text=True)
    assert run.returncode == 0, (run.returncode, run.stdout, run.stderr)
    assert "c abi ok" in run.stdout
