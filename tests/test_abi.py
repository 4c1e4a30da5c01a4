"""The C-ABI library loads and exports every entry point the header declares.

No kernel is launched here (CPU-only); the host-side helpers that need no
device (workspace sizing, status strings) are exercised.
"""

import os
import re
import subprocess

import pytest

from kshipra_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "kshipra_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ksh_[a-z0-9_]+)\s*\(", src)))


def test_library_exists_and_loads():
    assert os.path.exists(_lib.LIB_PATH), "run `python -m kshipra_b200.build`"
    h = _lib.lib()
    assert h.ksh_abi_version() == 1


def test_every_declared_symbol_is_exported():
    names = declared_functions()
    assert len(names) >= 20
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (ksh_[a-z0-9_]+)", out))
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    # and the ctypes table covers them all
    assert set(names) <= set(_lib.SIGNATURES), set(names) - set(_lib.SIGNATURES)


def test_status_strings():
    h = _lib.lib()
    assert h.ksh_status_string(0) == b"ok"
    for st in (-1, -2, -3, -4, -5):
        assert h.ksh_status_string(st) != b"unknown status"


def test_workspace_helpers_need_no_device():
    h = _lib.lib()
    ws = h.ksh_paged_attention_workspace_size(1, 14, 2, 64, 1, 562)
    assert ws > 0 and ws % 256 == 0
    assert h.ksh_paged_attention_workspace_size(64, 32, 8, 128, 1, 4096) >= 64 * 8 * 4
    assert h.ksh_lm_head_workspace_size(1, 151936) > 256
    assert h.ksh_paged_attention_workspace_size(1, 3, 2, 64, 1, 10) == 0   # bad GQA ratio


def test_argument_errors_are_reported_without_a_launch():
    h = _lib.lib()
    # n == 0 is a shape error; detected on the host before any launch
    assert h.ksh_pack_int8(None, 0, 4, None, None, None, None) == -1
    assert h.ksh_pack_int4(None, 4, 4, 3, None, None, None, None) == -1
    with pytest.raises(_lib.KshipraLibraryError):
        _lib.call("ksh_rmsnorm", None, None, None, 1, 0, 1e-6, None)


def test_bounded_wait_check_rejects_bad_limits_on_the_host():
    h = _lib.lib()
    fake = 256          # never dereferenced: the limits are checked before any launch
    assert h.ksh_check_bounded_wait(0, 0, fake, fake, None, None) == -1
    assert h.ksh_check_bounded_wait(1 << 25, 0, fake, fake, None, None) == -1
    assert h.ksh_check_bounded_wait(100, 0, None, fake, None, None) == -1


def test_noalloc_scratch_covers_the_largest_argmax_grid():
    """The fused lm_head GEMV's argmax grid is at most 8 CTAs per SM
    (gemv.cu, gemv_argmax_grid) and keeps one (max, index) pair of 8 bytes
    per CTA and row behind a 256-byte header; for the 16 rows the
    no-allocation entry point accepts, on a 148-SM B200, that must fit its
    fixed array."""
    h = _lib.lib()
    sms, max_rows = 148, 16
    assert 256 + sms * 8 * max_rows * 8 <= h.ksh_lm_head_argmax_noalloc_max_bytes()
