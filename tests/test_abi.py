"""The C ABI without a GPU: the library loads, exports every symbol include/enx.h declares,
and rejects bad arguments with a status (no CUDA work involved)."""

import ctypes as C
import re
import subprocess

import pytest

from conftest import ROOT


@pytest.fixture(scope="module")
def lib():
    from enargeia_b200 import build, _lib

    build.build()
    return _lib.load()


def declared():
    h = (ROOT / "include" / "enx.h").read_text()
    return sorted(set(re.findall(r"ENX_API\s+[\w\s\*]+?\b(enx_\w+)\s*\(", h)))


def test_every_declared_symbol_is_exported(lib):
    names = declared()
    assert len(names) >= 30
    out = subprocess.run(["nm", "-D", "--defined-only", str(ROOT / "enargeia_b200" / "libenx.so")],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r" T (enx_\w+)", out))
    assert set(names) <= exported, set(names) - exported
    from enargeia_b200._lib import SIGNATURES
    assert set(names) == set(SIGNATURES), set(names) ^ set(SIGNATURES)


def test_version(lib):
    assert b"sm_100a" in lib.enx_version()


def test_null_arguments_are_rejected(lib):
    from enargeia_b200._lib import MatmulQ4Dims, check, EnxError

    d = MatmulQ4Dims(1, 8, 64, 0, 64, 1, 8, 0, 8, 0, 0, 0)
    assert lib.enx_matmul_q4(None, None, None, None, None, None, C.byref(d), None) == 1
    assert b"null" in lib.enx_last_error()
    with pytest.raises(EnxError):
        check(1)


def test_bad_dims_are_rejected(lib):
    from enargeia_b200._lib import MatmulQ4Dims

    d = MatmulQ4Dims(1, 8, 60, 0, 64, 1, 8, 0, 8, 0, 0, 0)
    p = C.c_void_p(16)
    assert lib.enx_matmul_q4(p, p, p, p, None, p, C.byref(d), None) == 1
    assert b"multiple of 64" in lib.enx_last_error()


def test_workspace_sizes(lib):
    # float attention scores: heads x positions rounded up to the 64-position split
    assert lib.enx_attn_decode_workspace_bytes(2048, 14, 64) == 14 * 2048 * 4
    assert lib.enx_attn_decode_workspace_bytes(100, 14, 64) == 14 * 128 * 4
    assert lib.enx_attn_prefill_workspace_bytes(256, 2048, 14, 64) == 256 * 14 * 2048 * 4
