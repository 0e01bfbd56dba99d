"""CPU checks of the C ABI: the library loads, exports exactly what
include/flashdecode.h declares, and rejects bad arguments with status codes
before touching a device."""
import ctypes
import os
import re

import pytest

import flashdecode
from flashdecode import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(__file__)), "include", "flashdecode.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"\b([A-Za-z_][A-Za-z0-9_]*)\s*\(", text)
    skip = {"if", "defined"}
    return sorted({n for n in names if n not in skip and (n.startswith("fd_") or n == "run_kernel")})


def test_header_declares_the_reference_entry_point():
    assert "run_kernel" in declared_functions()


def test_library_exports_every_declared_symbol(lib):
    names = declared_functions()
    assert len(names) >= 9
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures out of sync with the header"


def test_version_and_error_strings(lib):
    assert lib.fd_version().decode().startswith("flashdecode-sm100")
    assert lib.fd_error_string(0) == b"ok"
    assert lib.fd_error_string(5) == b"in-kernel wait timed out"
    assert lib.fd_error_string(6) == b"page id outside the KV pool"


def _call(lib, **kw):
    args = dict(q=1024, k=1024, v=1024, out=1024, lse=None, sl=1024, bt=1024, bt_stride=1, B=1,
                Hq=8, Hkv=2, D=128, page=16, num_blocks=4, dtype=0, out_dtype=0, scale=0.1,
                max_len=0, ws=None, ws_bytes=0, stream=None)
    args.update(kw)
    return lib.fd_decode_paged(*args.values())


@pytest.mark.parametrize("kw,code", [
    (dict(q=None), 1), (dict(B=0), 1), (dict(Hkv=3), 1), (dict(page=0), 1),
    (dict(dtype=2), 1), (dict(out_dtype=1), 1), (dict(scale=float("nan")), 1),
    (dict(D=96), 2), (dict(num_blocks=1 << 40), 2),
])
def test_bad_arguments_return_status(lib, kw, code):
    assert _call(lib, **kw) == code
    status, msg = flashdecode.last_error()
    assert status == code and msg


def test_run_kernel_rejects_bad_arguments_silently(lib):
    # Reference semantics: void return, nothing done; the reason is kept.
    flashdecode.run_kernel(None, None, None, None, None, None, 1, 16, 0, 32, 8, 128, 16, 1, 0)
    assert flashdecode.last_error()[0] == 1  # seqlen_q must be >= 1
    flashdecode.run_kernel(None, None, None, None, None, None, 1, 16, 2, 32, 8, 128, 16, 1, 1)
    assert flashdecode.last_error()[0] == 1  # null tensors
    flashdecode.run_kernel(None, None, None, None, None, None, 4, 16, 1, 32, 8, 128, 16, 2, 0)
    assert flashdecode.last_error()[0] == 1  # num_blocks < batch: blocks_per_batch == 0


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(ImportError):
        _lib.load_library(tmp_path / "nope.so")
