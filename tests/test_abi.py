"""The C-ABI library loads and exports every entry point include/sokutou_b200.h declares; argument
validation answers with error codes before touching any device (no GPU needed)."""

import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "sokutou_b200.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^SK_API\s+(?:int|size_t)\s+(sk_\w+)\s*\(", src, re.M)))


def test_header_declares_the_boundary():
    syms = declared_symbols()
    for s in ("sk_dit_attention", "sk_dit_qkv_prologue", "sk_decode_attention", "sk_decode_workspace_bytes",
              "sk_device_error", "sk_version"):
        assert s in syms


def test_library_exports_every_declared_symbol(native_lib):
    for s in declared_symbols():
        assert hasattr(native_lib, s), s
    from sokutou_b200 import _lib
    assert set(_lib.SIGNATURES) == set(declared_symbols())


def test_version(native_lib):
    assert native_lib.sk_version() >= 100


def test_argument_errors_without_device(native_lib):
    P = ctypes.c_void_p
    fake = P(4096)  # never dereferenced: validation fails first
    # null q
    assert native_lib.sk_dit_attention(None, fake, fake, None, None, None, fake, 1, 1, 1, 1, 0, 64, 0, 0, 0, 0.0, None) == -1
    # unsupported head dim
    assert native_lib.sk_dit_attention(fake, fake, fake, None, None, None, fake, 1, 1, 1, 1, 0, 96, 0, 0, 0, 0.0, None) == -2
    # misaligned pointer
    assert native_lib.sk_dit_attention(P(4100), fake, fake, None, None, None, fake, 1, 1, 1, 1, 0, 64, 0, 0, 0, 0.0, None) == -1
    # unsupported dtype
    assert native_lib.sk_dit_attention(fake, fake, fake, None, None, None, fake, 1, 1, 1, 1, 0, 64, 0, 0, 7, 0.0, None) == -2
    # decode: nq must be 2*nkv, hd 128
    f = ctypes.c_float
    assert native_lib.sk_decode_attention(fake, fake, fake, f(1e-6), fake, fake, fake, None, 0, 16, 4, 4, 128, fake,
                                          None, 0, 0, None) == -2
    assert native_lib.sk_decode_attention(fake, fake, fake, f(1e-6), fake, fake, fake, None, 0, 16, 4, 2, 64, fake,
                                          None, 0, 0, None) == -2
    # decode: split-KV needs a workspace when max_len spans several chunks
    assert native_lib.sk_decode_attention(fake, fake, fake, f(1e-6), fake, fake, fake, None, 0, 1024, 4, 2, 128, fake,
                                          None, 0, 0, None) == -5
    assert native_lib.sk_decode_workspace_bytes(1024, 16, 8, 128, 0) > 0
    assert native_lib.sk_decode_workspace_bytes(0, 16, 8, 128, 0) == 0


def test_ops_raise_on_missing_library(monkeypatch, tmp_path):
    from sokutou_b200 import _lib
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "missing.so"))
    with pytest.raises(_lib.SokutouError):
        _lib.lib()
