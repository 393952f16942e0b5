"""The C-ABI library loads and exports every symbol include/chpe.h declares;
host-only semantics that need no GPU (NULL handling, validation, path and
init failures, and the engine's refusal to start without a usable GPU).  No
compute call is made here."""
import ctypes as C
import os
import re
import struct

import numpy as np
import pytest

import chpe_qwen_engine_b200 as chpe
import oracle_py as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    src = open(os.path.join(ROOT, "include", "chpe.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(chpe_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    L = C.CDLL(chpe.LIBCHPE_PATH)
    names = header_symbols()
    assert len(names) >= 25
    for n in names:
        assert hasattr(L, n), n
    bound = {n for n, _, _ in chpe.SYMBOLS}
    assert bound == set(names)


def test_reference_symbols_present():
    # chpe_c_api.zig:25-143
    ref = ["chpe_init", "chpe_forward_tokens", "chpe_get_last_logits", "chpe_get_vocab_size",
           "chpe_get_hidden_dim", "chpe_get_num_layers", "chpe_get_last_elapsed_ns",
           "chpe_get_last_argmax", "chpe_get_last_max_logit", "chpe_get_last_token0_logit",
           "chpe_get_last_hidden_norm", "chpe_free"]
    assert set(ref) <= set(header_symbols())


def test_null_context_semantics():
    L = chpe.lib()
    # NULL ctx answers for Qwen2.5-3B (chpe_c_api.zig:89-105), 0 for results (:107-135)
    assert L.chpe_get_vocab_size(None) == 151936
    assert L.chpe_get_hidden_dim(None) == 2048
    assert L.chpe_get_num_layers(None) == 36
    assert L.chpe_get_last_elapsed_ns(None) == 0
    assert L.chpe_get_last_argmax(None) == 0
    assert L.chpe_get_last_max_logit(None) == 0.0
    assert L.chpe_get_last_token0_logit(None) == 0.0
    assert L.chpe_get_last_hidden_norm(None) == 0.0
    toks = np.array([1, 2], np.uint32)
    assert L.chpe_forward_tokens(None, toks.ctypes.data_as(C.POINTER(C.c_uint32)), 2, None) == -1
    out = np.zeros(4, np.float32)
    assert L.chpe_get_last_logits(None, out.ctypes.data_as(C.POINTER(C.c_float)), 4) == 0
    L.chpe_free(None)


def test_init_missing_path_returns_null():
    assert chpe.lib().chpe_init(b"/nonexistent/archive.chpe") is None
    assert chpe.lib().chpe_last_error(None)


def _hdr(magic=0x57415243, version=1, header_bytes=4096, count=0, rec=20480, cell=17408, pre=3072,
         flags=0):
    return struct.pack("<IIQQQQQQQ", magic, version, header_bytes, count, count, rec, cell, pre, flags)


def test_validate_matches_oracle():
    cases = []
    cases.append(bytearray(100))
    b = bytearray(4096); b[:64] = _hdr(magic=0xDEADBEEF); cases.append(b)
    b = bytearray(4096); b[:64] = _hdr(rec=20544); cases.append(b)
    b = bytearray(4096); b[:64] = _hdr(count=1); cases.append(b)
    b = bytearray(4096); b[:64] = _hdr(version=2); cases.append(b)
    b = bytearray(4096); b[:64] = _hdr(header_bytes=64); cases.append(b)
    b = bytearray(4096 + 17408); b[:64] = _hdr(magic=0x45504843, count=1, rec=17408, pre=0); cases.append(b)
    b = bytearray(4096 + 16384); b[:64] = _hdr(count=1, rec=16384, cell=16384, pre=0); cases.append(b)
    b = bytearray(4096 + 16384); b[:64] = _hdr(count=1, rec=16384, cell=17408, pre=0); cases.append(b)
    for c in cases:
        assert chpe.validate_archive(c) == O.validate(c)[0]


def test_init_rejects_invalid_file(tmp_path):
    p = tmp_path / "bad.chpe"
    p.write_bytes(bytes(8192))
    assert chpe.lib().chpe_init(str(p).encode()) is None
    assert b"validation" in chpe.lib().chpe_last_error(None)


def _gpu_present() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.mark.skipif(_gpu_present(), reason="checks the failure without a usable GPU")
def test_engine_without_gpu_fails_loudly():
    """No CPU fallback: without a usable GPU the engine (the mock archive the
    reference's own test uses, chpe_engine.zig:1893-1933) refuses to start,
    with the CUDA error in the message and through chpe_last_error."""
    with pytest.raises(chpe.ChpeError, match="cuda|CUDA"):
        chpe.Engine.from_bytes(np.zeros(8192, np.uint8), chpe.ARCH_3B, 16)
    buf = np.zeros(8192, np.uint8)
    ctx = chpe.lib().chpe_init_bytes(buf.ctypes.data, buf.size, chpe.ARCH_3B, 16, 0)
    assert ctx is None
    assert b"CUDA" in chpe.lib().chpe_last_error(None) or b"cuda" in chpe.lib().chpe_last_error(None)
