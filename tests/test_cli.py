"""The chpe_fwd command line (the reference's src/main.zig contract): flags,
raw u32 tokens file, raw f32 logits of the last token, receipt lines.  The
CPU tests run only what needs no GPU (help, argument errors, the architecture
rule, the prompt limit); the GPU test decodes a synthetic archive and checks
the logits file against the oracle."""
import os
import re
import struct
import subprocess

import numpy as np
import pytest

import chpe_qwen_engine_b200 as chpe
import oracle_py as O
from chpe_qwen_engine_b200 import build as B
from _util import archive, assert_logits_match, oracle_threads


def _cli():
    if not os.path.exists(B.CHPE_FWD):
        B.build_all()
    return B.CHPE_FWD


def test_cli_help_and_missing_archive(tmp_path):
    r = subprocess.run([_cli(), "--help"], capture_output=True, text=True)
    assert r.returncode == 0
    for flag in ("--archive", "--tokens-file", "--out-logits", "--arch", "--bench", "--max-seq-len"):
        assert flag in r.stderr
    r = subprocess.run([_cli(), "--archive", str(tmp_path / "none.chpe")], capture_output=True, text=True)
    assert r.returncode == 1 and "Failed to open weight archive" in r.stderr
    toks = tmp_path / "empty.bin"
    toks.write_bytes(b"")
    arc = tmp_path / "x.chpe"
    arc.write_bytes(b"\0" * 64)
    r = subprocess.run([_cli(), str(arc), "--tokens-file", str(toks)], capture_output=True, text=True)
    assert r.returncode == 1 and "EmptyTokensFile" in r.stderr


@pytest.mark.parametrize("name,override,want", [
    ("Qwen2.5-3B.w2.chpe", None, "Qwen2.5-3B"),
    ("Qwen3.5-9B.w4.chpe", None, "Qwen3.5-9B"),
    ("qwen35.w4.chpe", None, "Qwen3.5-9B"),
    ("qwen2.5-72b.w4.chpe", None, "Qwen2.5-72B"),
    ("Qwen2.5-3B.w2.chpe", "qwen2_5_72b", "Qwen2.5-72B"),
    ("Qwen2.5-72B.chpe", "qwen3_5_9b", "Qwen3.5-9B"),
])
def test_cli_arch_rule_and_prompt_limit(tmp_path, name, override, want):
    """src/main.zig:86-106: --arch wins, else the archive path's substring
    picks the model; a prompt longer than --max-seq-len is refused before any
    GPU work; the receipt lines report the archive's record count."""
    arc = tmp_path / name
    hdr = struct.pack("<IIQQQQQQQ", 0x57415243, 1, 4096, 7, 7, 20480, 17408, 3072, 0)
    arc.write_bytes(hdr + b"\0" * (4096 - len(hdr)))
    toks = tmp_path / "p.bin"
    np.arange(5, dtype="<u4").tofile(toks)
    cmd = [_cli(), str(arc), "--tokens-file", str(toks), "--max-seq-len", "4"]
    if override:
        cmd += ["--arch", override]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 1
    assert f"Model Arch     : {want} " in r.stderr
    assert "7 tiles" in r.stderr
    assert "Loaded 5 tokens" in r.stderr and "5 tokens exceed --max-seq-len 4" in r.stderr


@pytest.mark.gpu
def test_cli_decodes_and_writes_logits(tmp_path):
    path = tmp_path / "Qwen2.5-3B.w2.chpe"
    chpe.synth_write(str(path), chpe.SYNTH_3B_W2)
    toks = np.array([151644, 872, 9707, 11, 3000], np.uint32)
    tf = tmp_path / "prompt.bin"
    toks.astype("<u4").tofile(tf)
    out = tmp_path / "logits.bin"
    r = subprocess.run([_cli(), "--archive", str(path), "--tokens-file", str(tf), "--out-logits", str(out),
                        "--bench", "2", "--max-seq-len", "64"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    got = np.fromfile(out, dtype=np.float32)
    a = archive(chpe.SYNTH_3B_W2)
    o = O.OracleEngine(a, O.ARCH_3B, 64, threads=oracle_threads())
    for p, t in enumerate(toks):
        rr = o.forward_decode(int(t), p)
    assert got.size == 151936
    assert_logits_match(got, o.logits(), "chpe_fwd logits")
    m = re.search(r"Argmax Decoded Token ID : (\d+)", r.stderr)
    assert m and int(m.group(1)) == int(np.argmax(got))
    assert "[Iter 2/2]" in r.stderr and "Throughput" in r.stderr
    assert "100% FINITE" in r.stderr
