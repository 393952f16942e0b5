"""The synthetic archive generator: deterministic, valid, laid out where the
reference's tensor maps look (CPU only)."""
import hashlib
import struct

import numpy as np

import chpe_qwen_engine_b200 as chpe
import oracle_py as O


def test_sizes_match_reference_record_counts():
    assert chpe.synth_lib().chpe_synth_bytes(chpe.SYNTH_3B_FP16_RAW, 0) == 4096 + 376853 * 16384
    assert chpe.synth_lib().chpe_synth_bytes(chpe.SYNTH_3B_W4, 0) == 4096 + 94349 * 17408
    assert chpe.synth_lib().chpe_synth_bytes(chpe.SYNTH_3B_W4, chpe.SYNTH_STANDARD) == 4096 + 94349 * 20480
    assert chpe.synth_lib().chpe_synth_bytes(chpe.SYNTH_9B_W4, 0) == 4096 + 546681 * 17408
    assert chpe.synth_lib().chpe_synth_bytes(chpe.SYNTH_72B_W4, 0) == 4096 + 2219153 * 17408


def test_deterministic_across_thread_counts():
    a = chpe.synth_archive(chpe.SYNTH_3B_W2, 0, seed=7, threads=1)
    b = chpe.synth_archive(chpe.SYNTH_3B_W2, 0, seed=7, threads=5)
    assert hashlib.sha256(a).digest() == hashlib.sha256(b).digest()
    c = chpe.synth_archive(chpe.SYNTH_3B_W2, 0, seed=8, threads=5)
    assert hashlib.sha256(a).digest() != hashlib.sha256(c).digest()


def test_layout_seen_by_oracle():
    a = chpe.synth_archive(chpe.SYNTH_3B_W4)
    assert O.validate(a)[0] == 0
    e = O.OracleEngine(a, O.ARCH_3B, 8)
    f = e.facts()
    assert f["is_dense"] == 1 and f["quant_bits"] == 4 and f["weights_per_tile"] == 32768
    li = e.layer_info(0)
    assert np.all(e.unpack_norm(li["input_norm"], 2048) == 1.0)
    assert np.all(e.unpack_bias(li["q_bias"], 2048) == 0.0)
    # a row-tiled q cell: 4-bit, group-128 flag, 16 x 2048
    off = 4096 + li["q_proj"] * 17408 + 16448
    assert a[off + 20] == 4
    flags = struct.unpack("<Q", a[off + 24:off + 32].tobytes())[0]
    rows, cols = struct.unpack("<II", a[off + 40:off + 48].tobytes())
    assert flags & 1 and rows == 16 and cols == 2048


def test_raw_fp16_layout():
    n = chpe.synth_lib().chpe_synth_bytes(chpe.SYNTH_3B_FP16_RAW, 0)
    a = np.empty(n, np.uint8)
    assert chpe.synth_lib().chpe_synth_fill(chpe.SYNTH_3B_FP16_RAW, 0, 0, a.ctypes.data, n, 8) == 0
    e = O.OracleEngine(a, O.ARCH_3B, 8)
    f = e.facts()
    assert f["is_raw"] == 1 and f["is_raw_fp16"] == 1 and f["weights_per_tile"] == 8192
    w = a[4096 + 37984 * 16384 + 16384:4096 + 37984 * 16384 + 2 * 16384].view(np.float16).astype(np.float32)
    assert 0.015 < float(w.std()) < 0.025
