"""Archive converters (chpe_convert_archive; weight_archive.zig:617-776) against
the oracle's restatement, byte for byte: standard records -> dense cells,
-> raw tiles, -> raw FP16 tiles (BF16 rounded to FP16 on the GPU, 1-D cells
copied verbatim).  The archives are small and hand-built: random bytes, so
every BF16 class occurs (zeros, subnormals, values that overflow FP16, ties,
infinities, NaNs), and some cells marked quant_bits 32 (1-D data).  The
dense and raw conversions need no GPU and also run in the CPU suite."""
import struct

import numpy as np
import pytest

import chpe_qwen_engine_b200 as chpe
import oracle_py as O

N_REC = 3000


def _standard_archive(rng) -> np.ndarray:
    a = rng.integers(0, 256, 4096 + N_REC * 20480, dtype=np.uint8)
    hdr = struct.pack("<IIQQQQQQQ", 0x57415243, 1, 4096, N_REC, N_REC, 20480, 17408, 3072, 0x10)
    a[:4096] = 0
    a[:64] = np.frombuffer(hdr, np.uint8)
    for i in range(N_REC):  # quant_bits of each cell: 32 (1-D) for every 7th, else 16
        a[4096 + i * 20480 + 3072 + 16448 + 20] = 32 if i % 7 == 0 else 16
    return a


def _check(path, src, mode):
    got = np.fromfile(path, np.uint8)
    stride = 17408 if mode == chpe.CONVERT_DENSE else 16384
    assert got.size == 4096 + N_REC * stride
    assert np.array_equal(got[:4096], O.convert_header(src, mode))
    for i in range(N_REC):
        ref = O.convert_record(src, mode, i)
        if not np.array_equal(got[4096 + i * stride:4096 + (i + 1) * stride], ref):
            raise AssertionError(f"mode {mode} record {i} differs")


def test_oracle_rounding_matches_numpy():
    """The oracle's f32 -> f16 rounding against numpy's (nearest, ties to even)
    on every BF16 bit pattern that is not a NaN."""
    b = np.arange(65536, dtype=np.uint32)
    f = (b << 16).view(np.float32)
    keep = ~np.isnan(f)
    a = np.zeros(4096 + 20480, np.uint8)
    a[:64] = np.frombuffer(struct.pack("<IIQQQQQQQ", 0x57415243, 1, 4096, 1, 1, 16384, 16384, 0, 0), np.uint8)
    want = np.empty(65536, np.uint16)
    with np.errstate(over="ignore"):
        want[:] = f.astype(np.float16).view(np.uint16)
    for part in range(8):
        tile = np.zeros(4096 + 16384, np.uint8)
        tile[:4096] = a[:4096]
        tile[4096:] = (b[part * 8192:(part + 1) * 8192].astype(np.uint16)).view(np.uint8)
        out = O.convert_record(tile, 2, 0).view(np.uint16)
        sl = slice(part * 8192, (part + 1) * 8192)
        assert np.array_equal(out[keep[sl]], want[sl][keep[sl]])
        nan = ~keep[sl]
        assert np.all((out[nan] & 0x7C00) == 0x7C00) and np.all((out[nan] & 0x3FF) != 0)


@pytest.mark.gpu
@pytest.mark.parametrize("mode", [chpe.CONVERT_DENSE, chpe.CONVERT_RAW, chpe.CONVERT_RAW_FP16])
def test_convert_matches_oracle(tmp_path, mode):
    src = _standard_archive(np.random.default_rng(12 + mode))
    sp = tmp_path / "src.chpe"
    src.tofile(sp)
    dp = tmp_path / "dst.chpe"
    chpe.convert_archive(str(sp), str(dp), mode)
    _check(dp, src, mode)
    if mode != chpe.CONVERT_DENSE:  # a raw source converts again, to raw FP16
        raw = np.fromfile(dp, np.uint8)
        d2 = tmp_path / "dst2.chpe"
        chpe.convert_archive(str(dp), str(d2), chpe.CONVERT_RAW_FP16)
        got = np.fromfile(d2, np.uint8)
        assert np.array_equal(got[:4096], O.convert_header(raw, chpe.CONVERT_RAW_FP16))
        for i in range(0, N_REC, 97):
            assert np.array_equal(got[4096 + i * 16384:4096 + (i + 1) * 16384],
                                  O.convert_record(raw, chpe.CONVERT_RAW_FP16, i)), i


@pytest.mark.parametrize("mode", [chpe.CONVERT_DENSE, chpe.CONVERT_RAW])
def test_convert_host_modes(tmp_path, mode):
    """The dense and raw conversions are byte copies on the host (no GPU
    needed): byte for byte against the oracle, and a raw source refused for
    the dense conversion (it holds no cells)."""
    src = _standard_archive(np.random.default_rng(40 + mode))
    sp = tmp_path / "src.chpe"
    src.tofile(sp)
    dp = tmp_path / "dst.chpe"
    chpe.convert_archive(str(sp), str(dp), mode)
    _check(dp, src, mode)
    if mode == chpe.CONVERT_RAW:
        with pytest.raises(chpe.ChpeError, match="raw archive"):
            chpe.convert_archive(str(dp), str(tmp_path / "d.chpe"), chpe.CONVERT_DENSE)


def test_convert_rejects_bad_input(tmp_path):
    bad = tmp_path / "bad.chpe"
    bad.write_bytes(b"\0" * 8192)
    with pytest.raises(chpe.ChpeError, match="validation"):
        chpe.convert_archive(str(bad), str(tmp_path / "o.chpe"), chpe.CONVERT_RAW)
    with pytest.raises(chpe.ChpeError, match="mode"):
        chpe.convert_archive(str(bad), str(tmp_path / "o.chpe"), 9)
