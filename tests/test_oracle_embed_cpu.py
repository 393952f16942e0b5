"""Embedding lookup, tied LM head, norms and biases restated a second time in
numpy float64 and checked against the C oracle on hand-built archives with
random contents (CPU only):

* unpackEmbedRowCell (chpe_engine.zig:1288-1394): 8-bit rows under 8 only
  (later rows leave the output as it was, Q3), 2-bit and 4-bit rows with
  group-128 scales and outliers that REPLACE their column, the 4-bit
  scale/bias form, and for D = 4096 / 8192 the reads past the cell's codes
  and scale area (Q4), which land in the payload and the next record;
* unpackEmbedRow (:1491-1552): cell archives at tok / 16 for every D (Q2),
  raw FP16 / BF16 rows (8192 / D per tile), raw INT8 rows (16384 / D per
  tile, x 0.00373708), and the formula fallback past the archive;
* computeLmHead, tied forms (:1582-1660): every cell record in order with
  TileDims.rows rows (16 when 0) through unpackEmbedRowCell, a row buffer
  that keeps the previous row where a row is not written, and raw FP16 /
  BF16 tiles of 8192 / D rows;
* unpackNorm / unpackBias (:1144-1192): f32 (BF16 for the 9B raw archive),
  gains of 1.0 for a non-finite or all-zero norm, biases with non-finite
  entries set to 0."""
import struct

import numpy as np

import oracle_py as O

CELL, PAYLOAD, CODES = 17408, 16448, 64
CODEBOOK_W2 = np.array([0.0, 1.0, -2.0, -1.0])


def _archive(records, rec_bytes, flags=0):
    hdr = np.zeros(4096, np.uint8)
    hdr[:64] = np.frombuffer(struct.pack("<IIQQQQQQQ", 0x57415243, 1, 4096, len(records), len(records),
                                         rec_bytes, rec_bytes, 0, flags), np.uint8)
    return np.concatenate([hdr] + [r.astype(np.uint8) for r in records])


def _cell(rng, quant_bits, flags, rows=16, cols=2048, scale=0.0, bias=0.0):
    c = np.zeros(CELL, np.uint8)
    c[CODES:CODES + 16384] = rng.integers(0, 256, 16384, dtype=np.uint8)
    pl = PAYLOAD
    c[pl + 20] = quant_bits
    c[pl + 24:pl + 32] = np.frombuffer(struct.pack("<Q", flags), np.uint8)
    c[pl + 32:pl + 48] = np.frombuffer(struct.pack("<ffII", scale, bias, rows, cols), np.uint8)
    c[pl + 48:pl + 560] = np.abs(rng.normal(0, 0.01, 256)).astype(np.float16).view(np.uint8)
    c[pl + 560:pl + 816] = rng.normal(0, 0.5, 128).astype(np.float16).view(np.uint8)
    c[pl + 816:pl + 832] = rng.integers(0, 2400, 8).astype(np.uint16).view(np.uint8)
    # the rest of the payload: small finite FP16 values (read by the Q4 over-reads)
    c[pl + 832:pl + 960] = np.abs(rng.normal(0, 0.01, 64)).astype(np.float16).view(np.uint8)
    return c


def embed_row_cell(arc, off, row, D, out):
    """unpackEmbedRowCell on the cell at byte offset `off` of the archive;
    reads may run past the cell, as the reference's do."""
    pl = off + PAYLOAD
    qb = int(arc[pl + 20])
    flags = struct.unpack("<Q", arc[pl + 24:pl + 32].tobytes())[0]
    scale, bias = struct.unpack("<ff", arc[pl + 32:pl + 40].tobytes())
    codes = arc[off + CODES:]
    ng = D // 128

    def gs(i):
        return float(arc[pl + 48 + 2 * i:pl + 50 + 2 * i].copy().view(np.float16)[0])

    def replace_outliers():
        if flags & 1:
            cols = arc[pl + 816:pl + 832].copy().view(np.uint16)
            ws = arc[pl + 560:pl + 816].copy().view(np.float16).astype(np.float64)
            for k in range(8):
                if cols[k] < D:
                    out[cols[k]] = ws[row * 8 + k]

    if qb == 8:
        if row >= 8:
            return out
        w = codes[row * D:(row + 1) * D].copy().view(np.int8).astype(np.float64)
        for g in range(ng):
            out[g * 128:(g + 1) * 128] = w[g * 128:(g + 1) * 128] * gs(row * ng + g)
        return out
    if qb == 2:
        if row >= 16:
            return out
        b = codes[row * (D // 4):(row + 1) * (D // 4)]
        q = CODEBOOK_W2[np.stack([(b >> s) & 3 for s in (0, 2, 4, 6)], axis=-1).reshape(-1)]
        for g in range(ng):
            out[g * 128:(g + 1) * 128] = q[g * 128:(g + 1) * 128] * gs(row * ng + g)
        replace_outliers()
        return out
    b = codes[row * (D // 2):(row + 1) * (D // 2)]
    q = np.stack([b & 0x0F, b >> 4], axis=-1).reshape(-1).astype(np.float64) - 8.0
    if flags & 1 or qb == 4:
        if row >= 16:
            return out
        for g in range(ng):
            out[g * 128:(g + 1) * 128] = q[g * 128:(g + 1) * 128] * gs(row * ng + g)
        replace_outliers()
        return out
    out[:] = q * scale + bias
    return out


def _mixed_cells(rng, n):
    kinds = [(4, 1), (2, 1), (8, 0), (16, 0), (16, 1), (4, 0), (2, 0)]
    cells = []
    for i in range(n):
        qb, fl = kinds[i % len(kinds)]
        cells.append(_cell(rng, qb, fl, scale=0.01 + 0.001 * i, bias=0.002 * (i % 3 - 1)))
    return cells


def test_cell_embedding_rows():
    rng = np.random.default_rng(21)
    for arch, D in ((O.ARCH_3B, 2048), (O.ARCH_9B, 4096), (O.ARCH_72B, 8192)):
        cells = _mixed_cells(rng, 16)
        arc = _archive(cells, CELL)
        e = O.OracleEngine(arc, arch, 4)
        # rows of D / 2 bytes run 16 rows past a 16 KiB code area for D > 2048:
        # keep the reads inside the archive (the last two cells are only read)
        for t in range(len(cells) - (2 if D > 2048 else 0)):
            for r in range(16):
                tok = 16 * t + r
                init = rng.standard_normal(D).astype(np.float32)
                got = e.embed(tok, init.copy())
                # over-read scale bytes may decode to NaN or inf, as in the reference
                with np.errstate(invalid="ignore", over="ignore"):
                    want = embed_row_cell(arc, 4096 + t * CELL, r, D, init.astype(np.float64).copy())
                assert np.allclose(got, want, rtol=1e-6, atol=1e-9, equal_nan=True), (D, t, r)
        # rows of an 8-bit cell past row 7 leave the hidden as it was (Q3)
        init = rng.standard_normal(D).astype(np.float32)
        assert np.array_equal(e.embed(16 * 2 + 11, init.copy()), init)


def test_raw_embedding_rows():
    rng = np.random.default_rng(22)
    n = 6
    fallback = lambda tok, D: 0.05 * (((np.arange(D) + tok) % 17) - 8)
    for kind in ("fp16", "bf16", "int8"):
        if kind == "int8":
            arch, D, rpt, flags = O.ARCH_9B, 4096, 4, 0x08
            tiles = [rng.integers(-128, 128, 16384).astype(np.int8).view(np.uint8) for _ in range(n)]
            rows = [t.view(np.int8).astype(np.float64) * float(np.float32(0.00373708)) for t in tiles]
        else:
            arch, D, rpt = O.ARCH_3B, 2048, 4
            w = [rng.normal(0, 0.02, 8192) for _ in range(n)]
            if kind == "fp16":
                flags = 0x04
                tiles = [v.astype(np.float16).view(np.uint8) for v in w]
                rows = [t.copy().view(np.float16).astype(np.float64) for t in tiles]
            else:
                flags = 0
                tiles = [(v.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16).view(np.uint8) for v in w]
                rows = [(t.copy().view(np.uint16).astype(np.uint32) << 16).view(np.float32).astype(np.float64)
                        for t in tiles]
        e = O.OracleEngine(_archive(tiles, 16384, flags), arch, 4)
        for tok in range(n * rpt):
            t, r = divmod(tok, rpt)
            assert np.allclose(e.embed(tok), rows[t][r * D:(r + 1) * D], rtol=1e-6, atol=0), (kind, tok)
        for tok in (n * rpt, n * rpt + 5, 151000):   # past the archive: the formula
            assert np.allclose(e.embed(tok), fallback(tok, D), rtol=1e-6, atol=1e-9), (kind, tok)


def test_tied_lm_head_cells():
    rng = np.random.default_rng(23)
    D = 2048
    cells = _mixed_cells(rng, 14)
    rows = [16, 0, 16, 12, 16, 16, 20, 16, 8, 16, 16, 3, 16, 16]   # TileDims.rows; 0 reads as 16
    for c, n in zip(cells, rows):
        c[PAYLOAD + 40:PAYLOAD + 44] = np.frombuffer(struct.pack("<I", n), np.uint8)
    arc = _archive(cells, CELL)
    e = O.OracleEngine(arc, O.ARCH_3B, 4)
    x = rng.standard_normal(D).astype(np.float32)
    got = e.lm_head(x)
    buf = np.zeros(D)
    want = []
    for t, n in enumerate(rows):
        for r in range(n or 16):
            buf = embed_row_cell(arc, 4096 + t * CELL, r, D, buf)
            want.append(float(buf @ x.astype(np.float64)))
    want = np.array(want)
    np.testing.assert_allclose(got[:want.size], want, rtol=0, atol=2e-5 * np.abs(want).max())


def test_tied_lm_head_raw():
    rng = np.random.default_rng(24)
    D, n = 2048, 9
    for flags in (0x04, 0):
        w = [rng.normal(0, 0.02, 8192) for _ in range(n)]
        if flags:
            tiles = [v.astype(np.float16).view(np.uint8) for v in w]
            W = np.concatenate([t.copy().view(np.float16).astype(np.float64) for t in tiles])
        else:
            tiles = [(v.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16).view(np.uint8) for v in w]
            W = np.concatenate([(t.copy().view(np.uint16).astype(np.uint32) << 16).view(np.float32)
                                .astype(np.float64) for t in tiles])
        e = O.OracleEngine(_archive(tiles, 16384, flags), O.ARCH_3B, 4)
        x = rng.standard_normal(D).astype(np.float32)
        got = e.lm_head(x)
        want = W.reshape(-1, D) @ x.astype(np.float64)
        np.testing.assert_allclose(got[:want.size], want, rtol=0, atol=2e-5 * np.abs(want).max())


def test_norms_and_biases():
    rng = np.random.default_rng(25)
    D = 2048
    good = rng.normal(1.0, 0.1, 4096).astype(np.float32)
    nan = good.copy()
    nan[77] = np.nan
    bias = rng.normal(0, 0.02, 4096).astype(np.float32)
    bias[[3, 900]] = [np.inf, np.nan]
    tiles = [t.view(np.uint8) for t in (good, nan, np.zeros(4096, np.float32), bias)]
    e = O.OracleEngine(_archive(tiles, 16384, 0x04), O.ARCH_3B, 4)
    assert np.array_equal(e.unpack_norm(0, D), good[:D])
    assert np.array_equal(e.unpack_norm(1, D), np.ones(D, np.float32))        # a non-finite gain
    assert np.array_equal(e.unpack_norm(2, D), np.ones(D, np.float32))        # all zero
    assert np.array_equal(e.unpack_norm(9, D), np.ones(D, np.float32))        # past the archive
    want = np.where(np.isfinite(bias[:D]), bias[:D], 0.0).astype(np.float32)
    assert np.array_equal(e.unpack_bias(3, D), want)
    assert np.array_equal(e.unpack_bias(9, D), np.zeros(D, np.float32))
    # the 9B raw archive stores 1-D tensors as BF16
    D9 = 4096
    g9 = rng.normal(1.0, 0.1, 8192).astype(np.float32)
    t9 = (g9.view(np.uint32) >> 16).astype(np.uint16).view(np.uint8)
    e9 = O.OracleEngine(_archive([t9], 16384, 0x08), O.ARCH_9B, 4)
    want9 = ((t9.copy().view(np.uint16).astype(np.uint32) << 16).view(np.float32))[:D9]
    assert np.array_equal(e9.unpack_norm(0, D9), want9)
