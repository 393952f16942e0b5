"""A second, independent restatement of the reference's tile formats, in
numpy float64, checked against the C oracle's gemvLinear on hand-built
archives with random contents (CPU only).  The known-answer tests pin the
oracle on constant cells; this pins every format branch on arbitrary codes,
scales, outliers and replacement lists:

* row-tiled cells (c_total <= 2048) through gemvTilePolymorphic
  (chpe_engine.zig:732-751): gemvTileW2 (:223-324), gemvTileW4 (:326-419)
  with group-128 scales or per-tile scale/bias and the additive row outliers,
  gemvTileW8 (:421-473), gemvTileF16 IEEE and BF16 (:475-542), gemvTileF32
  (:544-582); rows past TileDims.rows or past y, and the rows == 0 stop of
  gemvLinear (:1396-1489);
* flat cells (c_total > 2048) through gemvCellFlat (:584-730): 4-bit and
  2-bit cells with group scales or scale/bias, the down_aux replacements
  (count <= 64, offsets below the tile), cells of other widths read as
  zeros, rows wrapping across cells and stopping at r_total;
* raw tiles through dotSegment (:1194-1286): FP16, BF16 and INT8 (global
  scale 0.00373708);
* the archive converters (weight_archive.zig:617-776) on the byte level,
  from standard, dense and raw sources.

The oracle accumulates in f32 in the reference's order; the restatement sums
in float64, so the comparison allows 2e-5 of the largest output."""
import struct

import numpy as np
import pytest

import oracle_py as O

CELL, PAYLOAD, CODES = 17408, 16448, 64
CODEBOOK_W2 = np.array([0.0, 1.0, -2.0, -1.0])


def _archive(records: list[np.ndarray], rec_bytes: int, flags: int = 0) -> np.ndarray:
    hdr = np.zeros(4096, np.uint8)
    hdr[:64] = np.frombuffer(struct.pack("<IIQQQQQQQ", 0x57415243, 1, 4096, len(records), len(records),
                                         rec_bytes, rec_bytes, 0, flags), np.uint8)
    return np.concatenate([hdr] + [r.astype(np.uint8) for r in records])


def _cell(rng, quant_bits: int, flags: int, rows: int, cols: int, scale=0.0, bias=0.0) -> np.ndarray:
    """A dense cell with random codes and payload, and the given metadata."""
    c = np.zeros(CELL, np.uint8)
    c[CODES:CODES + 16384] = rng.integers(0, 256, 16384, dtype=np.uint8)
    pl = PAYLOAD
    c[pl + 20] = quant_bits
    c[pl + 24:pl + 32] = np.frombuffer(struct.pack("<Q", flags), np.uint8)
    c[pl + 32:pl + 48] = np.frombuffer(struct.pack("<ffII", scale, bias, rows, cols), np.uint8)
    # group scales |N(0, 0.01)| as f16, row outlier weights and columns
    c[pl + 48:pl + 560] = np.abs(rng.normal(0, 0.01, 256)).astype(np.float16).view(np.uint8)
    c[pl + 560:pl + 816] = rng.normal(0, 0.05, 128).astype(np.float16).view(np.uint8)
    c[pl + 816:pl + 832] = rng.integers(0, 2048, 8).astype(np.uint16).view(np.uint8)
    return c


def _f16(b: np.ndarray) -> np.ndarray:
    return b.view(np.float16).astype(np.float64)


def _bf16(b: np.ndarray) -> np.ndarray:
    return (b.view(np.uint16).astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def _codes4(b: np.ndarray) -> np.ndarray:
    """Nibbles, low first, minus 8."""
    return np.stack([b & 0x0F, b >> 4], axis=-1).reshape(*b.shape[:-1], -1).astype(np.float64) - 8.0


def _codes2(b: np.ndarray) -> np.ndarray:
    """2-bit codes, least significant first, through the codebook."""
    q = np.stack([(b >> s) & 3 for s in (0, 2, 4, 6)], axis=-1).reshape(*b.shape[:-1], -1)
    return CODEBOOK_W2[q]


def _meta(cell: np.ndarray):
    pl = cell[PAYLOAD:PAYLOAD + 960]
    flags = struct.unpack("<Q", pl[24:32].tobytes())[0]
    scale, bias, rows, cols = struct.unpack("<ffII", pl[32:48].tobytes())
    return int(pl[20]), flags, float(scale), float(bias), rows, cols


def tile_rows(cell: np.ndarray, x: np.ndarray, nrows: int) -> np.ndarray:
    """Row sums of one row-tiled cell for its first nrows rows."""
    qb, flags, scale, bias, rows, cols = _meta(cell)
    pl = cell[PAYLOAD:PAYLOAD + 960]
    codes = cell[CODES:CODES + 16384]
    x = x.astype(np.float64)
    out = np.zeros(nrows)
    if qb not in (4, 8, 16, 32):
        qb = 2  # the dispatcher's fallback
    if qb in (2, 4):
        group = bool(flags & 1)
        per_byte = 2 if qb == 4 else 4
        dec = _codes4 if qb == 4 else _codes2
        row_bytes = cols // per_byte
        gs = _f16(pl[48:560].copy())
        for r in range(nrows):
            rb = codes[r * row_bytes:(r + 1) * row_bytes]
            if group:
                G, ng = cols // 128, min(cols // 128, x.size // 128)
                q = dec(rb[:ng * 128 // per_byte][None, :])[0]
                out[r] = sum(float(q[g * 128:(g + 1) * 128] @ x[g * 128:(g + 1) * 128]) * gs[r * G + g]
                             for g in range(ng))
            else:
                n = min(cols, x.size) // per_byte * per_byte
                q = dec(rb[:n // per_byte][None, :])[0]
                out[r] = float((q * scale + bias) @ x[:n])
        if group and rows == 16:
            ocol = pl[816:832].copy().view(np.uint16).astype(np.int64)
            xo = np.array([x[c] if c < x.size else 0.0 for c in ocol])
            ow = _f16(pl[560:816].copy()).reshape(16, 8)
            out += ow[:nrows] @ xo
    elif qb == 8:
        n = min(cols, x.size)
        w = codes.view(np.int8).astype(np.float64)
        for r in range(nrows):
            out[r] = float(w[r * cols:r * cols + n] @ x[:n]) * scale + bias
    else:
        n = min(cols, x.size)
        if qb == 16:
            w = _f16(codes.copy()) if flags & 0x04 else _bf16(codes.copy())
        else:
            w = codes.copy().view(np.float32).astype(np.float64)
        for r in range(nrows):
            out[r] = float(w[r * cols:r * cols + n] @ x[:n])
    return out


def linear_row_tiled(cells: list[np.ndarray], x, r_total, y0=None) -> np.ndarray:
    """gemvLinear over row-tiled cells: rows in cell order until r_total, a
    cell of zero rows, or the end of the tiles."""
    y = np.zeros(r_total) if y0 is None else y0.astype(np.float64).copy()
    row_base = 0
    for cell in cells:
        rows = _meta(cell)[4]
        if row_base >= r_total or rows == 0:
            break
        n = min(rows, r_total - row_base)
        y[row_base:row_base + n] += tile_rows(cell, x, n)
        row_base += rows
    return y


def flat_weights(cell: np.ndarray) -> np.ndarray:
    """The 32768 weights of a flat cell, with the down_aux replacements."""
    qb, flags, scale, bias, rows, cols = _meta(cell)
    pl = cell[PAYLOAD:PAYLOAD + 960]
    codes = cell[CODES:CODES + 16384]
    if qb not in (2, 4):
        return np.zeros(32768)
    dec, per_byte = (_codes4, 2) if qb == 4 else (_codes2, 4)
    q = dec(codes[:32768 // per_byte][None, :])[0]
    if flags & 1:
        w = q * np.repeat(_f16(pl[48:560].copy()), 128)
    else:
        w = q * scale + bias
    n = int(pl[560:562].copy().view(np.uint16)[0])
    if 0 < n <= 64:
        vals = _f16(pl[562:562 + 2 * n].copy())
        offs = pl[690:690 + 2 * n].copy().view(np.uint16)
        for v, o in zip(vals, offs):
            if o < 32768:
                w[o] = v
    return w


def _segments(weights_per_tile: list[np.ndarray], x, r_total, c_total, y, scale=1.0):
    """Tile t holds flat weights [t wpt, (t+1) wpt) of the row-major tensor;
    each row's part of a tile is one segment, rows stop at r_total."""
    x = x.astype(np.float64)
    for t, w in enumerate(weights_per_tile):
        wpt = w.size
        r, c = divmod(t * wpt, c_total)
        j = 0
        while j < wpt and r < r_total:
            seg = min(wpt - j, c_total - c)
            y[r] += float(w[j:j + seg] @ x[c:c + seg]) * scale
            j += seg
            c += seg
            if c == c_total:
                c, r = 0, r + 1
    return y


def _close(got, want, what):
    tol = 2e-5 * max(1.0, float(np.max(np.abs(want))))
    err = float(np.max(np.abs(got.astype(np.float64) - want)))
    assert err <= tol, (what, err, tol)


def _row_tiled_cells(rng) -> list[np.ndarray]:
    cells = [
        _cell(rng, 4, 1, 16, 2048),                          # W4, group-128 scales, row outliers
        _cell(rng, 4, 0, 16, 2048, scale=0.01, bias=0.001),  # W4, scale/bias
        _cell(rng, 2, 1, 16, 2048),                          # W2, group-128 scales, row outliers
        _cell(rng, 2, 0, 16, 2048, scale=0.02, bias=-0.003), # W2, scale/bias
        _cell(rng, 8, 0, 8, 2048, scale=0.004, bias=0.01),   # W8
        _cell(rng, 16, 4, 4, 2048),                          # IEEE FP16
        _cell(rng, 16, 0, 4, 2048),                          # BF16
        _cell(rng, 32, 0, 2, 2048),                          # F32
        _cell(rng, 7, 1, 16, 2048),                          # unknown width: the W2 path
        _cell(rng, 4, 1, 8, 2048),                           # W4 group, 8 rows: no outliers
    ]
    w = rng.normal(0, 0.02, 8192)
    cells[5][CODES:CODES + 16384] = w.astype(np.float16).view(np.uint8)
    cells[6][CODES:CODES + 16384] = (w.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16).view(np.uint8)
    cells[7][CODES:CODES + 16384] = rng.normal(0, 0.02, 4096).astype(np.float32).view(np.uint8)
    # outlier columns past x are read as 0
    cells[2][PAYLOAD + 816:PAYLOAD + 818] = np.frombuffer(struct.pack("<H", 5000), np.uint8)
    return cells


def test_row_tiled_cells_every_format():
    rng = np.random.default_rng(11)
    cells = _row_tiled_cells(rng)
    stop = _cell(rng, 4, 1, 0, 2048)                         # rows == 0: gemvLinear stops here
    after = _cell(rng, 4, 1, 16, 2048)
    arc = _archive(cells + [stop, after], CELL)
    e = O.OracleEngine(arc, O.ARCH_3B, 4)
    x = rng.standard_normal(2048).astype(np.float32)
    total = sum(_meta(c)[4] for c in cells)                  # 106 rows
    for r_total in (total, 40, 3, total + 20):
        got = e.gemv_linear(0, len(cells) + 2, x, r_total, 2048)
        _close(got, linear_row_tiled(cells + [stop, after], x, r_total), f"r_total {r_total}")
        if r_total > total:
            assert np.all(got[total:] == 0.0)
    # accumulate: y += W x
    y0 = rng.standard_normal(total).astype(np.float32)
    got = e.gemv_linear(0, len(cells), x, total, 2048, accumulate=True, y=y0.copy())
    _close(got, linear_row_tiled(cells, x, total, y0), "accumulate")
    # a shorter x: group loops stop at x's last whole group, the rest at x's end
    xs = x[:1000].copy()
    got = e.gemv_linear(0, len(cells), xs, total, 2048)
    _close(got, linear_row_tiled(cells, xs, total), "short x")


def _flat_cells(rng) -> list[np.ndarray]:
    def aux(c, n, offs=None):
        c[PAYLOAD + 560:PAYLOAD + 562] = np.frombuffer(struct.pack("<H", n), np.uint8)
        k = min(n, 64)
        c[PAYLOAD + 562:PAYLOAD + 562 + 2 * k] = rng.normal(0, 0.5, k).astype(np.float16).view(np.uint8)
        o = rng.integers(0, 32768, k).astype(np.uint16) if offs is None else np.array(offs, np.uint16)
        c[PAYLOAD + 690:PAYLOAD + 690 + 2 * k] = o.view(np.uint8)
        return c
    return [
        aux(_cell(rng, 4, 1, 0, 0), 5, [0, 77, 32767, 40000, 1234]),   # W4 group; one offset past the tile
        aux(_cell(rng, 2, 1, 0, 0), 3),                               # W2 group
        aux(_cell(rng, 4, 0, 0, 0, scale=0.01, bias=0.002), 70),      # W4 scale/bias; count > 64: ignored
        _cell(rng, 8, 0, 0, 0, scale=1.0),                            # 8-bit: zeros in the flat path
        aux(_cell(rng, 2, 0, 0, 0, scale=0.02, bias=-0.001), 64),     # W2 scale/bias, 64 replacements
        aux(_cell(rng, 4, 1, 0, 0), 0),                               # W4 group, none
    ]


@pytest.mark.parametrize("c_total,r_total", [(11008, 17), (11008, 9), (29568, 6), (4096, 48), (2112, 60)])
def test_flat_cells(c_total, r_total):
    rng = np.random.default_rng(c_total + r_total)
    cells = _flat_cells(rng)
    arc = _archive(cells, CELL)
    e = O.OracleEngine(arc, O.ARCH_72B, 4)
    x = rng.standard_normal(c_total).astype(np.float32)
    want = _segments([flat_weights(c) for c in cells], x, r_total, c_total, np.zeros(r_total))
    _close(e.gemv_linear(0, len(cells), x, r_total, c_total), want, "flat")
    # tiles past the archive's end are not read
    _close(e.gemv_linear(0, len(cells) + 5, x, r_total, c_total), want, "flat, span past the end")


@pytest.mark.parametrize("kind", ["fp16", "bf16", "int8"])
@pytest.mark.parametrize("c_total", [2048, 4096, 11008])
def test_raw_tiles(kind, c_total):
    rng = np.random.default_rng(c_total)
    n_tiles = 12
    if kind == "int8":
        tiles = [rng.integers(-128, 128, 16384).astype(np.int8).view(np.uint8) for _ in range(n_tiles)]
        weights = [t.view(np.int8).astype(np.float64) for t in tiles]
        arch, flags, scale = O.ARCH_9B, 0x08, float(np.float32(0.00373708))
    else:
        w = [rng.normal(0, 0.02, 8192) for _ in range(n_tiles)]
        if kind == "fp16":
            tiles = [v.astype(np.float16).view(np.uint8) for v in w]
            weights = [_f16(t.copy()) for t in tiles]
            flags = 0x04
        else:
            tiles = [(v.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16).view(np.uint8) for v in w]
            weights = [_bf16(t.copy()) for t in tiles]
            flags = 0
        arch, scale = O.ARCH_3B, 1.0
    arc = _archive(tiles, 16384, flags)
    e = O.OracleEngine(arc, arch, 4)
    wpt = weights[0].size
    r_total = n_tiles * wpt // c_total
    x = rng.standard_normal(c_total).astype(np.float32)
    for r in (r_total, max(1, r_total // 3)):
        want = _segments(weights, x, r, c_total, np.zeros(r), scale)
        _close(e.gemv_linear(0, n_tiles, x, r, c_total), want, f"{kind} rows {r}")


# weight_archive.zig:617-776: convertToDensePosix, convertToRawContiguousPosix,
# convertToRawFp16ContiguousPosix, restated on the byte level
def _convert_header(src: np.ndarray, mode: int) -> np.ndarray:
    out = np.zeros(4096, np.uint8)
    out[:64] = src[:64]
    put = lambda off, v: out.__setitem__(slice(off, off + 8), np.frombuffer(struct.pack("<Q", v), np.uint8))
    if mode == 0:        # dense: record_bytes = cell bytes, no prefetch area
        put(32, 17408)
        put(48, 0)
    else:                # raw: 16 KiB tiles of codes only
        put(32, 16384)
        put(40, 16384)
        put(48, 0)
        if mode == 2:
            put(56, struct.unpack("<Q", src[56:64].tobytes())[0] | 0x04)
    return out


def _convert_record(src: np.ndarray, mode: int, i: int) -> np.ndarray:
    count, rb, pb = (struct.unpack("<Q", src[o:o + 8].tobytes())[0] for o in (16, 32, 48))
    raw = rb == 16384 and pb == 0
    cell = 4096 + i * rb + pb
    if mode == 0:
        return src[cell:cell + 17408].copy()
    tile = src[4096 + i * 16384:4096 + (i + 1) * 16384] if raw else src[cell + 64:cell + 64 + 16384]
    if mode == 1:
        return tile.copy()
    one_d = (count == 376853 and (i == 376852 or (i >= 37984 and (i - 37984) % 9413 in (0, 513, 578, 643, 1156))))
    one_d = one_d or (not raw and src[cell + 16448 + 20] == 32)
    if one_d:
        return tile.copy()
    f = (tile.copy().view(np.uint16).astype(np.uint32) << 16).view(np.float32)
    with np.errstate(over="ignore", invalid="ignore"):
        return f.astype(np.float16).view(np.uint8)


def test_converters_match_restatement():
    rng = np.random.default_rng(31)
    n = 40
    for rb, pb in ((20480, 3072), (17408, 0), (16384, 0)):
        recs = [rng.integers(0, 256, rb, dtype=np.uint8) for _ in range(n)]
        if rb != 16384:
            for i, r in enumerate(recs):   # quant_bits 32 (1-D) for every 5th cell, else 16
                r[pb + 16448 + 20] = 32 if i % 5 == 0 else 16
        hdr = np.zeros(4096, np.uint8)
        hdr[:64] = np.frombuffer(struct.pack("<IIQQQQQQQ", 0x57415243, 1, 4096, n, n, rb,
                                             16384 if rb == 16384 else 17408, pb, 0x10), np.uint8)
        src = np.concatenate([hdr] + recs)
        for mode in (0, 1, 2):
            if mode == 0 and rb == 16384:
                continue   # a raw archive holds no cells to keep
            assert np.array_equal(O.convert_header(src, mode), _convert_header(src, mode)), (rb, mode)
            for i in range(n):
                got, want = O.convert_record(src, mode, i), _convert_record(src, mode, i)
                if mode == 2 and got.size == 16384 and not np.array_equal(got, want):
                    # NaN payloads: both NaN with the same sign; every other value exact
                    g, w = got.view(np.uint16), want.view(np.uint16)
                    nan = (w & 0x7C00) == 0x7C00
                    nan &= (w & 0x3FF) != 0
                    assert np.array_equal(g[~nan], w[~nan]), (rb, i)
                    assert np.all(((g[nan] & 0x7C00) == 0x7C00) & ((g[nan] & 0x3FF) != 0))
                    assert np.array_equal(g[nan] >> 15, w[nan] >> 15)
                else:
                    assert np.array_equal(got, want), (rb, mode, i)
