"""Kernel-level parity on the GPU, through the C ABI probes, against the CPU
oracle: bit-exact dequantised tiles and embedding rows; GEMV per call site
within f32 accumulation-order tolerance."""
import numpy as np
import pytest

import chpe_qwen_engine_b200 as chpe
import oracle_py as O
from _util import archive, assert_close_vec, oracle_threads

pytestmark = pytest.mark.gpu

CELL_CONFIGS = [
    (chpe.SYNTH_3B_W4, 0),
    (chpe.SYNTH_3B_W2, 0),
    (chpe.SYNTH_3B_W4, chpe.SYNTH_OUTLIERS),
    (chpe.SYNTH_3B_W4, chpe.SYNTH_NONGROUP | chpe.SYNTH_STANDARD),
    (chpe.SYNTH_3B_W4, chpe.SYNTH_MIXED | chpe.SYNTH_BIAS),
]


def engines(cfg, flags, max_seq=64):
    a = archive(cfg, flags)
    e = chpe.Engine.from_bytes(a, chpe.SYNTH_ARCH[cfg], max_seq)
    o = O.OracleEngine(a, chpe.SYNTH_ARCH[cfg], max_seq, threads=oracle_threads())
    return a, e, o


@pytest.mark.parametrize("cfg,flags", CELL_CONFIGS)
def test_dequant_cells_bit_exact(cfg, flags):
    a, e, o = engines(cfg, flags)
    stride = 20480 if flags & chpe.SYNTH_STANDARD else 17408
    pre = 3072 if flags & chpe.SYNTH_STANDARD else 0
    tiles = []
    for l in (0, 1, 7, 21, 35):
        li = o.layer_info(l)
        for name in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj"):
            tiles.append((li[name], False))
            tiles.append((li[name] + 3, False))
        tiles.append((li["down_proj"], True))
        tiles.append((li["down_proj"] + 100, True))
    tiles += [(0, False), (9495, False)]
    for t, flat in tiles:
        cell = a[4096 + t * stride + pre:4096 + t * stride + pre + 17408]
        ref = O.dequant_cell(np.ascontiguousarray(cell), flat)
        got = e.probe_dequant_cell(t, flat)
        assert got.shape == ref.shape, (t, flat)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), (t, flat)


@pytest.mark.parametrize("cfg,flags", CELL_CONFIGS + [(chpe.SYNTH_3B_FP16_RAW, 0), (chpe.SYNTH_3B_BF16_RAW, 0)])
def test_embedding_rows_bit_exact(cfg, flags):
    a, e, o = engines(cfg, flags)
    rng = np.random.default_rng(3)
    for tok in [0, 1, 15, 16, 151935, 151936, 200000] + list(rng.integers(0, 151936, 12)):
        init = np.full(o.hidden_dim, 7.0, np.float32)
        ref = o.embed(int(tok), init.copy())
        got = e.probe_embed(int(tok), init.copy())
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), tok


def _call_sites(o, l):
    li = o.layer_info(l)
    D, F, qd, kvd = 2048, 11008, 2048, 256
    return [
        ("q", li["q_proj"], li["q_tiles"], qd, D, D, False, li["q_bias"]),
        ("k", li["k_proj"], li["k_tiles"], kvd, D, D, False, li["k_bias"]),
        ("v", li["v_proj"], li["v_tiles"], kvd, D, D, False, li["v_bias"]),
        ("o", li["o_proj"], li["o_tiles"], D, D, D, True, -1),
        ("gate", li["gate_proj"], li["gate_tiles"], F, D, D, False, -1),
        ("up", li["up_proj"], li["up_tiles"], F, D, D, False, -1),
        ("down", li["down_proj"], li["down_tiles"], D, F, F, True, -1),
    ]


@pytest.mark.parametrize("as_flat", [False, True])
@pytest.mark.parametrize("cfg,flags", CELL_CONFIGS + [(chpe.SYNTH_3B_FP16_RAW, 0)])
def test_gemv_linear_call_sites(cfg, flags, as_flat, monkeypatch):
    # as_flat: the opt-in routing of 16x2048 row-tiled cells to the flat
    # kernel's aligned-cell mode (read when a call is planned)
    if as_flat:
        monkeypatch.setenv("CHPE_ROWTILE_AS_FLAT", "1")
    a, e, o = engines(cfg, flags)
    rng = np.random.default_rng(11)
    for l in (0, 5, 21):
        for name, ts, nt, r, c, xl, acc, bias in _call_sites(o, l):
            x = rng.standard_normal(xl).astype(np.float32)
            y0 = rng.standard_normal(r).astype(np.float32) if acc else np.zeros(r, np.float32)
            ref = o.gemv_linear(ts, nt, x, r, c, accumulate=acc, bias_tile=bias, y=y0.copy())
            got = e.probe_gemv_linear(ts, nt, x, r, c, accumulate=acc, bias_tile=bias, y=y0.copy())
            assert_close_vec(got, ref, 1e-4, f"layer {l} {name}")


def test_gemv_partial_spans_and_past_end():
    """Fewer tiles than rows (rows beyond stay 0), a start past the archive
    (synthetic pattern / no-op), and a span cut by the archive's end."""
    a, e, o = engines(chpe.SYNTH_3B_W4, 0)
    rng = np.random.default_rng(5)
    li = o.layer_info(3)
    x = rng.standard_normal(2048).astype(np.float32)
    xf = rng.standard_normal(11008).astype(np.float32)
    cases = [
        (li["q_proj"], 40, 2048, 2048, x, False),   # 40 row-tiled cells cover 640 rows
        (li["down_proj"], 100, 2048, 11008, xf, False),  # flat: first 100 tiles only
        (94349 + 5, 10, 300, 2048, x, False),        # past the end: pattern
        (94349 + 5, 10, 300, 2048, x, True),         # past the end, accumulate: untouched
        (94340, 50, 160, 2048, x, False),            # cut by the archive end
    ]
    for ts, nt, r, c, xv, acc in cases:
        y0 = rng.standard_normal(r).astype(np.float32)
        ref = o.gemv_linear(ts, nt, xv, r, c, accumulate=acc, y=y0.copy())
        got = e.probe_gemv_linear(ts, nt, xv, r, c, accumulate=acc, y=y0.copy())
        assert_close_vec(got, ref, 1e-4, f"{ts},{nt},{r},{c},{acc}")


# (rows, cols) read from the 3B down-projection tiles (688 flat cells, or 2752
# raw FP16 tiles): the widths of the 9B/72B tensors (4096, 8192, 12288,
# 29568; 4096 and 8192 take the aligned-cell path), widths just past one
# consumer warp's run, a handful of rows, a width that is not a multiple of
# the chunk width, and spans longer than the tiles given (not covered in
# full, aligned and not).
FLAT_SHAPES = [(2048, 8192), (700, 29568), (4000, 4096), (1500, 12288), (9000, 2112), (5, 8192),
               (3, 29568), (1, 4096), (700, 30000), (770, 29568), (2800, 8192), (8, 4096)]


@pytest.mark.parametrize("colown", [False, True])
@pytest.mark.parametrize("cfg", [chpe.SYNTH_3B_W4, chpe.SYNTH_3B_W2, chpe.SYNTH_3B_FP16_RAW])
def test_gemv_flat_widths(cfg, colown, monkeypatch):
    # colown: the column-owner mode (default for rows of 384..960 16-byte
    # chunks, e.g. 29568 4-bit columns) or, with CHPE_FLAT_COLOWN=0, the
    # stream mode for the same calls; read when a call is planned
    monkeypatch.setenv("CHPE_FLAT_COLOWN", "1" if colown else "0")
    a, e, o = engines(cfg, 0)
    li = o.layer_info(4)
    rng = np.random.default_rng(17)
    for r, c in FLAT_SHAPES:
        for acc in (False, True):
            x = rng.standard_normal(c).astype(np.float32)
            y0 = rng.standard_normal(r).astype(np.float32)
            ref = o.gemv_linear(li["down_proj"], li["down_tiles"], x, r, c, accumulate=acc, y=y0.copy())
            got = e.probe_gemv_linear(li["down_proj"], li["down_tiles"], x, r, c, accumulate=acc, y=y0.copy())
            assert_close_vec(got, ref, 1e-4, f"{r}x{c} acc={acc}")


# Aligned 4-bit shapes for the tensor-core decode: whole 16-row blocks of
# 8192 / 4096 columns read from the 3B down-projection cells (688 cells), one
# more than the cells hold (2800 x 8192: the FFMA decode takes it), and
# single blocks.
MMA_SHAPES = [(2048, 8192), (4000, 4096), (16, 8192), (32, 4096), (1600, 8192), (2800, 8192)]


@pytest.mark.parametrize("mma", [False, True])
@pytest.mark.parametrize("cfg,flags", [(chpe.SYNTH_3B_W4, 0), (chpe.SYNTH_3B_W4, chpe.SYNTH_OUTLIERS)])
def test_gemv_flat_mma(cfg, flags, mma, monkeypatch):
    """mma.sync decode (code bytes as the u8 operand, x as int8 pieces under a
    per-group exponent, exact s32 sums) of aligned 4-bit group-scaled cells
    against the oracle, the tensor cores taken wherever they apply
    (CHPE_FLAT_MMA=1); with CHPE_FLAT_MMA=0 the FFMA
    decode of the same calls.  x spans a wide range: a few entries 1e4 times
    the rest."""
    monkeypatch.setenv("CHPE_FLAT_MMA", "1" if mma else "0")
    a, e, o = engines(cfg, flags)
    li = o.layer_info(4)
    rng = np.random.default_rng(29)
    for r, c in MMA_SHAPES:
        for acc in (False, True):
            x = rng.standard_normal(c).astype(np.float32)
            x[rng.integers(0, c, 4)] *= 1e4
            y0 = rng.standard_normal(r).astype(np.float32)
            ref = o.gemv_linear(li["down_proj"], li["down_tiles"], x, r, c, accumulate=acc, y=y0.copy())
            got = e.probe_gemv_linear(li["down_proj"], li["down_tiles"], x, r, c, accumulate=acc, y=y0.copy())
            assert_close_vec(got, ref, 1e-4, f"{r}x{c} acc={acc} mma={mma}")


# Row-block shapes for the tensor-core decode of rows that do not start at
# cell boundaries (rows in whole 8-row units, every row in the 688 cells):
# CTAs of 16-row blocks with an 8-row tail (5320 x 4224: 33 groups, a
# two-group last chunk), the 9B / 72B down widths, a single 8-row block, and
# rows that give one or two 8-row units per CTA.
ROWBLK_SHAPES = [(5320, 4224), (1824, 12288), (752, 29568), (8, 29568), (24, 11008), (2000, 11008),
                 (16, 4224), (2960, 6272)]


@pytest.mark.parametrize("rowblk", [True, False])
def test_gemv_rowblk(rowblk, monkeypatch):
    """Row-block tensor-core decode (gemv_rowblk_kernel: per-row bulk copies
    of 16-group chunks, the int8-piece B of every group in shared memory)
    against the oracle; with CHPE_FLAT_ROWBLK=0 the FFMA decode of the same
    calls (CHPE_FLAT_ROWBLK=1 takes the tensor cores wherever they apply).  x
    spans a wide range: a few entries 1e4 times the rest."""
    monkeypatch.setenv("CHPE_FLAT_ROWBLK", "1" if rowblk else "0")
    a, e, o = engines(chpe.SYNTH_3B_W4, 0)
    li = o.layer_info(4)
    rng = np.random.default_rng(31)
    for r, c in ROWBLK_SHAPES:
        for acc in (False, True):
            x = rng.standard_normal(c).astype(np.float32)
            x[rng.integers(0, c, 4)] *= 1e4
            y0 = rng.standard_normal(r).astype(np.float32)
            ref = o.gemv_linear(li["down_proj"], li["down_tiles"], x, r, c, accumulate=acc, y=y0.copy())
            got = e.probe_gemv_linear(li["down_proj"], li["down_tiles"], x, r, c, accumulate=acc, y=y0.copy())
            assert_close_vec(got, ref, 1e-4, f"{r}x{c} acc={acc} rowblk={rowblk}")


@pytest.mark.parametrize("arch", [chpe.ARCH_3B, chpe.ARCH_9B, chpe.ARCH_72B])
def test_attention_against_oracle(arch):
    """RoPE + KV append + GQA softmax (chpe_engine.zig:1688-1734) over a
    growing cache, one call per position, against the oracle's f32 path."""
    mock = np.zeros(8192, np.uint8)  # the attention op does not read weights
    e = chpe.Engine.from_bytes(mock, arch, 96)
    A = {chpe.ARCH_3B: (16, 2, 128), chpe.ARCH_9B: (16, 4, 256), chpe.ARCH_72B: (64, 8, 128)}[arch]
    H, KV, HD = A
    rng = np.random.default_rng(arch + 7)
    kc = np.zeros((96, KV * HD), np.float32)
    vc = np.zeros((96, KV * HD), np.float32)
    for pos in list(range(0, 40)) + [40, 41]:
        q = rng.standard_normal(H * HD).astype(np.float32)
        k = rng.standard_normal(KV * HD).astype(np.float32)
        v = rng.standard_normal(KV * HD).astype(np.float32)
        got = e.probe_attention(2, pos, q, k, v)
        qr = O.apply_rope(q, pos, H, HD)
        kc[pos] = O.apply_rope(k, pos, KV, HD)
        vc[pos] = v
        ref = O.gqa_attention(qr, kc[:pos + 1], vc[:pos + 1], pos, H, KV, HD)
        # the cache holds FP16 (the reference holds f32): tolerance of fp16 rounding
        assert_close_vec(got, ref, 4e-3, f"pos {pos}")
