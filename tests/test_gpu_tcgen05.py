"""The tcgen05 integer MMA path on its own (chpe_probe_tc_i8): A in tensor
memory (written with tcgen05.st), B in shared memory (K-major, no swizzle),
two K=32 MMAs into an s32 accumulator in tensor memory, read with
tcgen05.ld.  Exact against the integer product."""
import numpy as np
import pytest

import chpe_qwen_engine_b200 as chpe

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [16, 32])
def test_tcgen05_i8_product_exact(n):
    rng = np.random.default_rng(n)
    a = rng.integers(0, 256, (128, 64), dtype=np.uint8)
    b = rng.integers(-128, 128, (n, 64), dtype=np.int8)
    d = np.zeros((128, n), np.int32)
    rc = chpe.lib().chpe_probe_tc_i8(a.ctypes.data, b.ctypes.data, n, d.ctypes.data, 0)
    assert rc == 0, chpe.lib().chpe_last_error(None)
    ref = a.astype(np.int64) @ b.astype(np.int64).T
    assert np.array_equal(d.astype(np.int64), ref)


# (rows, cols) read from the 3B down-projection cells (688 flat 4-bit cells):
# the 9B/72B widths, rows that straddle cells (29568, 12288 columns), split-K
# ranges of one and several groups
BG_SHAPES = [(2048, 8192), (1024, 4096), (640, 29568), (512, 12288), (128, 128 * 40), (256, 2176)]


@pytest.mark.parametrize("nt", [4, 8])
def test_batched_gemm_matches_oracle(nt):
    flags = 0
    """The tcgen05 batched GEMM (chpe_probe_bgemm) against the oracle's
    gemvLinear token by token, store and accumulate, x with a few entries
    1e4 times the rest (the int8 pieces' range under the group exponent)."""
    import oracle_py as O
    from _util import archive, assert_close_vec, oracle_threads
    a = archive(chpe.SYNTH_3B_W4, flags)
    e = chpe.Engine.from_bytes(a, chpe.ARCH_3B, 16)
    o = O.OracleEngine(a, O.ARCH_3B, 16, threads=oracle_threads())
    li = o.layer_info(4)
    rng = np.random.default_rng(nt + flags)
    for r, c in BG_SHAPES:
        for acc in (False, True):
            x = rng.standard_normal((nt, c)).astype(np.float32)
            x[:, rng.integers(0, c, 3)] *= 1e4
            y0 = rng.standard_normal((nt, r)).astype(np.float32)
            got = e.probe_bgemm(li["down_proj"], li["down_tiles"], x, r, c, accumulate=acc, y=y0)
            for t in range(nt):
                ref = o.gemv_linear(li["down_proj"], li["down_tiles"], x[t], r, c, accumulate=acc, y=y0[t].copy())
                assert_close_vec(got[t], ref, 1e-4, f"{r}x{c} acc={acc} token {t}")
    e.close()


def test_batched_gemm_refuses_what_it_cannot_run():
    """down_aux replacement cells, and rows that are not whole 128-row blocks,
    are refused (the decode step then keeps the per-token path)."""
    import oracle_py as O
    from _util import archive
    a = archive(chpe.SYNTH_3B_W4, chpe.SYNTH_OUTLIERS)
    e = chpe.Engine.from_bytes(a, chpe.ARCH_3B, 16)
    o = O.OracleEngine(a, O.ARCH_3B, 16)
    li = o.layer_info(4)
    x = np.ones((4, 8192), np.float32)
    with pytest.raises(chpe.ChpeError):
        e.probe_bgemm(li["down_proj"], li["down_tiles"], x, 1024, 8192)
    a0 = archive(chpe.SYNTH_3B_W4)
    e0 = chpe.Engine.from_bytes(a0, chpe.ARCH_3B, 16)
    with pytest.raises(chpe.ChpeError):
        e0.probe_bgemm(li["down_proj"], li["down_tiles"], x, 1000, 8192)
