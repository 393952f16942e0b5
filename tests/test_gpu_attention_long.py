"""Decode attention at long context over the paged KV cache, against the
oracle's f32 attention (chpe_engine.zig:1688-1734).

A layer's cache is prefilled through chpe_kv_load with FP16-representable
rows (the same rows go into the oracle's f32 cache), then the attention step
runs at positions where every split of the positions holds data and the
split merge takes all its batches: max_seq_len 2304 gives 64 splits per kv
head for the Qwen2.5-3B and Qwen3.5-9B geometries and 37 for Qwen2.5-72B's.
Pages are handed out in a seeded random order, so logical and physical
pages differ everywhere."""
import numpy as np
import pytest

import chpe_qwen_engine_b200 as chpe
import oracle_py as O
from _util import assert_close_vec

pytestmark = pytest.mark.gpu

GEOM = {chpe.ARCH_3B: (16, 2, 128), chpe.ARCH_9B: (16, 4, 256), chpe.ARCH_72B: (64, 8, 128)}
MAXS = 2304
POSITIONS = (511, 1023, 2047, 2303)


def fp16_rows(rng, n, width, scale=1.0):
    """Random rows that FP16 holds exactly (the GPU cache is FP16)."""
    return (rng.standard_normal((n, width)) * scale).astype(np.float16).astype(np.float32)


@pytest.mark.parametrize("permuted", [False, True])
@pytest.mark.parametrize("arch", [chpe.ARCH_3B, chpe.ARCH_9B, chpe.ARCH_72B])
def test_attention_long_context_paged(arch, permuted):
    H, KV, HD = GEOM[arch]
    e = chpe.Engine.from_bytes(np.zeros(8192, np.uint8), arch, MAXS)
    rng = np.random.default_rng(100 + arch)
    page = chpe.lib().chpe_kv_page_size()
    _, npages = e.kv_page_table()
    assert npages == (MAXS + page - 1) // page
    order = rng.permutation(npages).astype(np.uint32) if permuted else np.arange(npages, dtype=np.uint32)
    e.kv_set_page_order(order)
    layer = 3
    # keys spread the scores over a few units, so every split carries weight
    kc = fp16_rows(rng, MAXS, KV * HD, 1.5)
    vc = fp16_rows(rng, MAXS, KV * HD)
    e.kv_load(layer, 0, kc, vc)
    table, _ = e.kv_page_table()
    assert np.array_equal(table, order[:len(table)]) and len(table) == npages
    for pos in POSITIONS:
        q = rng.standard_normal(H * HD).astype(np.float32)
        k = rng.standard_normal(KV * HD).astype(np.float32)
        v = rng.standard_normal(KV * HD).astype(np.float32)
        got = e.probe_attention(layer, pos, q, k, v)
        qr = O.apply_rope(q, pos, H, HD)
        kc[pos] = O.apply_rope(k, pos, KV, HD)
        vc[pos] = v
        ref = O.gqa_attention(qr, kc[:pos + 1], vc[:pos + 1], pos, H, KV, HD)
        # the appended entry is rounded to FP16 (the reference keeps f32)
        assert_close_vec(got, ref, 4e-3, f"arch {arch} pos {pos} permuted {permuted}")
    e.close()


def test_kv_pages_follow_the_sequence():
    """Pages map as positions are reached and all return at position 0."""
    e = chpe.Engine.from_bytes(np.zeros(8192, np.uint8), chpe.ARCH_3B, 300)
    page = chpe.lib().chpe_kv_page_size()
    order = np.array([4, 2, 0, 3, 1], np.uint32)
    e.kv_set_page_order(order)
    H, KV, HD = GEOM[chpe.ARCH_3B]
    rng = np.random.default_rng(7)
    q = rng.standard_normal(H * HD).astype(np.float32)
    kv = rng.standard_normal(KV * HD).astype(np.float32)
    e.probe_attention(0, page + 3, q, kv, kv)  # reaches the second page
    table, n = e.kv_page_table()
    assert n == 5 and list(table) == [4, 2]
    e.forward_tokens(np.array([1, 2, 3], np.uint32))  # a new sequence: pages come back in order
    table, _ = e.kv_page_table()
    assert list(table) == [4]
    with pytest.raises(chpe.ChpeError):
        e.kv_set_page_order(np.array([0, 1, 2, 3, 3], np.uint32))
    e.close()
