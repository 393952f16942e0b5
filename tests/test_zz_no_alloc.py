"""The allocation-free attention entry point (chpe_attention_decode_noalloc).

Serving runtimes that hand out device memory only from their own pre-sized
pools, and plugins inside a host process that owns all GPU allocation, cannot
let this library call cudaMalloc.  They call this entry point with their own
device buffers; its scratch is a static device array inside the library.

The test prefills a cache at long context (511 positions, so all 16 splits
of the positions hold data and the split merge combines them), then calls the
entry point twice in a row, at positions 511 and 512 (the second call reads
what the first appended), and checks each output against the engine's
attention entry point (chpe_probe_attention, which uses the engine's
allocated scratch) fed the same cache and inputs, and against the CPU
oracle, within the attention tolerance of the parity suite.  A geometry no
model has (head_dim 256 with 8 query heads per kv head) is checked against
the oracle alone.  It sits in its own file, collected last, and runs alone or
after the others.
"""
import numpy as np
import pytest

import chpe_qwen_engine_b200 as chpe
import oracle_py as O
from _util import assert_close_vec

pytestmark = pytest.mark.gpu

MAXS = 1024
CTX = 511
GEOM = {chpe.ARCH_3B: (16, 2, 128), chpe.ARCH_9B: (16, 4, 256), chpe.ARCH_72B: (64, 8, 128)}


def _fp16_rows(rng, n, width, scale=1.0):
    return (rng.standard_normal((n, width)) * scale).astype(np.float16).astype(np.float32)


def _run(torch, H, KV, HD, rng, eng=None):
    """Two calls in a row at CTX and CTX+1 over a prefilled cache; returns the
    largest deviation seen, after checking every output."""
    L = chpe.lib()
    dev = torch.device("cuda:0")
    stream = torch.cuda.current_stream().cuda_stream
    kc = _fp16_rows(rng, MAXS, KV * HD, 1.5)
    vc = _fp16_rows(rng, MAXS, KV * HD)
    tkc = torch.from_numpy(kc.reshape(MAXS, KV, HD)).to(dev).half()
    tvc = torch.from_numpy(vc.reshape(MAXS, KV, HD)).to(dev).half()
    out = torch.empty(H * HD, dtype=torch.float32, device=dev)
    if eng is not None:
        eng.kv_load(0, 0, kc[:CTX], vc[:CTX])
    for pos in (CTX, CTX + 1):  # the second call reads what the first appended
        q = rng.standard_normal(H * HD).astype(np.float32)
        k = rng.standard_normal(KV * HD).astype(np.float32)
        v = rng.standard_normal(KV * HD).astype(np.float32)
        tq, tk, tv = (torch.from_numpy(a).to(dev) for a in (q, k, v))
        rc = L.chpe_attention_decode_noalloc(tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), tkc.data_ptr(),
                                             tvc.data_ptr(), out.data_ptr(), pos, MAXS, H, KV, HD,
                                             1000000.0, stream)
        assert rc == 0, L.chpe_last_error(None).decode()
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        kc[pos] = O.apply_rope(k, pos, KV, HD)
        vc[pos] = v
        ref = O.gqa_attention(O.apply_rope(q, pos, H, HD), kc[:pos + 1], vc[:pos + 1], pos, H, KV, HD)
        assert_close_vec(got, ref, 4e-3, f"oracle, pos {pos}")
        if eng is not None:
            alloc = eng.probe_attention(0, pos, q, k, v)
            assert_close_vec(got, alloc, 4e-3, f"allocating entry point, pos {pos}")


@pytest.mark.parametrize("arch", [chpe.ARCH_3B, chpe.ARCH_9B, chpe.ARCH_72B])
def test_noalloc_attention_matches_allocating_entry_point(arch):
    torch = pytest.importorskip("torch")
    assert torch.cuda.is_available()
    H, KV, HD = GEOM[arch]
    eng = chpe.Engine.from_bytes(np.zeros(8192, np.uint8), arch, MAXS)
    _run(torch, H, KV, HD, np.random.default_rng(42 + arch), eng)
    eng.close()


def test_noalloc_attention_hd256_g8_and_limits():
    torch = pytest.importorskip("torch")
    assert torch.cuda.is_available()
    _run(torch, 32, 4, 256, np.random.default_rng(77))
    # sizes beyond the scratch limit are rejected, not run, with a reason
    L = chpe.lib()
    dev = torch.device("cuda:0")
    buf = torch.zeros(1 << 20, dtype=torch.float32, device=dev)
    p = buf.data_ptr()
    stream = torch.cuda.current_stream().cuda_stream
    assert L.chpe_attention_decode_noalloc(p, p, p, p, p, p, 0, 16, 512, 64, 256, 1000000.0, stream) == -2
    assert b"scratch" in L.chpe_last_error(None)
    assert L.chpe_attention_decode_noalloc(p, p, p, p, p, p, 16, 16, 16, 2, 128, 1000000.0, stream) == -1
    assert b"pos" in L.chpe_last_error(None)
