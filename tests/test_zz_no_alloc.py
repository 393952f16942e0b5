"""The allocation-free attention entry point (chpe_attention_decode_noalloc).

Callers that cannot allocate device memory -- code recorded into a CUDA
graph, runtimes with their own fixed pools, plugins in a process that owns
all allocation -- call it with their own device buffers; its scratch is a
static device array inside the library.  This test runs it twice in a row on
consecutive positions and checks each output against the engine's attention
entry point (chpe_probe_attention, which uses the engine's allocated scratch)
fed the same inputs, within the attention tolerance of the parity suite.
It sits in its own file, collected last, and runs alone or after the others.
"""
import ctypes as C

import numpy as np
import pytest

import chpe_qwen_engine_b200 as chpe
from _util import assert_close_vec

pytestmark = pytest.mark.gpu


def test_noalloc_attention_matches_allocating_entry_point():
    torch = pytest.importorskip("torch")
    assert torch.cuda.is_available()
    H, KV, HD, MAXS = 16, 2, 128, 64  # Qwen2.5-3B attention geometry
    eng = chpe.Engine.from_bytes(np.zeros(8192, np.uint8), chpe.ARCH_3B, MAXS)
    dev = torch.device("cuda:0")
    kc = torch.zeros((MAXS, KV, HD), dtype=torch.float16, device=dev)
    vc = torch.zeros((MAXS, KV, HD), dtype=torch.float16, device=dev)
    out = torch.empty(H * HD, dtype=torch.float32, device=dev)
    rng = np.random.default_rng(42)
    L = chpe.lib()
    stream = torch.cuda.current_stream().cuda_stream
    for pos in (0, 1):  # two calls in a row; the second reads what the first appended
        q = rng.standard_normal(H * HD).astype(np.float32)
        k = rng.standard_normal(KV * HD).astype(np.float32)
        v = rng.standard_normal(KV * HD).astype(np.float32)
        ref = eng.probe_attention(0, pos, q, k, v)
        tq, tk, tv = (torch.from_numpy(a).to(dev) for a in (q, k, v))
        rc = L.chpe_attention_decode_noalloc(tq.data_ptr(), tk.data_ptr(), tv.data_ptr(),
                                             kc.data_ptr(), vc.data_ptr(), out.data_ptr(), pos, MAXS,
                                             H, KV, HD, 1000000.0, stream)
        assert rc == 0
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert_close_vec(got, ref, 4e-3, f"pos {pos}")
    # sizes beyond the scratch limit are rejected, not run
    assert L.chpe_attention_decode_noalloc(tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), kc.data_ptr(),
                                           vc.data_ptr(), out.data_ptr(), 0, MAXS, 512, 64, 256,
                                           1000000.0, stream) == -2
    eng.close()
