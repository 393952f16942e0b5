"""Batch-M verification (chpe_verify) on the GPU: m candidates scored at
positions pos..pos+m-1 must equal m sequential forwardDecode steps (same
kernels: bit-identical logits) and the CPU oracle under the per-step gate;
verifying a second candidate set at the same position (rollback) must equal a
fresh sequential decode of that set."""
import numpy as np
import pytest

import chpe_qwen_engine_b200 as chpe
import oracle_py as O
from _util import archive, assert_logits_match, oracle_threads

pytestmark = pytest.mark.gpu

PROMPT = np.array([11, 2222, 33333, 151000, 7], np.uint32)


@pytest.mark.parametrize("cfg,m", [(chpe.SYNTH_3B_W4, 4), (chpe.SYNTH_3B_FP16_RAW, 8)])
def test_verify_equals_sequential_decode_and_oracle(cfg, m):
    a = archive(cfg)
    arch = chpe.SYNTH_ARCH[cfg]
    rng = np.random.default_rng(9)
    cand = rng.integers(0, 151936, m).astype(np.uint32)
    cand2 = rng.integers(0, 151936, m).astype(np.uint32)
    pos = PROMPT.size

    e = chpe.Engine.from_bytes(a, arch, 64)
    e.forward_tokens(PROMPT)
    lg, am = e.verify(cand, pos)
    assert lg.shape == (m, e.vocab) and am.shape == (m,)
    assert e.last_result().argmax_token == int(am[-1])
    # rollback: a second candidate set at the same position
    lg2, am2 = e.verify(cand2, pos)

    s = chpe.Engine.from_bytes(a, arch, 64)
    o = O.OracleEngine(a, arch, 64, threads=oracle_threads())
    for p, t in enumerate(PROMPT):
        o.forward_decode(int(t), p)
    s.forward_tokens(PROMPT)
    for i, t in enumerate(cand):
        s.forward_decode(int(t), pos + i)
        assert np.array_equal(lg[i], s.logits()), i
        assert int(am[i]) == int(np.argmax(lg[i]))
        o.forward_decode(int(t), pos + i)
        assert_logits_match(lg[i], o.logits(), f"verify cfg {cfg} cand {i}")
    s.forward_tokens(PROMPT)
    for i, t in enumerate(cand2):
        s.forward_decode(int(t), pos + i)
        assert np.array_equal(lg2[i], s.logits()), i
        assert int(am2[i]) == int(np.argmax(lg2[i]))


def test_verify_rejects_bad_arguments():
    a = archive(chpe.SYNTH_3B_W4)
    e = chpe.Engine.from_bytes(a, chpe.ARCH_3B, 16)
    with pytest.raises(chpe.ChpeError):
        e.verify(np.arange(8, dtype=np.uint32), 12)  # past max_seq_len
    L = chpe.lib()
    assert L.chpe_verify(e.ctx, None, 4, 0, None, None) == -1
    t = np.array([1], np.uint32)
    assert L.chpe_verify(e.ctx, t.ctypes.data_as(chpe._U32P), 0, 0, None, None) == -1
