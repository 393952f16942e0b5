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


def _prefill(e, oracles, L, KV, HD, ctx, rng):
    for l in range(L):
        k = (rng.standard_normal((ctx, KV * HD)) * 1.5).astype(np.float16).astype(np.float32)
        v = rng.standard_normal((ctx, KV * HD)).astype(np.float16).astype(np.float32)
        e.kv_load(l, 0, k, v)
        for o in oracles:
            o.kv_load(l, 0, k, v)


@pytest.fixture(scope="module")
def archive_9b():
    import gc
    a = chpe.synth_archive(chpe.SYNTH_9B_W4)
    yield a
    del a
    gc.collect()


def test_batched_prefill_9b(archive_9b, monkeypatch):
    """Batched prefill: a 21-token prompt through chpe_forward_tokens runs two
    chunks of 8 through the batched tcgen05 step and 5 tokens one by one; the
    last logits match the same prompt on the single-token step and the oracle."""
    a = archive_9b
    prompt = np.random.default_rng(4).integers(0, 248320, 21).astype(np.uint32)
    e = chpe.Engine.from_bytes(a, chpe.ARCH_9B, 64)
    got = np.empty(e.vocab, np.float32)
    e.forward_tokens(prompt, got)
    assert e.position() == 21
    monkeypatch.setenv("CHPE_PREFILL_BATCHED", "0")
    seq = np.empty(e.vocab, np.float32)
    e.forward_tokens(prompt, seq)
    monkeypatch.delenv("CHPE_PREFILL_BATCHED")
    assert_logits_match(got, seq, "batched prefill vs single-token steps")
    o = O.OracleEngine(a, O.ARCH_9B, 64, threads=oracle_threads())
    for p, t in enumerate(prompt):
        o.forward_decode(int(t), p)
    assert_logits_match(got, o.logits(), "batched prefill vs oracle")
    o.close()
    e.close()


@pytest.mark.parametrize("ctx", [5, 2048])
def test_batched_verify_9b(ctx, monkeypatch, archive_9b):
    """Config 4: Qwen3.5-9B 4-bit, batch-4/8 verification through the batched
    tcgen05 step, against the same candidates run as sequential decode steps
    (CHPE_VERIFY_BATCHED=0) and against the oracle; at ctx 5 after a real
    prompt, at ctx 2048 over a prefilled KV cache.  m = 3 pads the batch of 4;
    a second candidate set at the same position checks the rollback."""
    a = archive_9b
    if True:
        e = chpe.Engine.from_bytes(a, chpe.ARCH_9B, ctx + 16)
        assert e.verify_batched_unavailable(8) == ""
        o = O.OracleEngine(a, O.ARCH_9B, ctx + 16, threads=oracle_threads())
        o16 = O.OracleEngine(a, O.ARCH_9B, ctx + 16, threads=oracle_threads())
        o16.set_kv_fp16(True)
        rng = np.random.default_rng(ctx)
        if ctx == 5:
            e.forward_tokens(PROMPT)
            for p, t in enumerate(PROMPT):
                o.forward_decode(int(t), p)
                o16.forward_decode(int(t), p)
        else:
            _prefill(e, (o, o16), 32, 4, 256, ctx, rng)
        for m in (4, 8, 3):
            cand = rng.integers(0, e.vocab, m).astype(np.uint32)
            lg, am = e.verify(cand, ctx)
            assert e.last_verify_batched(), e.verify_batched_unavailable(m)
            monkeypatch.setenv("CHPE_VERIFY_BATCHED", "0")
            lg_seq, am_seq = e.verify(cand, ctx)  # rollback to the same position
            assert not e.last_verify_batched()
            monkeypatch.delenv("CHPE_VERIFY_BATCHED")
            for i, t in enumerate(cand):
                assert_logits_match(lg[i], lg_seq[i], f"ctx {ctx} m {m} cand {i} vs sequential")
                assert int(am[i]) == int(np.argmax(lg[i]))
                o.forward_decode(int(t), ctx + i)
                o16.forward_decode(int(t), ctx + i)
                assert_logits_match(lg[i], o.logits(), f"ctx {ctx} m {m} cand {i} vs oracle")
                assert_logits_match(lg[i], o16.logits(), f"ctx {ctx} m {m} cand {i} vs oracle, FP16 KV")
        o.close()
        o16.close()
        e.close()


def test_all_batched_prompt_then_single_token_steps(monkeypatch):
    """A prompt whose every token goes through the batched step (a multiple
    of 8) leaves the engine ready for single-token steps: greedy steps on the
    device and host-driven steps run, and their results equal those after
    the same prompt decoded token by token (within f32 summation order)."""
    a = archive(chpe.SYNTH_3B_W4)
    prompt = np.random.default_rng(4).integers(0, 151936, 16).astype(np.uint32)
    res = []
    for batched in ("1", "0"):
        monkeypatch.setenv("CHPE_PREFILL_BATCHED", batched)
        e = chpe.Engine.from_bytes(a, chpe.ARCH_3B, 64)
        e.forward_tokens(prompt)
        first = e.logits().copy()
        e.bench_greedy(3)
        r = e.last_result()
        _, lg = e.bench_host(np.array([5, 77], np.uint32))
        res.append((first, r.argmax_token, lg))
        e.close()
    (f1, t1, l1), (f0, t0, l0) = res
    assert_logits_match(f1, f0, "batched vs sequential prompt")
    assert t1 == t0
    assert_logits_match(l1, l0, "host steps after the prompt")
