"""Speculative greedy decoding (chpe_speculative_generate) around chpe_verify:
prompt-lookup drafts, greedy acceptance, rollback by overwriting the KV
entries of rejected draft tokens.  Its output must equal plain greedy
generation (chpe_generate) token for token, and the draft counters must be
consistent.  The 4-bit synthetic model keeps one argmax across positions, so
its drafts are accepted; the FP16 model's are mostly rejected, which
exercises the rollback on every round."""
import numpy as np
import pytest

import chpe_qwen_engine_b200 as chpe
from _util import archive

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cfg,draft", [(chpe.SYNTH_3B_W4, 4), (chpe.SYNTH_3B_FP16_RAW, 8),
                                       (chpe.SYNTH_3B_W2, 3)])
def test_speculative_equals_greedy(cfg, draft):
    a = archive(cfg)
    e = chpe.Engine.from_bytes(a, chpe.SYNTH_ARCH[cfg], 128)
    prompt = np.array([11, 2222, 33333, 11, 2222, 151000, 7, 11, 2222], np.uint32)
    n_gen = 40
    ref = e.generate(prompt, n_gen)
    got, st = e.speculative_generate(prompt, n_gen, draft_len=draft, ngram=2)
    assert np.array_equal(got, ref), (got, ref)
    assert 1 <= st["rounds"] <= n_gen
    assert st["accepted"] <= st["proposed"] <= st["rounds"] * draft
    # every round emits its accepted drafts plus one token
    assert st["accepted"] + st["rounds"] >= n_gen - 1
    if cfg == chpe.SYNTH_3B_W4:
        assert st["accepted"] > 0
    e.close()
