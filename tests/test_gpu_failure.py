"""Failure detection on the GPU without a GPU fault: a bounded device wait of
the kind the tensor-parallel exchanges use is given an arrival that nothing
sends, under a short poll limit.  The kernel must give up and return, the
host must report the timeout through chpe_last_error, and the context must
decode correctly afterwards."""
import time

import numpy as np
import pytest

import chpe_qwen_engine_b200 as chpe
from _util import archive

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_stays_usable():
    e = chpe.Engine.from_bytes(archive(chpe.SYNTH_3B_W4), chpe.ARCH_3B, 32)
    toks = np.array([5, 77, 1024], np.uint32)
    e.forward_tokens(toks)
    before = e.logits()
    L = chpe.lib()
    t0 = time.time()
    rc = L.chpe_probe_wait_timeout(e.ctx, 20000)
    took = time.time() - t0
    assert rc == -1
    assert b"timed out" in L.chpe_last_error(e.ctx)
    assert took < 30.0
    # the flag was cleared: the same sequence decodes to the same logits
    e.forward_tokens(toks)
    assert np.array_equal(e.logits(), before)
    assert e.last_result().all_finite
    e.close()
