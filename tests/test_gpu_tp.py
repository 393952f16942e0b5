"""Tensor-parallel decode on 2 GPUs (skipped with fewer): two processes, one
per GPU, each building rank r of Engine.tensor_parallel over the same seeded
9B 4-bit archive, exchanging the IPC handles over a gloo group on 127.0.0.1.
Both ranks must report the same logits and results (every element is computed
on one rank and copied to the other), and those must match the CPU oracle
under the per-step gate (max-abs-err <= 2e-2, cosine >= 0.9999, argmax where
the margin exceeds 1e-3) and the single-GPU engine within f32 summation
order.  Each rank holds only the archive tiles it reads (under 60 % of the
archive at 2 ranks)."""
import os
import socket

import numpy as np
import pytest

import chpe_qwen_engine_b200 as chpe
import oracle_py as O
from _util import assert_close_vec, assert_logits_match, oracle_threads

pytestmark = pytest.mark.gpu

TOKENS = [5, 248000, 77, 1234]


def _gpus() -> int:
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, cfg, q):
    try:
        _rank_body(rank, world, port, cfg, q)
    except BaseException:  # report to the parent at once instead of leaving it waiting
        import traceback
        q.put((rank, "error", traceback.format_exc()))
        raise


def _rank_body(rank, world, port, cfg, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=120))
    try:
        a = chpe.synth_archive(cfg, threads=max(1, (os.cpu_count() or 2) // world))
        e = chpe.Engine.tensor_parallel(a, chpe.SYNTH_ARCH[cfg], rank, world, max_seq_len=64)
        out = []
        for pos, t in enumerate(TOKENS):
            r = e.forward_decode(t, pos)
            out.append((r.argmax_token, r.max_logit, r.token0_logit, r.hidden_norm, r.all_finite,
                        e.logits().copy()))
        gen = e.generate(np.array([11, 2222, 33333], np.uint32), 4)
        # the rank holds only the tiles it reads: its slices and the embedding
        assert e.device_archive_bytes() < 0.6 * a.size, (e.device_archive_bytes(), a.size)
        q.put((rank, out, [int(x) for x in gen]))
        e.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("rowblk", ["0", "1"])
def test_tp2_decode_matches_oracle_and_single_gpu(rowblk, monkeypatch):
    """rowblk "1": the down projections on the row-block tensor-core kernel
    (its exchange: outputs broadcast to both ranks, one arrival per CTA)."""
    import torch.multiprocessing as mp
    monkeypatch.setenv("CHPE_FLAT_ROWBLK", rowblk)  # inherited by the spawned ranks
    cfg, world = chpe.SYNTH_9B_W4, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, cfg, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, out, gen = q.get(timeout=600)
            assert out != "error", f"rank {r} failed:\n{gen}"
            res[r] = (out, gen)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for p in procs:
        assert p.exitcode == 0
    # ranks agree exactly
    for i in range(len(TOKENS)):
        a0, a1 = res[0][0][i], res[1][0][i]
        assert a0[:5] == a1[:5]
        assert np.array_equal(a0[5], a1[5])
    assert res[0][1] == res[1][1]
    a = chpe.synth_archive(cfg)
    arch = chpe.SYNTH_ARCH[cfg]
    o = O.OracleEngine(a, arch, 64, threads=oracle_threads())
    e1 = chpe.Engine.from_bytes(a, arch, 64)
    for pos, t in enumerate(TOKENS):
        r_ref = o.forward_decode(t, pos)
        r1 = e1.forward_decode(t, pos)
        tp = res[0][0][pos]
        assert_logits_match(tp[5], o.logits(), f"tp2 pos {pos}")
        assert_close_vec(tp[5], e1.logits(), 1e-5, f"tp2 vs 1 GPU pos {pos}")
        assert tp[4] == bool(r_ref.all_finite)
        assert abs(tp[3] - r1.hidden_norm) <= 1e-4 * max(1.0, r1.hidden_norm)
        assert tp[0] == int(np.argmax(tp[5])) and tp[2] == tp[5][0]
    gen1 = e1.generate(np.array([11, 2222, 33333], np.uint32), 4)
    assert res[0][1] == [int(x) for x in gen1]
