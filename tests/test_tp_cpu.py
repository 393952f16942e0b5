"""Tensor-parallel host logic without a GPU, on gloo ranks (world size 2 and
4, 127.0.0.1): every rank computes its slices with chpe_tp_slice (the
function the engine's tensor-parallel step uses), the ranks all-gather them,
and together they must tile the query heads, the hidden, FFN and vocabulary
rows exactly once, with every query head's kv head owned by its rank.  The
IPC-handle exchange of Engine.tensor_parallel (all_gather_object over the
default group) is exercised with stand-in 64-byte handles."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import chpe_qwen_engine_b200 as chpe

ARCHS = {chpe.ARCH_3B: (2048, 11008, 16, 2, 151936), chpe.ARCH_9B: (4096, 12288, 16, 4, 248320),
         chpe.ARCH_72B: (8192, 29568, 64, 8, 152064)}


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        slices = {}
        for arch in ARCHS:
            try:
                mine = chpe.tp_slice(arch, rank, world)
            except ValueError:
                mine = None
            got = [None] * world
            dist.all_gather_object(got, mine)
            slices[arch] = got
        # the handle exchange the engine uses, with stand-in handles
        h = bytes([rank]) * 64
        out = [None] * world
        dist.all_gather_object(out, h)
        if rank == 0:
            q.put((slices, out))
    finally:
        dist.destroy_process_group()


def _run(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return res


def _covers(parts, total):
    """(count, first) pairs tile [0, total) once, in rank order."""
    pos = 0
    for n, first in parts:
        assert first == pos
        pos += n
    assert pos == total


@pytest.mark.parametrize("world", [2, 4])
def test_tp_slices_tile_every_dimension(world):
    slices, handles = _run(world)
    assert handles == [bytes([r]) * 64 for r in range(world)]
    for arch, (D, F, H, KV, V) in ARCHS.items():
        per = slices[arch]
        assert all(s is not None for s in per), (arch, world)
        _covers([(s["hq"], s["h0"]) for s in per], H)
        _covers([(s["dl"], s["d0"]) for s in per], D)
        _covers([(s["fl"], s["f0"]) for s in per], F)
        _covers([(s["vl"], s["v0"]) for s in per], V)
        G = H // KV
        for s in per:
            for h in range(s["h0"], s["h0"] + s["hq"]):
                assert s["kv0"] <= h // G < s["kv0"] + s["kvl"]
            assert s["hq"] // s["kvl"] * s["kvl"] == s["hq"]  # whole local groups


def test_tp_slice_rejects_uneven_splits():
    with pytest.raises(ValueError):
        chpe.tp_slice(chpe.ARCH_72B, 0, 3)  # 64 heads over 3 ranks
    with pytest.raises(ValueError):
        chpe.tp_slice(chpe.ARCH_72B, 5, 4)  # rank out of range
    s = chpe.tp_slice(chpe.ARCH_72B, 7, 8)
    assert (s["hq"], s["h0"], s["kv0"], s["kvl"]) == (8, 56, 7, 1)
    s = chpe.tp_slice(chpe.ARCH_9B, 5, 8)  # 2 query heads of kv group 2 (4 per group)
    assert (s["hq"], s["h0"], s["kv0"], s["kvl"]) == (2, 10, 2, 1)
