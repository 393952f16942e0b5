"""Tensor-parallel host logic without a GPU, on gloo ranks (world size 2, 4
and 8, 127.0.0.1): every rank computes its slices with chpe_tp_slice (the
function the engine's tensor-parallel step uses), the ranks all-gather them,
and together they must tile the query heads, the hidden, FFN and vocabulary
rows exactly once, with every query head's kv head owned by its rank.  The
IPC-handle exchange of Engine.tensor_parallel (all_gather_object over the
default group) is exercised with stand-in 64-byte handles.  The sharded
loader's tile runs are checked against the oracle's tensor maps, and the
sharded math itself runs on CPU ranks: row slices computed from each rank's
tiles, exchanged by an all-gather, equal the unsharded oracle bit for bit;
a rank that leaves or never arrives ends the exchange with an error."""
import bisect
import os
import socket
import struct

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


@pytest.mark.parametrize("world", [2, 4, 8])
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


# Sharded loading: the tiles one rank uploads (chpe_tp_tile_runs, the function
# the engine's loader calls) against what its kernels read, derived here from
# the oracle's tensor maps (getLayerInfo, chpe_engine.zig:1035-1142) and the
# untied LM head spans (qwen35_tensor_map.zig LM_HEAD_TILE, qwen72b_tensor_map.zig
# LM_HEAD_RECORD_START).  A flat GEMV over rows [r0, r0+n) with C columns from
# tile `start` reads tiles start + r0*C // 32768 .. ceil((r0+n)*C / 32768),
# never past the tensor's own tiles.
TOTAL = {chpe.ARCH_9B: 546681, chpe.ARCH_72B: 2219153}
LM_HEAD = {chpe.ARCH_9B: (484601, 62080), chpe.ARCH_72B: (2181137, 38016)}
HEAD_DIM = {chpe.ARCH_9B: 256, chpe.ARCH_72B: 128}
LAYERS = {chpe.ARCH_9B: 32, chpe.ARCH_72B: 80}


def _reads(start, tiles, r0, n, C, wpt=32768):
    if start < 0:
        return None
    hi = min(start + -(-(r0 + n) * C // wpt), start + tiles)
    return (start + r0 * C // wpt, hi)


def _needed(arch, layers, s):
    D, F, H, KV, V = ARCHS[arch]
    HD = HEAD_DIM[arch]
    out = [(0, -(-V // 16) + 2)]  # embedding records and two past them
    for li in layers:
        out += [_reads(li["q_proj"], li["q_tiles"], s["h0"] * HD, s["hq"] * HD, D),
                _reads(li["k_proj"], li["k_tiles"], s["kv0"] * HD, s["kvl"] * HD, D),
                _reads(li["v_proj"], li["v_tiles"], s["kv0"] * HD, s["kvl"] * HD, D),
                _reads(li["o_proj"], li["o_tiles"], s["d0"], s["dl"], D),
                _reads(li["gate_proj"], li["gate_tiles"], s["f0"], s["fl"], D),
                _reads(li["up_proj"], li["up_tiles"], s["f0"], s["fl"], D),
                _reads(li["down_proj"], li["down_tiles"], s["d0"], s["dl"], F)]
    out.append(_reads(*LM_HEAD[arch], s["v0"], s["vl"], D))
    return [r for r in out if r is not None and r[1] > r[0]]


@pytest.mark.parametrize("arch", [chpe.ARCH_9B, chpe.ARCH_72B])
def test_tp_tile_runs_hold_every_slice(arch):
    import bisect

    import numpy as np
    import oracle_py as O
    total = TOTAL[arch]
    e = O.OracleEngine(np.zeros(8192, np.uint8), arch, 4)  # maps only; no archive bytes read
    layers = [e.layer_info(l) for l in range(LAYERS[arch])]
    D, F, H, KV, V = ARCHS[arch]
    whole = {"hq": H, "h0": 0, "kv0": 0, "kvl": KV, "dl": D, "d0": 0, "fl": F, "f0": 0, "vl": V, "v0": 0}
    for world in (2, 4, 8):
        union = np.zeros(total, bool)
        for rank in range(world):
            runs = chpe.tp_tile_runs(arch, False, 32768, total, rank, world)
            assert runs and all(0 <= lo < hi <= total for lo, hi in runs)
            assert all(a[1] < b[0] for a, b in zip(runs, runs[1:])), "runs disjoint, ascending, merged"
            los = [lo for lo, _ in runs]
            for lo, hi in _needed(arch, layers, chpe.tp_slice(arch, rank, world)):
                i = bisect.bisect_right(los, lo) - 1
                assert i >= 0 and runs[i][0] <= lo and hi <= runs[i][1], (world, rank, lo, hi)
            held = sum(hi - lo for lo, hi in runs)
            embed = -(-V // 16) + 2
            # a rank holds the embedding plus about 1/world of the rest
            assert held <= embed + (total - embed) / world * 1.05 + 8 * len(layers), (world, rank, held)
            for lo, hi in runs:
                union[lo:hi] = True
        # together the ranks hold everything one GPU's kernels read
        for lo, hi in _needed(arch, layers, whole):
            assert union[lo:hi].all(), (world, lo, hi)
    # a rank of the 9B at 2 ranks uploads under 60 % of the archive (the
    # tensor-parallel GPU test checks the same bound on the device)
    if arch == chpe.ARCH_9B:
        held = sum(hi - lo for lo, hi in chpe.tp_tile_runs(arch, False, 32768, total, 0, 2))
        assert held < 0.6 * total


def test_tp_tile_runs_rejects_uneven_splits():
    with pytest.raises(ValueError):
        chpe.tp_tile_runs(chpe.ARCH_72B, False, 32768, TOTAL[chpe.ARCH_72B], 0, 3)


# ---- sharded math on CPU ranks ------------------------------------------------
# Each gloo rank computes its row slice of every projection of two 9B layers
# (a Q8 linear layer and a full-attention layer) from the tiles its sharded
# loader would upload (chpe_tp_tile_runs), tile by tile in the reference's
# order through the oracle's gemvCellFlat; an all-gather stands in for the
# peer-memory exchange, and the gathered outputs must equal the unsharded
# oracle's gemvLinear bit for bit (each output element is computed whole on
# one rank with the same f32 arithmetic).  A rank that never arrives makes
# the others' exchange end with an error within the group's timeout.
LAYERS_9B = (0, 3)
CELL9 = 17408


def _sparse_9b_archive(path: str) -> None:
    """A dense 9B-sized archive file whose only written records are random
    4-bit group-scaled cells (some with down_aux replacements) at the tiles
    of LAYERS_9B's projections and record 0; the rest are holes."""
    import numpy as np
    import oracle_py as O
    total = TOTAL[chpe.ARCH_9B]
    hdr = np.zeros(4096, np.uint8)
    hdr[:64] = np.frombuffer(struct.pack("<IIQQQQQQQ", 0x57415243, 1, 4096, total, total, CELL9, CELL9, 0, 0),
                             np.uint8)
    e = O.OracleEngine(np.zeros(8192, np.uint8), O.ARCH_9B, 4)  # maps only
    rng = np.random.default_rng(17)
    tiles = {0}
    for l in LAYERS_9B:
        li = e.layer_info(l)
        for p in ("q", "k", "v", "o", "gate", "up", "down"):
            tiles.update(range(li[f"{p}_proj"], li[f"{p}_proj"] + li[f"{p}_tiles"]))
    with open(path, "wb") as f:
        f.truncate(4096 + total * CELL9)
        f.write(hdr.tobytes())
        for t in sorted(tiles):
            c = np.zeros(CELL9, np.uint8)
            c[64:64 + 16384] = rng.integers(0, 256, 16384, dtype=np.uint8)
            pl = 16448
            c[pl + 20] = 4
            c[pl + 24] = 1  # group-128 scales
            c[pl + 48:pl + 560] = np.abs(rng.normal(0, 0.01, 256)).astype(np.float16).view(np.uint8)
            n = int(rng.integers(0, 5)) if t % 7 == 0 else 0
            c[pl + 560:pl + 562] = np.frombuffer(struct.pack("<H", n), np.uint8)
            c[pl + 562:pl + 562 + 2 * n] = rng.normal(0, 0.5, n).astype(np.float16).view(np.uint8)
            c[pl + 690:pl + 690 + 2 * n] = rng.integers(0, 32768, n).astype(np.uint16).view(np.uint8)
            f.seek(4096 + t * CELL9)
            f.write(c.tobytes())


def _projections(li, s, D, F, HD):
    """(name, first tile, tiles, rank's first row, rows, all rows, columns)."""
    return [("q", li["q_proj"], li["q_tiles"], s["h0"] * HD, s["hq"] * HD, 16 * HD, D),
            ("k", li["k_proj"], li["k_tiles"], s["kv0"] * HD, s["kvl"] * HD, 4 * HD, D),
            ("v", li["v_proj"], li["v_tiles"], s["kv0"] * HD, s["kvl"] * HD, 4 * HD, D),
            ("o", li["o_proj"], li["o_tiles"], s["d0"], s["dl"], D, D),
            ("gate", li["gate_proj"], li["gate_tiles"], s["f0"], s["fl"], F, D),
            ("up", li["up_proj"], li["up_tiles"], s["f0"], s["fl"], F, D),
            ("down", li["down_proj"], li["down_tiles"], s["d0"], s["dl"], D, F)]


def _inputs(D, F):
    import numpy as np
    rng = np.random.default_rng(23)
    return rng.standard_normal(D).astype(np.float32), rng.standard_normal(F).astype(np.float32)


def _shard_worker(rank, world, port, path, skip_rank, skip_mode, timeout_s, q):
    import time

    import numpy as np
    import oracle_py as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=timeout_s))
    try:
        if rank == skip_rank:
            # this rank never arrives at the exchange: it leaves the group at
            # once ("exit"), or stays alive past the group's timeout ("stall")
            if skip_mode == "stall":
                time.sleep(timeout_s + 6)
            return
        D, F, HD = 4096, 12288, 256
        a = np.memmap(path, dtype=np.uint8, mode="r")
        e = O.OracleEngine(np.zeros(8192, np.uint8), O.ARCH_9B, 4)
        s = chpe.tp_slice(chpe.ARCH_9B, rank, world)
        runs = chpe.tp_tile_runs(chpe.ARCH_9B, False, 32768, TOTAL[chpe.ARCH_9B], rank, world)
        los = [lo for lo, _ in runs]
        xd, xf = _inputs(D, F)
        mine, used = {}, 0
        for l in LAYERS_9B:
            for name, start, tiles, r0, n, rows, cols in _projections(e.layer_info(l), s, D, F, HD):
                x = xf if cols == F else xd
                y = np.zeros(rows, np.float32)
                t_hi = min(-(-(r0 + n) * cols // 32768), tiles)
                for t in range(r0 * cols // 32768, t_hi):
                    g = start + t
                    i = bisect.bisect_right(los, g) - 1
                    assert i >= 0 and g < runs[i][1], ("tile outside this rank's upload", g)
                    cell = np.asarray(a[4096 + g * CELL9:4096 + (g + 1) * CELL9])
                    O.gemv_cell_flat(cell, t, rows, cols, x, y)
                    used += 1
                mine[(l, name)] = y[r0:r0 + n].copy()
        out = [None] * world
        dist.all_gather_object(out, (rank, mine, used))
        if rank == 0:
            q.put(("ok", out))
    except Exception as ex:  # the exchange with a missing rank ends here
        q.put(("error", rank, type(ex).__name__, str(ex)[:200]))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run_shards(world, path, skip_rank=-1, skip_mode="exit", timeout_s=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_shard_worker, args=(r, world, port, path, skip_rank, skip_mode, timeout_s, q),
                         daemon=True) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = q.get(timeout=300)
    finally:
        for p in procs:  # the processes this call started, by handle
            p.join(timeout=120)
            if p.is_alive():
                p.terminate()
    return res, [p.exitcode for p in procs]


@pytest.fixture(scope="module")
def sparse_9b(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("tp") / "sparse_9b.chpe")
    _sparse_9b_archive(path)
    return path


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_projections_equal_unsharded_oracle(sparse_9b, world):
    import numpy as np
    import oracle_py as O
    res, codes = _run_shards(world, sparse_9b)
    assert res[0] == "ok", res
    assert codes == [0] * world
    parts = sorted(res[1], key=lambda t: t[0])
    a = np.memmap(sparse_9b, dtype=np.uint8, mode="r")
    e = O.OracleEngine(a, O.ARCH_9B, 4, threads=8)
    D, F, HD = 4096, 12288, 256
    xd, xf = _inputs(D, F)
    whole = chpe.tp_slice(chpe.ARCH_9B, 0, 1)
    for l in LAYERS_9B:
        for name, start, tiles, _, _, rows, cols in _projections(e.layer_info(l), whole, D, F, HD):
            want = e.gemv_linear(start, tiles, xf if cols == F else xd, rows, cols)
            got = np.concatenate([p[1][(l, name)] for p in parts])  # rank order = row order
            assert np.array_equal(got, want), (l, name, float(np.max(np.abs(got - want))))
    assert all(p[2] > 0 for p in parts)
    # the ranks together read each needed tile about once (row slices split tiles only at their edges)
    assert sum(p[2] for p in parts) < 1.01 * _run_tiles_needed(e) + 2 * world * 7 * len(LAYERS_9B)


def _run_tiles_needed(e) -> int:
    n = 0
    for l in LAYERS_9B:
        for _, start, tiles, _, _, rows, cols in _projections(e.layer_info(l), chpe.tp_slice(chpe.ARCH_9B, 0, 1),
                                                              4096, 12288, 256):
            n += min(-(-rows * cols // 32768), tiles)
    return n


@pytest.mark.parametrize("mode", ["exit", "stall"])
def test_missing_rank_ends_the_exchange_with_an_error(sparse_9b, mode):
    """A rank that leaves, or one that never arrives, makes rank 0's
    exchange raise (connection closed, or the group's 8 s timeout) instead
    of waiting for good; every process then exits normally."""
    import time
    t0 = time.time()
    res, codes = _run_shards(2, sparse_9b, skip_rank=1, skip_mode=mode, timeout_s=8)
    assert res[0] == "error" and res[1] == 0, res
    assert codes == [0, 0] and time.time() - t0 < 120
