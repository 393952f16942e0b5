"""Pin the CPU oracle to the known answers in the reference's own unit tests.

Each test cites the reference test it restates (chpe-qwen-engine, path:line).
These run on CPU only.
"""
import json
import os
import struct

import numpy as np
import pytest

import oracle_py as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def make_cell(quant_bits, flags=0, scale=0.0, bias=0.0, rows=0, cols=0):
    """A zeroed 17408-byte Cell with TileMetadata/TileDims filled in
    (geometry.zig:243-256, weight_archive.zig:92-105, chpe_engine.zig:150-155)."""
    c = np.zeros(17408, np.uint8)
    pl = 16448
    c[pl + 20] = quant_bits
    c[pl + 24:pl + 32] = np.frombuffer(struct.pack("<Q", flags), np.uint8)
    c[pl + 32:pl + 48] = np.frombuffer(struct.pack("<ffII", scale, bias, rows, cols), np.uint8)
    return c


# chpe_engine.zig:1814-1838 "polymorphic GEMV 2-bit cell"
def test_gemv_2bit_cell_kat():
    c = make_cell(2, 0, 0.5, 0.0, 4, 128)
    c[64:72] = 0x55  # fingerprints[0].words[0] = 0x5555555555555555 -> code 1
    y = O.gemv_tile(c, np.ones(128, np.float32), 4)
    assert y[0] == 16.0 and y[0] > 0 and not np.isnan(y[0])
    assert list(y[1:]) == [0.0, 0.0, 0.0]


# chpe_engine.zig:1840-1865 "polymorphic GEMV 4-bit cell"
def test_gemv_4bit_cell_kat():
    c = make_cell(4, 0, 0.25, 0.0, 4, 128)
    c[64:64 + 64] = 0x99  # nibble 9 -> +1
    y = O.gemv_tile(c, np.ones(128, np.float32), 4)
    assert y[0] == 32.0
    assert list(y[1:]) == [-256.0] * 3  # zero bytes decode to -8


# chpe_engine.zig:1867-1891 "polymorphic GEMV 8-bit cell"
def test_gemv_8bit_cell_kat():
    c = make_cell(8, 0, 0.1, 0.0, 4, 128)
    c[64:64 + 128] = 10
    y = O.gemv_tile(c, np.ones(128, np.float32), 4)
    assert y[0] == np.float32(1280.0) * np.float32(0.1)
    assert abs(y[0] - 128.0) < 1e-4
    assert list(y[1:]) == [0.0] * 3


# chpe_engine.zig:1893-1933: forwardDecode(151644, 0) over 8192 zero bytes.
@pytest.mark.parametrize("arch", [O.ARCH_3B, O.ARCH_9B, O.ARCH_72B])
def test_mock_archive_forward(arch):
    mock = np.zeros(8192, np.uint8)
    e = O.OracleEngine(mock, arch, 16)
    r = e.forward_decode(151644, 0)
    assert r.all_finite and not np.isnan(r.hidden_norm) and r.hidden_norm > 0
    # Synthetic fallbacks: logits 0.001*((v%13)-6) -> first v with v%13 == 12.
    assert r.argmax_token == 12
    assert r.max_logit == np.float32(0.001) * np.float32(6.0)
    assert r.token0_logit == np.float32(0.001) * np.float32(-6.0)
    f = e.facts()
    assert f["archive_valid"] == 0 and f["quant_bits"] == 2


# qwen_rope.zig:90-103 (pos 0 identity), :105-124 (norm), :149-162 (KAT at pos 1)
def test_rope_kats():
    vec = (np.arange(128, dtype=np.float32) + 1) * np.float32(0.1)
    assert np.array_equal(O.apply_rope(vec, 0, 1, 128), vec)
    r = O.apply_rope(vec, 1, 1, 128)
    assert abs(r[0] - -5.415531) < 1e-4
    assert abs(r[1] - -4.622832) < 1e-4
    assert abs(r[64] - 3.596112) < 1e-4
    assert abs(r[65] - 4.714808) < 1e-4
    n0, n1 = float(np.sum(vec * vec)), float(np.sum(r * r))
    assert abs(n1 - n0) / n0 < 1e-4


# qwen_rope.zig:126-147: multi-head == per-head
def test_rope_multihead_consistency():
    v = (np.arange(4 * 128, dtype=np.float32) + 1) * np.float32(0.01)
    multi = O.apply_rope(v, 2, 4, 128)
    for h in range(4):
        single = O.apply_rope(v[h * 128:(h + 1) * 128], 2, 1, 128)
        assert np.array_equal(single, multi[h * 128:(h + 1) * 128])


# qwen_mlp.zig:92-111: silu and SwiGLU
def test_silu_swiglu_kats():
    assert O.silu(0.0) == 0.0
    assert abs(O.silu(1.0) - 0.7310586) < 1e-5
    gate = [0.0, 1.0, -1.0, 2.0]
    up = [5.0, 2.0, 3.0, 0.5]
    out = [np.float32(O.silu(g)) * np.float32(u) for g, u in zip(gate, up)]
    assert out[0] == 0.0
    assert abs(out[1] - 1.462117) < 1e-4


# qwen_rmsnorm.zig:73-90
def test_rmsnorm_kat():
    y = O.rms_norm(np.ones(2048, np.float32), np.full(2048, 2.0, np.float32))
    assert np.all(np.abs(y - 2.0) < 1e-4)


# qwen_attention.zig:144-169 (seq 1 pass-through) and :171-190 (bounds at seq 2)
def test_attention_kats():
    H, KV, HD = 16, 2, 128
    k0 = np.full(KV * HD, 0.5, np.float32)
    v0 = (np.arange(KV * HD, dtype=np.float32) + 1) * np.float32(0.1)
    out = O.gqa_attention(np.ones(H * HD, np.float32), k0[None], v0[None], 0, H, KV, HD)
    for h in range(H):
        kv = h // (H // KV)
        assert np.array_equal(out[h * HD:(h + 1) * HD], v0[kv * HD:(kv + 1) * HD])
    kc = np.stack([np.full(KV * HD, 0.2, np.float32), np.full(KV * HD, 0.4, np.float32)])
    vc = np.stack([np.full(KV * HD, 1.0, np.float32), np.full(KV * HD, 3.0, np.float32)])
    out = O.gqa_attention(np.full(H * HD, 0.5, np.float32), kc, vc, 1, H, KV, HD)
    assert np.all((out >= 1.0) & (out <= 3.0))


# qwen3b_tensor_map.zig:21-538 (full table, parsed into the golden fixture)
def test_3b_cell_map_matches_reference_table():
    g = json.load(open(os.path.join(GOLDEN, "tensor_maps.json")))["qwen3b_cell"]
    names = ["input_norm", "q_proj", "q_bias", "k_proj", "k_bias", "v_proj", "v_bias",
             "o_proj", "post_norm", "gate_proj", "up_proj", "down_proj"]
    for l, ref in enumerate(g["layers"]):
        mine = dict(zip(names, O.map_3b_cell_layer(l)))
        assert mine == {k: ref[k] for k in names}, l
    assert g["consts"]["FINAL_NORM_RECORD"] == 94348


# qwen72b_tensor_map.zig:89-112
def test_72b_map_matches_reference_test():
    g = json.load(open(os.path.join(GOLDEN, "tensor_maps.json")))["qwen72b"]["checks"]
    names = ["input_norm", "q_proj", "q_bias", "k_proj", "k_bias", "v_proj", "v_bias",
             "o_proj", "post_norm", "gate_proj", "up_proj", "down_proj"]
    consts = {"RECORDS_PER_LAYER": 26789, "EMBED_TOKENS_RECORDS": 38016,
              "FINAL_NORM_RECORD": 2181136, "LM_HEAD_RECORD_START": 2181137,
              "TOTAL_RECORDS": 2219153}
    for chk in g:
        expr, val = chk["expr"], chk["value"]
        if expr.startswith("LAYERS["):
            l = int(expr[7:expr.index("]")])
            field = expr.split(".")[1]
            assert dict(zip(names, O.map_72b_layer(l)))[field] == val, expr
        else:
            assert consts[expr] == val, expr


# qwen35_tensor_map.zig:7-1015 through getLayerInfo (chpe_engine.zig:1108-1131)
def test_9b_map_matches_reference_table():
    g = json.load(open(os.path.join(GOLDEN, "tensor_maps.json")))["qwen35_9b"]
    e = O.OracleEngine(np.zeros(8192, np.uint8), O.ARCH_9B, 4)
    for l, m in enumerate(g["layers"]):
        li = e.layer_info(l)
        full = m["is_full_attn"]
        assert full == (l % 4 == 3)
        assert li["input_norm"] == m["input_norm_tile"]
        assert li["post_norm"] == m["post_norm_tile"]
        for t in ("gate", "up", "down"):
            assert li[f"{t}_proj"] == m[f"{t}_proj_tile"]
            assert li[f"{t}_tiles"] == m[f"{t}_proj_tiles"]
        if full:
            for t in ("q", "k", "v", "o"):
                assert li[f"{t}_proj"] == m[f"{t}_proj_tile"]
                assert li[f"{t}_tiles"] == m[f"{t}_proj_tiles"]
        else:  # Q8 reference-mode substitution
            assert li["q_proj"] == m["in_proj_qkv_tile"] and li["q_tiles"] == m["in_proj_qkv_tiles"]
            assert li["k_proj"] == m["in_proj_z_tile"] and li["k_tiles"] == m["in_proj_z_tiles"]
            assert li["v_proj"] == m["in_proj_a_tile"] and li["v_tiles"] == 1
            assert li["o_proj"] == m["out_proj_tile"] and li["o_tiles"] == m["out_proj_tiles"]
        assert li["q_bias"] == li["k_bias"] == li["v_bias"] == -1
    assert e.final_norm_index() == g["consts"]["FINAL_NORM_TILE"]


def _hdr(magic=0x57415243, version=1, header_bytes=4096, count=0, rec=20480, cell=17408,
         pre=3072, flags=0):
    return struct.pack("<IIQQQQQQQ", magic, version, header_bytes, count, count, rec, cell, pre,
                       flags)


# weight_archive.zig:1048-1078 corruption errors, :1080-1107 dense support
def test_archive_validation_errors():
    assert O.validate(bytearray(100))[0] == 6  # FileTooSmall
    buf = bytearray(4096)
    buf[:64] = _hdr(magic=0xDEADBEEF)
    assert O.validate(buf)[0] == 1  # InvalidMagic
    buf[:64] = _hdr(rec=20480 + 64)
    assert O.validate(buf)[0] == 3  # BadGeometry
    buf[:64] = _hdr(count=1)
    assert O.validate(buf)[0] == 4  # Truncated
    dense = bytearray(4096 + 17408)
    dense[:64] = _hdr(magic=0x45504843, count=1, rec=17408, cell=17408, pre=0)
    rc, h = O.validate(dense)
    assert rc == 0 and h.record_bytes == 17408 and h.prefetch_bytes == 0
    raw = bytearray(4096 + 16384)
    raw[:64] = _hdr(count=1, rec=16384, cell=16384, pre=0, flags=4)
    assert O.validate(raw)[0] == 0
    raw[:64] = _hdr(count=1, rec=16384, cell=17408, pre=0)
    assert O.validate(raw)[0] == 3
    buf[:64] = _hdr(version=2)
    assert O.validate(buf)[0] == 2
    buf[:64] = _hdr(header_bytes=8192)
    assert O.validate(buf)[0] == 10


def test_deltanet_step_matches_transformers_golden():
    """The Gated DeltaNet decode step (no reference function) against outputs
    of the installed transformers package's Qwen3.5 functions
    (tests/golden/gen_deltanet.py): three consecutive steps, outputs and the
    final conv history and recurrent state."""
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "deltanet_step.npz"))
    nk, nv, dk, dv, t0 = (int(g[k]) for k in ("nk", "nv", "dk", "dv", "t0"))
    hist = g["hist0"].copy()
    state = g["state0"].copy()
    for s in range(g["mixed"].shape[0]):
        out = O.deltanet_step(g["mixed"][s], g["z"][s], g["a"][s], g["b"][s], g["conv_w"], hist, t0 + s,
                              g["a_log"], g["dt_bias"], g["norm_w"], state, nk, nv, dk, dv, float(g["eps"]))
        ref = g["out"][s]
        assert np.max(np.abs(out - ref)) <= 2e-5 * max(1.0, float(np.max(np.abs(ref)))), s
    assert np.array_equal(hist, g["hist_end"])
    assert np.max(np.abs(state - g["state_end"])) <= 1e-5 * max(1.0, float(np.max(np.abs(g["state_end"]))))


def _defines(path: str) -> dict:
    import re
    out = {}
    for m in re.finditer(r"^#define\s+(\w+)\s+(\d+)u?\b", open(path).read(), re.M):
        out[m.group(1)] = int(m.group(2))
    return out


# geometry.zig:431-443 "cell is cache-line aligned and record is sector
# aligned" / "the 4.25 ratio", :483-499 "cell struct matches 17,408 bytes" /
# "record struct matches 20,480 bytes"; weight_archive.zig:897-910
# "WeightArchiveHeader layout" / "TileMetadata layout fits in semantic payload"
def test_archive_layout_constants_match_reference_tests():
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    prod = _defines(os.path.join(root, "chpe_qwen_engine_b200", "csrc", "chpe_maps.h"))
    orac = _defines(os.path.join(root, "oracle", "chpe_oracle.c"))
    cell, record, prefetch, header, tile = 17408, 20480, 3072, 4096, 16384
    payload_off, payload_bytes, cell_header = 16448, 960, 64
    assert cell % 64 == 0 and cell // 64 == 272 and record // 4096 == 5 and cell % 4096 != 0
    assert cell + prefetch == record and cell_header + tile + payload_bytes == cell
    assert cell_header + tile == payload_off
    for d, names in ((prod, ("CHPE_CELL_BYTES", "CHPE_RECORD_BYTES", "CHPE_PREFETCH_BYTES",
                             "CHPE_HEADER_BYTES", "CHPE_TILE_CODE_BYTES", "CHPE_PAYLOAD_OFF")),
                     (orac, ("CELL_BYTES", "RECORD_BYTES", "PREFETCH_LABEL_BYTES", "HEADER_BYTES",
                             "TILE_CODE_BYTES", "PAYLOAD_OFF"))):
        assert [d[n] for n in names] == [cell, record, prefetch, header, tile, payload_off], names
    assert prod["CHPE_CELL_HEADER_BYTES"] == cell_header
    assert prod["CHPE_PAYLOAD_FROM_CODES"] == tile
    # TileMetadata is 32 bytes at the payload start (quant_bits u8 @20,
    # custom_flags u64 @24); TileDims follows at @32 and the group scales at @48
    assert 32 <= payload_bytes and 48 + 2 * 256 <= payload_bytes
    c = make_cell(4, flags=1, scale=0.5, bias=0.25, rows=16, cols=2048)
    assert c[payload_off + 20] == 4
    assert struct.unpack("<Q", c[payload_off + 24:payload_off + 32].tobytes())[0] == 1
    assert struct.unpack("<ffII", c[payload_off + 32:payload_off + 48].tobytes()) == (0.5, 0.25, 16, 2048)


# weight_archive.zig:912-1007 "createArchive, mmap open, record slicing":
# three standard records with known patterns, flags 0x1234; the file is
# 4096 + 3 * 20480 = 65536 bytes, its header reads back, and each record's
# cell, code tile and TileMetadata sit at the offsets the engine reads
def test_created_archive_reads_back():
    import chpe_qwen_engine_b200 as chpe
    recs = np.zeros((3, 20480), np.uint8)
    for i in range(3):
        recs[i, :16] = 0xA0 + i                                          # prefetch seal
        recs[i, 3072:3080] = np.frombuffer(struct.pack("<Q", 0x100 + i), np.uint8)  # bytecode opcode
        for fp in range(32):                                             # fingerprint words
            o = 3072 + 64 + fp * 512
            recs[i, o:o + 4] = np.frombuffer(struct.pack("<I", 0xCAFE0000 + i), np.uint8)
        pl = 3072 + 16448                                                # TileMetadata
        recs[i, pl:pl + 32] = np.frombuffer(struct.pack("<IIQIB3xQ", i, 10 + i, 17408 * (i + 1), 4, 4, 0x55AA),
                                            np.uint8)
    hdr = np.zeros(4096, np.uint8)
    hdr[:64] = np.frombuffer(struct.pack("<IIQQQQQQQ", 0x57415243, 1, 4096, 3, 3, 20480, 17408, 3072, 0x1234),
                             np.uint8)
    a = np.concatenate([hdr, recs.reshape(-1)])
    assert a.size == 65536
    rc, h = O.validate(a)
    assert rc == 0 and chpe.validate_archive(a) == 0
    assert (h.record_count, h.record_bytes, h.cell_bytes, h.prefetch_bytes, h.flags) == (3, 20480, 17408, 3072,
                                                                                         0x1234)
    f = O.OracleEngine(a, O.ARCH_3B, 4).facts()
    assert (f["archive_valid"], f["record_count"], f["is_dense"], f["is_raw"], f["quant_bits"]) == (1, 3, 0, 0, 4)
    for i in range(3):
        rec = a[4096 + i * 20480:4096 + (i + 1) * 20480]
        cell = rec[3072:]
        assert rec[0] == 0xA0 + i
        assert struct.unpack("<Q", cell[:8].tobytes())[0] == 0x100 + i
        assert struct.unpack("<I", cell[64:68].tobytes())[0] == 0xCAFE0000 + i
        meta = struct.unpack("<IIQIB3xQ", cell[16448:16480].tobytes())
        assert meta == (i, 10 + i, 17408 * (i + 1), 4, 4, 0x55AA)
    # a file that holds fewer records than its header promises is refused
    assert O.validate(a[:65536 - 1])[0] == chpe.validate_archive(a[:65536 - 1]) != 0
