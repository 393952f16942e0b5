"""ctypes binding of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py.  It is the checker, never the thing measured or
shipped.  The oracle restates chpe-qwen-engine's decode path
(src/chpe_engine.zig); see oracle/chpe_oracle.h for its parity status.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

ARCH_3B, ARCH_9B, ARCH_72B = 0, 1, 2


class ForwardResult(C.Structure):
    _fields_ = [
        ("argmax_token", C.c_uint32),
        ("max_logit", C.c_float),
        ("token0_logit", C.c_float),
        ("elapsed_ns", C.c_uint64),
        ("hidden_norm", C.c_float),
        ("all_finite", C.c_int32),
    ]


class Header(C.Structure):
    _fields_ = [("magic", C.c_uint32), ("version", C.c_uint32)] + [
        (n, C.c_uint64)
        for n in ("header_bytes", "record_count", "tile_count", "record_bytes",
                  "cell_bytes", "prefetch_bytes", "flags")
    ]


class LayerInfo(C.Structure):
    _fields_ = [(n, C.c_int64) for n in (
        "input_norm", "q_proj", "q_tiles", "q_bias", "k_proj", "k_tiles", "k_bias",
        "v_proj", "v_tiles", "v_bias", "o_proj", "o_tiles", "post_norm", "gate_proj",
        "gate_tiles", "up_proj", "up_tiles", "down_proj", "down_tiles")]


def build() -> str:
    """Compile liboracle.so with the committed Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        P, F, S, I, U32, I64 = C.c_void_p, C.c_float, C.c_size_t, C.c_int, C.c_uint32, C.c_int64
        FP = C.POINTER(C.c_float)
        L.oracle_deltanet_step.argtypes = [FP, FP, FP, FP, FP, FP, U32, FP, FP, FP, FP, FP,
                                           U32, U32, U32, U32, F]
        L.oracle_deltanet_step.restype = None
        L.oracle_validate.argtypes = [P, S, C.POINTER(Header)]
        L.oracle_validate.restype = I
        L.oracle_engine_new.argtypes = [P, S, I, S]
        L.oracle_engine_new.restype = P
        L.oracle_engine_free.argtypes = [P]
        L.oracle_set_threads.argtypes = [P, I]
        L.oracle_set_kv_fp16.argtypes = [P, I]
        L.oracle_forward_decode.argtypes = [P, U32, S, C.POINTER(ForwardResult)]
        L.oracle_kv_load.argtypes = [P, S, S, S, FP, FP]
        L.oracle_kv_load.restype = I
        L.oracle_logits.argtypes = [P]
        L.oracle_logits.restype = FP
        L.oracle_hidden.argtypes = [P]
        L.oracle_hidden.restype = FP
        L.oracle_vocab.argtypes = [P]
        L.oracle_vocab.restype = S
        L.oracle_hidden_dim.argtypes = [P]
        L.oracle_hidden_dim.restype = S
        L.oracle_engine_facts.argtypes = [P, C.POINTER(C.c_int64)]
        L.oracle_layer_info.argtypes = [P, S, C.POINTER(LayerInfo)]
        L.oracle_final_norm_index.argtypes = [P]
        L.oracle_final_norm_index.restype = I64
        L.oracle_gemv_linear.argtypes = [P, S, S, FP, S, FP, S, S, I, I64]
        L.oracle_unpack_norm.argtypes = [P, S, FP, S]
        L.oracle_unpack_bias.argtypes = [P, S, FP, S]
        L.oracle_unpack_embed_row.argtypes = [P, U32, FP]
        L.oracle_compute_lm_head.argtypes = [P, FP, FP]
        L.oracle_gemv_tile_polymorphic.argtypes = [P, FP, S, FP, S, S, I]
        L.oracle_gemv_cell_flat.argtypes = [P, S, S, S, S, FP, FP]
        L.oracle_dequant_cell.argtypes = [P, I, FP, S]
        L.oracle_dequant_cell.restype = S
        L.oracle_unpack_embed_row_cell.argtypes = [P, S, FP, S]
        L.oracle_silu.argtypes = [F]
        L.oracle_silu.restype = F
        L.oracle_rms_norm.argtypes = [FP, FP, FP, S, F]
        L.oracle_apply_rope.argtypes = [FP, S, S, S, F]
        L.oracle_gqa_attention.argtypes = [FP, FP, FP, S, S, S, S, FP]
        L.oracle_convert_header.argtypes = [P, I, P]
        L.oracle_convert_record.argtypes = [P, I, S, P]
        L.oracle_convert_record.restype = S
        L.oracle_map_3b_cell_layer.argtypes = [S, C.POINTER(C.c_int64)]
        L.oracle_map_72b_layer.argtypes = [S, C.POINTER(C.c_int64)]
        _lib = L
    return _lib


def fptr(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.POINTER(C.c_float))


def bptr(a) -> int:
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    return C.addressof(C.c_char.from_buffer(a))


def validate(buf) -> tuple[int, Header]:
    h = Header()
    arr = np.frombuffer(buf, dtype=np.uint8)
    rc = lib().oracle_validate(arr.ctypes.data if arr.size else None, arr.size, C.byref(h))
    return rc, h


class OracleEngine:
    """Mirror of CHPEEngine (chpe_engine.zig:820) over borrowed archive bytes."""

    def __init__(self, archive: np.ndarray, arch: int, max_seq_len: int = 2048, threads: int = 1):
        self._arc = archive  # keep the bytes alive: the engine borrows them
        L = lib()
        self.h = L.oracle_engine_new(archive.ctypes.data, archive.size, arch, max_seq_len)
        if not self.h:
            raise ValueError("bad arch")
        L.oracle_set_threads(self.h, threads)
        self.vocab = L.oracle_vocab(self.h)
        self.hidden_dim = L.oracle_hidden_dim(self.h)

    def close(self):
        if self.h:
            lib().oracle_engine_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_threads(self, n: int):
        lib().oracle_set_threads(self.h, n)

    def set_kv_fp16(self, on: bool = True):
        """Test option: round cached K/V rows to FP16 (the reference keeps f32)."""
        lib().oracle_set_kv_fp16(self.h, int(on))

    def forward_decode(self, token: int, pos: int) -> ForwardResult:
        r = ForwardResult()
        lib().oracle_forward_decode(self.h, token, pos, C.byref(r))
        return r

    def kv_load(self, layer: int, pos0: int, k: np.ndarray, v: np.ndarray):
        """K/V rows [n][kv_heads*head_dim] at positions pos0.. of one layer."""
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        if lib().oracle_kv_load(self.h, layer, pos0, k.shape[0], fptr(k), fptr(v)) != 0:
            raise ValueError("KV rows do not fit the cache")

    def logits(self) -> np.ndarray:
        p = lib().oracle_logits(self.h)
        return np.ctypeslib.as_array(p, shape=(self.vocab,)).copy()

    def hidden(self) -> np.ndarray:
        p = lib().oracle_hidden(self.h)
        return np.ctypeslib.as_array(p, shape=(self.hidden_dim,)).copy()

    def facts(self) -> dict:
        o = (C.c_int64 * 7)()
        lib().oracle_engine_facts(self.h, o)
        keys = ("is_raw", "is_raw_fp16", "is_dense", "quant_bits", "weights_per_tile",
                "archive_valid", "record_count")
        return dict(zip(keys, list(o)))

    def layer_info(self, l: int) -> dict:
        li = LayerInfo()
        lib().oracle_layer_info(self.h, l, C.byref(li))
        return {n: getattr(li, n) for n, _ in LayerInfo._fields_}

    def final_norm_index(self) -> int:
        return lib().oracle_final_norm_index(self.h)

    def gemv_linear(self, tile_start, num_tiles, x, r_total, c_total, accumulate=False,
                    bias_tile=-1, y=None):
        x = np.ascontiguousarray(x, dtype=np.float32)
        if y is None:
            y = np.zeros(r_total, dtype=np.float32)
        lib().oracle_gemv_linear(self.h, tile_start, num_tiles, fptr(x), x.size, fptr(y),
                                 r_total, c_total, int(accumulate), bias_tile)
        return y

    def unpack_norm(self, tile, n):
        o = np.empty(n, np.float32)
        lib().oracle_unpack_norm(self.h, tile, fptr(o), n)
        return o

    def unpack_bias(self, tile, n):
        o = np.empty(n, np.float32)
        lib().oracle_unpack_bias(self.h, tile, fptr(o), n)
        return o

    def embed(self, token, out=None):
        if out is None:
            out = np.zeros(self.hidden_dim, np.float32)
        lib().oracle_unpack_embed_row(self.h, token, fptr(out))
        return out

    def lm_head(self, normed):
        normed = np.ascontiguousarray(normed, dtype=np.float32)
        out = np.empty(self.vocab, np.float32)
        lib().oracle_compute_lm_head(self.h, fptr(normed), fptr(out))
        return out


def silu(z: float) -> float:
    return lib().oracle_silu(z)


def rms_norm(x, gamma, eps=1e-6):
    x = np.ascontiguousarray(x, np.float32)
    g = np.ascontiguousarray(gamma, np.float32)
    y = np.empty_like(x)
    lib().oracle_rms_norm(fptr(x), fptr(g), fptr(y), x.size, eps)
    return y


def apply_rope(vec, pos, num_heads, head_dim, theta=1e6):
    v = np.array(vec, dtype=np.float32)
    lib().oracle_apply_rope(fptr(v), pos, num_heads, head_dim, theta)
    return v


def gqa_attention(q, k_cache, v_cache, pos, num_heads, num_kv_heads, head_dim):
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k_cache, np.float32)
    v = np.ascontiguousarray(v_cache, np.float32)
    out = np.empty(num_heads * head_dim, np.float32)
    lib().oracle_gqa_attention(fptr(q), fptr(k), fptr(v), pos, num_heads, num_kv_heads,
                               head_dim, fptr(out))
    return out


def gemv_tile(cell: np.ndarray, x, y_len, row_base=0, accumulate=False, y=None):
    x = np.ascontiguousarray(x, np.float32)
    if y is None:
        y = np.zeros(y_len, np.float32)
    lib().oracle_gemv_tile_polymorphic(cell.ctypes.data, fptr(x), x.size, fptr(y), y.size,
                                       row_base, int(accumulate))
    return y


def gemv_cell_flat(cell: np.ndarray, t, r_total, c_total, x, y=None, wpt=32768):
    x = np.ascontiguousarray(x, np.float32)
    if y is None:
        y = np.zeros(r_total, np.float32)
    lib().oracle_gemv_cell_flat(cell.ctypes.data, t, wpt, r_total, c_total, fptr(x), fptr(y))
    return y


def dequant_cell(cell: np.ndarray, flat: bool) -> np.ndarray:
    out = np.empty(32768, np.float32)
    n = lib().oracle_dequant_cell(cell.ctypes.data, int(flat), fptr(out), out.size)
    return out[:n].copy()


def embed_row_cell(cell: np.ndarray, row, d, out=None):
    if out is None:
        out = np.zeros(d, np.float32)
    lib().oracle_unpack_embed_row_cell(cell.ctypes.data, row, fptr(out), d)
    return out


def map_3b_cell_layer(l):
    o = (C.c_int64 * 12)()
    lib().oracle_map_3b_cell_layer(l, o)
    return list(o)


def map_72b_layer(l):
    o = (C.c_int64 * 12)()
    lib().oracle_map_72b_layer(l, o)
    return list(o)


def deltanet_step(mixed, z, a, b, conv_w, conv_hist, t, a_log, dt_bias, norm_w, state,
                  nk, nv, dk, dv, eps=1e-6):
    """One Gated DeltaNet decode step (deltanet_oracle.c); conv_hist [4][conv_dim]
    and state [nv][dv][dk] are updated in place.  Returns the output [nv*dv]."""
    f = lambda x: np.ascontiguousarray(x, np.float32)
    for arr in (conv_hist, state):
        assert arr.dtype == np.float32 and arr.flags["C_CONTIGUOUS"]
    ins = [f(mixed), f(z), f(a), f(b), f(conv_w)]
    prm = [f(a_log), f(dt_bias), f(norm_w)]
    out = np.zeros(nv * dv, np.float32)
    lib().oracle_deltanet_step(fptr(ins[0]), fptr(ins[1]), fptr(ins[2]), fptr(ins[3]), fptr(ins[4]),
                               fptr(conv_hist), t, fptr(prm[0]), fptr(prm[1]), fptr(prm[2]),
                               fptr(state), fptr(out), nk, nv, dk, dv, eps)
    return out


def convert_header(src: np.ndarray, mode: int) -> np.ndarray:
    out = np.zeros(4096, np.uint8)
    lib().oracle_convert_header(src.ctypes.data, mode, out.ctypes.data)
    return out


def convert_record(src: np.ndarray, mode: int, i: int) -> np.ndarray:
    out = np.zeros(17408, np.uint8)
    n = lib().oracle_convert_record(src.ctypes.data, mode, i, out.ctypes.data)
    return out[:n].copy()
