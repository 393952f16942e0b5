"""chpe_qwen_engine_b200 -- B200-native decode loop of chpe-qwen-engine.

The product is libchpe.so (CUDA sm_100a + C++), whose extern "C" surface is
declared in include/chpe.h and mirrors src/chpe_c_api.zig.  This module is
the ctypes binding a Python caller of the reference would write (the
reference's C ABI is documented for ctypes callers, chpe_c_api.zig:1-5), plus
an object wrapper shaped like CHPEEngine (init / forwardDecode / logits).

There is no CPU fallback: importing works without a GPU, but every compute
call goes through libchpe.so and raises if the library or the device is
missing.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

PKG = os.path.dirname(os.path.abspath(__file__))
LIBCHPE_PATH = os.path.join(PKG, "libchpe.so")
LIBSYNTH_PATH = os.path.join(PKG, "libchpe_synth.so")

ARCH_BY_PATH, ARCH_3B, ARCH_9B, ARCH_72B = -1, 0, 1, 2
ROLE_QKV, ROLE_ATTN, ROLE_O, ROLE_GATEUP, ROLE_DOWN, ROLE_LMHEAD, ROLE_EMBED = 1, 2, 3, 4, 5, 6, 7
ARCH_NAMES = {ARCH_3B: "Qwen2.5-3B", ARCH_9B: "Qwen3.5-9B", ARCH_72B: "Qwen2.5-72B"}

# Symbols of include/chpe.h: (name, restype, argtypes)
_P, _S, _I, _U32, _U64, _I64, _F = (C.c_void_p, C.c_size_t, C.c_int, C.c_uint32, C.c_uint64,
                                    C.c_int64, C.c_float)
_FP = C.POINTER(C.c_float)
_U32P = C.POINTER(C.c_uint32)
SYMBOLS = [
    ("chpe_init", _P, [C.c_char_p]),
    ("chpe_forward_tokens", _I, [_P, _U32P, _S, _FP]),
    ("chpe_get_last_logits", _S, [_P, _FP, _S]),
    ("chpe_get_vocab_size", _S, [_P]),
    ("chpe_get_hidden_dim", _S, [_P]),
    ("chpe_get_num_layers", _S, [_P]),
    ("chpe_get_last_elapsed_ns", _U64, [_P]),
    ("chpe_get_last_argmax", _U32, [_P]),
    ("chpe_get_last_max_logit", _F, [_P]),
    ("chpe_get_last_token0_logit", _F, [_P]),
    ("chpe_get_last_hidden_norm", _F, [_P]),
    ("chpe_free", None, [_P]),
    ("chpe_init_ex", _P, [C.c_char_p, _I, _U32, _I]),
    ("chpe_init_bytes", _P, [_P, _U64, _I, _U32, _I]),
    ("chpe_validate_archive", _I, [_P, _U64]),
    ("chpe_convert_archive", _I, [C.c_char_p, C.c_char_p, _I, _I]),
    ("chpe_decode_step", _I, [_P, _U32, _U32, _FP]),
    ("chpe_generate", _I, [_P, _U32P, _S, _S, _U32P]),
    ("chpe_speculative_generate", _I, [_P, _U32P, _S, _S, _U32, _U32, _U32P, C.POINTER(C.c_uint64)]),
    ("chpe_bench_greedy", _I, [_P, _S, _FP]),
    ("chpe_bench_host", _I, [_P, _U32P, _S, _FP, C.POINTER(C.c_double)]),
    ("chpe_bench_kernel", _I, [_P, _I, _I, _FP, C.POINTER(C.c_double), C.POINTER(C.c_int)]),
    ("chpe_role_kernel_name", C.c_char_p, [_P, _I]),
    ("chpe_bench_kernel_cold", _I, [_P, _I, _I, _FP, C.POINTER(C.c_double), C.POINTER(C.c_int)]),
    ("chpe_init_tp", _P, [C.c_char_p, _I, C.c_uint32, _I, _I, _I]),
    ("chpe_init_tp_bytes", _P, [_P, C.c_uint64, _I, C.c_uint32, _I, _I, _I]),
    ("chpe_tp_export_handle", _I, [_P, C.c_char_p]),
    ("chpe_tp_connect", _I, [_P, C.c_char_p, _I]),
    ("chpe_tp_slice", _I, [_I, _I, _I, _U32P]),
    ("chpe_tp_tile_runs", _I64, [_I, _I, _U64, _U64, _I, _I, C.POINTER(C.c_uint64), _S]),
    ("chpe_step_weight_bytes", C.c_double, [_P]),
    ("chpe_profile_step", _I, [_P, _FP, C.POINTER(C.c_int), _I]),
    ("chpe_verify", _I, [_P, _U32P, C.c_size_t, C.c_uint32, _FP, _U32P]),
    ("chpe_last_verify_batched", _I, [_P]),
    ("chpe_profile_verify", _I, [_P, C.c_size_t, _U32, _FP, C.POINTER(C.c_double), _I]),
    ("chpe_verify_batched_unavailable", C.c_char_p, [_P, _I]),
    ("chpe_deltanet_step", _I, [_P, _P, _P, _P, _P, _P, C.c_uint32, _P, _P, _P, _P, _P,
                                C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_float, _P]),
    ("chpe_get_last_all_finite", _I, [_P]),
    ("chpe_kernels_per_step", _I, [_P]),
    ("chpe_get_position", _U32, [_P]),
    ("chpe_device_archive_bytes", _U64, [_P]),
    ("chpe_last_error", C.c_char_p, [_P]),
    ("chpe_kv_page_size", _U32, []),
    ("chpe_kv_load", _I, [_P, _U32, _U32, _U32, _FP, _FP]),
    ("chpe_kv_set_page_order", _I, [_P, _U32P, _U32]),
    ("chpe_kv_page_table", _I, [_P, _U32P, _U32, _U32P]),
    ("chpe_probe_gemv_linear", _I, [_P, _U64, _U64, _FP, _U64, _FP, _U64, _U64, _I, _I64]),
    ("chpe_attention_decode_noalloc", _I, [_P, _P, _P, _P, _P, _P, _U32, _U32, _U32, _U32, _U32, _F, _P]),
    ("chpe_probe_attention", _I, [_P, _U32, _U32, _FP, _FP, _FP, _FP]),
    ("chpe_probe_embed", _I, [_P, _U32, _FP]),
    ("chpe_probe_wait_timeout", _I, [_P, _U32]),
    ("chpe_probe_tc_i8", _I, [_P, _P, _I, _P, _I]),
    ("chpe_probe_bgemm", _I, [_P, _U64, _U64, _FP, _I, _FP, _U64, _U64, _I]),
    ("chpe_probe_dequant_cell", _I, [_P, _U64, _I, _FP, _U64, C.POINTER(C.c_uint64)]),
]

_lib = None
_synth = None


def lib() -> C.CDLL:
    """Load libchpe.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIBCHPE_PATH):
            raise RuntimeError(f"{LIBCHPE_PATH} is missing: run python -m chpe_qwen_engine_b200.build")
        L = C.CDLL(LIBCHPE_PATH)
        for name, res, args in SYMBOLS:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def synth_lib() -> C.CDLL:
    global _synth
    if _synth is None:
        if not os.path.exists(LIBSYNTH_PATH):
            raise RuntimeError(f"{LIBSYNTH_PATH} is missing: run python -m chpe_qwen_engine_b200.build")
        L = C.CDLL(LIBSYNTH_PATH)
        L.chpe_synth_bytes.restype = C.c_uint64
        L.chpe_synth_bytes.argtypes = [C.c_int, C.c_uint32]
        L.chpe_synth_fill.restype = C.c_int
        L.chpe_synth_fill.argtypes = [C.c_int, C.c_uint32, C.c_uint64, C.c_void_p, C.c_uint64, C.c_int]
        L.chpe_synth_write.restype = C.c_int
        L.chpe_synth_write.argtypes = [C.c_int, C.c_uint32, C.c_uint64, C.c_char_p, C.c_int]
        _synth = L
    return _synth


# Synthetic archive configs (csrc/chpe_synth.h)
SYNTH_3B_FP16_RAW, SYNTH_3B_BF16_RAW, SYNTH_3B_W4, SYNTH_3B_W2 = 0, 1, 2, 3
SYNTH_9B_W4, SYNTH_72B_W4, SYNTH_72B_FP16_RAW, SYNTH_9B_I8_RAW = 4, 5, 6, 7
SYNTH_STANDARD, SYNTH_OUTLIERS, SYNTH_NONGROUP, SYNTH_BIAS, SYNTH_MIXED = 0x1, 0x2, 0x4, 0x8, 0x10
SYNTH_ARCH = {0: ARCH_3B, 1: ARCH_3B, 2: ARCH_3B, 3: ARCH_3B, 4: ARCH_9B, 5: ARCH_72B,
              6: ARCH_72B, 7: ARCH_9B}


def synth_archive(config: int, flags: int = 0, seed: int = 0, threads: int | None = None) -> np.ndarray:
    """A seeded synthetic .chpe archive as a uint8 array."""
    L = synth_lib()
    n = L.chpe_synth_bytes(config, flags)
    if n == 0:
        raise ValueError(f"unknown synthetic config {config}")
    buf = np.empty(n, dtype=np.uint8)
    rc = L.chpe_synth_fill(config, flags, seed, buf.ctypes.data, n, threads or os.cpu_count() or 8)
    if rc != 0:
        raise RuntimeError(f"chpe_synth_fill failed: {rc}")
    return buf


def synth_write(path: str, config: int, flags: int = 0, seed: int = 0, threads: int | None = None):
    rc = synth_lib().chpe_synth_write(config, flags, seed, path.encode(), threads or os.cpu_count() or 8)
    if rc != 0:
        raise RuntimeError(f"chpe_synth_write failed: {rc}")


@dataclass
class ForwardResult:
    """chpe_engine.zig:803-810"""
    argmax_token: int
    max_logit: float
    token0_logit: float
    elapsed_ns: int
    hidden_norm: float
    all_finite: bool


def _fp(a: np.ndarray):
    return a.ctypes.data_as(_FP)


def _u32p(a: np.ndarray):
    return a.ctypes.data_as(_U32P)


class ChpeError(RuntimeError):
    pass


def tp_slice(arch: int, rank: int, world: int) -> dict:
    """Rows one tensor-parallel rank owns (chpe_tp_slice); no GPU needed."""
    out = np.zeros(10, np.uint32)
    if lib().chpe_tp_slice(arch, rank, world, _u32p(out)) != 0:
        raise ValueError(f"architecture {arch} does not split over {world} ranks")
    keys = ("hq", "h0", "kv0", "kvl", "dl", "d0", "fl", "f0", "vl", "v0")
    return {k: int(v) for k, v in zip(keys, out)}


def tp_tile_runs(arch: int, is_raw: bool, wpt: int, record_count: int, rank: int,
                 world: int) -> list[tuple[int, int]]:
    """Archive tiles one tensor-parallel rank uploads (chpe_tp_tile_runs), as
    disjoint ascending runs [lo, hi); no GPU needed."""
    n = lib().chpe_tp_tile_runs(arch, int(is_raw), wpt, record_count, rank, world, None, 0)
    if n < 0:
        raise ValueError(f"architecture {arch} does not split over {world} ranks")
    out = (C.c_uint64 * (2 * n))()
    lib().chpe_tp_tile_runs(arch, int(is_raw), wpt, record_count, rank, world, out, n)
    return [(int(out[2 * i]), int(out[2 * i + 1])) for i in range(n)]


class Engine:
    """CHPEEngine over libchpe.so: one context = one device stream and KV cache."""

    def __init__(self, ctx: int, keepalive=None):
        if not ctx:
            raise ChpeError(lib().chpe_last_error(None).decode() or "chpe init failed")
        self.ctx = ctx
        self._keep = keepalive
        L = lib()
        self.vocab = L.chpe_get_vocab_size(ctx)
        self.hidden_dim = L.chpe_get_hidden_dim(ctx)
        self.num_layers = L.chpe_get_num_layers(ctx)

    @classmethod
    def from_path(cls, path: str, arch: int = ARCH_BY_PATH, max_seq_len: int = 2048, device: int = 0):
        return cls(lib().chpe_init_ex(path.encode(), arch, max_seq_len, device))

    @classmethod
    def from_bytes(cls, archive: np.ndarray, arch: int, max_seq_len: int = 2048, device: int = 0):
        """CHPEEngine.init over caller-held bytes (kept alive by the engine)."""
        a = np.ascontiguousarray(archive, dtype=np.uint8)
        return cls(lib().chpe_init_bytes(a.ctypes.data, a.size, arch, max_seq_len, device), keepalive=a)

    @classmethod
    def tensor_parallel(cls, archive, arch: int, rank: int, world: int, max_seq_len: int = 2048,
                        device: int | None = None, all_gather=None):
        """Rank `rank` of a tensor-parallel engine over `world` GPUs of this node
        (one process per GPU).  `archive` is a path (every rank maps the same
        file) or a uint8 array.  `all_gather(bytes) -> list[bytes]` exchanges the
        64-byte CUDA IPC handles between ranks in rank order; by default it is
        torch.distributed.all_gather_object on the default process group."""
        L = lib()
        dev = rank if device is None else device
        if isinstance(archive, (str, bytes, os.PathLike)):
            ctx = L.chpe_init_tp(os.fsencode(archive), arch, max_seq_len, dev, rank, world)
            keep = None
        else:
            keep = np.ascontiguousarray(archive, dtype=np.uint8)
            ctx = L.chpe_init_tp_bytes(keep.ctypes.data, keep.size, arch, max_seq_len, dev, rank, world)
        eng = cls(ctx, keepalive=keep)
        h = C.create_string_buffer(64)
        if L.chpe_tp_export_handle(eng.ctx, h) != 0:
            raise ChpeError(eng._err())
        if all_gather is None:
            import torch.distributed as dist

            def all_gather(b):
                out = [None] * world
                dist.all_gather_object(out, b)
                return out
        handles = all_gather(h.raw)
        if len(handles) != world or any(len(x) != 64 for x in handles):
            raise ChpeError("tensor parallel: bad handle exchange")
        if L.chpe_tp_connect(eng.ctx, b"".join(handles), world) != 0:
            raise ChpeError(eng._err())
        return eng

    def close(self):
        if getattr(self, "ctx", None):
            lib().chpe_free(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _err(self) -> str:
        return lib().chpe_last_error(self.ctx).decode()

    def forward_tokens(self, tokens, out_logits: np.ndarray | None = None) -> int:
        """chpe_forward_tokens: positions 0..n-1 (fresh sequence)."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        r = lib().chpe_forward_tokens(self.ctx, _u32p(t), t.size, _fp(out_logits) if out_logits is not None else None)
        if r < 0:
            raise ChpeError(self._err() or "chpe_forward_tokens failed")
        return r

    def forward_decode(self, token: int, pos: int) -> ForwardResult:
        """forwardDecode(token, pos) continuing the current sequence."""
        r = lib().chpe_decode_step(self.ctx, token, pos, None)
        if r < 0:
            raise ChpeError(self._err() or "chpe_decode_step failed")
        return self.last_result()

    def last_result(self) -> ForwardResult:
        L = lib()
        return ForwardResult(L.chpe_get_last_argmax(self.ctx), L.chpe_get_last_max_logit(self.ctx),
                             L.chpe_get_last_token0_logit(self.ctx), L.chpe_get_last_elapsed_ns(self.ctx),
                             L.chpe_get_last_hidden_norm(self.ctx), bool(L.chpe_get_last_all_finite(self.ctx)))

    def logits(self) -> np.ndarray:
        out = np.empty(self.vocab, np.float32)
        n = lib().chpe_get_last_logits(self.ctx, _fp(out), out.size)
        assert n == self.vocab
        return out

    def verify(self, tokens, pos: int) -> tuple[np.ndarray, np.ndarray]:
        """chpe_verify: (logits [m, vocab], argmax [m]) of m candidates at pos.."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        lg = np.empty((t.size, self.vocab), np.float32)
        am = np.empty(t.size, np.uint32)
        if lib().chpe_verify(self.ctx, _u32p(t), t.size, pos, _fp(lg), _u32p(am)) != 0:
            raise ChpeError(self._err() or "chpe_verify failed")
        return lg, am

    def profile_verify(self, m: int, pos: int) -> tuple[np.ndarray, np.ndarray]:
        """(milliseconds, algorithmic bytes) per role of the batched step."""
        ms = np.zeros(8, np.float32)
        by = np.zeros(8, np.float64)
        if lib().chpe_profile_verify(self.ctx, m, pos, _fp(ms), by.ctypes.data_as(C.POINTER(C.c_double)), 8) < 0:
            raise ChpeError(self._err())
        return ms, by

    def last_verify_batched(self) -> bool:
        return bool(lib().chpe_last_verify_batched(self.ctx))

    def verify_batched_unavailable(self, m: int) -> str:
        return (lib().chpe_verify_batched_unavailable(self.ctx, m) or b"").decode()

    def generate(self, prompt, n_gen: int) -> np.ndarray:
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = np.zeros(max(n_gen, 1), np.uint32)
        if lib().chpe_generate(self.ctx, _u32p(p), p.size, n_gen, _u32p(out)) != 0:
            raise ChpeError(self._err() or "chpe_generate failed")
        return out[:n_gen]

    def speculative_generate(self, prompt, n_gen: int, draft_len: int = 4,
                             ngram: int = 3) -> tuple[np.ndarray, dict]:
        """chpe_speculative_generate: (tokens, {rounds, proposed, accepted})."""
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = np.zeros(max(n_gen, 1), np.uint32)
        st = (C.c_uint64 * 3)()
        if lib().chpe_speculative_generate(self.ctx, _u32p(p), p.size, n_gen, draft_len, ngram,
                                           _u32p(out), st) != 0:
            raise ChpeError(self._err() or "chpe_speculative_generate failed")
        return out[:n_gen], {"rounds": st[0], "proposed": st[1], "accepted": st[2]}

    def bench_greedy(self, n_steps: int) -> float:
        ms = C.c_float()
        if lib().chpe_bench_greedy(self.ctx, n_steps, C.byref(ms)) != 0:
            raise ChpeError(self._err())
        return ms.value

    def bench_host(self, tokens) -> tuple[float, np.ndarray]:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        logits = np.empty(self.vocab, np.float32)
        ms = C.c_double()
        if lib().chpe_bench_host(self.ctx, _u32p(t), t.size, _fp(logits), C.byref(ms)) != 0:
            raise ChpeError(self._err())
        return ms.value, logits

    def bench_kernel(self, role: int, rounds: int = 3) -> tuple[float, float, int]:
        """(avg ms per launch, algorithmic bytes per launch, launches)."""
        ms, b, n = C.c_float(), C.c_double(), C.c_int()
        if lib().chpe_bench_kernel(self.ctx, role, rounds, C.byref(ms), C.byref(b), C.byref(n)) != 0:
            raise ChpeError(self._err())
        return ms.value, b.value, n.value

    def bench_kernel_cold(self, role: int, rounds: int = 2) -> tuple[float, float, int]:
        """bench_kernel with an L2 flush before every launch."""
        ms, b, n = C.c_float(), C.c_double(), C.c_int()
        if lib().chpe_bench_kernel_cold(self.ctx, role, rounds, C.byref(ms), C.byref(b), C.byref(n)) != 0:
            raise ChpeError(self._err())
        return ms.value, b.value, n.value

    def op_kernel_name(self, role: int) -> str:
        """Kernel that runs the first op of `role`."""
        return (lib().chpe_role_kernel_name(self.ctx, role) or b"").decode()

    def profile_step(self) -> tuple[np.ndarray, np.ndarray]:
        """One greedy step op by op: (per-op ms, per-op role)."""
        cap = 4096
        ms = np.zeros(cap, np.float32)
        roles = np.zeros(cap, np.int32)
        n = lib().chpe_profile_step(self.ctx, _fp(ms), roles.ctypes.data_as(C.POINTER(C.c_int)), cap)
        if n < 0:
            raise ChpeError(self._err())
        n = min(n, cap)
        return ms[:n], roles[:n]

    def step_weight_bytes(self) -> float:
        """Algorithmic weight bytes one step streams on this rank."""
        return lib().chpe_step_weight_bytes(self.ctx)

    # -- paged KV cache -------------------------------------------------------
    def kv_load(self, layer: int, pos0: int, k, v):
        """chpe_kv_load: K (rotated) / V rows [n][kv_heads*head_dim] at pos0.."""
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        n = k.shape[0] if k.ndim > 1 else 1
        if lib().chpe_kv_load(self.ctx, layer, pos0, n, _fp(k), _fp(v)) != 0:
            raise ChpeError(self._err())

    def kv_set_page_order(self, order):
        o = np.ascontiguousarray(order, np.uint32)
        if lib().chpe_kv_set_page_order(self.ctx, _u32p(o), o.size) != 0:
            raise ChpeError(self._err())

    def kv_page_table(self) -> tuple[np.ndarray, int]:
        """(physical page of each mapped logical page, pages in the pool)."""
        npg = C.c_uint32()
        n = lib().chpe_kv_page_table(self.ctx, None, 0, C.byref(npg))
        out = np.zeros(max(n, 1), np.uint32)
        n = lib().chpe_kv_page_table(self.ctx, _u32p(out), out.size, C.byref(npg))
        if n < 0:
            raise ChpeError(self._err())
        return out[:n].copy(), int(npg.value)

    def kernels_per_step(self) -> int:
        return lib().chpe_kernels_per_step(self.ctx)

    def position(self) -> int:
        return lib().chpe_get_position(self.ctx)

    def device_archive_bytes(self) -> int:
        return lib().chpe_device_archive_bytes(self.ctx)

    # -- probes used by the parity suite ------------------------------------
    def probe_gemv_linear(self, tile_start, num_tiles, x, r_total, c_total, accumulate=False,
                          bias_tile=-1, y=None) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        y = np.zeros(r_total, np.float32) if y is None else np.ascontiguousarray(y, np.float32).copy()
        if lib().chpe_probe_gemv_linear(self.ctx, tile_start, num_tiles, _fp(x), x.size, _fp(y), r_total,
                                        c_total, int(accumulate), bias_tile) != 0:
            raise ChpeError(self._err())
        return y

    def probe_bgemm(self, tile_start, num_tiles, x, r_total, c_total, accumulate=False, y=None):
        """chpe_probe_bgemm: x [nt][c_total] -> y [nt][r_total] on the tensor cores."""
        x = np.ascontiguousarray(x, np.float32)
        nt = x.shape[0]
        y = np.zeros((nt, r_total), np.float32) if y is None else np.ascontiguousarray(y, np.float32).copy()
        if lib().chpe_probe_bgemm(self.ctx, tile_start, num_tiles, _fp(x), nt, _fp(y), r_total, c_total,
                                  int(accumulate)) != 0:
            raise ChpeError(self._err())
        return y

    def probe_attention(self, layer: int, pos: int, q, k, v) -> np.ndarray:
        q = np.ascontiguousarray(q, np.float32)
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        out = np.empty(q.size, np.float32)
        if lib().chpe_probe_attention(self.ctx, layer, pos, _fp(q), _fp(k), _fp(v), _fp(out)) != 0:
            raise ChpeError(self._err())
        return out

    def probe_embed(self, token: int, init: np.ndarray | None = None) -> np.ndarray:
        out = np.zeros(self.hidden_dim, np.float32) if init is None else np.array(init, np.float32)
        if lib().chpe_probe_embed(self.ctx, token, _fp(out)) != 0:
            raise ChpeError(self._err())
        return out

    def probe_dequant_cell(self, tile: int, flat: bool) -> np.ndarray:
        out = np.empty(32768, np.float32)
        n = C.c_uint64()
        if lib().chpe_probe_dequant_cell(self.ctx, tile, int(flat), _fp(out), out.size, C.byref(n)) != 0:
            raise ChpeError(self._err())
        return out[: n.value].copy()


CONVERT_DENSE, CONVERT_RAW, CONVERT_RAW_FP16 = 0, 1, 2


def convert_archive(src: str, dst: str, mode: int, device: int = 0) -> None:
    """chpe_convert_archive: rewrite an archive as dense cells, raw tiles, or
    raw FP16 tiles (BF16 -> FP16 on the GPU)."""
    if lib().chpe_convert_archive(os.fsencode(src), os.fsencode(dst), mode, device) != 0:
        raise ChpeError(lib().chpe_last_error(None).decode())


def validate_archive(buf) -> int:
    a = np.frombuffer(buf, dtype=np.uint8)
    return lib().chpe_validate_archive(a.ctypes.data if a.size else None, a.size)
