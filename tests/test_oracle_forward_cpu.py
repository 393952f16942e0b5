"""The composition of forwardDecode (chpe_engine.zig:1663-1803), restated a
second time in numpy float64 around the oracle's weight readers, against the
oracle's own forward pass (CPU only).

The restatement reads weights only through the oracle's gemvLinear, norm,
embedding and LM-head functions (pinned on their own by the known-answer and
format tests) and redoes in float64 everything between them: RMSNorm
(:163-193), RoPE rotate-half over the whole head (:195-216), the KV append
and GQA softmax attention with scale 1/sqrt(head_dim) (:1693-1734), the
residual adds of O and down, SwiGLU (:1744-1748), the final norm and the LM
head.  A mistake in the order of operations, in which buffer feeds which
projection, in the GQA head mapping or the RoPE pairing would show as a
difference far above f32 rounding."""
import numpy as np
import pytest

import chpe_qwen_engine_b200 as chpe
import oracle_py as O

# chpe_engine.zig:110-145: hidden, FFN, layers, query heads, kv heads, head dim
DIMS = {O.ARCH_3B: (2048, 11008, 36, 16, 2, 128), O.ARCH_9B: (4096, 12288, 32, 16, 4, 256)}
THETA, EPS = 1e6, 1e-6


def rms(x, g):
    x = x.astype(np.float64)
    return x / np.sqrt(np.mean(x * x) + EPS) * g.astype(np.float64)


def rope(v, pos, heads, hd):
    v = v.astype(np.float64).reshape(heads, hd).copy()
    i = np.arange(hd // 2, dtype=np.float64)
    ang = pos * (1.0 / THETA ** (2.0 * i / hd))
    c, s = np.cos(ang), np.sin(ang)
    x0, x1 = v[:, :hd // 2].copy(), v[:, hd // 2:].copy()
    v[:, :hd // 2] = x0 * c - x1 * s
    v[:, hd // 2:] = x0 * s + x1 * c
    return v.reshape(-1)


class Composition:
    """forwardDecode in float64 around the oracle's weight readers."""

    def __init__(self, e: O.OracleEngine, arch: int, k0=None, v0=None):
        self.e = e
        self.D, self.F, L, self.H, self.KV, self.HD = DIMS[arch]
        self.layers = [e.layer_info(l) for l in range(L)]
        # cached K/V rows [layer][position][kv_heads * head_dim]
        w = self.KV * self.HD
        self.kc = np.zeros((L, 0, w)) if k0 is None else k0.astype(np.float64)
        self.vc = np.zeros((L, 0, w)) if v0 is None else v0.astype(np.float64)

    def lin(self, start, tiles, x, rows, cols, bias=-1):
        return self.e.gemv_linear(start, tiles, x.astype(np.float32), rows, cols, bias_tile=bias).astype(np.float64)

    def step(self, tok, pos):
        e, D, F, H, KV, HD = self.e, self.D, self.F, self.H, self.KV, self.HD
        h = e.embed(tok).astype(np.float64)
        ks, vs = [], []
        for l, li in enumerate(self.layers):
            xn = rms(h, e.unpack_norm(li["input_norm"], D))
            q = self.lin(li["q_proj"], li["q_tiles"], xn, H * HD, D, li["q_bias"])
            k = self.lin(li["k_proj"], li["k_tiles"], xn, KV * HD, D, li["k_bias"])
            v = self.lin(li["v_proj"], li["v_tiles"], xn, KV * HD, D, li["v_bias"])
            q, k = rope(q, pos, H, HD), rope(k, pos, KV, HD)
            K = np.concatenate([self.kc[l], k[None]])  # positions 0..pos
            Vc = np.concatenate([self.vc[l], v[None]])
            ks.append(k)
            vs.append(v)
            out = np.zeros(H * HD)
            for qh in range(H):
                kv = qh // (H // KV)
                sc = K[:, kv * HD:(kv + 1) * HD] @ q[qh * HD:(qh + 1) * HD] / np.sqrt(HD)
                p = np.exp(sc - sc.max())
                out[qh * HD:(qh + 1) * HD] = (p / p.sum()) @ Vc[:, kv * HD:(kv + 1) * HD]
            h = h + self.lin(li["o_proj"], li["o_tiles"], out, D, D)
            xn = rms(h, e.unpack_norm(li["post_norm"], D))
            g = self.lin(li["gate_proj"], li["gate_tiles"], xn, F, D)
            u = self.lin(li["up_proj"], li["up_tiles"], xn, F, D)
            h = h + self.lin(li["down_proj"], li["down_tiles"], g / (1.0 + np.exp(-g)) * u, D, F)
        self.kc = np.concatenate([self.kc, np.stack(ks)[:, None]], axis=1)
        self.vc = np.concatenate([self.vc, np.stack(vs)[:, None]], axis=1)
        hn = rms(h, e.unpack_norm(e.final_norm_index(), D))
        logits = e.lm_head(hn.astype(np.float32)).astype(np.float64)
        return logits, float(np.sqrt(h @ h))


def _compare(comp, ref, toks, pos0):
    for i, tok in enumerate(toks):
        r = ref.forward_decode(tok, pos0 + i)
        want = ref.logits().astype(np.float64)
        got, hnorm = comp.step(tok, pos0 + i)
        scale = max(1.0, float(np.max(np.abs(want))))
        err = float(np.max(np.abs(got - want)))
        assert err <= 1e-4 * scale, (pos0 + i, err, scale)
        assert abs(hnorm - r.hidden_norm) <= 2e-5 * r.hidden_norm, (pos0 + i, hnorm, r.hidden_norm)


@pytest.mark.parametrize("cfg,arch,vscale", [(chpe.SYNTH_3B_FP16_RAW, O.ARCH_3B, 3.0),
                                              (chpe.SYNTH_9B_I8_RAW, O.ARCH_9B, 30.0)])
def test_forward_composition(cfg, arch, vscale):
    """Archives that behave like a random transformer (the residual stays
    near unit scale, so attention moves the logits): 3B FP16 with q/k/v
    biases, and the 9B INT8 raw archive (linear layers as GQA with v from one
    tile, Q8; BF16 norms).  Three tokens from position 0, then two more after
    24 cached positions of seeded K/V rows loaded into both, where the
    attention output dominates the residual: swapping the rotate-half
    pairing for an interleaved one, or the kv heads, moves the logits by more
    than their own scale, against ~1e-5 here."""
    a = chpe.synth_archive(cfg, chpe.SYNTH_BIAS if arch == O.ARCH_3B else 0, seed=3)
    L, KV, HD = DIMS[arch][2], DIMS[arch][4], DIMS[arch][5]
    ref = O.OracleEngine(a, arch, 40, threads=8)
    _compare(Composition(O.OracleEngine(a, arch, 40, threads=8), arch), ref, [151644, 872, 9707], 0)
    P = 24
    rng = np.random.default_rng(9)
    k0 = (rng.standard_normal((L, P, KV * HD)) * 3.0).astype(np.float32)
    v0 = (rng.standard_normal((L, P, KV * HD)) * vscale).astype(np.float32)
    ref = O.OracleEngine(a, arch, 40, threads=8)
    for l in range(L):
        ref.kv_load(l, 0, k0[l], v0[l])
    _compare(Composition(O.OracleEngine(a, arch, 40, threads=8), arch, k0, v0), ref, [5, 77], P)
