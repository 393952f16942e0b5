"""The Gated DeltaNet decode-step kernel (chpe_deltanet_step) on the GPU:
against the transformers golden vectors (tests/golden/deltanet_step.npz, 2
key / 4 value heads, three steps) and against the CPU oracle at the 9B head
counts (16 key / 32 value heads of 128, four steps from a random state),
outputs within f32 summation order and the conv history bit-exact."""
import ctypes as C
import os

import numpy as np
import pytest

import chpe_qwen_engine_b200 as chpe
import oracle_py as O

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _run_gpu(steps, nk, nv, conv_w, hist0, state0, a_log, dt_bias, norm_w, t0, eps):
    import torch
    dev = torch.device("cuda:0")
    T = lambda x: torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(dev)
    w, hist, state = T(conv_w), T(hist0), T(state0)
    al, dt, nw = T(a_log), T(dt_bias), T(norm_w)
    out = torch.zeros(nv * 128, dtype=torch.float32, device=dev)
    L = chpe.lib()
    outs = []
    for s, (mixed, z, a, b) in enumerate(steps):
        m_, z_, a_, b_ = T(mixed), T(z), T(a), T(b)
        rc = L.chpe_deltanet_step(m_.data_ptr(), z_.data_ptr(), a_.data_ptr(), b_.data_ptr(), w.data_ptr(),
                                  hist.data_ptr(), t0 + s, al.data_ptr(), dt.data_ptr(), nw.data_ptr(),
                                  state.data_ptr(), out.data_ptr(), nk, nv, 128, 128, eps, None)
        assert rc == 0
        torch.cuda.synchronize()
        outs.append(out.cpu().numpy().copy())
    return outs, hist.cpu().numpy(), state.cpu().numpy()


def test_deltanet_kernel_matches_transformers_golden():
    g = np.load(os.path.join(HERE, "golden", "deltanet_step.npz"))
    steps = [(g["mixed"][s], g["z"][s], g["a"][s], g["b"][s]) for s in range(g["mixed"].shape[0])]
    outs, hist, state = _run_gpu(steps, int(g["nk"]), int(g["nv"]), g["conv_w"], g["hist0"], g["state0"],
                                 g["a_log"], g["dt_bias"], g["norm_w"], int(g["t0"]), float(g["eps"]))
    for s, o in enumerate(outs):
        ref = g["out"][s]
        assert np.max(np.abs(o - ref)) <= 2e-5 * max(1.0, float(np.max(np.abs(ref)))), s
    assert np.array_equal(hist, g["hist_end"])
    assert np.max(np.abs(state - g["state_end"])) <= 1e-5 * max(1.0, float(np.max(np.abs(g["state_end"]))))


def test_deltanet_kernel_matches_oracle_at_9b_heads():
    nk, nv, eps, t0 = 16, 32, 1e-6, 0
    conv_dim = 2 * nk * 128 + nv * 128
    rng = np.random.default_rng(21)
    f = lambda *s, sc=1.0: (rng.standard_normal(s) * sc).astype(np.float32)
    conv_w = f(conv_dim, 4, sc=0.5)
    a_log = np.log(rng.uniform(1, 16, nv)).astype(np.float32)
    dt_bias = f(nv, sc=0.5)
    norm_w = (1.0 + f(128, sc=0.1)).astype(np.float32)
    hist0 = np.zeros((4, conv_dim), np.float32)  # a fresh sequence
    state0 = f(nv, 128, 128, sc=0.05)
    steps = [(f(conv_dim), f(nv * 128), f(nv), f(nv)) for _ in range(4)]
    outs, hist, state = _run_gpu(steps, nk, nv, conv_w, hist0, state0, a_log, dt_bias, norm_w, t0, eps)
    h_ref, s_ref = hist0.copy(), state0.copy()
    for s, (mixed, z, a, b) in enumerate(steps):
        ref = O.deltanet_step(mixed, z, a, b, conv_w, h_ref, t0 + s, a_log, dt_bias, norm_w, s_ref,
                              nk, nv, 128, 128, eps)
        assert np.max(np.abs(outs[s] - ref)) <= 2e-5 * max(1.0, float(np.max(np.abs(ref)))), s
    assert np.array_equal(hist, h_ref)
    assert np.max(np.abs(state - s_ref)) <= 1e-5 * max(1.0, float(np.max(np.abs(s_ref))))


def test_deltanet_rejects_bad_arguments():
    L = chpe.lib()
    assert L.chpe_deltanet_step(None, None, None, None, None, None, 0, None, None, None, None, None,
                                16, 32, 128, 128, 1e-6, None) == -1
