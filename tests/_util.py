"""Shared helpers for the parity tests (archives, comparisons)."""
from __future__ import annotations

import functools
import os

import numpy as np

import chpe_qwen_engine_b200 as chpe


@functools.lru_cache(maxsize=4)
def archive(config: int, flags: int = 0, seed: int = 0) -> np.ndarray:
    return chpe.synth_archive(config, flags, seed)


def oracle_threads() -> int:
    return max(1, min(os.cpu_count() or 1, 64))


def cosine(a: np.ndarray, b: np.ndarray) -> float:
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))


def assert_logits_match(got: np.ndarray, ref: np.ndarray, what: str = ""):
    """Per-step gate: max-abs-err <= 2e-2 and cosine >= 0.9999; identical
    argmax wherever the reference's top-1 margin exceeds 1e-3."""
    assert got.shape == ref.shape, what
    assert np.all(np.isfinite(got)) == np.all(np.isfinite(ref)), what
    err = float(np.max(np.abs(got.astype(np.float64) - ref.astype(np.float64))))
    cos = cosine(got, ref) if np.any(ref) or np.any(got) else 1.0
    assert err <= 2e-2, f"{what}: max-abs-err {err}"
    assert cos >= 0.9999, f"{what}: cosine {cos}"
    top2 = np.partition(ref, -2)[-2:]
    margin = float(top2[1] - top2[0])
    if margin > 1e-3:
        assert int(np.argmax(got)) == int(np.argmax(ref)), f"{what}: argmax differs (margin {margin})"
    return err, cos, margin


def assert_close_vec(got: np.ndarray, ref: np.ndarray, rel: float = 1e-4, what: str = ""):
    scale = max(1e-6, float(np.max(np.abs(ref))))
    err = float(np.max(np.abs(got.astype(np.float64) - ref.astype(np.float64))))
    assert err <= rel * scale, f"{what}: max-abs-err {err} vs scale {scale}"
    return err
