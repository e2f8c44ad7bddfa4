"""Helpers shared by the tests: parity metrics and the benchmark's synthetic inputs."""
from __future__ import annotations

import numpy as np


def max_rel_err(got, want):
    """max |got - want| / max |want| per stem (row 0 of the leading axis), the worst one."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    worst = 0.0
    for g, w in zip(got.reshape(got.shape[0], -1), want.reshape(want.shape[0], -1)):
        scale = np.abs(w).max()
        worst = max(worst, float(np.abs(g - w).max() / (scale if scale > 0 else 1.0)))
    return worst


def snr_db(got, want):
    """Worst per-stem SNR, 10 log10(sum ref^2 / sum (got - ref)^2) (tools/stems-parity.cpp:26-37)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    worst = np.inf
    for g, w in zip(got.reshape(got.shape[0], -1), want.reshape(want.shape[0], -1)):
        num, den = np.sum(w * w), np.sum((g - w) ** 2)
        worst = min(worst, np.inf if den == 0 else 10 * np.log10(num / den))
    return worst


def synth_audio(seed, length, channels=2, sr=44100):
    """The benchmark's synthetic mix: per channel 8 seeded sines (50-8000 Hz, amplitude
    0.05-0.2, random phase) plus white noise sigma 0.01, clipped to [-1, 1]."""
    rng = np.random.default_rng(seed)
    t = np.arange(length, dtype=np.float64) / sr
    out = np.empty((channels, length), np.float32)
    for c in range(channels):
        f = rng.uniform(50, 8000, 8)
        a = rng.uniform(0.05, 0.2, 8)
        ph = rng.uniform(0, 2 * np.pi, 8)
        x = (a[:, None] * np.sin(2 * np.pi * f[:, None] * t[None, :] + ph[:, None])).sum(0)
        x += 0.01 * rng.standard_normal(length)
        out[c] = np.clip(x, -1, 1)
    return out


def synth_mask(seed, n, sigma):
    return (sigma * np.random.default_rng(seed).standard_normal(n)).astype(np.float32)
