"""The small whole-separation cases pinned by tests/golden/golden.npz (see make_golden.py)."""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from common import synth_audio, synth_mask  # noqa: E402


def _bands(kind):
    import __graft_entry__
    b = __graft_entry__.load_package().bands
    return b.mel_bands() if kind == "mel" else b.bs_bands()


def _rf(kind, chunk, nov, length, zero_dc, complement):
    def params():
        sizes, freqs = _bands(kind)
        return oracle.rf_params(sizes, freqs, chunk=chunk, num_overlap=nov, zero_dc=zero_dc,
                                complement=complement)

    def mask_floats(p, length):
        sizes, _ = _bands(kind)
        T = chunk // 441 + 1
        return oracle.rf_n_chunks(p, length) * int(sizes.sum()) * 4 * T

    return dict(params=params, length=length, mask_floats=mask_floats, sigma=0.5,
                run=oracle.rf_separate, gpu=dict(arch="roformer", bands=kind, chunk=chunk, num_overlap=nov,
                                                  zero_dc=bool(zero_dc), complement=bool(complement)))


def _ht(segment, length, sources):
    def params():
        return oracle.ht_params(n_sources=sources, segment=segment)

    def mask_floats(p, length):
        return oracle.ht_n_segments(p, length) * sources * 4 * 2048 * oracle.ht_n_frames(p)

    return dict(params=params, length=length, mask_floats=mask_floats, sigma=1.0, run=oracle.ht_separate,
                gpu=dict(arch="htdemucs", segment=segment, sources=sources))


def _tfc(dim_t, chunking, overlap, length, compensate, complement):
    def params():
        return oracle.tfc_params(dim_t=dim_t, chunking=chunking, overlap=overlap, num_overlap=4,
                                 compensate=compensate, complement=complement)

    def mask_floats(p, length):
        return oracle.tfc_n_chunks(p, length) * 4 * 3072 * dim_t

    return dict(params=params, length=length, mask_floats=mask_floats, sigma=1.0, run=oracle.tfc_separate,
                gpu=dict(arch="tfc", dim_t=dim_t, chunking=chunking, overlap=overlap, compensate=compensate,
                         complement=bool(complement)))


# (source rate, destination rate) pairs of the resampler's golden vectors
RESAMPLE_RATES = [(48000, 44100), (44100, 48000), (22050, 44100), (44100, 32000), (8000, 44100)]

# VR primitives' golden vectors: (n_fft, hop) of vr_stft / vr_istft and resampler rate pairs
VR_STFTS = [(320, 80), (640, 160), (960, 480), (512, 128), (2048, 1024)]
VR_RESAMPLES = [(44100, 22050), (22050, 44100), (44100, 7350), (7350, 44100)]

CASES = {
    "rf_mel": _rf("mel", 441 * 20, 4, 441 * 45 + 7, 0, 0),
    "rf_bs": _rf("bs", 441 * 20, 2, 441 * 33 + 100, 1, 1),
    "ht": _ht(1024 * 12, 20000, 2),
    "tfc_uvr": _tfc(16, 0, 0.5, 25000, 1.009, 1),
    "tfc_msst": _tfc(16, 1, -1.0, 33333, 1.0, 0),
}


def inputs_for(case, seed=5):
    p = case["params"]()
    mix = synth_audio(seed, case["length"])
    mask = synth_mask(seed + 1, case["mask_floats"](p, case["length"]), case["sigma"])
    return p, mix, mask
