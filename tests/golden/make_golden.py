#!/usr/bin/env python
"""Writes tests/golden/golden.npz from the reference's own compiled DSP code.

Run where the reference sources are present (it needs oracle/_ref/libstems_ref.so, which
oracle/build.sh compiles from the reference's src/stft.h and src/vr_dsp.h):

    python tests/golden/make_golden.py

What it stores:
  * primitives computed by the reference itself (st::FFT, st::VRFFT, st::torch_stft/istft,
    st::htdemucs_spec/ispec, st::resample_planar, st::vr_stft/vr_istft/vr_resample) on small
    seeded inputs;
  * whole separations (RoFormer, HTDemucs, TFC-TDF host loops as restated in oracle.c, with
    the network replaced by a seeded mask) whose DSP primitives are the reference's own.
Inputs are regenerated from their seeds by the tests; a checksum of each input is stored so
that a change in numpy's generators is caught instead of read as a parity failure.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(HERE))

import oracle  # noqa: E402
from golden_cases import CASES, RESAMPLE_RATES, VR_RESAMPLES, VR_STFTS, inputs_for  # noqa: E402


def main():
    oracle.build(force=True)
    R = oracle.ref_lib()
    if R is None:
        sys.exit("the reference shim is not built (reference sources absent)")
    out = {}
    # -- primitives, straight from the reference ---------------------------------------------
    rng = np.random.default_rng(2024)
    x = rng.uniform(-1, 1, 4096) + 1j * rng.uniform(-1, 1, 4096)
    out["prim_fft4096_in"] = x.astype(np.complex128)
    out["prim_fft4096"] = oracle.fft(x, impl=R)
    v = np.zeros(7680, np.complex128)
    v[7] = 1.0
    v[100] = 0.5 - 0.25j
    out["prim_vrfft7680_in"] = v
    out["prim_vrfft7680"] = oracle.fft(v, impl=R)
    a = rng.uniform(-1, 1, 441 * 10 + 3).astype(np.float32)
    out["prim_stft_in"] = a
    s = oracle.torch_stft(a, 2048, 441, False, impl=R)
    out["prim_stft_2048_441"] = s
    out["prim_istft_2048_441"] = oracle.torch_istft(s, 2048, 441, False, impl=R)
    b = rng.uniform(-0.5, 0.5, 1024 * 8 + 100).astype(np.float32)
    out["prim_hspec_in"] = b
    h = oracle.htdemucs_spec(b, impl=R)
    out["prim_hspec_4096"] = h
    out["prim_hispec_4096"] = oracle.htdemucs_ispec(h, b.size, impl=R)
    # -- the input resampler, straight from the reference (src/audio.h resample_planar) -----
    io = np.random.default_rng(77).uniform(-1, 1, (3, 3001)).astype(np.float32)
    out["io_resample_in"] = io
    for src, dst in RESAMPLE_RATES:
        out[f"io_resample_{src}_{dst}"] = oracle.resample_planar(io, src, dst, impl=R)
    # -- VR primitives, straight from the reference (src/vr_dsp.h) --------------------------
    vw = np.random.default_rng(78).uniform(-0.5, 0.5, (2, 2000)).astype(np.float32)
    out["vr_wave_in"] = vw
    for nfft, hop in VR_STFTS:
        spec = oracle.vr_stft(vw, nfft, hop, impl=R)
        out[f"vr_stft_{nfft}_{hop}"] = spec
        out[f"vr_istft_{nfft}_{hop}"] = oracle.vr_istft(spec, nfft, hop, impl=R)
    for src, dst in VR_RESAMPLES:
        out[f"vr_fir_{src}_{dst}"] = oracle.vr_fir(src, dst)
        out[f"vr_resample_{src}_{dst}"] = oracle.vr_resample(vw, src, dst, out[f"vr_fir_{src}_{dst}"], impl=R)
    # -- whole separations with the reference's primitives ----------------------------------
    assert oracle.use_reference(True)
    for name, case in CASES.items():
        params, mix, mask = inputs_for(case)
        out[f"{name}_out"] = case["run"](params, mix, mask)
        out[f"{name}_mix_sum"] = np.float64(np.sum(mix, dtype=np.float64))
        out[f"{name}_mask_sum"] = np.float64(np.sum(mask, dtype=np.float64))
    oracle.use_reference(False)
    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path) / 1e6:.2f} MB, {len(out)} arrays)")


if __name__ == "__main__":
    main()
