"""GPU parity at the benchmark configurations' full sizes, against the CPU oracle (threads on
every host core). These are the five workloads bench.py times:

  cfg0  HTDemucs, 20 s, 4 stems, segment 343980, overlap 0.25
  cfg1  Mel-Band RoFormer (Kim), 60 s, chunk 352800, num_overlap 4, 60 mel bands
  cfg2  BS-RoFormer (viperx 317), 180 s, chunk 352800, num_overlap 2, zero_dc
  cfg3  MDX TFC-TDF (Kim_Vocal_2), 180 s, n_fft 7680, dim_f 3072, dim_t 256, UVR overlap 0.5
  cfg4  the batch of 240 s HTDemucs tracks, two of them here

Bar: per stem, max |got - ref| / max |ref| <= 1e-5, and an SNR of at least 100 dB. Besides the
oracle comparison, properties that hold at any size are checked: the RoFormer path with every
band mask 1 + 0i returns the mix (the whole chunked path is then the identity), and the
separation is linear in the mask.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

from common import max_rel_err, snr_db, synth_audio, synth_mask

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

SR = 44100
THREADS = os.cpu_count() or 1


def _gpu(plan, mix, mask):
    import torch
    d_out = torch.empty(plan.out_shape, device="cuda", dtype=torch.float32)
    plan.separate(torch.from_numpy(mix).cuda(), torch.from_numpy(mask).cuda(), d_out)
    torch.cuda.synchronize()
    return d_out.cpu().numpy()


def _check(got, want, what):
    err, snr = max_rel_err(got, want), snr_db(got, want)
    print(f"{what}: max rel err {err:.2e}, SNR {snr:.1f} dB")
    assert err <= 1e-5 and snr >= 100.0, f"{what}: max rel err {err:.3e}, SNR {snr:.1f} dB"


def test_cfg1_mel_roformer_60s(pkg, engine, oracle_mod):
    sizes, freqs = pkg.bands.mel_bands()
    n = 60 * SR
    plan = engine.plan_roformer(n, sizes, freqs, chunk=352800, num_overlap=4)
    assert plan.n_chunks == 36 and plan.n_frames == 801
    mix = synth_audio(1, n)
    mask = synth_mask(2, plan.mask_floats, 0.5)
    want = oracle_mod.rf_separate(oracle_mod.rf_params(sizes, freqs, chunk=352800, num_overlap=4,
                                                       threads=THREADS), mix, mask)
    _check(_gpu(plan, mix, mask), want, "cfg1")


def test_cfg2_bs_roformer_180s(pkg, engine, oracle_mod):
    sizes, freqs = pkg.bands.bs_bands()
    n = 180 * SR
    plan = engine.plan_roformer(n, sizes, freqs, chunk=352800, num_overlap=2, zero_dc=True)
    assert plan.n_chunks == 47
    mix = synth_audio(3, n)
    mask = synth_mask(4, plan.mask_floats, 0.5)
    want = oracle_mod.rf_separate(oracle_mod.rf_params(sizes, freqs, chunk=352800, num_overlap=2, zero_dc=1,
                                                       threads=THREADS), mix, mask)
    _check(_gpu(plan, mix, mask), want, "cfg2")


def test_cfg2_split_eight_ways_equals_whole(pkg, engine):
    """bench.py's strong-scaling record at 8 GPUs, on one: cfg2's output samples split into 8
    ranges (sharding.sample_range_for_rank), each written by stg_separate_part, give the same
    bits as the whole track."""
    import torch
    sizes, freqs = pkg.bands.bs_bands()
    n = 180 * SR
    plan = engine.plan_roformer(n, sizes, freqs, chunk=352800, num_overlap=2, zero_dc=True)
    d_mix = torch.from_numpy(synth_audio(3, n)).cuda()
    d_mask = torch.from_numpy(synth_mask(4, plan.mask_floats, 0.5)).cuda()
    whole = torch.empty(plan.out_shape, device="cuda")
    plan.separate(d_mix, d_mask, whole)
    split = torch.full(plan.out_shape, float("nan"), device="cuda")
    for r in range(8):
        b, e = pkg.sharding.sample_range_for_rank(n, r, 8)
        plan.separate_part(d_mix, d_mask, split, b, e)
    torch.cuda.synchronize()
    assert torch.equal(split, whole)


def test_cfg0_htdemucs_20s(engine, oracle_mod):
    n = 20 * SR
    plan = engine.plan_htdemucs(n, n_sources=4, segment=343980)
    assert plan.n_chunks == 4 and plan.n_frames == 336
    mix = synth_audio(5, n)
    mask = synth_mask(6, plan.mask_floats, 1.0)
    p = oracle_mod.ht_params(n_sources=4, segment=343980, mono_norm=1, cac_norm=1, threads=THREADS)
    want = oracle_mod.ht_separate(p, mix, mask)
    _check(_gpu(plan, mix, mask), want, "cfg0")


def test_cfg3_mdx_kim_vocal_180s(engine, oracle_mod):
    n = 180 * SR
    plan = engine.plan_tfc(n, n_fft=7680, hop=1024, dim_f=3072, dim_t=256, zero_bins=3, overlap=0.5,
                           compensate=1.009, complement=True)
    assert plan.n_chunks == 63
    mix = synth_audio(7, n)
    mask = synth_mask(8, plan.mask_floats, 1.0)
    p = oracle_mod.tfc_params(overlap=0.5, compensate=1.009, complement=1, threads=THREADS)
    want = oracle_mod.tfc_separate(p, mix, mask)
    _check(_gpu(plan, mix, mask), want, "cfg3")


def test_cfg4_batch_htdemucs_two_tracks(engine, oracle_mod):
    n = 240 * SR
    plan = engine.plan_htdemucs(n, n_sources=4, segment=343980)
    assert plan.n_chunks == 42
    p = oracle_mod.ht_params(n_sources=4, segment=343980, mono_norm=1, cac_norm=1, threads=THREADS)
    for track in range(2):
        mix = synth_audio(40 + track, n)
        mask = synth_mask(50 + track, plan.mask_floats, 1.0)
        _check(_gpu(plan, mix, mask), oracle_mod.ht_separate(p, mix, mask), f"cfg4 track {track}")


def test_roformer_identity_mask_returns_the_mix(pkg, engine):
    sizes, freqs = pkg.bands.mel_bands()
    n = 60 * SR
    plan = engine.plan_roformer(n, sizes, freqs, chunk=352800, num_overlap=4)
    T = plan.n_frames
    mask = np.zeros((plan.n_chunks, int(sizes.sum()) * 4 * T), np.float32)
    mask[:, 0::2] = 1.0
    mix = synth_audio(9, n)
    got = _gpu(plan, mix, mask.reshape(-1))
    assert np.abs(got[0] - mix).max() < 1e-5


def test_separation_is_linear_in_the_mask(pkg, engine):
    sizes, freqs = pkg.bands.bs_bands()
    n = 30 * SR
    plan = engine.plan_roformer(n, sizes, freqs, chunk=352800, num_overlap=2)
    mix = synth_audio(10, n)
    a = synth_mask(11, plan.mask_floats, 0.5)
    b = synth_mask(12, plan.mask_floats, 0.5)
    ya, yb, yab = _gpu(plan, mix, a), _gpu(plan, mix, b), _gpu(plan, mix, (2.0 * a + b).astype(np.float32))
    assert np.abs(yab - (2.0 * ya + yb)).max() <= 1e-5 * np.abs(yab).max()
