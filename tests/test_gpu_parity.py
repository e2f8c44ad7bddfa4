"""GPU parity: the fused CUDA path, called through the C ABI, against the CPU oracle.

Bar: per stem, max |got - ref| / max |ref| <= 1e-5 (the SNR is reported as well). Inputs
are seeded synthetic audio and masks of the benchmark configurations' kind;
sizes here keep the oracle to seconds.
"""
from __future__ import annotations

import numpy as np
import pytest

from common import max_rel_err, snr_db, synth_audio, synth_mask

pytestmark = pytest.mark.gpu

TOL = 1e-5


def run_gpu(plan, mix, mask):
    import torch
    d_mix = torch.from_numpy(np.ascontiguousarray(mix)).cuda()
    d_mask = torch.from_numpy(np.ascontiguousarray(mask)).cuda()
    d_out = torch.full(plan.out_shape, float("nan"), device="cuda", dtype=torch.float32)
    plan.separate(d_mix, d_mask, d_out)
    torch.cuda.synchronize()
    return d_out.cpu().numpy()


def check(got, want, what):
    err = max_rel_err(got, want)
    snr = snr_db(got, want)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    assert err <= TOL, f"{what}: max rel err {err:.3e} (SNR {snr:.1f} dB)"
    return err, snr


# ---- RoFormer ------------------------------------------------------------------------------
RF_CASES = [
    # name, bands, chunk, num_overlap, length, zero_dc, complement, normalized
    ("mel_ov4_pad", "mel", 441 * 40, 4, 441 * 80 + 1234, True, False, False),
    ("bs_ov2_complement", "bs", 441 * 40, 2, 441 * 100 + 17, True, True, False),
    ("mel_short_reflect_tail", "mel", 441 * 40, 2, 441 * 31, False, False, False),   # len < chunk
    ("bs_short_zero_tail", "bs", 441 * 40, 2, 441 * 15, False, False, True),        # tail <= chunk/2
    ("mel_no_border_pad", "mel", 441 * 40, 4, 441 * 50, True, False, False),         # len < 2*border
]


@pytest.mark.parametrize("case", RF_CASES, ids=[c[0] for c in RF_CASES])
def test_roformer_matches_oracle(case, pkg, engine, oracle_mod):
    name, kind, chunk, nov, length, zdc, comp, norm = case
    sizes, freqs = pkg.bands.mel_bands() if kind == "mel" else pkg.bands.bs_bands()
    plan = engine.plan_roformer(length, sizes, freqs, chunk=chunk, num_overlap=nov, zero_dc=zdc,
                                complement=comp, normalized=norm)
    mix = synth_audio(11, length)
    mask = synth_mask(12, plan.mask_floats, 0.5)
    got = run_gpu(plan, mix, mask)
    p = oracle_mod.rf_params(sizes, freqs, chunk=chunk, num_overlap=nov, zero_dc=int(zdc),
                             complement=int(comp), normalized=int(norm), threads=8)
    assert plan.n_chunks == oracle_mod.rf_n_chunks(p, length)
    want = oracle_mod.rf_separate(p, mix, mask)
    check(got, want, name)


# ---- HTDemucs ------------------------------------------------------------------------------
HT_CASES = [
    # name, segment, length, sources, overlap, channels, mono_norm, cac_norm
    ("seg24k_4src", 1024 * 24, 60000, 4, -1.0, 2, 1, 1),   # the reference's normalisations
    ("seg24k_raw", 1024 * 24, 60000, 4, -1.0, 2, 0, 0),
    ("seg24k_short", 1024 * 24, 9000, 2, -1.0, 2, 1, 1),   # one segment, centre-padded
    ("seg_odd_ov05", 1024 * 20 + 333, 51001, 4, 0.5, 2, 1, 1),
    ("seg24k_mono_norm_only", 1024 * 24, 70001, 4, -1.0, 2, 1, 0),
    ("seg24k_cac_norm_only", 1024 * 24, 70001, 6, -1.0, 2, 0, 1),
    ("seg24k_one_channel", 1024 * 24, 60000, 4, -1.0, 1, 1, 1),
]


@pytest.mark.parametrize("case", HT_CASES, ids=[c[0] for c in HT_CASES])
def test_htdemucs_matches_oracle(case, pkg, engine, oracle_mod):
    name, seg, length, S, ov, ch, mono, cac = case
    plan = engine.plan_htdemucs(length, n_channels=ch, n_sources=S, segment=seg, overlap=ov, mono_norm=mono,
                                cac_norm=cac)
    mix = synth_audio(21, length, channels=ch)
    mask = synth_mask(22, plan.mask_floats, 1.0)
    got = run_gpu(plan, mix, mask)
    p = oracle_mod.ht_params(n_channels=ch, n_sources=S, segment=seg, overlap=ov, mono_norm=mono, cac_norm=cac,
                             threads=8)
    assert plan.n_chunks == oracle_mod.ht_n_segments(p, length)
    want = oracle_mod.ht_separate(p, mix, mask)
    check(got, want, name)


# ---- random shifts (src/htdemucs.cpp:610-626, src/roformer.cpp:456-478) -----------------------
@pytest.mark.parametrize("shifts,seed", [(1, 0), (3, 17)])
def test_htdemucs_shifts_match_oracle(engine, oracle_mod, shifts, seed):
    seg, length, S = 1024 * 24, 60000, 4
    plan = engine.plan_htdemucs(length, n_sources=S, segment=seg, shifts=shifts, seed=seed)
    p = oracle_mod.ht_params(n_sources=S, segment=seg, mono_norm=1, cac_norm=1, shifts=shifts, seed=seed,
                             threads=8)
    assert plan.n_chunks == oracle_mod.ht_n_segments(p, length)
    mix = synth_audio(31, length)
    mask = synth_mask(32, plan.mask_floats, 1.0)
    check(run_gpu(plan, mix, mask), oracle_mod.ht_separate(p, mix, mask), f"ht shifts={shifts}")


@pytest.mark.parametrize("length", [441 * 100 + 33, 15000])   # 15000: only the shifted tracks are padded
def test_roformer_shifts_match_oracle(pkg, engine, oracle_mod, length):
    sizes, freqs = pkg.bands.bs_bands()
    chunk = 441 * 40
    plan = engine.plan_roformer(length, sizes, freqs, chunk=chunk, num_overlap=2, zero_dc=True, complement=True,
                                shifts=2, seed=9)
    p = oracle_mod.rf_params(sizes, freqs, chunk=chunk, num_overlap=2, zero_dc=1, complement=1, shifts=2, seed=9,
                             threads=8)
    assert plan.n_chunks == oracle_mod.rf_n_chunks(p, length)
    mix = synth_audio(33, length)
    mask = synth_mask(34, plan.mask_floats, 0.5)
    check(run_gpu(plan, mix, mask), oracle_mod.rf_separate(p, mix, mask), f"rf shifts, length {length}")


# ---- TFC-TDF -------------------------------------------------------------------------------
TFC_CASES = [
    # name, dim_t, chunking, overlap, length, compensate, complement
    ("uvr_dt32_ov05", 32, "uvr_mdx", 0.5, 70000, 1.009, True),
    ("uvr_dt32_default", 32, "uvr_mdx", -1.0, 50000, 1.0, False),
    ("msst_dt32", 32, "msst", -1.0, 90001, 1.0, True),
]


@pytest.mark.parametrize("case", TFC_CASES, ids=[c[0] for c in TFC_CASES])
def test_tfc_matches_oracle(case, pkg, engine, oracle_mod):
    name, dim_t, chunking, ov, length, comp, complement = case
    plan = engine.plan_tfc(length, n_fft=7680, hop=1024, dim_f=3072, dim_t=dim_t, zero_bins=3,
                           chunking=chunking, overlap=ov, num_overlap=4, compensate=comp,
                           complement=complement)
    mix = synth_audio(31, length)
    mask = synth_mask(32, plan.mask_floats, 1.0)
    got = run_gpu(plan, mix, mask)
    p = oracle_mod.tfc_params(dim_t=dim_t, chunking=0 if chunking == "uvr_mdx" else 1, overlap=ov,
                              num_overlap=4, compensate=comp, complement=int(complement), threads=8)
    assert plan.n_chunks == oracle_mod.tfc_n_chunks(p, length)
    want = oracle_mod.tfc_separate(p, mix, mask)
    check(got, want, name)


@pytest.mark.parametrize("hop,stems", [(1023, 1), (768, 2)], ids=["odd_hop_one_cta", "even_hop_pair_two_stems"])
def test_tfc_7680_hops(hop, stems, pkg, engine, oracle_mod):
    """n_fft 7680 runs on CTA pairs split by sample parity when the hop is even and on one CTA
    when it is odd; both against the oracle, the pair also with two stems."""
    length = 61001
    plan = engine.plan_tfc(length, n_fft=7680, hop=hop, dim_f=3072, dim_t=32, zero_bins=3, n_stems=stems,
                           chunking="uvr_mdx", overlap=0.5, compensate=1.0, complement=True)
    mix = synth_audio(35, length)
    mask = synth_mask(36, plan.mask_floats, 1.0)
    got = run_gpu(plan, mix, mask)
    p = oracle_mod.tfc_params(n_stems=stems, n_fft=7680, hop=hop, dim_t=32, chunking=0, overlap=0.5,
                              complement=1, threads=8)
    assert plan.n_chunks == oracle_mod.tfc_n_chunks(p, length)
    check(got, oracle_mod.tfc_separate(p, mix, mask), f"tfc hop {hop}")


# ---- determinism and the host-buffer entry point ---------------------------------------
def test_deterministic_and_host_entry(pkg, engine):
    sizes, freqs = pkg.bands.mel_bands()
    length = 441 * 90
    plan = engine.plan_roformer(length, sizes, freqs, chunk=441 * 40, num_overlap=4)
    mix = synth_audio(41, length)
    mask = synth_mask(42, plan.mask_floats, 0.5)
    a = run_gpu(plan, mix, mask)
    b = run_gpu(plan, mix, mask)
    c = plan.separate_host(mix, mask)
    assert np.array_equal(a, b), "two runs differ bitwise"
    assert np.array_equal(a, c), "host entry point differs from the device one"
    assert np.array_equal(a, plan.separate_host(mix, mask)), "second host call differs"


def test_host_entry_tfc_batches(pkg, engine):
    """The host entry point brings the masks in batch by batch (the TFC-TDF ones transposed per
    batch): the same floats as the device entry point, call after call."""
    length = 44100 * 8 + 17
    plan = engine.plan_tfc(length, dim_t=32, complement=True)
    assert plan.n_chunks >= 9
    mix = synth_audio(43, length)
    mask = synth_mask(44, plan.mask_floats, 1.0)
    a = run_gpu(plan, mix, mask)
    for _ in range(2):
        assert np.array_equal(a, plan.separate_host(mix, mask))


@pytest.mark.parametrize("shifts", [0, 2])
def test_host_entry_htdemucs_batches(pkg, engine, shifts):
    """HTDemucs through the host entry point: each batch's masks transposed as they arrive
    (with shifts, the batches cross from one shift pass's segments into the next)."""
    length = 44100 * 30 + 7
    plan = engine.plan_htdemucs(length, shifts=shifts, seed=5)
    assert plan.n_chunks >= 4
    mix = synth_audio(45, length)
    mask = synth_mask(46, plan.mask_floats, 1.0)
    a = run_gpu(plan, mix, mask)
    for _ in range(2):
        assert np.array_equal(a, plan.separate_host(mix, mask))


# ---- DualMono (src/separator.cpp:15-47) ----------------------------------------------------------
def test_dual_mono_roformer_matches_oracle(pkg, engine, oracle_mod):
    """A mono RoFormer (a dereverb model's layout) over a stereo mix, channel by channel."""
    import torch
    sizes, freqs = pkg.bands.bs_bands()
    chunk, n = 441 * 40, 441 * 90 + 11
    plan = engine.plan_roformer(n, sizes, freqs, n_channels=1, chunk=chunk, num_overlap=2, complement=True)
    mix = synth_audio(91, n)
    mask = synth_mask(92, 2 * plan.mask_floats, 0.5)   # left channel's masks, then the right's
    out = torch.empty((plan.n_out_sources, 2, n), device="cuda")
    plan.separate_dual_mono(torch.from_numpy(mix).cuda(), torch.from_numpy(mask).cuda(), out)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    p = oracle_mod.rf_params(sizes, freqs, n_channels=1, chunk=chunk, num_overlap=2, complement=1, threads=8)
    for c in range(2):
        want = oracle_mod.rf_separate(p, mix[c:c + 1], mask[c * plan.mask_floats:(c + 1) * plan.mask_floats])
        check(got[:, c:c + 1], want, f"dual mono channel {c}")


def test_misaligned_mask_is_rejected(pkg, engine):
    import torch
    sizes, freqs = pkg.bands.bs_bands()
    n = 441 * 60
    plan = engine.plan_roformer(n, sizes, freqs, chunk=441 * 40, num_overlap=2)
    mask = torch.zeros(plan.mask_floats + 4, device="cuda")
    with pytest.raises(pkg.StemsError) as e:
        plan.separate(torch.zeros((2, n), device="cuda"), mask[1:], torch.empty(plan.out_shape, device="cuda"))
    assert e.value.code == 1 and "aligned" in str(e.value)


# ---- a track split by output samples (stg_separate_part) -----------------------------------------
def _parts_equal_whole(pkg, plan, mix, mask, parts):
    import torch
    d_mix, d_mask = torch.from_numpy(mix).cuda(), torch.from_numpy(mask).cuda()
    whole = torch.empty(plan.out_shape, device="cuda")
    plan.separate(d_mix, d_mask, whole)
    split = torch.full(plan.out_shape, float("nan"), device="cuda")
    for r in range(parts):
        b, e = pkg.sharding.sample_range_for_rank(plan.n_samples, r, parts)
        plan.separate_part(d_mix, d_mask, split, b, e)
    torch.cuda.synchronize()
    assert torch.equal(split, whole)


@pytest.mark.parametrize("shifts", [0, 2])
def test_roformer_parts_equal_whole(pkg, engine, shifts):
    sizes, freqs = pkg.bands.mel_bands()
    n = 441 * 200 + 77
    plan = engine.plan_roformer(n, sizes, freqs, chunk=441 * 40, num_overlap=4, complement=True, shifts=shifts,
                                seed=4)
    _parts_equal_whole(pkg, plan, synth_audio(93, n), synth_mask(94, plan.mask_floats, 0.5), 3)


def test_htdemucs_parts_equal_whole(pkg, engine):
    n = 1024 * 24 * 5 + 123
    plan = engine.plan_htdemucs(n, n_sources=4, segment=1024 * 24)
    _parts_equal_whole(pkg, plan, synth_audio(95, n), synth_mask(96, plan.mask_floats, 1.0), 4)


def test_tfc_parts_equal_whole(pkg, engine):
    n = 120000
    plan = engine.plan_tfc(n, dim_t=32, overlap=0.5, compensate=1.009, complement=True)
    _parts_equal_whole(pkg, plan, synth_audio(97, n), synth_mask(98, plan.mask_floats, 1.0), 2)

