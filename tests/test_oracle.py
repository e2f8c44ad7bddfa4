"""The CPU oracle, pinned three ways (no GPU needed):

1. the reference's own known-answer tests, restated against the oracle's primitives
   (tests/dsp_test.cpp:53-96 and tests/vr_dsp_test.cpp:8-33 of the reference), and, where
   the reference was compiled here (oracle/_ref), the reference's own test binaries;
2. the golden vectors of tests/golden/golden.npz, produced by the reference's compiled
   st::FFT / st::VRFFT / st::torch_stft / st::htdemucs_spec (make_golden.py);
3. the live reference, when oracle/_ref is present: primitives bit for bit, and whole
   separations with the reference's primitives under the restated host loops.
"""
from __future__ import annotations

import os
import subprocess

import numpy as np
import pytest

from common import synth_audio
from golden_cases import CASES, RESAMPLE_RATES, VR_RESAMPLES, VR_STFTS, inputs_for

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden", "golden.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


# ---- 1. the reference's known-answer tests -----------------------------------------------
@pytest.mark.parametrize("binary", ["dsp_test", "vr_dsp_test"])
def test_reference_kat_binaries_pass(binary):
    path = os.path.join(ROOT, "oracle", "_ref", binary)
    if not os.path.exists(path):
        pytest.skip("reference not compiled on this machine")
    res = subprocess.run([path], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0 and "PASS" in res.stdout, res.stdout + res.stderr


def test_fft_inverse_is_identity(oracle_mod):                   # dsp_test.cpp:53-64
    rng = np.random.default_rng(1234)
    a = rng.uniform(-1, 1, 4096) + 1j * rng.uniform(-1, 1, 4096)
    back = oracle_mod.fft(oracle_mod.fft(a), inverse=True) / 4096
    assert np.abs(back - a).max() < 1e-12


@pytest.mark.parametrize("normalized", [False, True])
def test_stft_round_trip(oracle_mod, normalized):               # dsp_test.cpp:66-78
    rng = np.random.default_rng(99)
    x = rng.uniform(-1, 1, 441 * 200).astype(np.float32)
    y = oracle_mod.torch_istft(oracle_mod.torch_stft(x, 2048, 441, normalized), 2048, 441, normalized)
    assert y.size == x.size and np.abs(y - x).max() < 1e-5


def test_htdemucs_round_trip_away_from_edges(oracle_mod):       # dsp_test.cpp:80-96
    rng = np.random.default_rng(7)
    f, p, a = rng.uniform(40, 0.4 * 44100, 24), rng.uniform(0, 2 * np.pi, 24), rng.uniform(0.02, 0.2, 24)
    n = 1024 * 60
    t = np.arange(n)
    x = (a[:, None] * np.sin(2 * np.pi * f[:, None] * t / 44100 + p[:, None])).sum(0).astype(np.float32)
    spec = oracle_mod.htdemucs_spec(x)
    y = oracle_mod.htdemucs_ispec(spec, n)
    assert spec.shape[1] == n // 1024
    assert np.abs(y[4096:-4096] - x[4096:-4096]).max() < 1e-6


@pytest.mark.parametrize("n", [320, 512, 640, 960, 2048, 7680])
def test_vrfft_impulse_and_inverse(oracle_mod, n):               # vr_dsp_test.cpp:8-15
    x = np.zeros(n, np.complex128)
    x[7] = 1
    X = _vr(oracle_mod, x)                                      # Bluestein at every size, as there
    k = np.arange(n)
    assert np.abs(X - np.exp(-2j * np.pi * 7 * k / n)).max() < 1e-10
    back = _vr(oracle_mod, X, inverse=True)
    assert np.abs(back / n - x).max() < 1e-10


def _vr(oracle_mod, x, inverse=False):
    a = np.ascontiguousarray(x, np.complex128).copy()
    assert oracle_mod.lib().or_vrfft(a.size, a.view(np.float64), int(inverse)) == 0
    return a


def test_identity_mask_gives_back_the_mix(oracle_mod, pkg):
    """RoFormer with every band mask 1+0i: the whole chunked path is the identity."""
    sizes, freqs = pkg.bands.mel_bands()
    chunk = 441 * 20
    for length in (441 * 70 + 3, 441 * 15):
        p = oracle_mod.rf_params(sizes, freqs, chunk=chunk, num_overlap=4)
        T = chunk // 441 + 1
        m = np.zeros((oracle_mod.rf_n_chunks(p, length), int(sizes.sum()) * 4 * T), np.float32)
        m[:, 0::2] = 1.0
        x = synth_audio(3, length)
        y = oracle_mod.rf_separate(p, x, m)
        assert np.abs(y[0] - x).max() < 1e-6


# ---- the input resampler (src/audio.h:17-56) ---------------------------------------------------
@pytest.mark.parametrize("src,dst", RESAMPLE_RATES)
def test_resampler_matches_golden(oracle_mod, golden, src, dst):
    got = oracle_mod.resample_planar(golden["io_resample_in"], src, dst)
    assert np.array_equal(got, golden[f"io_resample_{src}_{dst}"])


def test_resampler_bit_exact_vs_reference(oracle_mod):
    R = oracle_mod.ref_lib()
    if R is None:
        pytest.skip("reference not compiled on this machine")
    x = np.random.default_rng(3).uniform(-1, 1, (2, 20011)).astype(np.float32)
    for src, dst in [(48000, 44100), (96000, 44100), (11025, 44100)]:
        assert np.array_equal(oracle_mod.resample_planar(x, src, dst), oracle_mod.resample_planar(x, src, dst, impl=R))


def test_resampler_passes_a_low_tone(oracle_mod):
    """A 440 Hz tone survives 48 kHz -> 44.1 kHz: the sinc kernel's passband, away from the edges."""
    n = 48000
    x = np.sin(2 * np.pi * 440 * np.arange(n) / 48000).astype(np.float32)[None]
    y = oracle_mod.resample_planar(x, 48000, 44100)[0]
    want = np.sin(2 * np.pi * 440 * np.arange(y.size) / 44100)
    assert y.size == 44100 and np.abs(y[200:-200] - want[200:-200]).max() < 1e-3


# ---- VR (src/vr_dsp.h) ----------------------------------------------------------------------
@pytest.mark.parametrize("n", [320, 512, 640, 960, 2048])
def test_vr_stft_round_trip(oracle_mod, n):                     # vr_dsp_test.cpp:17-24
    samples = 3 * n
    k = np.arange(2 * samples)
    wave = (0.2 * np.sin(0.017 * k)).astype(np.float32).reshape(2, samples)
    spec = oracle_mod.vr_stft(wave, n, n // 2)
    back = oracle_mod.vr_istft(spec, n, n // 2)
    assert back.shape == wave.shape and np.abs(back - wave).max() < 1e-6


def test_vr_band_filter_edges(oracle_mod):                       # vr_dsp_test.cpp:26-27
    L = oracle_mod.lib()
    assert L.or_vr_lowpass(24, 25, 53) == 1 and L.or_vr_lowpass(52, 25, 53) == 0
    assert L.or_vr_highpass(85, 130, 85) == 0 and L.or_vr_highpass(86, 130, 85) == 0
    assert L.or_vr_highpass(131, 130, 85) == 1


def test_vr_polyphase_alignment(oracle_mod):                     # vr_dsp_test.cpp:28-33
    x = np.array([[0, 1, 0, 0], [0, 1, 0, 0]], np.float32)
    y = oracle_mod.vr_resample(x, 1, 2, np.array([0.5, 1, 0.5], np.float32))
    assert y.shape == (2, 8)
    assert np.array_equal(y.reshape(-1), np.array([0, .5, 1, .5, 0, 0, 0, 0, 0, .5, 1, .5, 0, 0, 0, 0], np.float32))


@pytest.mark.parametrize("nfft,hop", VR_STFTS)
def test_vr_primitives_match_golden(oracle_mod, golden, nfft, hop):
    spec = oracle_mod.vr_stft(golden["vr_wave_in"], nfft, hop)
    assert np.array_equal(spec, golden[f"vr_stft_{nfft}_{hop}"])
    assert np.array_equal(oracle_mod.vr_istft(spec, nfft, hop), golden[f"vr_istft_{nfft}_{hop}"])


@pytest.mark.parametrize("src,dst", VR_RESAMPLES)
def test_vr_resampler_matches_golden(oracle_mod, golden, src, dst):
    got = oracle_mod.vr_resample(golden["vr_wave_in"], src, dst, golden[f"vr_fir_{src}_{dst}"])
    assert np.array_equal(got, golden[f"vr_resample_{src}_{dst}"])


def test_vr_primitives_bit_exact_vs_reference(oracle_mod):
    R = oracle_mod.ref_lib()
    if R is None:
        pytest.skip("reference not compiled on this machine")
    w = np.random.default_rng(4).uniform(-1, 1, (2, 7001)).astype(np.float32)
    for nfft, hop in [(640, 80), (1024, 256), (960, 320)]:
        s = oracle_mod.vr_stft(w, nfft, hop)
        assert np.array_equal(s, oracle_mod.vr_stft(w, nfft, hop, impl=R))
        assert np.array_equal(oracle_mod.vr_istft(s, nfft, hop), oracle_mod.vr_istft(s, nfft, hop, impl=R))
    h = oracle_mod.vr_fir(14700, 44100)
    assert np.array_equal(oracle_mod.vr_resample(w, 14700, 44100, h), oracle_mod.vr_resample(w, 14700, 44100, h, impl=R))


def test_vr_separation_of_silence_is_silence(oracle_mod):
    """A zero peak returns zeros (src/vr.cpp:361)."""
    p = oracle_mod.vr_params([dict(sr=44100, hop=512, nfft=1024, start=0, stop=480)], bins=480, pre_start=0,
                             pre_stop=1)
    n = 20000
    T = oracle_mod.vr_n_frames(p, n)
    y = oracle_mod.vr_separate(p, np.zeros((2, n), np.float32), np.full((2, 481, T), 0.5, np.float32))
    assert not y.any()


# ---- random shifts (src/htdemucs.cpp:610-626, src/roformer.cpp:456-478) ----------------------
def _mt19937_raw(seed, n):
    """Raw 32-bit outputs of std::mt19937(seed): numpy's legacy RandomState seeds MT19937 by
    the same init_genrand, and a full-range 32-bit draw is one raw output."""
    return np.random.RandomState(seed).randint(0, 2**32, size=n, dtype=np.uint64)


def _bounded(raw, hi, count):
    """uniform_int_distribution<int>(0, hi) over 32-bit raw draws: Lemire's multiply-shift
    with rejection of the biased low products."""
    out, it, span = [], iter(raw), hi + 1
    while len(out) < count:
        prod = int(next(it)) * span
        if (prod & 0xFFFFFFFF) < span:
            threshold = (2**32 - span) % span
            while (prod & 0xFFFFFFFF) < threshold:
                prod = int(next(it)) * span
        out.append(prod >> 32)
    return out


@pytest.mark.parametrize("seed,shifts,hi", [(0, 5, 22050), (42, 3, 22049), (7, 10, 3999)])
def test_shift_offsets_are_the_standard_library_sequence(oracle_mod, seed, shifts, hi):
    got = oracle_mod.shift_offsets(seed, shifts, hi)
    assert list(got) == _bounded(_mt19937_raw(seed, 4 * shifts + 8), hi, shifts)
    assert all(0 <= o <= hi for o in got)


def _sines(length, channels=2, seed=5):
    rng = np.random.default_rng(seed)
    t = np.arange(length) / 44100.0
    return np.stack([(rng.uniform(0.05, 0.2, 6)[:, None] *
                      np.sin(2 * np.pi * rng.uniform(60, 4000, 6)[:, None] * t)).sum(0)
                     for _ in range(channels)]).astype(np.float32)


def test_htdemucs_shift_schedule(oracle_mod):
    """Every shift runs split() over a view of len + max_shift - offset samples, offset in
    [0, max_shift] (src/htdemucs.cpp:612-621): the segment count is the views' sum."""
    length, seg = 30000, 1024 * 12
    p = oracle_mod.ht_params(n_sources=2, segment=seg, shifts=4, seed=3, sample_rate=8000)
    stride = int(0.75 * seg)
    offs = oracle_mod.shift_offsets(3, 4, 4000)
    want = sum(-(-(length + 4000 - int(o)) // stride) for o in offs)
    assert oracle_mod.ht_n_segments(p, length) == want


def test_roformer_shift_average_of_identity_is_the_mix(oracle_mod, pkg):
    sizes, freqs = pkg.bands.mel_bands()
    chunk = 441 * 20
    p = oracle_mod.rf_params(sizes, freqs, chunk=chunk, num_overlap=4, shifts=3, seed=11, sample_rate=8000,
                             complement=1)
    length = 441 * 50 + 7
    T = chunk // 441 + 1
    m = np.zeros((oracle_mod.rf_n_chunks(p, length), int(sizes.sum()) * 4 * T), np.float32)
    m[:, 0::2] = 1.0
    x = synth_audio(4, length)
    y = oracle_mod.rf_separate(p, x, m)
    assert np.abs(y[0] - x).max() < 1e-5 and np.abs(y[1]).max() < 1e-5


# ---- 2. golden vectors from the reference ----------------------------------------------------
def test_primitives_match_golden(oracle_mod, golden):
    g = golden
    assert np.array_equal(oracle_mod.fft(g["prim_fft4096_in"]), g["prim_fft4096"])
    assert np.abs(_vr(oracle_mod, g["prim_vrfft7680_in"]) - g["prim_vrfft7680"]).max() < 1e-12
    s = oracle_mod.torch_stft(g["prim_stft_in"], 2048, 441)
    assert np.array_equal(s, g["prim_stft_2048_441"])
    assert np.array_equal(oracle_mod.torch_istft(s, 2048, 441), g["prim_istft_2048_441"])
    h = oracle_mod.htdemucs_spec(g["prim_hspec_in"])
    assert np.array_equal(h, g["prim_hspec_4096"])
    assert np.array_equal(oracle_mod.htdemucs_ispec(h, g["prim_hspec_in"].size), g["prim_hispec_4096"])


@pytest.mark.parametrize("name", sorted(CASES))
def test_separation_matches_golden(oracle_mod, golden, name):
    case = CASES[name]
    params, mix, mask = inputs_for(case)
    assert np.sum(mix, dtype=np.float64) == golden[f"{name}_mix_sum"], "input generator drifted"
    assert np.sum(mask, dtype=np.float64) == golden[f"{name}_mask_sum"], "input generator drifted"
    got = case["run"](params, mix, mask)
    want = golden[f"{name}_out"]
    assert got.shape == want.shape
    assert np.abs(got - want).max() <= 1e-6 * max(1.0, np.abs(want).max())


# ---- 3. the live reference --------------------------------------------------------------------
@pytest.fixture(scope="module")
def ref(oracle_mod):
    R = oracle_mod.ref_lib()
    if R is None:
        pytest.skip("reference not compiled on this machine")
    return R


def test_primitives_bit_exact_vs_reference(oracle_mod, ref):
    rng = np.random.default_rng(5)
    for n in (2048, 4096, 16384):
        x = rng.standard_normal(n) + 1j * rng.standard_normal(n)
        assert np.array_equal(oracle_mod.fft(x), oracle_mod.fft(x, impl=ref))
    for n in (320, 7680):
        x = rng.standard_normal(n) + 1j * rng.standard_normal(n)
        assert np.array_equal(_vr(oracle_mod, x), oracle_mod.fft(x, impl=ref))
    x = rng.uniform(-1, 1, 441 * 30 + 11).astype(np.float32)
    for nfft, hop in ((2048, 441), (7680, 1024)):
        s = oracle_mod.torch_stft(x, nfft, hop)
        assert np.array_equal(s, oracle_mod.torch_stft(x, nfft, hop, impl=ref))
        assert np.array_equal(oracle_mod.torch_istft(s, nfft, hop), oracle_mod.torch_istft(s, nfft, hop, impl=ref))
    h = oracle_mod.htdemucs_spec(x)
    assert np.array_equal(h, oracle_mod.htdemucs_spec(x, impl=ref))
    assert np.array_equal(oracle_mod.htdemucs_ispec(h, x.size), oracle_mod.htdemucs_ispec(h, x.size, impl=ref))


@pytest.mark.parametrize("name", ["rf_bs", "tfc_uvr"])
def test_separation_with_reference_primitives(oracle_mod, ref, name):
    case = CASES[name]
    params, mix, mask = inputs_for(case, seed=77)
    mine = case["run"](params, mix, mask)
    assert oracle_mod.use_reference(True)
    try:
        theirs = case["run"](params, mix, mask)
    finally:
        oracle_mod.use_reference(False)
    assert np.array_equal(mine, theirs)


# ---- band tables (tools/convert_roformer.py:107-124) ---------------------------------------
def test_band_tables(pkg):
    sizes, freqs = pkg.bands.mel_bands()
    bpf = pkg.bands.bands_per_freq(sizes, freqs, 1025)
    assert sizes.size == 60 and sizes.sum() == 1979 and sizes.min() == 6 and sizes.max() == 130
    assert bpf.min() == 1 and bpf.max() == 2
    bs, bf = pkg.bands.bs_bands()
    assert bs.size == 62 and bs.sum() == 1025 and list(bs[-2:]) == [128, 129]
    assert np.array_equal(bf, np.arange(1025))


# ---- HTDemucs bag of models (src/htdemucs.cpp:585-642) ------------------------------------------
def _bag_inputs(oracle_mod, n_models, seg=1024 * 12, length=30000, S=4):
    p1 = oracle_mod.ht_params(n_sources=S, segment=seg, threads=4)
    per_model = oracle_mod.ht_n_segments(p1, length) * S * 4 * 2048 * oracle_mod.ht_n_frames(p1)
    rng = np.random.default_rng(41)
    mix = (0.2 * rng.standard_normal((2, length))).astype(np.float32)
    mask = rng.standard_normal(n_models * per_model).astype(np.float32)
    return mix, mask, per_model


@pytest.mark.parametrize("mono", [0, 1])
def test_bag_one_hot_picks_each_models_stem(oracle_mod, mono):
    """htdemucs_ft's bag: four models, one-hot weights. Stem s is model s's stem s alone: the sum
    over the bag adds it to zero once and divides by 1, so it equals a one-model run bit for bit."""
    S, seg, length = 4, 1024 * 12, 30000
    mix, mask, per = _bag_inputs(oracle_mod, 4)
    p = oracle_mod.ht_params(n_sources=S, segment=seg, mono_norm=mono, cac_norm=1, threads=4,
                             bag_weights=np.eye(4))
    got = oracle_mod.ht_separate(p, mix, mask)
    for s in range(S):
        one = oracle_mod.ht_params(n_sources=S, segment=seg, mono_norm=mono, cac_norm=1, threads=4)
        want = oracle_mod.ht_separate(one, mix, mask[s * per:(s + 1) * per])
        np.testing.assert_array_equal(got[s], want[s])


def test_bag_weights_follow_the_reference_arithmetic(oracle_mod):
    """Arbitrary weights: float32 products summed in model order, divided by the float32 sum of
    the weights (then the mono inverse, off here), against the models' own one-model runs."""
    S, seg, length = 4, 1024 * 12, 30000
    w = np.array([[0.5, 1.0, 0.0, 2.0], [1.5, 0.25, 1.0, 0.0], [0.0, 3.0, 1.0, 1.0]], np.float32)
    mix, mask, per = _bag_inputs(oracle_mod, 3)
    p = oracle_mod.ht_params(n_sources=S, segment=seg, mono_norm=0, cac_norm=1, threads=4, bag_weights=w)
    got = oracle_mod.ht_separate(p, mix, mask)
    est = np.zeros((S, 2, length), np.float32)
    tot = np.zeros(S, np.float32)
    for m in range(3):
        one = oracle_mod.ht_params(n_sources=S, segment=seg, mono_norm=0, cac_norm=1, threads=4)
        res = oracle_mod.ht_separate(one, mix, mask[m * per:(m + 1) * per])
        for s in range(S):
            tot[s] = np.float32(tot[s] + w[m, s])
            if w[m, s] != 0:
                est[s] = (est[s] + (w[m, s] * res[s]).astype(np.float32)).astype(np.float32)
    want = (est / tot[:, None, None]).astype(np.float32)
    np.testing.assert_array_equal(got, want)
