"""The VR spectral path on the device (src/vr.cpp:215-269, 349-377; src/vr_dsp.h) against the
oracle, with the network replaced by a given mask [2][bins+1][T].

The band layouts are made up for the test but obey the reference's model checks
(src/vr.cpp:296-327; equal frame durations, crops within bins, filters in range): one band
at n_fft 2048 / hop 1024, and multi-band layouts crossing 11.025/22.05/44.1 kHz and
7.35/14.7/44.1 kHz with the FFT sizes 320, 512, 640, 960 and 1024. The resampling FIRs are
designed as the reference's converter designs them (oracle.vr_fir). Tolerance: per stem,
max |got - ref| / max |ref| <= 1e-5 (the oracle runs in double, the device in float)."""
from __future__ import annotations

import numpy as np
import pytest

from common import max_rel_err, synth_audio

pytestmark = pytest.mark.gpu

TOL = 1e-5

LAYOUTS = {
    "1band_2048": dict(bins=1024, pre=(0, 1), bands=[
        dict(sr=44100, hop=1024, nfft=2048, start=0, stop=1024)]),
    "3band_640_960_1024": dict(bins=832, pre=(700, 832), bands=[
        dict(sr=11025, hop=128, nfft=640, start=0, stop=200, lp_start=150, lp_stop=200),
        dict(sr=22050, hop=256, nfft=960, start=100, stop=400, hp_start=120, hp_stop=100, lp_start=350,
             lp_stop=400),
        dict(sr=44100, hop=512, nfft=1024, start=200, stop=513, hp_start=230, hp_stop=210)]),
    "3band_320_512_960": dict(bins=608, pre=(500, 600), bands=[
        dict(sr=7350, hop=80, nfft=320, start=0, stop=100, lp_start=80, lp_stop=100),
        dict(sr=14700, hop=160, nfft=512, start=50, stop=200, hp_start=60, hp_stop=50, lp_start=180,
             lp_stop=200),
        dict(sr=44100, hop=480, nfft=960, start=150, stop=481, hp_start=170, hp_stop=150)]),
}


def _plan(engine, oracle_mod, layout, n):
    L = LAYOUTS[layout]
    p = oracle_mod.vr_params(L["bands"], bins=L["bins"], pre_start=L["pre"][0], pre_stop=L["pre"][1])
    rates = sorted({b["sr"] for b in L["bands"]})
    firs = {(s, d): oracle_mod.vr_fir(s, d) for s in rates for d in rates if s != d}
    bands = [dict(sample_rate=b["sr"], hop=b["hop"], n_fft=b["nfft"], crop_start=b["start"], crop_stop=b["stop"],
                  hpf_start=b.get("hp_start", -1), hpf_stop=b.get("hp_stop", -1), lpf_start=b.get("lp_start", -1),
                  lpf_stop=b.get("lp_stop", -1)) for b in L["bands"]]
    plan = engine.plan_vr(n, bands, firs, bins=L["bins"], pre_filter_start=L["pre"][0], pre_filter_stop=L["pre"][1])
    return plan, p


@pytest.mark.parametrize("layout", sorted(LAYOUTS))
def test_vr_matches_oracle(engine, oracle_mod, layout):
    import torch
    n = 44100 * 3 + 113
    plan, p = _plan(engine, oracle_mod, layout, n)
    assert plan.n_frames == oracle_mod.vr_n_frames(p, n)
    mix = synth_audio(81, n)
    mask = np.random.default_rng(82).uniform(0, 1, plan.mask_shape).astype(np.float32)
    out = torch.empty(plan.out_shape, device="cuda")
    plan.separate(torch.from_numpy(mix).cuda(), torch.from_numpy(mask).cuda(), out)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    want = oracle_mod.vr_separate(p, mix, mask)
    for s in range(2):
        assert max_rel_err(got[s], want[s]) <= TOL, f"{layout} stem {s}"


def test_vr_front_gives_the_network_input(engine, oracle_mod):
    """|spec| and its peak: the stems of the mask 1 and 0 agree with the two-call form."""
    import torch
    n = 44100 * 2 + 7
    plan, p = _plan(engine, oracle_mod, "3band_640_960_1024", n)
    d_mix = torch.from_numpy(synth_audio(83, n)).cuda()
    mag = torch.empty(plan.mask_shape, device="cuda")
    peak = torch.zeros(1, device="cuda")
    plan.front(d_mix, mag, peak)
    torch.cuda.synchronize()
    m = mag.cpu().numpy()
    assert (m >= 0).all() and float(peak.item()) == float(m.max()) and m.max() > 0
    mask = torch.from_numpy(np.random.default_rng(84).uniform(0, 1, plan.mask_shape).astype(np.float32)).cuda()
    a = torch.empty(plan.out_shape, device="cuda")
    plan.back(mask, a)
    b = torch.empty(plan.out_shape, device="cuda")
    plan.separate(d_mix, mask, b)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_vr_silence(engine, oracle_mod):
    import torch
    n = 30000
    plan, _ = _plan(engine, oracle_mod, "1band_2048", n)
    out = torch.full(plan.out_shape, 7.0, device="cuda")
    plan.separate(torch.zeros((2, n), device="cuda"), torch.full(plan.mask_shape, 0.3, device="cuda"), out)
    torch.cuda.synchronize()
    assert not out.any()


def test_vr_rejects_bad_layouts(engine, pkg):
    """The reference's model checks: frame durations must agree, the last band runs at the
    model rate, crops fit in bins."""
    good = dict(sample_rate=44100, hop=512, n_fft=1024, crop_start=0, crop_stop=400)
    with pytest.raises(pkg.StemsError):   # 22.05 kHz with the same hop: a different duration
        engine.plan_vr(30000, [dict(good, sample_rate=22050), good], {}, bins=800)
    with pytest.raises(pkg.StemsError):   # last band not at the model rate
        engine.plan_vr(30000, [dict(good, sample_rate=22050, hop=256)], {}, bins=416)
    with pytest.raises(pkg.StemsError):   # crops larger than bins
        engine.plan_vr(30000, [good], {}, bins=384)
