"""One track over several devices in one process (stg_separate_multi_host): plan d writes the
d-th range of output samples from the chunks that reach it, one host thread per device.

Every range is the floats one device writes for the whole track, so the result must equal
stg_separate_host's bit for bit. With one GPU the parts run on engines of the same device
(the split, the per-range mask copies and the threads are the same code); with more, on
distinct devices."""
from __future__ import annotations

import numpy as np
import pytest

from common import synth_audio, synth_mask

pytestmark = pytest.mark.gpu


def _plans(pkg, devices, make):
    engines = [pkg.Engine(d) for d in devices]
    return engines, [make(e) for e in engines]


def _check_parts(pkg, devices, make, seed):
    engines, plans = _plans(pkg, devices, make)
    p0 = plans[0]
    mix = synth_audio(seed, p0.n_samples, channels=p0.n_channels)
    mask = synth_mask(seed + 1, p0.mask_floats, 0.5)
    whole = p0.separate_host(mix, mask)
    out = np.full(p0.out_shape, np.nan, np.float32)
    pkg.separate_multi_host(plans, mix, mask, out)
    np.testing.assert_array_equal(out, whole)
    for p in plans:
        p.close()
    for e in engines:
        e.close()


@pytest.mark.parametrize("parts", [2, 3])
def test_roformer_parts_on_one_device(pkg, parts):
    sizes, freqs = pkg.bands.bs_bands()
    n = 441 * 150 + 77
    _check_parts(pkg, [0] * parts, lambda e: e.plan_roformer(n, sizes, freqs, chunk=441 * 40, num_overlap=2,
                                                              zero_dc=True, complement=True), 91)


def test_htdemucs_bag_parts_on_one_device(pkg):
    w = np.array([[1.0, 0.5, 1.0, 1.0], [0.5, 1.0, 2.0, 1.0]], np.float32)
    _check_parts(pkg, [0, 0], lambda e: e.plan_htdemucs(70000, segment=1024 * 24, bag_weights=w), 93)


def test_tfc_parts_on_one_device(pkg):
    _check_parts(pkg, [0, 0, 0], lambda e: e.plan_tfc(90001, dim_t=32, overlap=0.5, complement=True), 95)


def test_parts_across_devices(pkg):
    n_dev = pkg.device_count()
    if n_dev < 2:
        pytest.skip("one device visible")
    sizes, freqs = pkg.bands.mel_bands()
    n = 441 * 200
    _check_parts(pkg, list(range(min(n_dev, 4))),
                 lambda e: e.plan_roformer(n, sizes, freqs, chunk=441 * 40, num_overlap=4), 97)


def test_plans_must_match(pkg):
    e1, e2 = pkg.Engine(0), pkg.Engine(0)
    sizes, freqs = pkg.bands.bs_bands()
    a = e1.plan_roformer(441 * 100, sizes, freqs, chunk=441 * 40)
    b = e2.plan_roformer(441 * 101, sizes, freqs, chunk=441 * 40)
    mix = synth_audio(1, 441 * 100)
    with pytest.raises(pkg.StemsError):
        pkg.separate_multi_host([a, b], mix, np.zeros(a.mask_floats, np.float32))
    with pytest.raises(pkg.StemsError):   # one engine, two parts
        pkg.separate_multi_host([a, e1.plan_roformer(441 * 100, sizes, freqs, chunk=441 * 40)], mix,
                                np.zeros(a.mask_floats, np.float32))
