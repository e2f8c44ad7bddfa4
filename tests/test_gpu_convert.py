"""The request-side conversions on the device against the oracle (src/libstems.cpp:160-199,
src/audio.h:17-68): interleaved/planar input, to_channels, the Kaiser-sinc resampler and the
length pin of the stems. The device does the reference's double arithmetic with explicitly
rounded operations, so the results are compared for equality, float for float."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n_channels,interleaved,sr", [
    (2, True, 48000),     # the usual request: interleaved stereo at 48 kHz
    (1, True, 22050),     # mono is duplicated
    (3, False, 44100),    # extra channels dropped, same rate: a copy
    (2, False, 96000),
])
def test_prepare_input(engine, oracle_mod, n_channels, interleaved, sr):
    import torch
    n = 48011
    x = np.random.default_rng(sr + n_channels).uniform(-1, 1, n * n_channels).astype(np.float32)
    got = engine.prepare_input(torch.from_numpy(x).cuda(), n_channels, sr, interleaved=interleaved)
    torch.cuda.synchronize()
    want = oracle_mod.prepare_input(x, interleaved, n_channels, sr, 2, 44100)
    assert got.shape == want.shape
    assert np.array_equal(got.cpu().numpy(), want)


@pytest.mark.parametrize("sr", [48000, 32000, 44100])
def test_restore_output(engine, oracle_mod, sr):
    import torch
    n = 30001                                   # the request's length at sr
    length = oracle_mod.resampled_length(n, sr, 44100)
    stems = np.random.default_rng(sr).uniform(-1, 1, (4, 2, length)).astype(np.float32)
    got = engine.restore_output(torch.from_numpy(stems).cuda(), 44100, sr, n)
    torch.cuda.synchronize()
    want = oracle_mod.restore_output(stems.reshape(8, length), 44100, sr, n)
    assert got.shape == (8, n)
    assert np.array_equal(got.cpu().numpy(), want)


def test_round_trip_keeps_a_tone(engine):
    """48 kHz -> 44.1 kHz -> 48 kHz keeps a 1 kHz tone away from the edges."""
    import torch
    n = 48000
    x = (0.5 * np.sin(2 * np.pi * 1000 * np.arange(n) / 48000)).astype(np.float32)
    d = engine.prepare_input(torch.from_numpy(np.repeat(x, 2)).cuda(), 2, 48000)
    back = engine.restore_output(d, 44100, 48000, n).cpu().numpy()
    assert np.abs(back[:, 500:-500] - x[500:-500]).max() < 2e-3
