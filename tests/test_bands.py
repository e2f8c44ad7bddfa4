"""The RoFormer band tables against an independent implementation (CPU only).

The reference's converter builds the Mel-Band RoFormer table from librosa's filters.mel
(tools/convert_roformer.py:107-115): Slaney mel scale, Slaney area normalisation, fmin 0,
fmax sr/2, the first and last weights forced to 1, then ``fb > 0`` per band. librosa is not
installed here; torchaudio's melscale_fbanks with norm="slaney", mel_scale="slaney" computes
the same filterbank, so it pins bands.mel_bands() without our own formula on both sides.
"""
from __future__ import annotations

import numpy as np
import pytest


def _torchaudio_mel_bands(sr, n_fft, n_mels):
    ta = pytest.importorskip("torchaudio")
    fb = ta.functional.melscale_fbanks(n_fft // 2 + 1, 0.0, sr / 2.0, n_mels, sr, norm="slaney",
                                       mel_scale="slaney").numpy().T.copy()   # [n_mels][bins]
    fb[0][0] = 1.0                                                          # convert_roformer.py:111
    fb[-1, -1] = 1.0                                                        # :112
    mask = fb > 0
    assert mask.any(axis=0).all()
    rows = [np.nonzero(r)[0] for r in mask]
    return np.array([r.size for r in rows], np.int32), np.concatenate(rows).astype(np.int32)


@pytest.mark.parametrize("sr,n_fft,n_mels", [(44100, 2048, 60), (44100, 2048, 64), (44100, 4096, 60),
                                             (48000, 2048, 60)])
def test_mel_bands_match_torchaudio_slaney(pkg, sr, n_fft, n_mels):
    sizes, freqs = pkg.bands.mel_bands(sr=sr, n_fft=n_fft, n_mels=n_mels)
    want_sizes, want_freqs = _torchaudio_mel_bands(sr, n_fft, n_mels)
    np.testing.assert_array_equal(sizes, want_sizes)
    np.testing.assert_array_equal(freqs, want_freqs)


def test_mel_bands_kim_shape(pkg):
    """The Kim Mel-Band RoFormer table the benchmark uses: 60 bands, 1979 (band, bin) entries,
    every bin covered, no bin in more than two bands."""
    sizes, freqs = pkg.bands.mel_bands()
    assert sizes.size == 60 and int(sizes.sum()) == freqs.size == 1979
    bpf = pkg.bands.bands_per_freq(sizes, freqs, 1025)
    assert bpf.min() == 1 and bpf.max() == 2


def test_bs_bands_viperx():
    """BS-RoFormer viperx 317: 62 contiguous bands over 1025 bins, the last taking 129."""
    import __graft_entry__
    b = __graft_entry__.load_package().bands
    sizes, freqs = b.bs_bands()
    assert sizes.size == 62 and int(sizes.sum()) == 1025 and sizes[-1] == 129
    np.testing.assert_array_equal(freqs, np.arange(1025))
