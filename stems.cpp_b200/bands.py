"""RoFormer band tables (the roformer.band_sizes / roformer.band_freqs GGUF metadata).

The reference reads these int32 lists from the model file (src/roformer.cpp:394-411); its
converter writes them (tools/convert_roformer.py:107-124, 238-239). This module rebuilds the
same lists without a model file so the spectral path can be configured and benchmarked:

* ``bs_bands``: BS-RoFormer's contiguous ``freqs_per_bands`` (convert_roformer.py:118-124).
* ``mel_bands``: MelBandRoformer's binarised mel filterbank (convert_roformer.py:107-115),
  which the converter takes from librosa ``filters.mel`` (Slaney mel scale, Slaney area
  normalisation, fmin 0, fmax sr/2). librosa is not installed here, so the filterbank is
  restated from its published formula; only the sign of each weight matters (``fb > 0``),
  and the first and last weights are forced to 1 exactly as the converter does.
"""
from __future__ import annotations

import numpy as np

# BS-RoFormer (viperx 317 and the MSST defaults): 62 bands over the 1025 bins of n_fft 2048.
BS_ROFORMER_FREQS_PER_BANDS = ((2,) * 24 + (4,) * 12 + (12,) * 8 + (24,) * 8 + (48,) * 8
                               + (128, 129))


def bs_bands(freqs_per_bands=BS_ROFORMER_FREQS_PER_BANDS, n_fft=2048):
    """Contiguous bands as (band_sizes, band_freqs) int32 arrays."""
    sizes = np.asarray(freqs_per_bands, dtype=np.int32)
    if int(sizes.sum()) != n_fft // 2 + 1:
        raise ValueError(f"freqs_per_bands sum to {int(sizes.sum())}, not {n_fft // 2 + 1}")
    return sizes, np.arange(n_fft // 2 + 1, dtype=np.int32)


def _hz_to_mel(f):
    # Slaney: linear below 1 kHz (200/3 Hz per mel), logarithmic above.
    f = np.asarray(f, dtype=np.float64)
    f_sp = 200.0 / 3
    mels = f / f_sp
    min_log_hz, min_log_mel, logstep = 1000.0, 1000.0 / f_sp, np.log(6.4) / 27.0
    return np.where(f >= min_log_hz,
                    min_log_mel + np.log(np.maximum(f, 1e-300) / min_log_hz) / logstep, mels)


def _mel_to_hz(m):
    m = np.asarray(m, dtype=np.float64)
    f_sp = 200.0 / 3
    freqs = f_sp * m
    min_log_hz, min_log_mel, logstep = 1000.0, 1000.0 / f_sp, np.log(6.4) / 27.0
    return np.where(m >= min_log_mel, min_log_hz * np.exp(logstep * (m - min_log_mel)), freqs)


def mel_filterbank(sr=44100, n_fft=2048, n_mels=60):
    """Triangular Slaney mel filters [n_mels][n_fft/2 + 1] with Slaney area normalisation."""
    fftfreqs = np.linspace(0.0, sr / 2.0, 1 + n_fft // 2)
    mel_f = _mel_to_hz(np.linspace(_hz_to_mel(0.0), _hz_to_mel(sr / 2.0), n_mels + 2))
    fdiff = np.diff(mel_f)
    ramps = np.subtract.outer(mel_f, fftfreqs)
    w = np.zeros((n_mels, 1 + n_fft // 2), dtype=np.float64)
    for i in range(n_mels):
        lower = -ramps[i] / fdiff[i]
        upper = ramps[i + 2] / fdiff[i + 1]
        w[i] = np.maximum(0.0, np.minimum(lower, upper))
    enorm = 2.0 / (mel_f[2:n_mels + 2] - mel_f[:n_mels])
    return (w * enorm[:, None]).astype(np.float32)


def mel_bands(sr=44100, n_fft=2048, n_mels=60):
    """MelBandRoformer's band lists as (band_sizes, band_freqs) int32 arrays."""
    fb = mel_filterbank(sr, n_fft, n_mels)
    fb[0][0] = 1.0
    fb[-1, -1] = 1.0
    mask = fb > 0
    if not mask.any(axis=0).all():
        raise ValueError("every frequency must be covered by a band")
    rows = [np.nonzero(r)[0] for r in mask]
    sizes = np.array([r.size for r in rows], dtype=np.int32)
    return sizes, np.concatenate(rows).astype(np.int32)


def bands_per_freq(sizes, freqs, n_bins):
    """How many bands cover each bin (src/roformer.cpp:399, 408-411)."""
    bpf = np.zeros(n_bins, dtype=np.int32)
    np.add.at(bpf, np.asarray(freqs), 1)
    return bpf
