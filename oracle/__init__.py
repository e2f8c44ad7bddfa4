"""Python bindings for the CPU checker (oracle/liboracle.so). TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs
import this package, and only as the checker or as the timed CPU baseline. The product
(stems.cpp_b200) never imports it.

The C restatement follows the reference's src/stft.h, src/vr_dsp.h, src/htdemucs.cpp,
src/roformer.cpp and src/tfc_tdf.cpp line by line (see oracle.c). ``use_reference()`` swaps
its DSP primitives for the reference's own compiled code (oracle/_ref/libstems_ref.so).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libstems_ref.so")

_lib = None
_ref = None

_F32 = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_F64 = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_I32P = C.POINTER(C.c_int)


class HtParams(C.Structure):
    _fields_ = [("n_channels", C.c_int), ("n_sources", C.c_int), ("segment", C.c_int),
                ("overlap", C.c_float), ("cac_norm", C.c_int), ("mono_norm", C.c_int),
                ("sample_first", C.c_int), ("sample_count", C.c_int), ("threads", C.c_int),
                ("shifts", C.c_int), ("seed", C.c_uint), ("sample_rate", C.c_int),
                ("n_models", C.c_int), ("bag", C.POINTER(C.c_float))]


class RfParams(C.Structure):
    _fields_ = [("n_channels", C.c_int), ("n_stems", C.c_int), ("n_fft", C.c_int),
                ("hop", C.c_int), ("normalized", C.c_int), ("zero_dc", C.c_int),
                ("chunk", C.c_int), ("step", C.c_int), ("n_bands", C.c_int),
                ("band_sizes", _I32P), ("band_freqs", _I32P), ("complement", C.c_int),
                ("sample_first", C.c_int), ("sample_count", C.c_int), ("threads", C.c_int),
                ("shifts", C.c_int), ("seed", C.c_uint), ("sample_rate", C.c_int)]


class TfcParams(C.Structure):
    _fields_ = [("n_stems", C.c_int), ("n_fft", C.c_int), ("hop", C.c_int), ("dim_f", C.c_int),
                ("dim_t", C.c_int), ("zero_bins", C.c_int), ("chunking", C.c_int),
                ("overlap", C.c_float), ("num_overlap", C.c_int), ("compensate", C.c_float),
                ("complement", C.c_int), ("sample_first", C.c_int), ("sample_count", C.c_int),
                ("threads", C.c_int)]


class VrBand(C.Structure):
    _fields_ = [(k, C.c_int) for k in ("sr", "hop", "nfft", "start", "stop", "hp_start", "hp_stop",
                                      "lp_start", "lp_stop")]


class VrFir(C.Structure):
    _fields_ = [("src", C.c_int), ("dst", C.c_int), ("n_taps", C.c_int), ("taps", C.POINTER(C.c_float))]


class VrParams(C.Structure):
    _fields_ = [("sample_rate", C.c_int), ("bins", C.c_int), ("pre_start", C.c_int), ("pre_stop", C.c_int),
                ("n_bands", C.c_int), ("bands", C.POINTER(VrBand)), ("n_firs", C.c_int),
                ("firs", C.POINTER(VrFir))]


def build(force: bool = False) -> None:
    """Compile oracle.c (and the reference shim when the reference sources exist)."""
    if force or not os.path.exists(LIB_PATH):
        subprocess.run(["bash", os.path.join(HERE, "build.sh")], check=True,
                       stdout=subprocess.DEVNULL)


def lib():
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(LIB_PATH)
        L.or_fft.argtypes = [C.c_int, _F64, C.c_int]
        L.or_vrfft.argtypes = [C.c_int, _F64, C.c_int]
        L.or_torch_stft.argtypes = [C.c_int, _F32, C.c_int, C.c_int, C.c_int, _F64, _I32P]
        L.or_torch_istft.argtypes = [C.c_int, _F64, C.c_int, C.c_int, C.c_int, _F32]
        L.or_htdemucs_spec.argtypes = [C.c_int, _F32, C.c_int, _F64, _I32P]
        L.or_htdemucs_ispec.argtypes = [C.c_int, _F64, C.c_int, C.c_int, _F32]
        L.or_use_reference.argtypes = [C.c_char_p]
        L.or_shift_offsets.argtypes = [C.c_uint, C.c_int, C.c_int, _I32P]
        L.or_vr_stft.argtypes = [_F32, C.c_int, C.c_int, C.c_int, _F64, _I32P]
        L.or_vr_istft.argtypes = [_F64, C.c_int, C.c_int, C.c_int, _F32]
        L.or_vr_resampled_length.argtypes = [C.c_int, C.c_int, C.c_int]
        L.or_vr_resample.argtypes = [_F32, C.c_int, C.c_int, C.c_int, _F32, C.c_int, _F32]
        L.or_vr_lowpass.restype = C.c_float
        L.or_vr_lowpass.argtypes = [C.c_int, C.c_int, C.c_int]
        L.or_vr_highpass.restype = C.c_float
        L.or_vr_highpass.argtypes = [C.c_int, C.c_int, C.c_int]
        L.or_vr_n_frames.argtypes = [C.POINTER(VrParams), C.c_int]
        L.or_vr_separate.argtypes = [C.POINTER(VrParams), _F32, C.c_int, _F32, _F32]
        L.or_resampled_length.restype = C.c_longlong
        L.or_resampled_length.argtypes = [C.c_longlong, C.c_int, C.c_int]
        L.or_resample_planar.argtypes = [_F32, C.c_int, C.c_int, C.c_int, C.c_int, _F32, _I32P]
        L.or_ht_n_segments.argtypes = [C.POINTER(HtParams), C.c_int]
        L.or_ht_n_frames.argtypes = [C.POINTER(HtParams)]
        L.or_ht_separate.argtypes = [C.POINTER(HtParams), _F32, C.c_int, _F32, _F32]
        L.or_rf_n_chunks.argtypes = [C.POINTER(RfParams), C.c_int]
        L.or_rf_separate.argtypes = [C.POINTER(RfParams), _F32, C.c_int, _F32, _F32]
        L.or_rf_band_gather.argtypes = [C.POINTER(RfParams), _F64, C.c_int, _F32]
        L.or_tfc_n_chunks.argtypes = [C.POINTER(TfcParams), C.c_int]
        L.or_tfc_separate.argtypes = [C.POINTER(TfcParams), _F32, C.c_int, _F32, _F32]
        _lib = L
    return _lib


def reference_available() -> bool:
    return os.path.exists(REF_PATH)


def use_reference(on: bool = True) -> bool:
    """Route the glue's DSP primitives through the reference's compiled stft.h/vr_dsp.h."""
    L = lib()
    if not on:
        L.or_use_reference(None)
        return True
    if not reference_available():
        return False
    return L.or_use_reference(REF_PATH.encode()) == 0


def ref_lib():
    """The reference shim itself (ref_fft, ref_torch_stft, ...), or None when not built."""
    global _ref
    if _ref is None and reference_available():
        R = C.CDLL(REF_PATH)
        R.ref_fft.argtypes = [C.c_int, _F64, C.c_int]
        R.ref_vrfft.argtypes = [C.c_int, _F64, C.c_int]
        R.ref_torch_stft.argtypes = [C.c_int, _F32, C.c_int, C.c_int, C.c_int, _F64, _I32P]
        R.ref_torch_istft.argtypes = [C.c_int, _F64, C.c_int, C.c_int, C.c_int, _F32]
        R.ref_htdemucs_spec.argtypes = [C.c_int, _F32, C.c_int, _F64, _I32P]
        R.ref_htdemucs_ispec.argtypes = [C.c_int, _F64, C.c_int, C.c_int, _F32]
        R.ref_resample_planar.argtypes = [_F32, C.c_int, C.c_int, C.c_int, C.c_int, _F32, _I32P]
        R.ref_vr_stft.argtypes = [_F32, C.c_int, C.c_int, C.c_int, _F64, _I32P]
        R.ref_vr_istft.argtypes = [_F64, C.c_int, C.c_int, C.c_int, _F32]
        R.ref_vr_resample.argtypes = [_F32, C.c_int, C.c_int, C.c_int, _F32, C.c_int, _F32]
        _ref = R
    return _ref


def _check(rc, what):
    if rc != 0:
        raise ValueError(f"oracle: {what} failed ({rc})")


# ---- primitives -------------------------------------------------------------------------
def fft(x, inverse=False, impl=None):
    a = np.ascontiguousarray(x, dtype=np.complex128).copy()
    n = a.size
    L = impl or lib()
    pow2 = n >= 2 and not (n & (n - 1))
    f = (L.ref_fft if impl is not None else L.or_fft) if pow2 else (
        L.ref_vrfft if impl is not None else L.or_vrfft)
    _check(f(n, a.view(np.float64), int(inverse)), "fft")
    return a


def torch_stft(x, n_fft, hop, normalized=False, impl=None):
    x = np.ascontiguousarray(x, dtype=np.float32)
    T = x.size // hop + 1
    F = n_fft // 2 + 1
    out = np.zeros(F * T, np.complex128)
    nf = C.c_int(0)
    f = impl.ref_torch_stft if impl is not None else lib().or_torch_stft
    _check(f(n_fft, x, x.size, hop, int(normalized), out.view(np.float64), C.byref(nf)), "torch_stft")
    return out.reshape(F, T)


def torch_istft(spec, n_fft, hop, normalized=False, impl=None):
    spec = np.ascontiguousarray(spec, dtype=np.complex128)
    T = spec.shape[1]
    out = np.zeros(hop * (T - 1), np.float32)
    f = impl.ref_torch_istft if impl is not None else lib().or_torch_istft
    _check(f(n_fft, spec.reshape(-1).view(np.float64), T, hop, int(normalized), out), "torch_istft")
    return out


def htdemucs_spec(x, n_fft=4096, impl=None):
    x = np.ascontiguousarray(x, dtype=np.float32)
    hl = n_fft // 4
    T = (x.size + hl - 1) // hl
    out = np.zeros((n_fft // 2) * T, np.complex128)
    nf = C.c_int(0)
    f = impl.ref_htdemucs_spec if impl is not None else lib().or_htdemucs_spec
    _check(f(n_fft, x, x.size, out.view(np.float64), C.byref(nf)), "htdemucs_spec")
    return out.reshape(n_fft // 2, T)


def htdemucs_ispec(spec, length, n_fft=4096, impl=None):
    spec = np.ascontiguousarray(spec, dtype=np.complex128)
    out = np.zeros(length, np.float32)
    f = impl.ref_htdemucs_ispec if impl is not None else lib().or_htdemucs_ispec
    _check(f(n_fft, spec.reshape(-1).view(np.float64), spec.shape[1], length, out), "htdemucs_ispec")
    return out


# ---- the request's audio in and the stems out ----------------------------------------------
def resampled_length(n, src_rate, dst_rate):
    return int(lib().or_resampled_length(n, src_rate, dst_rate))


def resample_planar(x, src_rate, dst_rate, impl=None):
    """audio.h resample_planar of planar x [ch][n] -> [ch][out_n]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    ch, n = x.shape
    m = resampled_length(n, src_rate, dst_rate)
    out = np.zeros(ch * m, np.float32)
    got = C.c_int(0)
    f = impl.ref_resample_planar if impl is not None else lib().or_resample_planar
    _check(f(x.reshape(-1), n, ch, src_rate, dst_rate, out, C.byref(got)), "resample_planar")
    assert got.value == m
    return out.reshape(ch, m)


def to_channels(x, want):
    """audio.h to_channels: mono duplicated, extra channels dropped (planar [ch][n])."""
    ch = x.shape[0]
    return np.stack([x[0 if ch == 1 else min(c, ch - 1)] for c in range(want)])


def prepare_input(samples, interleaved, n_channels, sample_rate, model_channels, model_rate, impl=None):
    """libstems.cpp:160-169: interleaved/planar -> planar, to_channels, resample."""
    s = np.asarray(samples, np.float32).reshape(-1)
    n = s.size // n_channels
    planar = s.reshape(n, n_channels).T.copy() if interleaved else s.reshape(n_channels, n)
    return resample_planar(to_channels(planar, model_channels), sample_rate, model_rate, impl=impl)


def restore_output(stems, model_rate, sample_rate, n_samples, impl=None):
    """libstems.cpp:189-199: stems [rows][len] back to the request's rate, pinned to n_samples."""
    if model_rate == sample_rate:
        return np.asarray(stems, np.float32)
    y = resample_planar(stems, model_rate, sample_rate, impl=impl)
    out = np.zeros((y.shape[0], n_samples), np.float32)
    k = min(n_samples, y.shape[1])
    out[:, :k] = y[:, :k]
    return out


# ---- VR (src/vr_dsp.h, src/vr.cpp) ------------------------------------------------------------
def vr_stft(wave, nfft, hop, impl=None):
    """vr_stft of stereo wave [2][n]: complex128 [2][nfft/2+1][n/hop+1] (complex64 values)."""
    wave = np.ascontiguousarray(wave, np.float32)
    n = wave.shape[1]
    frames = n // hop + 1
    out = np.zeros(2 * (nfft // 2 + 1) * frames, np.complex128)
    got = C.c_int(0)
    f = impl.ref_vr_stft if impl is not None else lib().or_vr_stft
    _check(f(wave.reshape(-1), n, nfft, hop, out.view(np.float64), C.byref(got)), "vr_stft")
    return out.reshape(2, nfft // 2 + 1, frames)


def vr_istft(spec, nfft, hop, impl=None):
    spec = np.ascontiguousarray(spec, np.complex128)
    frames = spec.shape[2]
    out = np.zeros(2 * hop * (frames - 1), np.float32)
    f = impl.ref_vr_istft if impl is not None else lib().or_vr_istft
    _check(f(spec.reshape(-1).view(np.float64), frames, nfft, hop, out), "vr_istft")
    return out.reshape(2, -1)


def vr_resample(x, src, dst, fir, impl=None):
    x = np.ascontiguousarray(x, np.float32)
    fir = np.ascontiguousarray(fir, np.float32)
    n = x.shape[1]
    m = lib().or_vr_resampled_length(n, src, dst)
    out = np.zeros(2 * m, np.float32)
    f = impl.ref_vr_resample if impl is not None else lib().or_vr_resample
    _check(f(x.reshape(-1), n, src, dst, fir, fir.size, out), "vr_resample")
    return out.reshape(2, m)


def vr_fir(src, dst):
    """The model's resampling FIR as the reference's converter designs it (tools/convert_vr.py:
    199-211): scipy.signal.firwin(20*m + 1, 1/m, kaiser 5.0) * up, float32."""
    from math import gcd
    from scipy.signal import firwin
    g = gcd(src, dst)
    up, down = dst // g, src // g
    m = max(up, down)
    return (firwin(20 * m + 1, 1.0 / m, window=("kaiser", 5.0)).astype(np.float32) * up).astype(np.float32)


def vr_params(bands, sample_rate=44100, bins=None, pre_start=0, pre_stop=0):
    """bands: dicts with sr, hop, nfft, start, stop and optional hp_start/hp_stop/lp_start/lp_stop
    (-1 when absent), lowest rate first. The FIRs of every rate pair come from vr_fir."""
    bl = (VrBand * len(bands))()
    for i, b in enumerate(bands):
        bl[i] = VrBand(b["sr"], b["hop"], b["nfft"], b["start"], b["stop"], b.get("hp_start", -1),
                       b.get("hp_stop", -1), b.get("lp_start", -1), b.get("lp_stop", -1))
    rates = sorted({b["sr"] for b in bands} | {sample_rate})
    keep, firs = [], []
    for s in rates:
        for d in rates:
            if s != d:
                h = vr_fir(s, d)
                keep.append(h)
                firs.append(VrFir(s, d, h.size, h.ctypes.data_as(C.POINTER(C.c_float))))
    fl = (VrFir * max(1, len(firs)))(*firs)
    if bins is None:
        bins = sum(b["stop"] - b["start"] for b in bands)
    p = VrParams(sample_rate, bins, pre_start, pre_stop, len(bands), bl, len(firs), fl)
    p._keep = (bl, fl, keep, bands)
    return p


def vr_n_frames(p, length):
    return lib().or_vr_n_frames(C.byref(p), length)


def vr_separate(p, mix, mask):
    mix = np.ascontiguousarray(mix, np.float32)
    n = mix.shape[1]
    out = np.zeros(4 * n, np.float32)
    _check(lib().or_vr_separate(C.byref(p), mix.reshape(-1), n, np.ascontiguousarray(mask, np.float32).reshape(-1),
                                out), "vr_separate")
    return out.reshape(2, 2, n)


# ---- glue --------------------------------------------------------------------------------
def ht_params(n_channels=2, n_sources=4, segment=343980, overlap=-1.0, cac_norm=0, mono_norm=0,
              sample_first=0, sample_count=0, threads=1, shifts=0, seed=0, sample_rate=44100, n_models=1,
              bag_weights=None):
    p = HtParams(n_channels, n_sources, segment, overlap, cac_norm, mono_norm, sample_first,
                 sample_count, threads, shifts, seed, sample_rate, n_models)
    if bag_weights is not None:
        w = np.ascontiguousarray(bag_weights, dtype=np.float32).reshape(-1)
        p.n_models = w.size // n_sources
        p.bag = w.ctypes.data_as(C.POINTER(C.c_float))
        p._bag = w   # keeps the weights alive with the struct
    return p


def shift_offsets(seed, shifts, hi):
    """The separators' random-shift offsets (std::mt19937 + uniform_int_distribution(0, hi))."""
    out = np.zeros(max(shifts, 1), dtype=np.int32)
    if lib().or_shift_offsets(seed, shifts, hi, out.ctypes.data_as(_I32P)) != 0:
        raise ValueError("bad shift arguments")
    return out[:shifts].copy()


def ht_n_segments(p, length):
    return lib().or_ht_n_segments(C.byref(p), length)


def ht_n_frames(p):
    return lib().or_ht_n_frames(C.byref(p))


def ht_separate(p, mix, mask):
    mix = np.ascontiguousarray(mix, dtype=np.float32)
    length = mix.shape[-1]
    out = np.zeros((p.n_sources, p.n_channels, length), np.float32)
    _check(lib().or_ht_separate(C.byref(p), mix.reshape(-1), length,
                                np.ascontiguousarray(mask, np.float32).reshape(-1),
                                out.reshape(-1)), "ht_separate")
    return out


class _Bands:
    """Keeps the int arrays alive as long as the params that point at them."""

    def __init__(self, sizes, freqs):
        self.sizes = np.ascontiguousarray(sizes, dtype=np.int32)
        self.freqs = np.ascontiguousarray(freqs, dtype=np.int32)


def rf_params(band_sizes, band_freqs, n_channels=2, n_stems=1, n_fft=2048, hop=441,
              normalized=0, zero_dc=0, chunk=352800, step=None, complement=0,
              sample_first=0, sample_count=0, threads=1, num_overlap=2, shifts=0, seed=0,
              sample_rate=44100):
    keep = _Bands(band_sizes, band_freqs)
    p = RfParams(n_channels, n_stems, n_fft, hop, normalized, zero_dc, chunk,
                 chunk // num_overlap if step is None else step, keep.sizes.size,
                 keep.sizes.ctypes.data_as(_I32P), keep.freqs.ctypes.data_as(_I32P),
                 complement, sample_first, sample_count, threads, shifts, seed, sample_rate)
    p._keep = keep
    return p


def rf_n_chunks(p, length):
    return lib().or_rf_n_chunks(C.byref(p), length)


def rf_separate(p, mix, mask):
    mix = np.ascontiguousarray(mix, dtype=np.float32)
    length = mix.shape[-1]
    out = np.zeros((p.n_stems + (1 if p.complement else 0), p.n_channels, length), np.float32)
    _check(lib().or_rf_separate(C.byref(p), mix.reshape(-1), length,
                                np.ascontiguousarray(mask, np.float32).reshape(-1),
                                out.reshape(-1)), "rf_separate")
    return out


def rf_band_gather(p, z):
    z = np.ascontiguousarray(z, dtype=np.complex128)
    T = z.shape[-1]
    din = int(np.sum(p._keep.sizes)) * p.n_channels * 2
    feat = np.zeros(din * T, np.float32)
    _check(lib().or_rf_band_gather(C.byref(p), z.reshape(-1).view(np.float64), T, feat), "band_gather")
    return feat


def tfc_params(n_stems=1, n_fft=7680, hop=1024, dim_f=3072, dim_t=256, zero_bins=3, chunking=0,
               overlap=-1.0, num_overlap=4, compensate=1.0, complement=0, sample_first=0,
               sample_count=0, threads=1):
    return TfcParams(n_stems, n_fft, hop, dim_f, dim_t, zero_bins, chunking, overlap, num_overlap,
                     compensate, complement, sample_first, sample_count, threads)


def tfc_n_chunks(p, length):
    return lib().or_tfc_n_chunks(C.byref(p), length)


def tfc_separate(p, mix, mask):
    mix = np.ascontiguousarray(mix, dtype=np.float32)
    length = mix.shape[-1]
    out = np.zeros((p.n_stems + (1 if p.complement else 0), 2, length), np.float32)
    _check(lib().or_tfc_separate(C.byref(p), mix.reshape(-1), length,
                                 np.ascontiguousarray(mask, np.float32).reshape(-1),
                                 out.reshape(-1)), "tfc_separate")
    return out
