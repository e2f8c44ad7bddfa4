"""stems.cpp_b200 -- the B200 spectral front/back end of stems.cpp, from Python.

A thin ctypes layer over the C ABI in include/stems_gpu_v1.h (libstems_gpu.so, built
in-tree for sm_100a by build.py). It mirrors the reference's separator interface
(src/separator.h:19-54): a plan is made for one model configuration and one track length,
and ``separate`` runs chunking -> STFT -> mask -> iSTFT -> overlap-add on the GPU. The
network is out of scope; a mask buffer stands in for its output.

There is no CPU fallback: when the library is missing or no B200 is visible, every call
raises. Device buffers may be torch CUDA tensors (their data_ptr and the current stream are
used) or raw device pointers.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import bands  # noqa: F401  (band tables for RoFormer configurations)
from . import sharding  # noqa: F401  (work split across GPUs)

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libstems_gpu.so")

STATUS = {0: "OK", 1: "INVALID_ARGUMENT", 2: "UNSUPPORTED", 3: "CANCELLED", 4: "MODEL_ERROR",
          5: "IO_ERROR", 6: "OUT_OF_MEMORY", 7: "INTERNAL_ERROR"}
ARCH_ROFORMER, ARCH_HTDEMUCS, ARCH_TFC = 0, 1, 2

_I32P = C.POINTER(C.c_int32)


class StemsError(RuntimeError):
    def __init__(self, code, message):
        super().__init__(f"{STATUS.get(code, code)}: {message}")
        self.code = code


class Cancelled(StemsError):
    pass


class HTDemucsConfig(C.Structure):
    _fields_ = [("size", C.c_uint32), ("n_channels", C.c_int32), ("n_sources", C.c_int32),
                ("segment", C.c_int32), ("overlap", C.c_float), ("mono_norm", C.c_int32),
                ("cac_norm", C.c_int32), ("shifts", C.c_int32), ("seed", C.c_uint32),
                ("sample_rate", C.c_int32), ("n_models", C.c_int32), ("bag_weights", C.POINTER(C.c_float))]


class RoFormerConfig(C.Structure):
    _fields_ = [("size", C.c_uint32), ("n_channels", C.c_int32), ("n_stems", C.c_int32),
                ("n_fft", C.c_int32), ("hop", C.c_int32), ("normalized", C.c_int32),
                ("zero_dc", C.c_int32), ("chunk", C.c_int32), ("num_overlap", C.c_int32),
                ("overlap", C.c_float), ("n_bands", C.c_int32), ("band_sizes", _I32P),
                ("band_freqs", _I32P), ("complement", C.c_int32), ("shifts", C.c_int32),
                ("seed", C.c_uint32), ("sample_rate", C.c_int32)]


class TFCConfig(C.Structure):
    _fields_ = [("size", C.c_uint32), ("n_stems", C.c_int32), ("n_fft", C.c_int32),
                ("hop", C.c_int32), ("dim_f", C.c_int32), ("dim_t", C.c_int32),
                ("zero_bins", C.c_int32), ("chunking", C.c_int32), ("num_overlap", C.c_int32),
                ("overlap", C.c_float), ("compensate", C.c_float), ("complement", C.c_int32)]


class PlanInfo(C.Structure):
    _fields_ = [("size", C.c_uint32), ("arch", C.c_int32), ("n_samples", C.c_int64),
                ("n_channels", C.c_int32), ("n_out_sources", C.c_int32), ("n_chunks", C.c_int64),
                ("n_frames", C.c_int64), ("mask_floats_per_chunk", C.c_int64),
                ("out_floats", C.c_int64), ("scratch_bytes", C.c_int64), ("n_models", C.c_int32)]


class VrBandC(C.Structure):
    _fields_ = [(k, C.c_int32) for k in ("sample_rate", "hop", "n_fft", "crop_start", "crop_stop", "hpf_start",
                                        "hpf_stop", "lpf_start", "lpf_stop")]


class VrFirC(C.Structure):
    _fields_ = [("src_rate", C.c_int32), ("dst_rate", C.c_int32), ("n_taps", C.c_int32),
                ("taps", C.POINTER(C.c_float))]


class VrConfig(C.Structure):
    _fields_ = [("size", C.c_uint32), ("sample_rate", C.c_int32), ("bins", C.c_int32),
                ("pre_filter_start", C.c_int32), ("pre_filter_stop", C.c_int32), ("n_bands", C.c_int32),
                ("bands", C.POINTER(VrBandC)), ("n_firs", C.c_int32), ("firs", C.POINTER(VrFirC))]


PROGRESS_FN = C.CFUNCTYPE(None, C.c_void_p, C.c_int32, C.c_int32)
CANCEL_FN = C.CFUNCTYPE(C.c_int32, C.c_void_p)


class RunOptions(C.Structure):
    _fields_ = [("size", C.c_uint32), ("chunks_per_batch", C.c_int32),
                ("on_progress", PROGRESS_FN), ("should_cancel", CANCEL_FN), ("user", C.c_void_p)]


class NetworkInfo(C.Structure):
    _fields_ = [("size", C.c_uint32), ("net_in_floats_per_chunk", C.c_int64),
                ("net_out_floats_per_chunk", C.c_int64)]


NETWORK_FN = C.CFUNCTYPE(C.c_int32, C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p)


# Every symbol include/stems_gpu_v1.h declares, with its ctypes signature.
_SIGNATURES = {
    "stg_version": (C.c_char_p, []),
    "stg_device_count": (C.c_int, []),
    "stg_engine_create": (C.c_int32, [C.c_int, C.POINTER(C.c_void_p)]),
    "stg_engine_destroy": (None, [C.c_void_p]),
    "stg_engine_last_error": (C.c_char_p, [C.c_void_p]),
    "stg_engine_set_profiling": (C.c_int32, [C.c_void_p, C.c_int32]),
    "stg_plan_last_timing": (C.c_int32, [C.c_void_p, C.POINTER(C.c_float), C.POINTER(C.c_float),
                                         C.POINTER(C.c_int32)]),
    "stg_plan_last_timing_detail": (C.c_int32, [C.c_void_p, C.POINTER(C.c_float), C.POINTER(C.c_float),
                                                C.POINTER(C.c_float), C.POINTER(C.c_int32)]),
    "stg_plan_htdemucs": (C.c_int32, [C.c_void_p, C.POINTER(HTDemucsConfig), C.c_int64, C.POINTER(C.c_void_p)]),
    "stg_plan_roformer": (C.c_int32, [C.c_void_p, C.POINTER(RoFormerConfig), C.c_int64, C.POINTER(C.c_void_p)]),
    "stg_plan_tfc": (C.c_int32, [C.c_void_p, C.POINTER(TFCConfig), C.c_int64, C.POINTER(C.c_void_p)]),
    "stg_plan_destroy": (None, [C.c_void_p]),
    "stg_plan_get_info": (C.c_int32, [C.c_void_p, C.POINTER(PlanInfo)]),
    "stg_separate": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "stg_separate_part": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p,
                                      C.c_void_p]),
    "stg_separate_dual_mono": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "stg_separate_host": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "stg_separate_host_ex": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                         C.POINTER(RunOptions)]),
    "stg_separate_multi_host": (C.c_int32, [C.POINTER(C.c_void_p), C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p]),
    "stg_separate_ex": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                    C.POINTER(RunOptions)]),
    "stg_plan_network_info": (C.c_int32, [C.c_void_p, C.POINTER(NetworkInfo)]),
    "stg_front": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p]),
    "stg_back": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_void_p]),
    "stg_finish": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "stg_separate_network": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, NETWORK_FN, C.c_void_p,
                                         C.POINTER(RunOptions), C.c_void_p]),
    "stg_resampled_length": (C.c_int64, [C.c_int64, C.c_int32, C.c_int32]),
    "stg_prepare_input": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int64, C.c_int32, C.c_int32, C.c_int32,
                                      C.c_int32, C.c_void_p, C.c_void_p]),
    "stg_restore_output": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int64, C.c_int32, C.c_int32, C.c_int64,
                                       C.c_void_p, C.c_void_p]),
    "stg_plan_vr": (C.c_int32, [C.c_void_p, C.POINTER(VrConfig), C.c_int64, C.POINTER(C.c_void_p)]),
    "stg_vr_plan_destroy": (None, [C.c_void_p]),
    "stg_vr_plan_frames": (C.c_int32, [C.c_void_p, C.POINTER(C.c_int64)]),
    "stg_vr_front": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "stg_vr_back": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "stg_separate_vr": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "stg_model_open": (C.c_int32, [C.c_char_p, C.POINTER(C.c_void_p), C.c_char_p, C.c_size_t]),
    "stg_model_close": (None, [C.c_void_p]),
    "stg_model_architecture": (C.c_char_p, [C.c_void_p]),
    "stg_model_sample_rate": (C.c_int32, [C.c_void_p]),
    "stg_model_htdemucs_config": (C.c_int32, [C.c_void_p, C.POINTER(HTDemucsConfig), C.c_char_p, C.c_size_t]),
    "stg_model_roformer_config": (C.c_int32, [C.c_void_p, C.POINTER(RoFormerConfig), C.c_char_p, C.c_size_t]),
    "stg_model_tfc_config": (C.c_int32, [C.c_void_p, C.POINTER(TFCConfig), C.c_char_p, C.c_size_t]),
    "stg_model_vr_config": (C.c_int32, [C.c_void_p, C.POINTER(VrConfig), C.c_char_p, C.c_size_t]),
    "stg_torch_stft": (C.c_int32, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_int32, C.c_int64,
                                   C.c_void_p, C.c_void_p]),
    "stg_torch_istft": (C.c_int32, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_int32, C.c_int32,
                                    C.c_void_p, C.c_void_p]),
    "stg_htdemucs_spec": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int64, C.c_void_p, C.c_void_p]),
    "stg_htdemucs_ispec": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_int64, C.c_void_p,
                                       C.c_void_p]),
    "stg_separate_roformer_noalloc": (C.c_int32, [C.c_int, C.POINTER(RoFormerConfig), C.c_int64, C.c_void_p,
                                                  C.c_void_p, C.c_void_p, C.c_void_p, C.c_char_p, C.c_size_t]),
}

_lib = None


def library_path() -> str:
    return LIB_PATH


def lib():
    """The loaded C library. Raises when it has not been built (no silent fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise StemsError(7, f"{LIB_PATH} is missing: run __graft_entry__.build() first")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def version() -> str:
    return lib().stg_version().decode()


def device_count() -> int:
    return lib().stg_device_count()


def resampled_length(n_samples: int, src_rate: int, dst_rate: int) -> int:
    """Samples per channel after resampling (src/audio.h:20-21)."""
    return int(lib().stg_resampled_length(n_samples, src_rate, dst_rate))


def _ptr(x):
    """Device pointer of a torch tensor (checked contiguous, float32, CUDA) or an int."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        if not x.is_cuda:
            raise StemsError(1, "expected a CUDA tensor")
        if not x.is_contiguous():
            raise StemsError(1, "expected a contiguous tensor")
        return x.data_ptr()
    raise TypeError(f"cannot take a device pointer of {type(x)}")


def _stream_of(stream, *tensors):
    if stream is not None:
        return stream if isinstance(stream, int) else stream.cuda_stream
    for t in tensors:
        if hasattr(t, "device") and getattr(t, "is_cuda", False):
            import torch
            return torch.cuda.current_stream(t.device).cuda_stream
    return None


def separate_multi_host(plans, mix, mask, out=None):
    """One track over several devices (stg_separate_multi_host): plans[d], each of its own
    engine and all of one configuration and length, writes the d-th range of output samples.
    Host buffers (numpy float32); returns the [S][C][n] result."""
    if not plans:
        raise StemsError(1, "no plans")
    p0 = plans[0]
    mix = np.ascontiguousarray(mix, dtype=np.float32)
    mask = np.ascontiguousarray(mask, dtype=np.float32)
    if mix.size != p0.n_channels * p0.n_samples or mask.size != p0.mask_floats:
        raise StemsError(1, "buffer sizes do not match the plans")
    if out is None:
        out = np.empty(p0.out_shape, np.float32)
    handles = (C.c_void_p * len(plans))(*[p._h for p in plans])
    rc = lib().stg_separate_multi_host(handles, len(plans), mix.ctypes.data, mask.ctypes.data, out.ctypes.data)
    p0.engine._check(rc, "separate_multi_host")
    return out


class Engine:
    """One CUDA device (include/stems_gpu_v1.h: stg_engine_create)."""

    def __init__(self, device: int = 0):
        self._h = C.c_void_p()
        rc = lib().stg_engine_create(device, C.byref(self._h))
        if rc != 0:
            raise StemsError(rc, f"cannot create an engine on device {device}")
        self.device = device

    def close(self):
        if self._h:
            lib().stg_engine_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def last_error(self) -> str:
        return lib().stg_engine_last_error(self._h).decode()

    def set_profiling(self, enabled: bool = True):
        """Record CUDA events around every run's kernels (see Plan.last_timing)."""
        self._check(lib().stg_engine_set_profiling(self._h, int(enabled)), "set_profiling")

    def _check(self, rc, what):
        if rc != 0:
            msg = self.last_error()
            if rc == 3:
                raise Cancelled(rc, msg or what)
            raise StemsError(rc, f"{what}: {msg}")

    # -- the DSP primitives of src/stft.h on the device ----------------------------------
    def torch_stft(self, x, n_fft, hop, normalized=False, stream=None):
        """torch.stft of each channel of x [C][n] (CUDA float32): complex64 [C][n_fft/2+1][n/hop+1]."""
        import torch
        C_, n = x.shape
        T = n // hop + 1
        spec = torch.empty((C_, n_fft // 2 + 1, T), dtype=torch.complex64, device=x.device)
        self._check(lib().stg_torch_stft(self._h, n_fft, hop, int(normalized), _ptr(x), C_, n, spec.data_ptr(),
                                         _stream_of(stream, x)), "torch_stft")
        return spec

    def torch_istft(self, spec, n_fft, hop, normalized=False, stream=None):
        """torch.istft of complex64 [C][n_fft/2+1][T]: float32 [C][hop*(T-1)]."""
        import torch
        spec = spec.contiguous()
        C_, _, T = spec.shape
        y = torch.empty((C_, hop * (T - 1)), dtype=torch.float32, device=spec.device)
        self._check(lib().stg_torch_istft(self._h, n_fft, hop, int(normalized), spec.data_ptr(), C_, T, _ptr(y),
                                          _stream_of(stream, spec)), "torch_istft")
        return y

    def plan_vr(self, n_samples, bands, firs, sample_rate=44100, bins=None, pre_filter_start=0,
                pre_filter_stop=0):
        """A VR separation (src/vr.cpp). bands: dicts with sample_rate, hop, n_fft, crop_start,
        crop_stop and optional hpf_start/hpf_stop/lpf_start/lpf_stop (-1 = none), lowest rate
        first; firs: {(src_rate, dst_rate): float32 taps}, the model's resampling filters."""
        bl = (VrBandC * len(bands))()
        for i, b in enumerate(bands):
            bl[i] = VrBandC(b["sample_rate"], b["hop"], b["n_fft"], b["crop_start"], b["crop_stop"],
                            b.get("hpf_start", -1), b.get("hpf_stop", -1), b.get("lpf_start", -1),
                            b.get("lpf_stop", -1))
        taps = {k: np.ascontiguousarray(v, dtype=np.float32) for k, v in firs.items()}
        fl = (VrFirC * max(1, len(taps)))(*[VrFirC(s, d, t.size, t.ctypes.data_as(C.POINTER(C.c_float)))
                                             for (s, d), t in taps.items()])
        if bins is None:
            bins = sum(b["crop_stop"] - b["crop_start"] for b in bands)
        cfg = VrConfig(C.sizeof(VrConfig), sample_rate, bins, pre_filter_start, pre_filter_stop, len(bands), bl,
                       len(taps), fl)
        h = C.c_void_p()
        self._check(lib().stg_plan_vr(self._h, C.byref(cfg), n_samples, C.byref(h)), "plan_vr")
        return VrPlan(self, h, n_samples, bins)

    def plan_from_model(self, model: "Model", n_samples, **run):
        """A plan for a GGUF model (Model): the configuration its metadata gives, with the
        run options (overlap, shifts, seed; HTDemucs' mono_norm / cac_norm) overriding the
        reference's defaults. VR models give a VrPlan."""
        cfg = model.config()
        for k, v in run.items():
            if not hasattr(cfg, k):
                raise StemsError(1, f"{model.architecture} has no option {k}")
            setattr(cfg, k, v)
        h = C.c_void_p()
        if model.architecture == "vr_cascaded":
            self._check(lib().stg_plan_vr(self._h, C.byref(cfg), n_samples, C.byref(h)), "plan_vr")
            return VrPlan(self, h, n_samples, cfg.bins)
        fn = {"htdemucs": lib().stg_plan_htdemucs, "tfc_tdf": lib().stg_plan_tfc}.get(model.architecture,
                                                                                    lib().stg_plan_roformer)
        self._check(fn(self._h, C.byref(cfg), n_samples, C.byref(h)), "plan_from_model")
        return Plan(self, h)

    # -- the request's audio in and the stems out (src/libstems.cpp:160-199) -----------------
    def prepare_input(self, samples, n_channels, sample_rate, interleaved=True, model_channels=2,
                      model_rate=44100, out=None, stream=None):
        """Request audio (a flat CUDA tensor of n frames x n_channels, interleaved or planar)
        -> planar float32 [model_channels][resampled length] at model_rate."""
        import torch
        n = samples.numel() // n_channels
        m = resampled_length(n, sample_rate, model_rate)
        if out is None:
            out = torch.empty((model_channels, m), dtype=torch.float32, device=samples.device)
        self._check(lib().stg_prepare_input(self._h, _ptr(samples), int(bool(interleaved)), n, n_channels,
                                            sample_rate, model_channels, model_rate, _ptr(out),
                                            _stream_of(stream, samples)), "prepare_input")
        return out

    def restore_output(self, stems, model_rate, sample_rate, n_samples, out=None, stream=None):
        """Stems [rows][len] at model_rate -> [rows][n_samples] at sample_rate."""
        import torch
        stems = stems.reshape(-1, stems.shape[-1])
        rows, length = stems.shape
        if out is None:
            out = torch.empty((rows, n_samples), dtype=torch.float32, device=stems.device)
        self._check(lib().stg_restore_output(self._h, _ptr(stems), rows, length, model_rate, sample_rate, n_samples,
                                             _ptr(out), _stream_of(stream, stems)), "restore_output")
        return out

    def htdemucs_spec(self, x, stream=None):
        """HTDemucs _spec of x [C][n]: complex64 [C][2048][ceil(n/1024)]."""
        import torch
        C_, n = x.shape
        spec = torch.empty((C_, 2048, (n + 1023) // 1024), dtype=torch.complex64, device=x.device)
        self._check(lib().stg_htdemucs_spec(self._h, _ptr(x), C_, n, spec.data_ptr(), _stream_of(stream, x)),
                    "htdemucs_spec")
        return spec

    def htdemucs_ispec(self, spec, length, stream=None):
        """HTDemucs _ispec of complex64 [C][2048][T]: float32 [C][length]."""
        import torch
        spec = spec.contiguous()
        C_, _, T = spec.shape
        y = torch.empty((C_, length), dtype=torch.float32, device=spec.device)
        self._check(lib().stg_htdemucs_ispec(self._h, spec.data_ptr(), C_, T, length, _ptr(y),
                                             _stream_of(stream, spec)), "htdemucs_ispec")
        return y

    # -- plans ---------------------------------------------------------------------------
    def plan_htdemucs(self, n_samples, n_channels=2, n_sources=4, segment=343980, overlap=-1.0,
                      mono_norm=True, cac_norm=True, shifts=0, seed=0, sample_rate=44100, n_models=1,
                      bag_weights=None):
        """HTDemucs.separate (src/htdemucs.cpp:534-642). Both normalisations are on by default,
        as in the reference; mono_norm / cac_norm False leave the mix / spectrogram raw.
        shifts > 0 averages that many random shifts (offsets from std::mt19937(seed)); the
        plan's chunks are then every shift's segments, shift by shift. n_models > 1 or
        bag_weights ([n_models][n_sources]) make a bag of models: every model's masks, model
        after model, weighted per stem (:628-642)."""
        cfg = HTDemucsConfig(C.sizeof(HTDemucsConfig), n_channels, n_sources, segment, overlap,
                             int(bool(mono_norm)), int(bool(cac_norm)), shifts, seed, sample_rate)
        keep = None
        if bag_weights is not None:
            keep = np.ascontiguousarray(bag_weights, dtype=np.float32).reshape(-1)
            n_models = keep.size // n_sources
            if keep.size != n_models * n_sources or n_models < 1:
                raise StemsError(1, "bag_weights must be [n_models][n_sources]")
            cfg.bag_weights = keep.ctypes.data_as(C.POINTER(C.c_float))
        cfg.n_models = n_models
        h = C.c_void_p()
        self._check(lib().stg_plan_htdemucs(self._h, C.byref(cfg), n_samples, C.byref(h)), "plan_htdemucs")
        return Plan(self, h)

    def plan_roformer(self, n_samples, band_sizes, band_freqs, n_channels=2, n_stems=1, n_fft=2048,
                      hop=441, normalized=False, zero_dc=False, chunk=352800, num_overlap=2,
                      overlap=-1.0, complement=False, shifts=0, seed=0, sample_rate=44100):
        sizes = np.ascontiguousarray(band_sizes, dtype=np.int32)
        freqs = np.ascontiguousarray(band_freqs, dtype=np.int32)
        cfg = RoFormerConfig(C.sizeof(RoFormerConfig), n_channels, n_stems, n_fft, hop, int(normalized),
                             int(zero_dc), chunk, num_overlap, overlap, sizes.size,
                             sizes.ctypes.data_as(_I32P), freqs.ctypes.data_as(_I32P), int(complement),
                             shifts, seed, sample_rate)
        h = C.c_void_p()
        self._check(lib().stg_plan_roformer(self._h, C.byref(cfg), n_samples, C.byref(h)), "plan_roformer")
        return Plan(self, h)

    def plan_tfc(self, n_samples, n_stems=1, n_fft=7680, hop=1024, dim_f=3072, dim_t=256, zero_bins=3,
                 chunking="uvr_mdx", num_overlap=4, overlap=-1.0, compensate=1.0, complement=False):
        ch = {"uvr_mdx": 0, "msst": 1}[chunking] if isinstance(chunking, str) else int(chunking)
        cfg = TFCConfig(C.sizeof(TFCConfig), n_stems, n_fft, hop, dim_f, dim_t, zero_bins, ch, num_overlap,
                        overlap, compensate, int(complement))
        h = C.c_void_p()
        self._check(lib().stg_plan_tfc(self._h, C.byref(cfg), n_samples, C.byref(h)), "plan_tfc")
        return Plan(self, h)


class Plan:
    """A model configuration bound to one track length (stg_plan_*)."""

    def __init__(self, engine: Engine, handle):
        self.engine = engine
        self._h = handle
        info = PlanInfo()
        info.size = C.sizeof(PlanInfo)
        engine._check(lib().stg_plan_get_info(self._h, C.byref(info)), "plan_get_info")
        self.arch = info.arch
        self.n_samples = info.n_samples
        self.n_channels = info.n_channels
        self.n_out_sources = info.n_out_sources
        self.n_chunks = info.n_chunks
        self.n_frames = info.n_frames
        self.mask_floats_per_chunk = info.mask_floats_per_chunk
        self.mask_floats = info.mask_floats_per_chunk * info.n_chunks
        self.out_floats = info.out_floats
        self.scratch_bytes = info.scratch_bytes
        self.n_models = info.n_models

    @property
    def out_shape(self):
        return (self.n_out_sources, self.n_channels, self.n_samples)

    def close(self):
        if self._h:
            lib().stg_plan_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def separate_part(self, mix, mask, out, sample_begin, sample_end, stream=None):
        """Samples [sample_begin, sample_end) of every output row (out is the whole track's
        buffer), from the chunks that reach them only."""
        self.engine._check(lib().stg_separate_part(self._h, _ptr(mix), _ptr(mask), sample_begin, sample_end,
                                                   _ptr(out), _stream_of(stream, mix, mask, out)), "separate_part")

    def separate_dual_mono(self, mix, mask, out, stream=None):
        """A one-channel plan over both channels of a stereo mix (src/separator.cpp:15-47):
        mix [2][n], mask = the left channel's masks then the right's, out [S][2][n]."""
        self.engine._check(lib().stg_separate_dual_mono(self._h, _ptr(mix), _ptr(mask), _ptr(out),
                                                        _stream_of(stream, mix, mask, out)), "separate_dual_mono")

    @staticmethod
    def _options(chunks_per_batch, progress, should_cancel):
        """stg_run_options for the callbacks (SeparateOptions.progress / should_cancel), or None;
        the ctypes callbacks are kept alive on the returned struct."""
        if progress is None and should_cancel is None and chunks_per_batch <= 0:
            return None
        opts = RunOptions()
        opts.size = C.sizeof(RunOptions)
        opts.chunks_per_batch = chunks_per_batch
        opts.on_progress = PROGRESS_FN(lambda u, d, t: progress(d, t)) if progress else PROGRESS_FN()
        opts.should_cancel = (CANCEL_FN(lambda u: int(bool(should_cancel()))) if should_cancel
                              else CANCEL_FN())
        return opts

    def separate(self, mix, mask, out, stream=None, chunks_per_batch=0, progress=None, should_cancel=None):
        """Device buffers (torch CUDA tensors or pointers): mix [C][n], mask, out [S][C][n].
        progress(done, total) and should_cancel() as the reference's SeparateOptions; a
        cancelled run raises Cancelled."""
        st = _stream_of(stream, mix, mask, out)
        opts = self._options(chunks_per_batch, progress, should_cancel)
        if opts is None:
            rc = lib().stg_separate(self._h, _ptr(mix), _ptr(mask), _ptr(out), st)
        else:
            rc = lib().stg_separate_ex(self._h, _ptr(mix), _ptr(mask), _ptr(out), st, C.byref(opts))
        self.engine._check(rc, "separate")
        return out

    # -- the halves around a real network ------------------------------------------------
    def network_info(self):
        """(network input floats per chunk, network output floats per chunk)."""
        info = NetworkInfo()
        info.size = C.sizeof(NetworkInfo)
        self.engine._check(lib().stg_plan_network_info(self._h, C.byref(info)), "network_info")
        return info.net_in_floats_per_chunk, info.net_out_floats_per_chunk

    def front(self, mix, first_chunk, n_chunks, net_in, stream=None):
        self.engine._check(lib().stg_front(self._h, _ptr(mix), first_chunk, n_chunks, _ptr(net_in),
                                           _stream_of(stream, mix)), "front")

    def back(self, mix, net_out, first_chunk, n_chunks, stream=None):
        self.engine._check(lib().stg_back(self._h, _ptr(mix), _ptr(net_out), first_chunk, n_chunks,
                                          _stream_of(stream, net_out)), "back")

    def finish(self, mix, out, stream=None):
        self.engine._check(lib().stg_finish(self._h, _ptr(mix), _ptr(out), _stream_of(stream, out)), "finish")

    def separate_network(self, mix, out, network, chunks_per_batch=0, stream=None):
        """network(first_chunk, n_chunks, net_in_ptr, net_out_ptr, stream_handle) runs the model."""
        st = _stream_of(stream, mix, out)
        errors = []

        def cb(user, first, n, p_in, p_out, s):
            try:
                network(first, n, p_in, p_out, s)
                return 0
            except Exception as e:   # reported through the status
                errors.append(e)
                return 1
        fn = NETWORK_FN(cb)
        rc = lib().stg_separate_network(self._h, _ptr(mix), _ptr(out), chunks_per_batch, fn, None, None, st)
        if errors:
            raise errors[0]
        self.engine._check(rc, "separate_network")
        return out

    def last_timing(self):
        """(ms before the combine, combine kernel ms, kernel launches) of the last run."""
        a, b, n = C.c_float(), C.c_float(), C.c_int32()
        self.engine._check(lib().stg_plan_last_timing(self._h, C.byref(a), C.byref(b), C.byref(n)),
                           "last_timing")
        return a.value, b.value, n.value

    def last_timing_detail(self):
        """(preparation ms, fused kernel ms, combine kernel ms, kernel launches) of the last run."""
        a, b, c, n = C.c_float(), C.c_float(), C.c_float(), C.c_int32()
        self.engine._check(lib().stg_plan_last_timing_detail(self._h, C.byref(a), C.byref(b), C.byref(c),
                                                             C.byref(n)), "last_timing_detail")
        return a.value, b.value, c.value, n.value

    def separate_host_ptr(self, h_mix: int, h_mask: int, h_out: int, stream=None):
        """Host pointers (e.g. pinned torch tensors' data_ptr()); blocks until h_out is filled."""
        st = stream if (stream is None or isinstance(stream, int)) else stream.cuda_stream
        self.engine._check(lib().stg_separate_host(self._h, h_mix, h_mask, h_out, st), "separate_host")

    def separate_host(self, mix, mask, out=None, stream=None, chunks_per_batch=0, progress=None,
                      should_cancel=None):
        """Host buffers (numpy float32); returns the [S][C][n] result. With progress /
        should_cancel (stg_separate_host_ex), a cancelled run raises Cancelled and leaves out
        untouched."""
        mix = np.ascontiguousarray(mix, dtype=np.float32)
        mask = np.ascontiguousarray(mask, dtype=np.float32)
        if mix.size != self.n_channels * self.n_samples or mask.size != self.mask_floats:
            raise StemsError(1, "buffer sizes do not match the plan")
        if out is None:
            out = np.empty(self.out_shape, np.float32)
        st = stream if (stream is None or isinstance(stream, int)) else stream.cuda_stream
        opts = self._options(chunks_per_batch, progress, should_cancel)
        if opts is None:
            rc = lib().stg_separate_host(self._h, mix.ctypes.data, mask.ctypes.data, out.ctypes.data, st)
        else:
            rc = lib().stg_separate_host_ex(self._h, mix.ctypes.data, mask.ctypes.data, out.ctypes.data, st,
                                            C.byref(opts))
        self.engine._check(rc, "separate_host")
        return out


class VrPlan:
    """A VR model's spectral path bound to one track length (stg_plan_vr)."""

    def __init__(self, engine: Engine, handle, n_samples, bins):
        self.engine = engine
        self._h = handle
        self.n_samples = n_samples
        self.bins = bins
        t = C.c_int64()
        engine._check(lib().stg_vr_plan_frames(self._h, C.byref(t)), "vr_plan_frames")
        self.n_frames = t.value
        self.mask_shape = (2, bins + 1, self.n_frames)
        self.out_shape = (2, 2, n_samples)

    def front(self, mix, mag=None, peak=None, stream=None):
        self.engine._check(lib().stg_vr_front(self._h, _ptr(mix), _ptr(mag), _ptr(peak), _stream_of(stream, mix)),
                           "vr_front")

    def back(self, mask, out, stream=None):
        self.engine._check(lib().stg_vr_back(self._h, _ptr(mask), _ptr(out), _stream_of(stream, mask)), "vr_back")

    def separate(self, mix, mask, out, stream=None):
        self.engine._check(lib().stg_separate_vr(self._h, _ptr(mix), _ptr(mask), _ptr(out),
                                                 _stream_of(stream, mix, out)), "separate_vr")

    def close(self):
        if self._h:
            lib().stg_vr_plan_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Model:
    """A model's spectral-path configuration read from its GGUF file (stg_model_open): no
    weights are read and no GPU is needed."""

    def __init__(self, path: str):
        h = C.c_void_p()
        msg = C.create_string_buffer(512)
        rc = lib().stg_model_open(os.fsencode(path), C.byref(h), msg, 512)
        if rc != 0:
            raise StemsError(rc, msg.value.decode(errors="replace"))
        self._h = h
        self.architecture = lib().stg_model_architecture(h).decode()
        self.sample_rate = lib().stg_model_sample_rate(h)

    def config(self):
        """The architecture's configuration struct (HTDemucsConfig, RoFormerConfig, TFCConfig
        or VrConfig); its arrays belong to this Model."""
        kinds = {"htdemucs": (HTDemucsConfig, lib().stg_model_htdemucs_config),
                 "mel_band_roformer": (RoFormerConfig, lib().stg_model_roformer_config),
                 "bs_roformer": (RoFormerConfig, lib().stg_model_roformer_config),
                 "tfc_tdf": (TFCConfig, lib().stg_model_tfc_config),
                 "vr_cascaded": (VrConfig, lib().stg_model_vr_config)}
        if self.architecture not in kinds:
            raise StemsError(4, f"unknown architecture {self.architecture!r}")
        T, fn = kinds[self.architecture]
        cfg = T()
        cfg.size = C.sizeof(T)
        msg = C.create_string_buffer(512)
        rc = fn(self._h, C.byref(cfg), msg, 512)
        if rc != 0:
            raise StemsError(rc, msg.value.decode(errors="replace"))
        cfg._model = self
        return cfg

    def close(self):
        if self._h:
            lib().stg_model_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

