"""The entry point that allocates no device memory (stg_separate_roformer_noalloc).

It is for callers that cannot call cudaMalloc (plug-ins inside a host application that owns
the device memory, real-time code that must not wait on the allocator): its tables and
scratch live in a static device array of 64 MiB. Its output must match the ordinary entry
point's (a plan and stg_separate), within the tolerance of the other parity tests, on two
calls in a row, since every call reuses the same array. This file is collected last so that a
run stopping at the first failure has run every other test; it also passes on its own.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from common import max_rel_err, synth_audio, synth_mask

pytestmark = pytest.mark.gpu

TOL = 1e-5


def _config(pkg, sizes, freqs, chunk, num_overlap):
    cfg = pkg.RoFormerConfig(C.sizeof(pkg.RoFormerConfig), 2, 1, 2048, 441, 0, 0, chunk, num_overlap, -1.0,
                             sizes.size, sizes.ctypes.data_as(C.POINTER(C.c_int32)),
                             freqs.ctypes.data_as(C.POINTER(C.c_int32)), 0)
    return cfg


@pytest.mark.parametrize("chunk,num_overlap,seconds", [(441 * 40, 4, 3.0), (352800, 4, 10.0)])
def test_noalloc_matches_the_ordinary_entry_point(pkg, engine, chunk, num_overlap, seconds):
    import torch
    sizes, freqs = pkg.bands.mel_bands()
    length = int(seconds * 44100) + 123
    plan = engine.plan_roformer(length, sizes, freqs, chunk=chunk, num_overlap=num_overlap)
    mix = torch.from_numpy(synth_audio(51, length)).cuda()
    mask = torch.from_numpy(synth_mask(52, plan.mask_floats, 0.5)).cuda()
    want = torch.empty(plan.out_shape, device="cuda", dtype=torch.float32)
    plan.separate(mix, mask, want)
    torch.cuda.synchronize()
    want = want.cpu().numpy()

    cfg = _config(pkg, sizes, freqs, chunk, num_overlap)
    msg = C.create_string_buffer(512)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        out = torch.full(plan.out_shape, float("nan"), device="cuda", dtype=torch.float32)
        rc = pkg.lib().stg_separate_roformer_noalloc(0, C.byref(cfg), length, mix.data_ptr(), mask.data_ptr(),
                                                      out.data_ptr(), stream, msg, C.sizeof(msg))
        assert rc == 0, msg.value.decode()
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert np.isfinite(got).all()
        err = max_rel_err(got, want)
        assert err <= TOL, f"call {call}: max rel err {err:.3e}"


def test_noalloc_rejects_what_does_not_fit(pkg, engine):
    import torch
    sizes, freqs = pkg.bands.mel_bands()
    length = 120 * 44100                       # 120 s at num_overlap 4: far beyond 64 MiB of scratch
    cfg = _config(pkg, sizes, freqs, 352800, 4)
    mix = torch.zeros((2, length), device="cuda")
    mask = torch.zeros(16, device="cuda")
    out = torch.zeros((1, 2, length), device="cuda")
    msg = C.create_string_buffer(512)
    rc = pkg.lib().stg_separate_roformer_noalloc(0, C.byref(cfg), length, mix.data_ptr(), mask.data_ptr(),
                                                  out.data_ptr(), None, msg, C.sizeof(msg))
    assert rc == 1
    assert "MiB" in msg.value.decode()
