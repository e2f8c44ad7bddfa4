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


def _noalloc(pkg, cfg, length, mix_ptr, mask_ptr, out_ptr, stream):
    msg = C.create_string_buffer(512)
    rc = pkg.lib().stg_separate_roformer_noalloc(0, C.byref(cfg), length, mix_ptr, mask_ptr, out_ptr, stream, msg,
                                                  C.sizeof(msg))
    assert rc == 0, msg.value.decode()


def _plan_result(pkg, engine, sizes, freqs, chunk, num_overlap, length, mix, mask):
    import torch
    plan = engine.plan_roformer(length, sizes, freqs, chunk=chunk, num_overlap=num_overlap)
    want = torch.empty(plan.out_shape, device="cuda", dtype=torch.float32)
    plan.separate(torch.from_numpy(mix).cuda(), torch.from_numpy(mask).cuda(), want)
    torch.cuda.synchronize()
    return plan, want.cpu().numpy()


def test_noalloc_small_after_large_reads_nothing_stale(pkg, engine):
    """A 10 s call fills the array's scratch; a 3 s call after it, with a different chunk size,
    must not read any of it: its output equals the plan path's."""
    import torch
    sizes, freqs = pkg.bands.mel_bands()
    stream = torch.cuda.current_stream().cuda_stream
    runs = [(352800, 4, 10.0), (441 * 40, 2, 3.0), (441 * 40, 2, 3.0)]
    for chunk, nov, seconds in runs:
        length = int(seconds * 44100) + 77
        mix = synth_audio(57, length)
        n_mask = engine.plan_roformer(length, sizes, freqs, chunk=chunk, num_overlap=nov).mask_floats
        mask = synth_mask(58, n_mask, 0.5)
        plan, want = _plan_result(pkg, engine, sizes, freqs, chunk, nov, length, mix, mask)
        d_mix, d_mask = torch.from_numpy(mix).cuda(), torch.from_numpy(mask).cuda()
        out = torch.full(plan.out_shape, float("nan"), device="cuda", dtype=torch.float32)
        _noalloc(pkg, _config(pkg, sizes, freqs, chunk, nov), length, d_mix.data_ptr(), d_mask.data_ptr(),
                 out.data_ptr(), stream)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert np.isfinite(got).all()
        assert max_rel_err(got, want) <= TOL, f"{seconds} s after the previous call"


def test_noalloc_refuses_a_driver_created_context(pkg, engine):
    """A host that made its own (cuCtxCreate) context current: the call is refused with
    STG_UNSUPPORTED before any GPU work, and the caller's context is still current after it.
    The arena's address is resolved for the runtime's primary context only, so running there
    could hand a kernel an address the caller's context does not map."""
    cu = pytest.importorskip("cuda.bindings.driver")
    sizes, freqs = pkg.bands.mel_bands()
    chunk, nov, length = 441 * 40, 4, 2 * 44100

    def ok(r):
        err = r[0] if isinstance(r, tuple) else r
        assert int(err) == 0, f"driver call failed: {err}"
        return r[1] if isinstance(r, tuple) and len(r) == 2 else r

    ok(cu.cuInit(0))
    dev = ok(cu.cuDeviceGet(0))
    ctx = ok(cu.cuCtxCreate(0, dev))
    try:
        msg = C.create_string_buffer(512)
        cfg = _config(pkg, sizes, freqs, chunk, nov)
        # the buffers are never touched: the call stops before any GPU work
        rc = pkg.lib().stg_separate_roformer_noalloc(0, C.byref(cfg), length, 256, 256, 256, None, msg, C.sizeof(msg))
        assert rc == 2, msg.value.decode()
        assert "primary context" in msg.value.decode()
        assert int(ok(cu.cuCtxGetCurrent())) == int(ctx)
    finally:
        cu.cuCtxDestroy(ctx)


def test_noalloc_from_a_thread_without_a_context(pkg, engine):
    """A thread that never touched CUDA: the call makes the device's primary context current
    for itself and leaves the thread as it found it (no context current)."""
    import threading

    import torch
    cu = pytest.importorskip("cuda.bindings.driver")
    sizes, freqs = pkg.bands.mel_bands()
    chunk, nov = 441 * 40, 4
    length = int(2.0 * 44100) + 5
    mix = synth_audio(59, length)
    plan0 = engine.plan_roformer(length, sizes, freqs, chunk=chunk, num_overlap=nov)
    mask = synth_mask(60, plan0.mask_floats, 0.5)
    _, want = _plan_result(pkg, engine, sizes, freqs, chunk, nov, length, mix, mask)
    d_mix, d_mask = torch.from_numpy(mix).cuda(), torch.from_numpy(mask).cuda()
    out = torch.full(want.shape, float("nan"), device="cuda")
    torch.cuda.synchronize()
    result = {}

    def worker():
        before = cu.cuCtxGetCurrent()[1]
        msg = C.create_string_buffer(512)
        cfg = _config(pkg, sizes, freqs, chunk, nov)
        result["rc"] = pkg.lib().stg_separate_roformer_noalloc(0, C.byref(cfg), length, d_mix.data_ptr(),
                                                               d_mask.data_ptr(), out.data_ptr(), None, msg,
                                                               C.sizeof(msg))
        result["msg"] = msg.value.decode()
        result["before"], result["after"] = int(before), int(cu.cuCtxGetCurrent()[1])

    t = threading.Thread(target=worker)
    t.start()
    t.join()
    assert result["rc"] == 0, result["msg"]
    assert result["before"] == 0 and result["after"] == 0
    torch.cuda.synchronize()
    assert max_rel_err(out.cpu().numpy(), want) <= TOL


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
