"""GPU tests of the separate() contracts around the kernels, through the C ABI:

* the HTDemucs bag of models (src/htdemucs.cpp:585-642) against the oracle;
* progress and cancellation (SeparateOptions, src/separator.h:26-31) counted as each
  reference separator counts them: HTDemucs src/htdemucs.cpp:576-577, 593, 602; RoFormer
  src/roformer.cpp:444-451, 479; TFC-TDF src/tfc_tdf.cpp:411-425, 577-581;
* the host-buffer entry point on a cancellation: the caller's output buffer is untouched.

Bar for the numerics: per stem, max |got - ref| / max |ref| <= 1e-5.
"""
from __future__ import annotations

import numpy as np
import pytest

from common import max_rel_err, synth_audio, synth_mask

pytestmark = pytest.mark.gpu

TOL = 1e-5


def run_gpu(plan, mix, mask, **kw):
    import torch
    d_mix = torch.from_numpy(np.ascontiguousarray(mix)).cuda()
    d_mask = torch.from_numpy(np.ascontiguousarray(mask)).cuda()
    d_out = torch.full(plan.out_shape, float("nan"), device="cuda", dtype=torch.float32)
    plan.separate(d_mix, d_mask, d_out, **kw)
    torch.cuda.synchronize()
    return d_out.cpu().numpy()


# ---- bag of models -------------------------------------------------------------------------------
BAG_CASES = [
    # name, weights [n_models][S], shifts, mono_norm, cac_norm
    ("two_models", [[0.75, 1.0, 0.25, 2.0], [1.25, 0.5, 1.0, 0.0]], 0, 1, 1),
    ("ft_one_hot", np.eye(4).tolist(), 0, 1, 1),                 # htdemucs_ft: one model per stem
    ("three_models_shifts", [[1.0, 0.0, 1.0, 1.0], [0.5, 1.0, 0.0, 1.0], [1.0, 1.0, 1.0, 0.5]], 2, 1, 1),
    ("two_models_raw", [[1.0, 1.0, 1.0, 1.0], [3.0, 1.0, 0.5, 1.0]], 0, 0, 0),
]


@pytest.mark.parametrize("case", BAG_CASES, ids=[c[0] for c in BAG_CASES])
def test_htdemucs_bag_matches_oracle(case, engine, oracle_mod):
    name, w, shifts, mono, cac = case
    w = np.asarray(w, np.float32)
    seg, length, S = 1024 * 24, 60000, 4
    plan = engine.plan_htdemucs(length, n_sources=S, segment=seg, mono_norm=mono, cac_norm=cac, shifts=shifts,
                                seed=5, bag_weights=w)
    p = oracle_mod.ht_params(n_sources=S, segment=seg, mono_norm=mono, cac_norm=cac, shifts=shifts, seed=5,
                             threads=8, bag_weights=w)
    assert plan.n_models == w.shape[0]
    assert plan.n_chunks == w.shape[0] * oracle_mod.ht_n_segments(p, length)
    mix = synth_audio(51, length)
    mask = synth_mask(52, plan.mask_floats, 1.0)
    got = run_gpu(plan, mix, mask)
    want = oracle_mod.ht_separate(p, mix, mask)
    assert np.isfinite(got).all()
    err = max_rel_err(got, want)
    assert err <= TOL, f"{name}: max rel err {err:.3e}"
    # the host entry point streams every model's masks in batches and gives the same floats
    np.testing.assert_array_equal(plan.separate_host(mix, mask), got)


def test_htdemucs_bag_of_one_is_the_plain_path(engine):
    """One model of weight 1 given as a bag adds its stems to zero, divides by 1 and maps back
    once: the same floats as the plan without a bag."""
    seg, length = 1024 * 24, 50000
    mix = synth_audio(53, length)
    a = engine.plan_htdemucs(length, segment=seg)
    b = engine.plan_htdemucs(length, segment=seg, bag_weights=np.ones((1, 4), np.float32))
    mask = synth_mask(54, a.mask_floats, 1.0)
    np.testing.assert_array_equal(run_gpu(a, mix, mask), run_gpu(b, mix, mask))


def _view(ptr, n):
    """A torch float32 tensor over n floats of device memory at ptr (no copy)."""
    import torch

    class _A:
        __cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3}
    return torch.as_tensor(_A(), device="cuda")


def test_htdemucs_bag_through_the_network_loop(engine, oracle_mod):
    """stg_separate_network with a bag: member m's chunks reach the callback as m * G + k; a
    callback that writes ox = Z * M (the stand-in network) gives the oracle's bag."""
    import torch
    seg, length, S = 1024 * 24, 50000, 4
    w = np.array([[1.0, 0.5, 1.0, 1.0], [0.5, 1.0, 2.0, 1.0]], np.float32)
    plan = engine.plan_htdemucs(length, n_sources=S, segment=seg, bag_weights=w)
    mix = synth_audio(55, length)
    mask = synth_mask(56, plan.mask_floats, 1.0)
    d_mask = torch.from_numpy(mask).cuda()
    n_in, n_out = plan.network_info()
    T = plan.n_frames
    seen = []

    def net(first, k, p_in, p_out, stream):
        seen.append((first, k))
        x = _view(p_in, k * n_in).view(k, 1, 2, 2, 2048, T)            # [chunk][.][c][re/im][F][T]
        m = d_mask[first * n_out:(first + k) * n_out].view(k, S, 2, 2, 2048, T)
        re = x[:, :, :, 0] * m[:, :, :, 0] - x[:, :, :, 1] * m[:, :, :, 1]
        im = x[:, :, :, 0] * m[:, :, :, 1] + x[:, :, :, 1] * m[:, :, :, 0]
        _view(p_out, k * n_out).view(k, S, 2, 2, 2048, T).copy_(torch.stack([re, im], dim=3))

    d_mix = torch.from_numpy(mix).cuda()
    out = torch.empty(plan.out_shape, device="cuda")
    plan.separate_network(d_mix, out, net, chunks_per_batch=2)
    torch.cuda.synchronize()
    G = plan.n_chunks // 2
    assert seen == [(m * G + b, min(2, G - b)) for m in range(2) for b in range(0, G, 2)]
    p = oracle_mod.ht_params(n_sources=S, segment=seg, mono_norm=1, cac_norm=1, threads=8, bag_weights=w)
    assert max_rel_err(out.cpu().numpy(), oracle_mod.ht_separate(p, mix, mask)) <= TOL


# ---- progress and cancellation --------------------------------------------------------------------
def _ref_progress_htdemucs(n_models, shifts, length, stride, actual_chunks):
    """htdemucs.cpp:576-577, 602: progress(++done, total) after every segment pass."""
    total = n_models * max(1, shifts) * -(-length // stride)
    return [(k, total) for k in range(1, actual_chunks + 1)]


def _ref_progress_roformer(shifts, chunks_of_len, actual_chunks):
    """roformer.cpp:444-451, 479: tick before every chunk reports (done, total) once done > 0,
    then (total, total) at the end."""
    total = max(1, shifts) * chunks_of_len
    return [(k, total) for k in range(1, actual_chunks)] + [(total, total)]


def _ref_progress_tfc(actual_chunks):
    """tfc_tdf.cpp:425, 577-579: tick(++done, total) after every chunk."""
    return [(k, actual_chunks) for k in range(1, actual_chunks + 1)]


def _batched(seq, per, final_total=False):
    """The pairs a run in batches of `per` chunks reports: the reference's pair after each
    batch's last chunk (RoFormer's last report is (total, total))."""
    n = len(seq)
    ends = list(range(per, n, per)) + [n]
    return [seq[e - 1] for e in ends]


def _collect(plan, mix, mask, per, **kw):
    got = []
    run_gpu(plan, mix, mask, chunks_per_batch=per, progress=lambda d, t: got.append((d, t)), **kw)
    return got


@pytest.mark.parametrize("per", [1, 3])
def test_progress_htdemucs_bag_and_shifts(engine, per):
    seg, length, S, shifts = 1024 * 24, 60000, 4, 2
    w = np.array([[1.0, 1.0, 0.0, 1.0], [0.0, 1.0, 1.0, 1.0]], np.float32)
    plan = engine.plan_htdemucs(length, n_sources=S, segment=seg, shifts=shifts, seed=3, bag_weights=w)
    mix = synth_audio(61, length)
    mask = synth_mask(62, plan.mask_floats, 1.0)
    per_model = plan.n_chunks // 2
    ref = _ref_progress_htdemucs(2, shifts, length, int(0.75 * seg), plan.n_chunks)
    # batches never span two models: the reference's pair after each batch's last chunk
    ends = []
    for m in range(2):
        ends += [m * per_model + min(e, per_model) for e in range(per, per_model + per, per)]
    want = [ref[e - 1] for e in ends]
    assert _collect(plan, mix, mask, per) == want


@pytest.mark.parametrize("shifts,per", [(0, 1), (0, 4), (2, 1)])
def test_progress_roformer(pkg, engine, oracle_mod, shifts, per):
    sizes, freqs = pkg.bands.bs_bands()
    chunk, length = 441 * 40, 441 * 100 + 17
    plan = engine.plan_roformer(length, sizes, freqs, chunk=chunk, num_overlap=2, shifts=shifts, seed=4)
    p0 = oracle_mod.rf_params(sizes, freqs, chunk=chunk, num_overlap=2)
    ref = _ref_progress_roformer(shifts, oracle_mod.rf_n_chunks(p0, length), plan.n_chunks)
    want = _batched(ref, per)
    want[-1] = (ref[-1][1], ref[-1][1])
    mix = synth_audio(63, length)
    mask = synth_mask(64, plan.mask_floats, 0.5)
    assert _collect(plan, mix, mask, per) == want


@pytest.mark.parametrize("per", [1, 2])
def test_progress_tfc(engine, per):
    length = 70000
    plan = engine.plan_tfc(length, dim_t=32, overlap=0.5)
    mix = synth_audio(65, length)
    mask = synth_mask(66, plan.mask_floats, 1.0)
    assert _collect(plan, mix, mask, per) == _batched(_ref_progress_tfc(plan.n_chunks), per)


def _cancel_after(n_polls):
    calls = []

    def should_cancel():
        calls.append(1)
        return len(calls) > n_polls
    return should_cancel, calls


def test_cancel_after_first_batch_returns_cancelled(pkg, engine):
    """should_cancel is polled before every batch (src/roformer.cpp:448); true before the second
    abandons the job with STG_CANCELLED (3) after exactly one progress report."""
    sizes, freqs = pkg.bands.mel_bands()
    chunk, length = 441 * 40, 441 * 100
    plan = engine.plan_roformer(length, sizes, freqs, chunk=chunk, num_overlap=4)
    mix = synth_audio(67, length)
    mask = synth_mask(68, plan.mask_floats, 0.5)
    should_cancel, calls = _cancel_after(1)
    seen = []
    with pytest.raises(pkg.Cancelled) as ei:
        run_gpu(plan, mix, mask, chunks_per_batch=2, progress=lambda d, t: seen.append(d), should_cancel=should_cancel)
    assert ei.value.code == 3
    assert len(calls) == 2 and seen == [2]
    # the plan is still usable afterwards
    assert np.isfinite(run_gpu(plan, mix, mask)).all()


def test_tfc_polls_cancel_after_its_last_chunk(engine, pkg):
    """The reference's TFC-TDF tick after the last chunk polls should_cancel once more
    (src/tfc_tdf.cpp:425, 578): a cancel there still ends the job with Cancelled."""
    length = 50000
    plan = engine.plan_tfc(length, dim_t=32)
    n = plan.n_chunks
    mix = synth_audio(69, length)
    mask = synth_mask(70, plan.mask_floats, 1.0)
    should_cancel, calls = _cancel_after(n)   # false before every chunk, true after the last
    with pytest.raises(pkg.Cancelled):
        run_gpu(plan, mix, mask, chunks_per_batch=1, should_cancel=should_cancel)
    assert len(calls) == n + 1


def test_host_cancel_leaves_output_untouched(pkg, engine):
    """stg_separate_host_ex cancelled after its first batch: STG_CANCELLED, the caller's output
    buffer keeps its contents (the result is never copied back), and every copy from the
    caller's buffers has finished when the call returns, so the caller may free them."""
    sizes, freqs = pkg.bands.bs_bands()
    chunk, length = 441 * 40, 441 * 120
    plan = engine.plan_roformer(length, sizes, freqs, chunk=chunk, num_overlap=2)
    mix = synth_audio(71, length)
    mask = synth_mask(72, plan.mask_floats, 0.5)
    out = np.full(plan.out_shape, 7.0, np.float32)
    should_cancel, calls = _cancel_after(1)
    with pytest.raises(pkg.Cancelled):
        plan.separate_host(mix, mask, out=out, chunks_per_batch=1, should_cancel=should_cancel)
    assert (out == 7.0).all()
    mask[:] = np.nan   # the host buffers are the caller's again: nothing reads them any more
    mix[:] = np.nan
    mix2 = synth_audio(71, length)
    mask2 = synth_mask(72, plan.mask_floats, 0.5)
    np.testing.assert_array_equal(plan.separate_host(mix2, mask2), run_gpu(plan, mix2, mask2))
