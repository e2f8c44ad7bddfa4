"""The entry points around a real network, against the CPU oracle.

* The DSP primitives of src/stft.h on the device: stg_torch_stft / stg_torch_istft and
  stg_htdemucs_spec / stg_htdemucs_ispec against the restated torch_stft / torch_istft /
  htdemucs_spec / htdemucs_ispec (max |diff| / max |ref| <= 1e-5).
* The front half writes the network's input layouts: RoFormer band-major features
  (src/roformer.cpp:226-241) and HTDemucs CaC planes (src/htdemucs.cpp:423-433).
* stg_separate_network: front -> a network callback -> back -> finish, with the stand-in
  network computed by torch on the GPU, against the oracle's separation (and, for RoFormer,
  bit for bit against the fused entry point, which runs the same kernel on the same masks).
"""
from __future__ import annotations

import numpy as np
import pytest

from common import max_rel_err, synth_audio, synth_mask

pytestmark = pytest.mark.gpu

TOL = 1e-5


def _rel(got, want):
    got, want = np.asarray(got), np.asarray(want)
    return float(np.abs(got - want).max() / max(np.abs(want).max(), 1e-30))


# ---- primitives ----------------------------------------------------------------------------
@pytest.mark.parametrize("n_fft,hop,normalized,C,n", [
    (2048, 441, False, 2, 441 * 120 + 17),
    (2048, 441, True, 1, 30000),
    (4096, 1024, False, 2, 50001),
    (7680, 1024, False, 2, 1024 * 40 + 3),
])
def test_torch_stft_istft(engine, oracle_mod, n_fft, hop, normalized, C, n):
    import torch
    x = synth_audio(61, n, channels=C)
    spec = engine.torch_stft(torch.from_numpy(x).cuda(), n_fft, hop, normalized).cpu().numpy()
    for c in range(C):
        want = oracle_mod.torch_stft(x[c], n_fft, hop, normalized)
        assert spec[c].shape == want.shape
        assert _rel(spec[c], want) <= TOL, f"stft channel {c}"
    ref_spec = np.stack([oracle_mod.torch_stft(x[c], n_fft, hop, normalized) for c in range(C)])
    y = engine.torch_istft(torch.from_numpy(ref_spec.astype(np.complex64)).cuda(), n_fft, hop, normalized)
    y = y.cpu().numpy()
    for c in range(C):
        want = oracle_mod.torch_istft(ref_spec[c], n_fft, hop, normalized)
        assert _rel(y[c], want) <= TOL, f"istft channel {c}"


@pytest.mark.parametrize("n", [343980, 1024 * 30, 20000 + 7])
def test_htdemucs_spec_ispec(engine, oracle_mod, n):
    import torch
    x = synth_audio(62, n)
    spec = engine.htdemucs_spec(torch.from_numpy(x).cuda()).cpu().numpy()
    ref = np.stack([oracle_mod.htdemucs_spec(x[c]) for c in range(2)])
    assert spec.shape == ref.shape
    assert _rel(spec, ref) <= TOL
    y = engine.htdemucs_ispec(torch.from_numpy(ref.astype(np.complex64)).cuda(), n).cpu().numpy()
    for c in range(2):
        assert _rel(y[c], oracle_mod.htdemucs_ispec(ref[c], n)) <= TOL


# ---- front half layouts -------------------------------------------------------------------
def test_roformer_front_features(pkg, engine, oracle_mod):
    import torch
    sizes, freqs = pkg.bands.mel_bands()
    chunk = 441 * 40
    n = chunk + 5000                      # shorter than two borders: no border padding
    plan = engine.plan_roformer(n, sizes, freqs, chunk=chunk, num_overlap=4)
    n_in, _ = plan.network_info()
    mix = synth_audio(63, n)
    feat = torch.empty(n_in * plan.n_chunks, device="cuda")
    plan.front(torch.from_numpy(mix).cuda(), 0, plan.n_chunks, feat)
    torch.cuda.synchronize()
    p = oracle_mod.rf_params(sizes, freqs, chunk=chunk, num_overlap=4)
    z = np.stack([oracle_mod.torch_stft(mix[c, :chunk], 2048, 441) for c in range(2)])
    want = oracle_mod.rf_band_gather(p, z)
    got = feat[:n_in].cpu().numpy()
    assert _rel(got, want) <= TOL


def test_htdemucs_front_cac(engine, oracle_mod):
    import torch
    seg = 343980
    n = seg + 100000
    plan = engine.plan_htdemucs(n, n_sources=4, segment=seg, mono_norm=False, cac_norm=False)
    n_in, n_out = plan.network_info()
    assert n_out == plan.mask_floats_per_chunk
    mix = synth_audio(64, n)
    cac = torch.empty(n_in, device="cuda")
    plan.front(torch.from_numpy(mix).cuda(), 0, 1, cac)
    torch.cuda.synchronize()
    T = plan.n_frames
    got = cac.cpu().numpy().reshape(4, 2048, T)
    for c in range(2):
        z = oracle_mod.htdemucs_spec(mix[c, :seg])
        assert _rel(got[2 * c], z.real) <= TOL and _rel(got[2 * c + 1], z.imag) <= TOL


def test_htdemucs_front_cac_normalised(engine, oracle_mod):
    """The front half with both normalisations: the mix divided by its mono std, then the
    segment's CaC planes mapped to (v - mean) / (1e-5 + std) (src/htdemucs.cpp:434-436, 539-549)."""
    import torch
    seg = 1024 * 24
    n = 3 * seg
    plan = engine.plan_htdemucs(n, n_sources=4, segment=seg)
    n_in, _ = plan.network_info()
    mix = synth_audio(71, n)
    cac = torch.empty(n_in * 2, device="cuda")
    d_mix = torch.from_numpy(mix).cuda()
    plan.front(d_mix, 0, 2, cac)
    torch.cuda.synchronize()
    T = plan.n_frames
    mono = mix.astype(np.float64).mean(axis=0).astype(np.float32).astype(np.float64)
    mixn = ((mix - mono.mean()) / mono.std(ddof=1)).astype(np.float32)
    stride = int(0.75 * seg)
    for k in range(2):
        planes = np.concatenate([
            np.stack([z.real, z.imag]) for z in
            (oracle_mod.htdemucs_spec(mixn[c, k * stride:k * stride + seg]) for c in range(2))])
        v = planes.astype(np.float32).astype(np.float64)
        want = (v - v.mean()) / (1e-5 + v.std(ddof=1))
        got = cac[k * n_in:(k + 1) * n_in].cpu().numpy().reshape(4, 2048, T)
        assert _rel(got, want) <= TOL, f"segment {k}"
    # a later batch of the same track reads the normalised copy; a different track may not
    plan.front(d_mix, 1, 1, cac)
    with pytest.raises(Exception):
        plan.front(d_mix.clone(), 1, 1, cac)


# ---- whole separations through the network callback -----------------------------------------
def _run_network(plan, mix, net, per_batch):
    import torch
    d_mix = torch.from_numpy(mix).cuda()
    out = torch.empty(plan.out_shape, device="cuda")
    plan.separate_network(d_mix, out, net, chunks_per_batch=per_batch)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def _view(ptr, n):
    """A torch float32 tensor over n floats of device memory at ptr (no copy)."""
    import torch
    class _A:
        __cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3}
    return torch.as_tensor(_A(), device="cuda")


def test_roformer_network_loop_matches_fused(pkg, engine, oracle_mod):
    import torch
    sizes, freqs = pkg.bands.bs_bands()
    n = 441 * 100 + 33
    plan = engine.plan_roformer(n, sizes, freqs, chunk=441 * 40, num_overlap=2, zero_dc=True, complement=True)
    mix = synth_audio(65, n)
    mask = synth_mask(66, plan.mask_floats, 0.5)
    d_mask = torch.from_numpy(mask).cuda()
    n_in, n_out = plan.network_info()

    def net(first, k, p_in, p_out, stream):   # the "network" hands back this chunk batch's masks
        _view(p_out, k * n_out).copy_(d_mask[first * n_out:(first + k) * n_out])

    got = _run_network(plan, mix, net, per_batch=3)
    fused = torch.empty(plan.out_shape, device="cuda")
    plan.separate(torch.from_numpy(mix).cuda(), d_mask, fused)
    torch.cuda.synchronize()
    assert np.array_equal(got, fused.cpu().numpy())
    p = oracle_mod.rf_params(sizes, freqs, chunk=441 * 40, num_overlap=2, zero_dc=1, complement=1, threads=8)
    assert max_rel_err(got, oracle_mod.rf_separate(p, mix, mask)) <= TOL


@pytest.mark.parametrize("norm", [False, True], ids=["raw", "normalised"])
def test_htdemucs_network_loop(engine, oracle_mod, norm):
    import torch
    seg, n, S = 1024 * 24, 60000, 4
    plan = engine.plan_htdemucs(n, n_sources=S, segment=seg, mono_norm=norm, cac_norm=norm)
    mix = synth_audio(67, n)
    mask = synth_mask(68, plan.mask_floats, 1.0)
    d_mask = torch.from_numpy(mask).cuda()
    n_in, n_out = plan.network_info()
    T = plan.n_frames

    def net(first, k, p_in, p_out, stream):   # ox = Z * M per stem (the stand-in network)
        x = _view(p_in, k * n_in).view(k, 1, 2, 2, 2048, T)            # [chunk][.][c][re/im][F][T]
        m = d_mask[first * n_out:(first + k) * n_out].view(k, S, 2, 2, 2048, T)
        re = x[:, :, :, 0] * m[:, :, :, 0] - x[:, :, :, 1] * m[:, :, :, 1]
        im = x[:, :, :, 0] * m[:, :, :, 1] + x[:, :, :, 1] * m[:, :, :, 0]
        _view(p_out, k * n_out).view(k, S, 2, 2, 2048, T).copy_(torch.stack([re, im], dim=3))

    got = _run_network(plan, mix, net, per_batch=2)
    p = oracle_mod.ht_params(n_sources=S, segment=seg, mono_norm=int(norm), cac_norm=int(norm), threads=8)
    assert max_rel_err(got, oracle_mod.ht_separate(p, mix, mask)) <= TOL


def test_tfc_network_loop(engine, oracle_mod):
    import torch
    n = 70000
    plan = engine.plan_tfc(n, dim_t=32, overlap=0.5, compensate=1.009, complement=True)
    mix = synth_audio(69, n)
    mask = synth_mask(70, plan.mask_floats, 1.0)
    d_mask = torch.from_numpy(mask).cuda()
    n_in, n_out = plan.network_info()

    def net(first, k, p_in, p_out, stream):   # y = in * mask (the stand-in network)
        x = _view(p_in, k * n_in)
        _view(p_out, k * n_out).copy_(x * d_mask[first * n_out:(first + k) * n_out])

    got = _run_network(plan, mix, net, per_batch=4)
    p = oracle_mod.tfc_params(dim_t=32, overlap=0.5, compensate=1.009, complement=1, threads=8)
    assert max_rel_err(got, oracle_mod.tfc_separate(p, mix, mask)) <= TOL
