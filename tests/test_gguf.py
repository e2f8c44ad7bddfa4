"""Model configurations read from GGUF metadata (stg_model_*), against the keys the
reference's constructors read (src/htdemucs.cpp:478-500, src/roformer.cpp:360-412,
src/tfc_tdf.cpp:498-553, src/vr.cpp:296-327). The files are written by tests/gguf_writer.py
with the keys of the reference's converters; no GPU is needed except for the last tests,
which check that a plan made from a file separates like the plan made from the same
configuration by hand."""
from __future__ import annotations

import numpy as np
import pytest

import gguf_writer as G


def _common(arch, sources, complement=None):
    kv = {"general.architecture": (G.STRING, arch), "stems.model": (G.STRING, "test"),
          "stems.sources": (G.ARRAY, G.STRING, sources), "stems.samplerate": (G.U32, 44100),
          "stems.audio_channels": (G.U32, 2)}
    if complement:
        kv["stems.complement"] = (G.STRING, complement)
    return kv


def htdemucs_file(path):
    kv = _common("htdemucs", ["drums", "bass", "other", "vocals"])
    kv.update({"stems.segment_num": (G.U32, 39), "stems.segment_den": (G.U32, 5), "stems.n_models": (G.U32, 1),
               "stems.bag_weights": (G.ARRAY, G.F32, [1.0, 1.0, 1.0, 1.0])})
    G.write(path, kv, {"some.weight": np.ones((3, 4), np.float32)})


def roformer_file(path, pkg, arch="mel_band_roformer"):
    sizes, freqs = pkg.bands.mel_bands()
    kv = _common(arch, ["vocals"], complement="instrumental")
    kv.update({"roformer.dim": (G.U32, 384), "roformer.depth": (G.U32, 6), "roformer.stft_n_fft": (G.U32, 2048),
               "roformer.stft_hop_length": (G.U32, 441), "roformer.stft_normalized": (G.BOOL, 0),
               "roformer.zero_dc": (G.BOOL, 1), "roformer.chunk_size": (G.U32, 441 * 40),
               "roformer.num_overlap": (G.U32, 4), "roformer.rope_theta": (G.F32, 10000.0),
               "roformer.band_sizes": (G.ARRAY, G.I32, [int(v) for v in sizes]),
               "roformer.band_freqs": (G.ARRAY, G.I32, [int(v) for v in freqs])})
    G.write(path, kv)
    return sizes, freqs


def tfc_file(path, chunking="uvr_mdx"):
    kv = _common("tfc_tdf", ["vocals"], complement="instrumental")
    kv.update({"tfc_tdf.schema_version": (G.U32, 1), "tfc_tdf.variant": (G.STRING, "mdx_net"),
               "tfc_tdf.chunking": (G.STRING, chunking), "tfc_tdf.n_fft": (G.U32, 7680), "tfc_tdf.hop": (G.U32, 1024),
               "tfc_tdf.dim_f": (G.U32, 3072), "tfc_tdf.dim_t": (G.U32, 256), "tfc_tdf.compensate": (G.F32, 1.009),
               "tfc_tdf.act": (G.STRING, "relu")})
    kv["tfc_tdf.zero_bins" if chunking == "uvr_mdx" else "tfc_tdf.num_overlap"] = (G.U32, 3 if chunking == "uvr_mdx" else 4)
    G.write(path, kv)


VR_BANDS = [dict(sr=11025, hl=128, n_fft=640, crop_start=0, crop_stop=200, hpf_start=-1, hpf_stop=-1,
                 lpf_start=150, lpf_stop=200),
            dict(sr=44100, hl=512, n_fft=1024, crop_start=100, crop_stop=513, hpf_start=120, hpf_stop=100,
                 lpf_start=-1, lpf_stop=-1)]


def vr_file(path, oracle_mod):
    kv = _common("vr_cascaded", ["instrumental", "vocals"])
    kv.update({"vr.schema_version": (G.U32, 1), "vr.bins": (G.U32, 640), "vr.pre_filter_start": (G.U32, 600),
               "vr.pre_filter_stop": (G.U32, 640), "vr.band_count": (G.U32, len(VR_BANDS)),
               "vr.resampling": (G.STRING, "polyphase")})
    for i, b in enumerate(VR_BANDS):
        for k, v in b.items():
            kv[f"vr.band.{i}.{k}"] = (G.I32, v)
    firs = {f"resample.{s}.{d}": oracle_mod.vr_fir(s, d) for s, d in [(11025, 44100), (44100, 11025)]}
    G.write(path, kv, firs)
    return firs


def test_htdemucs_config(pkg, tmp_path):
    p = tmp_path / "h.gguf"
    htdemucs_file(p)
    m = pkg.Model(str(p))
    assert m.architecture == "htdemucs" and m.sample_rate == 44100
    c = m.config()
    assert (c.n_channels, c.n_sources, c.segment, c.mono_norm, c.cac_norm, c.shifts) == (2, 4, 343980, 1, 1, 0)
    assert c.overlap < 0


def test_htdemucs_bag_config(pkg, tmp_path):
    """htdemucs_ft-style file: stems.n_models 4 and one-hot stems.bag_weights (src/htdemucs.cpp:493-499)."""
    p = tmp_path / "ft.gguf"
    kv = _common("htdemucs", ["drums", "bass", "other", "vocals"])
    w = np.eye(4, dtype=np.float32)
    kv.update({"stems.segment_num": (G.U32, 39), "stems.segment_den": (G.U32, 5), "stems.n_models": (G.U32, 4),
               "stems.bag_weights": (G.ARRAY, G.F32, [float(x) for x in w.reshape(-1)])})
    G.write(p, kv)
    c = pkg.Model(str(p)).config()
    assert c.n_models == 4
    assert [c.bag_weights[i] for i in range(16)] == list(w.reshape(-1))
    # a bag whose weights do not match n_models x sources is a model error
    kv["stems.bag_weights"] = (G.ARRAY, G.F32, [1.0] * 15)
    q = tmp_path / "bad.gguf"
    G.write(q, kv)
    with pytest.raises(pkg.StemsError):
        pkg.Model(str(q)).config()


def test_roformer_config(pkg, tmp_path):
    p = tmp_path / "r.gguf"
    sizes, freqs = roformer_file(p, pkg)
    c = pkg.Model(str(p)).config()
    assert (c.n_stems, c.n_fft, c.hop, c.normalized, c.zero_dc, c.chunk, c.num_overlap, c.complement) == \
        (1, 2048, 441, 0, 1, 441 * 40, 4, 1)
    assert c.n_bands == len(sizes)
    assert [c.band_sizes[i] for i in range(c.n_bands)] == list(sizes)
    assert [c.band_freqs[i] for i in range(int(sum(sizes)))] == list(freqs)


@pytest.mark.parametrize("chunking", ["uvr_mdx", "msst"])
def test_tfc_config(pkg, tmp_path, chunking):
    p = tmp_path / "t.gguf"
    tfc_file(p, chunking)
    c = pkg.Model(str(p)).config()
    assert (c.n_stems, c.n_fft, c.hop, c.dim_f, c.dim_t, c.chunking, c.complement) == \
        (1, 7680, 1024, 3072, 256, int(chunking == "msst"), 1)
    assert (c.zero_bins, c.num_overlap) == ((3, 0) if chunking == "uvr_mdx" else (0, 4))
    assert abs(c.compensate - 1.009) < 1e-7


def test_vr_config_reads_bands_and_firs(pkg, oracle_mod, tmp_path):
    p = tmp_path / "v.gguf"
    firs = vr_file(p, oracle_mod)
    c = pkg.Model(str(p)).config()
    assert (c.sample_rate, c.bins, c.pre_filter_start, c.pre_filter_stop, c.n_bands) == (44100, 640, 600, 640, 2)
    b = c.bands[1]
    assert (b.sample_rate, b.hop, b.n_fft, b.crop_start, b.crop_stop, b.hpf_start, b.hpf_stop) == \
        (44100, 512, 1024, 100, 513, 120, 100)
    got = {(c.firs[k].src_rate, c.firs[k].dst_rate): np.ctypeslib.as_array(c.firs[k].taps, (c.firs[k].n_taps,))
           for k in range(c.n_firs)}
    assert set(got) == {(11025, 44100), (44100, 11025)}
    for (s, d), taps in got.items():
        assert np.array_equal(taps, firs[f"resample.{s}.{d}"])


def test_bad_files(pkg, tmp_path):
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"NOPE" + b"\0" * 40)
    with pytest.raises(pkg.StemsError) as e:
        pkg.Model(str(bad))
    assert e.value.code == 4
    with pytest.raises(pkg.StemsError) as e:
        pkg.Model(str(tmp_path / "absent.gguf"))
    assert e.value.code == 5
    p = tmp_path / "short.gguf"
    htdemucs_file(p)
    p.write_bytes(p.read_bytes()[:60])
    with pytest.raises(pkg.StemsError):
        pkg.Model(str(p))
    q = tmp_path / "nokey.gguf"
    G.write(q, {"general.architecture": (G.STRING, "htdemucs")})
    with pytest.raises(pkg.StemsError) as e:
        pkg.Model(str(q)).config()
    assert e.value.code == 4 and "stems." in str(e.value)


# ---- plans from files, on the GPU -------------------------------------------------------------
@pytest.mark.gpu
def test_roformer_plan_from_file_separates_like_the_config(pkg, engine, tmp_path):
    import torch
    p = tmp_path / "r.gguf"
    sizes, freqs = roformer_file(p, pkg)
    n = 441 * 90 + 5
    a = engine.plan_from_model(pkg.Model(str(p)), n)
    b = engine.plan_roformer(n, sizes, freqs, chunk=441 * 40, num_overlap=4, zero_dc=True, complement=True)
    assert a.n_chunks == b.n_chunks and a.mask_floats == b.mask_floats
    mix = torch.from_numpy(np.random.default_rng(1).uniform(-1, 1, (2, n)).astype(np.float32)).cuda()
    mask = torch.randn(a.mask_floats, device="cuda")
    oa, ob = torch.empty(a.out_shape, device="cuda"), torch.empty(b.out_shape, device="cuda")
    a.separate(mix, mask, oa)
    b.separate(mix, mask, ob)
    torch.cuda.synchronize()
    assert torch.equal(oa, ob)


@pytest.mark.gpu
def test_vr_plan_from_file(pkg, engine, oracle_mod, tmp_path):
    import torch
    p = tmp_path / "v.gguf"
    vr_file(p, oracle_mod)
    n = 44100 * 2 + 3
    plan = engine.plan_from_model(pkg.Model(str(p)), n)
    params = oracle_mod.vr_params([dict(sr=b["sr"], hop=b["hl"], nfft=b["n_fft"], start=b["crop_start"],
                                        stop=b["crop_stop"], hp_start=b["hpf_start"], hp_stop=b["hpf_stop"],
                                        lp_start=b["lpf_start"], lp_stop=b["lpf_stop"]) for b in VR_BANDS],
                                  bins=640, pre_start=600, pre_stop=640)
    mix = np.random.default_rng(2).uniform(-0.5, 0.5, (2, n)).astype(np.float32)
    mask = np.random.default_rng(3).uniform(0, 1, plan.mask_shape).astype(np.float32)
    out = torch.empty(plan.out_shape, device="cuda")
    plan.separate(torch.from_numpy(mix).cuda(), torch.from_numpy(mask).cuda(), out)
    torch.cuda.synchronize()
    want = oracle_mod.vr_separate(params, mix, mask)
    got = out.cpu().numpy()
    for s in range(2):
        assert np.abs(got[s] - want[s]).max() / np.abs(want[s]).max() <= 1e-5
