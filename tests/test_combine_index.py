"""The combine kernels' index arithmetic replayed on the host (CPU only).

tests/combine_index/emulate.cpp compiles the library's own scheduler (csrc/plan.cu) for the
host with stubs for the GPU side; launch_plan runs unchanged and every combine launch it makes
is replayed sample by sample (combine_kernel4 for one or two stereo stems, combine_kernel for
the rest) over the GPU parity tests' plans and the five BASELINE configurations, at four
resident-CTA counts (so four tile sizes). It asserts:
  * every chunk whose output reaches a sample lies in the kernel's chunk range;
  * every clamp of combine_kernel4 (uc, tc, uc2, the complement's min(s, nv - 1)) leaves its
    index unchanged wherever the loaded value is used, and every such address is inside its
    buffer (weight tables, Y, Tr, mix, out).
Where combine_kernel4 reads a chunk's four samples as 16-byte vectors (all four inside the chunk,
none on a tile boundary's partial sums, aligned rows), it checks that those are the samples the
per-sample loop would use and that the vector loads are aligned and inside their buffers.
It also reports where an unguarded load would have left its buffer: the weight table read at
u = -3..-1 when a chunk's first output sample falls inside a thread's four samples (chunk steps
that are not a multiple of 4), and the complement's mix read past the track's end (lengths that
are not a multiple of 4).
"""
from __future__ import annotations

import os
import shutil
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


@pytest.fixture(scope="module")
def replay(tmp_path_factory, pkg):
    if not shutil.which("g++") or not os.path.exists(os.path.join(CUDA, "include", "cuda_runtime.h")):
        pytest.skip("needs g++ and the CUDA headers")
    d = tmp_path_factory.mktemp("combine_index")
    exe = d / "emulate"
    cmd = ["g++", "-std=c++17", "-O2", "-x", "c++", f"-I{CUDA}/include", f"-I{ROOT}/stems.cpp_b200/csrc",
           f"{ROOT}/stems.cpp_b200/csrc/plan.cu", "-x", "c++", f"{ROOT}/tests/combine_index/emulate.cpp",
           "-o", str(exe), f"-L{CUDA}/lib64", "-lcudart", f"-Wl,-rpath,{CUDA}/lib64"]
    subprocess.run(cmd, check=True, capture_output=True)
    ms, mf = pkg.bands.mel_bands()
    bs, bf = pkg.bands.bs_bands()
    files = []
    for name, a in (("ms", ms), ("mf", mf), ("bs", bs), ("bf", bf)):
        f = d / f"{name}.bin"
        np.asarray(a, np.int32).tofile(f)
        files.append(str(f))
    out = subprocess.run([str(exe), *files], check=True, capture_output=True, text=True, timeout=600).stdout
    rows = {}
    for line in out.splitlines():
        name, rest = line.split(" ", 1)
        kv = dict(x.split("=", 1) for x in rest.split(" "))
        rows.setdefault(name, []).append(kv)
    return rows


def test_every_plan_replayed(replay):
    assert len(replay) == 27
    for name, runs in replay.items():
        assert len(runs) == 4, name
        for kv in runs:
            assert int(kv["launches"]) >= 1, name


def test_no_index_leaves_its_buffer_where_used(replay):
    bad = [(name, kv["slots"], kv["first"]) for name, runs in replay.items() for kv in runs
           if int(kv["violations"]) != 0]
    assert not bad, bad


def test_unguarded_candidates(replay):
    """Where the guards matter: chunk starts inside a group of four (weight table at u < 0) in
    the test plans whose step is not a multiple of 4, and the complement's mix read past the
    end of a track whose length is not a multiple of 4. The benchmark configurations hit
    neither."""
    w = {n for n, runs in replay.items() if int(runs[0]["oob_unguarded_W"]) > 0}
    mix = {n for n, runs in replay.items() if int(runs[0]["mix"]) > 0}
    assert "rf_mel_ov4_pad" in w and "rf_mel_no_border_pad" in w
    assert "rf_bs_ov2_complement" in mix and "tfc_msst_dt32" in mix
    for n, runs in replay.items():
        if n.startswith("cfg"):
            for kv in runs:
                assert (int(kv["oob_unguarded_W"]), int(kv["Y"]), int(kv["Tr"]), int(kv["mix"])) == (0, 0, 0, 0), n
        for kv in runs:   # Y and Tr reads never leave their buffers, guarded or not
            assert int(kv["Y"]) == 0 and int(kv["Tr"]) == 0, n


def test_vector_path_taken_on_the_benchmark_plans(replay):
    for name in ("cfg1_mel_roformer_60s", "cfg2_bs_roformer_180s", "cfg3_tfc_180s"):
        for kv in replay[name]:
            assert int(kv["vec"]) > 0, name
