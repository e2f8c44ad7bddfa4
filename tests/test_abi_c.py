"""The C ABI from compiled hosts, as the reference's own tests/abi_test.c checks libstems:
  * tests/abi/abi_test.c (C): dlopen + dlsym only, statuses, NULL handling, undersized structs;
    on a GPU also one separation from host buffers against the CPU oracle;
  * tests/abi/adapter_test.cpp (C++): include/stems_gpu.hpp, the Separator-shaped adapter whose
    RoFormer::separate code INTEGRATION.md shows, linked against the library; on a GPU the same
    separation against the oracle and a cancelled one."""
from __future__ import annotations

import os
import shutil
import subprocess

import numpy as np
import pytest

from common import synth_audio, synth_mask

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def abi_test(tmp_path_factory, pkg):
    if not shutil.which("gcc"):
        pytest.skip("needs gcc")
    exe = tmp_path_factory.mktemp("abi") / "abi_test"
    subprocess.run(["gcc", "-std=c11", "-O1", "-Wall", "-Werror", f"-I{ROOT}/include", f"{ROOT}/tests/abi/abi_test.c",
                    "-o", str(exe), "-ldl", "-lm"], check=True, capture_output=True, text=True)
    return str(exe)


@pytest.fixture(scope="module")
def adapter_test(tmp_path_factory, pkg):
    if not shutil.which("g++"):
        pytest.skip("needs g++")
    lib = pkg.library_path()
    exe = tmp_path_factory.mktemp("adapter") / "adapter_test"
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror", f"-I{ROOT}/include",
                    f"{ROOT}/tests/abi/adapter_test.cpp", "-o", str(exe), lib,
                    f"-Wl,-rpath,{os.path.dirname(lib)}"], check=True, capture_output=True, text=True)
    return str(exe)


def _case(pkg, oracle_mod, d):
    """A small Mel-RoFormer separation: inputs and the oracle's result, as files."""
    sizes, freqs = pkg.bands.mel_bands()
    chunk, nov = 441 * 40, 4
    n = 441 * 90 + 321
    p = oracle_mod.rf_params(sizes, freqs, chunk=chunk, num_overlap=nov, threads=8)
    n_chunks = oracle_mod.rf_n_chunks(p, n)
    mix = synth_audio(81, n)
    mask = synth_mask(82, n_chunks * int(sizes.sum()) * 4 * (chunk // 441 + 1), 0.5)
    want = oracle_mod.rf_separate(p, mix, mask)
    (d / "case.txt").write_text(f"{n} {chunk} {nov} {sizes.size}\n")
    np.asarray(sizes, np.int32).tofile(d / "sizes.i32")
    np.asarray(freqs, np.int32).tofile(d / "freqs.i32")
    mix.astype(np.float32).tofile(d / "mix.f32")
    mask.astype(np.float32).tofile(d / "mask.f32")
    want.astype(np.float32).tofile(d / "want.f32")
    return str(d)


def test_cpp_adapter_without_gpu_work(adapter_test):
    r = subprocess.run([adapter_test], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all passed" in r.stdout


@pytest.mark.gpu
def test_cpp_adapter_separation_matches_oracle(adapter_test, pkg, oracle_mod, tmp_path):
    r = subprocess.run([adapter_test, _case(pkg, oracle_mod, tmp_path)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all passed" in r.stdout


def test_c_host_without_gpu_work(abi_test, pkg):
    r = subprocess.run([abi_test, pkg.library_path()], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all passed" in r.stdout


@pytest.mark.gpu
def test_c_host_separation_matches_oracle(abi_test, pkg, oracle_mod, tmp_path):
    r = subprocess.run([abi_test, pkg.library_path(), _case(pkg, oracle_mod, tmp_path)], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all passed" in r.stdout
