"""The committed ncu summaries: each names the command that made it, and the per-kernel ones
carry the DRAM bytes per launch that bench.py reports as roofline.traffic."""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PROFILES = os.path.join(ROOT, "profiles")


def _files():
    return sorted(f for f in os.listdir(PROFILES) if f.endswith(".txt"))


@pytest.mark.parametrize("name", _files())
def test_summary_names_its_command(name):
    text = open(os.path.join(PROFILES, name)).read()
    assert "ncu " in text and "--clock-control none" in text, name
    assert "bench.py" in text, name


@pytest.mark.parametrize("name", [f for f in _files() if not f.startswith("launches_")])
def test_kernel_summary_traffic_line(name):
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    kernel, workload = re.match(r"(.+)_(cfg\d+|vr3band|io48k)\.txt$", name).groups()
    traffic = bench.profiled_traffic(kernel, workload)
    assert traffic is not None and traffic > 1e6, name
