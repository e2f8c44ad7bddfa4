"""The multi-GPU host logic on CPU: two gloo ranks split a batch of tracks round-robin, each
separates its share (the CPU oracle stands in for the GPU), and the union equals the serial
result; the max-over-ranks timing reduction used by bench.py returns the slowest rank."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n_tracks, length, out_dir):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "tests")]
    import torch.distributed as dist
    import __graft_entry__
    import oracle
    from common import synth_audio, synth_mask
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pkg = __graft_entry__.load_package()
        sizes, freqs = pkg.bands.bs_bands()
        p = oracle.rf_params(sizes, freqs, chunk=441 * 20, num_overlap=2)
        mine = pkg.sharding.tracks_for_rank(n_tracks, rank, world)
        for k in mine:
            mix = synth_audio(100 + k, length)
            n_mask = oracle.rf_n_chunks(p, length) * int(sizes.sum()) * 4 * 21
            out = oracle.rf_separate(p, mix, synth_mask(200 + k, n_mask, 0.5))
            np.save(os.path.join(out_dir, f"track{k}.npy"), out)
        slowest = pkg.sharding.max_over_ranks(float(rank + 1))
        np.save(os.path.join(out_dir, f"max{rank}.npy"), np.array([slowest]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n,world", [(1000, 1), (1000, 3), (7, 8), (2646000, 8)])
def test_sample_ranges_tile_the_track(pkg, n, world):
    got = [pkg.sharding.sample_range_for_rank(n, r, world) for r in range(world)]
    assert got[0][0] == 0 and got[-1][1] == n
    assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
    assert max(e - b for b, e in got) - min(e - b for b, e in got) <= 1


def test_round_robin_split_covers_every_track_once(pkg):
    world, n = 3, 10
    got = sorted(k for r in range(world) for k in pkg.sharding.tracks_for_rank(n, r, world))
    assert got == list(range(n))
    with pytest.raises(ValueError):
        pkg.sharding.tracks_for_rank(n, 3, 3)


def test_two_gloo_ranks_match_serial(tmp_path, oracle_mod, pkg):
    from common import synth_audio, synth_mask
    world, n_tracks, length = 2, 5, 441 * 30
    mp.start_processes(_worker, args=(world, _free_port(), n_tracks, length, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    sizes, freqs = pkg.bands.bs_bands()
    p = oracle_mod.rf_params(sizes, freqs, chunk=441 * 20, num_overlap=2)
    for k in range(n_tracks):
        mix = synth_audio(100 + k, length)
        n_mask = oracle_mod.rf_n_chunks(p, length) * int(sizes.sum()) * 4 * 21
        want = oracle_mod.rf_separate(p, mix, synth_mask(200 + k, n_mask, 0.5))
        assert np.array_equal(np.load(tmp_path / f"track{k}.npy"), want)
    for r in range(world):
        assert float(np.load(tmp_path / f"max{r}.npy")[0]) == float(world)
