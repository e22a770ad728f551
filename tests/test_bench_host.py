"""Host logic of bench.py without a GPU: how streams are dealt to ranks
(weak scaling by default, the fixed-job split on request) and where the
roofline's HBM peak comes from."""
import json

import bench


def test_weak_scaling_gives_every_rank_its_own_streams():
    world, n = 4, 64
    shards = [bench.streams_for_rank(n, world, r, split=False) for r in range(world)]
    assert all(len(s) == n for s in shards)
    ids = [i for s in shards for i in s]
    assert sorted(ids) == list(range(n * world))  # distinct seeds across ranks


def test_split_deals_one_job_round_robin():
    world, n = 8, 64
    shards = [bench.streams_for_rank(n, world, r, split=True) for r in range(world)]
    assert all(len(s) == n // world for s in shards)
    assert sorted(i for s in shards for i in s) == list(range(n))
    assert bench.streams_for_rank(1, 2, 1, split=True) == []  # bench refuses this before loading


def test_one_gpu_is_the_same_job_either_way():
    assert bench.streams_for_rank(64, 1, 0, split=False) == bench.streams_for_rank(64, 1, 0, split=True)


def test_peak_prefers_the_pod_file_then_the_build_copy(tmp_path, monkeypatch):
    monkeypatch.setattr(bench, "ROOT", str(tmp_path))
    assert bench.peaks() == (6650.0, "fallback")
    (tmp_path / "rai_b200").mkdir()
    (tmp_path / "rai_b200" / "measured_peaks.json").write_text(json.dumps({"hbm_gbs": 6400.0}))
    assert bench.peaks() == (6400.0, "measured")
    (tmp_path / "MEASURED_PEAKS.json").write_text(json.dumps({"hbm_gbs": 6553.0}))
    assert bench.peaks() == (6553.0, "measured")
    (tmp_path / "MEASURED_PEAKS.json").write_text("{not json")
    assert bench.peaks() == (6400.0, "measured")
