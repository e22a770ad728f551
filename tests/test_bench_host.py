"""Host logic of bench.py without a GPU: how streams are dealt to ranks
(one job dealt over the ranks by default, weak scaling on request), the
config object both arms print, the reference arm's model writer and where
the roofline's peak and traffic come from."""
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


class _Args:
    def __init__(self, weak=False):
        self.weak = weak


def test_config_two_deals_one_job_by_default(monkeypatch):
    monkeypatch.setattr(bench, "CFG", dict(bench.CONFIGS["tinyllama"]))
    js = bench.job_shape(_Args(), 8)
    assert js == {"mode": "dp", "weak": False, "split": True, "streams": 64, "per_gpu": 8}
    weak = bench.job_shape(_Args(weak=True), 8)
    assert weak["weak"] and weak["streams"] == 512 and weak["per_gpu"] == 64


def test_tensor_and_replica_modes(monkeypatch):
    monkeypatch.setattr(bench, "CFG", dict(bench.CONFIGS["llama8b"]))
    assert bench.job_shape(_Args(), 4)["mode"] == "tp"
    assert bench.job_shape(_Args(), 1)["mode"] == "dp"
    monkeypatch.setattr(bench, "CFG", dict(bench.CONFIGS["olmoe"]))
    assert bench.job_shape(_Args(), 2)["mode"] == "ep"
    monkeypatch.setattr(bench, "CFG", dict(bench.CONFIGS["qwen"]))
    js = bench.job_shape(_Args(), 4)
    assert js["weak"] and js["streams"] == 4  # one replica stream per GPU


def test_both_arms_print_the_same_config(monkeypatch):
    monkeypatch.setattr(bench, "CFG", dict(bench.CONFIGS["tinyllama"]))
    for world in (1, 2, 8):
        a = bench.config_object(_Args(), world)
        assert a == bench.config_object(_Args(), world)
        assert a["streams"] == 64 and a["k"] == 8 and a["streams_per_gpu"] == 64 // world


def test_oracle_writer_matches_the_product_writer(tmp_path):
    """The reference arm writes its model with the oracle's copy of the
    writer; both must produce the same bytes for the same preset and seed."""
    from oracle import oracle as O
    from rai_b200 import convert
    O.build()
    for name in ("tiny-llama", "tiny-qwen", "tiny-moe", "tiny-llama3"):
        a, b = tmp_path / f"{name}.a", tmp_path / f"{name}.b"
        convert.write_synthetic(str(a), name, seed=11, fast=True)
        convert.write_synthetic(str(b), name, seed=11, backend=O.WriterBackend)
        assert a.read_bytes() == b.read_bytes(), name


def test_profile_traffic_lookup_picks_the_nearest_capture(tmp_path, monkeypatch):
    monkeypatch.setattr(bench, "ROOT", str(tmp_path))
    assert bench.gemm_traffic_from_profile(9) is None
    (tmp_path / "profiles").mkdir()
    (tmp_path / "profiles" / "w4a8_gemm_tinyllama_gateup_m9.md").write_text("M: 9\ndram_bytes_per_launch: 100\n")
    (tmp_path / "profiles" / "w4a8_gemm_tinyllama_gateup_m104.md").write_text("M: 104\ndram_bytes_per_launch: 300\n")
    assert bench.gemm_traffic_from_profile(9) == 100
    assert bench.gemm_traffic_from_profile(96) == 300
