"""Host side of tensor / expert parallelism, without a GPU: the shard rules
of rai_gpu_model_create_tp (checked before any device work) and the handle
exchange of rai_b200.tp.connect over a 2-rank gloo group."""
import os
import socket

import pytest

from rai_b200 import native


def _create_tp(path, rank, world):
    import ctypes as C
    import numpy as np
    blob = np.fromfile(path, dtype=np.uint8)
    h = C.c_void_p()
    rc = native.lib().rai_gpu_model_create_tp(blob.ctypes.data_as(C.c_void_p), blob.size, 0, rank, world,
                                              C.byref(h))
    if rc == native.RAI_OK:
        native.lib().rai_gpu_model_destroy(h)
    return rc


def test_tp_shard_rules(tiny_model_paths):
    # tiny-llama: 8 heads, 2 KV heads, head_dim 32, ff 512, group 128.
    p = tiny_model_paths["tiny-llama"]
    assert _create_tp(p, 0, 3) == native.RAI_ERR_INVALID          # size not 1/2/4/8
    assert _create_tp(p, 2, 2) == native.RAI_ERR_INVALID          # rank out of range
    assert _create_tp(p, 0, 4) == native.RAI_ERR_UNSUPPORTED      # 2 KV heads over 4 ranks
    assert "KV heads" in native.last_error()
    # Mixture of experts (8 experts) splits by experts instead: the shard rules
    # pass and only the device step remains (no device here -> device error).
    assert _create_tp(tiny_model_paths["tiny-moe"], 1, 2) in (native.RAI_OK, native.RAI_ERR_DEVICE)
    # tiny-qwen: ff 384 = 3 groups, not whole groups per rank at 2 ranks.
    assert _create_tp(tiny_model_paths["tiny-qwen"], 0, 2) == native.RAI_ERR_UNSUPPORTED
    assert "ff slice" in native.last_error()


class _FakeShard:
    """Stands in for RaiModel: records the handles connect() passes."""

    def __init__(self, rank, world):
        self.tp_rank, self.tp_size = rank, world
        self.connected = None

    def tp_handle(self):
        return bytes([self.tp_rank + 1]) * 64

    def tp_connect(self, handles):
        self.connected = list(handles)


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from rai_b200 import tp
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    m = _FakeShard(rank, world)
    tp.connect(m)
    q.put((rank, m.connected))
    try:
        tp.connect(_FakeShard((rank + 1) % world, world))
        q.put((rank, "no error"))
    except ValueError as e:
        q.put((rank, str(e)))
    dist.destroy_process_group()


def test_connect_exchanges_handles_in_rank_order():
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in range(4)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    handles = [v for r, v in got if isinstance(v, list)]
    assert len(handles) == 2
    for h in handles:
        assert h == [bytes([1]) * 64, bytes([2]) * 64]
    errors = [v for r, v in got if isinstance(v, str)]
    assert all("rank" in e for e in errors) and len(errors) == 2
