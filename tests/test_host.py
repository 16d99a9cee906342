"""Host-side logic on CPU: seeded weights, FLOP accounting, crop sharding, and the 2-rank all-gather path
over the gloo backend (the NCCL path runs the same code on GPUs)."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from strix_halo_maxx_b200.config import TowerConfig, TapNextConfig
from strix_halo_maxx_b200 import weights as wg
from strix_halo_maxx_b200.multigpu import local_crop_ids, encode_sharded, frame_crop_slice, ShardedFrame


def test_weights_are_deterministic_and_independent():
    cfg = TowerConfig()
    a = wg.tower_weights(cfg, seed=0, n_blocks=1)
    b = wg.tower_weights(cfg, seed=0, n_blocks=1)
    c = wg.tower_weights(cfg, seed=1, n_blocks=1)
    for k in a:
        assert np.array_equal(a[k], b[k])
    assert not np.array_equal(a["blocks.0.qkv_w"], c["blocks.0.qkv_w"])
    assert abs(float(a["blocks.0.fc1_w"].std()) - 0.02) < 1e-3
    assert not a["blocks.0.qkv_b"].any() and (a["blocks.0.ln1_w"] == 1).all()


def test_flop_accounting_matches_survey():
    f = TowerConfig().flops_per_crop()
    assert abs(f["total"] / 1e9 - 666.45) < 0.01
    assert abs(TapNextConfig().flops_per_frame() / 1e9 - 314.4) < 0.5


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_crop_sharding_covers_every_crop_once(world):
    ids = sorted(i for r in range(world) for i in local_crop_ids(1040, world, r, 130))
    assert ids == list(range(1040))


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n_total, mb, T, W = 16, 2, 3, 4
        ids = local_crop_ids(n_total, world, rank, mb)
        pix = torch.tensor(ids, dtype=torch.float32)

        def forward(p, out):   # stand-in tower: feature = crop id broadcast
            out.copy_(p[:, None, None].expand(-1, T, W))
        feats = torch.full((n_total, T, W), -1.0)
        local = torch.empty(len(ids), T, W)
        encode_sharded(forward, pix, feats, local, mb)
        q.put((rank, bool(torch.equal(feats[:, 0, 0], torch.arange(n_total, dtype=torch.float32)))))
    finally:
        dist.destroy_process_group()


def test_two_rank_all_gather_over_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}


def _rank_leaving(rank, world, port, q):
    """Rank 1 leaves between steps, before the first all-gather (a host-side injected failure); rank 0 must get
    an error from its collective instead of waiting for good."""
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=15))
    if rank == 1:
        q.put((rank, "left"))
        q.close()
        q.join_thread()  # the message is sent before the process goes
        os._exit(3)
    try:
        n_total, mb, T, W = 16, 2, 3, 4
        ids = local_crop_ids(n_total, world, rank, mb)
        pix = torch.tensor(ids, dtype=torch.float32)
        feats = torch.empty(n_total, T, W)
        local = torch.empty(len(ids), T, W)
        encode_sharded(lambda p, out: out.copy_(p[:, None, None].expand(-1, T, W)), pix, feats, local, mb)
        q.put((rank, "completed"))
    except Exception as e:  # the collective's error: the peer is gone
        q.put((rank, "error " + type(e).__name__))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_a_rank_leaving_before_the_all_gather_ends_the_other_ranks_collective_with_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 30500 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_rank_leaving, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = dict(q.get(timeout=120) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert res[1] == "left"
    assert res[0].startswith("error"), res[0]
    assert procs[1].exitcode == 3


@pytest.mark.parametrize("n,world", [(13, 1), (13, 2), (13, 4), (13, 8), (3, 4), (1, 2)])
def test_frame_crop_slices_cover_the_frame_once_in_order(n, world):
    got = []
    for r in range(world):
        lo, hi, per = frame_crop_slice(n, world, r)
        assert 0 <= hi - lo <= per and (hi == lo or lo == r * per)
        got.extend(range(lo, hi))
    assert got == list(range(n))


class _FakeTower:
    """Stand-in for VisionTower on the CPU: the features of crop i are the value i; the frame's output lists the
    first feature of every crop it was given, in order."""
    T, W = 3, 4

    def forward(self, p, out=None):
        out = torch.empty(p.shape[0], self.T, self.W) if out is None else out
        out.copy_(p[:, None, None].expand(-1, self.T, self.W))
        return out

    def frame_from_features(self, feats):
        return feats[:, 0, 0].clone()


def _rank_frame(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        res = []
        for n in (13, 3, 1):
            sf = ShardedFrame(_FakeTower(), n, _FakeTower.T, _FakeTower.W, "cpu", dtype=torch.float32)
            crops = torch.arange(n, dtype=torch.float32) + 100
            res.append(bool(torch.equal(sf(crops), crops)))
        q.put((rank, all(res)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_frame_gathers_every_crop_in_order_on_every_rank(world):
    """ShardedFrame over gloo ranks: every rank ends with the features of all crops of the frame, in crop order,
    also when the crops do not divide evenly and some ranks hold fewer (or none: 1 crop over 2 or 3 ranks)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 31500 + world * 10 + (os.getpid() % 500)
    procs = [ctx.Process(target=_rank_frame, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = dict(q.get(timeout=120) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert res == {r: True for r in range(world)}
