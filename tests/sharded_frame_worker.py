"""torchrun worker for tests/test_multigpu_gpu.py (one process per GPU, NCCL): a 2-block tower with the
projection, one 13-crop frame sharded over the ranks (multigpu.ShardedFrame) against the whole frame on this
rank's GPU, and a crop batch through encode_sharded against single-GPU features.  Rank 0 prints one line."""
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from strix_halo_maxx_b200.config import TOWER  # noqa: E402
from strix_halo_maxx_b200.weights import tower_weights, crop_pixels  # noqa: E402
from strix_halo_maxx_b200.tower import VisionTower  # noqa: E402
from strix_halo_maxx_b200.multigpu import ShardedFrame, encode_sharded, local_crop_ids  # noqa: E402
from strix_halo_maxx_b200._lib import device_status  # noqa: E402


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        cfg = TOWER
        tower = VisionTower(tower_weights(cfg, seed=0, n_blocks=2), cfg, device=dev)
        crops = torch.from_numpy(crop_pixels(13, cfg, seed=1)).to(torch.bfloat16).to(dev)
        sf = ShardedFrame(tower, 13, cfg.ntok, cfg.width, dev)
        frame_ok = all(torch.equal(sf(crops), tower.frame(crops)) for _ in range(2))
        n_total, mb = 4 * world, 2
        ids = local_crop_ids(n_total, world, rank, mb)
        pix = torch.from_numpy(crop_pixels(n_total, cfg, seed=2)).to(torch.bfloat16).to(dev)
        feats = torch.empty(n_total, cfg.ntok, cfg.width, dtype=torch.bfloat16, device=dev)
        local_out = torch.empty(len(ids), cfg.ntok, cfg.width, dtype=torch.bfloat16, device=dev)
        encode_sharded(lambda p, out: tower.forward(p, out=out), pix[ids], feats, local_out, mb)
        gather_ok = torch.equal(feats, tower.forward(pix))
        ok = torch.tensor([1.0 if frame_ok and gather_ok and device_status() == 0 else 0.0], device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if rank == 0:
            print(f"SHARDED_OK {int(ok.item())} world={world} frame={frame_ok} gather={gather_ok}", flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
