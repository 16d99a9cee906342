"""Crop-batch data parallelism over GPUs: one process per GPU (torchrun), every GPU
runs whole towers on its slice of the crops, and the 729 x 1152 features are all-gathered with NCCL over
NVLink.  The reference has no multi-device path (a single iGPU); this is the B200 build's own.

Crop order: the batch is cut into chunks of world * mb crops; in chunk j, rank r owns crops
[j*world*mb + r*mb, j*world*mb + (r+1)*mb).  So after chunk j every rank has a contiguous slice of
the global output and one all_gather_into_tensor fills rows [j*world*mb, (j+1)*world*mb) in crop
order.  The collective of chunk j is asynchronous and runs while chunk j+1 is computed.

One frame's latency (BASELINE config 2 on N GPUs, ShardedFrame): the frame's 13 crops are cut the same way
(ceil(13 / N) consecutive crops per rank), one all-gather puts every crop's features on every rank in crop
order, and every rank runs the combine and the projection, so each ends with the whole frame's output.
"""
import torch
import torch.distributed as dist


def local_crop_ids(n_total, world, rank, mb):
    """Global crop ids of this rank, in the order its chunks are processed."""
    if n_total % (world * mb):
        raise ValueError(f"{n_total} crops do not split into chunks of {world} ranks x {mb}")
    ids = []
    for j in range(n_total // (world * mb)):
        base = j * world * mb + rank * mb
        ids.extend(range(base, base + mb))
    return ids


def encode_sharded(forward, pix_local, feats_all, local_out, mb, group=None, exposed=None):
    """forward(pix_chunk, out=chunk_out) computes one chunk; pix_local [n_local, ...] holds this rank's
    crops in local_crop_ids order; local_out [n_local, T, W] receives this rank's features and
    feats_all [n_total, T, W] the gathered features of every rank.  Returns feats_all.
    exposed: optional list; with more than one rank it gets a pair of CUDA events recorded on the current
    stream around the final waits for the collectives, i.e. the all-gather time not hidden behind compute."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    n_local = pix_local.shape[0]
    if n_local % mb:
        raise ValueError(f"{n_local} local crops are not a multiple of the micro-batch {mb}")
    works = []
    for j in range(n_local // mb):
        sl = slice(j * mb, (j + 1) * mb)
        if world == 1:
            forward(pix_local[sl], out=feats_all[sl])
            continue
        forward(pix_local[sl], out=local_out[sl])
        dst = feats_all[j * world * mb:(j + 1) * world * mb]
        works.append(dist.all_gather_into_tensor(dst, local_out[sl], group=group, async_op=True))
    if exposed is not None and works:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
    for w in works:
        w.wait()
    if exposed is not None and works:
        e1.record()
        exposed.append((e0, e1))
    return feats_all


class HostPipeline:
    """End-to-end public entry: crops in pinned host memory -> features in pinned host memory, with the
    host<->device copies overlapped with the towers: chunk j+1 is copied in on one stream while chunk j is
    computed, and chunk j's features are copied out on a third stream.  With more than one rank the
    features are also all-gathered on the devices (encode_sharded's crop order)."""

    def __init__(self, tower, n_local, mb):
        self.tower, self.n_local, self.mb = tower, n_local, mb
        cfg, dev = tower.cfg, tower.dev
        self.stage = [torch.empty(mb, cfg.in_ch, cfg.img, cfg.img, dtype=torch.bfloat16, device=dev) for _ in range(2)]
        self.local_out = torch.empty(n_local, cfg.ntok, cfg.width, dtype=torch.bfloat16, device=dev)
        self.s_in = torch.cuda.Stream(dev)
        self.s_out = torch.cuda.Stream(dev)

    def h2d_bytes(self):
        return self.n_local * self.stage[0][0].numel() * 2

    def d2h_bytes(self):
        return self.local_out.numel() * 2

    def run(self, pix_host, out_host, feats_all=None, group=None):
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        mb, n = self.mb, self.n_local // self.mb
        main = torch.cuda.current_stream()
        self.s_in.wait_stream(main)
        self.s_out.wait_stream(main)
        consumed = [None, None]
        ready = [None] * n

        def h2d(j):
            with torch.cuda.stream(self.s_in):
                if consumed[j % 2] is not None:
                    self.s_in.wait_event(consumed[j % 2])
                self.stage[j % 2].copy_(pix_host[j * mb:(j + 1) * mb], non_blocking=True)
                e = torch.cuda.Event()
                e.record(self.s_in)
                return e
        works = []
        ready[0] = h2d(0)
        for j in range(n):
            if j + 1 < n:
                ready[j + 1] = h2d(j + 1)
            main.wait_event(ready[j])
            sl = slice(j * mb, (j + 1) * mb)
            self.tower.forward(self.stage[j % 2], out=self.local_out[sl])
            consumed[j % 2] = torch.cuda.Event()
            consumed[j % 2].record(main)
            if world > 1:
                works.append(dist.all_gather_into_tensor(feats_all[j * world * mb:(j + 1) * world * mb],
                                                         self.local_out[sl], group=group, async_op=True))
            with torch.cuda.stream(self.s_out):
                self.s_out.wait_event(consumed[j % 2])
                out_host[sl].copy_(self.local_out[sl], non_blocking=True)
        for w in works:
            w.wait()
        main.wait_stream(self.s_out)
        main.wait_stream(self.s_in)
        return out_host


def frame_crop_slice(n_crops, world, rank):
    """(lo, hi, per_rank): the crops [lo, hi) of one n_crops-crop frame that `rank` computes when the frame is
    sharded over `world` ranks, ceil(n_crops / world) consecutive crops each (the last ranks fewer, maybe none)."""
    per = -(-n_crops // world)
    lo = min(rank * per, n_crops)
    return lo, min(lo + per, n_crops), per


class ShardedFrame:
    """One multi-crop frame with its crops sharded over the ranks, for latency: rank r runs
    the tower on crops frame_crop_slice(n, world, r), the [per_rank, T, W] features of every rank are
    all-gathered (rank-major, so rows 0..n-1 are the crops in order; a rank with fewer crops pads its block,
    and the padding rows land after row n-1), and every rank combines and projects the frame
    (tower.frame_from_features).  Per-crop features do not depend on which crops share a launch, so the
    result equals tower.frame on one GPU.  `tower` needs forward(pix, out=) and frame_from_features(feats)."""

    def __init__(self, tower, n_crops, T, W, device, group=None, dtype=torch.bfloat16):
        self.tower, self.n, self.group = tower, n_crops, group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.lo, self.hi, per = frame_crop_slice(n_crops, self.world, rank)
        self.local = torch.zeros(per, T, W, dtype=dtype, device=device)
        self.gathered = torch.empty(self.world * per, T, W, dtype=dtype, device=device)

    def __call__(self, crops):
        """crops [n_crops, ...]: the whole frame (each rank reads only its own slice) -> the frame's output."""
        if self.world == 1:
            return self.tower.frame_from_features(self.tower.forward(crops))
        if self.hi > self.lo:
            self.tower.forward(crops[self.lo:self.hi], out=self.local[:self.hi - self.lo])
        dist.all_gather_into_tensor(self.gathered, self.local, group=self.group)
        return self.tower.frame_from_features(self.gathered[:self.n])
