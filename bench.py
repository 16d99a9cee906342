#!/usr/bin/env python
"""Vision-tower crop-batch throughput on 1..8 B200.

A step = 1040 crops (80 frames x 13) through the 27-block moondream2-style tower of config 1 (patch-
embed, 27 pre-LN blocks, post-LN), sharded evenly over the ranks, each rank working in chunks of
130 crops, with the 729 x 1152 bf16 features all-gathered over NVLink by NCCL (async, overlapped with
the next chunk).  Total work is fixed as N grows ("scaling": "strong").  Synthetic seeded inputs:
pixels U[-1, 1], weights N(0, 0.02) (no checkpoints offline).

value  : crops/s of the whole job with the pixels already in HBM (CUDA events, max over ranks).
e2e    : crops/s through the public host-buffer API (strix_halo_maxx_b200.multigpu.HostPipeline):
         pinned host pixels -> H2D -> towers -> all-gather -> D2H of this rank's features, every step.
roofline: the tcgen05 GEMM kernel (all its launches in the timed region, CUDA events on the launching
         stream): achieved = algorithmic GEMM FLOPs / summed launch time, against the measured sustained
         cuBLAS bf16 peak (MEASURED_PEAKS.json).
cpu_baseline: the CPU fp32 oracle (a port of md2fast.FastMD2._vision) on one crop, rank 0 at N=1.
--impl reference: the same CPU oracle as the reference arm, a bounded sample per step.

Run:  python bench.py [--gpus N --steps K --warmup W]   (N > 1 under torchrun, one rank per GPU)
"""
import argparse
import contextlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "vision-tower crops/sec and ms per 13-crop frame at 1/2/4/8 B200; % bf16 TC peak"
UNIT = "crops/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="vt", choices=["vt", "reference"])
    ap.add_argument("--crops", type=int, default=1040)
    ap.add_argument("--mb", type=int, default=130,
                    help="crops per chunk and rank (at most; with N > 1 capped so every rank has >= 2 chunks)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-frame", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer pass (profiling runs)")
    ap.add_argument("--no-fold", action="store_true", help="LayerNorm as separate passes instead of folded into GEMMs")
    ap.add_argument("--no-tapnext", action="store_true",
                    help="skip the TAPNext per-frame step and text-decoder timings (N=1 only)")
    ap.add_argument("--tapnext-only", action="store_true",
                    help="profiling runs: only the config-3 and TAPNext++ per-frame steps, printed as one JSON line")
    return ap.parse_args()


def env_rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("bf16_tflops_sustained", 1400.0), d.get("bf16_tflops", 1590.0), d.get("hbm_gbs", 6650.0), "measured"
    return 1400.0, 1590.0, 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampled every 200 ms during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-i", str(self.idx), "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None
        return self

    def __exit__(self, *a):
        if self.p is not None:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()
        self.f.flush()

    def summary(self):
        rows = []
        for line in open(self.f.name):
            p = [x.strip() for x in line.split(",")]
            if len(p) >= 9 and p[1].replace(".", "").isdigit():
                rows.append(p)
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


class OpTimer:
    """CUDA events around every op launch of the tower (on the launching stream)."""

    def __init__(self):
        self.rec = []

    @contextlib.contextmanager
    def __call__(self, name, flops):
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        yield
        e.record()
        self.rec.append((name, flops, s, e))

    def summary(self):
        out = {}
        for name, flops, s, e in self.rec:
            d = out.setdefault(name, {"launches": 0, "ms": 0.0, "flops": 0})
            d["launches"] += 1
            d["ms"] += s.elapsed_time(e)
            d["flops"] += flops
        return out


def cpu_oracle_rate(W, cfg, n_crops, reps):
    """Crops/s of the CPU fp32 oracle (port of FastMD2._vision's tower) on all host threads."""
    from oracle import tower_ref
    from strix_halo_maxx_b200.weights import crop_pixels
    torch.set_num_threads(os.cpu_count() or 1)
    pix = torch.from_numpy(crop_pixels(n_crops, cfg, seed=1))
    tower_ref.tower(pix, W, cfg)             # warm-up
    ts = []
    for _ in range(reps):
        t = time.perf_counter()
        tower_ref.tower(pix, W, cfg)
        ts.append(time.perf_counter() - t)
    return n_crops / statistics.median(ts), torch.get_num_threads()


def run_reference(a):
    rank, world, _ = env_rank()
    if rank != 0:
        return
    from strix_halo_maxx_b200.config import TOWER
    from strix_halo_maxx_b200.weights import tower_weights, crop_pixels
    from oracle import tower_ref
    torch.set_num_threads(os.cpu_count() or 1)
    W = tower_weights(TOWER, seed=0, projection=False)
    pix = torch.from_numpy(crop_pixels(1, TOWER, seed=1))
    for _ in range(a.warmup):
        tower_ref.tower(pix, W, TOWER)
    t0 = time.perf_counter()
    for _ in range(a.steps):
        tower_ref.tower(pix, W, TOWER)
    dt = time.perf_counter() - t0
    v = a.steps / dt
    sample = f"1 crop per step (27 blocks + post-LN, fp32 torch CPU oracle, port of md2fast.FastMD2._vision) of the {a.crops}-crop workload"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": 1000 * dt / a.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded U[-1,1] pixels, N(0,0.02) weights)",
        "config": {"workload": f"config 4 ({a.crops} crops through the 27-block tower), bounded CPU sample",
                   "crops_per_step": 1},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}), flush=True)


def run_e2e(a, tower, n_local, mb, pix_host, feats_all, local_out, dev, world, barrier, max_over_ranks):
    """Crops/s through HostPipeline.run: pinned host pixels in, pinned host features out, every step."""
    from strix_halo_maxx_b200.multigpu import HostPipeline
    cfg = tower.cfg
    pipe = HostPipeline(tower, n_local, mb)
    out_host = torch.empty(n_local, cfg.ntok, cfg.width, dtype=torch.bfloat16).pin_memory()
    pipe.run(pix_host, out_host, feats_all)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(a.steps):
        pipe.run(pix_host, out_host, feats_all)
    f1.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(f0.elapsed_time(f1))
    # bytes of the whole job (every rank copies its own crops in and its features out)
    e2e = {"value": a.crops * a.steps / (e2e_ms / 1000.0), "unit": UNIT, "h2d_bytes_per_step": pipe.h2d_bytes() * world,
           "d2h_bytes_per_step": pipe.d2h_bytes() * world, "h2d_bytes_per_step_per_rank": pipe.h2d_bytes(),
           "api": "strix_halo_maxx_b200.multigpu.HostPipeline.run"}
    # the e2e output must equal the device-resident path
    e2e_ok = bool(torch.equal(out_host[:mb].to(dev), (local_out if world > 1 else feats_all)[:mb]))

    return e2e, e2e_ok


def run_vt(a):
    import torch.distributed as dist
    from datetime import timedelta
    from strix_halo_maxx_b200.config import TOWER
    from strix_halo_maxx_b200.weights import tower_weights, crop_pixels
    from strix_halo_maxx_b200.tower import VisionTower
    from strix_halo_maxx_b200.multigpu import local_crop_ids, encode_sharded, HostPipeline, ShardedFrame
    from strix_halo_maxx_b200 import ops
    from strix_halo_maxx_b200._lib import device_status

    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=300),
                                device_id=dev)
    cfg = TOWER
    # every rank gets at least two chunks when N > 1, so the all-gather of a chunk overlaps the next one's
    # compute (130 crops per chunk up to N = 4, 65 at N = 8)
    mb = min(a.mb, a.crops // world if world == 1 else max(1, a.crops // (2 * world)))
    ids = local_crop_ids(a.crops, world, rank, mb)
    n_local = len(ids)

    W = tower_weights(cfg, seed=0, projection=not a.no_frame)
    tower = VisionTower(W, cfg, device=dev, fold_ln=not a.no_fold)

    # this rank's crops, chunk by chunk (ids are runs of mb consecutive crops)
    pix_host = torch.empty(n_local, 3, cfg.img, cfg.img, dtype=torch.bfloat16).pin_memory()
    for j in range(n_local // mb):
        pix_host[j * mb:(j + 1) * mb] = torch.from_numpy(crop_pixels(mb, cfg, seed=1, first=ids[j * mb])).to(torch.bfloat16)
    pix_dev = pix_host.to(dev)
    feats_all = torch.empty(a.crops, cfg.ntok, cfg.width, dtype=torch.bfloat16, device=dev)
    local_out = torch.empty(n_local, cfg.ntok, cfg.width, dtype=torch.bfloat16, device=dev) if world > 1 else None
    fwd = lambda p, out: tower.forward(p, out=out)   # noqa: E731

    exposed = []

    def step():
        encode_sharded(fwd, pix_dev, feats_all, local_out, mb, exposed=exposed)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    device_status(clear=True)
    exposed.clear()

    # ---------------- timed: device-resident inputs
    timer = OpTimer()
    tower.op_timer = timer
    phys = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")
    gpu_index = phys[local] if len(phys) > local and phys[local].strip().isdigit() else str(local)
    l0 = ops.LAUNCHES
    barrier()
    torch.cuda.synchronize()
    with Clocks(gpu_index) as clk:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
    barrier()
    launches = ops.LAUNCHES - l0
    ms = max_over_ranks(e0.elapsed_time(e1))
    ag_exposed = max_over_ranks(sum(s.elapsed_time(e) for s, e in exposed) / a.steps) if world > 1 else 0.0
    tower.op_timer = None
    ops_summary = timer.summary()
    clocks = clk.summary()
    status = device_status(clear=True)
    value = a.crops * a.steps / (ms / 1000.0)

    gemm_ms = sum(v["ms"] for k, v in ops_summary.items() if k.startswith("gemm_"))
    gemm_fl = sum(v["flops"] for k, v in ops_summary.items() if k.startswith("gemm_"))
    gemm_n = sum(v["launches"] for k, v in ops_summary.items() if k.startswith("gemm_"))
    sustained, burst, hbm, src = peaks()
    achieved = gemm_fl / (gemm_ms / 1000.0) / 1e12
    traffic = None
    tp = os.path.join(ROOT, "profiles", "gemm_traffic.json")
    if os.path.exists(tp):
        traffic = json.load(open(tp)).get("bytes_per_launch")
    total_ms = sum(v["ms"] for v in ops_summary.values())
    breakdown = {k: {"launches": v["launches"], "ms_per_step": v["ms"] / a.steps,
                     "share": v["ms"] / total_ms if total_ms else None,
                     "tflops": (v["flops"] / (v["ms"] / 1000.0) / 1e12) if v["flops"] else None}
                 for k, v in sorted(ops_summary.items())}

    # ---------------- e2e: public host-buffer API, copies inside the timed region
    e2e, e2e_ok = None, None
    if not a.no_e2e:
        e2e, e2e_ok = run_e2e(a, tower, n_local, mb, pix_host, feats_all, local_out, dev, world, barrier,
                              max_over_ranks)
    # ---------------- config 2 latency: one 13-crop frame (tower + combine + projection)
    # one 13-crop frame's latency on the N GPUs of the run: at N = 1 the whole frame on this GPU; at N > 1 its
    # crops sharded over the ranks (ShardedFrame: ceil(13 / N) crops each, one NCCL all-gather of the features,
    # combine + projection on every rank), max over ranks; the sharded output is checked against one GPU's
    frame_ms = frame_ok = None
    if not a.no_frame:
        crops = torch.from_numpy(crop_pixels(13, cfg, seed=1, first=0)).to(torch.bfloat16).to(dev)
        sf = ShardedFrame(tower, 13, cfg.ntok, cfg.width, dev)
        for _ in range(3):
            sf(crops)
        torch.cuda.synchronize()
        barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        for _ in range(10):
            sf(crops)
        g1.record()
        torch.cuda.synchronize()
        frame_ms = max_over_ranks(g0.elapsed_time(g1) / 10)
        if world > 1:
            frame_ok = bool(torch.equal(sf(crops), tower.frame(crops)))
            frame_ok = max_over_ranks(0.0 if frame_ok else 1.0) == 0.0

    tap = txt = fin = None
    if world == 1 and not a.no_tapnext:
        tap = tapnext_frame_ms(dev)
        txt = text_ms(dev)
        fin = frame_input_ms(dev)

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        v, cores = cpu_oracle_rate(W, cfg, 4, 5)
        cpu = {"value": v, "unit": UNIT, "cores": cores, "kind": "port",
               "sample": "4 crops per run (27 blocks + post-LN, fp32 torch CPU oracle = port of md2fast.FastMD2._vision), median of 5 runs after 1 warm-up"}

    if rank == 0:
        fl = cfg.flops_per_crop()
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": ms / a.steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded U[-1,1] pixels, N(0,0.02) weights; no checkpoints offline)",
            "config": {"workload": f"config 4: {a.crops} crops (80 frames x 13) through the 27-block tower of config 1, "
                                   f"all-gathered [{a.crops},729,1152] bf16", "crops_per_step": a.crops,
                       "chunk_crops_per_rank": mb, "chunks_per_rank": n_local // mb,
                       "parallelism": f"dp{world} (crop sharding) + NCCL all-gather",
                       "l2": "inputs larger than L2 (pixels %.0f MB per step, activations GBs)" % (a.crops * 3 * 378 * 378 * 2 / 1e6)},
            "allgather_exposed_ms_per_step": ag_exposed,
            "ms_per_frame_13crop_throughput": 13 * 1000.0 / value,
            "ms_per_frame_13crop_latency": frame_ms,
            "frame_latency_mode": ("one GPU" if world == 1 else
                                   f"13 crops sharded over {world} GPUs ({-(-13 // world)} per rank), NCCL all-gather "
                                   "of the features, combine + projection on every rank; max over ranks"),
            "frame_sharded_matches_one_gpu": frame_ok,
            "tapnext_ms_per_frame": tap,
            "text_decoder": txt,
            "frame_input": fin,
            "tflops_whole_step": fl["total"] * a.crops * a.steps / (ms / 1000.0) / 1e12,
            "frac_of_peak_whole_step": fl["total"] * a.crops * a.steps / (ms / 1000.0) / 1e12 / (sustained * world),
            "roofline": {"kernel": "gemm_bf16_tc_pair_kernel (tcgen05 cta_group::2, all GEMM launches of the timed region)",
                         "bound": "tensor", "achieved": achieved, "peak": sustained, "unit": "TFLOP/s",
                         "frac": achieved / sustained, "traffic": traffic,
                         "traffic_source": "profiles/gemm_traffic.json: dram__bytes_read.sum + dram__bytes_write.sum per "
                                           "GEMM launch from an ncu capture of the 26-crop case, scaled to the bench's "
                                           "chunk by its rows (not measured in this run; writes still in L2 when a "
                                           "kernel ends are not counted)",
                         "peak_source": f"{src} bf16_tflops_sustained" + (" of measured" if src == "measured" else " of fallback"),
                         "launches": gemm_n, "avg_launch_ms": gemm_ms / max(gemm_n, 1)},
            "kernels": breakdown,
            "cpu_baseline": cpu,
            "e2e": e2e, "e2e_matches_device_path": e2e_ok,
            "gpu_launches": launches,
            "clocks": clocks,
            "device_status": status,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def text_ms(dev, reps=10):
    """The text decoder after the tower (24 layers, 2048 wide): image prefill of 730 tokens and the 32-token
    question, mean ms over `reps` (3 warm-ups).  Timing only, so the weights are drawn N(0, 0.02) (LayerNorm
    gamma 1, beta 0) directly on the device from a seeded generator instead of the host generator the parity
    tests use."""
    from strix_halo_maxx_b200.config import TEXT
    from strix_halo_maxx_b200.weights import text_weights_device
    from strix_halo_maxx_b200.text import TextDecoder
    W = text_weights_device(TEXT, dev, seed=0)
    g = torch.Generator(device=dev).manual_seed(1)
    emb = torch.randn(TEXT.prefix - 1, TEXT.dim, device=dev, generator=g)
    ids = torch.randint(1, TEXT.vocab, (TEXT.q_len,), device=dev, generator=g)

    def timed(dec):
        res = {}
        for name, fn in (("prefill_ms", lambda: dec.encode(emb, 0)), ("question_ms", lambda: dec.query(ids, TEXT.q_len - 1))):
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                fn()
            e1.record()
            torch.cuda.synchronize()
            res[name] = e0.elapsed_time(e1) / reps
        return res

    # bf16 linears (tlin_cls=HLin), then the W8A8 int8 ones (tlin_cls=HI8Lin, the reference's default)
    out = timed(TextDecoder(W, TEXT, device=dev))
    out["prefill_gemm_tflops"] = TEXT.flops(TEXT.prefix) / (out["prefill_ms"] / 1000) / 1e12
    i8 = timed(TextDecoder(W, TEXT, device=dev, int8=True))
    i8["prefill_gemm_tops"] = TEXT.flops(TEXT.prefix) / (i8["prefill_ms"] / 1000) / 1e12
    out["int8"] = i8
    del W
    return out


def frame_input_ms(dev, reps=20):
    """One 640 x 480 JPEG frame to the tower's 378 x 378 uint8 input: nvJPEG decode + the LANCZOS squash
    kernels on the device, next to Pillow's decode + resize on the host (the reference's FastMD2.set_image
    path, md2fast.py:223-228), mean ms over `reps`."""
    import io
    from PIL import Image
    from strix_halo_maxx_b200 import imgproc
    yy, xx = np.mgrid[0:480, 0:640].astype(np.float64)
    img = np.stack([np.sin(xx / 23.0) * np.cos(yy / 17.0), np.cos(xx / 31.0 + yy / 29.0), np.sin((xx + yy) / 41.0)], -1)
    buf = io.BytesIO()
    Image.fromarray((img * 100 + 128).clip(0, 255).astype(np.uint8)).save(buf, format="JPEG", quality=92)
    data = buf.getvalue()
    out = torch.empty(378, 378, 3, dtype=torch.uint8, device=dev)
    for _ in range(3):
        imgproc.load_frame(data, dev, out=out)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(reps):
        imgproc.load_frame(data, dev, out=out)
    torch.cuda.synchronize()
    gpu = (time.perf_counter() - t0) * 1000 / reps
    t0 = time.perf_counter()
    for _ in range(reps):
        Image.open(io.BytesIO(data)).convert("RGB").resize((378, 378), Image.Resampling.LANCZOS)
    host = (time.perf_counter() - t0) * 1000 / reps
    return {"gpu_ms": gpu, "pillow_host_ms": host, "jpeg": "640x480 q92", "timing": "host wall clock incl. launch"}


def tapnext_frame_ms(dev, n_frames=16):
    """Config 3 (the BASELINE simplification) and the full TAPNext++ step (blocks + tracking heads): 12 blocks,
    1280 tokens, the
    state carried over n_frames frames of one video; mean ms per frame (CUDA events, 4 warm-up frames, so
    that every CUDA graph the engines replay -- one per history-ring position -- is captured before the
    timed frames; a video's first frame always runs eagerly)."""
    from strix_halo_maxx_b200.config import TAPNEXT
    from strix_halo_maxx_b200.weights import tapnext_weights, tapnextpp_weights, tapnext_inputs, heads_weights
    from strix_halo_maxx_b200.tapnext import TapNextStep
    from strix_halo_maxx_b200.tapnextpp import TapNextPPStep
    frames, queries = tapnext_inputs(TAPNEXT, n_frames, seed=2)
    fr, qs = torch.from_numpy(frames).to(dev), torch.from_numpy(queries).to(dev)
    out = {}
    for name, cls, wfn in (("config3", TapNextStep, tapnext_weights), ("tapnextpp", TapNextPPStep, tapnextpp_weights)):
        if cls is TapNextPPStep:  # the reference's whole per-frame step: blocks + tracking heads (step8.py:316-325)
            eng = cls(wfn(TAPNEXT, seed=9), TAPNEXT, device=dev, heads=heads_weights(TAPNEXT, seed=21))
            run = eng.track
        else:
            eng = cls(wfn(TAPNEXT, seed=9), TAPNEXT, device=dev)
            run = eng.step
        for f in range(4):
            run(fr[f], qs[f])
        eng.reset()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for f in range(n_frames):
            run(fr[f], qs[f])
        e1.record()
        torch.cuda.synchronize()
        out[name] = e0.elapsed_time(e1) / n_frames
        del eng
    out["frames"] = n_frames
    return out


def main():
    a = parse()
    if a.tapnext_only:
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        print(json.dumps({"tapnext_ms_per_frame": tapnext_frame_ms(dev)}), flush=True)
        return
    if a.impl == "reference":
        run_reference(a)
    else:
        run_vt(a)


if __name__ == "__main__":
    main()
