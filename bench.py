#!/usr/bin/env python
"""Benchmark: map-frames/s of the scenemap objprob keyframe update.

Workload (per GPU): 64 independent box-room maps (config-0 generator, per-map seeds), 640x480
fp32 depth + uint16 labels, 8-24 detections per frame, 1152-d bf16 embeddings, 512x512 grid.
A step = one keyframe of every map (Mapper2D::keyframe + ObjectMap::update + addPoints).
The maps first run `--preroll` untimed frames (so the timed window sees a populated memory),
then W warm-up steps, then K timed steps.  Each step reads fresh frames (118 MB of new input
per step at 64 maps; the timed window reads K x that from HBM), so no L2 flush is inserted.

  python bench.py [--gpus N --steps K --warmup W] [--impl reference]

Multi-GPU (torchrun): every rank owns its own 64 maps (weak scaling, no collective on the
path); per-map ApStats are gathered to rank 0 with NCCL after the timed region.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "robot-agent_b200"))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

METRIC = "map-frames/s of scenemap objprob update"
D_EMB = 1152


def alg_bytes(work, D):
    """Algorithmic HBM bytes per step from the work counters: the per-unit terms of the path's
    byte count (depth fp32 + label u16 per scanned pixel, bf16 detection embeddings, memory
    vectors read by association, r_frag fp32 read + write and one fp16 view per update, 20-byte
    cloud points, int16 log-odds read + write per updated cell, 12-byte scan points, depth
    pixels read by makeScan).  Per kernel: the terms that kernel moves."""
    w = work
    per = {
        "k_obs": 6 * w["obs_px"],
        "k_assoc": 2 * D * (w["det"] + w["vec16"]),
        "k_update": 10 * D * w["upd"],
        "k_cloud_add": 20 * w["cloud_pts"],
        "k_grid": 4 * w["scan_px"] + 12 * w["scan_pts"] + 4 * w["cells"],
    }
    return per, float(sum(per.values()))


def ncu_traffic():
    """DRAM bytes per launch from the committed ncu summary (profiles/ncu_traffic.txt:
    '<kernel> <bytes per launch>' lines), or {} when absent."""
    out = {}
    pth = os.path.join(ROOT, "profiles", "ncu_traffic.txt")
    if os.path.exists(pth):
        for line in open(pth):
            f = line.split()
            if len(f) >= 2 and not line.startswith("#"):
                try:
                    out[f[0]] = float(f[1])
                except ValueError:
                    pass
    return out


def rooflines(kt, work, step_s, D):
    peaks_p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    peaks = json.load(open(peaks_p)) if os.path.exists(peaks_p) else {}
    hbm = peaks.get("hbm_gbs", 6650.0)
    src = "measured (MEASURED_PEAKS.json hbm_gbs)" if peaks else "fallback 6650 GB/s"
    per, tot = alg_bytes(work, D)
    traffic = ncu_traffic()
    allk = {}
    for k, b in per.items():
        if k not in kt or kt[k][1] == 0:
            continue
        avg_s = kt[k][0] / kt[k][1] / 1e3
        allk[k] = {"alg_bytes_per_launch": b, "avg_launch_ms": avg_s * 1e3, "achieved_gbs": b / avg_s / 1e9,
                   "frac": b / avg_s / 1e9 / hbm}
    dom = max(allk, key=lambda k: allk[k]["avg_launch_ms"])
    d = allk[dom]
    roof = {"kernel": dom, "bound": "hbm", "achieved": d["achieved_gbs"], "peak": hbm, "unit": "GB/s",
            "frac": d["frac"], "traffic": traffic.get(dom), "alg_bytes_per_launch": d["alg_bytes_per_launch"],
            "avg_launch_ms": d["avg_launch_ms"], "peak_source": src}
    step = {"kernel": "whole keyframe chain (all kernels of a step)", "bound": "hbm", "achieved": tot / step_s / 1e9,
            "peak": hbm, "unit": "GB/s", "frac": tot / step_s / 1e9 / hbm, "alg_bytes_per_step": tot}
    return roof, step, allk
UNIT = "map-frames/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--preroll", type=int, default=100)
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--kt-steps", type=int, default=10, help="steps of the separate per-kernel timing pass")
    ap.add_argument("--maps", type=int, default=None, help="maps per GPU (default 64 for objprob, 1 for occ)")
    ap.add_argument("--max-objects", type=int, default=1024)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--cpu-timed", type=int, default=10,
                    help="CPU baseline: timed keyframes per map (the first of the device arm's timed frames)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="objprob: skip the short config-2 / config-3 runs recorded under extra_workloads")
    ap.add_argument("--assoc-frames", type=int, default=32,
                    help="config 2: frames per association call (their detections as one row block against the bank)")
    ap.add_argument("--workload", default="objprob", choices=["objprob", "occ", "assoc", "walls"],
                    help="objprob = config 1 (headline); occ = config 3 (grid insert + correlative scan matching); "
                         "assoc = config 2 (association GEMM); walls = wall extraction from the config-1 grids")
    ap.add_argument("--scans", type=int, default=5000, help="config 3: scans per map")
    ap.add_argument("--mask-grid", type=int, default=0, metavar="S",
                    help="detections as the detector's bit masks on an S-pixel grid (sm_detections form) instead of "
                         "the label image; both arms read the same masks")
    ap.add_argument("--no-reencode-pass", action="store_true",
                    help="skip the extra timed pass (and CPU baseline) without the re-encode stage")
    ap.add_argument("--max-clouds", type=int, default=None,
                    help="cloud slots per map (smg_create_pooled; default = --max-objects)")
    ap.add_argument("--width", type=int, default=640, help="depth image width (config 4: 848)")
    ap.add_argument("--dets", type=int, default=24, help="detections per frame at most (config 4: 32)")
    ap.add_argument("--boxes", type=int, default=20, help="boxes per room")
    ap.add_argument("--check-run", type=int, default=0, metavar="FRAMES",
                    help="checked run instead of the benchmark: push --maps maps (device-resident config-1 frames, "
                         "--max-objects slots) for FRAMES keyframes; after every 16 frames print the device error word "
                         "and the first failed bounds check (nonzero only in a -DSMG_CHECKS library, chosen with the "
                         "SMG_LIB environment variable) and stop at the first nonzero one.  Also the small case that "
                         "ncu captures are taken on")
    return ap.parse_args()


# ------------------------------------------------------------------ clocks
class Clocks:
    """SM clock and clock-event (throttle) reasons sampled while the timed region runs: NVML
    every 2 ms in a thread (a short timed region still gets samples), else `nvidia-smi -lms 200`
    into a temporary CSV.  Reading only; nothing is set."""
    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap"}

    def __init__(self, gpu_index: int, path: str, torch_dev=None):
        self.path, self.proc, self.thread = path, None, None
        self.sm, self.mx, self.bits = [], None, 0
        self.stop_ev = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            h = None
            try:   # the GPU torch runs on, by PCI address (indices differ under CUDA_VISIBLE_DEVICES)
                import torch
                pr = torch.cuda.get_device_properties(torch_dev if torch_dev is not None else gpu_index)
                h = pynvml.nvmlDeviceGetHandleByPciBusId(f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0")
            except Exception:
                h = pynvml.nvmlDeviceGetHandleByIndex(gpu_index)
            self.mx = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            reasons_fn = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons

            def run():
                while not self.stop_ev.is_set():
                    try:
                        self.sm.append(float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)))
                        self.bits |= int(reasons_fn(h))
                    except Exception:
                        pass
                    self.stop_ev.wait(0.002)
            self.thread = threading.Thread(target=run, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.thread = None
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={gpu_index}", f"--query-gpu={q}", "--format=csv,noheader",
                                          "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.thread is not None:
            self.stop_ev.set()
            self.thread.join(timeout=5)
            reasons = sorted(name for bit, name in self.REASONS.items() if self.bits & bit)
            return {"sm_mhz": statistics.median(self.sm) if self.sm else None, "sm_max_mhz": self.mx, "reasons": reasons,
                    "samples": len(self.sm), "source": "nvml, 2 ms"}
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], None, set()
        for line in open(self.path):
            p = [x.strip() for x in line.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1].split()[0]))
                mx = float(p[2].split()[0])
            except ValueError:
                continue
            for name, v in zip(["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"], p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        try:
            os.unlink(self.path)
        except OSError:
            pass
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvidia-smi, 200 ms"}


# ------------------------------------------------------------------ CPU baseline (reference scenemap code)
def cpu_reference(M_sample: int, lead: int, timed: int, threads: int, base_seed: int = 1000, obj_kv: str = "",
                  mask_grid: int = 0, reencode: bool = True):
    """The reference scenemap (oracle/_ref, compiled from the reference sources) on the host cores:
    one map per thread.  Every map runs `lead` untimed keyframes, then `timed` timed ones: the
    same frames (same seeds, same frame indices) the device arm pre-rolls and times.  Inputs come
    from the same generator (the device renderer when a GPU is present, else the host one, which
    renders the same bytes) in chunks of 10 frames; the threads meet at every chunk, and the
    timed span is the sum over chunks of the slowest thread's timed work in that chunk."""
    from oracle import ref
    from scenemap_b200 import synth
    if not ref.available():
        return None
    M_sample = min(M_sample, threads)
    frames = lead + timed
    gen_dev = False
    try:
        import torch
        gen_dev = torch.cuda.is_available()
    except Exception:
        pass
    if gen_dev:
        from scenemap_b200.workload import RoomBatch
        wl = RoomBatch(M_sample, base_seed, frames, D=D_EMB, bf16=True, max_det=24, mask_grid=mask_grid)
    else:
        gens = [synth.BoxRoom(seed=synth.map_seed(base_seed, m), n_frames=frames, bf16=True, max_det=24, mask_grid=mask_grid)
                for m in range(M_sample)]
    maps = [ref.RefMap(obj_kv) for _ in range(M_sample)]
    for R in maps:
        R.set_reencode(reencode)
    span = 0.0
    for f0 in range(0, frames, 10):
        nf = min(10, frames - f0)
        if gen_dev:
            R = wl.render(f0, nf)
            chunk = [wl.host_frames(R, fi) for fi in range(nf)]
        else:
            chunk = [[g.frame(f0 + fi) for g in gens] for fi in range(nf)]
        t_m = [0.0] * M_sample

        def work(m):
            for fi in range(nf):
                t0 = time.perf_counter()
                maps[m].frame(chunk[fi][m])
                if f0 + fi >= lead:
                    t_m[m] += time.perf_counter() - t0

        ths = [threading.Thread(target=work, args=(m,)) for m in range(M_sample)]
        for t in ths:
            t.start()
        for t in ths:
            t.join()
        span += max(t_m)
    value = M_sample * timed / span
    return dict(value=value, unit=UNIT, cores=M_sample, kind="reference", frames_timed=f"{lead}..{frames - 1}",
                sample=f"{M_sample} maps, keyframes {lead}..{frames - 1} timed after {lead} untimed, one map per host "
                       f"thread, reference scenemap C++ (-O2) from oracle/_ref"
                       + ("" if reencode else ", buildReencode not run"))


# ------------------------------------------------------------------ B200 arm
def run_b200(args, rank, world, local_rank):
    import torch
    from scenemap_b200 import smg
    from scenemap_b200.workload import RoomBatch
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    M = args.maps
    n_total = args.preroll + args.warmup + args.steps + args.kt_steps + args.e2e_steps
    from scenemap_b200 import dist
    n_total += 0 if args.no_reencode_pass else args.steps
    W, H = args.width, 480
    wl = RoomBatch(M, 1000, n_total, D=1152, bf16=True, w=W, h=H, max_det=args.dets,
                   map_offset=dist.rank_maps(rank, world, M)[0], device=str(dev), mask_grid=args.mask_grid,
                   n_boxes=args.boxes)
    B = smg.Batch(M, max_objects=args.max_objects, emb_dim=1152, max_w=W, max_h=H, max_det=args.dets,
                  grid=(512, 512, -256 + 60, -256 + 50), dev=local_rank, **pool_kw(args))
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    f = 0
    # untimed pre-roll + warm-up
    chunk = max(1, min(16, int(4e9 // (M * W * H * 6))))   # rendered frames held at once: <= ~4 GB
    while f < args.preroll + args.warmup:
        nf = min(chunk, args.preroll + args.warmup - f)
        R = wl.render(f, nf, sp)
        for fi in range(nf):
            keep = []
            B.push(None, smg.SMG_MEM_DEVICE, structs=wl.structs(R, fi, keep), stream=sp)
        f += nf
    torch.cuda.synchronize()
    assert B.error_word() == 0, "device error word set during warm-up"
    # timed window: inputs resident in HBM before the clock starts
    R = wl.render(f, args.steps, sp)
    keep = []
    structs = [wl.structs(R, fi, keep) for fi in range(args.steps)]
    work0 = B.work()
    launches0 = B.launches()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clk = Clocks(local_rank, os.path.join(tempfile.gettempdir(), f"smg_bench_clocks_{os.getpid()}_r{rank}.csv"))
    if clk.thread is None:
        time.sleep(0.3)   # nvidia-smi's first sample
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for fi in range(args.steps):
        B.push(None, smg.SMG_MEM_DEVICE, structs=structs[fi], stream=sp)
    e1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    clocks = clk.stop()
    t = e0.elapsed_time(e1) / 1e3
    launches = B.launches() - launches0
    work1 = B.work()
    work = {k: (work1[k] - work0[k]) / args.steps for k in work0}   # per step (all maps of this GPU)
    err = B.error_word()
    f += args.steps
    del R, structs
    # the same chain without the re-encode stage, on the next K keyframes (its CPU baseline times
    # the same keyframes): the reference's stage fills a whole mask grid per candidate object
    t_nr, f_nr = None, f
    if not args.no_reencode_pass:
        R = wl.render(f, args.steps, sp)
        keep = []
        structs = [wl.structs(R, fi, keep) for fi in range(args.steps)]
        B.set_reencode(False)
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for fi in range(args.steps):
            B.push(None, smg.SMG_MEM_DEVICE, structs=structs[fi], stream=sp)
        e1.record(stream)
        torch.cuda.synchronize()
        t_nr = e0.elapsed_time(e1) / 1e3
        B.set_reencode(True)
        f += args.steps
        del R, structs
    # per-kernel breakdown: a separate pass with event timing around every launch (the chain
    # then runs as one stream group, so each kernel's time is its own)
    R = wl.render(f, args.kt_steps, sp)
    keep = []
    structs = [wl.structs(R, fi, keep) for fi in range(args.kt_steps)]
    torch.cuda.synchronize()
    B.timing_read()
    B.timing(True)
    for fi in range(args.kt_steps):
        B.push(None, smg.SMG_MEM_DEVICE, structs=structs[fi], stream=sp)
    torch.cuda.synchronize()
    kt = B.timing_read()
    B.timing(False)
    f += args.kt_steps
    del R, structs
    # e2e: host (pinned) inputs through the C ABI, association read back every step
    # (pinned host frames of at most ~8 GB: fewer e2e steps for very large batches)
    E = max(2, min(args.e2e_steps, int(8e9 // (M * W * H * 6))))
    R = wl.render(f, E, sp)
    depth_h = torch.empty((E, M, H, W), dtype=torch.float32, pin_memory=True)
    label_h = torch.empty((E, M, H, W), dtype=torch.int16, pin_memory=True)
    emb_h = torch.empty(R["emb"].shape, dtype=torch.int16, pin_memory=True)
    depth_h.copy_(R["depth"])
    label_h.copy_(R["label"].view(torch.int16))
    emb_h.copy_(R["emb"].view(torch.int16))
    masks_h = None
    if R["masks"] is not None:
        masks_h = torch.empty(R["masks"].shape, dtype=torch.int32, pin_memory=True)
        masks_h.copy_(R["masks"])
    torch.cuda.synchronize()
    e_structs, keep2 = [], []
    h2d = 0
    for fi in range(E):
        arr = (smg.SmgFrame * M)()
        for m in range(M):
            fd = wl.frame_dict(R, fi, m)
            d = R["dets"][fi * M + m]
            ptrs = dict(depth=depth_h[fi, m].data_ptr(), label=label_h[fi, m].data_ptr(),
                        emb=emb_h.data_ptr() + d["emb_off"] * 1152 * 2 if d["n"] else None)
            if masks_h is not None:
                ptrs["mask_bits"] = masks_h[fi * M + m].data_ptr()
            arr[m] = smg.Batch.frame_struct(fd, keep2, smg.SMG_EMB_BF16, ptrs=ptrs)
            h2d += W * H * 6 + d["n"] * 1152 * 2
        e_structs.append(arr)
    h2d //= E
    d2h = M * args.dets * 4   # uint32 object id per detection slot
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    h2d_0 = B.work()["h2d"]
    # pipelined like a streaming caller: push keyframe k + 1 (its host copies overlap keyframe
    # k's chain) before waiting for keyframe k's association, which every step reads back
    outs = [torch.empty((M, args.dets), dtype=torch.int32, pin_memory=True) for _ in range(2)]
    t0 = time.perf_counter()
    prev = None
    for fi in range(E):
        B.push(None, smg.SMG_MEM_HOST, structs=e_structs[fi], stream=sp)
        tk = B.assoc_all_async(outs[fi % 2].data_ptr())
        if prev is not None:
            B.wait_read(prev)
        prev = tk
    B.wait_read(prev)
    torch.cuda.synchronize()
    t_e2e = time.perf_counter() - t0
    # bytes that crossed to the device: the library counts its copies and the pixels it read in
    # place from the pinned frames (the input frames themselves are h2d_input per step)
    h2d_input = h2d
    h2d = (B.work()["h2d"] - h2d_0) // E
    if world > 1:
        torch.distributed.barrier()
    err |= B.error_word()
    # per-map statistics gathered to rank 0 (NCCL over NVLink when world > 1)
    stats = np.zeros((M, 16), np.int64)
    for m in range(M):
        s = B.stats(m)
        stats[m] = list(s.values())
    from scenemap_b200 import dist
    all_stats = dist.gather_stats(stats, world, dev)          # NCCL all_gather when world > 1
    if t_nr is not None:
        t, t_e2e, t_nr = dist.max_over_ranks([t, t_e2e, t_nr], world, dev)   # device times: max over ranks
    else:
        t, t_e2e = dist.max_over_ranks([t, t_e2e], world, dev)
    n_obj = [len(B.objects(m)) for m in range(min(M, 4))]
    B.close()
    return dict(t=t, t_e2e=t_e2e, E=E, t_nr=t_nr, f_nr=f_nr, kt=kt, launches=launches, err=err, clocks=clocks, work=work,
                stats=all_stats, h2d=h2d, h2d_input=h2d_input, d2h=d2h, n_obj=n_obj)


def pool_kw(args) -> dict:
    """smg_create_pooled's cloud pool size when --max-clouds is given."""
    return {"max_clouds": args.max_clouds} if args.max_clouds else {}


def check_run(args, local_rank):
    """Checked run of the config-1 workload (see --check-run)."""
    import torch
    from scenemap_b200 import smg
    from scenemap_b200.workload import RoomBatch
    torch.cuda.set_device(local_rank)
    M, NF = args.maps, args.check_run
    wl = RoomBatch(M, 1000, NF, D=D_EMB, bf16=True, max_det=24, device=f"cuda:{local_rank}")
    B = smg.Batch(M, max_objects=args.max_objects, emb_dim=D_EMB, max_w=640, max_h=480, max_det=24,
                  grid=(512, 512, -256 + 60, -256 + 50), dev=local_rank)
    for f0 in range(0, NF, 16):
        nf = min(16, NF - f0)
        R = wl.render(f0, nf, 0)
        for fi in range(nf):
            keep = []
            B.push(None, smg.SMG_MEM_DEVICE, structs=wl.structs(R, fi, keep), stream=0)
        torch.cuda.synchronize()
        err, chk = B.error_word(), B.debug_check()
        print("frames", f0, f0 + nf, "err", err, "chk", chk, flush=True)
        if err or any(chk):
            B.close()
            sys.exit(1)
    print("work", B.work())
    B.close()


def run_occ(args, rank, world, local_rank):
    """Config 3: every step is one scan per map: correlative scan match around the initial pose,
    then the insert at the matched pose (smg_occ_track).  `value` = scans/s with the scans'
    host-to-device staging inside the step and no per-step readback; `e2e` = the same with the
    matched pose, index, score and changed count read back after every step."""
    import torch
    from scenemap_b200.floorplan import FloorPlan
    from scenemap_b200.occ import OccBatch, config3_csm
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    M = args.maps
    N = args.scans
    plans = [FloorPlan(seed=7000 + rank * M + m, n_scans=N) for m in range(M)]
    scans = [[p.scan(k) for p in plans] for k in range(N)]
    G = OccBatch(M, (1024, 1024, -100, -100), max_points=1024, dev=local_rank)
    csm = config3_csm()
    st = torch.cuda.current_stream(dev)
    W = args.warmup
    n_hits = float(np.mean([len(s["hits"]) for row in scans for s in row]))
    n_cand = 41 * 13 * 13
    for k in range(W):
        G.track(scans[k], [s["pose0"] for s in scans[k]], csm, stream=st.cuda_stream)
    torch.cuda.synchronize()
    K = min(args.steps if args.steps != 100 else N - W, N - W)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0.record(st)
    from scenemap_b200 import occ as occ_mod
    L = occ_mod._lib()
    import ctypes as C
    for k in range(W, W + K):   # asynchronous steps (outputs stay on the device)
        arr, keep = G._scans(scans[k])
        P0 = np.ascontiguousarray([s["pose0"] for s in scans[k]], np.float64)
        rc = L.smg_occ_track(G.h, arr, P0.ctypes.data_as(C.POINTER(C.c_double)), C.byref(csm), M, None, None, None, None,
                             C.c_void_p(st.cuda_stream))
        assert rc == 0
    e1.record(st)
    torch.cuda.synchronize()
    t = e0.elapsed_time(e1) / 1e3
    # end to end: results read back every step (what a scan-matching front end waits for)
    G2 = OccBatch(M, (1024, 1024, -100, -100), max_points=1024, dev=local_rank)
    KE = min(K, 1000)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for k in range(KE):
        G2.track(scans[k], [s["pose0"] for s in scans[k]], csm, stream=st.cuda_stream)
    t_e2e = time.perf_counter() - t0
    if world > 1:
        tt = torch.tensor([t, t_e2e], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
        t, t_e2e = float(tt[0]), float(tt[1])
    G.close(); G2.close()
    cb = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import ref
        if ref.available() and ref.port_available():
            R = ref.RefOcc()
            ns = min(200, N)
            t0 = time.perf_counter()
            for k in range(ns):
                s = scans[k][0]
                bi, bs, bp = ref.csm(R.cells(), s["hits"], s["pose0"])
                R.insert(s["hits"], s["free"], bp)
            tc = time.perf_counter() - t0
            cb = {"value": ns / tc, "unit": "scans/s", "cores": 1, "kind": "port",
                  "sample": f"{ns} scans of map 0: restated matcher (oracle/port) + reference OccGrid::insert (oracle/_ref)"}
    return dict(t=t, K=K, t_e2e=t_e2e, KE=KE, n_hits=n_hits, n_cand=n_cand, cb=cb)


def run_assoc(args, rank, world, local_rank):
    """Config 2: each step associates F frames of 256 detections with the 16384-vector bank in
    one call (the frames' detections as consecutive rows; tcgen05 GEMM + fused gate/top-1 +
    certification).  Frames are pre-generated and resident; the bank (37.7 MB) stays resident
    across steps.  Per-kernel CUDA-event times give the GEMM's TFLOP/s."""
    import torch
    from scenemap_b200.assoc import AssocGPU, AssocWorkload
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    W = AssocWorkload(seed=100 + rank)
    F = max(1, args.assoc_frames)
    n_batches = 8
    frames = [W.frame(k) for k in range(F * n_batches)]
    to_d = lambda a, dt=None: (torch.from_numpy(np.ascontiguousarray(a)).view(dt) if dt is not None
                               else torch.from_numpy(np.ascontiguousarray(a))).to(dev)
    zb = [np.concatenate([frames[i * F + j][0] for j in range(F)]) for i in range(n_batches)]
    bb = [np.concatenate([frames[i * F + j][1] for j in range(F)]) for i in range(n_batches)]
    Z = [to_d(z, torch.int16) for z in zb]
    Bx = [to_d(b) for b in bb]
    mem, mbox = to_d(W.mem, torch.int16), to_d(W.mem_box)
    A = AssocGPU(W.n_det * F, W.n_mem, W.dim, dev=local_rank)
    st = torch.cuda.current_stream(dev)
    for k in range(args.warmup):
        A.match(Z[k % n_batches], Bx[k % n_batches], mem, mbox, stream=st.cuda_stream)
    torch.cuda.synchronize()
    K = args.steps
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    outs = []
    for k in range(K):
        outs.append(A.match(Z[k % n_batches], Bx[k % n_batches], mem, mbox, stream=st.cuda_stream))
    e1.record(st)
    torch.cuda.synchronize()
    t = e0.elapsed_time(e1) / 1e3
    cert = float(np.mean([o[2].float().mean().item() for o in outs[:16]]))
    matched = float(np.mean([(o[0] >= 0).float().mean().item() for o in outs[:16]]))
    # end to end: host batches (pinned) in, decisions out, every step
    hz = [torch.from_numpy(z.view(np.int16)).pin_memory() for z in zb]
    hb = [torch.from_numpy(b).pin_memory() for b in bb]
    zd, bd = torch.empty_like(Z[0]), torch.empty_like(Bx[0])
    KE = min(K, 200)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for k in range(KE):
        zd.copy_(hz[k % n_batches], non_blocking=True)
        bd.copy_(hb[k % n_batches], non_blocking=True)
        m, s, c = A.match(zd, bd, mem, mbox, stream=st.cuda_stream)
        m.cpu()
    t_e2e = time.perf_counter() - t0
    if world > 1:
        tt = torch.tensor([t, t_e2e], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
        t, t_e2e = float(tt[0]), float(tt[1])
    err = A.error()
    A.close()
    cb = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import assoc_oracle as ao
        ns = 8
        t0 = time.perf_counter()
        for k in range(ns):
            ao.decide(frames[k][0], frames[k][1], W.mem, W.mem_box)
        cb = {"value": ns / (time.perf_counter() - t0), "unit": "frames/s", "cores": 1, "kind": "port",
              "sample": f"{ns} frames: numpy restatement (float32 gate over all pairs, fp64 index-order dots of gated pairs)"}
    return dict(t=t, K=K, t_e2e=t_e2e, KE=KE, cert=cert, matched=matched, err=err, cb=cb, F=F,
                flops=2.0 * W.n_det * W.n_mem * W.dim, bytes=2.0 * W.dim * (W.n_mem + W.n_det), n_det=W.n_det)


def assoc_line(r: dict, args, world: int) -> dict:
    """The config-2 JSON line of a run_assoc result."""
    F = r["F"]
    v = world * r["K"] * F / r["t"]
    peaks_p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    peaks = json.load(open(peaks_p)) if os.path.exists(peaks_p) else {}
    tf = r["flops"] * r["K"] * F / r["t"] / 1e12
    pk = peaks.get("bf16_tflops", 1590.0)
    out = {"metric": "frames/s of association stress (config 2)", "value": v, "unit": "frames/s", "n_gpus": world,
           "steps": r["K"], "warmup": args.warmup, "ms_per_step": 1e3 * r["t"] / r["K"], "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (fp32 accumulate)", "data": "synthetic",
           "config": {"workload": "config 2: 256 detections x 16384 memories x 1152, IoU gate 0.1, cos 0.8, top-1",
                      "frames_per_step": F,
                      "l2": "bank (37.7 MB) resident in L2 across steps"},
           "roofline": {"kernel": "k_assoc_gemm + k_assoc_decide", "bound": "tensor", "achieved": tf, "peak": pk,
                        "unit": "TFLOP/s", "frac": tf / pk, "traffic": None,
                        "peak_source": "measured (MEASURED_PEAKS.json bf16_tflops)" if peaks else "fallback"},
           "certified_fraction": r["cert"], "matched_fraction": r["matched"], "device_error_word": r["err"],
           "e2e": {"value": world * r["KE"] * F / r["t_e2e"], "unit": "frames/s",
                   "h2d_bytes_per_step": int(F * r["n_det"] * (1152 * 2 + 24)),
                   "d2h_bytes_per_step": int(F * r["n_det"] * 4)}}
    return out


def occ_line(r: dict, args, world: int) -> dict:
    """The config-3 JSON line of a run_occ result."""
    M = args.maps
    v = M * world * r["K"] / r["t"]
    out = {"metric": "scans/s of occupancy insert + correlative scan match (config 3)", "value": v, "unit": "scans/s",
           "n_gpus": world, "steps": r["K"], "warmup": args.warmup, "ms_per_step": 1e3 * r["t"] / r["K"],
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "i32 scores / f64 poses",
           "data": "synthetic", "config": {"workload": f"config 3: {M} map(s) per GPU, 12-room floor plan, 720 beams, "
                                                       "8 m, 1024^2 grid at 0.05 m, 13x13x41 search",
                                           "maps_per_gpu": M},
           "csm_lookups_per_s": v * r["n_hits"] * r["n_cand"],
           "e2e": {"value": M * world * r["KE"] / r["t_e2e"], "unit": "scans/s",
                   "h2d_bytes_per_step": int(M * (8 * 720 + 64)), "d2h_bytes_per_step": int(M * 56)}}
    return out


def main():
    args = parse()
    if args.maps is None:
        args.maps = 64 if args.workload in ("objprob", "walls") else 1
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.check_run:
        check_run(args, local_rank)
        return
    if args.workload == "walls":   # the wall-extraction line alone (one GPU)
        if rank == 0:
            print(json.dumps(run_walls(args, local_rank)))
        return
    masks = ("u16 label image (mask grid = image grid)" if args.mask_grid <= 0 else
             f"detector bit masks on a {args.mask_grid}-pixel grid (sm_detections form)")
    big = args.maps > 64 or args.width != 640
    cfg = {"workload": f"config {4 if big else 1}: {args.maps} box-room maps per GPU ({args.boxes} boxes), {args.width}x480 fp32 "
                       f"depth + {masks}, <= {args.dets} dets, 1152-d bf16 embeddings, <={args.max_objects} object slots"
                       + (f" ({args.max_clouds} cloud slots)" if args.max_clouds else "") + ", 512x512 grid",
           "detections": masks,
           "keyframe": "Mapper2D::keyframe + ObjectMap::update + addPoints + buildReencode (capi.cpp:811-1010)",
           "maps_per_gpu": args.maps, "frames_timed": f"{args.preroll + args.warmup}..{args.preroll + args.warmup + args.steps - 1}",
           "l2": f"fresh frames every step ({args.maps * args.width * 480 * 6 / 1e6:.0f} MB/step of depth + labels), no flush",
           "parallelism": f"dp{world} (maps)"}
    if args.impl == "reference":
        if rank != 0:
            return
        cores = os.cpu_count() or 1
        # the same keyframes the device arm times: frames preroll+W .. preroll+W+K-1 of the same
        # maps, after the same untimed pre-roll and warm-up frames
        lead = args.preroll + args.warmup
        cb = cpu_reference(min(cores, 64), lead, args.steps, min(cores, 64), mask_grid=args.mask_grid)
        if cb is None:
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libscenemap_ref.so not built"}))
            return
        extra = {}
        if not args.no_reencode_pass:   # the keyframes the device arm times without the stage
            cb_nr = cpu_reference(min(cores, 64), lead + args.steps, args.steps, min(cores, 64), mask_grid=args.mask_grid,
                                  reencode=False)
            extra = {"value_without_reencode": cb_nr["value"], "frames_timed_without_reencode": cb_nr["frames_timed"]}
        print(json.dumps({"metric": METRIC, "value": cb["value"], "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
                          "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
                          "vs_baseline": None, "dtype": "f64/f32", "data": "synthetic", "config": cfg, "impl": "reference",
                          "frames_timed": cb["frames_timed"], **extra,
                          "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
                          "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return
    if world > 1:
        import datetime
        import torch
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    if args.workload == "assoc":
        r = run_assoc(args, rank, world, local_rank)
        if world > 1:
            import torch
            torch.distributed.destroy_process_group()
        if rank == 0:
            out = assoc_line(r, args, world)
            if r["cb"]:
                out["cpu_baseline"] = r["cb"]
            print(json.dumps(out))
        return
    if args.workload == "occ":
        r = run_occ(args, rank, world, local_rank)
        if world > 1:
            import torch
            torch.distributed.destroy_process_group()
        if rank == 0:
            out = occ_line(r, args, world)
            if r["cb"]:
                out["cpu_baseline"] = r["cb"]
            print(json.dumps(out))
        return
    r = run_b200(args, rank, world, local_rank)
    if world > 1:
        import torch
        torch.distributed.destroy_process_group()
    if rank != 0:
        return
    K, M = args.steps, args.maps
    value = M * world * K / r["t"]
    e2e = M * world * r["E"] / r["t_e2e"]
    # roofline: algorithmic bytes from the device work counters (one launch per kernel per step)
    roof, roof_step, roof_all = rooflines(r["kt"], r["work"], r["t"] / K, D_EMB)
    cb = cb_nr = None
    if not args.no_cpu_baseline and world == 1:
        cores = os.cpu_count() or 1
        cb = cpu_reference(min(cores, 64), args.preroll + args.warmup, args.cpu_timed, min(cores, 64), mask_grid=args.mask_grid)
        if r["t_nr"] is not None:
            cb_nr = cpu_reference(min(cores, 64), r["f_nr"], args.cpu_timed, min(cores, 64), mask_grid=args.mask_grid,
                                  reencode=False)
    out = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K, "warmup": args.warmup,
           "ms_per_step": 1e3 * r["t"] / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": "f64/f32 (bf16 embeddings)", "data": "synthetic", "config": cfg,
           "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": r["d2h"],
                   "host_input_bytes_per_step": r["h2d_input"]},
           "gpu_launches": r["launches"], "roofline": roof, "roofline_step": roof_step,
           "roofline_kernels": roof_all, "work_per_step": r["work"], "clocks": r["clocks"],
           "kernel_ms_per_step": {k: v[0] / max(v[1], 1) for k, v in r["kt"].items()},
           "device_error_word": r["err"], "objects_first_maps": r["n_obj"],
           "stats_sum": {k: int(v) for k, v in zip(["n_through", "n_obs", "n_wall", "n_wall_name", "n_ceil", "n_floor",
                                                     "n_assoc", "n_new", "n_merge", "n_obj_struct", "n_reenc_req",
                                                     "n_reenc_done", "n_blocked", "n_wall_tall", "n_so_big", "n_bridge"],
                                                    r["stats"].sum(0))}}
    if r["t_nr"] is not None:
        out["value_without_reencode"] = M * world * K / r["t_nr"]
        out["frames_timed_without_reencode"] = f"{r['f_nr']}..{r['f_nr'] + K - 1}"
    if cb is not None:
        out["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
        ratios = {"with_reencode": value / cb["value"]}
        if cb_nr is not None:
            out["cpu_baseline_without_reencode"] = {k: cb_nr[k] for k in ("value", "unit", "cores", "kind", "sample")}
            ratios["without_reencode"] = out["value_without_reencode"] / cb_nr["value"]
        out["vs_cpu_baseline"] = ratios
    if world == 1 and not args.no_extra:
        out["extra_workloads"] = extra_workloads(args, local_rank)
    print(json.dumps(out))


def run_walls(args, local_rank: int, n_frames: int = 40) -> dict:
    """Wall extraction (smg_set_walls) on the config-1 maps: every keyframe's grid insert changes
    visible cells, so k_walls re-extracts all 64 maps each keyframe (the direction every 2 s of
    stamps).  Device time of k_walls per launch by CUDA events (timing mode), and the reference's
    walls.cpp (wallAngle + wallSegments) on the same final grids on one host core."""
    import torch
    from scenemap_b200 import smg
    from scenemap_b200.workload import RoomBatch
    torch.cuda.set_device(local_rank)
    M = args.maps
    grid = (512, 512, -256 + 60, -256 + 50)
    wl = RoomBatch(M, 1000, n_frames, D=1152, bf16=True, max_det=24, device=f"cuda:{local_rank}")
    B = smg.Batch(M, max_objects=args.max_objects, emb_dim=1152, max_w=640, max_h=480, max_det=24, grid=grid, dev=local_rank,
                  **pool_kw(args))
    B.set_walls(True)
    B.timing(True)
    for f0 in range(0, n_frames, 8):
        nf = min(8, n_frames - f0)
        R = wl.render(f0, nf, 0)
        for fi in range(nf):
            keep = []
            if f0 + fi == n_frames // 2:
                B.timing_read()   # the first half fills the grids
            B.push(None, smg.SMG_MEM_DEVICE, structs=wl.structs(R, fi, keep), stream=0)
        torch.cuda.synchronize()
    kt = B.timing_read()
    ms, n = kt.get("k_walls", (0.0, 0))
    per = ms / max(1, n // 2)   # k_wall_rects + k_walls: two launches per keyframe
    nseg = []
    for m in range(M):
        w = B.wall_segments(m)
        nseg.append(0 if w is None else len(w))
    err = B.error_word()
    cells = [B.grid_cells(m)["c8"] for m in range(M)]
    B.close()
    res = 0.05
    ox, oy = grid[2] * float(np.float32(res)), grid[3] * float(np.float32(res))
    line = {"metric": "wall extractions/s (every map's grid, one launch)", "value": M / (per * 1e-3) if per > 0 else None,
            "unit": "map-extractions/s", "ms_per_launch": per, "maps": M, "segments_per_map": float(np.mean(nseg)),
            "error_word": err,
            "roofline": {"bound": "latency (one CTA per map; the chaining warp walks every row and column)",
                         "alg_bytes_per_map": 512 * 512, "achieved_gbs": M * 512 * 512 / (per * 1e-3) / 1e9 if per > 0 else None}}
    try:
        import time
        from oracle import ref
        if ref.available():
            # the same mix as the device run: an extraction every keyframe, the direction every
            # 2 s of stamps (every 20th keyframe at 10 Hz)
            t0 = time.perf_counter()
            for c in cells:
                ref.wall_segments_grid(c, float(np.float32(res)), ox, oy, mode=0)
            t_seg = time.perf_counter() - t0
            t0 = time.perf_counter()
            for c in cells:
                ref.wall_segments_grid(c, float(np.float32(res)), ox, oy, mode=1)
            t_ang = time.perf_counter() - t0
            line["cpu_baseline"] = {"value": M / (t_seg + t_ang / 20), "unit": "map-extractions/s", "cores": 1, "kind": "reference",
                                    "sample": f"walls.cpp wallSegments on the {M} final grids, plus wallAngle once per 20",
                                    "wallSegments_ms_per_map": 1e3 * t_seg / M, "wallAngle_ms_per_map": 1e3 * t_ang / M}
    except Exception as e:
        line["cpu_baseline"] = {"error": f"{type(e).__name__}: {e}"}
    return line


def _workload_child(argv: list, local_rank: int) -> dict:
    """One `bench.py --workload …` run in a process of its own, on the same GPU; its JSON line.
    In the config-1 process, after the 64-map chain and the 16-thread CPU baseline, the config-2
    association ran at a quarter of its own process's rate (25.9 k vs 109.6 k frames/s at 32
    frames per call), so each configuration is timed the way its own `--workload` run times it."""
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_WORLD_SIZE", "GROUP_RANK",
                                                            "ROLE_RANK", "MASTER_ADDR", "MASTER_PORT")}
    env["LOCAL_RANK"] = str(local_rank)
    p = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py")] + argv, env=env, cwd=ROOT,
                       capture_output=True, text=True, timeout=600)
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
    if p.returncode != 0 or not lines:
        raise RuntimeError(f"rc {p.returncode}: {(p.stderr or p.stdout)[-300:]}")
    line = json.loads(lines[-1])
    line["process"] = "own: bench.py " + " ".join(argv)
    return line


def extra_workloads(args, local_rank: int) -> dict:
    """Short device-timed runs of the other configurations, so the default run records them:
    config 2 (association GEMM, 32 frames per call) and config 3 (occupancy insert + scan match,
    one map), each as its own `--workload` process with fewer steps and no CPU baseline; then
    the wall extraction on this process's config-1 maps."""
    out = {}
    # 200 calls (about 60 ms): a 20-call window (6 ms) was seen to catch the clocks ramping
    try:
        out["config2"] = _workload_child(["--workload", "assoc", "--steps", "200", "--warmup", "20",
                                          "--assoc-frames", "32", "--no-cpu-baseline"], local_rank)
    except Exception as e:   # recorded, not fatal to the headline line
        out["config2"] = {"error": f"{type(e).__name__}: {e}"}
    try:
        out["config3"] = _workload_child(["--workload", "occ", "--steps", "30", "--warmup", "3", "--maps", "1",
                                          "--scans", "200", "--no-cpu-baseline"], local_rank)
    except Exception as e:
        out["config3"] = {"error": f"{type(e).__name__}: {e}"}
    try:
        out["walls"] = run_walls(args, local_rank)
    except Exception as e:
        out["walls"] = {"error": f"{type(e).__name__}: {e}"}
    return out


if __name__ == "__main__":
    main()
