#!/usr/bin/env python
"""Benchmark of the B200 hot path: full-page OCR, pages/s (BASELINE metric; config 4 by default).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--pages B] [--impl b200|reference]
                    [--workload pp4|pp4ink|det1|...] [--lanes L] [--merge M]

Default workload (`pp4`): the PP-OCRv6 page pipeline of the reference's bench
(src/bin/ocr-bench.rs:133-310, 458-585 with DET=ppocr REC=ppocr): per page detection
(NdGraph::det_input + the DB detector, seed 3), DB boxes at 0.3 (`ppdet::boxes`), line images
(`ppocr::line_input`, batched 16 by width) and recognition (the SVTR recogniser, seed 2, arg-max
per step).  A step is B synthetic 2550 x 3300 pages per GPU through `wocr_pp_pages` (L lanes on
the GPU, recognitions merged M pages at a time per lane).  Pages shard across GPUs with no
collective (weak scaling): one process per GPU (torchrun), timed on the device, max over ranks.

  value  - pages/s with the pages already in HBM (B pages = 303 MB > L2 per step)
  e2e    - pages/s through the same public call from pinned host pages: the pages' upload and
           the read-back of every line's arg-max classes inside the timed region
  roofline - the kernel with the largest share of device time in a CUDA-event profile of the
           same workload (one lane): algorithmic bytes (or FLOPs) per launch / its mean time
  cpu_baseline - the CPU oracle (a C/numpy restatement of the reference's arithmetic, OpenMP)
           on a bounded sample of pages, on this host's cores

`--workload det1` is config 1 (ocrs detection alone); the others are secondary measurements.
`--impl reference` times the reference's CPU implementation stand-in (the oracle; the reference
itself is Rust + wgpu and cannot run here) on the same workload, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
from concurrent.futures import ThreadPoolExecutor
import os
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "wgpu-ocr_b200"))

W_PAGE, H_PAGE = 2550, 3300
THRESHOLD = 0.5
WORKLOAD = "config 1: ocrs detection U-Net (16/32/64/128 ch, 800x600 model input, He-normal seed 1), " \
           "2550x3300 RGB u8 synthetic pages, threshold 0.5, bit-mask output"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=30)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--pages", type=int, default=12, help="pages per GPU per step")
    p.add_argument("--impl", default="b200", choices=["b200", "reference"])
    p.add_argument("--cpu-sample", type=int, default=2, help="pages of the CPU-baseline sample")
    p.add_argument("--workload", default="pp4",
                   choices=["pp4", "pp4ink", "ocrs2", "ocrs2ink", "det1", "rec0", "pp3", "ctc3", "ppdet4", "ppdb4",
                            "pplines", "words1"],
                   help="pp4 (default, the driver's line): config 4, the full PP-OCRv6 page pipeline (pp4ink: "
                        "with a hand-set ink detector, hundreds of lines a page); ocrs2: config 2, the full ocrs page "
                        "pipeline (ocrs2ink: with a hand-set ink detector, 36 lines a page); det1: config 1 detection; rec0 / "
                        "pp3 / ppdet4: configs 0, 3 and 4 through their public calls; ctc3: config 3's CTC head alone over "
                        "all its steps' rows; ppdb4: config 4 with the DB "
                        "mask and box scores on the device; pplines: PP line extraction; words1: word rectangles "
                        "of config 1 detection masks (secondary measurements)")
    p.add_argument("--lanes", type=int, default=4,
                   help="workers per GPU: page-pipeline lanes (pp4, pp4ink, ocrs2, ocrs2ink); contexts with a "
                        "host thread each over the width batches (pp3)")
    p.add_argument("--merge", type=int, default=3, help="pages whose recognitions a lane runs together")
    p.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU-baseline sample length (pp4, pp4ink)")
    return p.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(path))
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "src": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


def traffic_per_launch(kernel: str):
    """DRAM bytes per launch of `kernel` (dram__bytes_read.sum + dram__bytes_write.sum averaged
    over one step's launches) from the committed ncu summary, or None."""
    path = os.path.join(ROOT, "profiles", "tconv_config1.md")
    try:
        for line in open(path):
            if line.startswith("traffic per launch (bytes):"):
                for item in line.split(":", 1)[1].split():
                    name, _, val = item.partition("=")
                    if name == kernel:
                        return float(val)
    except OSError:
        pass
    return None


def roofline(top, total_ms: float, with_traffic: bool = True):
    """Roofline of the dominant kernel: algorithmic FLOPs and bytes per launch over its average
    launch time (CUDA events).  The bound is the resource whose peak would take longer for that
    work (HBM at the measured copy bandwidth, or the tensor cores at the measured dense bf16
    rate); the other one is reported beside it."""
    pk = peaks()
    n = max(top["launches"], 1)
    t = top["ms"] / n / 1e3
    flops, nbytes = top["flops"] / n, top["bytes"] / n
    hbm = {"achieved": nbytes / t / 1e9, "peak": pk["hbm_gbs"], "unit": "GB/s"}
    hbm["frac"] = hbm["achieved"] / hbm["peak"]
    ten = {"achieved": flops / t / 1e12, "peak": pk["bf16_tflops"], "unit": "TFLOP/s"}
    ten["frac"] = ten["achieved"] / ten["peak"]
    t_hbm = nbytes / (pk["hbm_gbs"] * 1e9)
    t_ten = flops / (pk["bf16_tflops"] * 1e12)
    if flops > 0 and t_ten > t_hbm:
        roof, other, oname = dict(bound="tensor", **ten), hbm, "hbm"
        src = " (dense bf16 cuBLAS burst)"
    else:
        roof, other, oname = dict(bound="hbm", **hbm), ten, "tensor"
        src = " (copy bandwidth)"
    tr = traffic_per_launch(top["kernel"]) if with_traffic else None
    roof.update({"traffic": tr, "kernel": top["kernel"], "share": top["ms"] / total_ms,
                 "algorithmic_bytes_per_launch": nbytes, "algorithmic_flops_per_launch": flops,
                 "peak_source": pk["src"] + src, oname: other})
    return roof


class Clocks:
    """SM clock and throttle reasons of this process's GPU, sampled every 200 ms by NVML in a
    thread while the timed region runs (nvidia-smi's own 100 ms loop over every GPU of the box
    was seen to stall the timed kernels)."""

    def __init__(self, bus_id):
        self.bus = bus_id if isinstance(bus_id, int) else None   # torch's pci_bus_id (an int)
        self.samples = []
        self.stop_flag = threading.Event()
        self.err = None

    def _handle(self, nv):
        n = nv.nvmlDeviceGetCount()
        for i in range(n):
            h = nv.nvmlDeviceGetHandleByIndex(i)
            if self.bus is None or nv.nvmlDeviceGetPciInfo(h).bus == self.bus:
                return h
        return nv.nvmlDeviceGetHandleByIndex(0)

    def _run(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = self._handle(nv)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            bits = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                    "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                    "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                    "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap}
            while not self.stop_flag.is_set():
                mhz = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((mhz, [k for k, b in bits.items() if r & b]))
                self.stop_flag.wait(0.2)
            nv.nvmlShutdown()
        except Exception as e:  # no NVML: report it instead of clocks
            self.err = str(e)

    def start(self):
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()

    def stop(self):
        time.sleep(0.05)
        self.stop_flag.set()
        self.t.join(timeout=5)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.err or "no samples"], "samples": 0}
        sm = sorted(s[0] for s in self.samples)
        reasons = sorted({r for s in self.samples for r in s[1]})
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": getattr(self, "max_mhz", None), "reasons": reasons,
                "samples": len(sm)}


def dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def make_pages(rank: int, n: int):
    """This rank's pages (weak scaling: n per rank, global page g from seed 1000 + g)."""
    import numpy as np
    from wocr import synth
    from wocr.shard import weak_pages_of
    return np.stack([synth.page(1000 + g, W_PAGE, H_PAGE) for g in weak_pages_of(rank, n)])


def cpu_baseline(sample: int):
    """The oracle on `sample` pages with all host threads: pages/s."""
    from oracle import ref
    from wocr import synth
    m = synth.ocrs_det_model()
    pgs = [synth.page(7000 + k, W_PAGE, H_PAGE) for k in range(sample + 1)]
    ref.set_threads(os.cpu_count() or 1)
    ref.detect_page(m, pgs[0], THRESHOLD)            # warm-up (library load, page-in)
    t0 = time.perf_counter()
    for p in pgs[1:]:
        ref.detect_page(m, p, THRESHOLD)
    dt = time.perf_counter() - t0
    return {"value": sample / dt, "unit": "pages/s", "cores": ref.threads(), "kind": "port",
            "sample": f"{sample} pages of config 1 through the C oracle (grey/resize, U-Net, mask), "
                      f"{dt:.2f} s"}


PP_MAX_SIDE = 960
PP_DB = (0.3, 0.45, 1.4, 3.0)


def pp_workload(ink: bool):
    """Config 4's models and its description (pp4ink: the ink detector in place of the DB's)."""
    from wocr import synth
    det_m = synth.pp_ink_det_model() if ink else synth.pp_det_model()
    detector = ("a hand-set ink detector (darkness, 3x9 box average, sigmoid) standing in for trained DB weights, "
                "which marks word blobs" if ink else
                "the PP-OCRv6-style DB detector with random-init weights (seed 3), which mark most of each page, "
                "so a page gives about one page-sized box")
    desc = (f"config 4 full page: {detector}; 2550x3300 RGB u8 synthetic pages (36 text bands), det input "
            f"3x960x736, DB boxes at 0.3 on the device, lines grown 0.1 x height, cut to height 48 and batched "
            f"16 by width on the device, PP-OCRv6-style recognition (seed 2, 18,709 classes), arg-max per step")
    return det_m, synth.pp_rec_model(), desc


def oracle_pp_page(det_m, rec_m, page):
    """One page of config 4 through the CPU oracle: detection, DB boxes, line images,
    recognition arg-max.  Returns the number of lines."""
    from oracle import ref
    x, tp = ref.det_input(page, PP_MAX_SIDE)
    prob = ref.run_onnx(det_m, x)[0, 0]
    boxes = ref.db_boxes(prob, tp, *PP_DB)
    batches, _ = ref.pp_batches(page, ref.pp_line_rects(boxes, 0.1))
    for data, _, _ in batches:
        lg = ref.run_onnx(rec_m, data, stop_before_softmax=True)
        ref.argmax(lg.reshape(-1, lg.shape[-1]))
    return len(boxes)


def ocrs_workload(ink: bool):
    """Config 2's models and its description (ocrs2ink: the ink detector in place of the U-Net)."""
    from wocr import synth
    det_m = synth.ocrs_ink_det_model() if ink else synth.ocrs_det_model()
    detector = ("a hand-set ink detector (darkness, 3x5 box sum, sigmoid) standing in for trained ocrs weights, "
                "which marks words" if ink else
                "the ocrs-style detection U-Net with random-init weights (seed 1), whose mask is noise-like, so a "
                "page gives about one page-sized word and line")
    desc = (f"config 2 full ocrs page: {detector}; 2550x3300 RGB u8 synthetic pages (36 text bands), grey/resize "
            f"to 800x600, mask at 0.5, word rectangles (expand 3, min area 100), text lines (ocrs line grouping "
            f"restated), lines padded 0.15 / 0.1 x median height, 64-row line images batched by width, ocrs-style "
            f"recognition (conv trunk + 2-layer biGRU(256) + Linear 512->97, seed 0), arg-max per step")
    return det_m, synth.ocrs_rec_model(), desc


def oracle_ocrs_page(det_m, rec_m, page):
    """One page of config 2 through the CPU oracle: detection, word rectangles, lines, line
    images, recognition.  Returns the number of lines."""
    from oracle import ref
    h, w = page.shape[:2]
    bits, _, _ = ref.detect_page(det_m, page, THRESHOLD)
    lines = ref.ocrs_page_lines(bits, w, h)
    if lines:
        batches, _, _ = ref.ocrs_line_batches(page, lines)
        ref.recognize(rec_m, batches)
    return len(lines)


def page_workload(name: str):
    """(models, description, oracle page function) of a full-page workload."""
    if name in ("pp4", "pp4ink"):
        det_m, rec_m, desc = pp_workload(name == "pp4ink")
        return det_m, rec_m, desc, oracle_pp_page
    det_m, rec_m, desc = ocrs_workload(name == "ocrs2ink")
    return det_m, rec_m, desc, oracle_ocrs_page


def run_reference(args):
    world, rank, _ = dist()
    if rank != 0:
        return 0
    if args.workload in ("pp4", "pp4ink", "ocrs2", "ocrs2ink"):
        return run_reference_pages(args)
    from oracle import ref
    from wocr import synth
    m = synth.ocrs_det_model()
    page = synth.page(7000, W_PAGE, H_PAGE)
    ref.set_threads(os.cpu_count() or 1)
    for _ in range(args.warmup):
        ref.detect_page(m, page, THRESHOLD)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        ref.detect_page(m, page, THRESHOLD)
    dt = time.perf_counter() - t0
    v = args.steps / dt
    line = {"impl": "reference", "metric": "pages/s", "value": v, "unit": "pages/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "step": "1 page per step (bounded CPU sample)",
                       "parallelism": "host threads"},
            "cpu_baseline": {"value": v, "unit": "pages/s", "cores": ref.threads(), "kind": "port",
                             "sample": "1 page per step through the C oracle (the reference is Rust + wgpu over "
                                       "Vulkan and cannot run here)"},
            "e2e": {"value": v, "unit": "pages/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def run_b200(args):
    import numpy as np
    import torch
    import torch.distributed as tdist

    import wocr
    from wocr import synth

    world, rank, local = dist()
    if world > 1:
        from datetime import timedelta
        tdist.init_process_group("nccl", timeout=timedelta(seconds=300))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    B = args.pages
    words = (W_PAGE + 31) // 32

    gpu = wocr.Gpu(lines=8, device=local)
    det = wocr.Detector(gpu, synth.ocrs_det_model())
    host_pages = make_pages(rank, B)
    d_rgb = torch.from_numpy(host_pages).to(dev)
    d_mask = torch.empty(B * H_PAGE * words, dtype=torch.int32, device=dev)
    torch.cuda.synchronize(dev)
    stream = torch.cuda.ExternalStream(gpu.stream, device=dev)

    def step():
        det.detect_pages_device(d_rgb.data_ptr(), B, W_PAGE, H_PAGE, THRESHOLD, d_mask.data_ptr())

    from wocr import shard

    def barrier():
        shard.barrier(local)
        torch.cuda.synchronize(dev)

    def max_over_ranks(v: float) -> float:
        return shard.max_over_ranks(v, dev)

    # ---- device-resident throughput --------------------------------------------------
    for _ in range(max(args.warmup, 3)):
        step()
    gpu.submit_wait()
    barrier()
    bus = None
    try:
        bus = torch.cuda.get_device_properties(dev).pci_bus_id
    except Exception:
        bus = None
    clocks = Clocks(bus)
    clocks.start()
    l0 = gpu.launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    e1.synchronize()
    launches = gpu.launches() - l0
    clk = clocks.stop()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1))
    value = world * B * args.steps / (ms / 1e3)

    # ---- per-kernel profile of the same workload (separate pass) -----------------------
    psteps = min(args.steps, 5)
    gpu.profile(True)
    for _ in range(psteps):
        step()
    rep = gpu.profile_report()
    gpu.profile(False)
    total_ms = sum(r["ms"] for r in rep) or 1.0
    top = max(rep, key=lambda r: r["ms"])
    roof = roofline(top, total_ms)
    kernels = {r["kernel"]: {"launches": r["launches"] // psteps, "ms_per_step": r["ms"] / psteps,
                             "share": r["ms"] / total_ms} for r in rep}

    # ---- end to end through the public API, pinned host buffers -------------------------
    import ctypes
    nbytes = host_pages.nbytes
    hp = ctypes.c_void_p()
    wocr.lib().wocr_host_alloc(nbytes, ctypes.byref(hp))
    hm = ctypes.c_void_p()
    mbytes = B * H_PAGE * words * 4
    wocr.lib().wocr_host_alloc(mbytes, ctypes.byref(hm))
    ctypes.memmove(hp.value, host_pages.ctypes.data, nbytes)

    def e2e_step():
        wocr._lib.check(wocr.lib().wocr_detect_pages(det.h, hp, B, W_PAGE, H_PAGE, THRESHOLD, hm))

    for _ in range(2):
        e2e_step()
    barrier()
    e0.record(stream)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    e1.synchronize()
    wall = time.perf_counter() - t0
    ems = max_over_ranks(max(e0.elapsed_time(e1), 1e3 * wall))
    # the bytes that crossed PCIe in one call (tall pages go up compacted to the rows they use)
    h2d_step, d2h_step = det.last_transfer_bytes()
    e2e = {"value": world * B * args.steps / (ems / 1e3), "unit": "pages/s", "h2d_bytes_per_step": int(h2d_step),
           "d2h_bytes_per_step": int(d2h_step), "host_page_bytes_per_step": int(nbytes)}
    wocr.lib().wocr_host_free(hp)
    wocr.lib().wocr_host_free(hm)

    cpu = None
    if rank == 0 and world == 1:
        cpu = cpu_baseline(args.cpu_sample)

    flops_step, _ = det.stats()
    if rank == 0:
        line = {"metric": "pages/s", "value": value, "unit": "pages/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": WORKLOAD, "pages_per_gpu_per_step": B, "global_batch": B * world,
                           "parallelism": f"pages sharded over {world} GPU(s), no collective",
                           "l2": f"inputs {B * W_PAGE * H_PAGE * 3 / 1e6:.0f} MB per GPU per step > 126 MB L2"},
                "e2e": e2e, "gpu_launches": int(launches), "roofline": roof, "cpu_baseline": cpu,
                "clocks": clk, "kernels": kernels,
                "algorithmic_gflop_per_page": det.stats()[0] / B / 1e9 if flops_step else None}
        print(json.dumps(line), flush=True)
    det.close()
    gpu.close()
    if world > 1:
        tdist.barrier(device_ids=[local])
        tdist.destroy_process_group()
    return 0


def run_reference_pages(args):
    """The reference arm on config 4: the CPU oracle, one page per step, all host threads."""
    from oracle import ref
    from wocr import synth
    det_m, rec_m, desc, oracle_page = page_workload(args.workload)
    pages = [synth.page(7000 + k, W_PAGE, H_PAGE) for k in range(max(args.steps, 1) + max(args.warmup, 1))]
    ref.set_threads(os.cpu_count() or 1)
    for k in range(args.warmup):
        oracle_page(det_m, rec_m, pages[k])
    t0 = time.perf_counter()
    nl = 0
    for k in range(args.steps):
        nl += oracle_page(det_m, rec_m, pages[args.warmup + k])
    dt = time.perf_counter() - t0
    v = args.steps / dt
    line = {"impl": "reference", "metric": "pages/s", "value": v, "unit": "pages/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": desc, "step": "1 page per step (bounded CPU sample)", "parallelism": "host threads",
                       "lines_per_page": nl / max(args.steps, 1)},
            "cpu_baseline": {"value": v, "unit": "pages/s", "cores": ref.threads(), "kind": "port",
                             "sample": "1 page per step through the CPU oracle (the reference is Rust + wgpu over "
                                       "Vulkan and cannot run here)"},
            "e2e": {"value": v, "unit": "pages/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def run_pages(args):
    """Configs 4 (default) and 2: a whole page pipeline, B pages per GPU per step."""
    import ctypes

    import numpy as np
    import torch
    import torch.distributed as tdist

    import wocr
    from wocr import shard, synth

    world, rank, local = dist()
    if world > 1:
        from datetime import timedelta
        tdist.init_process_group("nccl", timeout=timedelta(seconds=300))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    B, L, M = args.pages, max(1, args.lanes), max(1, args.merge)
    det_m, rec_m, desc, oracle_page = page_workload(args.workload)
    ocrs = args.workload.startswith("ocrs")
    gpu = wocr.Gpu(lines=8, device=local)
    pp = (wocr.OcrsPipeline if ocrs else wocr.PPPipeline)(gpu, det_m, rec_m)
    host_np = [synth.page(3000 + g, W_PAGE, H_PAGE) for g in shard.weak_pages_of(rank, B)]
    held = []

    def pinned(a):
        p = ctypes.c_void_p()
        wocr._lib.check(wocr.lib().wocr_host_alloc(a.nbytes, ctypes.byref(p)))
        held.append(p)
        out = np.frombuffer((ctypes.c_char * a.nbytes).from_address(p.value), dtype=a.dtype,
                            count=a.size).reshape(a.shape)
        out[...] = a
        return out

    host = [pinned(a) for a in host_np]
    d_pages = [torch.from_numpy(a).to(dev) for a in host_np]
    d_ptrs = [t.data_ptr() for t in d_pages]
    torch.cuda.synchronize(dev)

    def barrier():
        shard.barrier(local)
        torch.cuda.synchronize(dev)

    def step(src, lanes=L):
        if ocrs:
            return pp.pages(src, W_PAGE, H_PAGE, threshold=THRESHOLD, merge=M, lanes=lanes)
        return pp.pages(src, W_PAGE, H_PAGE, max_side=PP_MAX_SIDE, db=PP_DB, merge=M, lanes=lanes)

    # warm-up: every lane captures its graphs for every batch shape of these pages
    for _ in range(max(args.warmup, 3)):
        res = step(d_ptrs)
    if ocrs:
        lines_per_page = sum(len(ls) for ls in res) / B
        steps_per_page = sum(sum(len(b) for _, _, b in ls) for ls in res) / B
    else:
        lines_per_page = sum(len(b) for b, _ in res) / B
        steps_per_page = sum(sum(len(x) for x in ls) for _, ls in res) / B
    barrier()
    bus = None
    try:
        bus = torch.cuda.get_device_properties(dev).pci_bus_id
    except Exception:
        bus = None
    # the call is synchronous and spreads over L streams; events on a stream of their own bracket
    # it, so the elapsed time covers every lane's work and the host steps between
    ts = torch.cuda.Stream(device=dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = Clocks(bus)
    clocks.start()
    l0 = pp.launches()
    e0.record(ts)
    for _ in range(args.steps):
        step(d_ptrs)
    e1.record(ts)
    e1.synchronize()
    clk = clocks.stop()
    launches = pp.launches() - l0
    barrier()
    ms = shard.max_over_ranks(e0.elapsed_time(e1), dev)
    value = world * B * args.steps / (ms / 1e3)

    # end to end: pinned host pages in, every line's classes out
    for _ in range(2):
        step(host)
    barrier()
    e0.record(ts)
    for _ in range(args.steps):
        step(host)
    e1.record(ts)
    e1.synchronize()
    h2d, d2h = pp.last_bytes
    barrier()
    ems = shard.max_over_ranks(e0.elapsed_time(e1), dev)
    e2e = {"value": world * B * args.steps / (ems / 1e3), "unit": "pages/s", "h2d_bytes_per_step": int(h2d),
           "d2h_bytes_per_step": int(d2h)}

    # per-kernel profile of one more step on one lane (the profile records the caller's context)
    gpu.profile(True)
    step(d_ptrs, lanes=1)
    rep = gpu.profile_report()
    gpu.profile(False)
    total_ms = sum(r["ms"] for r in rep) or 1.0
    top = max(rep, key=lambda r: r["ms"])
    roof = roofline(top, total_ms, with_traffic=False)
    roof["traffic"] = pp_traffic(top["kernel"])
    if top["kernel"] in LATENCY_KERNELS:
        # the dominant share is a latency chain (a block per page component); beside it, the
        # roofline of the largest kernel that fills the GPU (FLOPs or bytes recorded for it)
        roof["note"] = LATENCY_KERNELS[top["kernel"]]
        fill = [r for r in rep if r["kernel"] not in LATENCY_KERNELS and (r["flops"] > 0 or r["bytes"] > 0)]
        if fill:
            ft = max(fill, key=lambda r: r["ms"])
            fr = roofline(ft, total_ms, with_traffic=False)
            fr["traffic"] = pp_traffic(ft["kernel"])
            roof["largest_throughput_kernel"] = fr
    kernels = {r["kernel"]: {"launches": r["launches"], "ms_per_step": r["ms"], "share": r["ms"] / total_ms}
               for r in rep}

    cpu = None
    if rank == 0 and world == 1:
        from oracle import ref
        ref.set_threads(os.cpu_count() or 1)
        oracle_page(det_m, rec_m, host_np[0])  # warm-up
        t0, k, nl = time.perf_counter(), 0, 0
        while k < 2 or (time.perf_counter() - t0 < args.cpu_seconds and k < B):
            nl += oracle_page(det_m, rec_m, host_np[k % B])
            k += 1
        dt = time.perf_counter() - t0
        cpu = {"value": k / dt, "unit": "pages/s", "cores": ref.threads(), "kind": "port",
               "sample": f"{k} pages ({nl} lines) of this workload through the CPU oracle (detection, DB boxes, "
                         f"line images, recognition arg-max), {dt:.1f} s"}
    if rank == 0:
        line = {"metric": "pages/s", "value": value, "unit": "pages/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": desc, "pages_per_gpu_per_step": B, "global_batch": B * world,
                           "lanes_per_gpu": L, "merge": M, "lines_per_page": lines_per_page,
                           "recognition_steps_per_page": steps_per_page,
                           "parallelism": f"pages sharded over {world} GPU(s), no collective",
                           "l2": f"inputs {B * W_PAGE * H_PAGE * 3 / 1e6:.0f} MB per GPU per step > 126 MB L2"},
                "e2e": e2e, "gpu_launches": int(launches),
                "roofline": roof, "cpu_baseline": cpu, "clocks": clk, "kernels": kernels}
        print(json.dumps(line), flush=True)
    pp.close()
    gpu.close()
    for p_ in held:
        wocr.lib().wocr_host_free(p_)
    if world > 1:
        tdist.barrier(device_ids=[local])
        tdist.destroy_process_group()
    return 0


# kernels whose time is a dependent chain, not bytes or FLOPs: the roofline fraction of HBM or the
# tensor cores is not their bound
LATENCY_KERNELS = {
    "word_rect": "latency-bound: one block per page component runs its Douglas-Peucker levels in "
                 "sequence (927 levels of a 5,471-point border for a page-sized component), so the "
                 "HBM fraction is not its bound",
    "word_trace": "latency-bound: one warp per component follows its border a point at a time",
    "word_label": "bound by the union-find's atomic links on the page-sized component's roots",
}


def pp_traffic(kernel: str):
    """DRAM bytes per launch of `kernel` in config 4's page pipeline from the committed ncu
    summary, or None."""
    path = os.path.join(ROOT, "profiles", "pp_page_config4.md")
    try:
        for line in open(path):
            if line.startswith("traffic per launch (bytes):"):
                for item in line.split(":", 1)[1].split():
                    name, _, val = item.partition("=")
                    if name == kernel:
                        return float(val)
    except OSError:
        pass
    return None


def run_workload(args):
    """Configs 0, 3 and 4 and the next rows through the public calls a user makes (host inputs in
    pinned memory, as the reference's Recognizer::recognize, NdGraph::run + argmax and the PP
    detection page take them; device pages for the line and word kernels).  `value`: units over
    the context stream's busy time (CUDA events; the H2D copies the call makes are inside);
    `e2e`: the same over wall-clock time of the calls."""
    import numpy as np
    import torch

    import wocr
    from oracle import ref
    from wocr import synth

    world, rank, local = dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    gpu = wocr.Gpu(lines=8, device=local)
    stream = torch.cuda.ExternalStream(gpu.stream, device=dev)
    ref.set_threads(os.cpu_count() or 1)
    held = []

    def pinned(a):
        """A copy of `a` in page-locked host memory (`wocr_host_alloc`): the timed calls' inputs
        come from pinned memory, as the driver's end-to-end contract asks."""
        import ctypes
        p = ctypes.c_void_p()
        wocr._lib.check(wocr.lib().wocr_host_alloc(max(a.nbytes, 1), ctypes.byref(p)))
        held.append(p)
        out = np.frombuffer((ctypes.c_char * max(a.nbytes, 1)).from_address(p.value), dtype=a.dtype,
                            count=a.size).reshape(a.shape)
        out[...] = a
        return out

    serial_step = None  # the one-lane step the per-kernel profile runs (default: step)

    def lane_launches():
        return 0

    def close_lanes():
        pass

    if args.workload == "rec0":
        model = synth.ocrs_rec_model()
        batches, _, _ = synth.ocrs_batches(synth.ocrs_lines(0, n=64))
        batches = [(pinned(np.ascontiguousarray(d, np.float32)), n, w) for d, n, w in batches]
        handle = wocr.Recognizer(gpu, model)
        units, unit, workload = 64, "lines/s", ("config 0: ocrs recognition, 64 lines 1x64xW (W ~ U{64..1024}), "
                                                "conv trunk + 2-layer biGRU(256) + Linear 512->97, seed 0")
        tmax, ntot, classes = handle.dims(batches)
        h2d = sum(b[0].nbytes for b in batches)
        d2h = tmax * ntot * (classes + 1) * 4

        def step():
            handle.recognize(batches, want_logits=True)

        sample = batches[:1]

        def cpu():
            ref.recognize(model, sample)
            return sum(b[1] for b in sample), f"{sum(b[1] for b in sample)} lines (the first width bucket)"
    elif args.workload == "pp3":
        model = synth.pp_rec_model()
        batches, _ = synth.pp_batches(synth.pp_lines(2, n=256))
        batches = [(pinned(np.ascontiguousarray(d, np.float32)), n, w) for d, n, w in batches]
        handle = wocr.NdGraph(gpu, model, stop_before_softmax=True)
        # lanes: more contexts (each its own stream and graph), a host thread each; the width
        # batches go to the least loaded lane, widest first (a batch's cost ~ lines x width)
        L = max(1, args.lanes)
        lane_gpus = [wocr.Gpu(lines=8, device=local) for _ in range(L - 1)]
        lane_handles = [handle] + [wocr.NdGraph(g_, model, stop_before_softmax=True) for g_ in lane_gpus]
        plan, load = [[] for _ in range(L)], [0] * L
        for i in sorted(range(len(batches)), key=lambda i: -batches[i][1] * batches[i][2]):
            k_ = load.index(min(load))
            plan[k_].append(i)
            load[k_] += batches[i][1] * batches[i][2]
        pool = ThreadPoolExecutor(L) if L > 1 else None
        units, unit, workload = 256, "lines/s", ("config 3: PP-OCRv6-style recognition, 256 lines 3x48xW "
                                                 "(W ~ U{96..1280}), trunk + 2 SVTR blocks + CTC head 120->18709, "
                                                 f"seed 2, arg-max per step; {len(batches)} width batches over {L} "
                                                 "lane(s) (a context and a host thread each)")
        h2d = sum(b[0].nbytes for b in batches)
        d2h = sum(b[1] * (b[2] // 8) * 8 for b in batches)  # classes and maxima, 4 bytes each a step

        # the classes per step, as the reference's NdGraph::argmax gives them (no log-sum-exp)
        def run_lane(k_):
            for i in plan[k_]:
                lane_handles[k_].argmax(batches[i][0], lse=False)

        def step():
            if pool is None:
                run_lane(0)
            else:
                list(pool.map(run_lane, range(L)))

        def serial_step():
            for data, _, _ in batches:
                handle.argmax(data, lse=False)

        def lane_launches():
            return sum(g_.launches() for g_ in lane_gpus)

        def close_lanes():
            if pool is not None:
                pool.shutdown()
            for h_ in lane_handles[1:]:
                h_.close()
            for g_ in lane_gpus:
                g_.close()

        def cpu():
            data, n, _ = batches[0]
            logits = ref.run_onnx(model, data, stop_before_softmax=True)
            ref.argmax(logits.reshape(-1, logits.shape[-1]))
            return n, f"{n} lines (the narrowest batch)"
    elif args.workload == "ctc3":
        # the CTC head of config 3 (120 -> 18,709 with the fused arg-max, classes only as the
        # reference's argmax) once over the rows of all 16 width batches (sum of lines x steps)
        batches, _ = synth.pp_batches(synth.pp_lines(2, n=256))
        rows = sum(n_ * (w_ // 8) for _, n_, w_ in batches)
        b_ = synth._Builder(2)
        model = b_.model("x", b_.linear("x", 120, 18709))
        handle = wocr.NdGraph(gpu, model)
        xin = pinned(np.random.default_rng(5).standard_normal((1, rows, 120)).astype(np.float32))
        units, unit, workload = rows, "rows/s", (f"config 3 CTC head alone: Linear 120 -> 18709 (random init, seed 2) "
                                                 f"with the fused row arg-max over {rows} rows (the 256 lines' steps "
                                                 f"of all width batches at once), classes read back")
        h2d, d2h = xin.nbytes, rows * 8

        def step():
            handle.argmax(xin, lse=False)

        def cpu():
            sub = np.ascontiguousarray(xin[:, :512])
            logits = ref.run_onnx(model, sub)
            ref.argmax(logits.reshape(-1, logits.shape[-1]))
            return 512, "512 rows through the CPU oracle (matmul + arg-max)"
    elif args.workload == "pplines":
        handle = None
        npg = 12
        seeds = [3000 + k for k in range(npg)]
        pages_np = [synth.page(sd, W_PAGE, H_PAGE) for sd in seeds]
        boxes = [synth.page_line_boxes(sd, W_PAGE, H_PAGE) for sd in seeds]
        d_pages = [torch.from_numpy(pg).to(dev) for pg in pages_np]
        cap = max(gpu.pp_lines(0, W_PAGE, H_PAGE, b)[2] for b in boxes)
        d_out = torch.empty(cap, dtype=torch.float32, device=dev)
        torch.cuda.synchronize()
        units = sum(len(b) for b in boxes)
        unit, workload = "lines/s", (f"config 3/4 line extraction: {units} PP-OCR recognition lines cut from {npg} "
                                     "device-resident 2550x3300 pages (36 text bands each, boxes padded 0.1 x height), "
                                     "resized to height 48 (Triangle), normalised, batched 16 by width")
        h2d = sum(len(b) for b in boxes) * 32  # the line plans
        d2h = 0

        def step():
            for dp, b in zip(d_pages, boxes):
                gpu.pp_lines(dp.data_ptr(), W_PAGE, H_PAGE, b, 16, d_out.data_ptr(), cap)

        def cpu():
            ref.pp_batches(pages_np[0], boxes[0])
            return len(boxes[0]), f"{len(boxes[0])} lines (one page)"
    elif args.workload == "words1":
        handle = None
        npg = 12
        masks = synth.pack_mask(np.stack([synth.page_word_mask(2000 + k, W_PAGE, H_PAGE) for k in range(npg)]))
        d_masks = torch.from_numpy(masks.view(np.int32)).to(dev)
        torch.cuda.synchronize()
        nrects = sum(len(r) for r in gpu.word_rects(None, W_PAGE, H_PAGE, d_mask=d_masks.data_ptr(), n=npg))
        units, unit, workload = npg, "pages/s", (f"config 1 word rectangles: word_rects (external contours, "
                                                 f"Douglas-Peucker 2 px, minimum-area rectangles, expand 3, min "
                                                 f"area 100) of {npg} device-resident 2550x3300 text masks of "
                                                 f"synthetic pages (seeds 2000..2011: each page's ink rectangles "
                                                 f"grown 8 x 3 px into word blobs, as a trained detector marks "
                                                 f"words), {nrects} rectangles read back")
        h2d, d2h = 0, nrects * 24 + npg * 4

        def step():
            gpu.word_rects(None, W_PAGE, H_PAGE, d_mask=d_masks.data_ptr(), n=npg)

        def cpu():
            ref.word_rects(masks[0], W_PAGE, H_PAGE)
            return 1, "1 page"
    elif args.workload == "ppdb4":
        model = synth.pp_det_model()
        page = pinned(synth.page(3, W_PAGE, H_PAGE))
        handle = wocr.NdGraph(gpu, model)
        _, tp = handle.ppdet_page(page, W_PAGE, H_PAGE, 960, read_map=False)
        rects = synth.page_db_candidates(3, W_PAGE, H_PAGE, tp)
        units, unit, workload = 1, "pages/s", (f"config 4 detection + DB scoring: PP-OCRv6-style DB detector on a "
                                               f"2550x3300 page resized to 3x960x736, seed 3, the map kept on the "
                                               f"device, its p > 0.2 bit mask read back and {len(rects)} candidate "
                                               "boxes (the page's ink rectangles and lines) scored on the device")
        h2d, d2h = page.nbytes + len(rects) * 40, 960 * (736 // 32) * 4 + len(rects) * 4

        def step():
            handle.ppdet_page(page, W_PAGE, H_PAGE, 960, read_map=False)
            handle.db_mask(0.2)
            handle.db_scores(rects)

        def cpu():
            x, _ = ref.det_input(page, 960)
            prob = ref.run_onnx(model, x)[0, 0]
            np.packbits(prob > np.float32(0.2), axis=1, bitorder="little")
            ref.db_scores(prob, rects)
            return 1, "1 page"
    else:
        model = synth.pp_det_model()
        page = pinned(synth.page(3, W_PAGE, H_PAGE))
        handle = wocr.NdGraph(gpu, model)
        units, unit, workload = 1, "pages/s", ("config 4 detection: PP-OCRv6-style DB detector on a 2550x3300 "
                                               "page resized to 3x960x736, seed 3, probability map read back")
        h2d, d2h = page.nbytes, 960 * 736 * 4

        def step():
            handle.ppdet_page(page, W_PAGE, H_PAGE, 960)

        def cpu():
            x, _ = ref.det_input(page, 960)
            ref.run_onnx(model, x)
            return 1, "1 page"

    for _ in range(max(args.warmup, 3)):
        step()
    gpu.submit_wait()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    l0 = gpu.launches() + lane_launches()
    e0.record(stream)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    # every lane's calls have returned (they wait for their results): the context stream's event
    # closes the region
    e1.record(stream)
    e1.synchronize()
    wall = time.perf_counter() - t0
    launches = gpu.launches() + lane_launches() - l0
    ms = e0.elapsed_time(e1)
    gpu.profile(True)
    (serial_step or step)()
    rep = gpu.profile_report()
    gpu.profile(False)
    total_ms = sum(r["ms"] for r in rep) or 1.0
    top = max(rep, key=lambda r: r["ms"])
    roof = roofline(top, total_ms, with_traffic=False)  # the committed ncu traffic is config 1's
    cpu_v = None
    if rank == 0:
        c0 = time.perf_counter()
        n, what = cpu()
        dt = time.perf_counter() - c0
        cpu_v = {"value": n / dt, "unit": unit, "cores": ref.threads(), "kind": "port",
                 "sample": f"{what} through the CPU oracle, {dt:.2f} s"}
        line = {"metric": unit, "value": units * args.steps / (ms / 1e3), "unit": unit, "n_gpus": 1,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic", "config": {"workload": workload, "units_per_step": units},
                "e2e": {"value": units * args.steps / wall, "unit": unit, "h2d_bytes_per_step": int(h2d),
                        "d2h_bytes_per_step": int(d2h)},
                "gpu_launches": int(launches), "roofline": roof, "cpu_baseline": cpu_v,
                "kernels": {r["kernel"]: {"launches": r["launches"], "ms_per_step": r["ms"],
                                          "share": r["ms"] / total_ms} for r in rep}}
        print(json.dumps(line), flush=True)
    close_lanes()
    if handle is not None:
        handle.close()
    for p in held:
        wocr.lib().wocr_host_free(p)
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload in ("pp4", "pp4ink", "ocrs2", "ocrs2ink"):
        return run_pages(args)
    if args.workload != "det1":
        return run_workload(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
