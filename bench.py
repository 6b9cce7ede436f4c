#!/usr/bin/env python
"""Throughput benchmark of the PP-OCRv6 hot path on B200 (driver contract).

Default workload: the tiny detector forward at 416x736 (benchmark configs 1
and 3: the reference's ppocr-gpu-bench --kind det shape, batched 32 images per
GPU), seeded uniform-RGB8 inputs, seeded random-init weights in the exact
reference checkpoint layout, FP32.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                  [--kind det|rec|e2e] [--size tiny|small|medium] [--batch B]

One process per GPU (torchrun for N > 1); images shard across ranks with no
collective on the data path (weak scaling).  A step is one forward of the
rank's batch.  `value` is device-timed throughput with inputs resident in HBM
(the model's own input slot), each step bracketed by CUDA events on the
launching stream with an L2 flush between steps; `e2e` is the same metric
through the C ABI's host-buffer forward (pinned H2D input, D2H output).

The default line also carries two secondary figures of the same run
(`secondary`): the medium recognizer in BF16 (config 4, crops/s, device-timed)
and end-to-end pages (config 5: 1920x1080 synthetic pages through the OCR
engine -- detector, DB postprocess, rectification, recognizer, CTC text --
pages/s by wall clock around the public batch call).  `--kind e2e` makes the
page pipeline the headline.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (os.path.join(ROOT, "ppocr-rs_b200"), ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

HBM_FALLBACK_GBS = 6650.0
BF16_FALLBACK_TFLOPS = 1590.0


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return HBM_FALLBACK_GBS, BF16_FALLBACK_TFLOPS, "fallback"


def _workload(args):
    if args.kind == "det":
        h, w = 416, 736
        shape = (args.batch, 3, h, w)
        name = f"{args.size} detector forward, {args.batch}x3x{h}x{w} per GPU"
        unit = "img/s"
        metric = f"det img/s @416x736 ({args.size} detector, batch {args.batch}/GPU)"
    else:
        h, w = 48, 320
        shape = (args.batch, 3, h, w)
        name = f"{args.size} recognizer forward + greedy CTC, {args.batch}x3x{h}x{w} per GPU"
        unit = "crops/s"
        metric = f"rec crops/s @48x320 ({args.size} recognizer, batch {args.batch}/GPU)"
    return shape, name, unit, metric


def _inputs(kind, shape, seed):
    from ppocr_b200 import seeded

    if kind == "det":
        return seeded.det_batch(shape[0], shape[2], shape[3], seed=seed)
    return seeded.rec_batch(shape[0], shape[3], seed=seed)


class _Clocks:
    """nvidia-smi sampler for the timed region."""

    def __init__(self, device):
        self.path = tempfile.mktemp(suffix=".csv")
        self.proc = None
        self.device = device

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        sms, maxs, reasons = [], [], set()
        try:
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sms.append(float(parts[1]))
                    maxs.append(float(parts[2]))
                except ValueError:
                    continue
                for name, val in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"),
                                     parts[5:9]):
                    if val.lower() == "active":
                        reasons.add(name)
        except OSError:
            pass
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxs), "reasons": sorted(reasons),
                "samples": len(sms)}


def _device_view(ptr, count, torch):
    """A torch float32 view of `count` floats at device address `ptr`."""

    class _Ptr:
        __cuda_array_interface__ = {"shape": (count,), "typestr": "<f4", "data": (ptr, False), "version": 2}

    return torch.as_tensor(_Ptr(), device="cuda")


def _cpu_forms(args, shape):
    """The CPU restatements of the reference's CPU path for this workload, as
    (name, forward(x), per-step sample, description) on all host threads:
    the torch port (oracle/model.py, intra-op threads, one image per call) and,
    for the tiny / small detector, the C++ restatement (oracle/cpu_detector.cpp,
    -O3 -march=native -fopenmp, images spread over the threads)."""
    import torch

    from oracle import model as om
    from ppocr_b200 import seeded

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    w = om.Weights(seeded.make_weights(args.kind, args.size, 0, "spec"))
    m = om.Detector(w, args.size) if args.kind == "det" else om.Recognizer(w, args.size)
    forms = [("torch", m.forward, 1 if args.kind == "det" else min(shape[0], 8),
              f"torch-CPU FP32 port of src/cpu/model.rs, {threads} intra-op threads")]
    if args.kind == "det" and args.size in ("tiny", "small"):
        from oracle.cpu_detector import CpuDetector

        tmp = tempfile.mkdtemp(prefix="ppocr_cpu_")
        path = os.path.join(tmp, "w.safetensors")
        seeded.write_weights(path, args.kind, args.size, 0, "spec")
        cpp = CpuDetector(path, args.size)
        forms.append(("c++", lambda x: cpp.forward(x, threads), min(shape[0], max(threads, 2)),
                      f"C++ restatement of src/cpu/model.rs (g++ -O3 -march=native -fopenmp), images over {threads} threads"))
    return forms, threads


def _time_form(fwd, x, seconds):
    fwd(x)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds or n < 2:
        fwd(x)
        n += 1
    return n, time.perf_counter() - t0


def cpu_baseline(args, shape, seconds=12.0):
    """Both CPU restatements on a bounded sample of the workload, all host threads;
    the faster one is the baseline (both rates are listed)."""
    forms, threads = _cpu_forms(args, shape)
    unit = "img/s" if args.kind == "det" else "crops/s"
    rates = {}
    best = None
    for name, fwd, sample, desc in forms:
        x = _inputs(args.kind, (sample,) + tuple(shape[1:]), seed=99)
        n, dt = _time_form(fwd, x, seconds / len(forms))
        rate = n * sample / dt
        rates[name] = round(rate, 3)
        if best is None or rate > best[0]:
            best = (rate, f"{n} calls of {sample}x{shape[1]}x{shape[2]}x{shape[3]} ({args.size}): {desc}")
    return {"value": round(best[0], 3), "unit": unit, "cores": threads, "kind": "port", "sample": best[1],
            "rates": rates}


def run_reference(args):
    """--impl reference: the reference's CPU algorithm (the oracle port; the Rust crate cannot be built here)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if args.kind == "e2e":
        tmp = tempfile.mkdtemp(prefix="ppocr_e2e_ref_")
        cpu = cpu_baseline_e2e(tmp, seconds=20.0)
        line = {"impl": "reference", "metric": "e2e pages/s @1920x1080 (tiny det + DB postprocess + tiny rec + CTC)",
                "value": cpu["value"], "unit": "pages/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(1000.0 / cpu["value"], 3) if cpu["value"] else None, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": "config 5 pages through the CPU restatement of the reference pipeline"},
                "cpu_baseline": cpu,
                "e2e": {"value": cpu["value"], "unit": "pages/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    shape, name, unit, metric = _workload(args)
    # The faster CPU restatement (a short probe of each), then K timed steps of it.
    forms, threads = _cpu_forms(args, shape)
    best = None
    for form in forms:
        name_f, fwd, sample_f, desc = form
        x = _inputs(args.kind, (sample_f,) + tuple(shape[1:]), seed=99)
        n, dt = _time_form(fwd, x, 3.0)
        if best is None or n * sample_f / dt > best[0]:
            best = (n * sample_f / dt, form, x)
    _, (form_name, fwd, sample, desc), x = best
    for _ in range(max(args.warmup, 1)):
        fwd(x)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        fwd(x)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = sample * args.steps / total
    line = {
        "impl": "reference", "metric": metric, "value": round(value, 3), "unit": unit, "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 * total / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": name, "sample_per_step": sample},
        "cpu_baseline": {"value": round(value, 3), "unit": unit, "cores": threads, "kind": "port",
                         "sample": f"{sample} of the {shape[0]} inputs per step: {desc} (the faster CPU restatement; "
                                   f"ppocr-cpu-bench needs a Rust toolchain, absent here)"},
        "e2e": {"value": round(value, 3), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


E2E_SIZE = (1080, 1920)


def _e2e_pages(count, rank, world):
    """Config 5 pages for this rank (page ids dealt round-robin): 30-80 dark stroke blocks,
    height 16-40, width 40-600, +-15 degrees, on a light noisy background."""
    from ppocr_b200 import seeded, sharding

    ids = sharding.round_robin(count * world, world, rank)
    return [seeded.text_page_rgb8(E2E_SIZE[0], E2E_SIZE[1], seed=5000 + i, blocks=(30, 80), block_h=(16, 40),
                                  block_w=(40, 600), max_angle=15.0, background=(180, 250)) for i in ids]


def _e2e_models(tmp):
    from ppocr_b200 import seeded

    det = seeded.write_weights(os.path.join(tmp, "e2e_det_tiny.safetensors"), "det", "tiny", 0, "spec")
    rec = seeded.write_weights(os.path.join(tmp, "e2e_rec_tiny.safetensors"), "rec", "tiny", 0, "spec")
    d = os.path.join(tmp, "e2e_dict.txt")
    with open(d, "w", encoding="utf-8") as f:
        f.write("\n".join(seeded.synthetic_dictionary("tiny")) + "\n")
    return det, rec, d


def measure_e2e(gpu, pages_per_rank, steps, warmup, world, rank, barrier, tmp, rec_precision=None):
    """Pages/s of the OCR engine's batch call over this rank's pages (max over ranks of the wall time).
    rec_precision: None runs both models in FP32 (the reference's arithmetic); "bf16" runs the
    recognizer on the tcgen05 BF16 path."""
    import ppocr_b200 as P
    from ppocr_b200 import sharding

    det, rec, d = _e2e_models(tmp)
    pages = _e2e_pages(pages_per_rank, rank, world)
    eng = P.Engine(gpu, det, rec, d, recognizer_precision=rec_precision)
    for _ in range(max(1, warmup)):
        res = eng.recognize_batch(pages)
    lines = sum(len(r["lines"]) for r in res)
    barrier()
    t0 = time.perf_counter()
    step_ms = []
    for _ in range(steps):
        ts = time.perf_counter()
        eng.recognize_batch(pages)
        step_ms.append(round(1000 * (time.perf_counter() - ts), 2))
    dt = sharding.max_over_ranks(time.perf_counter() - t0)
    stages = eng.stage_times()
    eng.close()
    value = pages_per_rank * world * steps / dt
    name = "e2e pages/s @1920x1080 (tiny det + DB postprocess + tiny rec + CTC)"
    if rec_precision:
        name += f", recognizer {rec_precision}"
    return {"metric": name, "value": round(value, 2), "last_call_stage_ms": {k: round(v, 2) for k, v in stages.items()},
            "unit": "pages/s", "ms_per_page": round(1000 * dt / (pages_per_rank * steps), 3),
            "pages_per_step_per_gpu": pages_per_rank, "steps": steps, "step_ms": step_ms,
            "lines_per_page": round(lines / len(pages), 1),
            "api": "ppocr_engine_recognize_batch (host RGB8 pages in, JSON out)",
            "h2d_bytes_per_step": int(sum(p.size for p in pages)),
            "data": "synthetic config-5 pages, seeded random-init (spec) weights"}


def cpu_baseline_e2e(tmp, seconds=12.0):
    """The oracle pipeline (torch-CPU detector + restated DB postprocess + recognizer + CTC) on pages."""
    import torch

    from oracle import model as om
    from oracle import pipeline as opl
    from oracle import postprocess as opost
    from oracle import preprocess as opre
    from ppocr_b200 import seeded

    torch.set_num_threads(os.cpu_count() or 1)
    det, rec, _ = _e2e_models(tmp)
    odet, orec = om.load_detector(det, "tiny"), om.load_recognizer(rec, "tiny")
    words = seeded.synthetic_dictionary("tiny")
    pages = _e2e_pages(2, 0, 1)
    n, t0 = 0, time.perf_counter()
    for page in pages:
        h, w = page.shape[:2]
        iw, ih = opre.detector_input_size(w, h, 736)
        prob = odet.forward(opre.prepare_detector(page, iw, ih))[0, 0]
        dets = opl.extract_detections(prob, ih, iw, (w, h), (iw, ih))
        for idx, width, contents in opl.recognition_batches(dets):
            x = np.concatenate([opre.prepare_recognizer_crop(page, dets[i].polygon, width, c)
                                for i, c in zip(idx, contents)])
            probs = orec.forward(x)
            for k, c in enumerate(contents):
                opost.decode_ctc_greedy(probs[k], words, c, width)
        n += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": round(n / dt, 4), "unit": "pages/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{n} config-5 pages through the torch-CPU oracle pipeline"}


def family_roofline(model, precision, families=None):
    """The dominant kernel family of a model's plan (per-op CUDA events, 3 runs)
    against its roof: FLOP/s vs the BF16 tensor peak for the BF16 tcgen05 GEMMs,
    algorithmic bytes/s vs HBM for everything else (the FP32 split GEMMs are
    HBM-bound: three BF16 pieces per operand, six products, tensor pipe
    ~5-10 %).  Returns (roofline dict, per-family table, ops, per-op ms)."""
    ops = model.ops()
    prof = model.profile(runs=3)
    fam = {}
    for op, ms in zip(ops, prof):
        f = fam.setdefault(op["kind"], {"ms": 0.0, "bytes": 0.0, "flops": 0.0, "launches": 0})
        f["ms"] += ms
        f["bytes"] += op["bytes"]
        f["flops"] += op["flops"]
        f["launches"] += 1
    dom_kind = max(fam, key=lambda k: fam[k]["ms"]) if families is None else families
    dom = fam[dom_kind]
    hbm, tflops, peak_src = _peaks()
    launches = dom["launches"]
    per_launch_s = dom["ms"] / launches / 1000.0
    if dom_kind == "gemm" and precision == "bf16":
        achieved = dom["flops"] / launches / per_launch_s / 1e12
        roof = {"bound": "tensor", "achieved": round(achieved, 2), "peak": tflops, "unit": "TFLOP/s",
                "frac": round(achieved / tflops, 4)}
        # Each GEMM against the roof that bounds it: at an arithmetic intensity
        # (algorithmic FLOPs per algorithmic byte) above the ridge point
        # (tensor peak / HBM bandwidth) the tensor pipe, below it HBM.
        ridge = tflops * 1e12 / (hbm * 1e9)
        groups = {"tensor": [0.0, 0.0, 0], "hbm": [0.0, 0.0, 0]}   # work, seconds, launches
        for op, ms in zip(ops, prof):
            if op["kind"] != "gemm" or ms <= 0:
                continue
            bound = "tensor" if op["flops"] / max(op["bytes"], 1.0) >= ridge else "hbm"
            g = groups[bound]
            g[0] += op["flops"] if bound == "tensor" else op["bytes"]
            g[1] += ms / 1000.0
            g[2] += 1
        per = {}
        for bound, (work, secs, n) in groups.items():
            if n == 0:
                continue
            rate = work / secs / (1e12 if bound == "tensor" else 1e9)
            peak = tflops if bound == "tensor" else hbm
            per[bound] = {"launches": n, "achieved": round(rate, 2), "peak": peak,
                          "unit": "TFLOP/s" if bound == "tensor" else "GB/s", "frac": round(rate / peak, 4),
                          "ms": round(secs * 1000.0, 4)}
        roof["per_roof"] = per
        roof["ridge_flops_per_byte"] = round(ridge, 1)
    else:
        achieved = dom["bytes"] / launches / per_launch_s / 1e9
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(achieved / hbm, 4)}
        if dom_kind == "gemm" and precision == "fp32":
            # Tensor-pipe view of the split GEMMs: six BF16 products per FP32 MAC.
            bf16_tf = 6 * dom["flops"] / launches / per_launch_s / 1e12
            roof["tensor_view"] = {"achieved": round(bf16_tf, 2), "peak": tflops, "unit": "TFLOP/s (BF16, six products)",
                                   "frac": round(bf16_tf / tflops, 4)}
    roof.update({"kernel": dom_kind, "launches_per_step": launches, "time_share": round(dom["ms"] / sum(prof), 4),
                 "peak_source": peak_src, "algorithmic_bytes_per_launch": round(dom["bytes"] / launches),
                 "algorithmic_flops_per_launch": round(dom["flops"] / launches)})
    table = {k: {"ms": round(v["ms"], 4), "launches": v["launches"],
                 "GBps": round(v["bytes"] / (v["ms"] / 1000.0) / 1e9, 1),
                 "TFLOPs": round(v["flops"] / (v["ms"] / 1000.0) / 1e12, 2)} for k, v in fam.items()}
    return roof, table, ops, prof


def _timed(models_inputs, steps, warmup, barrier):
    """Device time (ms, summed over `steps`) of one step = one graph replay of
    every model in order, each on its resident input slot, with a 256 MiB L2
    flush before each step; CUDA events on the launching stream."""
    import torch

    stream = torch.cuda.Stream()
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    for _ in range(warmup):
        for m in models_inputs:
            m.run(stream.cuda_stream)
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    barrier()
    with torch.cuda.stream(stream):
        for i in range(steps):
            flush.fill_(i & 0xFF)
            starts[i].record(stream)
            for m in models_inputs:
                m.run(stream.cuda_stream)
            ends[i].record(stream)
    torch.cuda.synchronize()
    del flush
    return sum(s.elapsed_time(e) for s, e in zip(starts, ends))


def _load_resident(P, gpu, path, kind, size, shape, precision, x, shared=None):
    import torch

    M = P.Detector if kind == "det" else P.Recognizer
    model = M.load(gpu, path, size, shape, precision=precision) if kind == "det" else \
        M.load(gpu, path, size, shape, precision=precision, shared_weights=shared)
    din, _ = model.device_buffers()
    _device_view(din, x.size, torch).copy_(torch.from_numpy(np.ascontiguousarray(x).reshape(-1)))
    return model


def _cpu_rate(kind, size, shape, seconds=3.0):
    """The faster CPU restatement (torch port, C++ for tiny / small detectors)
    on a small sample of this configuration, all host threads."""
    class A:
        pass

    a = A()
    a.kind, a.size = kind, size
    forms, threads = _cpu_forms(a, shape)
    best = None
    for name, fwd, sample, desc in forms:
        x = _inputs(kind, (sample,) + tuple(shape[1:]), seed=99)
        n, dt = _time_form(fwd, x, seconds / len(forms))
        rate = n * sample / dt
        if best is None or rate > best["value"]:
            best = {"value": round(rate, 3), "unit": "img/s" if kind == "det" else "crops/s", "cores": threads,
                    "kind": "port", "sample": f"{n} calls of {sample}x{shape[1]}x{shape[2]}x{shape[3]}: {desc}"}
    return best


def measure_config(gpu, world, rank, barrier, tmp, kind, size, batch, precision, text, steps=10, warmup=3, cpu=False):
    """Configs 3 (small / medium detector, batch 32 per GPU, text-like pages)
    and the like: device throughput with inputs resident (max over ranks), the
    dominant family's roofline, and (rank 0 of a 1-GPU run) the CPU rate."""
    import ppocr_b200 as P
    from ppocr_b200 import seeded, sharding

    path = os.path.join(tmp, f"{kind}_{size}.safetensors")
    if not os.path.exists(path):
        seeded.write_weights(path, kind, size, 0, "spec")
    shape = (batch, 3, 416, 736) if kind == "det" else (batch, 3, 48, 320)
    x = seeded.det_batch(batch, 416, 736, seed=3000 + rank, text=text) if kind == "det" else \
        seeded.rec_batch(batch, 320, seed=3000 + rank)
    model = _load_resident(P, gpu, path, kind, size, shape, precision, x)
    total = sharding.max_over_ranks(_timed([model], steps, warmup, barrier))
    roof, table, _, _ = family_roofline(model, precision)
    model.close()
    unit = "img/s" if kind == "det" else "crops/s"
    out = {"metric": f"{kind} {unit} @{shape[2]}x{shape[3]} ({size}, batch {batch}/GPU{', text-like pages' if text else ''})",
           "value": round(batch * world * steps / (total / 1000.0), 2), "unit": unit,
           "ms_per_step": round(total / steps, 4), "dtype": "f32" if precision == "fp32" else "bf16",
           "roofline": roof, "families": table}
    if cpu and rank == 0 and world == 1:
        out["cpu_baseline"] = _cpu_rate(kind, size, shape)
    return out


def measure_latency_b1(gpu, tmp, kind, size, precision, warmup=5, runs=30, cpu=False):
    """Configs 1 / 2 as the reference's bench reports them (src/bin/benchmark.rs:
    303-320): batch 1, `warmup` untimed and `runs` timed forwards on the resident
    input (Detector::benchmark), average / p50 / p90 / p95 in ms."""
    import ppocr_b200 as P
    from ppocr_b200 import seeded

    path = os.path.join(tmp, f"{kind}_{size}.safetensors")
    if not os.path.exists(path):
        seeded.write_weights(path, kind, size, 0, "spec")
    shape = (1, 3, 416, 736) if kind == "det" else (1, 3, 48, 320)
    x = seeded.det_batch(1, 416, 736, seed=1) if kind == "det" else seeded.rec_batch(1, 320, seed=1)
    M = P.Detector if kind == "det" else P.Recognizer
    model = M.load(gpu, path, size, shape, precision=precision)
    samples = sorted(1000.0 * t for t in model.benchmark(x, warmup, runs))   # seconds -> ms
    roof, _, _, _ = family_roofline(model, precision)
    model.close()
    pct = lambda q: samples[int(round((len(samples) - 1) * q))]
    avg = sum(samples) / len(samples)
    out = {"metric": f"{kind} latency @{shape[2]}x{shape[3]} ({size}, batch 1)", "average_ms": round(avg, 4),
           "p50_ms": round(pct(0.5), 4), "p90_ms": round(pct(0.9), 4), "p95_ms": round(pct(0.95), 4),
           "throughput": round(1000.0 / avg, 2), "unit": "img/s" if kind == "det" else "crops/s", "runs": runs,
           "warmup": warmup, "dtype": "f32" if precision == "fp32" else "bf16", "roofline": roof}
    if cpu:
        out["cpu_baseline"] = _cpu_rate(kind, size, shape)
    return out


def measure_config4(gpu, world, rank, barrier, tmp, crops=4096, batch=256, steps=3, warmup=2, cpu=False):
    """Config 4: 4096 crops per GPU, widths drawn uniformly from {160, 320, 480},
    bucketed by width into batches of 256, medium recognizer in BF16.  One step
    runs every batch of the rank's crops (one graph replay each, inputs
    resident); value = crops of all ranks / (max over ranks of the step time)."""
    import ppocr_b200 as P
    from ppocr_b200 import seeded, sharding

    path = os.path.join(tmp, "rec_medium.safetensors")
    if not os.path.exists(path):
        seeded.write_weights(path, "rec", "medium", 0, "spec")
    rng = np.random.default_rng(4000 + rank)
    widths = rng.choice([160, 320, 480], size=crops)
    runs, models, shared = [], [], None
    counts = {}
    for wdt in (160, 320, 480):
        count = int((widths == wdt).sum())
        counts[wdt] = count
        if count == 0:
            continue
        x = seeded.rec_batch(batch, wdt, seed=5000 + rank + wdt)
        m = _load_resident(P, gpu, path, "rec", "medium", (batch, 3, 48, wdt), "bf16", x, shared)
        shared = shared or m
        models.append(m)
        runs += [m] * ((count + batch - 1) // batch)
    total = sharding.max_over_ranks(_timed(runs, steps, warmup, barrier))
    roof, table, _, _ = family_roofline(models[len(models) // 2], "bf16")
    for m in models:
        m.close()
    out = {"metric": "rec crops/s (medium, 4096 crops/GPU, widths {160,320,480} bucketed into batches of 256)",
           "value": round(crops * world * steps / (total / 1000.0), 2), "unit": "crops/s",
           "ms_per_step": round(total / steps, 3), "batches_per_step": len(runs), "crops_per_width": counts,
           "dtype": "bf16", "roofline_w320": roof, "families_w320": table}
    if cpu and rank == 0 and world == 1:
        out["cpu_baseline"] = _cpu_rate("rec", "medium", (batch, 3, 48, 320))
    return out


def measure_rec(gpu, world, barrier, tmp, steps=10, warmup=3, batch=256):
    """Medium recognizer BF16 at width 320, batch 256: crops/s device-timed (max
    over ranks), the tcgen05 GEMM family against the BF16 tensor peak."""
    import ppocr_b200 as P
    from ppocr_b200 import seeded, sharding

    path = os.path.join(tmp, "rec_medium.safetensors")
    if not os.path.exists(path):
        seeded.write_weights(path, "rec", "medium", 0, "spec")
    shape = (batch, 3, 48, 320)
    x = seeded.rec_batch(batch, 320, seed=2000 + int(os.environ.get("RANK", "0")))
    model = _load_resident(P, gpu, path, "rec", "medium", shape, "bf16", x)
    total = sharding.max_over_ranks(_timed([model], steps, warmup, barrier))
    roof, table, _, _ = family_roofline(model, "bf16", families="gemm")
    # End to end from pinned host crops to host CTC classes and probabilities:
    # one ppocr_recognizer_forward_pipelined_ctc call over e_steps batches.
    import ctypes as C

    import torch

    e_steps = 5
    rows = batch * model.output_shape[1]
    hin = torch.from_numpy(np.tile(x.reshape(-1), e_steps)).pin_memory()
    hidx = torch.empty(rows * e_steps, dtype=torch.int32).pin_memory()
    hprob = torch.empty(rows * e_steps, dtype=torch.float32).pin_memory()
    lib = P.library()
    args = (model._h, C.cast(C.c_void_p(hin.data_ptr()), C.POINTER(C.c_float)), batch * e_steps,
            C.cast(C.c_void_p(hidx.data_ptr()), C.POINTER(C.c_int32)),
            C.cast(C.c_void_p(hprob.data_ptr()), C.POINTER(C.c_float)), rows * e_steps)
    for _ in range(2):
        P._check(lib.ppocr_recognizer_forward_pipelined_ctc(*args))
    barrier()
    t0 = time.perf_counter()
    P._check(lib.ppocr_recognizer_forward_pipelined_ctc(*args))
    et = sharding.max_over_ranks(time.perf_counter() - t0)
    model.close()
    return {"metric": "rec crops/s @48x320 (medium recognizer, batch 256/GPU)",
            "value": round(batch * world * steps / (total / 1000.0), 2), "unit": "crops/s",
            "ms_per_step": round(total / steps, 4), "dtype": "bf16", "gemm_roofline": roof, "families": table,
            "e2e": {"value": round(batch * e_steps * world / et, 2), "unit": "crops/s",
                    "h2d_bytes_per_step": int(x.size * 4), "d2h_bytes_per_step": int(rows * 8), "steps": e_steps,
                    "api": "ppocr_recognizer_forward_pipelined_ctc (pinned host crops in, CTC class + probability out)"}}


def run_e2e(args):
    import torch
    import torch.distributed as dist

    import ppocr_b200 as P

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    tmp = tempfile.mkdtemp(prefix=f"ppocr_e2e_{rank}_")
    gpu = P.Gpu(local)
    with _Clocks(local) as clocks:
        r = measure_e2e(gpu, args.batch, args.steps, args.warmup, world, rank, barrier, tmp)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_e2e(tmp)
    if rank == 0:
        line = {"metric": r["metric"], "value": r["value"], "unit": "pages/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(r["ms_per_page"] * args.batch, 3), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": r["data"],
                "config": {"workload": "config 5: 1920x1080 pages -> tiny det -> DB -> rectify -> tiny rec -> CTC",
                           "pages_per_step_per_gpu": args.batch, "parallelism": f"dp{world} (pages sharded, no collective)",
                           "lines_per_page": r["lines_per_page"]},
                "roofline": None, "cpu_baseline": cpu,
                "e2e": {"value": r["value"], "unit": "pages/s", "h2d_bytes_per_step": r["h2d_bytes_per_step"],
                        "d2h_bytes_per_step": None, "api": r["api"]},
                "clocks": clocks.summary()}
        print(json.dumps(line), flush=True)
    gpu.close()
    if world > 1:
        dist.destroy_process_group()


def run_b200(args):
    import torch
    import torch.distributed as dist

    import ppocr_b200 as P
    from ppocr_b200 import seeded, sharding

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    shape, name, unit, metric = _workload(args)
    precision = args.precision or ("fp32" if args.kind == "det" else "bf16")
    tmp = tempfile.mkdtemp(prefix=f"ppocr_bench_{rank}_")
    wpath = os.path.join(tmp, f"{args.kind}_{args.size}.safetensors")
    seeded.write_weights(wpath, args.kind, args.size, 0, "spec")
    gpu = P.Gpu(local)
    Model = P.Detector if args.kind == "det" else P.Recognizer
    model = Model.load(gpu, wpath, args.size, shape, precision=precision)
    x = _inputs(args.kind, shape, seed=1000 + rank)
    # A dedicated (non-default) stream: the forward, the L2 flush and the
    # timing events all go to it, so the events bracket exactly the forward.
    stream = torch.cuda.Stream()
    sptr = stream.cuda_stream
    din, dout = model.device_buffers()
    _device_view(din, x.size, torch).copy_(torch.from_numpy(x.reshape(-1)))
    torch.cuda.synchronize()

    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    for _ in range(args.warmup):
        model.run(sptr)
    torch.cuda.synchronize()

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with _Clocks(local) as clocks:
        barrier()
        torch.cuda.synchronize()
        w0 = time.perf_counter()
        with torch.cuda.stream(stream):
            for i in range(args.steps):
                flush.fill_(i & 0xFF)
                starts[i].record(stream)
                model.run(sptr)
                ends[i].record(stream)
        torch.cuda.synchronize()
        barrier()
        wall = time.perf_counter() - w0
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = sharding.max_over_ranks(sum(step_ms))
    units = shape[0] * world * args.steps
    value = units / (total_ms / 1000.0)

    # Output sanity: the device forward produced finite values.
    out = _device_view(dout, model.output_elements, torch)
    finite = bool(torch.isfinite(out).all().item())

    # Per-kernel timing (events around every op) for the roofline.
    roof, table, ops, prof = family_roofline(model, precision)
    dom_kind = roof["kernel"]
    top = sorted(zip(ops, prof), key=lambda t: -t[1])[:8]
    roof["top_ops"] = [{"op": o["name"], "kind": o["kind"], "ms": round(ms, 4),
                        "GBps": round(o["bytes"] / (ms / 1000.0) / 1e9, 1),
                        "TFLOPs": round(o["flops"] / (ms / 1000.0) / 1e12, 2)} for o, ms in top]
    roof["families"] = table
    roof["traffic"] = None
    traffic_path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(traffic_path):
        try:
            with open(traffic_path) as f:
                t = json.load(f).get(f"{args.kind}_{args.size}_{precision}", {}).get(dom_kind)
            if t is not None:
                roof["traffic"] = t
        except Exception:
            pass

    # End to end through the C ABI with pinned host buffers: one pipelined call
    # over e_steps batches (a distinct host copy of the input per batch), which
    # uploads batch i + 1 and downloads batch i - 1 while batch i runs; every
    # batch's host-to-device and device-to-host copies are inside the timed
    # region.  The detector downloads its probability maps
    # (ppocr_model_forward_pipelined); the recognizer only the greedy-CTC class
    # and probability per step (ppocr_recognizer_forward_pipelined_ctc), which is
    # all the reference's decoder reads (src/ocr.rs:800-853).
    e2e = None
    if not args.no_e2e:
        import ctypes as C

        # As many batches as timed steps: the pipeline's first upload and last
        # download (which nothing overlaps) spread over the whole run.
        e_steps = max(3, args.steps) if args.kind == "det" else 5
        images = shape[0] * e_steps
        hin = torch.from_numpy(np.tile(x.reshape(-1), e_steps)).pin_memory()
        fin = C.cast(C.c_void_p(hin.data_ptr()), C.POINTER(C.c_float))
        lib = P.library()
        if args.kind == "det":
            per_out = model.output_elements
            hout = [torch.empty(per_out * e_steps, dtype=torch.float32).pin_memory()]
            fout = C.cast(C.c_void_p(hout[0].data_ptr()), C.POINTER(C.c_float))
            d2h = per_out * 4

            def call():
                P._check(lib.ppocr_model_forward_pipelined(model._h, fin, images, fout, per_out * e_steps))
            api = f"ppocr_model_forward_pipelined (one call over {e_steps} batches of {shape[0]}, pinned host buffers)"
        else:
            rows = shape[0] * model.output_shape[1]
            hout = [torch.empty(rows * e_steps, dtype=torch.int32).pin_memory(),
                    torch.empty(rows * e_steps, dtype=torch.float32).pin_memory()]
            iout = C.cast(C.c_void_p(hout[0].data_ptr()), C.POINTER(C.c_int32))
            pout = C.cast(C.c_void_p(hout[1].data_ptr()), C.POINTER(C.c_float))
            d2h = rows * 8

            def call():
                P._check(lib.ppocr_recognizer_forward_pipelined_ctc(model._h, fin, images, iout, pout, rows * e_steps))
            api = (f"ppocr_recognizer_forward_pipelined_ctc (one call over {e_steps} batches of {shape[0]}, "
                   "pinned host buffers, CTC class + probability per step downloaded)")
        for _ in range(2):
            call()
        barrier()
        t0 = time.perf_counter()
        call()
        et = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(et, op=dist.ReduceOp.MAX)
        e2e = {"value": round(images * world / float(et.item()), 2), "unit": unit,
               "h2d_bytes_per_step": int(x.size * 4), "d2h_bytes_per_step": int(d2h),
               "steps": e_steps, "api": api}
        del hin, hout

    # The secondary figures run before the CPU baseline, whose torch thread pool
    # would otherwise compete with the engine's host threads.
    secondary = None
    if args.kind == "det" and not args.no_secondary:
        model.close()
        cpu_ok = not args.no_cpu_baseline
        secondary = {"rec": measure_rec(gpu, world, barrier, tmp),
                     "config4_rec": measure_config4(gpu, world, rank, barrier, tmp, cpu=cpu_ok),
                     "config3_small_det": measure_config(gpu, world, rank, barrier, tmp, "det", "small", 32, "fp32", True,
                                                         cpu=cpu_ok),
                     "config3_medium_det": measure_config(gpu, world, rank, barrier, tmp, "det", "medium", 32, "fp32", True,
                                                          steps=5, cpu=cpu_ok),
                     "e2e_pages": measure_e2e(gpu, 8, 10, 2, world, rank, barrier, tmp),
                     "e2e_pages_rec_bf16": measure_e2e(gpu, 8, 10, 2, world, rank, barrier, tmp, rec_precision="bf16")}
        if rank == 0:
            secondary["config1_det_b1"] = measure_latency_b1(gpu, tmp, "det", "tiny", "fp32")
            secondary["config2_rec_b1"] = measure_latency_b1(gpu, tmp, "rec", "tiny", "fp32", cpu=cpu_ok and world == 1)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args, shape)

    launches_per_step = sum(1 for op in ops)
    if rank == 0:
        line = {
            "metric": metric, "value": round(value, 2), "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32" if precision == "fp32" else "bf16",
            "data": "synthetic (seeded uniform RGB8 inputs, seeded random-init weights in the reference layout)",
            "config": {"workload": name, "batch_per_gpu": shape[0], "precision": precision,
                       "parallelism": f"dp{world} (images sharded, no collective)",
                       "l2": "256 MiB flush between timed steps", "cuda_graph": True},
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks.summary(), "wall_s": round(wall, 3), "output_finite": finite,
            "step_ms_min_max": [round(min(step_ms), 4), round(max(step_ms), 4)],
            "secondary": secondary,
        }
        print(json.dumps(line), flush=True)
    model.close()
    gpu.close()
    if world > 1:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--kind", default="det", choices=["det", "rec", "e2e"])
    ap.add_argument("--size", default="tiny", choices=["tiny", "small", "medium"])
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--precision", default=None, choices=[None, "fp32", "bf16", "fp32tc"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.batch is None:
        args.batch = {"det": 32, "rec": 256, "e2e": 16}[args.kind]
    if args.impl == "reference":
        run_reference(args)
    elif args.kind == "e2e":
        run_e2e(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
