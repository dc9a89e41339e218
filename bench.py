#!/usr/bin/env python
"""Benchmark of the unoq-dsp INT8 CNN execution path on B200.

Headline (BASELINE.json metric, config 4): MobileNetV4-Conv-Small-224 INT8 images/sec over a
global batch (default 4096) batch-sharded across N GPUs, one process per GPU, each GPU
replaying one CUDA graph of the whole network; YOLO26n-320 (global batch 1024) is reported in
the same line under "yolo26n_320". Weights are the bundled .uqmodel plans (staged into models/
by __graft_entry__.build()); inputs are seeded uniform int8 images (synthetic, no dataset).

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]

value  -- images/sec with inputs already in HBM: W untimed steps, then exactly K steps between
          a barrier + device sync on both sides, CUDA-event timed, max over ranks.
e2e    -- the same images/sec through the public batch call ug_infer_batch with pinned host
          buffers: per step the input H2D copy, the graph and the output D2H copy.
detect_e2e (YOLO) -- the detector's path through ug_detect_batch: uint8 pixels H2D, the byte
          table, the network and the top-k decode on the GPU, 20 records per image D2H.
--impl reference -- the reference's own C runtime (oracle/_ref/libug_ref.so, built from the
          reference sources) on all host cores; rank 0 only.
"""
import argparse
import ctypes as C
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT / "unoq-dsp_b200"), str(ROOT)]

METRIC = "INT8 images/sec (MobileNetV4-S 224, YOLO26n 320) at 1/2/4/8 B200; % INT8/HBM roofline"
MODELS = {
    "mobilenetv4-small": {"shape": (1, 224, 224, 3), "batch": 4096, "key": "mobilenetv4_small_224"},
    "yolo26n-320": {"shape": (1, 320, 320, 3), "batch": 1024, "key": "yolo26n_320"},
}
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


# --------------------------------------------------------------------------- reference CPU
_REF = {}


def _ref_init(plan_path):
    """Pool initializer: each worker process loads the reference runtime and the plan once."""
    sys.path[:0] = [str(ROOT), str(ROOT / "unoq-dsp_b200")]
    from oracle.oracle import Reference
    from unoq_dsp.bundle import load
    plan = load(plan_path).plan
    ref = Reference()
    if ref.load(plan):
        raise RuntimeError("reference ug_load failed")
    _REF.update(ref=ref, plan=plan)


def _ref_worker(args):
    shape, images, seed = args
    ref, plan = _REF["ref"], _REF["plan"]
    x = np.random.default_rng(seed).integers(-128, 128, size=shape, dtype=np.int64).astype(np.int8)
    t0 = time.perf_counter()
    for _ in range(images):
        ref.run(plan, x)
    return time.perf_counter() - t0


def reference_throughput(shape, images_per_proc, procs, pool):
    """Images/sec of the reference runtime (single-threaded C off Hexagon): `procs` worker
    processes, each running `images_per_proc` whole images of the already-loaded plan."""
    jobs = [(shape, images_per_proc, 1000 + i) for i in range(procs)]
    t0 = time.perf_counter()
    times = pool.map(_ref_worker, jobs, chunksize=1)
    wall = time.perf_counter() - t0
    return procs * images_per_proc / wall, wall, max(times)


def make_pool(procs, plan_path):
    import multiprocessing as mp
    return mp.get_context("spawn").Pool(procs, initializer=_ref_init, initargs=(str(plan_path),))


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock and clock-event reasons polled through NVML (read-only queries) every few
    milliseconds while the timed region runs."""
    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"),
               ("hw_power_brake", "nvmlClocksEventReasonHwPowerBrakeSlowdown"))

    def __init__(self, device, period=0.005):
        self.device, self.period = device, period
        self.rows, self.max_mhz, self.nvml = [], None, None
        self.stop = threading.Event()

    def __enter__(self):
        try:
            import pynvml as N
            N.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            index = int(vis.split(",")[self.device]) if vis and vis.split(",")[0].isdigit() else self.device
            self.handle = N.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(self.handle, N.NVML_CLOCK_SM)
            self.nvml = N
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
        except Exception:  # no NVML: the line says "unsampled"
            self.nvml = None
        return self

    def _poll(self):
        N = self.nvml
        while not self.stop.is_set():
            try:
                self.rows.append((N.nvmlDeviceGetClockInfo(self.handle, N.NVML_CLOCK_SM),
                                  N.nvmlDeviceGetCurrentClocksEventReasons(self.handle)))
            except Exception:
                pass
            time.sleep(self.period)

    def __exit__(self, *a):
        self.stop.set()
        if self.nvml:
            self.thread.join(timeout=5)
            self.nvml.nvmlShutdown()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"]}
        N = self.nvml or __import__("pynvml")
        reasons = {name for name, attr in self.REASONS for _, bits in self.rows
                   if getattr(N, attr, 0) and bits & getattr(N, attr)}
        return {"sm_mhz": statistics.median(r[0] for r in self.rows), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(self.rows), "source": "NVML, 5 ms polling"}


# --------------------------------------------------------------------------- distributed
class Dist:
    def __init__(self, gpus):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
            self.dist = dist
            self.pg = True

    def barrier(self):
        if self.pg:
            self.dist.barrier()

    def max(self, value):
        if not self.pg:
            return value
        import torch
        t = torch.tensor([float(value)], dtype=torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def sum(self, value):
        if not self.pg:
            return value
        import torch
        t = torch.tensor([float(value)], dtype=torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM)
        return float(t.item())

    def broadcast_bytes(self, data, size):
        """Rank 0's `data` (bytes of length `size`) on every rank, over the gloo group."""
        if not self.pg:
            return data
        obj = [data if self.rank == 0 else None]
        self.dist.broadcast_object_list(obj, src=0)
        if len(obj[0]) != size:
            raise RuntimeError("bad broadcast")
        return obj[0]

    def gather_object(self, obj):
        """Every rank's `obj` as a list on rank 0 (None elsewhere), over the gloo group."""
        if not self.pg:
            return [obj]
        out = [None] * self.world if self.rank == 0 else None
        self.dist.gather_object(obj, out, dst=0)
        return out

    def close(self):
        if self.pg:
            self.dist.destroy_process_group()


def shard(global_batch, world, rank):
    """Contiguous slice [start, start + count) of the global batch for `rank` (equal slices;
    the global batch must divide evenly so every rank replays the same graph)."""
    if global_batch % world:
        raise ValueError(f"global batch {global_batch} does not divide over {world} GPUs")
    per = global_batch // world
    return rank * per, per


def image_input(index, ni):
    """Seeded synthetic image `index` of the global batch (uniform int8). Each image has its own
    random stream, so the output check can regenerate any sample without the rest of the batch."""
    return np.random.default_rng([1234, index]).integers(-128, 128, size=ni, dtype=np.int8)


def sample_rows(per_gpu):
    """Local image indices checked on every rank: the first, middle and last of its shard."""
    return sorted({0, per_gpu // 2, per_gpu - 1})


def verify_outputs(plan, ni, samples, dist):
    """Rank 0: compare sampled output rows with the reference runtime's outputs for the same seeded
    images (oracle/_ref/libug_ref.so in a spawn pool; outside every timed region). `samples` maps
    a path name to {global image index: output bytes}. Returns the line's "verify" entry."""
    from oracle.refpool import checker_kind, reference_outputs
    index = sorted({g for rows in samples.values() for g in rows})
    expect = dict(zip(index, reference_outputs(plan, [image_input(g, ni) for g in index])))
    mismatch = {path: [g for g, row in rows.items() if row != expect[g].tobytes()] for path, rows in samples.items()}
    return {"images": len(index), "mismatch": sum(len(v) for v in mismatch.values()),
            "checked": {path: len(rows) for path, rows in samples.items()},
            "mismatched_images": {p: v[:8] for p, v in mismatch.items() if v}, "checker": checker_kind(),
            "ranks": dist.world}


def join_gather(lib, handle, dist):
    """Multi-GPU: rank 0 makes the NCCL id, every rank receives it and joins the output gather."""
    if dist.world == 1:
        return
    idbuf = C.create_string_buffer(128)
    if dist.rank == 0 and lib.ug_dist_unique_id(idbuf, 128):
        raise RuntimeError(f"ug_dist_unique_id: {lib.ug_last_error()}")
    data = dist.broadcast_bytes(idbuf.raw if dist.rank == 0 else None, 128)
    idbuf = C.create_string_buffer(data, 128)
    rc = lib.ug_dist_init(handle, dist.rank, dist.world, idbuf, 128)
    if rc:
        raise RuntimeError(f"ug_dist_init rc={rc}: {lib.ug_last_error()}")


# --------------------------------------------------------------------------- roofline
def op_traffic(plan, images):
    """Algorithmic bytes and int8 ops per plan op for `images` images: every activation input
    read once, the output written once, constants (weights, tables) read once per launch."""
    import struct
    magic, version, nt, no, arena, inp, out, flags = struct.unpack_from("<8I", plan)
    ts = [struct.unpack_from("<12I", plan, 32 + 48 * i) for i in range(nt)]
    ops = [struct.unpack_from("<8I", plan, 32 + 48 * nt + 32 * i) for i in range(no)]
    meta = 32 + 48 * nt + 32 * no
    rows = []
    for o in ops:
        code, a, b, z = o[:4]
        abytes, bbytes, zbytes = ts[a][1], ts[b][1], ts[z][1]
        const_b = ts[b][8]
        byt = (abytes + zbytes) * images
        mac = 0
        if code in (14, 15):
            q = [int(v) for v in np.frombuffer(plan, dtype="<i4", count=20, offset=meta + ts[o[4]][0])]
            kh, kw, oh, ow, ic, oc = q[0], q[1], q[10], q[11], q[16], q[17]
            k = kh * kw * (1 if code == 15 else ic)
            mac = int(ts[z][4]) * int(oh) * int(ow) * int(oc) * int(k) * images
            byt += bbytes + (20 + 3 * oc) * 4
        elif code in (18, 20, 25, 27):
            byt += bbytes * (1 if const_b else images)
        rows.append({"code": code, "bytes": int(byt), "ops": 2 * int(mac)})
    return rows


def roofline(lib, handle, plan, images, iters, peaks, kernel_names):
    n_ops = len(op_traffic(plan, 1))
    ns = (C.c_uint64 * 512)()
    total = C.c_float()
    rc = lib.ug_profile_batch(handle, images, iters, ns, 512, C.byref(total))
    if rc:
        return None, None
    traffic = op_traffic(plan, images)
    per_kind = {}
    for i in range(n_ops):
        kind = kernel_names.get(traffic[i]["code"], f"op{traffic[i]['code']}")
        d = per_kind.setdefault(kind, {"ns": 0, "bytes": 0, "ops": 0, "launches": 0})
        d["ns"] += ns[i] / iters
        d["bytes"] += traffic[i]["bytes"]
        d["ops"] += traffic[i]["ops"]
        d["launches"] += 1 if traffic[i]["code"] != 5 else 0
    top = max(per_kind, key=lambda k: per_kind[k]["ns"])
    d = per_kind[top]
    t = d["ns"] * 1e-9
    gbs = d["bytes"] / t / 1e9
    tops = d["ops"] / t / 1e12
    int8_peak = peaks.get("int8_tops") or 2 * peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"])
    hbm = peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"])
    ai = d["ops"] / max(d["bytes"], 1)
    bound = "hbm" if ai < int8_peak * 1e12 / (hbm * 1e9) else "tensor"
    if bound == "hbm":
        roof = {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s", "frac": round(gbs / hbm, 4)}
    else:
        roof = {"bound": "tensor", "achieved": round(tops, 1), "peak": int8_peak, "unit": "TOPS",
                "frac": round(tops / int8_peak, 4)}
    roof.update({"kernel": top, "traffic": None, "launches_per_step": d["launches"],
                 "ms_per_step": round(d["ns"] / 1e6, 4), "int8_tops": round(tops, 1),
                 "algorithmic_bytes_per_step": d["bytes"], "share_of_eager_step": round(d["ns"] / 1e6 / total.value * iters, 3)})
    top_ops = sorted(range(n_ops), key=lambda i: -ns[i])[:12]
    roof["top_ops"] = [{"op": i, "code": traffic[i]["code"], "ms": round(ns[i] / iters / 1e6, 4),
                        "GB/s": round(traffic[i]["bytes"] / (ns[i] / iters * 1e-9) / 1e9, 1) if ns[i] else None,
                        "TOPS": round(traffic[i]["ops"] / (ns[i] / iters * 1e-9) / 1e12, 1) if ns[i] else None}
                       for i in top_ops]
    breakdown = {k: {"ms": round(v["ns"] / 1e6, 4), "GB/s": round(v["bytes"] / (v["ns"] * 1e-9) / 1e9, 1) if v["ns"] else None,
                     "TOPS": round(v["ops"] / (v["ns"] * 1e-9) / 1e12, 1) if v["ns"] else None}
                 for k, v in sorted(per_kind.items(), key=lambda kv: -kv[1]["ns"])}
    return roof, breakdown


KERNEL_NAMES = {14: "conv", 15: "depthwise", 16: "pool", 17: "softmax_table", 18: "add", 19: "pack", 20: "concat",
                21: "resize", 22: "lut", 23: "pad", 24: "mean", 25: "mul", 26: "slice", 27: "bmm", 28: "softmax_exact",
                10: "permute", 5: "alias"}


# --------------------------------------------------------------------------- one model
def pcie_h2d_gbs(nbytes, device):
    """Host-to-device bandwidth of one plain pinned copy of `nbytes` (the step's input), timed with
    CUDA events: the ceiling of the e2e leg, which moves those bytes every step."""
    try:
        import torch
        src = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
        dst = torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{device}")
        s = torch.cuda.Stream(device=device)
        with torch.cuda.stream(s):
            dst.copy_(src, non_blocking=True)
            s.synchronize()
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record(s)
            for _ in range(3):
                dst.copy_(src, non_blocking=True)
            t1.record(s)
        t1.synchronize()
        gbs = 3 * nbytes / (t0.elapsed_time(t1) / 1e3) / 1e9
        del src, dst
        return round(gbs, 2)
    except Exception:  # torch absent or no pinned memory: the figure is context only
        return None


def detect_leg(lib, handle, model, h_in, per_gpu, global_batch, steps, dist, k=20):
    """The detector's own end-to-end path (ug_detect_batch): uint8 pixels from pinned host memory,
    the bundle's byte table and the one-to-one YOLO top-k on the GPU, k records per image back."""
    from unoq_dsp.modern import YOLODecoder, profile_lookup
    from unoq_dsp.native import RECORD_DTYPE
    md = model.metadata
    decoder = YOLODecoder(md["task"], md["outputs"], md["input"]["shape"])
    config = decoder.device_config()
    prof, q = md["task"]["preprocessing"], md["input"]["quantization"]
    table = np.ascontiguousarray(profile_lookup(tuple(float(v) for v in prof["mean"]),
                                                tuple(float(v) for v in prof["std"]), q["scale"], q["zero_point"], "|i1"))
    if lib.ug_set_yolo_decode(handle, C.byref(config)) or lib.ug_set_input_table(handle, table.ctypes.data, 3):
        raise RuntimeError(f"decoder set-up: {lib.ug_last_error()}")
    h_rec = lib.ug_host_alloc(RECORD_DTYPE.itemsize * k * per_gpu)
    try:
        for _ in range(2):
            lib.ug_detect_batch(handle, h_in, per_gpu, k, h_rec)
        dist.barrier()
        total = 0.0
        for _ in range(steps):
            rc = lib.ug_detect_batch(handle, h_in, per_gpu, k, h_rec)
            if rc:
                raise RuntimeError(f"detect rc={rc}: {lib.ug_last_error()}")
            total += lib.ug_last_infer_ms(handle)
        dist.barrier()
        t = dist.max(total / 1e3)
    finally:
        lib.ug_set_input_table(handle, None, 0)
        lib.ug_set_yolo_decode(handle, None)
        lib.ug_host_free(h_rec)
    ni = int(np.prod(md["input"]["shape"]))
    return {"value": round(global_batch * steps / t, 2), "unit": "images/s", "h2d_bytes_per_step": ni * global_batch,
            "d2h_bytes_per_step": RECORD_DTYPE.itemsize * k * global_batch, "records_per_image": k,
            "ms_per_step": round(t / steps * 1e3, 4),
            "path": "ug_detect_batch: uint8 pixels -> byte table -> network -> top-k decode on the GPU -> records"}


def bench_model(lib, dist, name, global_batch, steps, warmup, peaks, want_roofline, detect=False):
    from unoq_dsp.bundle import load
    spec = MODELS[name]
    model = load(ROOT / "models" / f"{name}.uqmodel")
    plan = model.plan
    start, per_gpu = shard(global_batch, dist.world, dist.rank)
    err = C.c_int()
    buf = C.create_string_buffer(plan, len(plan))
    handle = lib.ug_open_mode(buf, len(plan), 0, C.byref(err))
    if not handle:
        raise RuntimeError(f"ug_open_mode failed {err.value}: {lib.ug_last_error()}")
    try:
        d_in, d_out = C.c_void_p(), C.c_void_p()
        rc = lib.ug_batch_buffers(handle, per_gpu, C.byref(d_in), C.byref(d_out))
        if rc:
            raise RuntimeError(f"batch setup rc={rc}: {lib.ug_last_error()}")
        join_gather(lib, handle, dist)
        ni = int(np.prod(spec["shape"]))
        no = int(model.metadata["output"]["bytes"])
        # seeded synthetic images, pinned host staging for the e2e leg
        h_in = lib.ug_host_alloc(ni * per_gpu)
        # rank 0 receives the gathered outputs of every rank
        out_images = per_gpu * (dist.world if dist.rank == 0 else 1)
        h_out = lib.ug_host_alloc(no * out_images)
        x_host = np.ctypeslib.as_array(C.cast(h_in, C.POINTER(C.c_int8)), shape=(ni * per_gpu,))
        for i in range(per_gpu):
            x_host[i * ni:(i + 1) * ni] = image_input(start + i, ni)
        # device-resident inputs: the seeded images are uploaded once into the batch's arena
        rc = lib.ug_upload_batch(handle, h_in, per_gpu)
        if rc:
            raise RuntimeError(f"ug_upload_batch rc={rc}: {lib.ug_last_error()}")
        kernels = lib.ug_batch_kernel_count(handle, per_gpu)
        for _ in range(warmup):
            lib.ug_launch_batch(handle, per_gpu)
        lib.ug_synchronize(handle)
        dist.barrier()
        ms = C.c_float()
        with ClockSampler(dist.local) as clocks:
            rc = lib.ug_time_batch(handle, per_gpu, steps, C.byref(ms))
        if rc:
            raise RuntimeError(f"timed run rc={rc}: {lib.ug_last_error()}")
        dist.barrier()
        t_dev = dist.max(ms.value / 1e3)
        value = global_batch * steps / t_dev
        # outputs of the device-resident graph that was just timed, sampled on every rank
        rc = lib.ug_download_batch(handle, h_out, per_gpu)
        if rc:
            raise RuntimeError(f"ug_download_batch rc={rc}: {lib.ug_last_error()}")
        y_host = np.ctypeslib.as_array(C.cast(h_out, C.POINTER(C.c_int8)), shape=(no * out_images,))
        local = {start + i: y_host[i * no:(i + 1) * no].tobytes() for i in sample_rows(per_gpu)}
        resident = dist.gather_object(local)
        # e2e through the public batch API (pinned host buffers, copies inside the timed region)
        for _ in range(1):
            rc = lib.ug_infer_batch(handle, h_in, per_gpu, h_out)
            if rc:
                raise RuntimeError(f"e2e warm-up rc={rc}: {lib.ug_last_error()}")
        dist.barrier()
        e2e_ms = 0.0
        for _ in range(steps):
            rc = lib.ug_infer_batch(handle, h_in, per_gpu, h_out)
            if rc:
                raise RuntimeError(f"e2e rc={rc}: {lib.ug_last_error()}")
            e2e_ms += lib.ug_last_infer_ms(handle)
        dist.barrier()
        t_e2e = dist.max(e2e_ms / 1e3)
        verify = None
        if dist.rank == 0:
            # rank 0 holds the whole gathered batch of the last ug_infer_batch call, rank-major
            gathered = {r * per_gpu + i: y_host[(r * per_gpu + i) * no:(r * per_gpu + i + 1) * no].tobytes()
                        for r in range(dist.world) for i in sample_rows(per_gpu)}
            merged = {g: row for part in resident for g, row in part.items()}
            verify = verify_outputs(plan, ni, {"device_resident": merged, "ug_infer_batch": gathered}, dist)
        gather = None
        if dist.world > 1:
            # the one collective alone: every rank's outputs into GPU 0, timed on the device (max
            # over ranks), the bytes that cross NVLink per step being the other ranks' outputs
            gms = C.c_float()
            dist.barrier()  # rank 0 has just run the output check on the host
            rc = lib.ug_time_gather(handle, per_gpu, steps, C.byref(gms))
            if rc:
                raise RuntimeError(f"ug_time_gather rc={rc}: {lib.ug_last_error()}")
            t_g = dist.max(gms.value / 1e3) / steps
            moved = no * per_gpu * (dist.world - 1)
            gather = {"ms_per_step": round(t_g * 1e3, 4), "bytes_into_gpu0_per_step": moved,
                      "GB/s": round(moved / t_g / 1e9, 1), "share_of_step": round(t_g / (t_dev / steps), 4)}
        h2d_gbs = pcie_h2d_gbs(ni * per_gpu, dist.local)
        roof = breakdown = None
        if want_roofline:
            roof, breakdown = roofline(lib, handle, plan, per_gpu, max(1, min(steps, 3)), peaks, KERNEL_NAMES)
        detected = detect_leg(lib, handle, model, h_in, per_gpu, global_batch, steps, dist) if detect else None
        lib.ug_host_free(h_in)
        lib.ug_host_free(h_out)
        return {
            "value": value, "ms_per_step": t_dev / steps * 1e3, "per_gpu_batch": per_gpu, "kernels_per_step": kernels,
            "e2e": {"value": global_batch * steps / t_e2e, "unit": "images/s", "h2d_bytes_per_step": ni * global_batch,
                    "d2h_bytes_per_step": no * global_batch, "ms_per_step": t_e2e / steps * 1e3,
                    "pcie_h2d_gbs": h2d_gbs,
                    "h2d_bound_images_per_s": round(h2d_gbs * 1e9 / ni * dist.world, 1) if h2d_gbs else None},
            "clocks": clocks.summary(), "roofline": roof, "breakdown": breakdown, "detect_e2e": detected,
            "verify": verify, "gather": gather,
        }
    finally:
        lib.ug_close(handle)


# --------------------------------------------------------------------------- BASELINE configs 0-3
class L2Flush:
    """Writes a buffer twice the L2 size between timed launches, so that a config whose working
    set fits in the 126 MB L2 is still timed from HBM."""

    def __init__(self, device):
        import torch
        self.torch = torch
        self.buf = torch.empty(256 << 20, dtype=torch.uint8, device=f"cuda:{device}")
        self.n = 0

    def __call__(self):
        self.n += 1
        self.buf.fill_(self.n & 255)
        self.torch.cuda.synchronize()


def time_plan(lib, plan, images, reps, flush):
    """Median milliseconds of one graph launch of `plan` at `images` (device-resident seeded inputs),
    L2 flushed before each launch, CUDA events on the session stream (ug_time_batch, 1 iteration)."""
    err = C.c_int()
    buf = C.create_string_buffer(plan, len(plan))
    h = lib.ug_open_mode(buf, len(plan), 0, C.byref(err))
    if not h:
        raise RuntimeError(f"ug_open_mode {err.value}: {lib.ug_last_error()}")
    try:
        ni = lib_input_bytes(plan)
        x = np.random.default_rng(5).integers(-128, 128, size=ni * images, dtype=np.int8)
        if lib.ug_upload_batch(h, x.ctypes.data, images):
            raise RuntimeError(lib.ug_last_error())
        ms = C.c_float()
        for _ in range(3):
            lib.ug_time_batch(h, images, 1, C.byref(ms))
        times = []
        for _ in range(reps):
            flush()
            if lib.ug_time_batch(h, images, 1, C.byref(ms)):
                raise RuntimeError(lib.ug_last_error())
            times.append(ms.value)
        return statistics.median(times)
    finally:
        lib.ug_close(h)


def lib_input_bytes(plan):
    import struct
    inp = struct.unpack_from("<I", plan, 20)[0]
    return struct.unpack_from("<12I", plan, 32 + 48 * inp)[1]


def infer_latency(lib, plan, reps=100):
    """Batch-1 latency of the public single-image call ug_infer (pageable host buffers in and out,
    synchronous): median and 99th percentile wall-clock milliseconds over `reps` calls."""
    err = C.c_int()
    buf = C.create_string_buffer(plan, len(plan))
    h = lib.ug_open_mode(buf, len(plan), 0, C.byref(err))
    if not h:
        raise RuntimeError(f"ug_open_mode {err.value}: {lib.ug_last_error()}")
    try:
        import struct
        out_t = struct.unpack_from("<I", plan, 24)[0]
        ni, no = lib_input_bytes(plan), struct.unpack_from("<12I", plan, 32 + 48 * out_t)[1]
        x = np.random.default_rng(6).integers(-128, 128, size=ni, dtype=np.int8)
        y = np.empty(no, dtype=np.int8)
        for _ in range(10):
            lib.ug_infer(h, x.ctypes.data, ni, y.ctypes.data, no)
        t = []
        for _ in range(reps):
            t0 = time.perf_counter()
            if lib.ug_infer(h, x.ctypes.data, ni, y.ctypes.data, no):
                raise RuntimeError(lib.ug_last_error())
            t.append((time.perf_counter() - t0) * 1e3)
        t.sort()
        return {"median_ms": round(statistics.median(t), 4), "p99_ms": round(t[int(0.99 * (len(t) - 1))], 4),
                "calls": reps, "device_ms": round(lib.ug_last_infer_ms(h), 4)}
    finally:
        lib.ug_close(h)


def bench_configs(lib, device, peaks, int8_peak, cores):
    """BASELINE configs 0-3 on one GPU, each beside the reference C path on this host (1 core and
    all cores): config 0 (pointwise conv) and config 1 (16 depthwise layers) per layer at batch 1
    and 256 with GB/s against the measured HBM copy rate; config 2 (MobileNetV4) at batch 1 / 64 /
    256 and config 3 (YOLO26n) at batch 1 / 128 in images/s; and ug_infer batch-1 latency."""
    from unoq_dsp import synth
    from unoq_dsp.bundle import load
    hbm = peaks["hbm_gbs"]
    flush = L2Flush(device)
    gpu, jobs = {}, []
    for name, _ in synth.baseline_config_cases():
        plan, xs, _ = synth.baseline_config(name)
        row = {}
        for images in (1, 256):
            ms = time_plan(lib, plan, images, 9, flush)
            t = op_traffic(plan, images)
            byt, ops = sum(r["bytes"] for r in t), sum(r["ops"] for r in t)
            row[f"b{images}"] = {"ms": round(ms, 5), "GB/s": round(byt / (ms * 1e-3) / 1e9, 1),
                                 "frac_hbm": round(byt / (ms * 1e-3) / 1e9 / hbm, 4),
                                 "TOPS": round(ops / (ms * 1e-3) / 1e12, 2),
                                 "frac_int8": round(ops / (ms * 1e-3) / 1e12 / int8_peak, 4),
                                 "images_per_s": round(images / (ms * 1e-3), 1), "algorithmic_bytes": byt}
        gpu[name] = row
        jobs.append((name, plan, int(np.prod(xs)), 3 if name.startswith("config1") else 5))
    models = {"mobilenetv4-small": (1, 64, 256), "yolo26n-320": (1, 128)}
    latency = {}
    for name, batches in models.items():
        plan = load(ROOT / "models" / f"{name}.uqmodel").plan
        row = {}
        for images in batches:
            ms = time_plan(lib, plan, images, 5, flush)
            row[f"b{images}"] = {"ms": round(ms, 4), "images_per_s": round(images / (ms * 1e-3), 1)}
        gpu[name] = row
        latency[name] = infer_latency(lib, plan)
        jobs.append((name, plan, lib_input_bytes(plan), 2))
    del flush
    from oracle.refpool import reference_timings
    ref = reference_timings(jobs, cores)
    return {"gpu": gpu, "ug_infer_batch1_latency": latency, "reference_cpu": ref,
            "timing": "CUDA events around one graph launch, L2 flushed (256 MB write) before each, median; "
                      "device-resident seeded inputs", "int8_peak_tops": int8_peak,
            "reference_kind": "oracle/_ref/libug_ref.so (the reference runtime's C, gcc -O2, VISION_FLAGS)"}


TRAFFIC_FILE = ROOT / "profiles" / "dram_traffic.json"
CONV_KERNELS = ("conv_tc_kernel", "conv_rows_kernel", "conv_taps_kernel", "conv_small_kernel", "conv_simt_kernel")


def traffic_from_ncu_csv(csv_path, images, step_launches=None):
    """DRAM bytes per image of the conv launches in an ncu launch list (--csv, with the metrics
    dram__bytes_read.sum and dram__bytes_write.sum) of one step at `images` images per launch:
    the first `step_launches` model launches of the list (all when None), after the INT8 peak
    measurement's launches that bench.py makes first."""
    import csv
    total, launches = 0.0, set()
    with open(csv_path, newline="") as f:
        rows = [r for r in csv.reader(line for line in f if line.startswith('"'))]
    head = rows[0]
    col = {k: head.index(k) for k in ("ID", "Kernel Name", "Metric Name", "Metric Unit", "Metric Value")}
    scale = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9, "KB": 1024, "MB": 1024 ** 2, "GB": 1024 ** 3}
    model_ids = sorted({int(r[col["ID"]]) for r in rows[1:] if "int8_mma_peak" not in r[col["Kernel Name"]]})
    keep = set(model_ids if step_launches is None else model_ids[:step_launches])
    for r in rows[1:]:
        if int(r[col["ID"]]) not in keep:
            continue
        if r[col["Metric Name"]] in ("dram__bytes_read.sum", "dram__bytes_write.sum") and \
                any(k in r[col["Kernel Name"]] for k in CONV_KERNELS):
            total += float(r[col["Metric Value"]].replace(",", "")) * scale.get(r[col["Metric Unit"]], 1)
            launches.add(r[col["ID"]])
    return {"conv_dram_bytes_per_image": int(round(total / images)), "conv_launches": len(launches),
            "images_per_launch": images, "step_launches": step_launches, "csv": Path(csv_path).name}


def write_traffic(model, csv_path, images, step_launches):
    """Record one model's conv DRAM traffic per image in profiles/dram_traffic.json."""
    data = json.loads(TRAFFIC_FILE.read_text()) if TRAFFIC_FILE.is_file() else {}
    data[model] = traffic_from_ncu_csv(csv_path, images, step_launches)
    TRAFFIC_FILE.write_text(json.dumps(data, indent=1, sort_keys=True) + "\n")
    return data[model]


def attach_traffic(roof, model, images):
    """Fill roofline.traffic of the conv family from profiles/dram_traffic.json (written from the
    ncu launch-list CSV by `bench.py --write-traffic`), scaled to this step's images: every image
    is an independent slice of each launch, so DRAM traffic grows with the images processed."""
    if roof is None or roof.get("kernel") != "conv" or not TRAFFIC_FILE.is_file():
        return
    entry = json.loads(TRAFFIC_FILE.read_text()).get(model)
    if entry:
        roof["traffic"] = entry["conv_dram_bytes_per_image"] * images
        roof["traffic_source"] = (f"ncu dram__bytes_read.sum + dram__bytes_write.sum of the {entry['conv_launches']} "
                                  f"conv launches of one step at {entry['images_per_launch']} images "
                                  f"(profiles/dram_traffic.json from {entry['csv']}), scaled by images")


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.is_file():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return dict(PEAKS_FALLBACK, source="fallback")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--global-batch", type=int, default=MODELS["mobilenetv4-small"]["batch"])
    ap.add_argument("--yolo-batch", type=int, default=MODELS["yolo26n-320"]["batch"])
    ap.add_argument("--no-yolo", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip the BASELINE config 0-3 section (1 GPU only)")
    ap.add_argument("--yolo-only", action="store_true",
                    help="profiling aid: run only the YOLO26n section and print its fields")
    ap.add_argument("--write-traffic", nargs=4, metavar=("MODEL", "CSV", "IMAGES", "STEP_LAUNCHES"),
                    help="record a model's conv DRAM traffic from the first STEP_LAUNCHES launches (one step) "
                         "of an ncu launch-list CSV, then exit")
    args = ap.parse_args()
    if args.write_traffic:
        model, csv_path, images, step = args.write_traffic
        print(json.dumps(write_traffic(model, csv_path, int(images), int(step))))
        return
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    mpath = ROOT / "models" / "mobilenetv4-small.uqmodel"
    cores = os.cpu_count() or 1
    config = {"workload": f"MobileNetV4-Conv-Small-224 INT8, global batch {args.global_batch} batch-sharded over "
                          f"{world} GPU(s) (BASELINE config 4); YOLO26n-320 INT8 global batch {args.yolo_batch} "
                          "alongside", "model": "mobilenetv4-small.uqmodel (bundled weights)",
              "global_batch": args.global_batch, "image": "224x224x3 int8 NHWC", "parallelism": f"dp{world}",
              "l2": "inputs larger than L2 (616 MB per 4096 images); no flush needed",
              "collective": "int8 outputs gathered into GPU 0 over NCCL inside every timed step" if world > 1
              else "none (1 GPU)"}

    if args.impl == "reference":
        if rank != 0:
            return
        from oracle.oracle import REF_LIB
        if not REF_LIB.is_file():
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libug_ref.so not built"}))
            return
        pool = make_pool(cores, mpath)
        per_proc = 1
        for _ in range(args.warmup):
            reference_throughput(MODELS["mobilenetv4-small"]["shape"], per_proc, cores, pool)
        t0 = time.perf_counter()
        n = 0
        for _ in range(args.steps):
            reference_throughput(MODELS["mobilenetv4-small"]["shape"], per_proc, cores, pool)
            n += per_proc * cores
        wall = time.perf_counter() - t0
        pool.close()
        value = n / wall
        sample = f"{per_proc} image(s) per process per step x {cores} processes, seeded int8 input"
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "images/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": wall / args.steps * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8 (u8 x s8 -> s32)",
            "data": "synthetic seeded images", "config": config,
            "cpu_baseline": {"value": round(value, 3), "unit": "images/s", "cores": cores, "kind": "reference",
                             "sample": sample},
            "e2e": {"value": round(value, 3), "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return

    # CPU baseline pool is spawned before the first CUDA call in this process.
    pool = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle.oracle import REF_LIB
        if REF_LIB.is_file():
            pool = make_pool(cores, mpath)

    from unoq_dsp.native import load_library
    lib = load_library()
    dist = Dist(args.gpus)
    if lib.ug_set_device(dist.local) != 0:
        raise SystemExit(f"cannot select CUDA device {dist.local}")
    peaks = load_peaks()
    # the INT8 tensor-core peak of this device, measured (tcgen05 kind::i8 on shared-memory operands)
    tops, peak_ms = C.c_float(), C.c_float()
    if lib.ug_measure_int8_peak(8192, C.byref(tops), C.byref(peak_ms)) == 0 and tops.value > 0:
        peaks["int8_tops"] = round(float(tops.value), 1)
        peaks["int8_source"] = f"measured: ug_measure_int8_peak, {peak_ms.value:.2f} ms launch, burst"
    if args.yolo_only:
        yolo = bench_model(lib, dist, "yolo26n-320", args.yolo_batch, args.steps, args.warmup, peaks, True, detect=True)
        dist.close()
        if rank == 0:
            print(json.dumps({"model": "yolo26n-320", **{k: yolo[k] for k in ("value", "ms_per_step", "e2e", "detect_e2e",
                                                                              "roofline", "kernels_per_step")}}))
        return
    res = bench_model(lib, dist, "mobilenetv4-small", args.global_batch, args.steps, args.warmup, peaks, True)
    yolo = None
    if not args.no_yolo:
        yolo = bench_model(lib, dist, "yolo26n-320", args.yolo_batch, args.steps, args.warmup, peaks, True, detect=True)
    cpu = None
    if pool is not None:
        # bounded sample: about 25 s of CPU work in total, spread over every host core
        _, _, t1 = reference_throughput(MODELS["mobilenetv4-small"]["shape"], 1, cores, pool)
        per_proc = max(1, min(32, int(25.0 / (cores * max(t1, 1e-3)))))
        value, wall, _ = reference_throughput(MODELS["mobilenetv4-small"]["shape"], per_proc, cores, pool)
        pool.close()
        cpu = {"value": round(value, 3), "unit": "images/s", "cores": cores, "kind": "reference",
               "sample": f"{per_proc * cores} MobileNetV4 images ({per_proc} per process on {cores} processes), "
                         f"{wall:.1f} s wall"}
    configs = None
    if world == 1 and not args.no_configs:
        int8 = peaks.get("int8_tops") or 2 * peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"])
        configs = bench_configs(lib, dist.local, peaks, int8, cores)
    launches = int(dist.sum(res["kernels_per_step"] * args.steps))  # whole job: every rank's launches
    dist.close()
    if rank != 0:
        return
    roof = res["roofline"]
    if roof is not None:
        roof["peak_source"] = peaks["source"]
        attach_traffic(roof, "mobilenetv4-small", res["per_gpu_batch"])
    if yolo is not None and yolo["roofline"] is not None:
        yolo["roofline"]["peak_source"] = peaks["source"]
        attach_traffic(yolo["roofline"], "yolo26n-320", yolo["per_gpu_batch"])
    line = {
        "metric": METRIC, "value": round(res["value"], 2), "unit": "images/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(res["ms_per_step"], 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8 (s8 x s8 -> s32, int64 requant)",
        "data": "synthetic seeded int8 images; bundled model weights", "config": config,
        "e2e": {k: (round(v, 2) if isinstance(v, float) else v) for k, v in res["e2e"].items()},
        "roofline": roof, "cpu_baseline": cpu, "clocks": res["clocks"], "gpu_launches": launches,
        "per_gpu_batch": res["per_gpu_batch"], "kernel_breakdown": res["breakdown"],
        "int8_peak": {"tops": peaks.get("int8_tops"), "source": peaks.get("int8_source", "2 x measured bf16 (stand-in)")},
        "gather": res["gather"],
    }
    if configs is not None:
        line["baseline_configs"] = configs
    checks = {"mobilenetv4-small": res["verify"]}
    if yolo is not None:
        checks["yolo26n-320"] = yolo["verify"]
    line["verify"] = {"images": sum(c["images"] for c in checks.values()),
                      "mismatch": sum(c["mismatch"] for c in checks.values()), "models": checks,
                      "what": "first, middle and last image of every rank's shard, from the timed device-resident "
                              "graph and from the gathered ug_infer_batch output, against the reference runtime"}
    if yolo is not None:
        line[MODELS["yolo26n-320"]["key"]] = {
            "value": round(yolo["value"], 2), "unit": "images/s", "global_batch": args.yolo_batch,
            "ms_per_step": round(yolo["ms_per_step"], 4), "e2e": yolo["e2e"], "detect_e2e": yolo["detect_e2e"],
            "roofline": yolo["roofline"],
            "kernels_per_step": yolo["kernels_per_step"], "kernel_breakdown": yolo["breakdown"], "clocks": yolo["clocks"],
            "gather": yolo["gather"]}
    print(json.dumps(line))


if __name__ == "__main__":
    main()
