#!/usr/bin/env python
"""ZTCP cold-page codec benchmark on B200 -- prints one JSON line (rank 0).

Workload: the reference's headline configuration (its benchmark's config 0) -- batches of 256 GQA pages
(64 tokens x 8 KV heads x 128, separate K and V in bf16, 256 KiB hot per page), INT4_SYM + PRESERVE_FP8,
N(0,1) values with four x15 RoPE outlier channels per head, random 256-bit ChaCha20 key, 128-bit SipHash
key and 64-bit base nonce.  A batch round trip is egress (quantize, pack, encrypt, tag) of the 256 pages
followed by ingress (verify, decrypt, dequantize) of the blobs it produced.

One step = one window of --inflight (default 32) independent 256-page batch round trips, batch j of every
window on CUDA stream j.  A page's tag is one serial SipHash chain (~0.6 ms), so throughput comes from many
batches in flight; timing whole windows back to back keeps the pipeline's fill and drain (one chain
latency each) small against the timed work at any --steps.  value = (egress + ingress) hot bytes / time,
SI GB/s, inputs resident in HBM (32 input sets, > L2).

Also on the line: integer-ALU ceilings of the codec's primitives measured on this GPU in the same run
(ztcp_measure_int_peaks), every kernel's launch time split by phase marks with its roofline against
max(HBM time, ALU time), the end-to-end rate through host memory (e2e), the other benchmark
configurations (K8V4_ASYM 64-page, MLA 256-page, fidelity of config 2) and the 4,096-page prefix sweep
(config 4), and the reference codec timed on the host cores (cpu_baseline).

Multi-GPU: pages are independent, so every rank runs its own windows with no collective on the data path
(weak scaling); the only collectives are the barriers and the max-over-ranks reduction of the timings.

--impl reference times the reference codec (built from its own source into oracle/_ref) on the host
cores: one process per core, each running the reference's peak egress and peak ingress entry points on
its share of a 256-page batch, plus the reference's threaded batch encode.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "vlx-tee_b200"))
# One hardware work queue per in-flight batch (the driver default is 8; a batch waiting on its own
# 0.6 ms tag chain would otherwise stall the batches that share its queue).  Process-local: read by
# the CUDA driver when this process creates its context.
os.environ.setdefault("CUDA_DEVICE_MAX_CONNECTIONS", "32")

PAGE_HOT_BYTES = 2 * 64 * 8 * 128 * 2       # K + V, bf16/fp16
EXPECTED_PAYLOAD = 98304                     # INT4_SYM + PRESERVE_FP8, GQA 64x8x128
BLOB_BYTES = 32 + EXPECTED_PAYLOAD + 16
METRIC = "egress+ingress hot-byte GB/s (INT4_SYM+PRESERVE_FP8 256-page GQA batch)"
WORKLOAD = "cfg0: 256-page GQA 64x8x128 INT4_SYM+PRESERVE_FP8 egress+ingress round trip"


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20, help="timed steps (one window of --inflight batches each)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--pages", type=int, default=256, help="pages per batch")
    ap.add_argument("--inflight", type=int, default=32, help="batches per step, each on its own CUDA stream")
    ap.add_argument("--e2e-inflight", type=int, default=8,
                    help="batches per end-to-end step (host<->device copies are link-bound; a few streams keep "
                         "both copy directions busy)")
    ap.add_argument("--graphs", action="store_true",
                    help="launch each timed round trip as a CUDA graph captured from the same codec calls (one "
                         "graph per input set), instead of calling the codec API every step")
    ap.add_argument("--cpu-seconds", type=float, default=8.0, help="bounded CPU baseline sample length")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip the config 1/2/3 legs")
    ap.add_argument("--prefix-pages", type=int, default=4096,
                    help="pages of the full-prefix sweep (benchmark config 4), split over the ranks (0 = skip)")
    ap.add_argument("--prefix-chunk", type=int, default=0,
                    help="pages per codec call in the prefix sweep (0 = a rank's whole shard in one call per direction; "
                         "calls of 1,024 pages or more run the egress in wire order)")
    ap.add_argument("--prefix-reps", type=int, default=3)
    return ap.parse_args()


def measured_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def committed_traffic():
    """Per-launch DRAM traffic of each kernel from the committed ncu summaries, if any."""
    try:
        with open(os.path.join(REPO, "profiles", "traffic.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


def host_cpu():
    model = "unknown"
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    return model, cores


# ------------------------------------------------------------------------------------------------
# clocks during the timed region
# ------------------------------------------------------------------------------------------------
class ClockSampler:
    """Polls NVML every 5 ms from a background thread while the timed region runs (SM clock and clock
    event reasons), so even a region of a few milliseconds gets samples."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown"}

    def __init__(self, dev_index: int):
        self.dev_index = dev_index
        self.samples, self.reason_bits, self.max_mhz = [], 0, None
        self._stop = None

    def _handle(self, nv):
        import torch

        p = torch.cuda.get_device_properties(self.dev_index)
        try:
            return nv.nvmlDeviceGetHandleByPciBusId(f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0")
        except Exception:  # noqa: BLE001  (older torch: no PCI ids; fall back to the visible-device order)
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            idx = int(vis.split(",")[self.dev_index]) if vis else self.dev_index
            return nv.nvmlDeviceGetHandleByIndex(idx)

    def __enter__(self):
        import threading

        try:
            import pynvml as nv

            nv.nvmlInit()
            h = self._handle(nv)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        except Exception:  # noqa: BLE001
            return self
        self._stop = threading.Event()

        def run():
            while not self._stop.is_set():
                try:
                    self.samples.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
                    self.reason_bits |= int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))
                except Exception:  # noqa: BLE001
                    pass
                self._stop.wait(0.005)

        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._stop is not None:
            self._stop.set()
            self._thread.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml unavailable"], "samples": 0}
        reasons = sorted(n for b, n in self.REASONS.items() if self.reason_bits & b)
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples), "sm_mhz_min": min(self.samples)}


# ------------------------------------------------------------------------------------------------
# reference codec on the host cores
# ------------------------------------------------------------------------------------------------
def _ref_inputs(pages, seed):
    import torch

    from ztcp_b200 import workload

    k32, v32 = workload.kv_pages_np(pages, workload.GQA, seed=seed)
    k = torch.from_numpy(k32).to(torch.bfloat16).half()   # the reference codec accepts fp16 only
    v = torch.from_numpy(v32).to(torch.bfloat16).half()
    toks = torch.from_numpy(workload.token_hashes(pages, seed + 1))
    return k, v, toks, workload.session_material(7)


def _load_ref():
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import build_ref

    try:
        return build_ref.load_module()
    except FileNotFoundError:
        return None


def _ref_worker(args):
    """One process: the reference's peak egress + peak ingress on `pages` pages until `seconds` pass.

    Runs the reference codec built from its own source (oracle/_ref); where that build is absent, the
    oracle's C restatement of it (same work per page, kind "port").  Returns (pages, seconds, kind)."""
    worker, pages, seconds = args
    import numpy as np
    import torch

    torch.set_num_threads(1)
    k, v, toks, m = _ref_inputs(pages, 42 + worker)
    key, mk = m["key"], m["mac_key"]
    ref = _load_ref()
    if ref is None:
        import ztcp_oracle as port

        kb, vb, tk = k.numpy().view(np.uint16), v.numpy().view(np.uint16), toks.numpy()

        def round_trip(it):
            blobs = port.encode_batch(kb, vb, tk, rope_dim=64, preset=1, rope_mode=1,
                                      expected_payload=EXPECTED_PAYLOAD, tenant=m["tenant"], model=m["model"],
                                      layer=m["layer"], head_group=m["head_group"],
                                      base_seq=(m["base_seq"] + it * pages + worker * 2**32) % 2**64, key=key,
                                      mac_key=mk)
            port.decode_batch(blobs, tk, num_tokens=64, num_heads=8, head_dim=128, rope_dim=64, is_mla=False,
                              tenant=m["tenant"], model=m["model"], layer=m["layer"], key=key, mac_key=mk)
        kind = "port"
    else:
        out = torch.empty((pages, BLOB_BYTES), dtype=torch.uint8)
        kd, vd = torch.empty_like(k), torch.empty_like(v)

        def round_trip(it):
            ref.fused_encode_cold_pages_peak_into_cpu(k, v, toks, out, 1, 1, 64, EXPECTED_PAYLOAD, m["tenant"],
                                                      m["model"], m["layer"], m["head_group"],
                                                      (m["base_seq"] + it * pages + worker * 2**32) % 2**64,
                                                      key[0], key[1], mk[0], mk[1], key[2], key[3])
            ref.fused_decode_cold_pages_peak_into_cpu(out, toks, kd, vd, 64, False, m["tenant"], m["model"],
                                                      m["layer"], key[0], key[1], mk[0], mk[1], key[2], key[3])
        kind = "reference"
    done, it = 0, 0
    t0 = time.perf_counter()
    while True:
        round_trip(it)
        done += pages
        it += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            return done, el, kind


def _ref_threaded_encode(args):
    """One process: the reference's own multi-threaded batch egress (fused_encode_cold_pages_batch_cpu, one
    std::thread per hardware thread over contiguous page chunks, csrc:1858-1899) on `pages` pages until
    `seconds` pass.  Returns (pages, seconds) or None without the reference build."""
    pages, seconds = args
    k, v, toks, m = _ref_inputs(pages, 4242)
    key, mk = m["key"], m["mac_key"]
    ref = _load_ref()
    if ref is None:
        return None
    done, it = 0, 0
    t0 = time.perf_counter()
    while True:
        ref.fused_encode_cold_pages_batch_cpu(k, v, toks, 1, 1, 64, EXPECTED_PAYLOAD, m["tenant"], m["model"],
                                              m["layer"], m["head_group"], (m["base_seq"] + it * pages) % 2**64,
                                              key[0], key[1], mk[0], mk[1], key[2], key[3])
        done += pages
        it += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            return done, el


def reference_baseline(seconds: float, batch_pages: int = 256):
    """The reference codec on every host core: one process per core, each running the reference's peak
    egress + peak ingress on its share of a `batch_pages`-page batch (a harness-level split: on Linux the
    reference's peak entry points are serial loops), then the reference's threaded batch egress alone."""
    import multiprocessing as mp

    model, cores = host_cpu()
    per = -(-batch_pages // cores)
    ctx = mp.get_context("spawn")
    with ctx.Pool(cores) as pool:
        res = pool.map(_ref_worker, [(w, per, seconds) for w in range(cores)])
    pages = sum(r[0] for r in res)
    wall = max(r[1] for r in res)
    kind = res[0][2]
    gbs = 2 * pages * PAGE_HOT_BYTES / wall / 1e9
    what = ("reference fused_encode_cold_pages_peak_into_cpu + fused_decode_cold_pages_peak_into_cpu (oracle/_ref, "
            "the reference's own source, scalar x86-64 build, 1 thread each)" if kind == "reference" else
            "the oracle's C restatement of the reference codec, batch encode + decode (oracle/_ref absent), "
            "1 thread each")
    out = {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": kind, "cpu_model": model,
           "nproc": os.cpu_count(),
           "sample": (f"{cores} processes x {per}-page batches (a {batch_pages}-page batch split over the cores) for "
                      f"{seconds:g} s: {what}; {pages} pages round-tripped")}
    with ctx.Pool(1) as pool:
        thr = pool.map(_ref_threaded_encode, [(batch_pages, max(1.0, seconds / 2))])[0]
    if thr is not None:
        out["threaded_batch_egress"] = {
            "egress_hot_gbs": round(thr[0] * PAGE_HOT_BYTES / thr[1] / 1e9, 3),
            "sample": (f"reference fused_encode_cold_pages_batch_cpu on {batch_pages}-page batches in one process "
                       f"(its own std::thread per hardware thread) for {thr[1]:.1f} s, {thr[0]} pages")}
    return out


def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    base = reference_baseline(args.cpu_seconds, args.pages)
    per_batch_ms = 2 * args.pages * PAGE_HOT_BYTES / (base["value"] * 1e9) * 1e3
    line = {"metric": METRIC, "value": base["value"], "unit": "GB/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(per_batch_ms * args.inflight, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u32+f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "pages_per_batch": args.pages, "batches_per_step": args.inflight,
                       "host_cores": base["cores"], "cpu_model": base["cpu_model"]},
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


# ------------------------------------------------------------------------------------------------
# our arm
# ------------------------------------------------------------------------------------------------
class Leg:
    """One benchmark configuration: `n_sets` resident input sets of `pages`-page batches on one GPU, with
    the egress / ingress calls of one batch.  Set j always runs on stream j % len(streams)."""

    def __init__(self, name, shape, preset, rope_mode, pages, n_sets, dev, rank, m, keys, seed0):
        import torch

        from ztcp_b200 import capi, codec, sharding, workload

        self.name, self.shape, self.preset, self.rope_mode, self.pages = name, shape, preset, rope_mode, pages
        self.m, self.keys = m, keys
        g = capi.geometry(shape.num_tokens, shape.num_heads, shape.head_dim, shape.rope_dim, shape.mla)
        self.payload = int(capi.load().ztcp_spec_payload_bytes(preset, rope_mode, C.byref(g), 0 if shape.mla else 1))
        self.blob = 48 + self.payload
        self.hot = (1 if shape.mla else 2) * shape.vecs * shape.head_dim * 2
        dims = (pages, shape.num_tokens, shape.num_heads, shape.head_dim)
        self.sets = []
        for s in range(n_sets):
            seed = seed0 + 1000 * rank + s
            k, v = workload.kv_pages_torch(pages, shape, seed=seed, device=dev)
            self.sets.append({
                "k": k, "v": v, "toks": torch.from_numpy(workload.token_hashes(pages, seed)).to(dev),
                "seq": (m["base_seq"] + sharding.global_page_base(rank, s, n_sets, pages)) % 2**64,
                "blobs": torch.empty((pages, self.blob), dtype=torch.uint8, device=dev),
                "kout": torch.empty(dims, dtype=torch.float16, device=dev),
                "vout": None if shape.mla else torch.empty(dims, dtype=torch.float16, device=dev),
                "status": torch.empty(pages, dtype=torch.int32, device=dev),
                "fail": torch.zeros(1, dtype=torch.int32, device=dev),
            })

        # each set's egress and ingress through the public API, checked and packed once (codec.prepare_*):
        # a timed call only enqueues its two kernels on the given stream
        self.calls = []
        for S in self.sets:
            enc = codec.prepare_encode(S["k"], S["v"], S["toks"], S["blobs"], rope_dim=shape.rope_dim, preset=preset,
                                       rope_mode=rope_mode, expected_payload_bytes=self.payload,
                                       tenant_id_hash=m["tenant"], model_id_hash=m["model"], layer_id=m["layer"],
                                       head_group_id=m["head_group"], base_sequence_nonce=S["seq"], keys=keys)
            dec = codec.prepare_decode(S["blobs"], S["toks"], S["kout"], S["vout"], rope_dim=shape.rope_dim,
                                       is_mla=shape.mla, tenant_id_hash=m["tenant"], model_id_hash=m["model"],
                                       layer_id=m["layer"], keys=keys, status=S["status"], any_fail=S["fail"])
            self.calls.append((enc, dec))

    def egress(self, j, stream=None):
        self.calls[j % len(self.calls)][0](stream)

    def ingress(self, j, stream=None):
        self.calls[j % len(self.calls)][1](stream)

    def round_trip(self, i, stream=None):
        enc, dec = self.calls[i % len(self.calls)]
        enc(stream)
        dec(stream)

    def check(self, what):
        bad = sum(int(S["fail"].item()) for S in self.sets)
        if bad:
            raise RuntimeError(f"{self.name} {what}: a round trip failed verification")


def windows(streams, first, count, step_fn, dev):
    """`count` windows of len(streams) batches (batch j of a window on stream j, passed to step_fn), bracketed
    by events on the current stream; returns (start, end)."""
    import torch

    D = len(streams)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    main = torch.cuda.current_stream(dev)
    start.record(main)
    for st in streams:
        st.wait_event(start)
    for w in range(first, first + count):
        for j in range(D):
            step_fn(w * D + j, streams[j])
    for st in streams:
        done = torch.cuda.Event()
        done.record(st)
        main.wait_event(done)
    end.record(main)
    return start, end


def kernel_times(leg, iters, lib):
    """Per-kernel launch durations of one batch in flight (inputs cycling over the resident sets, larger than
    L2): CUDA events around each codec call, split between its two kernels by a phase mark.  Medians, ms."""
    import torch

    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(6)] for _ in range(iters)]
    for row in ev:  # the raw events exist once recorded
        for e in row:
            e.record()
    torch.cuda.synchronize()
    for i in range(iters):
        e = ev[i]
        e[0].record()
        lib.ztcp_mark_phase(C.c_void_p(e[1].cuda_event))
        leg.egress(i)
        e[2].record()
        e[3].record()
        lib.ztcp_mark_phase(C.c_void_p(e[4].cuda_event))
        leg.ingress(i)
        e[5].record()
    torch.cuda.synchronize()
    leg.check("kernel timing")
    med = lambda a, b: statistics.median(ev[i][a].elapsed_time(ev[i][b]) for i in range(iters))  # noqa: E731
    return {"egress_tile_kernel": med(0, 1), "mac_kernel<sign>": med(1, 2), "egress_call": med(0, 2),
            "mac_kernel<verify>": med(3, 4), "ingress_tile_kernel": med(4, 5), "ingress_call": med(3, 5)}


def kernel_rooflines(leg, kt, peaks, hbm_peak, traffic):
    """Roofline of each kernel for one launch of `leg.pages` pages: the slower of its algorithmic HBM bytes
    at the measured copy bandwidth and its integer work at the ceilings measured in this run (ChaCha20
    blocks for the tile kernels, SipHash words over every SM for the chains); chains also against the latency
    floor of one page's chain (its words at the register-only chain's cycles per word)."""
    n, blocks = leg.pages, leg.payload // 64
    words = (32 + leg.payload) // 8 + 1
    per_page = {
        "egress_tile_kernel": (leg.hot + 8, 32 + leg.payload, "chacha", blocks),
        "mac_kernel<sign>": (32 + leg.payload, 16, "sip", words),
        "mac_kernel<verify>": (leg.blob + 8, 4, "sip", words),
        "ingress_tile_kernel": (32 + leg.payload, leg.hot, "chacha", blocks),
    }
    out = {}
    chain_floor_ms = peaks["sip_chain_ms"] * words / 12293.0
    for name, (rd, wr, kind, units) in per_page.items():
        ms = kt[name]
        byts = n * (rd + wr)
        t_hbm = byts / (hbm_peak * 1e9) * 1e3
        rate = peaks["chacha20_blocks_per_s"] if kind == "chacha" else peaks["sip_words_per_s"]
        t_alu = n * units / rate * 1e3
        bound_ms = max(t_hbm, t_alu)
        e = {"launch_ms": round(ms, 4), "pages": n, "algorithmic_bytes": byts,
             "achieved_gbs": round(byts / (ms * 1e-3) / 1e9, 1),
             "hbm_ms": round(t_hbm, 4), "alu_ms": round(t_alu, 4),
             "alu_work": f"{n * units} {'ChaCha20 blocks' if kind == 'chacha' else 'SipHash words'}",
             "bound": "hbm" if t_hbm >= t_alu else "alu", "frac": round(bound_ms / ms, 4),
             "traffic": traffic.get(name, {}).get("dram_bytes_per_launch")}
        if e["traffic"] is not None:
            e["traffic"] = int(e["traffic"] * n / traffic[name].get("pages_per_launch", n))
        if kind == "sip":
            e["chain_floor_ms"] = round(chain_floor_ms, 4)
            e["frac_of_chain_floor"] = round(chain_floor_ms / ms, 4)
        out[name] = e
    return out


def ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    from ztcp_b200 import capi, codec, offload, sharding, workload

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    # baseline sample first: the spawn pool starts before this process does GPU work
    cpu_base = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu_base = reference_baseline(args.cpu_seconds, args.pages)

    lib = capi.load()
    # integer ceilings of the codec's primitives on this GPU (roofline denominators of the ALU terms)
    scratch = torch.empty(capi.MEASURE_SCRATCH_BYTES, dtype=torch.uint8, device=dev)
    pk = capi.IntPeaks()
    capi.check(lib.ztcp_measure_int_peaks(scratch.data_ptr(), scratch.numel(), C.byref(pk)))
    peaks = {f: getattr(pk, f) for f, _ in capi.IntPeaks._fields_ if f != "reserved"}
    del scratch

    n = args.pages
    D = max(1, args.inflight)
    m = workload.session_material(7)
    keys = capi.keys(*m["key"], *m["mac_key"])
    leg = Leg("cfg0", workload.GQA, 1, 1, n, D, dev, rank, m, keys, 42)
    streams = [torch.cuda.Stream(device=dev) for _ in range(D)]

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    windows(streams, 0, args.warmup, leg.round_trip, dev)
    torch.cuda.synchronize()
    leg.check("warm-up")

    step_fn = leg.round_trip
    graphs = []
    if args.graphs:
        # the same egress + ingress calls, captured once per input set on the set's stream; a timed batch
        # replays its set's graph (same kernels and work, one launch call instead of two API calls)
        for j in range(D):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=streams[j]):
                leg.round_trip(j)
            graphs.append(g)
        torch.cuda.synchronize()

        def step_fn(i, stream):
            with torch.cuda.stream(stream):
                graphs[i % D].replay()

        windows(streams, 0, args.warmup, step_fn, dev)
        torch.cuda.synchronize()
        leg.check("graph warm-up")

    K = args.steps
    with ClockSampler(local) as clocks:
        barrier()
        torch.cuda.synchronize()
        h0 = time.perf_counter()
        t0, t1 = windows(streams, args.warmup, K, step_fn, dev)
        host_enqueue_ms = (time.perf_counter() - h0) * 1e3
        torch.cuda.synchronize()
        wall_ms = (time.perf_counter() - h0) * 1e3
        barrier()
    total_ms = t0.elapsed_time(t1)
    leg.check("timed region")

    # per-kernel launch times (one batch in flight) and single-batch latency of each direction
    kt = kernel_times(leg, 12, lib)

    # end to end through the public API with pinned host buffers: every batch uploads its K/V and token
    # hashes, encodes, downloads the blobs, uploads them again, decodes, and downloads K/V and the status.
    DE = max(1, min(args.e2e_inflight, D))
    host = []
    for j in range(DE):
        S = leg.sets[j]
        host.append({"k": S["k"].cpu().pin_memory(), "v": S["v"].cpu().pin_memory(),
                     "toks": S["toks"].cpu().pin_memory(),
                     "blobs": torch.empty((n, BLOB_BYTES), dtype=torch.uint8).pin_memory(),
                     "kout": torch.empty((n, 64, 8, 128), dtype=torch.float16).pin_memory(),
                     "vout": torch.empty((n, 64, 8, 128), dtype=torch.float16).pin_memory()})

    # through ztcp_b200.offload.OffloadPipeline: each batch's egress (upload K/V -> encode -> download blobs)
    # and ingress (upload blobs -> decode -> download K/V + status) on the pipeline's slots; a batch's egress
    # waits for the ingress that last used the same host buffers.
    pipe = offload.OffloadPipeline(dev, slots=2 * DE)
    last_ingress = [None] * DE

    def e2e_batch(i):
        H, S = host[i % DE], leg.sets[i % DE]
        t = pipe.egress(H["k"], H["v"], H["toks"], H["blobs"], rope_dim=64, preset=1, rope_mode=1,
                        expected_payload_bytes=EXPECTED_PAYLOAD, tenant_id_hash=m["tenant"], model_id_hash=m["model"],
                        layer_id=m["layer"], head_group_id=m["head_group"], base_sequence_nonce=S["seq"], keys=keys,
                        after=last_ingress[i % DE])
        last_ingress[i % DE] = pipe.ingress(H["blobs"], H["toks"], H["kout"], H["vout"], rope_dim=64, is_mla=False,
                                            tenant_id_hash=m["tenant"], model_id_hash=m["model"], layer_id=m["layer"],
                                            keys=keys, after=t)

    for i in range(DE):
        e2e_batch(i)
    for tk in last_ingress:
        tk.wait()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for sl in pipe._slots:
        sl.stream.wait_event(e0)
    for i in range(DE, DE + K * DE):
        e2e_batch(i)
    for sl in pipe._slots:
        torch.cuda.current_stream(dev).wait_event(sl.idle)
    e1.record()
    torch.cuda.synchronize()
    for tk in last_ingress:
        tk.wait()  # raises the reference's error if any page failed
    if not torch.equal(host[0]["kout"], leg.sets[0]["kout"].cpu()):
        raise RuntimeError("end-to-end output differs from the device-resident run")
    del host, pipe

    # the other benchmark configurations: K8V4_ASYM 64-page batches (config 1), MLA 576-wide 256-page batches
    # (config 3), each timed like config 0 over fewer windows, and config 2's fidelity (config 0's bytes
    # decoded, 32 seed-99 queries per head, attention-output cosine against the bf16 input)
    configs = None
    if not args.no_configs:
        configs = {}
        cos = workload.attention_cosine(leg.sets[0]["k"].float(), leg.sets[0]["v"].float(),
                                        leg.sets[0]["kout"].float(), leg.sets[0]["vout"].float(), n_queries=32, seed=99)
        configs["cfg2"] = {"workload": "cfg2: config 0's 256 pages decoded; attention-output cosine against the bf16 "
                                       "pages, 32 N(0,1) queries per head from seed 99, float64",
                           "attention_output_cosine": round(cos, 6)}
        for name, shape, preset, pages, desc in (
                ("cfg1", workload.GQA, 2, 64, "cfg1: 64-page GQA 64x8x128 K8V4_ASYM+PRESERVE_FP8 round trip"),
                ("cfg3", workload.MLA, 1, 256, "cfg3: 256-page MLA 64x1x576 (RoPE-first) INT4_SYM+PRESERVE_FP8 round trip")):
            L2 = Leg(name, shape, preset, 1, pages, D, dev, rank, m, keys, 77)
            cw = max(2, K // 2)
            windows(streams, 0, 2, L2.round_trip, dev)
            torch.cuda.synchronize()
            barrier()
            a, b = windows(streams, 2, cw, L2.round_trip, dev)
            torch.cuda.synchronize()
            L2.check("timed region")
            ms = a.elapsed_time(b)
            kt2 = kernel_times(L2, 8, lib)
            entry = {"workload": desc, "pages_per_batch": pages, "batches_per_step": D, "steps": cw,
                     "ms_per_step": round(ms / cw, 4), "payload_bytes": L2.payload, "blob_bytes": L2.blob,
                     "hot_gbs": round(2 * pages * L2.hot * D * cw * world / (ms * 1e-3) / 1e9, 2),
                     "wire_gbs": round(2 * pages * L2.blob * D * cw * world / (ms * 1e-3) / 1e9, 2),
                     "single_batch": {"egress_ms": round(kt2["egress_call"], 4),
                                      "ingress_ms": round(kt2["ingress_call"], 4)},
                     "kernels_ms": {k: round(v, 4) for k, v in kt2.items() if not k.endswith("_call")}}
            if name == "cfg3":
                S = L2.sets[0]
                entry["softmax_weights_cosine"] = round(workload.attention_cosine(
                    S["k"].float(), None, S["kout"].float(), None, n_queries=16, seed=99), 6)
            configs[name] = entry
            del L2
        torch.cuda.synchronize()

    # benchmark config 4: a 4,096-page prefix (64 layers x 64 pages) addressed through a seeded shuffled
    # block-table list, split into contiguous shards over the ranks (strong scaling).  Each rank holds only
    # its own blocks; egress of the whole shard, then ingress, for INT4_SYM and K8V4_ASYM, in chunks of
    # --prefix-chunk pages over the streams.
    prefix = None
    if args.prefix_pages > 0:
        P = args.prefix_pages
        p0, pc = sharding.shard_range(P, world, rank)
        order = np.random.default_rng(4096).permutation(P)          # list position -> global block id
        mine = order[p0:p0 + pc]
        slot = {int(b): i for i, b in enumerate(np.sort(mine))}    # global block id -> local pool slot
        table = torch.tensor([slot[int(b)] for b in mine], dtype=torch.int32, device=dev)
        pk_, pv_ = workload.kv_pages_torch(pc, workload.GQA, seed=4242 + rank, device=dev)
        ptoks = torch.from_numpy(workload.token_hashes(P, 4096)[p0:p0 + pc].copy()).to(dev)
        pseq = torch.tensor([(m["base_seq"] + (1 << 40) + p0 + i) % 2**64 for i in range(pc)],
                            dtype=torch.uint64).to(dev)
        pko = torch.empty((pc, 64, 8, 128), dtype=torch.float16, device=dev)
        pvo = torch.empty_like(pko)
        pst = torch.empty(pc, dtype=torch.int32, device=dev)
        step = args.prefix_chunk if args.prefix_chunk > 0 else pc
        chunks = [(a, min(a + step, pc)) for a in range(0, pc, step)]
        pfail = torch.zeros(max(1, len(chunks)), dtype=torch.int32, device=dev)
        pool = streams[:max(1, min(len(chunks), len(streams)))]
        prefix = {}
        for name, preset, payload in (("int4_sym", 1, EXPECTED_PAYLOAD), ("k8v4_asym", 2, 114688)):
            pblobs = torch.empty((pc, 48 + payload), dtype=torch.uint8, device=dev)

            def p_egress(ci, stream, preset=preset, payload=payload, pblobs=pblobs):
                a, b = chunks[ci]
                codec.encode_pages(pk_, pv_, ptoks[a:b], pblobs[a:b], rope_dim=64, preset=preset, rope_mode=1,
                                   expected_payload_bytes=payload, tenant_id_hash=m["tenant"],
                                   model_id_hash=m["model"], layer_id=m["layer"], head_group_id=m["head_group"],
                                   base_sequence_nonce=0, keys=keys, block_table=table[a:b],
                                   sequence_nonces=pseq[a:b], check_block_table=False, stream=stream)

            def p_ingress(ci, stream, pblobs=pblobs):
                a, b = chunks[ci]
                codec.decode_pages(pblobs[a:b], ptoks[a:b], pko, pvo, rope_dim=64, is_mla=False,
                                   tenant_id_hash=m["tenant"], model_id_hash=m["model"], layer_id=m["layer"],
                                   keys=keys, block_table=table[a:b], status=pst[a:b], any_fail=pfail[ci:ci + 1],
                                   check_block_table=False, stream=stream)

            t_e, t_i = [], []
            for rep in range(1 + args.prefix_reps):
                barrier()
                torch.cuda.synchronize()
                a0, a1 = windows(pool, 0, -(-len(chunks) // len(pool)),
                                 lambda i, s: p_egress(i, s) if i < len(chunks) else None, dev)
                b0, b1 = windows(pool, 0, -(-len(chunks) // len(pool)),
                                 lambda i, s: p_ingress(i, s) if i < len(chunks) else None, dev)
                torch.cuda.synchronize()
                if int(pfail.sum().item()):
                    raise RuntimeError("prefix sweep: a page failed verification")
                if rep:
                    t_e.append(a0.elapsed_time(a1))
                    t_i.append(b0.elapsed_time(b1))
            prefix[name] = (statistics.median(t_e), statistics.median(t_i), payload)
            del pblobs

    kt_names = list(kt)
    red = sharding.max_over_ranks([total_ms, e0.elapsed_time(e1), host_enqueue_ms, wall_ms] + [kt[k] for k in kt_names],
                                  device=dev)
    total_ms, e2e_total_ms, host_enqueue_max, wall_max = red[:4]
    kt = dict(zip(kt_names, red[4:]))
    if prefix is not None:
        flat = sharding.max_over_ranks([x for nm in prefix for x in prefix[nm][:2]], device=dev)
        prefix = {nm: (flat[2 * j], flat[2 * j + 1], prefix[nm][2]) for j, nm in enumerate(prefix)}

    if rank == 0:
        batches = K * D * world
        hot_batch = 2 * n * PAGE_HOT_BYTES
        value = hot_batch * batches / (total_ms * 1e-3) / 1e9
        peak, peak_kind = measured_peaks()
        traffic = committed_traffic()
        roof = kernel_rooflines(leg, kt, peaks, peak, traffic)
        eg = roof["egress_tile_kernel"]
        clk = clocks.summary()
        step_bytes = n * (PAGE_HOT_BYTES + BLOB_BYTES) * 2 * D    # read + write, egress + ingress, per GPU
        # integer work of a step at the all-SM rates measured in this run: both directions' keystream blocks and
        # both directions' tag-chain words (the two share the SMs' ALU pipes, so their times add); the
        # quantizers' and dequantizers' integer work is left out, so the bound is a lower bound
        chacha_step_ms = 2 * n * D * (EXPECTED_PAYLOAD // 64) / peaks["chacha20_blocks_per_s"] * 1e3
        sip_step_ms = 2 * n * D * ((32 + EXPECTED_PAYLOAD) // 8 + 1) / peaks["sip_words_per_s"] * 1e3
        alu_step_ms = chacha_step_ms + sip_step_ms
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": round(total_ms / K, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u32+f32",
            "data": "synthetic (seeded N(0,1), x15 RoPE outlier channels)",
            "config": {"workload": WORKLOAD,
                       "step": f"one window of {D} independent {n}-page batch round trips, batch j on CUDA stream j",
                       "pages_per_batch": n, "batches_per_step": D,
                       "io": "bf16 K/V in; INT4/INT8 + fp16 scales on the wire; fp16 K/V out",
                       "launch": ("CUDA graph per input set, captured from the codec API calls" if args.graphs
                                  else "codec API calls every batch"),
                       "arithmetic": "32-bit integer ARX (ChaCha20, SipHash-2-4 in 32-bit halves), "
                                     "fp32/fp16 quantization",
                       "parallelism": f"pages sharded, {world} GPU(s), no collective",
                       "l2": f"{D} input sets, {D * n * (PAGE_HOT_BYTES * 2 + BLOB_BYTES) / 1e9:.2f} GB "
                             f"working set > 126 MB L2"},
            "ms_per_batch": round(total_ms / (K * D), 5),
            "wire_gbs": round(2 * n * BLOB_BYTES * batches / (total_ms * 1e-3) / 1e9, 2),
            "single_batch": {"egress_ms": round(kt["egress_call"], 4), "ingress_ms": round(kt["ingress_call"], 4),
                             "round_trip_gbs": round(hot_batch / ((kt["egress_call"] + kt["ingress_call"]) * 1e-3) / 1e9, 2),
                             "note": "one batch in flight; bounded below by one page's tag chain per direction"},
            "roofline": {"kernel": "egress_tile_kernel (quantize + pack + ChaCha20, one CTA per 64-vec tile of a page)",
                         "bound": eg["bound"], "achieved": eg["achieved_gbs"],
                         "peak": round(eg["algorithmic_bytes"] / (max(eg["hbm_ms"], eg["alu_ms"]) * 1e-3) / 1e9, 1),
                         "unit": "GB/s", "frac": eg["frac"], "traffic": eg["traffic"],
                         "definition": ("frac = max(HBM time, ALU time) / launch time, for one 256-page launch timed with "
                                        "CUDA events in this run; peak = algorithmic bytes / max(HBM time, ALU time); "
                                        "HBM time at MEASURED_PEAKS.json hbm_gbs (" + peak_kind + f", {peak} GB/s), ALU "
                                        "time at the ChaCha20 block rate measured in this run"),
                         "int_peaks": {k: (round(v, 4) if isinstance(v, float) else v) for k, v in peaks.items()},
                         "kernels": roof},
            "path_roofline": {
                "bytes_per_step": step_bytes,
                "hbm_bound_ms": round(step_bytes / (peak * 1e9) * 1e3, 4),
                "alu_bound_ms": round(alu_step_ms, 4),
                "alu_chacha20_ms": round(chacha_step_ms, 4),
                "alu_siphash_ms": round(sip_step_ms, 4),
                "chain_sm_ms_per_step": round(D * -(-n // 128) * (kt["mac_kernel<sign>"] + kt["mac_kernel<verify>"]), 3),
                "achieved_ms_per_step": round(total_ms / K, 4),
                "frac": round(max(step_bytes / (peak * 1e9) * 1e3, alu_step_ms) / (total_ms / K), 4),
                "note": "per GPU and step: hot K/V and blob bytes of both directions (each read or written once) at "
                        "the measured copy bandwidth; ALU = ChaCha20 blocks and SipHash words of both directions at "
                        "the all-SM rates measured in this run (quantizer work not counted); frac = max(HBM, ALU) / "
                        "achieved; chain_sm_ms_per_step = SM-milliseconds the SM-exclusive tag chains hold per step"},
            "clocks": clk,
            "host": {"enqueue_ms_max_over_ranks": round(host_enqueue_max, 3), "enqueue_ms_rank0": round(host_enqueue_ms, 3),
                     "wall_ms_max_over_ranks": round(wall_max, 3), "gpu_ms_max_over_ranks": round(total_ms, 3),
                     "gpus_active": world},
            "e2e": {"value": round(hot_batch * K * DE * world / (e2e_total_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": DE * n * (PAGE_HOT_BYTES + BLOB_BYTES + 8),
                    "d2h_bytes_per_step": DE * (n * (BLOB_BYTES + PAGE_HOT_BYTES) + 4),
                    "path": f"ztcp_b200.offload.OffloadPipeline ({2 * DE} slots, {DE} host buffer sets), {K} steps of "
                            f"{DE} batches, pinned host K/V, blobs and outputs; every batch uploads its K/V and token "
                            f"hashes, encodes, downloads the blobs, uploads them again, decodes, downloads K/V and status"},
            "gpu_launches": 4 * K * D,
        }
        if configs is not None:
            line["configs"] = configs
        if prefix is not None:
            P = args.prefix_pages
            sweep = {"workload": f"cfg4: {P}-page prefix (64 layers x 64 pages of 64x8x128 GQA K+V bf16), seeded "
                                 f"shuffled block table, contiguous shards over {world} GPU(s), "
                                 f"{chunks[0][1] - chunks[0][0]}-page codec calls on up to {len(pool)} stream(s) per GPU"
                                 + (" (egress in wire order)" if chunks[0][1] - chunks[0][0] >= 1024 else ""),
                     "pages_total": P, "pages_per_gpu": -(-P // world), "hot_bytes": P * PAGE_HOT_BYTES}
            for nm, (te, ti, payload) in prefix.items():
                sweep[nm] = {"egress_ms": round(te, 4), "ingress_ms": round(ti, 4),
                             "egress_hot_gbs": round(P * PAGE_HOT_BYTES / (te * 1e-3) / 1e9, 2),
                             "ingress_hot_gbs": round(P * PAGE_HOT_BYTES / (ti * 1e-3) / 1e9, 2),
                             "round_trip_hot_gbs": round(2 * P * PAGE_HOT_BYTES / ((te + ti) * 1e-3) / 1e9, 2),
                             "wire_gbs": round(2 * P * (48 + payload) / ((te + ti) * 1e-3) / 1e9, 2)}
            sweep["note"] = ("strong scaling is bounded below by one page's tag chain per direction "
                             f"(~{kt['mac_kernel<verify>']:.2f} ms measured): per-GPU time cannot fall under it however "
                             "few pages a GPU holds")
            line["prefix_sweep"] = sweep
        if cpu_base is not None:
            line["cpu_baseline"] = cpu_base
        print(json.dumps(line), file=sys.stdout, flush=True)
    graphs.clear()  # release captured graphs before the process group goes away
    torch.cuda.synchronize()
    if world > 1:
        dist.destroy_process_group()


def main():
    args = parse_args()
    if args.impl == "reference":
        reference_arm(args)
    else:
        ours(args)


if __name__ == "__main__":
    main()
