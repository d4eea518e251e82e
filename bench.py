#!/usr/bin/env python
"""ZTCP cold-page codec benchmark on B200 -- prints one JSON line (rank 0).

Workload: the reference's headline configuration (its benchmark's config 0) -- a batch of 256 GQA pages (64 tokens x 8 KV heads x 128, separate
K and V in bf16, 256 KiB hot per page), INT4_SYM + PRESERVE_FP8, N(0,1) values with four x15 RoPE
outlier channels per head, random 256-bit ChaCha20 key, 128-bit SipHash key and 64-bit base nonce.
One step = egress (quantize, pack, encrypt, tag) of the batch followed by ingress (verify, decrypt,
dequantize) of the blobs it produced.  value = (egress + ingress) hot bytes / time, SI GB/s.

Multi-GPU: pages are independent, so every rank encodes and decodes its own 256-page batch with no
collective on the data path (weak scaling); the only collectives are the barrier and the max-over-ranks
reduction of the timings.

--impl reference times the reference codec (built from its own source into oracle/_ref) on the host
cores: one process per core, each running the reference's peak egress and peak ingress entry points on
its share of pages.
"""
from __future__ import annotations

import argparse
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
CHACHA_BLOCKS_PER_PAGE = EXPECTED_PAYLOAD // 64
SIP_WORDS_PER_PAGE = (32 + EXPECTED_PAYLOAD) // 8 + 1
METRIC = "egress+ingress hot-byte GB/s (INT4_SYM+PRESERVE_FP8 256-page GQA batch)"
WORKLOAD = "cfg0: 256-page GQA 64x8x128 INT4_SYM+PRESERVE_FP8 egress+ingress round trip"
# Integer ceilings of the codec's primitives on B200, from vlx-tee_b200/ubench/int_peaks.cu
# (profiles/int_alu_peaks.md): ChaCha20 blocks/s and SipHash words/s with every SM busy, and the
# cycles/word of one chain whose input is in registers.
CHACHA_BLOCKS_PER_S = 2.88e10
SIP_WORDS_PER_S = 4.15e11
REG_CHAIN_CYCLES_PER_WORD = 89.0


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256,
                    help="timed steps (one 256-page round trip each); the pipeline needs a few times --inflight "
                         "steps to reach steady state")
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--pages", type=int, default=256, help="pages per GPU per step")
    ap.add_argument("--sets", type=int, default=4, help="input sets (rounded up to a multiple of --inflight)")
    ap.add_argument("--inflight", type=int, default=32, help="batches in flight (CUDA streams)")
    ap.add_argument("--e2e-steps", type=int, default=256)
    ap.add_argument("--e2e-inflight", type=int, default=8,
                    help="batches in flight in the end-to-end run (host<->device copies are link-bound; a few "
                         "streams keep both copy directions busy)")
    ap.add_argument("--graphs", action="store_true",
                    help="launch each timed round trip as a CUDA graph captured from the same codec calls (one "
                         "graph per input set), instead of calling the codec API every step")
    ap.add_argument("--cpu-seconds", type=float, default=8.0, help="bounded CPU baseline sample length")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--prefix-pages", type=int, default=4096,
                    help="pages of the full-prefix sweep (benchmark config 4), split over the ranks (0 = skip)")
    ap.add_argument("--prefix-chunk", type=int, default=256, help="pages per launch in the prefix sweep")
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
    """Per-launch DRAM traffic of the dominant kernel from the committed ncu summary, if any."""
    try:
        with open(os.path.join(REPO, "profiles", "traffic.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


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
def _ref_worker(args):
    """One process: the reference's peak egress + peak ingress on `pages` pages until `seconds` pass.

    Runs the reference codec built from its own source (oracle/_ref); where that build is absent, the
    oracle's C restatement of it (same work per page, kind "port").  Returns (pages, seconds, kind)."""
    worker, pages, seconds = args
    import numpy as np

    sys.path.insert(0, os.path.join(REPO, "oracle"))
    sys.path.insert(0, os.path.join(REPO, "vlx-tee_b200"))
    import torch

    import build_ref
    from ztcp_b200 import workload

    torch.set_num_threads(1)
    k32, v32 = workload.kv_pages_np(pages, workload.GQA, seed=42 + worker)
    k = torch.from_numpy(k32).to(torch.bfloat16).half()   # the reference codec accepts fp16 only
    v = torch.from_numpy(v32).to(torch.bfloat16).half()
    m = workload.session_material(7)
    toks = torch.from_numpy(workload.token_hashes(pages, 11 + worker))
    key, mk = m["key"], m["mac_key"]
    try:
        ref = build_ref.load_module()
    except FileNotFoundError:
        ref = None
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


def reference_baseline(seconds: float, pages_per_worker: int = 8):
    import multiprocessing as mp

    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    ctx = mp.get_context("spawn")
    with ctx.Pool(cores) as pool:
        res = pool.map(_ref_worker, [(w, pages_per_worker, seconds) for w in range(cores)])
    pages = sum(r[0] for r in res)
    wall = max(r[1] for r in res)
    kind = res[0][2]
    gbs = 2 * pages * PAGE_HOT_BYTES / wall / 1e9
    what = ("reference fused_encode_cold_pages_peak_into_cpu + fused_decode_cold_pages_peak_into_cpu (oracle/_ref, "
            "the reference's own source, scalar x86-64 build, 1 thread each)" if kind == "reference" else
            "the oracle's C restatement of the reference codec, batch encode + decode (oracle/_ref absent), "
            "1 thread each")
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": kind,
            "sample": (f"{cores} processes x {pages_per_worker}-page batches for {seconds:g} s: {what}; "
                       f"{pages} pages round-tripped")}


def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    base = reference_baseline(args.cpu_seconds)
    per_step_ms = 2 * args.pages * PAGE_HOT_BYTES / (base["value"] * 1e9) * 1e3
    line = {"metric": METRIC, "value": base["value"], "unit": "GB/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_step_ms, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u32+f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "pages_per_gpu": args.pages, "host_cores": base["cores"]},
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


# ------------------------------------------------------------------------------------------------
# our arm
# ------------------------------------------------------------------------------------------------
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
        cpu_base = reference_baseline(args.cpu_seconds)

    n = args.pages
    D = max(1, args.inflight)
    n_sets = D * -(-max(args.sets, D) // D)  # a multiple of D: set j always runs on stream j % D
    m = workload.session_material(7)
    keys = capi.keys(*m["key"], *m["mac_key"])
    sets = []
    for s in range(n_sets):
        seed = 42 + 1000 * rank + s
        k, v = workload.kv_pages_torch(n, workload.GQA, seed=seed, device=dev)
        sets.append({
            "k": k, "v": v, "toks": torch.from_numpy(workload.token_hashes(n, seed)).to(dev),
            "seq": (m["base_seq"] + sharding.global_page_base(rank, s, n_sets, n)) % 2**64,
            "blobs": torch.empty((n, BLOB_BYTES), dtype=torch.uint8, device=dev),
            "kout": torch.empty((n, 64, 8, 128), dtype=torch.float16, device=dev),
            "vout": torch.empty((n, 64, 8, 128), dtype=torch.float16, device=dev),
            "status": torch.empty(n, dtype=torch.int32, device=dev),
            "fail": torch.zeros(1, dtype=torch.int32, device=dev),
        })
    streams = [torch.cuda.Stream(device=dev) for _ in range(D)]

    def egress(S):
        codec.encode_pages(S["k"], S["v"], S["toks"], S["blobs"], rope_dim=64, preset=1, rope_mode=1,
                           expected_payload_bytes=EXPECTED_PAYLOAD, tenant_id_hash=m["tenant"],
                           model_id_hash=m["model"], layer_id=m["layer"], head_group_id=m["head_group"],
                           base_sequence_nonce=S["seq"], keys=keys)

    def ingress(S):
        codec.decode_pages(S["blobs"], S["toks"], S["kout"], S["vout"], rope_dim=64, is_mla=False,
                           tenant_id_hash=m["tenant"], model_id_hash=m["model"], layer_id=m["layer"], keys=keys,
                           status=S["status"], any_fail=S["fail"])

    def verify(S):
        codec.verify_pages(S["blobs"], S["toks"], num_tokens=64, num_heads=8, head_dim=128, rope_dim=64,
                           is_mla=False, tenant_id_hash=m["tenant"], model_id_hash=m["model"], layer_id=m["layer"],
                           keys=keys, status=S["status"], any_fail=S["fail"])

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def streamed(first, count, step_fn, pool=None):
        """Steps first..first+count-1 round-robin on `pool` (default: the D streams), bracketed by events on
        the current stream."""
        pool = streams if pool is None else pool
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        main = torch.cuda.current_stream(dev)
        start.record(main)
        for st in pool:
            st.wait_event(start)
        for i in range(first, first + count):
            with torch.cuda.stream(pool[i % len(pool)]):
                step_fn(i)
        for st in pool:
            done = torch.cuda.Event()
            done.record(st)
            main.wait_event(done)
        end.record(main)
        return start, end

    def round_trip(i):
        S = sets[i % n_sets]
        egress(S)
        ingress(S)

    def check(what):
        bad = sum(int(S["fail"].item()) for S in sets)
        if bad:
            raise RuntimeError(f"{what}: a round trip failed verification")

    streamed(0, args.warmup, round_trip)
    torch.cuda.synchronize()
    check("warm-up")

    step_fn = round_trip
    graphs = []
    if args.graphs:
        # the same egress + ingress calls, captured once per input set on the set's stream; a timed step
        # replays its set's graph (same kernels and work, one launch call instead of two API calls)
        for j in range(n_sets):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=streams[j % D]):
                round_trip(j)
            graphs.append(g)
        torch.cuda.synchronize()

        def step_fn(i):
            graphs[i % n_sets].replay()

        streamed(0, args.warmup, step_fn)
        torch.cuda.synchronize()
        check("graph warm-up")

    K = args.steps
    with ClockSampler(local) as clocks:
        barrier()
        torch.cuda.synchronize()
        h0 = time.perf_counter()
        t0, t1 = streamed(args.warmup, K, step_fn)
        host_enqueue_ms = (time.perf_counter() - h0) * 1e3
        torch.cuda.synchronize()
        barrier()
    total_ms = t0.elapsed_time(t1)
    check("timed region")

    # single-batch latency: the same round trip with one batch in flight
    L = max(3, min(K, 8))
    lat = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(L)]
    for i in range(L):
        S = sets[i % n_sets]
        lat[i][0].record()
        egress(S)
        lat[i][1].record()
        ingress(S)
        lat[i][2].record()
    # dominant kernel (SipHash chain): verify-only launches, timed live with events
    mac_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(L)]
    for i in range(L):
        S = sets[i % n_sets]
        mac_ev[i][0].record()
        verify(S)
        mac_ev[i][1].record()
    torch.cuda.synchronize()
    check("latency run")
    egress_ms = statistics.median(e[0].elapsed_time(e[1]) for e in lat)
    ingress_ms = statistics.median(e[1].elapsed_time(e[2]) for e in lat)
    mac_ms = statistics.median(a.elapsed_time(b) for a, b in mac_ev)

    # end to end through the public API with pinned host buffers: every step uploads its K/V and token
    # hashes, encodes, downloads the blobs, uploads them again, decodes, and downloads K/V and the status.
    DE = max(1, min(args.e2e_inflight, n_sets))
    host = []
    for j in range(DE):
        S = sets[j]
        host.append({"k": S["k"].cpu().pin_memory(), "v": S["v"].cpu().pin_memory(),
                     "toks": S["toks"].cpu().pin_memory(),
                     "blobs": torch.empty((n, BLOB_BYTES), dtype=torch.uint8).pin_memory(),
                     "kout": torch.empty((n, 64, 8, 128), dtype=torch.float16).pin_memory(),
                     "vout": torch.empty((n, 64, 8, 128), dtype=torch.float16).pin_memory(),
                     })

    # through ztcp_b200.offload.OffloadPipeline: each step's egress (upload K/V -> encode -> download blobs) and
    # ingress (upload blobs -> decode -> download K/V + status) on the pipeline's slots; a step's egress waits
    # for the ingress that last used the same host buffers.
    pipe = offload.OffloadPipeline(dev, slots=2 * DE)
    last_ingress = [None] * DE

    def e2e_step(i):
        H, S = host[i % DE], sets[i % DE]
        t = pipe.egress(H["k"], H["v"], H["toks"], H["blobs"], rope_dim=64, preset=1, rope_mode=1,
                        expected_payload_bytes=EXPECTED_PAYLOAD, tenant_id_hash=m["tenant"], model_id_hash=m["model"],
                        layer_id=m["layer"], head_group_id=m["head_group"], base_sequence_nonce=S["seq"], keys=keys,
                        after=last_ingress[i % DE])
        last_ingress[i % DE] = pipe.ingress(H["blobs"], H["toks"], H["kout"], H["vout"], rope_dim=64, is_mla=False,
                                            tenant_id_hash=m["tenant"], model_id_hash=m["model"], layer_id=m["layer"],
                                            keys=keys, after=t)

    E = max(4 * DE, args.e2e_steps)
    for i in range(DE):
        e2e_step(i)
    for tk in last_ingress:
        tk.wait()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for sl in pipe._slots:
        sl.stream.wait_event(e0)
    for i in range(DE, DE + E):
        e2e_step(i)
    for sl in pipe._slots:
        torch.cuda.current_stream(dev).wait_event(sl.idle)
    e1.record()
    torch.cuda.synchronize()
    for tk in last_ingress:
        tk.wait()  # raises the reference's error if any page failed
    if not torch.equal(host[0]["kout"], sets[0]["kout"].cpu()):
        raise RuntimeError("end-to-end output differs from the device-resident run")

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
        pk, pv = workload.kv_pages_torch(pc, workload.GQA, seed=4242 + rank, device=dev)
        ptoks = torch.from_numpy(workload.token_hashes(P, 4096)[p0:p0 + pc].copy()).to(dev)
        pseq = torch.tensor([(m["base_seq"] + (1 << 40) + p0 + i) % 2**64 for i in range(pc)],
                            dtype=torch.uint64).to(dev)
        pko = torch.empty((pc, 64, 8, 128), dtype=torch.float16, device=dev)
        pvo = torch.empty_like(pko)
        pst = torch.empty(pc, dtype=torch.int32, device=dev)
        chunks = [(a, min(a + args.prefix_chunk, pc)) for a in range(0, pc, args.prefix_chunk)]
        pfail = torch.zeros(max(1, len(chunks)), dtype=torch.int32, device=dev)
        pool = streams[:max(1, min(len(chunks), len(streams)))]
        prefix = {}
        for name, preset, payload in (("int4_sym", 1, EXPECTED_PAYLOAD), ("k8v4_asym", 2, 114688)):
            pblobs = torch.empty((pc, 48 + payload), dtype=torch.uint8, device=dev)

            def p_egress(ci, preset=preset, payload=payload, pblobs=pblobs):
                a, b = chunks[ci]
                codec.encode_pages(pk, pv, ptoks[a:b], pblobs[a:b], rope_dim=64, preset=preset, rope_mode=1,
                                   expected_payload_bytes=payload, tenant_id_hash=m["tenant"],
                                   model_id_hash=m["model"], layer_id=m["layer"], head_group_id=m["head_group"],
                                   base_sequence_nonce=0, keys=keys, block_table=table[a:b],
                                   sequence_nonces=pseq[a:b], check_block_table=False)

            def p_ingress(ci, pblobs=pblobs):
                a, b = chunks[ci]
                codec.decode_pages(pblobs[a:b], ptoks[a:b], pko, pvo, rope_dim=64, is_mla=False,
                                   tenant_id_hash=m["tenant"], model_id_hash=m["model"], layer_id=m["layer"],
                                   keys=keys, block_table=table[a:b], status=pst[a:b], any_fail=pfail[ci:ci + 1],
                                   check_block_table=False)

            t_e, t_i = [], []
            for rep in range(1 + args.prefix_reps):
                barrier()
                torch.cuda.synchronize()
                a0, a1 = streamed(0, len(chunks), p_egress, pool)
                b0, b1 = streamed(0, len(chunks), p_ingress, pool)
                torch.cuda.synchronize()
                if int(pfail.sum().item()):
                    raise RuntimeError("prefix sweep: a page failed verification")
                if rep:
                    t_e.append(a0.elapsed_time(a1))
                    t_i.append(b0.elapsed_time(b1))
            prefix[name] = (statistics.median(t_e), statistics.median(t_i), payload)
            del pblobs

    total_ms, egress_ms, ingress_ms, mac_ms, e2e_total_ms = sharding.max_over_ranks(
        [total_ms, egress_ms, ingress_ms, mac_ms, e0.elapsed_time(e1)], device=dev)
    if prefix is not None:
        flat = sharding.max_over_ranks([x for nm in prefix for x in prefix[nm][:2]], device=dev)
        prefix = {nm: (flat[2 * j], flat[2 * j + 1], prefix[nm][2]) for j, nm in enumerate(prefix)}

    if rank == 0:
        hot_step = 2 * n * PAGE_HOT_BYTES * world
        wire_step = 2 * n * BLOB_BYTES * world
        value = hot_step * K / (total_ms * 1e-3) / 1e9
        peak, peak_kind = measured_peaks()
        mac_bytes = n * BLOB_BYTES
        achieved = mac_bytes / (mac_ms * 1e-3) / 1e9
        traffic = committed_traffic().get("mac_kernel<verify>", {}).get("dram_bytes_per_launch")
        clk = clocks.summary()
        mhz = clk.get("sm_mhz") or 1965.0
        cycles_per_word = mac_ms * 1e-3 * mhz * 1e6 / SIP_WORDS_PER_PAGE
        step_bytes = n * (PAGE_HOT_BYTES + BLOB_BYTES) * 2 * world   # read + write, egress + ingress
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": round(total_ms / K, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u32+f32",
            "data": "synthetic (seeded N(0,1), x15 RoPE outlier channels)",
            "config": {"workload": WORKLOAD,
                       "pages_per_gpu": n, "batches_in_flight": D,
                       "io": "bf16 K/V in; INT4/INT8 + fp16 scales on the wire; fp16 K/V out",
                       "launch": ("CUDA graph per input set, captured from the codec API calls" if args.graphs
                                  else "codec API calls every step"),
                       "arithmetic": "32-bit integer ARX (ChaCha20, SipHash-2-4 in 32-bit halves), "
                                     "fp32/fp16 quantization",
                       "parallelism": f"pages sharded, {world} GPU(s), no collective",
                       "l2": f"{n_sets} input sets, {n_sets * n * (PAGE_HOT_BYTES * 2 + BLOB_BYTES) / 1e9:.2f} GB "
                             f"working set > 126 MB L2"},
            "wire_gbs": round(wire_step * K / (total_ms * 1e-3) / 1e9, 2),
            "single_batch": {"egress_ms": round(egress_ms, 4), "ingress_ms": round(ingress_ms, 4),
                             "round_trip_gbs": round(hot_step / ((egress_ms + ingress_ms) * 1e-3) / 1e9, 2),
                             "egress_gbs": round(n * world * PAGE_HOT_BYTES / (egress_ms * 1e-3) / 1e9, 2),
                             "ingress_gbs": round(n * world * PAGE_HOT_BYTES / (ingress_ms * 1e-3) / 1e9, 2)},
            "roofline": {"kernel": "mac_kernel<verify> (SipHash-2-4-128 chain, one lane per page)", "bound": "hbm",
                         "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 5), "traffic": traffic,
                         "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})",
                         "algorithmic_bytes_per_launch": mac_bytes, "launch_ms": round(mac_ms, 4),
                         "chain": {"cycles_per_word": round(cycles_per_word, 1),
                                   "register_chain_cycles_per_word": REG_CHAIN_CYCLES_PER_WORD,
                                   "frac_of_register_chain": round(REG_CHAIN_CYCLES_PER_WORD / cycles_per_word, 3),
                                   "note": "one chain = one page; the floor is the same SipHash code with its input in "
                                           "registers, ALU-pipe bound (profiles/int_alu_peaks.md)"}},
            "path_roofline": {
                "bytes_per_step": step_bytes,
                "hbm_bound_ms": round(step_bytes / (peak * 1e9) * 1e3, 4),
                "alu_bound_ms": round(2 * n * (CHACHA_BLOCKS_PER_PAGE / CHACHA_BLOCKS_PER_S
                                               + SIP_WORDS_PER_PAGE / SIP_WORDS_PER_S) * 1e3, 4),
                "achieved_ms_per_step": round(total_ms / K, 4),
                "frac_hbm": round(step_bytes / (peak * 1e9) * 1e3 / (total_ms / K), 4),
                "note": "alu bound = ChaCha20 keystream at its all-SM rate + SipHash words at the all-SM chain "
                        "rate (profiles/int_alu_peaks.md); per GPU"},
            "clocks": clk,
            "host_enqueue_ms": round(host_enqueue_ms, 3),
            "e2e": {"value": round(hot_step * E / (e2e_total_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": n * (PAGE_HOT_BYTES + BLOB_BYTES + 8),
                    "d2h_bytes_per_step": n * (BLOB_BYTES + PAGE_HOT_BYTES) + 4,
                    "path": f"ztcp_b200.offload.OffloadPipeline ({2 * DE} slots, {DE} host buffer sets), {E} steps, "
                            f"pinned host K/V, blobs and outputs; every step uploads its K/V and token hashes, "
                            f"encodes, downloads the blobs, uploads them again, decodes, downloads K/V and status"},
            "gpu_launches": 4 * K,
        }
        if prefix is not None:
            P = args.prefix_pages
            sweep = {"workload": f"cfg4: {P}-page prefix (64 layers x 64 pages of 64x8x128 GQA K+V bf16), seeded "
                                 f"shuffled block table, contiguous shards over {world} GPU(s), {args.prefix_chunk}-page "
                                 f"launches on up to {len(pool)} streams per GPU",
                     "pages_total": P, "pages_per_gpu": -(-P // world), "hot_bytes": P * PAGE_HOT_BYTES}
            for nm, (te, ti, payload) in prefix.items():
                sweep[nm] = {"egress_ms": round(te, 4), "ingress_ms": round(ti, 4),
                             "egress_hot_gbs": round(P * PAGE_HOT_BYTES / (te * 1e-3) / 1e9, 2),
                             "ingress_hot_gbs": round(P * PAGE_HOT_BYTES / (ti * 1e-3) / 1e9, 2),
                             "round_trip_hot_gbs": round(2 * P * PAGE_HOT_BYTES / ((te + ti) * 1e-3) / 1e9, 2),
                             "wire_gbs": round(2 * P * (48 + payload) / ((te + ti) * 1e-3) / 1e9, 2)}
            sweep["note"] = ("strong scaling is bounded below by one page's tag chain per direction "
                             f"(~{mac_ms:.2f} ms measured): per-GPU time cannot fall under it however few pages a GPU holds")
            line["prefix_sweep"] = sweep
        if cpu_base is not None:
            line["cpu_baseline"] = cpu_base
        print(json.dumps(line))
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
