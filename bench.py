"""bench.py - KV handoff GB/s and p50/p99 ms per 32K-token sequence on B200 (the BASELINE.json metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference] [--tokens T]

A step is one handoff of one sequence's whole cache: the K/V of the 12 full-attention layers (fp16, 2 KV
heads x head_dim 256, 256-token blocks at seed-random pool slots) plus the 36 linear-attention layers'
recurrent + conv state (fp32) plus the token ids.  Bytes per sequence B(T) = 24,576*T + 79,036,416 + 4*T.

  N = 1   config 2(a): pool -> pool on one GPU, source and destination block tables independent
          seed-random permutations of two 4,096-block pools.  ONE skv_copy launch per step.
  N > 1   config 3: N/2 prefill -> decode pairs (even rank -> next odd rank); by default the decode GPU pulls
          the sequence straight into its own pool over NVLink through CUDA-IPC peer pointers in ONE launch
          (skv_copy_gated: it waits for the prefill GPU's READY flag and releases DONE on the prefill GPU
          itself, both bounded); --p2p pull / push / push-tma select the others.  At N = 2 the line adds config
          3's length sweep and the split-role record, at N = 4 config 4 (fan-out), at N = 8 config 5.
  e2e     park (pool -> pinned host image) + resume (host image -> another pool) through the C ABI, host
          copies inside the timed region: the host-mediated handoff a user of the reference's park path gets.
  --impl reference
          the reference's own host park/resume (conversation_snapshot_save + _restore from
          oracle/_ref/libstrata_ref.so, cudaMemcpy link-wrapped to memcpy) on the host cores.

One JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "strata-concurrent_b200"))

import handoff_schedule  # noqa: E402
import skv  # noqa: E402

METRIC = "KV handoff GB/s & p50/p99 ms per 32K-token sequence"
UNIT = "GB/s"
PEAKS_FILE = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_HBM_GBS = 6650.0
NVLINK_PEER_COPY_GBS = 770.0     # an earlier measurement of the pool's peer copy per direction (900 nominal): the
                                 # rate used only where a line has no same-run probe (the standalone scenarios)


def link_rate(probe: dict | None) -> tuple:
    """(GB/s per direction, what it is) for a line's NVLink roofline: the same-run copy-engine probe (pull direction)
    when the run measured one, else the earlier figure."""
    if probe:
        return probe["pull_gbs_median"], "peer copy of this run (peer_copy_probe, pull direction)"
    return NVLINK_PEER_COPY_GBS, "earlier measured peer copy (770 GB/s; no probe in this run)"
PROFILE_TRAFFIC = os.path.join(ROOT, "profiles", "traffic.json")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--tokens", type=int, default=32768)
    ap.add_argument("--engine", default="tma", choices=["tma", "vec"])
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--pool-blocks", type=int, default=4096, help="slots per pool (the configs use 4,096)")
    ap.add_argument("--p2p", default="pull-gated", choices=["pull", "pull-gated", "push", "push-tma"],
                    help="N > 1: the decode GPU pulls (TMA loads of peer memory; pull-gated: the READY wait and the "
                         "DONE release inside the copy launch, skv_copy_gated), or the prefill GPU pushes (vector "
                         "engine remote stores, or TMA bulk stores to peer memory)")
    ap.add_argument("--scenario", default="auto", choices=["auto", "pairs", "sweep", "fanout", "mixed", "p2p-local"],
                    help="N > 1: pairs = N/2 prefill->decode pairs; fanout = one prefill to N-1 decodes (config 4); "
                         "mixed = N/2 prefill + N/2 decode GPUs, 64 log-uniform sequences, host parks (config 5); "
                         "auto = pairs, plus config 3's sweep and the split-role record at N = 2, config 4 at N = 4 "
                         "and config 5 at N = 8 embedded in the same line; sweep = pairs and config 3's sweep only")
    ap.add_argument("--chunk-mb", type=int, default=16,
                    help="fan-out chain: pipeline chunk size (16 / 32 / 64 MB measured 1,936 / 1,910 / 1,869 GB/s)")
    ap.add_argument("--mixed-order", default="phased",
                    choices=["phased", "phased-tail", "phased-unfused", "per-source", "serial"],
                    help="config 5: a decode GPU pulls on one stream per source prefill GPU, or one sequence at a "
                         "time, or in port-exclusive phases (phased_schedule; back-to-back runs from one source "
                         "fused into one launch unless phased-unfused; phased-tail: the last, small phases without "
                         "hand-over waits, on one stream per source)")
    ap.add_argument("--handover", default="gated", choices=["launch", "gated"],
                    help="config 5, phased orders: a run waits for its source's hand-over and signals the next "
                         "reader inside its copy launch (gated, the default: skv_copy_gated; a run's time then "
                         "includes its wait; 8 GPUs: 2,411 vs 2,377 GB/s) or with launches of their own around "
                         "its copy (launch)")
    ap.add_argument("--tuning", default=None,
                    help="copy-engine geometry for this run, STAGES,TILE_BYTES,TMA_CTAS_PER_SM[,VEC_CTAS_PER_SM] "
                         "(skv_set_copy_tuning); default: the library's")
    ap.add_argument("--relay-mb", type=int, default=RELAY_CHUNK_BYTES >> 20, help="N = 1 e2e relay: piece size")
    ap.add_argument("--relay-lanes", type=int, default=2, choices=[1, 2],
                    help="N = 1 e2e relay: streams per direction the pieces alternate over")
    ap.add_argument("--relay-ramp", default="off", choices=["on", "off"],
                    help="N = 1 e2e relay: graded pieces at both ends of the stream (on) or per-segment pieces (off)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-length-sweep", action="store_true",
                    help="N = 1: leave out the 1K / 4K / 128K pool->pool lines the headline line carries")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--timeline", action="store_true",
                    help="config 5, phased order: add every decode GPU's per-run timeline of the last timed step "
                         "(start and end from the step's start, bytes, source, phase, whether it waited)")
    ap.add_argument("--sweep", action="store_true",
                    help="with --impl reference: the reference's host path phase by phase (save, encode, decode, "
                         "restore) on one pinned core at 1K / 4K / 32K / 64K / 128K tokens, one JSON line per length")
    return ap.parse_args()


def peaks() -> tuple:
    try:
        with open(PEAKS_FILE) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def traffic_for(kernel: str, workload: str):
    try:
        with open(PROFILE_TRAFFIC) as f:
            return json.load(f).get(f"{kernel}:{workload}")
    except Exception:
        return None


class Clocks:
    """SM clock and clock-event reasons sampled DURING the timed region: NVML polled from a thread every
    ~1 ms (a 32K handoff step is ~0.3 ms, far below nvidia-smi's sampling interval)."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4,
               "hw_power_brake_slowdown": 0x80}

    def __init__(self, cuda_index: int, sample: bool = True):
        self.cuda_index = cuda_index
        self.sample = sample   # False: no polling thread in this process (the other ranks of a multi-GPU run)
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None

    def _handle(self, nv):
        import torch
        p = torch.cuda.get_device_properties(self.cuda_index)
        bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        try:
            return nv.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(self.cuda_index)

    def __enter__(self):
        if not self.sample:
            return self
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = self._handle(nv)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        except Exception:
            return self

        def poll():
            while not self._stop.is_set():
                try:
                    self.samples.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                                         int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))))
                except Exception:
                    pass
                time.sleep(0.001)

        self._thread = threading.Thread(target=poll, daemon=True)
        self._thread.start()
        time.sleep(0.003)
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"], "samples": 0}
        sm = [c for c, _ in self.samples]
        reasons = sorted({n for _, bits in self.samples for n, b in self.REASONS.items() if bits & b})
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples), "source": "NVML, 1 ms polling during the timed region"}


# ------------------------------------------------------------------------------------------------ workloads

class SeqOnGpu:
    """One sequence resident in a pool on the current GPU, filled with fp16 N(0,1) K/V, fp32 N(0,0.02) state
    and uniform ids (torch RNG on the device).

    ipc=False: the pool and the state are torch tensors (single-process use).
    ipc=True:  the pool and a state arena (GDN rows | ids | flags, `state_layout`) are cudaMalloc'd by the
               library, so CUDA IPC can export their base addresses to the peer process."""

    def __init__(self, torch, kg: skv.KvGeometry, tokens: int, n_blocks: int, seed: int, fill: bool, ipc: bool = False):
        self.kg, self.tokens, self.ipc = kg, tokens, ipc
        dev = torch.cuda.current_device()
        gen = torch.Generator(device="cuda").manual_seed(seed)
        ids_words = ((4 * tokens + 15) // 16) * 4
        if ipc:
            lay = state_layout(kg, tokens)
            self.pool_mem = None
            self.pool = skv.Pool(dev, n_blocks, kg.block_bytes)
            self.state = skv.Pool(dev, 1, lay["bytes"])
            self.state_bytes = lay["bytes"]
            self.gdn, self.ids = self.state.base, self.state.base + lay["ids"]
            self.flag = self.state.base + lay["flag"]
            zero = torch.zeros(lay["bytes"], dtype=torch.uint8, device="cuda")
            skv.copy([skv.segment(zero, self.state.base, lay["bytes"])], skv.COPY_VEC)
            if fill:
                chunk = 256 << 20
                total = n_blocks * kg.block_bytes
                for at in range(0, total, chunk):
                    n = min(chunk, total - at)
                    r = torch.randn(n // 2, generator=gen, device="cuda", dtype=torch.float16)
                    skv.copy([skv.segment(r, self.pool.base + at, n)], skv.COPY_VEC)
                    torch.cuda.synchronize()
                gdn = torch.randn(kg.gdn_bytes // 4, generator=gen, device="cuda") * 0.02
                ids = torch.randint(0, 151936, (ids_words,), generator=gen, device="cuda", dtype=torch.int32)
                skv.copy([skv.segment(gdn, self.gdn, kg.gdn_bytes), skv.segment(ids, self.ids, 4 * ids_words)],
                         skv.COPY_VEC)
                torch.cuda.synchronize()
        else:
            self.pool_mem = torch.empty(n_blocks * kg.block_bytes, dtype=torch.uint8, device="cuda")
            self.pool = skv.Pool(dev, n_blocks, kg.block_bytes, memory=self.pool_mem)
            if fill:
                self.pool_mem.view(torch.float16).copy_(
                    torch.randn(self.pool_mem.numel() // 2, generator=gen, device="cuda", dtype=torch.float16))
            self.gdn = (torch.randn(kg.gdn_bytes // 4, generator=gen, device="cuda") * 0.02 if fill
                        else torch.zeros(kg.gdn_bytes // 4, device="cuda"))
            self.ids = (torch.randint(0, 151936, (ids_words,), generator=gen, device="cuda", dtype=torch.int32)
                        if fill else torch.zeros(ids_words, device="cuda", dtype=torch.int32))
        self.pool.scramble(seed)
        nb = kg.blocks(tokens)
        self.blocks = np.stack([self.pool.alloc(nb) for _ in range(kg.n_qsa)])
        self.host_tables = skv.PooledSequence.host_tables(kg, self.blocks)
        self.tables = torch.from_numpy(self.host_tables.reshape(-1).copy()).cuda()
        self.ps = skv.PooledSequence(kg, self.pool, tokens, kg.n_qsa, self.blocks, self.tables, self.gdn, self.ids)

    def logical(self, torch):
        """Every layer's K/V pages read back through this sequence's own table (for the parity check)."""
        pages = self.kg.pages(self.tokens)
        tab = self.tables.view(self.kg.n_qsa, 2, -1)[:, :, :pages].long().reshape(-1)
        return self.pool_mem.view(-1, self.kg.page_bytes)[tab]

    def packed(self, torch):
        """The whole sequence packed through its table by the gather kernel (K/V, GDN rows, ids)."""
        off = skv.image_offsets(self.kg, self.tokens, self.kg.n_qsa)
        image = torch.zeros(off["total"], dtype=torch.uint8, device="cuda")
        skv.copy(skv.pack_segments(self.ps, image), skv.COPY_TMA)
        torch.cuda.synchronize()
        return image


def percentiles(ms: list) -> tuple:
    a = np.asarray(ms)
    return float(np.percentile(a, 50)), float(np.percentile(a, 99))


class quiet_gc:
    """Python's cyclic garbage collector paused for a timed region (a collection of a large heap can stall the
    launching thread for milliseconds, and a stalled rank stalls its pair); collected once before and after."""

    def __enter__(self):
        import gc
        gc.collect()
        self.was = gc.isenabled()
        gc.disable()
        return self

    def __exit__(self, *a):
        import gc
        if self.was:
            gc.enable()


def time_steps(torch, stream, fn, steps: int, warmup: int) -> tuple:
    """W warm-up calls, then K timed calls bracketed by synchronize; per-step CUDA events on `stream`."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    with quiet_gc():
        ev[0].record(stream)
        for i in range(steps):
            fn()
            ev[i + 1].record(stream)
        torch.cuda.synchronize()
    per = [ev[i].elapsed_time(ev[i + 1]) for i in range(steps)]
    return ev[0].elapsed_time(ev[steps]), per


def pcie_probe(torch, nbytes: int = 1 << 30, reps: int = 5) -> dict:
    """The box's pinned-host copy rates (the park/resume roofline): one direction at a time, then both at once
    on two streams.  Median of `reps`, CUDA events."""
    host_a = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    host_b = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    dev_a = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    dev_b = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()

    def timed(fn):
        out = []
        for _ in range(reps + 1):
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s1)
            s2.wait_event(e0)
            fn()
            done = torch.cuda.Event()
            done.record(s2)
            s1.wait_event(done)
            e1.record(s1)
            torch.cuda.synchronize()
            out.append(e0.elapsed_time(e1))
        return float(np.median(out[1:]))

    def d2h():
        with torch.cuda.stream(s1):
            host_a.copy_(dev_a, non_blocking=True)

    def h2d():
        with torch.cuda.stream(s1):
            dev_b.copy_(host_b, non_blocking=True)

    def both():
        with torch.cuda.stream(s1):
            host_a.copy_(dev_a, non_blocking=True)
        with torch.cuda.stream(s2):
            dev_b.copy_(host_b, non_blocking=True)

    t_d2h, t_h2d, t_both = timed(d2h), timed(h2d), timed(both)
    gb = nbytes / 1e9
    return {"d2h_gbs": round(gb / (t_d2h / 1e3), 2), "h2d_gbs": round(gb / (t_h2d / 1e3), 2),
            "both_directions_gbs": round(2 * gb / (t_both / 1e3), 2),
            "probe": f"{nbytes >> 20} MiB pinned <-> device copies, median of {reps}"}


RELAY_CHUNK_BYTES = 32 << 20


def relay_pieces(park_segs: list, resume_segs: list, piece_bytes: int = RELAY_CHUNK_BYTES, ramp: bool = False) -> list:
    """A pipelined host relay's pieces, as (park segments, resume segments) pairs in order.  Without `ramp`: every
    park segment and its resume twin cut into the same pieces of at most `piece_bytes`.  With `ramp`: the whole
    byte stream (the segments back to back) cut at graded points - pieces of 1/16, 1/16, 1/8, 1/4 and 1/2 of
    `piece_bytes` at the start, whole pieces in the middle, the same ramp reversed at the end - so the resume
    direction starts after a small first piece and the park direction's last piece is small too (the pipeline's
    fill and drain), and no piece is a segment's short leftover."""
    if not ramp:
        return [([p], [r]) for ps, rs in zip(park_segs, resume_segs)
                for p, r in zip(skv.split_segment(ps, piece_bytes), skv.split_segment(rs, piece_bytes))]
    total = sum(sg.bytes for sg in park_segs)
    steps = [piece_bytes // 16, piece_bytes // 16, piece_bytes // 8, piece_bytes // 4, piece_bytes // 2]
    head, cuts, at = [], [0], 0
    for n in steps:
        at += n
        head.append(at)
    if 2 * head[-1] >= total:     # too short to ramp both ways: whole pieces only
        cuts += list(range(piece_bytes, total, piece_bytes))
    else:
        tail = [total - c for c in reversed(head)]
        span = tail[0] - head[-1]                       # the middle, in equal pieces of at most piece_bytes
        n = -(-span // piece_bytes)
        cuts += head + [head[-1] + (span * i // n) // 65536 * 65536 for i in range(1, n)] + tail
    cuts.append(total)
    out = []
    for a, b in zip(cuts, cuts[1:]):
        pp, rp = skv.slice_segments(park_segs, a, b), skv.slice_segments(resume_segs, a, b)
        if pp:
            out.append((pp, rp))
    return out


def e2e_park_resume(torch, kg, src: SeqOnGpu, dst: SeqOnGpu, steps: int, warmup: int, side_steps: int,
                    piece_bytes: int = RELAY_CHUNK_BYTES, lanes: int = 1, ramp: bool = False) -> dict:
    """Host-mediated handoff through the C ABI: park to pinned host, resume into another table.

    relay (the reported e2e, fixed in advance): skv_park and skv_resume chunk by chunk on two streams - the park
           of chunk c+1 (device -> host) runs while the resume of chunk c (host -> device) runs, so both PCIe
           directions are busy at once.  Timed over `steps` steps.  lanes = 2 alternates the pieces over two
           streams per direction, so piece c+1's gather kernel runs beside piece c's device-to-host copy (and piece
           c's scatter beside piece c+1's host-to-device copy) instead of holding the copy engine idle.  ramp: graded
           pieces at both ends of the stream (relay_pieces).
    staged / direct (extra keys): one skv_park then one skv_resume of the whole sequence, staged through device
           memory or with the kernel reading and writing mapped host memory.  Timed over `side_steps` steps."""
    off = skv.image_offsets(kg, src.tokens, kg.n_qsa)
    host = skv.HostBuffer(off["total"])
    staging = torch.empty(off["total"] + 256 * 64, dtype=torch.uint8, device="cuda")
    staging_b = torch.empty(off["total"] + 256 * 64, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()
    side = torch.cuda.Stream()
    park_streams = [stream] + [torch.cuda.Stream() for _ in range(lanes - 1)]
    resume_streams = [side] + [torch.cuda.Stream() for _ in range(lanes - 1)]
    park_segs = skv.pack_segments(src.ps, host.ptr)
    resume_segs = skv.unpack_segments(host.ptr, dst.ps)
    chunks = relay_pieces(park_segs, resume_segs, piece_bytes, ramp)
    chunk_off = []
    at = 0
    for pp, _ in chunks:
        chunk_off.append(at)
        at += sum((sg.bytes + 255) & ~255 for sg in pp)
    parked = [torch.cuda.Event() for _ in chunks]
    resumed = [torch.cuda.Event() for _ in resume_streams]
    parity, modes, results = {}, {}, {}
    b = kg.metric_bytes(src.tokens)
    for mode, name, n_steps in ((skv.PARK_STAGED, "relay", steps), (skv.PARK_STAGED, "staged", side_steps),
                                (skv.PARK_DIRECT, "direct", side_steps)):
        if name == "relay":
            def step():
                for ps in park_streams[1:]:
                    ps.wait_stream(stream)   # the previous step (and its resumes) finished before any park
                for k, (pp, rp) in enumerate(chunks):
                    ps, rs = park_streams[k % lanes], resume_streams[k % lanes]
                    a = staging.data_ptr() + chunk_off[k]
                    skv.park(pp, mode, a, staging.numel() - chunk_off[k], ps)
                    parked[k].record(ps)
                    rs.wait_event(parked[k])
                    b2 = staging_b.data_ptr() + chunk_off[k]
                    skv.resume(rp, mode, b2, staging_b.numel() - chunk_off[k], rs)
                for ev_r, rs in zip(resumed, resume_streams):
                    ev_r.record(rs)
                    stream.wait_event(ev_r)
        else:
            def step():
                skv.park(park_segs, mode, staging, staging.numel(), stream)
                skv.resume(resume_segs, mode, staging, staging.numel(), stream)
        dst.pool_mem.zero_()
        dst.gdn.zero_()
        dst.ids.zero_()
        total, per = time_steps(torch, stream, step, n_steps, warmup)
        parity[name] = (bool(torch.equal(dst.logical(torch), src.logical(torch))) and bool(torch.equal(dst.gdn, src.gdn))
                        and bool(torch.equal(dst.ids, src.ids)))
        results[name] = {"value": b * n_steps / (total / 1e3) / 1e9, "ms_per_step": total / n_steps, "steps": n_steps,
                         "p50_ms": percentiles(per)[0], "p99_ms": percentiles(per)[1],
                         # bytes over PCIe in both directions together (B down + B up per step) per second
                         "pcie_gbs_both_directions": 2 * b * n_steps / (total / 1e3) / 1e9}
        modes[name] = round(results[name]["value"], 3)
    host.close()
    r = results["relay"]
    return {"value": round(r["value"], 3), "unit": UNIT, "h2d_bytes_per_step": b, "d2h_bytes_per_step": b,
            "mode": "relay", "piece_mb": piece_bytes >> 20, "lanes": lanes, "ramp": ramp, "pieces": len(chunks),
            "steps": r["steps"], "p50_ms": round(r["p50_ms"], 3), "p99_ms": round(r["p99_ms"], 3),
            "pcie_gbs_both_directions": round(r["pcie_gbs_both_directions"], 3),
            "other_modes_gbs": {k: v for k, v in modes.items() if k != "relay"}, "other_modes_steps": side_steps,
            "api": f"skv_park + skv_resume (C ABI), pinned host image, {piece_bytes >> 20} MB pieces"
                   f"{' (graded at both ends)' if ramp else ''} over {lanes} stream(s) per direction",
            "parity": parity["relay"], "parity_by_mode": parity}


def host_info() -> dict:
    """The host the CPU arms ran on: its CPU model and how many cores it offers this process."""
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            model = next((ln.split(":", 1)[1].strip() for ln in f if ln.startswith("model name")), None)
    except OSError:
        pass
    try:
        usable = len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        usable = os.cpu_count()
    return {"cpu_model": model, "cores_total": os.cpu_count(), "cores_usable": usable}


def cpu_baseline(tokens: int, reps: int = 20) -> dict | None:
    """The reference's own host park/resume on ONE host core (this thread pinned to one core for the run), a
    bounded sample: `reps` park + resume round trips of one sequence, median and p50/p99."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    try:
        import oracle as O
    except Exception:
        return None
    g = O.Geometry()
    if not O.ref_available():
        return None
    src, dst, ids = reference_pools(O, g, tokens)
    try:
        before = os.sched_getaffinity(0)
        os.sched_setaffinity(0, {min(before)})
    except (AttributeError, OSError):
        before = None
    try:
        save, restore = O.ref_time_park_resume(src, dst, ids, reps)
    finally:
        if before is not None:
            os.sched_setaffinity(0, before)
    t = save + restore
    b = O.metric_bytes(g, tokens)
    return {"value": round(float(b / (np.median(t) / 1e3) / 1e9), 3), "unit": UNIT, "cores": 1, "kind": "reference",
            "sample": f"{reps} x conversation_snapshot_save+_restore of one {tokens}-token sequence (reference "
                      f"sources, host pools) on one pinned core, median",
            "save_ms": round(float(np.median(save)), 2), "restore_ms": round(float(np.median(restore)), 2),
            "p50_ms": round(float(np.percentile(t, 50)), 2), "p99_ms": round(float(np.percentile(t, 99)), 2),
            "pinned": before is not None, "host": host_info()}


def reference_pools(O, g, tokens: int):
    """Host identity-layout pools for the reference (cheap deterministic fill: speed is data independent)."""
    s = O.Sequence(g, tokens, 0)
    n = s.pages * g.page_bytes
    rng = np.random.default_rng(0)
    proto = rng.integers(0, 256, n, dtype=np.uint8)
    s.k = [proto for _ in range(g.n_qsa + 1)]
    s.v = [proto for _ in range(g.n_qsa + 1)]
    s.pooled = [np.zeros(s.pooled_capacity_rows * g.idx_key_dim, np.float32) for _ in range(g.n_qsa)]
    s.tail = [np.zeros(3 * g.idx_key_dim, np.float32) for _ in range(g.n_qsa)]
    s.dead = [np.zeros(g.idx_key_dim, np.float32) for _ in range(g.n_qsa)]
    s.block_pos = [np.zeros(1, np.int32) for _ in range(g.n_qsa)]
    s.gdn = rng.standard_normal(g.n_gdn * g.gdn_row_floats, dtype=np.float32)
    s.ids = rng.integers(0, 151936, tokens, dtype=np.int32)
    return O.RefPools(s), O.RefPools(s, empty=True), s.ids


# ------------------------------------------------------------------------------------------------ arms

def run_reference_sweep(O) -> None:
    """The reference's own host hand-off path phase by phase, on one pinned core: conversation_snapshot_save,
    conversation_wire_encode (with its FNV-1a), conversation_wire_decode, conversation_snapshot_restore.  Per
    length a bounded sample (about 20 s of timed work, 2 to 20 repetitions; the long lengths take minutes to set
    up), p50/p99 per phase; the split-role figure is B(T) over all four phases, the park/resume figure over save +
    restore."""
    g = O.Geometry()
    host = host_info()   # before pinning: the host's cores, not the one this run keeps
    try:
        before = os.sched_getaffinity(0)
        os.sched_setaffinity(0, {min(before)})
    except (AttributeError, OSError):
        before = None
    try:
        for t in (1024, 4096, 32768, 65536, 131072):
            src, dst, ids = reference_pools(O, g, t)
            save, restore = O.ref_time_park_resume(src, dst, ids, 1)   # one rep sizes the sample
            payload, _ = O.ref_snapshot_encode(src, ids)
            enc, dec = O.ref_time_wire(payload, 1)
            one = float(save[0] + restore[0] + enc[0] + dec[0])
            reps = int(max(2, min(20, 20000 // max(one, 1.0))))
            save, restore = O.ref_time_park_resume(src, dst, ids, reps)
            enc, dec = O.ref_time_wire(payload, reps)
            b = O.metric_bytes(g, t)
            pct = lambda a: {"p50": round(float(np.percentile(a, 50)), 2),  # noqa: E731
                             "p99": round(float(np.percentile(a, 99)), 2)}
            print(json.dumps({"impl": "reference", "sweep": True, "tokens": t, "bytes": b, "payload_bytes": len(payload),
                              "reps": reps, "save_ms": pct(save), "encode_ms": pct(enc), "decode_ms": pct(dec),
                              "restore_ms": pct(restore),
                              "park_resume_gbs": round(b / (np.median(save + restore) / 1e3) / 1e9, 3),
                              "split_role_gbs": round(b / (np.median(save + enc + dec + restore) / 1e3) / 1e9, 3),
                              "cores": 1, "pinned": before is not None, "host": host}), flush=True)
            del src, dst, payload
    finally:
        if before is not None:
            os.sched_setaffinity(0, before)


REFERENCE_BUDGET_S = 150.0   # wall-time cap of the reference arm's timed steps


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    if not O.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libstrata_ref.so was not built "
                          "(needs the reference tree at build time)"}))
        return
    if args.sweep:
        run_reference_sweep(O)
        return
    g = O.Geometry()
    try:
        import psutil
        avail = psutil.virtual_memory().available
    except Exception:
        avail = 16 << 30
    per_thread = 3 * O.metric_bytes(g, args.tokens) + (1 << 30)
    threads = max(1, min(os.cpu_count() or 1, 16, int(avail * 0.6 // per_thread)))
    pools = [reference_pools(O, g, args.tokens) for _ in range(threads)]
    b = O.metric_bytes(g, args.tokens)
    warm = [0.0] * threads
    results = [None] * threads

    def warm_up(i):
        src, dst, ids = pools[i]
        s, r = O.ref_time_park_resume(src, dst, ids, max(1, args.warmup // 2))   # page faults etc.
        warm[i] = float(np.max(s + r)) / 1e3

    def worker(i, n):
        src, dst, ids = pools[i]
        results[i] = O.ref_time_park_resume(src, dst, ids, n)

    def run_all(fn, *extra):
        ts = [threading.Thread(target=fn, args=(i, *extra)) for i in range(threads)]
        for t in ts:
            t.start()
        for t in ts:
            t.join()

    run_all(warm_up)
    # the same step count as the device arm, unless that would take the host arm past REFERENCE_BUDGET_S
    per_step = max(1, min(args.steps, int(REFERENCE_BUDGET_S // max(max(warm), 1e-3))))
    t0 = time.perf_counter()
    run_all(worker, per_step)
    wall = time.perf_counter() - t0
    lat = np.concatenate([(s + r) for s, r in results])
    # aggregate: every thread moved per_step sequences; the slowest thread bounds the job
    slowest = max(float(np.sum(s + r)) for s, r in results) / 1e3
    value = threads * per_step * b / slowest / 1e9
    line = {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": per_step, "warmup": args.warmup, "ms_per_step": round(float(np.median(lat)), 3),
            "p50_ms": round(float(np.percentile(lat, 50)), 3), "p99_ms": round(float(np.percentile(lat, 99)), 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
            "data": "synthetic", "config": {"workload": f"host park/resume of a {args.tokens}-token sequence "
                                                       "(12 fp16 KV layers + 36 fp32 GDN rows + ids)",
                                            "tokens": args.tokens, "threads": threads},
            "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "reference",
                             "sample": f"{threads} threads x {per_step} conversation_snapshot_save+_restore each, "
                                       f"wall {wall:.1f} s", "host": host_info()},
            "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if per_step != args.steps:
        line["steps_note"] = (f"{args.steps} steps requested; one step of every thread took {max(warm):.2f} s in "
                              f"warm-up, so {per_step} steps keep the host arm within {REFERENCE_BUDGET_S:.0f} s")
    print(json.dumps(line))


def run_single(args, torch) -> None:
    kg = skv.KvGeometry()
    t = args.tokens
    engine = skv.COPY_TMA if args.engine == "tma" else skv.COPY_VEC
    torch.cuda.set_device(0)
    n_blocks = max(args.pool_blocks, kg.n_qsa * kg.blocks(t))
    src = SeqOnGpu(torch, kg, t, n_blocks, seed=args.seed, fill=True)
    dst = SeqOnGpu(torch, kg, t, n_blocks, seed=args.seed + 1000, fill=False)
    segs = skv.kv_segments_pool_to_pool(src.ps, dst.ps) + skv.state_segments(src.ps, dst.gdn, dst.ids)
    arr = (skv.Segment * len(segs))(*segs)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    L = skv.lib()

    def step():
        rc = L.skv_copy(arr, len(segs), engine, sp)
        if rc:
            skv.check(rc)

    skv.clear_status(0)
    with Clocks(0) as clk:
        total, per = time_steps(torch, stream, step, args.steps, args.warmup)
    status = skv.query_status(0)
    parity = (status == 0 and bool(torch.equal(dst.logical(torch), src.logical(torch)))
              and bool(torch.equal(dst.gdn, src.gdn)) and bool(torch.equal(dst.ids, src.ids)))
    b = kg.metric_bytes(t)
    value = b * args.steps / (total / 1e3) / 1e9
    p50, p99 = percentiles(per)
    hbm, hbm_kind = peaks()
    achieved = 2 * b / (total / args.steps / 1e3) / 1e9
    kernel = "copy_tma_kernel" if engine == skv.COPY_TMA else "copy_vec_kernel"
    workload = f"pool_to_pool_{t // 1024}k"
    line = {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(total / args.steps, 4), "p50_ms": round(p50, 4),
            "p99_ms": round(p99, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "u8", "data": "synthetic",
            "config": {"workload": f"config 2(a): 1xB200 intra-device pool->pool handoff of one {t}-token "
                                   "sequence (12 fp16 KV layers in 256-token blocks at seed-random slots of a "
                                   "4,096-block pool -> independent random slots of a second pool, + 36 fp32 "
                                   "GDN/conv rows + ids)", "tokens": t, "bytes_per_step": b,
                       "l2": "inputs larger than L2 (884 MB per step vs 126 MB)", "engine": args.engine,
                       "parallelism": "1 GPU"},
            "parity": parity, "gpu_launches": args.steps,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "peak_kind": f"{hbm_kind} copy (read+write)",
                         "traffic": traffic_for(kernel, workload), "kernel": kernel,
                         "algorithmic_bytes_per_launch": 2 * b}}
    line["clocks"] = clk.summary()
    if not args.no_length_sweep:
        line["length_sweep"] = [pool_to_pool_length(args, torch, kg, n, engine, hbm)
                                for n in SWEEP_TOKENS if n != t]
    if not args.no_e2e:
        e2e = e2e_park_resume(torch, kg, src, dst, args.steps, max(3, args.warmup), max(3, args.steps // 4),
                              args.relay_mb << 20, args.relay_lanes, args.relay_ramp == "on")
        pcie = pcie_probe(torch)
        e2e["pcie_peak"] = pcie
        # the relay keeps both directions busy, so its bound is the two-direction probe
        e2e["pcie_frac"] = round(e2e["pcie_gbs_both_directions"] / pcie["both_directions_gbs"], 4)
        line["e2e"] = e2e
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(t)
    print(json.dumps(line))


def pool_to_pool_length(args, torch, kg, t: int, engine: int, hbm: float) -> dict:
    """Config 2(a)'s operation at another length of config 3's sweep: two fresh pools, min(K, 50) timed steps after
    the warm-up, CUDA events per step, parity, and the kernel's fraction of the HBM copy peak (2 B(T) per step)."""
    n_blocks = max(args.pool_blocks, kg.n_qsa * kg.blocks(t))
    src = SeqOnGpu(torch, kg, t, n_blocks, seed=args.seed + t, fill=True)
    dst = SeqOnGpu(torch, kg, t, n_blocks, seed=args.seed + t + 1000, fill=False)
    segs = skv.kv_segments_pool_to_pool(src.ps, dst.ps) + skv.state_segments(src.ps, dst.gdn, dst.ids)
    arr = (skv.Segment * len(segs))(*segs)
    stream = torch.cuda.current_stream()
    L = skv.lib()
    steps = min(args.steps, 50)

    def step():
        skv.check(L.skv_copy(arr, len(segs), engine, stream.cuda_stream))

    skv.clear_status(0)
    total, per = time_steps(torch, stream, step, steps, max(3, args.warmup))
    parity = (skv.query_status(0) == 0 and bool(torch.equal(dst.logical(torch), src.logical(torch)))
              and bool(torch.equal(dst.gdn, src.gdn)) and bool(torch.equal(dst.ids, src.ids)))
    b = kg.metric_bytes(t)
    p50, p99 = percentiles(per)
    achieved = 2 * b / (total / steps / 1e3) / 1e9
    del src, dst
    torch.cuda.empty_cache()
    return {"tokens": t, "bytes": b, "steps": steps, "value": round(b * steps / (total / 1e3) / 1e9, 3),
            "ms_per_step": round(total / steps, 4), "p50_ms": round(p50, 4), "p99_ms": round(p99, 4),
            "hbm_frac": round(achieved / hbm, 4), "parity": parity}


def run_p2p_local(args, torch) -> None:
    """One process, two GPUs: the decode GPU (cuda:1) pulls one sequence from the prefill GPU's pool (cuda:0) into
    independent random slots of its own pool with the TMA engine (bulk loads of peer memory over NVLink, no
    multicast), K steps timed with CUDA events on the decode GPU's stream.  The case a single-process profiler
    capture of the NVLink counters runs on; the multi-process pairs (torchrun) are the headline."""
    if torch.cuda.device_count() < 2:
        print(json.dumps({"scenario": "p2p-local", "unavailable": "needs two GPUs"}))
        return
    kg = skv.KvGeometry()
    t = args.tokens
    n_blocks = max(args.pool_blocks, kg.n_qsa * kg.blocks(t))
    skv.check(skv.lib().skv_enable_peer(1, 0))
    with torch.cuda.device(0):
        src = SeqOnGpu(torch, kg, t, n_blocks, seed=args.seed, fill=True)
        torch.cuda.synchronize()
    torch.cuda.set_device(1)
    dst = SeqOnGpu(torch, kg, t, n_blocks, seed=args.seed + 1000, fill=False)
    segs = skv.kv_segments_pool_to_pool(src.ps, dst.ps) + skv.state_segments(src.ps, dst.gdn, dst.ids)
    arr = (skv.Segment * len(segs))(*segs)
    stream = torch.cuda.current_stream(1)
    L = skv.lib()

    def step():
        skv.check(L.skv_copy(arr, len(segs), skv.COPY_TMA, stream.cuda_stream))

    skv.clear_status(1)
    total, per = time_steps(torch, stream, step, args.steps, args.warmup)
    parity = (skv.query_status(1) == 0 and bool(torch.equal(dst.logical(torch).cpu(), src.logical(torch).cpu()))
              and bool(torch.equal(dst.gdn.cpu(), src.gdn.cpu())) and bool(torch.equal(dst.ids.cpu(), src.ids.cpu())))
    b = kg.metric_bytes(t)
    p50, p99 = percentiles(per)
    print(json.dumps({"scenario": "p2p-local", "metric": METRIC, "value": round(b * args.steps / (total / 1e3) / 1e9, 3),
                      "unit": UNIT, "tokens": t, "bytes_per_step": b, "steps": args.steps, "warmup": args.warmup,
                      "ms_per_step": round(total / args.steps, 4), "p50_ms": round(p50, 4), "p99_ms": round(p99, 4),
                      "parity": parity, "kernel": "copy_tma_kernel on cuda:1 loading cuda:0's pool",
                      "tuning": dict(zip(("tma_stages", "tma_tile_bytes", "tma_ctas_per_sm", "vec_ctas_per_sm"),
                                         skv.get_copy_tuning()))}))


# ------------------------------------------------------------------------------------------------ N > 1: pairs

def pair_role(rank: int, world: int) -> tuple:
    """(role, peer, active): even ranks prefill, the next odd rank decodes; an unpaired last rank idles."""
    pairs = world // 2
    role = "prefill" if rank % 2 == 0 else "decode"
    peer = rank + 1 if role == "prefill" else rank - 1
    return role, peer, rank < 2 * pairs


FLAGS = 128   # 8-byte flag words per state arena (chunk flags of a pipelined fan-out, completion flags)


def state_layout(kg: skv.KvGeometry, tokens: int) -> dict:
    """The decode GPU's per-sequence state arena: GDN rows | ids (16-byte rounded) | FLAGS flag words."""
    ids_off = kg.gdn_bytes
    flag_off = (ids_off + ((4 * tokens + 15) // 16) * 16 + 255) // 256 * 256
    total = (flag_off + 8 * FLAGS + 1023) // 1024 * 1024
    return {"ids": ids_off, "flag": flag_off, "bytes": total}


def summarize_pairs(max_elapsed_ms: float, per_step_ms: np.ndarray, pairs: int, seq_bytes: int, steps: int) -> dict:
    """Whole-job numbers from the max-over-ranks timed region and the per-step max-over-ranks latencies."""
    value = pairs * seq_bytes * steps / (max_elapsed_ms / 1e3) / 1e9
    per_pair = seq_bytes / (max_elapsed_ms / steps / 1e3) / 1e9
    return {"value": value, "per_pair_gbs": per_pair, "ms_per_step": max_elapsed_ms / steps,
            "p50_ms": float(np.percentile(per_step_ms, 50)), "p99_ms": float(np.percentile(per_step_ms, 99))}


def pair_parity(torch, dist, seq, role: str, peer: int, active: bool) -> list:
    """Each side packs its copy through ITS OWN table with the gather kernel; the decode side ships its image to
    the prefill side, which compares it with the image of the source.  One bool per pair (pair p = ranks 2p and
    2p+1), the same list on every rank."""
    ok = torch.ones(1, device="cuda")
    if active:
        image = seq.packed(torch)
        if role == "decode":
            dist.send(image, peer)
        else:
            got = torch.empty_like(image)
            dist.recv(got, peer)
            ok[0] = float(bool(torch.equal(got, image)))
    every = [torch.zeros_like(ok) for _ in range(dist.get_world_size())]
    dist.all_gather(every, ok)
    return [a == 1.0 and b == 1.0 for a, b in per_pair([float(e.item()) for e in every])]


def per_pair(values: list) -> list:
    """One value per rank -> one (prefill's, decode's) tuple per pair: pair p is ranks 2p and 2p + 1 (an unpaired
    last rank is left out)."""
    return [(values[2 * p], values[2 * p + 1]) for p in range(len(values) // 2)]


def cudart():
    """The CUDA runtime the library itself loaded (for the copy-engine probe's cudaMemcpyAsync)."""
    rt = ctypes.CDLL("libcudart.so.12")
    rt.cudaMemcpyAsync.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p]
    rt.cudaMemcpyAsync.restype = ctypes.c_int
    return rt


PROBE_BYTES = 1 << 30


def peer_copy_probe(torch, dist, role: str, active: bool, local_base: int, peer_base: int, nbytes: int,
                    stream, reps: int = 5) -> dict:
    """The NVLink reference of this run, on the same pairs: copy-engine copies (cudaMemcpyAsync between this GPU's
    memory and the peer's CUDA-IPC mapping) of `nbytes` between the two GPUs of every pair, all pairs at once,
    each direction in turn, median of `reps` after one untimed copy (CUDA events on the copying GPU's stream).
    pull: the decode GPU copies the prefill GPU's pool into its own pool; push: the prefill GPU copies its pool
    into the decode GPU's pool.  Only decode pools are written, and the hand-off overwrites them afterwards."""
    rt = cudart()
    world = dist.get_world_size()
    out = {"bytes": nbytes, "reps": reps, "how": "cudaMemcpyAsync over the pair's CUDA-IPC mapping, every pair at "
                                                 "once, median of reps, CUDA events"}
    for direction, mover in (("pull", "decode"), ("push", "prefill")):
        times = []
        for _ in range(reps + 1):
            torch.cuda.synchronize()
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            if active and role == mover:
                dst, src = (local_base, peer_base) if direction == "pull" else (peer_base, local_base)
                rc = rt.cudaMemcpyAsync(dst, src, nbytes, 4, stream.cuda_stream)   # 4 = cudaMemcpyDefault
                if rc:
                    raise RuntimeError(f"peer copy probe: cudaMemcpyAsync returned {rc}")
            e1.record(stream)
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        mine = torch.tensor([float(np.median(times[1:])) if active and role == mover else 0.0], device="cuda")
        every = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(every, mine)
        who = 1 if mover == "decode" else 0
        gbs = [round(nbytes / (pair[who] / 1e3) / 1e9, 1) for pair in per_pair([float(e.item()) for e in every])]
        out[f"{direction}_gbs"] = gbs
        out[f"{direction}_gbs_median"] = round(float(np.median(gbs)), 1)
    dist.barrier()
    return out


def host_relay_pairs(args, torch, dist, kg, t: int, seq, role: str, peer: int, active: bool, stream,
                     pairs: int) -> dict:
    """e2e at N GPUs: the same hand-off through pinned host memory, the route the reference's multi-GPU split
    takes.  The prefill rank parks into a shared-memory buffer both ranks registered with CUDA
    (skv.SharedHostBuffer) and the decode rank resumes from it, piece by piece: after each piece's device-to-host
    copy the prefill GPU raises that piece's flag in the same host buffer, the decode GPU waits for it (bounded) and
    copies the piece in, so both PCIe links and both directions stay busy; the decode GPU raises DONE at the end.
    C-ABI calls only (skv_park, skv_resume, skv_signal, skv_wait_flag).  The decode pool is cleared first and the
    pairs' parity is checked again afterwards."""
    L = skv.lib()
    sp = stream.cuda_stream
    off = skv.image_offsets(kg, t, kg.n_qsa)
    shared, handle = None, None
    if active and role == "prefill":
        shared = skv.SharedHostBuffer(off["total"] + 8 * FLAGS)   # a fresh memfd reads as zeros: flags start at 0
        handle = shared.handle()
    handles = [None] * dist.get_world_size()
    dist.all_gather_object(handles, handle)
    if active and role == "decode":
        shared = skv.SharedHostBuffer(off["total"] + 8 * FLAGS, handle=handles[peer])
    steps, warmup = max(3, min(args.steps, 20)), 2
    step = None
    counter = [0]
    if active:
        flags = shared.ptr + off["total"]
        done = flags + 8 * (FLAGS - 1)
        staging = torch.empty(off["total"] + 256 * 64, dtype=torch.uint8, device="cuda")
        if role == "prefill":
            segs = [p for s in skv.pack_segments(seq.ps, shared.ptr) for p in skv.split_segment(s, RELAY_CHUNK_BYTES)]
        else:
            segs = [p for s in skv.unpack_segments(shared.ptr, seq.ps) for p in skv.split_segment(s, RELAY_CHUNK_BYTES)]
        if len(segs) > FLAGS - 1:
            raise SystemExit(f"{len(segs)} relay pieces; at most {FLAGS - 1}")
        at, coff = 0, []
        for p in segs:
            coff.append(at)
            at += (p.bytes + 255) & ~255
        arrs = [(skv.Segment * 1)(p) for p in segs]
        base = staging.data_ptr()
        if role == "decode":   # the P2P run already filled this pool: clear it, the bytes must come from the host
            zero = torch.zeros(256 << 20, dtype=torch.uint8, device="cuda")
            for region, total in ((seq.pool.base, seq.pool.n_blocks * kg.block_bytes), (seq.state.base, seq.state_bytes)):
                for a in range(0, total, zero.numel()):
                    skv.copy([skv.segment(zero, region + a, min(zero.numel(), total - a))], skv.COPY_VEC)
            torch.cuda.synchronize()

        def step():
            counter[0] += 1
            v = counter[0]
            if role == "prefill":
                skv.check(L.skv_wait_flag(done, v - 1, 5_000_000_000, sp))        # the host buffer is free again
                for k, a in enumerate(arrs):
                    skv.check(L.skv_park(a, 1, skv.PARK_STAGED, base + coff[k], staging.numel() - coff[k], sp))
                    skv.check(L.skv_signal(flags + 8 * k, v, sp))                  # piece k is in host memory
            else:
                for k, a in enumerate(arrs):
                    skv.check(L.skv_wait_flag(flags + 8 * k, v, 5_000_000_000, sp))
                    skv.check(L.skv_resume(a, 1, skv.PARK_STAGED, base + coff[k], staging.numel() - coff[k], sp))
                skv.check(L.skv_signal(done, v, sp))                               # the host buffer may be reused
    dist.barrier()
    for _ in range(warmup):
        if step:
            step()
    torch.cuda.synchronize()
    dist.barrier()
    device_align(torch, dist)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        if step:
            step()
    e1.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    el = torch.tensor([e0.elapsed_time(e1), float(skv.query_status(torch.cuda.current_device()) != 0)], device="cuda")
    dist.all_reduce(el, op=dist.ReduceOp.MAX)
    ok = pair_parity(torch, dist, seq, role, peer, active)
    if shared is not None:
        shared.close()
    b = kg.metric_bytes(t)
    value = pairs * b * steps / (float(el[0].item()) / 1e3) / 1e9
    return {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": pairs * b, "d2h_bytes_per_step": pairs * b,
            "ms_per_step": round(float(el[0].item()) / steps, 4), "per_pair_gbs": round(value / pairs, 3),
            "parity": all(ok) and el[1].item() == 0, "parity_by_pair": ok, "steps": steps,
            "api": "skv_park on the prefill GPU into pinned memory shared with its decode rank (memfd + "
                   "skv_host_register), skv_resume on the decode GPU, per-piece flags in that host memory",
            "note": "the reference's multi-GPU route (through pinned RAM), PCIe-bound per pair"}


def run_pairs(args, torch, tokens: int | None = None, steps: int | None = None, e2e: bool = True,
              probe: dict | None = None) -> tuple:
    """N/2 prefill->decode pairs.  pull (default): the decode GPU's copy kernel reads the prefill GPU's pool
    pages over NVLink (TMA bulk loads from peer memory, no multicast) and writes its own pool; push: the
    prefill GPU's vector kernel stores into the decode GPU's pool.  Either way the destination slots are written
    directly, with no intermediate contiguous copy.  Protocol per step (flags are 8-byte words, release
    stores / bounded acquire polls): pull = prefill raises READY on the decode GPU, decode waits READY, pulls,
    raises DONE on the prefill GPU (whose blocks may then be freed), prefill waits DONE; push = prefill pushes
    and raises ARRIVED, decode waits ARRIVED.

    `probe`: the peer-copy reference of this run; measured here (before the hand-offs) when None.  Returns
    (rank 0's line or None, the probe)."""
    import torch.distributed as dist
    rank, world, local = ranks()
    kg = skv.KvGeometry()
    t = tokens or args.tokens
    n_steps = steps or args.steps
    pairs = world // 2
    role, peer, active = pair_role(rank, world)
    lay = state_layout(kg, t)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    L = skv.lib()
    n_blocks = max(args.pool_blocks, kg.n_qsa * kg.blocks(t))
    pull = args.p2p in ("pull", "pull-gated")
    gated = args.p2p == "pull-gated"
    push_engine = skv.COPY_TMA if args.p2p == "push-tma" else skv.COPY_VEC
    seq = None
    mine = None
    if active:
        seq = SeqOnGpu(torch, kg, t, n_blocks, seed=args.seed + 1000 * (role == "decode") + rank,
                       fill=role == "prefill", ipc=True)
        mine = {"pool": skv.ipc_export(seq.pool.base), "state": skv.ipc_export(seq.state.base),
                "tables": seq.host_tables}
        torch.cuda.synchronize()
    handles = [None] * world
    dist.all_gather_object(handles, mine)
    imported = []
    step = None
    peer_pool = 0
    if active:
        other = handles[peer]
        peer_pool = skv.ipc_import(local, other["pool"])
        peer_state = skv.ipc_import(local, other["state"])
        imported = [peer_pool, peer_state]
        peer_flag = peer_state + lay["flag"]
        peer_tables = torch.from_numpy(other["tables"].reshape(-1).copy()).cuda()
        peer_seq = skv.PooledSequence(kg, skv.Pool(local, n_blocks, kg.block_bytes, memory=peer_pool), t, kg.n_qsa,
                                      None, peer_tables, peer_state, peer_state + lay["ids"])
        counter = [0]
        if gated and role == "decode":
            segs = skv.kv_segments_pool_to_pool(peer_seq, seq.ps) + skv.state_segments(peer_seq, seq.gdn, seq.ids)
            arr = (skv.Segment * len(segs))(*segs)

            def step():
                counter[0] += 1   # one launch: wait for READY, pull over NVLink, release DONE on the prefill GPU
                skv.check(L.skv_copy_gated(arr, len(segs), seq.flag, counter[0], 5_000_000_000, peer_flag, counter[0],
                                           sp))
        elif pull and role == "decode":
            segs = skv.kv_segments_pool_to_pool(peer_seq, seq.ps) + skv.state_segments(peer_seq, seq.gdn, seq.ids)
            arr = (skv.Segment * len(segs))(*segs)

            def step():
                counter[0] += 1
                skv.check(L.skv_wait_flag(seq.flag, counter[0], 5_000_000_000, sp))    # READY
                skv.check(L.skv_copy(arr, len(segs), skv.COPY_TMA, sp))              # pull over NVLink
                skv.check(L.skv_signal(peer_flag, counter[0], sp))                   # DONE
        elif pull:
            def step():
                counter[0] += 1
                skv.check(L.skv_signal(peer_flag, counter[0], sp))                   # READY
                skv.check(L.skv_wait_flag(seq.flag, counter[0], 5_000_000_000, sp))  # DONE
        elif role == "prefill":
            segs = (skv.kv_segments_pool_to_pool(seq.ps, peer_seq, dst_base=peer_pool)
                    + skv.state_segments(seq.ps, peer_state, peer_state + lay["ids"]))
            arr = (skv.Segment * len(segs))(*segs)

            def step():
                counter[0] += 1
                skv.check(L.skv_copy(arr, len(segs), push_engine, sp))               # remote stores
                skv.check(L.skv_signal(peer_flag, counter[0], sp))                   # ARRIVED
        else:
            def step():
                counter[0] += 1
                skv.check(L.skv_wait_flag(seq.flag, counter[0], 5_000_000_000, sp))  # ARRIVED
    if step is None:
        def step():
            pass
    if probe is None:
        probe = peer_copy_probe(torch, dist, role, active, seq.pool.base if active else 0, peer_pool,
                                min(PROBE_BYTES, n_blocks * kg.block_bytes), stream)
    skv.clear_status(local)
    dist.barrier()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(n_steps + 1)]
    # host-side preparation (the collection, the clock sampler's start) first, then the device-side alignment, then
    # at once the start event and the steps: anything a host does after the alignment is skew in the first step
    with Clocks(local, sample=rank == 0) as clk, quiet_gc():
        device_align(torch, dist)
        ev[0].record(stream)
        for i in range(n_steps):
            step()
            ev[i + 1].record(stream)
        torch.cuda.synchronize()
    dist.barrier()
    per = torch.tensor([ev[i].elapsed_time(ev[i + 1]) for i in range(n_steps)], device="cuda")
    status = skv.query_status(local)
    red = torch.tensor([ev[0].elapsed_time(ev[n_steps]), float(status != 0)], device="cuda")
    dist.all_reduce(red, op=dist.ReduceOp.MAX)
    dist.all_reduce(per, op=dist.ReduceOp.MAX)
    ok = pair_parity(torch, dist, seq, role, peer, active)
    relay = None
    if e2e and not args.no_e2e:
        relay = host_relay_pairs(args, torch, dist, kg, t, seq, role, peer, active, stream, pairs)
    res = summarize_pairs(float(red[0].item()), per.cpu().numpy(), pairs, kg.metric_bytes(t), n_steps)
    line = None
    if rank == 0:
        ref = probe["pull_gbs_median"] if pull else probe["push_gbs_median"]
        line = {"metric": METRIC, "value": round(res["value"], 3), "unit": UNIT, "n_gpus": world, "steps": n_steps,
                "warmup": args.warmup, "ms_per_step": round(res["ms_per_step"], 4), "p50_ms": round(res["p50_ms"], 4),
                "p99_ms": round(res["p99_ms"], 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "u8", "data": "synthetic",
                "config": {"workload": f"config 3/5: {pairs} prefill->decode pair(s), one {t}-token sequence per pair "
                                       f"per step moved over NVLink ({args.p2p}: CUDA IPC peer pointers) straight "
                                       f"into independent random slots of the decode GPU's {n_blocks}-block pool",
                           "tokens": t, "pairs": pairs, "p2p": args.p2p, "bytes_per_step_per_pair": kg.metric_bytes(t),
                           "l2": "inputs larger than L2", "parallelism": f"{pairs} prefill/decode pairs"},
                "parity": all(ok) and red[1].item() == 0, "parity_by_pair": ok,
                # per pair and step: pull = wait+copy+signal and signal+wait; pull-gated = gated copy and signal+wait;
                # push = copy+signal and wait
                "gpu_launches": n_steps * (3 if gated else 5 if pull else 3) * pairs,
                "roofline": {"bound": "nvlink", "achieved": round(res["per_pair_gbs"], 1), "peak": ref,
                             "unit": "GB/s", "frac": round(res["per_pair_gbs"] / ref, 4),
                             "frac_of_nominal_900": round(res["per_pair_gbs"] / 900.0, 4),
                             "peak_kind": f"peer copy of this run ({'pull' if pull else 'push'} direction, "
                                          "peer_copy_probe); 900 GB/s per direction nominal",
                             "traffic": None, "kernel": {"push": "copy_vec_kernel", "pull-gated": "copy_tma_gated_kernel"}.get(args.p2p, "copy_tma_kernel")},
                "peer_copy_probe": probe,
                "clocks": clk.summary()}
        if relay is not None:
            line["e2e"] = relay
    torch.cuda.synchronize()
    dist.barrier()
    for p in imported:
        skv.ipc_close(p)
    dist.barrier()
    return (line if rank == 0 else None), probe


SWEEP_TOKENS = (1024, 4096, 32768, 131072)   # config 3's lengths


def pair_sweep(args, torch, probe: dict, headline: dict | None) -> list | None:
    """Config 3's length sweep on the same pairs and probe: every length of SWEEP_TOKENS but the headline's own
    (reused), each a short run of its own with parity."""
    rows = []
    for t in SWEEP_TOKENS:
        if t == args.tokens:
            sub = headline
        else:
            sub, _ = run_pairs(args, torch, tokens=t, steps=min(args.steps, 50), e2e=False, probe=probe)
        if sub is not None:
            rows.append({"tokens": t, "bytes": sub["config"]["bytes_per_step_per_pair"], "steps": sub["steps"],
                         "value": sub["value"], "ms_per_step": sub["ms_per_step"], "p50_ms": sub["p50_ms"],
                         "p99_ms": sub["p99_ms"], "per_pair_gbs": sub["roofline"]["achieved"],
                         "frac_of_probe": sub["roofline"]["frac"],
                         "frac_of_nominal_900": sub["roofline"]["frac_of_nominal_900"], "parity": sub["parity"]})
    return rows if headline is not None else None


SPLIT_ROLE_TOKENS = (4096, 32768)


def split_roles(torch, rank: int) -> list | None:
    """Row f2 on this run's GPUs 0 and 1: the split-role hand-off across two processes with only a device
    descriptor in the hand-off slot (tests/cpp/handoff_device_gpu_test.cpp: prefill process on GPU 0 packs the
    whole session into its HBM and publishes the descriptor; decode process on GPU 1 reads the slot, mounts
    straight from GPU 0's HBM and checks every byte), at config 1's length and at 32K.  Rank 0 runs it while every
    rank holds no work on its GPU: the other ranks wait on the rendezvous store (a host wait), not in a
    collective.  Returns rank 0's records."""
    import re
    import subprocess
    import tempfile
    from datetime import timedelta

    import torch.distributed as dist
    store = dist.distributed_c10d._get_default_store()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    key = "skv_split_roles_done"
    rows = None
    if rank == 0:
        rows = []
        try:
            sys.path.insert(0, os.path.join(ROOT, "tests"))
            from test_cpp_gpu import build as build_cpp_test
            exe = build_cpp_test("handoff_device_gpu_test")
            for t in SPLIT_ROLE_TOKENS:
                with tempfile.TemporaryDirectory() as d:
                    r = subprocess.run([exe, d, str(t)], capture_output=True, text=True, timeout=400)
                out = r.stdout
                pub = re.search(r"publish \(pack into HBM \+ descriptor\) ([0-9.]+) ms; fastest claim-to-release "
                                r"\(publish, DONE, decode mount, ACK, release\) ([0-9.]+) ms for ([0-9]+) payload bytes", out)
                mnt = re.search(r"read the slot \+ mount from the peer's HBM ([0-9.]+) ms", out)
                phases = {side: dict(zip(("prepare_ms", "issue_ms", "complete_ms", "total_ms"),
                                         (float(x) for x in m.groups())))
                          for side, m in (("pack", re.search(r"pack phases prepare ([0-9.]+) issue ([0-9.]+) complete "
                                                             r"([0-9.]+) total ([0-9.]+) ms", out)),
                                          ("mount", re.search(r"mount phases prepare ([0-9.]+) issue ([0-9.]+) complete "
                                                              r"([0-9.]+) total ([0-9.]+) ms", out))) if m}
                checks = [int(c) for c in re.findall(r"([0-9]+) checks passed", out)]
                row = {"tokens": t, "rc": r.returncode, "parity": r.returncode == 0 and "both instances passed" in out,
                       "checks": sum(checks)}
                if pub and mnt:
                    nbytes = int(pub.group(3))
                    row.update({"payload_bytes": nbytes, "publish_ms": float(pub.group(1)),
                                "mount_ms": float(mnt.group(1)), "claim_to_release_ms": float(pub.group(2)),
                                "mount_gbs_over_nvlink": round(nbytes / (float(mnt.group(1)) / 1e3) / 1e9, 1)})
                if phases:
                    row["phases"] = phases
                if r.returncode:
                    row["tail"] = (out + r.stderr)[-400:]
                rows.append(row)
        except Exception as e:   # the record says why; the headline stands
            rows.append({"error": f"{type(e).__name__}: {e}"[:400]})
        finally:
            store.set(key, "1")
    else:
        store.wait([key], timedelta(seconds=1200))
    dist.barrier()
    return rows


# ------------------------------------------------------------------------------------------------ fan-out

def run_fanout(args, torch, tokens: int | None = None, steps: int | None = None, probe: dict | None = None) -> dict | None:
    """Config 4: rank 0 (prefill) holds one sequence; ranks 1..N-1 (decode) each receive the whole cache into
    their own pool at independent random slots.  Four ways, each timed over the same K steps:

      p2p    every receiver pulls the whole sequence from rank 0's pool at once (the source's NVLink egress
             carries the cache N-1 times);
      nccl   rank 0 packs the sequence into a contiguous image (gather kernel), ncclBroadcast sends it, each
             receiver scatters it into its pool (the reference-style collective path);
      chain  receiver k pulls chunk c of the cache from receiver k-1's pool as soon as k-1 signals it landed, so
             every NVLink hop carries the cache once and the hops overlap chunk by chunk;
      chain_push  the same pipeline driven from the sending side: GPU k bulk-stores chunk c from its own pool
             into GPU k+1's pool and raises k+1's flag for it (no read requests cross NVLink).

    value = receivers x B(T) x K / max-over-ranks timed region (fan-out counts every receiver's bytes)."""
    import torch.distributed as dist
    rank, world, local = ranks()
    kg = skv.KvGeometry()
    t = tokens or args.tokens
    n_steps = steps or args.steps
    receivers = world - 1
    lay = state_layout(kg, t)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    L = skv.lib()
    n_blocks = max(args.pool_blocks, kg.n_qsa * kg.blocks(t))
    seq = SeqOnGpu(torch, kg, t, n_blocks, seed=args.seed + 1000 * rank, fill=rank == 0, ipc=True)
    mine = {"pool": skv.ipc_export(seq.pool.base), "state": skv.ipc_export(seq.state.base), "tables": seq.host_tables}
    torch.cuda.synchronize()
    handles = [None] * world
    dist.all_gather_object(handles, mine)
    maps = {}                    # rank -> (pool base, state base) mapped here

    def peer(r):
        if r not in maps:
            maps[r] = (skv.ipc_import(local, handles[r]["pool"]), skv.ipc_import(local, handles[r]["state"]))
        return maps[r]

    def peer_seq(r):
        pool, state = peer(r)
        tables = torch.from_numpy(handles[r]["tables"].reshape(-1).copy()).cuda()
        return skv.PooledSequence(kg, skv.Pool(local, n_blocks, kg.block_bytes, memory=pool), t, kg.n_qsa, None,
                                  tables, state, state + lay["ids"]), tables

    flag = lambda base, i: base + lay["flag"] + 8 * i            # noqa: E731
    DONE = FLAGS - 1 - receivers                                  # rank 0's flags DONE+1 .. DONE+receivers
    wait_ns = 5_000_000_000
    off = skv.image_offsets(kg, t, kg.n_qsa)
    image = torch.empty(off["total"], dtype=torch.uint8, device="cuda")
    chunk_bytes = args.chunk_mb << 20
    keep = []                    # tables of mapped peers stay alive
    results = {}
    counter = [0]

    def timed(step):
        dist.barrier()
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        dist.barrier()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(n_steps + 1)]
        with quiet_gc():
            device_align(torch, dist)   # after the collection: nothing of the host's lands in the first step
            ev[0].record(stream)
            for i in range(n_steps):
                step()
                ev[i + 1].record(stream)
            torch.cuda.synchronize()
        dist.barrier()
        per = torch.tensor([ev[i].elapsed_time(ev[i + 1]) for i in range(n_steps)], device="cuda")
        tot = torch.tensor([ev[0].elapsed_time(ev[n_steps])], device="cuda")
        dist.all_reduce(tot, op=dist.ReduceOp.MAX)
        dist.all_reduce(per, op=dist.ReduceOp.MAX)
        return float(tot.item()), per.cpu().numpy()

    def parity():
        """Every receiver's cache, packed through its own table, equals the source's packed cache."""
        mine_img = seq.packed(torch)
        ref = mine_img if rank == 0 else torch.empty_like(mine_img)
        dist.broadcast(ref, 0)
        ok = torch.tensor([float(bool(torch.equal(ref, mine_img)))], device="cuda")
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        return bool(ok.item() == 1.0)

    def clear_receiver():
        if rank:
            zero = torch.zeros(1 << 28, dtype=torch.uint8, device="cuda")
            total = n_blocks * kg.block_bytes
            for at in range(0, total, zero.numel()):
                n = min(zero.numel(), total - at)
                skv.copy([skv.segment(zero, seq.pool.base + at, n)], skv.COPY_VEC)
            skv.copy([skv.segment(zero, seq.gdn, kg.gdn_bytes)], skv.COPY_VEC)
            torch.cuda.synchronize()
        dist.barrier()

    # ---- p2p: every receiver pulls from rank 0 at once
    if rank == 0:
        rflags = [peer(r)[1] for r in range(1, world)]

        def step():
            counter[0] += 1
            for r, st in enumerate(rflags):
                skv.check(L.skv_signal(flag(st, 0), counter[0], sp))                 # READY
            for r in range(receivers):
                skv.check(L.skv_wait_flag(flag(seq.state.base, DONE + 1 + r), counter[0], wait_ns, sp))
    else:
        src, tab = peer_seq(0)
        keep.append(tab)
        segs = skv.kv_segments_pool_to_pool(src, seq.ps) + skv.state_segments(src, seq.gdn, seq.ids)
        arr = (skv.Segment * len(segs))(*segs)
        done0 = flag(peer(0)[1], DONE + rank)

        def step():
            counter[0] += 1
            skv.check(L.skv_wait_flag(flag(seq.state.base, 0), counter[0], wait_ns, sp))
            skv.check(L.skv_copy(arr, len(segs), skv.COPY_TMA, sp))
            skv.check(L.skv_signal(done0, counter[0], sp))
    clear_receiver()
    skv.clear_status(local)
    results["p2p"] = timed(step) + (parity(),)

    # ---- nccl: pack, broadcast, scatter
    pack = (skv.Segment * len(s0 := skv.pack_segments(seq.ps, image)))(*s0)
    unpack = (skv.Segment * len(s1 := skv.unpack_segments(image, seq.ps)))(*s1)

    def step():
        if rank == 0:
            skv.check(L.skv_copy(pack, len(s0), skv.COPY_TMA, sp))
        dist.broadcast(image, 0)
        if rank:
            skv.check(L.skv_copy(unpack, len(s1), skv.COPY_TMA, sp))
    clear_receiver()
    results["nccl"] = timed(step) + (parity(),)

    # ---- chain: receiver k pulls chunk c from receiver k-1 once k-1 has it
    counter[0] = 10 ** 6          # flag values keep growing across methods
    if rank == 0:
        first = flag(peer(1)[1], 0)

        def step():
            counter[0] += 1
            skv.check(L.skv_signal(first, counter[0], sp))                           # READY to receiver 1
            skv.check(L.skv_wait_flag(flag(seq.state.base, DONE + receivers), counter[0], wait_ns, sp))
        n_chunks = 0
    else:
        up, tab = peer_seq(rank - 1)
        keep.append(tab)
        whole = skv.kv_segments_pool_to_pool(up, seq.ps) + skv.state_segments(up, seq.gdn, seq.ids)
        pieces = [p for w in whole for p in skv.split_segment(w, chunk_bytes)]
        n_chunks = len(pieces)
        if n_chunks > FLAGS - 1 - receivers:
            raise SystemExit(f"--chunk-mb {args.chunk_mb} gives {n_chunks} chunks; at most {FLAGS - 1 - receivers}")
        # one chained launch per group of at most SKV_COPY_MAX_SEGMENTS chunks: in-kernel waits on this GPU's
        # chunk flags (set by the previous receiver), in-kernel release stores to the next receiver's flags
        groups = [(g0, (skv.Segment * len(pieces[g0:g0 + skv.MAX_SEGMENTS]))(*pieces[g0:g0 + skv.MAX_SEGMENTS]))
                  for g0 in range(0, n_chunks, skv.MAX_SEGMENTS)]
        down = peer(rank + 1)[1] if rank < receivers else None
        done0 = flag(peer(0)[1], DONE + receivers)

        def step():
            counter[0] += 1
            if rank == 1:
                skv.check(L.skv_wait_flag(flag(seq.state.base, 0), counter[0], wait_ns, sp))   # READY
            for g0, arr in groups:
                wait = None if rank == 1 else flag(seq.state.base, g0)
                signal = flag(down, g0) if down else None
                skv.check(L.skv_copy_chained(arr, len(arr), wait, signal, counter[0], wait_ns, sp))
            if not down:
                skv.check(L.skv_signal(done0, counter[0], sp))
    clear_receiver()
    results["chain"] = timed(step) + (parity(),)

    # ---- chain_push: GPU k stores chunk c into GPU k+1's pool, then raises k+1's flag c
    counter[0] = 2 * 10 ** 6
    if rank < receivers:
        dn, tab = peer_seq(rank + 1)
        keep.append(tab)
        whole = skv.kv_segments_pool_to_pool(seq.ps, dn) + skv.state_segments(seq.ps, dn.gdn, dn.ids)
        pieces = [p for w in whole for p in skv.split_segment(w, chunk_bytes)]
        if len(pieces) > FLAGS - 1 - receivers:
            raise SystemExit(f"--chunk-mb {args.chunk_mb} gives {len(pieces)} chunks; at most {FLAGS - 1 - receivers}")
        groups = [(g0, (skv.Segment * len(pieces[g0:g0 + skv.MAX_SEGMENTS]))(*pieces[g0:g0 + skv.MAX_SEGMENTS]))
                  for g0 in range(0, len(pieces), skv.MAX_SEGMENTS)]
        down = peer(rank + 1)[1]
        done_at = flag(seq.state.base if rank == 0 else peer(0)[1], DONE + receivers)

        def step():
            counter[0] += 1
            for g0, arr in groups:
                wait = flag(seq.state.base, g0) if rank else None
                skv.check(L.skv_copy_chained(arr, len(arr), wait, flag(down, g0), counter[0], wait_ns, sp))
            if rank and rank == receivers - 1:        # the last store into the last receiver has landed
                skv.check(L.skv_signal(done_at, counter[0], sp))
            if rank == 0 and receivers > 1:
                skv.check(L.skv_wait_flag(done_at, counter[0], wait_ns, sp))
    else:
        def step():                                   # the last receiver only receives
            counter[0] += 1
    clear_receiver()
    results["chain_push"] = timed(step) + (parity(),)
    status = torch.tensor([float(skv.query_status(local) != 0)], device="cuda")
    dist.all_reduce(status, op=dist.ReduceOp.MAX)

    b = kg.metric_bytes(t)
    line = None
    if rank == 0:
        methods = {}
        for name, (tot, per, ok) in results.items():
            methods[name] = {"value": round(receivers * b * n_steps / (tot / 1e3) / 1e9, 3),
                             "ms_per_step": round(tot / n_steps, 4),
                             "p50_ms": round(float(np.percentile(per, 50)), 4),
                             "p99_ms": round(float(np.percentile(per, 99)), 4),
                             "per_receiver_gbs": round(b * n_steps / (tot / 1e3) / 1e9, 3), "parity": ok}
        best = "chain_push"   # the reported method, fixed in advance; the others are kept beside it in `methods`
        rate, rate_kind = link_rate(probe)
        m = methods[best]
        line = {"metric": METRIC, "value": m["value"], "unit": UNIT, "n_gpus": world, "steps": n_steps,
                "warmup": args.warmup, "ms_per_step": m["ms_per_step"], "p50_ms": m["p50_ms"], "p99_ms": m["p99_ms"],
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
                "config": {"workload": f"config 4: 1 prefill GPU fans one {t}-token cache out to {receivers} decode "
                                       f"GPUs (independent random tables); reported: the chained push (p2p, nccl "
                                       f"broadcast and chained pull timed beside it)",
                           "tokens": t, "receivers": receivers, "method": best, "chunk_mb": args.chunk_mb,
                           "l2": "inputs larger than L2", "parallelism": f"1 -> {receivers} fan-out"},
                "methods": methods, "parity": all(v["parity"] for v in methods.values()) and status.item() == 0,
                "roofline": {"bound": "nvlink", "achieved": m["per_receiver_gbs"], "peak": rate, "unit": "GB/s",
                             "frac": round(m["per_receiver_gbs"] / rate, 4),
                             "frac_of_nominal_900": round(m["per_receiver_gbs"] / 900.0, 4),
                             "peak_kind": rate_kind + "; each receiver's ingress",
                             "traffic": None, "kernel": "copy_tma_chain_kernel"}}
    torch.cuda.synchronize()
    dist.barrier()
    for pool, state in maps.values():
        skv.ipc_close(pool)
        skv.ipc_close(state)
    dist.barrier()
    return line if rank == 0 else None


# ------------------------------------------------------------------------------------------------ mixed (config 5)

MIXED_SEQUENCES = 64
MIXED_TOKENS = (1024, 131072)      # log-uniform lengths (mean ~26.8K tokens)
SERVE_SLOTS = 8                    # serve slots per decode GPU, parked to and resumed from host during the handoffs
SLOT_TOKENS = 4096


def mixed_plan(world: int, seed: int) -> dict:
    """Config 5's workload, identical on every rank: seeded log-uniform lengths on [1K, 128K], each sequence's
    prefill owner (an even rank) and decode target (an odd rank) drawn at random."""
    rng = np.random.default_rng(seed)
    lo, hi = MIXED_TOKENS
    lengths = np.exp(rng.uniform(np.log(lo), np.log(hi), MIXED_SEQUENCES)).astype(np.int64)
    prefill = [r for r in range(world) if r % 2 == 0]
    decode = [r for r in range(world) if r % 2 == 1]
    return {"lengths": [int(x) for x in lengths], "owner": [int(x) for x in rng.choice(prefill, MIXED_SEQUENCES)],
            "target": [int(x) for x in rng.choice(decode, MIXED_SEQUENCES)]}


def mixed_demand(plan: dict, sizes: list) -> dict:
    """Config 5's bytes per (prefill rank, decode rank)."""
    demand = {}
    for i, (o, d) in enumerate(zip(plan["owner"], plan["target"])):
        demand[(o, d)] = demand.get((o, d), 0) + int(sizes[i])
    return demand


def phased_schedule(plan: dict, sizes: list, world: int) -> dict:
    """Config 5's pulls in port-exclusive phases (handoff_schedule.schedule): prefill ranks (even) are the
    sources, decode ranks (odd) the destinations."""
    return handoff_schedule.schedule(mixed_demand(plan, sizes), [r for r in range(world) if r % 2 == 0],
                                     [r for r in range(world) if r % 2 == 1])


TAIL_FRAC = 0.05   # phased-tail: a phase whose largest run moves less than this share of the busiest port's bytes


def tail_start(sched: dict, frac: float = TAIL_FRAC) -> int | None:
    """The first phase of the schedule's tail: the longest run of LAST phases whose largest run (over every
    destination) moves less than `frac` of the busiest port's bytes; None when the last phase is not that small.
    Waits point only at earlier phases, so no run before the tail waits for a run inside it."""
    weight = {}
    for runs in sched["runs"].values():
        for r in runs:
            weight[r["phase"]] = max(weight.get(r["phase"], 0), r["hi"] - r["lo"])
    start = None
    for k in sorted(weight, reverse=True):
        if weight[k] >= frac * sched["bound_bytes"]:
            break
        start = k
    return start


def phase_runs(rank: int, plan: dict, sizes: list, segs_of: dict, world: int) -> list:
    """Decode GPU `rank`'s runs under phased_schedule, ready to launch (handoff_schedule.launch_list).  `sizes[i]`
    = sequence i's bytes (all 64, for the global schedule); `segs_of[i]` = the segments moving sequence i into this
    GPU (each sequence it receives).  A flow's sequences go shortest first: the cuts are by bytes, so the order
    moves no phase, and most sequences land early."""
    for i, segs in segs_of.items():
        if sum(g.bytes for g in segs) != sizes[i]:
            raise ValueError(f"sequence {i}: its segments move {sum(g.bytes for g in segs)} bytes, not {sizes[i]}")
    flows = {}
    for i in sorted(segs_of, key=lambda i: (plan["lengths"][i], i)):
        flows.setdefault(plan["owner"][i], []).append((i, segs_of[i]))
    return handoff_schedule.launch_list(phased_schedule(plan, sizes, world), rank, flows)


def port_bound(plan: dict, sizes: list, world: int, rate_gbs: float = NVLINK_PEER_COPY_GBS) -> dict:
    """Config 5's schedule-independent bound: the busiest NVLink port's bytes at the measured peer-copy rate."""
    return handoff_schedule.port_bound(mixed_demand(plan, sizes), rate_gbs)


class SeqSet:
    """Several sequences in ONE library-allocated block pool (CUDA-IPC exportable) plus one state arena with each
    sequence's GDN rows and ids (`state_layout` per sequence), every layer's blocks at seed-random slots."""

    def __init__(self, torch, kg: skv.KvGeometry, lengths: list, seed: int, fill: bool):
        dev = torch.cuda.current_device()
        self.kg, self.lengths = kg, list(lengths)
        self.n_blocks = sum(kg.n_qsa * kg.blocks(t) for t in lengths) + 1
        self.pool = skv.Pool(dev, self.n_blocks, kg.block_bytes)
        self.offs, at = [], 0
        for t in lengths:
            self.offs.append(at)
            at += state_layout(kg, t)["bytes"]
        self.state_bytes = max(at, 1024)
        self.state = skv.Pool(dev, 1, self.state_bytes)
        gen = torch.Generator(device="cuda").manual_seed(seed)
        chunk = 256 << 20
        for base, total, floats in ((self.pool.base, self.n_blocks * kg.block_bytes, False),
                                    (self.state.base, self.state_bytes, True)):
            for a in range(0, total, chunk):
                n = min(chunk, total - a)
                if not fill:
                    r = torch.zeros(n, dtype=torch.uint8, device="cuda")
                elif floats:
                    r = torch.randn(n // 4, generator=gen, device="cuda") * 0.02
                else:
                    r = torch.randn(n // 2, generator=gen, device="cuda", dtype=torch.float16)
                skv.copy([skv.segment(r, base + a, n)], skv.COPY_VEC)
                torch.cuda.synchronize()
        self.pool.scramble(seed)
        self.blocks = [np.stack([self.pool.alloc(kg.blocks(t)) for _ in range(kg.n_qsa)]) for t in lengths]
        self.tables = [torch.from_numpy(skv.PooledSequence.host_tables(kg, b).reshape(-1).copy()).cuda()
                       for b in self.blocks]
        self.seqs = [self.view(i, self.pool, self.state.base, self.tables[i]) for i in range(len(lengths))]

    def view(self, i: int, pool: skv.Pool, state_base: int, tables) -> skv.PooledSequence:
        t = self.lengths[i]
        lay = state_layout(self.kg, t)
        return skv.PooledSequence(self.kg, pool, t, self.kg.n_qsa, self.blocks[i] if pool is self.pool else None,
                                  tables, state_base + self.offs[i], state_base + self.offs[i] + lay["ids"])


HANDOVER_WAIT_NS = 5_000_000_000   # every config-5 hand-over wait ends by itself after 5 s of device time


def issue_phase_run(L, arrays: list, wait, done, value: int, sp, gated: bool, on_start, on_end) -> None:
    """Enqueue one run of config 5's phased order on stream `sp`: its copy launches (one per (segment array, count)
    in `arrays`) after the hand-over it waits for (`wait`: a flag address, or None) and before the one it releases
    (`done`, or None), both at `value`.  launch: skv_wait_flag, the copies and skv_signal are launches of their own;
    gated: the wait rides in the first copy launch and the release in the last (skv_copy_gated), so a one-array run
    is a single launch.  on_start / on_end record the run's timing events around its copies (with gated hand-overs
    the wait falls between them)."""
    if gated:
        on_start()
        last = len(arrays) - 1
        for q, (arr, n) in enumerate(arrays):
            w, d = (wait if q == 0 else None), (done if q == last else None)
            if w is None and d is None:
                skv.check(L.skv_copy(arr, n, skv.COPY_TMA, sp))
            else:
                skv.check(L.skv_copy_gated(arr, n, w, value, HANDOVER_WAIT_NS, d, value, sp))
        on_end()
        return
    if wait is not None:
        skv.check(L.skv_wait_flag(wait, value, HANDOVER_WAIT_NS, sp))
    on_start()
    for arr, n in arrays:
        skv.check(L.skv_copy(arr, n, skv.COPY_TMA, sp))
    on_end()
    if done is not None:
        skv.check(L.skv_signal(done, value, sp))


def run_mixed(args, torch, probe: dict | None = None) -> dict | None:
    """Config 5: the even ranks prefill, the odd ranks decode.  64 sequences with seeded log-uniform lengths on
    [1K, 128K] live in their prefill owner's pool; each decode GPU pulls the sequences assigned to it (random
    pairing, so several decode GPUs may want one prefill GPU at once) with skv_copy (TMA, peer loads, no
    multicast) straight into its own pool, in one of three orders (--mixed-order):

      phased      (default) port-exclusive phases from phased_schedule: one stream, each prefill GPU read by one
                  decode GPU at a time, hand-overs by device flags (skv_signal / skv_wait_flag); back-to-back runs
                  from one source with no hand-over between them are one launch (handoff_schedule.fuse_runs;
                  phased-unfused keeps every run a launch of its own; each run's wait and signal ride inside
                  its copy launch, skv_copy_gated, unless --handover launch);
      per-source  one stream per source prefill GPU, one skv_copy per sequence, all sources at once;
      serial      one skv_copy per sequence, back to back.

    Meanwhile a side stream on every decode GPU parks its 8 serve slots (4,096-token conversations) to pinned
    host memory and resumes them (skv_park / skv_resume, staged).  value = all 64 sequences' B(T) per step / the
    max-over-ranks handoff window; a sequence's latency runs from the step's start to its last byte landing."""
    import torch.distributed as dist
    rank, world, local = ranks()
    kg = skv.KvGeometry()
    plan = mixed_plan(world, args.seed)
    lengths, owner, target = plan["lengths"], plan["owner"], plan["target"]
    steps, warmup = min(args.steps, 5), max(1, min(args.warmup, 2))
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    L = skv.lib()
    mine_out = [i for i in range(MIXED_SEQUENCES) if owner[i] == rank]
    mine_in = [i for i in range(MIXED_SEQUENCES) if target[i] == rank]
    decode = rank % 2 == 1
    # prefill side: its sequences resident; decode side: room for what it receives, plus its serve slots
    held = SeqSet(torch, kg, [lengths[i] for i in (mine_in if decode else mine_out)], args.seed + 7 * rank,
                  fill=not decode)
    slots = SeqSet(torch, kg, [SLOT_TOKENS] * (2 * SERVE_SLOTS), args.seed + 7 * rank + 3, fill=True) if decode else None
    phased = args.mixed_order in ("phased", "phased-tail", "phased-unfused")
    gated = phased and args.handover == "gated"
    flags = None
    if decode and phased:            # one 8-byte word per run of this GPU's phased order (phased_schedule)
        flags = skv.Pool(local, 1, 4096)
        zero = torch.zeros(512, dtype=torch.int64, device="cuda")
        skv.copy([skv.segment(zero, flags.base, 4096)], skv.COPY_VEC)
    info = {"flags": skv.ipc_export(flags.base) if flags else None} if decode else {
        "pool": skv.ipc_export(held.pool.base), "state": skv.ipc_export(held.state.base),
        "n_blocks": held.n_blocks, "seqs": mine_out, "offs": held.offs, "blocks": held.blocks}
    torch.cuda.synchronize()
    infos = [None] * world
    dist.all_gather_object(infos, info)
    maps, keep, pulls, segs_of = {}, [], [], {}
    for k, i in enumerate(mine_in if decode else []):
        p = owner[i]
        if p not in maps:
            maps[p] = (skv.ipc_import(local, infos[p]["pool"]), skv.ipc_import(local, infos[p]["state"]))
        pool_base, state_base = maps[p]
        j = infos[p]["seqs"].index(i)
        t = lengths[i]
        blocks = infos[p]["blocks"][j]
        tables = torch.from_numpy(skv.PooledSequence.host_tables(kg, blocks).reshape(-1).copy()).cuda()
        peer_pool = skv.Pool(local, infos[p]["n_blocks"], kg.block_bytes, memory=pool_base)
        lay = state_layout(kg, t)
        src = skv.PooledSequence(kg, peer_pool, t, kg.n_qsa, None, tables, state_base + infos[p]["offs"][j],
                                 state_base + infos[p]["offs"][j] + lay["ids"])
        dst = held.seqs[k]
        segs = skv.kv_segments_pool_to_pool(src, dst) + skv.state_segments(src, dst.gdn, dst.ids)
        keep += [tables, peer_pool]
        pulls.append((i, (skv.Segment * len(segs))(*segs), len(segs)))
        segs_of[i] = segs
    runs, peer_flags = [], {}
    tail_from = None   # phased-tail: the first phase run without hand-overs, on per-source streams
    if decode and phased:
        stream_bytes = lambda t: (2 * kg.n_qsa * kg.pages(t) * kg.page_bytes + kg.gdn_bytes  # noqa: E731
                                  + 16 * ((4 * t + 15) // 16))
        order = phase_runs(rank, plan, [stream_bytes(t) for t in lengths], segs_of, world)
        if args.mixed_order in ("phased", "phased-tail"):
            order = handoff_schedule.fuse_runs(order)
        if args.mixed_order == "phased-tail":
            tail_from = tail_start(phased_schedule(plan, [stream_bytes(t) for t in lengths], world))
        for run in order:
            pieces = run["pieces"]
            arrays = [((skv.Segment * len(pieces[a:a + skv.MAX_SEGMENTS]))(*pieces[a:a + skv.MAX_SEGMENTS]),
                       len(pieces[a:a + skv.MAX_SEGMENTS])) for a in range(0, len(pieces), skv.MAX_SEGMENTS)]
            if run["signal"] and run["signal"][0] not in peer_flags:
                peer_flags[run["signal"][0]] = skv.ipc_import(local, infos[run["signal"][0]]["flags"])
            runs.append(dict(run, arrays=arrays))
    side = torch.cuda.Stream()
    per_source = args.mixed_order == "per-source"
    source_stream = {p: torch.cuda.Stream() for p in sorted(set(owner[i] for i in mine_in))}
    tuning = skv.get_copy_tuning()
    if per_source:
        # one issuing CTA per SM per pull (NVLink-bound, it needs no more) so up to three pulls share the GPU at once
        skv.set_copy_tuning(tuning[0], tuning[1], 1, tuning[3])
    if decode:
        off = skv.image_offsets(kg, SLOT_TOKENS, kg.n_qsa)
        hosts = [skv.HostBuffer(off["total"]) for _ in range(SERVE_SLOTS)]
        staging = torch.empty(off["total"] + 256 * 64, dtype=torch.uint8, device="cuda")
        park_segs = [skv.pack_segments(slots.seqs[j], hosts[j].ptr) for j in range(SERVE_SLOTS)]
        resume_segs = [skv.unpack_segments(hosts[j].ptr, slots.seqs[SERVE_SLOTS + j]) for j in range(SERVE_SLOTS)]
    lat = []       # per-sequence pull times (ms), timed steps
    landed = []    # per-sequence time from the step's start (every sequence ready) to its last byte landing
    windows = []   # (handoff window, park window) per timed step, this rank
    idle = []      # phased: per timed step, the window minus this GPU's copy time
    timeline = []  # phased, --timeline: the last timed step's runs on this GPU
    gc_pause = quiet_gc().__enter__()   # paused for the whole step loop (resumed after it)
    for it in range(warmup + steps):
        dist.barrier()
        torch.cuda.synchronize()
        device_align(torch, dist)
        h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in pulls]
        h0.record(stream)
        side.wait_stream(stream)
        p0.record(side)
        if phased:
            # this GPU's runs in phase order on one stream; a run from a prefill GPU another decode GPU read
            # before waits for that GPU's signal, and each run signals the next reader of its source
            rev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in runs]
            tail_streams = set()
            for j, (run, (a, b)) in enumerate(zip(runs, rev)):
                if tail_from is not None and run["phase"] >= tail_from:
                    # the tail: no hand-over; each run on its source's stream, after this GPU's exclusive runs
                    st = source_stream[run["src"]]
                    if st not in tail_streams:
                        st.wait_stream(stream)
                        tail_streams.add(st)
                    a.record(st)
                    for arr, n in run["arrays"]:
                        skv.check(L.skv_copy(arr, n, skv.COPY_TMA, st.cuda_stream))
                    b.record(st)
                    continue
                wait = flags.base + 8 * run["wait"] if run["wait"] is not None else None
                done = peer_flags[run["signal"][0]] + 8 * run["signal"][1] if run["signal"] is not None else None
                issue_phase_run(L, run["arrays"], wait, done, it + 1, sp, gated,
                                lambda: a.record(stream), lambda: b.record(stream))
            for st in tail_streams:
                stream.wait_stream(st)
            first = {i: rev[j][0] for j in reversed(range(len(runs))) for i in runs[j]["starts"]}
            last = {i: rev[j][1] for j in range(len(runs)) for i in runs[j]["ends"]}
            ev = [(first[i], last[i]) for i, _, _ in pulls]
        for (i, arr, n), (a, b) in zip(pulls, ev) if not phased else ():
            # one stream per source prefill GPU: pulls from different sources run at once, so a source that
            # another decode GPU is also reading does not leave this GPU's NVLink ingress idle
            st = source_stream[owner[i]] if per_source else stream
            if st is not stream:
                st.wait_event(h0)
            a.record(st)
            skv.check(L.skv_copy(arr, n, skv.COPY_TMA, st.cuda_stream))
            b.record(st)
        # the serve-slot parks are enqueued AFTER the pulls: their ~430 launches and copies take the host about a
        # millisecond, which the pulls would otherwise wait out at the start of every step
        if decode:
            for j in range(SERVE_SLOTS):
                skv.park(park_segs[j], skv.PARK_STAGED, staging, staging.numel(), side)
                skv.resume(resume_segs[j], skv.PARK_STAGED, staging, staging.numel(), side)
        p1.record(side)
        for st in set(source_stream.values()) if per_source else ():
            stream.wait_stream(st)
        h1.record(stream)
        torch.cuda.synchronize()
        if it >= warmup:
            windows.append((h0.elapsed_time(h1), p0.elapsed_time(p1)))
            lat += [a.elapsed_time(b) for a, b in ev]
            landed += [h0.elapsed_time(b) for a, b in ev]
            if phased and runs:      # the share of the window this GPU spent waiting for hand-overs
                idle.append(h0.elapsed_time(h1) - sum(a.elapsed_time(b) for a, b in rev))
                timeline = [[round(h0.elapsed_time(a), 3), round(h0.elapsed_time(b), 3), r["hi"] - r["lo"],
                             r["src"], r["phase"], r["wait"] is not None] for r, (a, b) in zip(runs, rev)]
    gc_pause.__exit__()
    skv.set_copy_tuning(*tuning)
    status = torch.tensor([float(skv.query_status(local) != 0)], device="cuda")
    dist.all_reduce(status, op=dist.ReduceOp.MAX)
    win = torch.tensor([w[0] for w in windows], device="cuda")
    dist.all_reduce(win, op=dist.ReduceOp.MAX)
    # parity: every handed-off sequence, packed through the decode GPU's table, equals its prefill original; every
    # resumed serve slot equals the slot it was parked from
    ok = True
    for i in range(MIXED_SEQUENCES):
        p, d = owner[i], target[i]
        if rank == d:
            img = pack_image(torch, held.seqs[mine_in.index(i)])
            dist.send(img, p)
            del img
        elif rank == p:
            img = pack_image(torch, held.seqs[mine_out.index(i)])
            got = torch.empty_like(img)
            dist.recv(got, d)
            ok = ok and bool(torch.equal(img, got))
            del img, got
    if decode:
        for j in range(SERVE_SLOTS):
            ok = ok and bool(torch.equal(pack_image(torch, slots.seqs[j]), pack_image(torch, slots.seqs[SERVE_SLOTS + j])))
    okt = torch.tensor([float(ok)], device="cuda")
    dist.all_reduce(okt, op=dist.ReduceOp.MIN)
    # gather per-rank facts to rank 0
    facts = {"lat": lat, "landed": landed, "park_ms": [w[1] for w in windows], "hand_ms": [w[0] for w in windows],
             "bytes_in": sum(kg.metric_bytes(lengths[i]) for i in mine_in), "decode": decode,
             "idle_ms": round(float(np.mean(idle)), 3) if idle else None, "timeline": timeline, "rank": rank,
             "launches": (sum(len(r["arrays"]) + (not gated) * ((r["wait"] is not None) + (r["signal"] is not None))
                              for r in runs) if phased else len(pulls))}
    allf = [None] * world
    dist.all_gather_object(allf, facts)
    torch.cuda.synchronize()
    dist.barrier()
    del pulls, keep, runs
    for pool_base, state_base in maps.values():
        skv.ipc_close(pool_base)
        skv.ipc_close(state_base)
    for ptr in peer_flags.values():
        skv.ipc_close(ptr)
    dist.barrier()
    if rank != 0:
        return None
    total = sum(kg.metric_bytes(t) for t in lengths)
    rate, rate_kind = link_rate(probe)
    bound = port_bound(plan, [kg.metric_bytes(t) for t in lengths], world, rate)
    wins = win.cpu().numpy()
    value = total * steps / (float(wins.sum()) / 1e3) / 1e9
    lat_all = np.concatenate([np.asarray(f["lat"]) for f in allf if f["lat"]])
    landed_all = np.concatenate([np.asarray(f["landed"]) for f in allf if f["landed"]])
    slot_bytes = 2 * SERVE_SLOTS * kg.metric_bytes(SLOT_TOKENS)
    dec = [f for f in allf if f["decode"]]
    per_decode = [round(f["bytes_in"] / (np.mean(f["hand_ms"]) / 1e3) / 1e9, 1) for f in dec]
    parks = [round(slot_bytes / (np.mean(f["park_ms"]) / 1e3) / 1e9, 2) for f in dec]
    mean_ingress = float(np.mean(per_decode))
    return {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": steps, "warmup": warmup,
            "ms_per_step": round(float(wins.mean()), 4), "p50_ms": round(float(np.percentile(landed_all, 50)), 4),
            "p99_ms": round(float(np.percentile(landed_all, 99)), 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u8", "data": "synthetic",
            "config": {"workload": f"config 5: {world // 2} prefill + {world // 2} decode GPUs, {MIXED_SEQUENCES} "
                                   f"sequences with seeded log-uniform lengths on [1K, 128K] tokens, random "
                                   f"prefill->decode pairing, pulled over NVLink straight into the decode pools while "
                                   f"{SERVE_SLOTS} serve slots of {SLOT_TOKENS} tokens per decode GPU park to and "
                                   f"resume from pinned host memory",
                       "sequences": MIXED_SEQUENCES, "mean_tokens": round(float(np.mean(lengths)), 1),
                       "bytes_per_step": total, "serve_slots": SERVE_SLOTS, "slot_tokens": SLOT_TOKENS,
                       "order": args.mixed_order, **({"handover": args.handover} if phased else {}),
                       "parallelism": f"{world // 2} prefill + {world // 2} decode"},
            **({"timeline": {f["rank"]: f["timeline"] for f in dec}} if args.timeline else {}),
            **({"phases": phase_summary([f["timeline"] for f in dec])} if phased else {}),
            "handoffs": {"per_decode_gpu_gbs": per_decode, "idle_ms_per_decode_gpu": [f["idle_ms"] for f in dec],
                         "landed_p50_ms": round(float(np.percentile(landed_all, 50)), 4),
                         "landed_p99_ms": round(float(np.percentile(landed_all, 99)), 4),
                         "pull_p50_ms": round(float(np.percentile(lat_all, 50)), 4),
                         "pull_p99_ms": round(float(np.percentile(lat_all, 99)), 4),
                         "note": "landed: from the step's start (every sequence ready on its prefill GPU) to the "
                                 "sequence's last byte in the decode pool - the line's p50/p99; pull: the device time "
                                 "from its first byte's copy to its last byte's (concurrent pulls share the links; "
                                 "phased: a sequence may span phases); idle: phased only, the window minus the GPU's "
                                 "copy time (waits for hand-overs, idle padding)"},
            "parks": {"per_decode_gpu_gbs": parks, "bytes_per_step_per_gpu": slot_bytes,
                      "note": "park + resume of every serve slot, staged, on a side stream during the handoffs"},
            "parity": bool(okt.item() == 1.0) and status.item() == 0,
            "gpu_launches": steps * (sum(f["launches"] for f in dec) + len(dec) * SERVE_SLOTS * 2),
            "roofline": {"bound": "nvlink", "achieved": round(mean_ingress, 1), "peak": rate, "unit": "GB/s",
                         "frac": round(mean_ingress / rate, 4),
                         "peak_kind": rate_kind + "; mean decode-GPU ingress over its window",
                         "traffic": None, "kernel": "copy_tma_kernel"},
            "port_bound": dict(bound, frac=round(value / bound["gbs"], 4), rate_gbs=rate, rate_kind=rate_kind,
                               note="the busiest NVLink port's bytes (a prefill GPU's egress or a decode GPU's "
                                    "ingress) at the peer-copy rate: no order of the pulls ends sooner")}


def phase_summary(timelines: list) -> list:
    """Per phase of the port-exclusive order, from the last timed step's runs on every decode GPU (each run
    [start_ms, end_ms, bytes, source, phase, waited], times from that GPU's step start): the phase's bytes, its
    span (earliest start to latest end over the GPUs), the aggregate rate over the span, and its slowest run's
    rate - which phase or boundary limits the step."""
    by_phase = {}
    for runs in timelines:
        for start, end, nbytes, _src, phase, _waited in runs:
            by_phase.setdefault(phase, []).append((start, end, nbytes))
    out = []
    for phase in sorted(by_phase):
        runs = by_phase[phase]
        span = max(e for _, e, _ in runs) - min(a for a, _, _ in runs)
        nbytes = sum(n for _, _, n in runs)
        slowest = min(n / max(e - a, 1e-6) / 1e6 for a, e, n in runs)
        out.append({"phase": phase, "runs": len(runs), "bytes": nbytes, "span_ms": round(span, 3),
                    "gbs": round(nbytes / max(span, 1e-6) / 1e6, 1), "slowest_run_gbs": round(slowest, 1)})
    return out


def pack_image(torch, ps: skv.PooledSequence):
    """A sequence packed through its own table (K/V, GDN rows, ids) by the gather kernel."""
    off = skv.image_offsets(ps.g, ps.tokens, ps.layers)
    image = torch.zeros(off["total"], dtype=torch.uint8, device="cuda")
    skv.copy(skv.pack_segments(ps, image), skv.COPY_TMA)
    torch.cuda.synchronize()
    return image


def device_align(torch, dist) -> None:
    """Line the GPUs up on the device before a multi-GPU timed region: a one-element all-reduce that the current
    stream waits for, so each GPU's next operation (the timing event, then the first step) starts when the last rank
    has reached this point.  Without it the ranks' host skew after the barrier lands in the first timed step (a
    prefill GPU starts its clock while its decode rank has not launched yet).  Every rank calls it at the same
    points."""
    t = torch.ones(1, device="cuda" if torch.cuda.is_available() else "cpu")
    dist.all_reduce(t)


def ranks() -> tuple:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    return rank, world, int(os.environ.get("LOCAL_RANK", rank))


def brief(line: dict | None, keys=("value", "ms_per_step", "p50_ms", "p99_ms", "parity")) -> dict | None:
    """The headline fields of a scenario's line, plus its config and method table, for embedding."""
    if line is None:
        return None
    out = {k: line[k] for k in keys if k in line}
    for k in ("config", "methods", "roofline", "handoffs", "parks", "port_bound", "phases"):
        if k in line:
            out[k] = line[k]
    return out


def apply_tuning(spec: str | None) -> None:
    """--tuning: set the copy-engine geometry for the whole run (the line's config records it)."""
    if not spec:
        return
    parts = [int(x) for x in spec.split(",")]
    cur = skv.get_copy_tuning()
    stages, tile, ctas = parts[:3]
    vec = parts[3] if len(parts) > 3 else cur[3]
    skv.set_copy_tuning(stages, tile, ctas, vec)


def main() -> None:
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    apply_tuning(args.tuning)
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world == 1 and args.scenario == "p2p-local":
        run_p2p_local(args, torch)
        return
    if world == 1:
        run_single(args, torch)
        return
    import torch.distributed as dist
    from datetime import timedelta
    rank, world, local = ranks()
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    try:
        if args.scenario == "fanout":
            line = run_fanout(args, torch)
        elif args.scenario == "mixed":
            line = run_mixed(args, torch)
        else:
            # the headline: N/2 pairs (configs 3/5 throughput, weak scaling); at N = 4 and N = 8 the same run also
            # measures BASELINE's own 4- and 8-GPU configs and embeds them
            line, probe = run_pairs(args, torch)
            if args.scenario in ("auto", "sweep") and world == 2:
                sweep = pair_sweep(args, torch, probe, line)
                if line is not None:
                    line["config3_sweep"] = sweep
            if args.scenario == "auto" and world == 2:
                roles = split_roles(torch, rank)
                if line is not None:
                    line["split_roles_device_descriptor"] = roles
            if args.scenario == "auto" and world == 4:
                sub = run_fanout(args, torch, tokens=65536, steps=min(args.steps, 40), probe=probe)
                if line is not None:
                    line["config4_fanout"] = brief(sub)
            if args.scenario == "auto" and world == 8:
                sub = run_mixed(args, torch, probe=probe)
                if line is not None:
                    line["config5_mixed"] = brief(sub)
        if rank == 0 and line is not None:
            print(json.dumps(line))
    finally:
        torch.cuda.synchronize()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
