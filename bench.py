"""Benchmark of the LAL decode tail on B200 -- prints ONE JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2_qwen]
    python bench.py --impl reference ...

A step is one decode-tail pass (quantize hidden, int8 LM head over all vocab
rows, repetition penalty, top-k, temperature softmax, draw, history push) for
the B streams of the config, on seeded synthetic inputs with the BASELINE
shapes (no real weights exist for this path).  Default workload: c2_qwen, the
Qwen2.5-7B-shaped tail at B=1 (V=152064, d=3584, 545 MB int8 LM head).

Reported:
  value      tokens/s with the step's inputs already in HBM (CUDA events on the
             context's stream around the K timed steps)
  e2e        tokens/s through the public C ABI (lal_tail_step) from host
             buffers: H2D of hidden + draws and D2H of tokens + status inside
             the timed region, host wall clock per call
  roofline   the fused kernel's algorithmic bytes per launch / its average
             duration (CUDA events per launch), against MEASURED_PEAKS.json
  cpu_baseline  the reference's own C (oracle/_ref: quantize, |xq|, OpenMP
             LM head, lal_sample_token) on the host's cores, bounded sample

Before the timed region: W warm-up steps through the public call, then about
0.3 s of untimed device steps (the same count on every rank).

Multi-GPU (torchrun, --gpus N): each rank owns a contiguous vocab slice
(vocab-sharded, strong scaling: a step is the same B tokens at any N).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from lal_b200 import synth  # noqa: E402

METRIC = "Qwen7B LM-head+top-k tail tokens/s at B=1/64, % HBM BW peak, 1/2/4/8 B200"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
L2_BYTES = 126 << 20


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--config", default="c2_qwen", choices=sorted(synth.CONFIGS))
    ap.add_argument("--sampler", default="library", choices=["library", "server", "gpt2"],
                    help="the fused context's sampler: lal_sampling.h (default), the "
                         "Qwen server's, or the GPT-2 server's tail (one GPU)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=12.0,
                    help="bound of the CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def algorithmic_bytes(cfg, B, rows=None):
    """Per step: int8 W + fp32 row scales (this slice) + per stream fp32 hidden,
    int32 history and the int32 token (logits stay on chip / in L2)."""
    V = cfg.vocab if rows is None else rows
    return V * cfg.n_embd + 4 * V + B * (4 * cfg.n_embd + 4 * cfg.hist + 4)


def cpu_gbs(cfg, tokens_per_s):
    """A CPU rate as the algorithmic bytes of the whole vocabulary it streams:
    (V*d + 4V + B*(4d + 4H + 4)) per step of B tokens, in GB/s."""
    return round(tokens_per_s / cfg.streams * algorithmic_bytes(cfg, cfg.streams) / 1e9, 3)


INT8_DENSE_TOPS_NOMINAL = 4500.0  # B200 dense int8 (no measured int8 figure)


def tensor_roofline(cfg, B, rows, kern_ms):
    """int8 tensor-core rate of the batched GEMM: 2*B*rows*d ops per launch."""
    ops = 2.0 * B * rows * cfg.n_embd
    achieved = ops / (kern_ms * 1e-3) / 1e12
    return {"achieved": round(achieved, 1), "peak": INT8_DENSE_TOPS_NOMINAL, "unit": "TOPS",
            "frac": round(achieved / INT8_DENSE_TOPS_NOMINAL, 4),
            "note": "of nominal dense int8 (MEASURED_PEAKS.json has no int8 figure)"}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


def load_traffic(cfg_name, n_gpus):
    """dram read+write bytes per launch of the fused kernel from the committed
    ncu summary (profiles/traffic.json), or None."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        d = json.load(f)
    return d.get(f"{cfg_name}@{n_gpus}")


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled every `ms` milliseconds.
    Started (and its first sample awaited, at most 5 s) before the untimed
    warm-up, so that nvidia-smi's start-up is over before the timed region;
    mark() at the region's start drops the samples taken before it."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, ms: int = 20):
        self.gpu = gpu_index
        self.ms = ms
        self.proc = None
        self.lines = []
        self.skip = 0
        self.out = ""

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line)

    def _kill(self):
        if self.proc and self.proc.poll() is None:
            self.proc.kill()

    def __enter__(self):
        import atexit
        import threading
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", str(self.ms)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return self
        atexit.register(self._kill)
        threading.Thread(target=self._read, daemon=True).start()
        t0 = time.time()
        while not self.lines and time.time() - t0 < 5.0 and self.proc.poll() is None:
            time.sleep(0.01)
        return self

    def mark(self):
        """The timed region starts: earlier samples are left out of summary()."""
        self.skip = len(self.lines)

    def __exit__(self, *a):
        if self.proc:
            time.sleep(2.5 * self.ms / 1000.0)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        self.out = "".join(self.lines[self.skip:])

    def summary(self):
        rows = []
        for line in (self.out or "").splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                rows.append(dict(sm=float(f[1]), max=float(f[2]), hw=f[5], hwt=f[6], swt=f[7],
                                 pcap=f[8]))
            except ValueError:
                continue
        if not rows:
            return None
        reasons = set()
        for r in rows:
            for k, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"),
                            ("swt", "sw_thermal_slowdown"), ("pcap", "sw_power_cap")):
                if r[k].lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in rows),
                "sm_max_mhz": max(r["max"] for r in rows), "reasons": sorted(reasons),
                "samples": len(rows)}


# ---------------------------------------------------------------- CPU arm ---

def quantized_lm_head_host(cfg, rows=None):
    """int8 LM head + scales on the host, quantized by the reference's own
    lal_quantize_q8_per_row (oracle/_ref) when built, else the restatement."""
    import oracle
    V = cfg.vocab
    q = np.empty((V, cfg.n_embd), np.int8)
    s = np.empty(V, np.float32)
    which = "ref" if oracle.have_ref() else "port"
    step = 8192
    for r0 in range(0, V, step):
        r1 = min(V, r0 + step)
        q[r0:r1], s[r0:r1] = oracle.quantize_rows(synth.lm_head_f32(cfg, r0, r1), which)
    return q, s


def cpu_tail_gpt2(cfg, q, s, steps, threads, seconds):
    """Time the GPT-2 server's tail on the host: its own lm_head_int8_parallel
    (oracle/_ref, the int8 logits and the float re-score; the server caps its
    threads at 8) and the restated sampler with the recent-token ring.  The
    server's sampler sits inside its forward function, so the sampler is
    always the restatement ('reference' names the LM head's origin)."""
    import oracle
    V, d = cfg.vocab, cfg.n_embd
    ref = oracle.have_ref_gpt2() and (V, d) == (50257, 768)
    g = np.random.default_rng(cfg.seed)
    loops = [oracle.Gpt2PortLoop(q, s, synth.history(cfg, b), max(1, cfg.hist),
                                 float(synth.temperatures(cfg)[b]), cfg.top_k, cfg.rep_penalty)
             for b in range(cfg.streams)]
    nt = min(8, threads)
    done, t_tot = 0, 0.0
    for step in range(steps):
        hid = synth.hidden(cfg, step)
        t0 = time.perf_counter()
        for b, lp in enumerate(loops):
            u = np.float32(g.integers(0, 1000000) / 1e6)
            if ref:
                logits, _ = oracle.gpt2_lm_head(hid[b], q, s, "ref", n_threads=nt)
                tok, _, lp.logits = oracle.gpt2_sample(logits, lp.T, lp.k, lp.p,
                                                       lp.rec[:lp.n.value], u)
                oracle.port().orc_recent_push(lp.rec, oracle.C.byref(lp.n), lp.cap, int(tok))
            else:
                lp.step(hid[b], u)
        t_tot += time.perf_counter() - t0
        done += 1
        if t_tot > seconds:
            break
    return cfg.streams * done / t_tot, "reference" if ref else "port", done, nt if ref else 1


def cpu_tail(cfg, q, s, steps, threads, seconds, sampler="library"):
    """Time the reference's decode tail (qwen7b_server.c:829-850) on the host:
    oracle/_ref when built ('reference'), else the C restatement ('port').
    Runs at most `steps` steps or `seconds` of work per stream.  Returns
    (tokens/s, kind, steps done, cores)."""
    import ctypes as C

    import oracle
    if sampler == "gpt2":
        return cpu_tail_gpt2(cfg, q, s, steps, threads, seconds)
    B = cfg.streams
    V, d = cfg.vocab, cfg.n_embd
    # lal_sample_token's heap holds 64 (lal_sampling.h:74): larger k runs on
    # the uncapped restatement
    kind = "reference" if oracle.have_ref() and min(cfg.top_k, V) <= 64 else "port"
    temps = synth.temperatures(cfg)
    draws = synth.Draws(cfg)
    cap = max(1, cfg.hist)
    pad = max(32, -(-d // 32) * 32)
    xq = np.zeros(pad, np.int8)
    ax = np.zeros(pad, np.uint8)
    logits = np.zeros(V, np.float32)
    hists, loops = [], []
    for b in range(B):
        h0 = synth.history(cfg, b)
        rec = np.zeros(cap, np.int32)
        rec[:h0.size] = h0
        hists.append((rec, C.c_int(h0.size)))
        if kind == "port":
            loops.append(oracle.PortLoop(q, s, h0, cap, float(temps[b]), cfg.top_k,
                                         cfg.rep_penalty, 0))
    if kind == "reference":
        R = oracle.ref()
        if cfg.draws == "rand":
            R.ref_srand(cfg.seed)
    done = 0
    t_tot = 0.0
    for step in range(steps):
        hid = synth.hidden(cfg, step)
        t0 = time.perf_counter()
        for b in range(B):
            if kind == "reference":
                rec, n = hists[b]
                R.ref_tail_step(hid[b], xq, ax, logits, q.reshape(-1), s, V, d,
                                np.float32(temps[b]), cfg.top_k, np.float32(cfg.rep_penalty),
                                rec, C.byref(n), cap, threads, 0)
            else:
                loops[b].step(hid[b], draws.u(b))
        t_tot += time.perf_counter() - t0
        done += 1
        if t_tot > seconds:
            break
    return B * done / t_tot, kind, done, threads


def host_cpu():
    """The host CPU's model name and logical CPU count."""
    model = "unknown"
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"model": model, "nproc": os.cpu_count()}


def run_reference_arm(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    q, s = quantized_lm_head_host(cfg)
    # warm-up, then the timed steps (each a full step of the workload; bounded
    # by --cpu-seconds of host time)
    cpu_tail(cfg, q, s, max(1, min(args.warmup, 2)), threads, 5.0, args.sampler)
    val, kind, done, cores = cpu_tail(cfg, q, s, args.steps, threads, args.cpu_seconds * 2,
                                      args.sampler)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(val, 3), "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": done, "warmup": args.warmup,
        "ms_per_step": round(1000.0 * cfg.streams / val, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {**workload(cfg, args.gpus),
                   **({"sampler": args.sampler} if args.sampler != "library" else {})},
        "cpu_baseline": {"value": round(val, 3), "unit": "tokens/s", "cores": cores,
                         "kind": kind, "host": host_cpu(), "gbs": cpu_gbs(cfg, val),
                         "sample": f"{done} full decode-tail steps of {cfg.name} "
                                   + ("(gpt2_server.c's lm_head_int8_parallel and the "
                                      "restated sampler of :2862-3013)"
                                      if args.sampler == "gpt2" else
                                      "(reference tail sequence of qwen7b_server.c:829-850)")},
        "e2e": {"value": round(val, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    emit(line)


def workload(cfg, n):
    return {"workload": f"{cfg.name}: V={cfg.vocab} d={cfg.n_embd} B={cfg.streams} "
                        f"top_k={cfg.top_k} H={cfg.hist} p={cfg.rep_penalty}",
            "vocab": cfg.vocab, "n_embd": cfg.n_embd, "streams": cfg.streams,
            "top_k": cfg.top_k, "history": cfg.hist, "parallelism": f"vocab-sharded x{n}",
            "l2": l2_policy(cfg, n)}


def lm_head_copies(cfg, n):
    """Copies of a rank's LM-head slice used in turn so that one rotation
    covers at least twice L2 (1: the slice alone is that large).  Only the
    single-stream step rotates; batched steps keep the L2 flush."""
    slice_bytes = (cfg.vocab // n) * cfg.n_embd
    if slice_bytes >= 2 * L2_BYTES or cfg.streams > 1:
        return 1
    return -(-2 * L2_BYTES // slice_bytes)


def l2_policy(cfg, n):
    slice_bytes = (cfg.vocab // n) * cfg.n_embd
    if slice_bytes >= 2 * L2_BYTES:
        return (f"inputs larger than L2: each rank streams a {slice_bytes / 1e6:.0f} MB LM-head "
                f"slice per step (L2 126 MB), steps back to back")
    c = lm_head_copies(cfg, n)
    if c > 1:
        return (f"inputs larger than L2: each rank steps through {c} identical device copies "
                f"of its {slice_bytes / 1e6:.0f} MB LM-head slice in turn "
                f"({c * slice_bytes / 1e6:.0f} MB a rotation against the 126 MB L2), so every "
                f"step streams its slice from HBM; steps back to back")
    return (f"L2 flushed before each timed step: a 512 MB read on the tail's stream "
            f"(the {slice_bytes / 1e6:.0f} MB slice could stay in the 126 MB L2)")


# ---------------------------------------------------------------- GPU arm ---

def run_ours(args, cfg):
    import torch

    import lal_b200 as L

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    B = cfg.streams
    K, W = args.steps, args.warmup
    sampler = {"library": L.LAL_SAMPLER_LIBRARY, "server": L.LAL_SAMPLER_SERVER,
               "gpt2": L.LAL_SAMPLER_GPT2}[args.sampler]
    if args.sampler == "gpt2" and world > 1:
        raise SystemExit("--sampler gpt2 runs on one GPU (the GPT-2 tail has no sharded step)")
    if world > 1:
        from lal_b200.sharded import ShardedDecodeTail
        # vocab slice per rank; records all-gathered over NCCL each step
        t = ShardedDecodeTail(cfg.vocab, cfg.n_embd, device=local, max_streams=B,
                              max_top_k=max(cfg.top_k, 1), history_cap=cfg.hist,
                              sampler=sampler)
    else:
        t = L.DecodeTail(cfg.vocab, cfg.n_embd, max_streams=B, max_top_k=max(cfg.top_k, 1),
                         history_cap=cfg.hist, sampler=sampler, device=local)
    # LM head slice: fp32 rows generated in blocks, quantized on the GPU
    blk = 8192
    for r in range(0, t.n_rows, blk):
        n = min(blk, t.n_rows - r)
        t.load_lm_head_f32(synth.lm_head_f32(cfg, t.row0 + r, t.row0 + r + n), r)
    temps = synth.temperatures(cfg)
    t.set_sampling(temps, [cfg.top_k] * B, [cfg.rep_penalty] * B)
    for b in range(B):
        t.set_history(b, synth.history(cfg, b))
    draws = synth.Draws(cfg)
    nsteps = W + 2 * K
    hid = np.stack([synth.hidden(cfg, i) for i in range(nsteps)]).astype(np.float32)
    us = np.array([[draws.u(b) for b in range(B)] for _ in range(nsteps)], np.float32)

    stream = torch.cuda.ExternalStream(t.stream(), device=local)
    # steps run back to back when this rank's slice is at least twice L2
    # (126 MB), or when the single-stream step rotates copies of a smaller
    # slice that together are; otherwise a 512 MB read evicts the slice
    # before each step
    slice_bytes = t.n_rows * cfg.n_embd
    copies = lm_head_copies(cfg, world)
    if copies > 1:
        t.set_lm_head_copies(copies)
    flush = (torch.ones(128 << 20, dtype=torch.float32, device=local)
             if slice_bytes * copies < 2 * L2_BYTES else None)
    flush_out = torch.empty((), dtype=torch.float32, device=local)

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()

    align = torch.zeros(1, device=local) if dist is not None else None

    def evict_and_align():
        """Untimed, on the tail's stream: evict the slice from L2, then (N > 1)
        a one-element all-reduce so that every rank starts the step together
        (the host enqueues it all ahead, so no idle time is timed)."""
        with torch.cuda.stream(stream):
            torch.sum(flush, 0, out=flush_out)
            if align is not None:
                dist.all_reduce(align)

    # clocks sampled from here on; the summary keeps the timed region's samples
    clk = ClockSampler(local)
    clk.__enter__()

    # warm-up through the public call
    for i in range(W):
        t.step(hid[i], us[i])

    d_hid = torch.from_numpy(hid[W:W + K]).to(local)
    d_u = torch.from_numpy(us[W:W + K]).to(local)
    d_tok = torch.empty((K, B), dtype=torch.int32, device=local)
    # Untimed device steps for about WARM_S seconds before the timed region:
    # the first process on a freshly leased GPU ran its back-to-back steps ~9%
    # slower without them (C2: 102-103 us a step against 93-94 us; 0.3 s of
    # steps removed it, later processes never showed it). Rank 0's clock
    # decides after each chunk and the decision is all-reduced, so every rank
    # takes the same number of steps (the sharded step exchanges records).
    WARM_S, chunk = 0.3, 64
    go = torch.ones(1, dtype=torch.int32, device=local)
    t_w = time.perf_counter()
    while True:
        for j in range(chunk):
            i = j % K
            t.step_device(d_hid[i].data_ptr(), B, d_u[i].data_ptr(), d_tok[i].data_ptr())
        t.sync()
        go.fill_(int(rank != 0 or time.perf_counter() - t_w < WARM_S))
        if dist is not None:
            dist.all_reduce(go, op=dist.ReduceOp.MIN)
        if not int(go.item()):
            break

    # ---- value: inputs resident in HBM, device-timed ----
    n_ev = 1 if flush is None else K
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(n_ev)]
    barrier()
    clk.mark()
    try:  # the timed region and the roofline pass, clocks sampled throughout
        if flush is None:
            # back-to-back steps (the slice is larger than L2): one bracket
            ev[0][0].record(stream)
            for i in range(K):
                t.step_device(d_hid[i].data_ptr(), B, d_u[i].data_ptr(), d_tok[i].data_ptr())
            ev[0][1].record(stream)
        else:
            # the slice could stay in L2: a 512 MB read on the same stream
            # evicts it before each step, and the ranks line up, outside the
            # step's event pair (the host enqueues the step meanwhile: no idle
            # gap is timed)
            for i in range(K):
                evict_and_align()
                ev[i][0].record(stream)
                t.step_device(d_hid[i].data_ptr(), B, d_u[i].data_ptr(), d_tok[i].data_ptr())
                ev[i][1].record(stream)
        t.sync()
        barrier()
        dev_ms = sum(a.elapsed_time(b) for a, b in ev)

        # ---- kernel duration for the roofline: the same steps again with a
        # CUDA-event pair around every fused launch on the context's stream ----
        t.set_timing(True)
        t.kernel_time()
        for i in range(K):
            if flush is not None:
                evict_and_align()
            t.step_device(d_hid[i].data_ptr(), B, d_u[i].data_ptr(), d_tok[i].data_ptr())
        t.sync()
        kern_ms, n_launch = t.kernel_time()
        t.set_timing(False)
        barrier()
    finally:
        clk.__exit__(None, None, None)

    # ---- exchange share (N > 1, peer exchange): phase stamps of each step's
    # last CTA -- its record published, every rank's record arrived, merged
    # and drawn -- on the same back-to-back steps, read after each step ----
    peer = world > 1 and getattr(t, "p2p", False) and B == 1
    exch = None
    if peer:
        t.debug_phases(True)
        wait_us, merge_us = [], []
        for i in range(min(K, 100)):
            t.step_device(d_hid[i].data_ptr(), B, d_u[i].data_ptr(), d_tok[i].data_ptr())
            t.sync()
            _, last = t.phase_times()
            if last[5] and last[6] and last[7]:
                wait_us.append((last[6] - last[5]) / 1e3)
                merge_us.append((last[7] - last[5]) / 1e3)
        t.debug_phases(False)
        barrier()
        if merge_us:
            exch = {"publish_to_all_records_us": round(statistics.median(wait_us), 2),
                    "publish_to_token_us": round(statistics.median(merge_us), 2)}

    # ---- e2e: host buffers through the C ABI's lal_tail_step (bound once;
    # the step's hidden, draws and tokens are host arrays) ----
    barrier()
    e2e_s = 0.0
    c_step = L.lib().lal_tail_step if (world == 1 or peer) else None
    tok_host = np.empty(B, np.int32)
    ptr = lambda a: a.__array_interface__["data"][0]  # noqa: E731
    for i in range(K):
        if flush is not None:
            torch.sum(flush, 0, out=flush_out)
            torch.cuda.synchronize()
            if dist is not None:
                dist.barrier()  # every rank calls the step together (untimed)
        h = hid[W + K + i]
        u = us[W + K + i]
        hp, up, tp = ptr(h), ptr(u), ptr(tok_host)
        if c_step is not None:
            t0 = time.perf_counter()
            rc = c_step(t.h, hp, B, up, tp)
            e2e_s += time.perf_counter() - t0
            if rc:
                raise L.LalTailError(rc, L.lib().lal_tail_last_error().decode())
        else:
            t0 = time.perf_counter()
            t.step(h, u)
            e2e_s += time.perf_counter() - t0
    barrier()

    # max over ranks
    vals = torch.tensor([dev_ms, e2e_s * 1000.0, kern_ms], dtype=torch.float64, device=local)
    if dist is not None:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    dev_ms, e2e_ms, kern_ms = vals.tolist()

    out = None
    if rank == 0:
        peaks, pk_kind = load_peaks()
        rows = t.n_rows
        kind = t.step_kind(B)
        gpt2 = kind == "gpt2"
        batched = kind == "batched"
        if gpt2:
            # the GPT-2 server's tail: LM head with its quantizer (the timed
            # kernel), the 512-candidate select, the float re-score + sampler
            launches_per_step = 3 * B
            alg = algorithmic_bytes(cfg, 1, rows)
            kname = ("LM-head kernel (tail_kernel<MODE_LMHEAD>), one of the GPT-2 tail's three "
                     "launches a step")
        elif batched:
            # quantize + tensor-core GEMM + per-stream select: the GEMM streams
            # the slice once for all B streams (the timed kernel)
            launches_per_step = 3
            alg = algorithmic_bytes(cfg, B, rows)
            kname = "tcgen05 kind::i8 GEMM (gemm_i8_kernel)"
        else:
            # one fused launch per stream: it streams this slice's W and scales
            # once and reads / writes one stream's hidden, history and token
            launches_per_step = B
            alg = algorithmic_bytes(cfg, 1, rows)
            kname = "fused tail kernel (tail_kernel<MODE_FUSED>)"
        if world > 1 and not peer:
            launches_per_step += 1  # the merge (the NCCL all-gather is not ours)
        achieved = alg / (kern_ms * 1e-3) / 1e9
        # lal_tail_step hands the token back through a mapped completion word
        # (the library's own samplers, unsharded or peer-exchange steps)
        notified = not gpt2 and (world == 1 or peer)
        peak = float(peaks["hbm_gbs"])
        traffic = load_traffic(cfg.name, world)
        tokens = K * B
        out = {
            "metric": METRIC, "value": round(tokens / (dev_ms * 1e-3), 3), "unit": "tokens/s",
            "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": round(dev_ms / K, 5),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int8", "data": "synthetic",
            "config": {**workload(cfg, world),
                       **({"sampler": args.sampler} if args.sampler != "library" else {})},
            "e2e": {"value": round(tokens / (e2e_ms * 1e-3), 3), "unit": "tokens/s",
                    # unsharded, or one stream on peer-connected shards:
                    # hidden + draws + the step number pulled from pinned
                    # memory, one 8-byte completion word per stream written
                    # back; otherwise copies of hidden + draws up and of the
                    # tokens + status word down
                    "h2d_bytes_per_step": int(hid[0].nbytes + us[0].nbytes
                                              + (4 if notified else 0)),
                    "d2h_bytes_per_step": int(8 * B if notified else 4 * B + 4),
                    "path": "lal_tail_step (C ABI) from host arrays" if c_step is not None
                            else "ShardedDecodeTail.step (stage, select, NCCL all-gather, "
                                 "merge, fetch)"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1),
                         "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": traffic,
                         "note": f"{kname}; {alg} algorithmic bytes per launch on "
                                 f"rank 0's slice ({rows} rows); peak {pk_kind} "
                                 f"(MEASURED_PEAKS.json hbm_gbs)"},
            "gpu_launches": int(K * launches_per_step),
            **({"exchange": "peer: each rank's last CTA writes its candidate record into every "
                            "rank's buffer over NVLink and merges (one kernel per step)"
                if peer else "NCCL all-gather of the candidate records + merge kernel"}
               if world > 1 else {}),
            **({"exchange_time": {**exch,
                                  "share_of_step": round(exch["publish_to_token_us"]
                                                         / (1e3 * dev_ms / K), 4),
                                  "what": "rank 0's last CTA, median over steps: from its "
                                          "record published to every rank's record arrived, "
                                          "and to its token drawn (the merge)"}}
               if exch else {}),
            **({"tensor": tensor_roofline(cfg, B, rows, kern_ms)} if batched else {}),
            "kernel_ms": round(kern_ms, 5),
            "step_kind": kind,
            "clocks": clk.summary(),
        }
    # ---- CPU baseline (rank 0, N=1 only) ----
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        q, s = t.read_lm_head()
        val, kind, done, cores = cpu_tail(cfg, q, s, 10_000, os.cpu_count() or 1,
                                          args.cpu_seconds, args.sampler)
        val1, _, done1, _ = cpu_tail(cfg, q, s, 10_000, 1, args.cpu_seconds / 2, args.sampler)
        out["cpu_baseline"] = {"value": round(val, 3), "unit": "tokens/s", "cores": cores,
                               "kind": kind, "gbs": cpu_gbs(cfg, val),
                               "sample": f"{done} decode-tail steps of {cfg.name} "
                                         f"(~{args.cpu_seconds:.0f} s bound)",
                               "one_thread": {"value": round(val1, 3), "unit": "tokens/s",
                                              "cores": 1, "gbs": cpu_gbs(cfg, val1),
                                              "sample": f"{done1} steps "
                                                        f"(~{args.cpu_seconds / 2:.0f} s bound)"},
                               "host": host_cpu()}
    if out is not None:
        emit(out)
    t.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


_RESULT_OUT = None


def emit(line: dict):
    """The one JSON line, on the process's real stdout."""
    out = _RESULT_OUT or sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def main():
    global _RESULT_OUT
    # libraries (NCCL's version banner, ...) may print to fd 1: keep a private
    # handle on the real stdout for the result line, send fd 1 to stderr
    sys.stdout.flush()
    _RESULT_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    args = parse()
    cfg = synth.CONFIGS[args.config]
    if args.impl == "reference":
        run_reference_arm(args, cfg)
    else:
        run_ours(args, cfg)


if __name__ == "__main__":
    main()
