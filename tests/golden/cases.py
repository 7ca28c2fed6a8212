"""Seeded input cases shared by make_golden.py (which runs the reference on
them) and the tests (which run the oracle and the GPU on them).

Every input is a pure function of the case's seed, so the committed fixture
holds outputs and input hashes only.
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from lal_b200 import synth  # noqa: E402


def _rng(*seed):
    return np.random.Generator(np.random.PCG64(np.random.SeedSequence(list(seed))))


def quantize_x_inputs():
    """Vectors for lal_quantize_x_int8: both shapes, n%8 tails (truncation),
    the 1e-8 scale floor, exact .5 products (round-half-even vs truncation)."""
    g = _rng(11)
    xs = []
    for n in (768, 3584):
        x = g.standard_normal(n).astype(np.float32)
        x[g.choice(n, n // 100, replace=False)] *= 16
        xs.append(x)
    for n in (100, 37, 8, 1, 4099):
        xs.append((g.standard_normal(n) * 3).astype(np.float32))
    xs.append(np.zeros(64, np.float32))
    xs.append((g.standard_normal(48) * 1e-12).astype(np.float32))
    # max |x| = 127 -> scale 1, inv 1: every k + 0.5 is exact, exercising RNE
    half = (np.arange(-60, 61, dtype=np.float32) + np.float32(0.5)).astype(np.float32)
    half[0] = 127.0
    xs.append(half)
    return xs


def rms_norm_inputs():
    """(x, w, eps) for the final RMSNorm (runtime/lal_simd_optim.h:32-58): both
    model widths, other multiples of 8 (the only lengths with a fixed sum
    order: see orc_rms_norm), tiny and large scales, the 4096 limit."""
    g = _rng(23)
    out = []
    for n, scale, eps in ((3584, 1.0, 1e-6), (3584, 40.0, 1e-6), (768, 3.0, 1e-5),
                          (776, 0.5, 1e-6), (16, 7.0, 1e-6), (8, 2.0, 0.0),
                          (4096, 1e-3, 1e-6), (64, 1e-20, 1e-6)):
        x = (g.standard_normal(n) * scale).astype(np.float32)
        w = (1.0 + 0.25 * g.standard_normal(n)).astype(np.float32)
        out.append((x, w, np.float32(eps)))
    return out


def gpt2_lm_inputs():
    """(name, q, s, x) for the GPT-2 server's LM head (V=50257, d=768, the
    sizes its source fixes): the synthetic C1 head, and the same head with the
    row at place 505 copied over 20 rows ranked below it, so that 21 rows tie
    at the 512th largest logit and the server's heap history decides which 8
    of them it re-scores."""
    import oracle
    from lal_b200 import synth
    cfg = synth.CONFIGS["c1_gpt2"]
    q, s = oracle.quantize_rows(synth.lm_head_f32(cfg), "port")
    x = synth.hidden(cfg, 3)[0]
    out = [("plain", q, s, x)]
    sx, xq = oracle.gpt2_quantize_x(x, "port")
    lg = (sx * s) * (q.astype(np.int32) @ xq.astype(np.int32)).astype(np.float32)
    order = np.argsort(-lg, kind="stable")
    src = order[504]
    q2, s2 = q.copy(), s.copy()
    for r in order[600:620]:
        q2[r] = q[src]
        s2[r] = s[src]
    out.append(("boundary_ties", q2, s2, x))
    return out


def lm_head_inputs():
    """(W fp32 [V,d], x fp32 [d], [(v0, v1), ...]) for the LM-head kernels."""
    out = []
    for i, (V, d, ranges) in enumerate([
        (67, 96, [(0, 67), (5, 60), (66, 67)]),
        (1000, 768, [(0, 1000), (123, 877)]),
        (301, 100, [(0, 301), (7, 8)]),
        (64, 3584, [(0, 64)]),
    ]):
        g = _rng(21, i)
        W = (g.standard_normal((V, d)) * 0.02).astype(np.float32)
        W[min(3, V - 1)] = 0.0                      # all-zero row: scale floor
        x = g.standard_normal(d).astype(np.float32)
        x[g.choice(d, max(1, d // 200), replace=False)] *= 16
        out.append((W, x, ranges))
    return out


def sampler_cases():
    """Sampler parameter sets (both reference variants)."""
    cs = []
    seed = 100
    for V, T, k, p, nrec, kind in [
        (1000, 0.8, 40, 1.1, 64, "normal"),
        (1000, 0.7, 40, 1.1, 256, "normal"),
        (1000, 1.3, 1, 1.1, 10, "normal"),
        (1000, 0.8, 64, 1.3, 300, "dups"),
        (997, 0.8, 40, 1.1, 64, "ties"),
        (997, 0.5, 17, 1.1, 64, "ties"),
        (2048, 0.9, 50, 1.1, 128, "negative"),
        (2048, 0.9, 50, 1.0, 128, "normal"),      # penalty off (p <= 1)
        (500, 0.8, 600, 1.1, 32, "normal"),       # k > V
        (500, 0.0, 40, 1.1, 32, "normal"),        # greedy by temperature
        (500, 0.8, 0, 1.1, 32, "normal"),         # greedy by top_k
        (500, 0.0, 40, 1.1, 32, "ties"),          # greedy over tied maxima
        (300, 0.8, 40, 1.1, 40, "outofrange"),    # history ids outside [0, V)
        (3000, 0.6, 40, 1.1, 256, "spiky"),
        (3000, 0.8, 200, 1.1, 64, "normal"),      # k > 64: server variant only
        (3000, 0.8, 512, 1.2, 64, "ties"),        # server heap capacity
        (4096, 2.0, 40, 1.1, 0, "normal"),        # no history
        (1000, 1e-3, 40, 1.1, 16, "normal"),      # tiny temperature
        (64, 0.8, 64, 1.1, 8, "const"),           # every logit equal
    ]:
        cs.append(dict(V=V, temperature=T, top_k=k, penalty=p, n_recent=nrec, kind=kind,
                       seed=seed))
        seed += 1
    return cs


def sampler_logits(c):
    g = _rng(31, c["seed"])
    V = c["V"]
    kind = c["kind"]
    if kind == "ties":
        lg = np.round(g.standard_normal(V) * 2.0).astype(np.float32)
    elif kind == "negative":
        lg = (-np.abs(g.standard_normal(V)) * 4 - 1).astype(np.float32)
    elif kind == "spiky":
        lg = (g.standard_normal(V) * 2).astype(np.float32)
        lg[g.choice(V, 5, replace=False)] += 15
    elif kind == "const":
        lg = np.full(V, 1.25, np.float32)
    else:
        lg = (g.standard_normal(V) * 3).astype(np.float32)
    return lg


def sampler_recent(c):
    g = _rng(41, c["seed"])
    V, n = c["V"], c["n_recent"]
    if n == 0:
        return np.zeros(0, np.int32)
    if c["kind"] == "dups":
        base = g.integers(0, V, size=max(1, n // 4))
        return base[g.integers(0, base.size, size=n)].astype(np.int32)
    rec = g.integers(0, V, size=n).astype(np.int32)
    if c["kind"] == "outofrange":
        rec[::5] = -1
        rec[1::7] = V + 3
    return rec


def loop_cases():
    """Decode loops: (config, steps, variant) run through the server's tail
    sequence (quantize, |xq|, OpenMP LM head, sampler, history push)."""
    return {
        "tiny_lib": dict(base="c1_gpt2", vocab=997, n_embd=96, steps=64, top_k=40, hist=64,
                         temperature=0.8, variant=0, seed=5),
        "tiny_srv": dict(base="c1_gpt2", vocab=997, n_embd=96, steps=64, top_k=40, hist=64,
                         temperature=0.8, variant=1, seed=6),
        "odd_shape": dict(base="c1_gpt2", vocab=1531, n_embd=200, steps=32, top_k=33, hist=20,
                          temperature=1.1, variant=0, seed=7),
        "c1_gpt2": dict(base="c1_gpt2", vocab=50257, n_embd=768, steps=48, top_k=40, hist=64,
                        temperature=0.8, variant=0, seed=0),
        "c5_like": dict(base="c5_stress", vocab=4099, n_embd=256, steps=24, top_k=64, hist=512,
                        temperature=0.7, variant=1, seed=3000),
    }


def loop_config(spec) -> synth.TailConfig:
    base = synth.CONFIGS[spec["base"]]
    return base.with_(vocab=spec["vocab"], n_embd=spec["n_embd"], streams=1,
                      top_k=spec["top_k"], hist=spec["hist"], steps=spec["steps"],
                      temperature=spec["temperature"], temperature_hi=None,
                      seed=spec["seed"], draws="rand")


def loop_inputs(spec):
    """(cfg, W fp32, initial history) of a loop case."""
    cfg = loop_config(spec)
    return cfg, synth.lm_head_f32(cfg), synth.history(cfg, 0)


def run_ref_loop(spec) -> np.ndarray:
    """Tokens of the reference's own tail over spec['steps'] steps."""
    import oracle
    R = oracle.ref()
    cfg, W, hist0 = loop_inputs(spec)
    q, s = oracle.quantize_rows(W, "ref")
    V, d = cfg.vocab, cfg.n_embd
    pad = max(32, -(-d // 32) * 32)
    xq = np.zeros(pad, np.int8)
    ax = np.zeros(pad, np.uint8)
    logits = np.zeros(V, np.float32)
    cap = max(1, cfg.hist)
    rec = np.zeros(cap, np.int32)
    rec[:hist0.size] = hist0
    import ctypes as C
    n = C.c_int(hist0.size)
    R.ref_srand(cfg.seed)
    toks = []
    for step in range(cfg.steps):
        hdn = synth.hidden(cfg, step)[0]
        t = R.ref_tail_step(hdn, xq, ax, logits, q.reshape(-1), s, V, d,
                            np.float32(cfg.temperature), cfg.top_k,
                            np.float32(cfg.rep_penalty), rec, C.byref(n), cap, 4,
                            spec["variant"])
        assert t >= 0, t
        toks.append(t)
    return np.array(toks, np.int32)
