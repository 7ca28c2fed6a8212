"""Seeded synthetic inputs for the decode-tail workloads.

The reference ships no weights or datasets for this path, so every workload is
synthetic, with the shapes and value distributions of the five BASELINE
configurations:

=========  =======  =====  ===  =====  ====  =============================
name       V        d      B    top_k  H     notes
=========  =======  =====  ===  =====  ====  =============================
c1_gpt2    50257    768    1    40     64    T=0.8, 1% outliers x8, W~N(0,.02)
c2_qwen    152064   3584   1    40     256   T=0.7, 0.5% outliers x16
c3_batch   152064   3584   64   50     256   T~U(0.5,1) per stream
c4_dense   152064   3584   256  40/1   0     greedy and top-k 40
c5_stress  152064   3584   8    1024   4096  p=1.3, 30% repeats, 5% dup rows
=========  =======  =====  ===  =====  ====  =============================

Every array is a pure function of (config seed, purpose, block index), so any
vocab slice of the LM head can be generated on its own (each GPU of a
vocab-sharded run generates only its rows) and two processes always agree.

Random draws for the sampler come from glibc itself, called through ctypes:
``rand()`` after ``srand(seed)`` for the single-stream configs (the server's
generator, qwen7b_server.c:992 and lal_sampling.h:116) and one ``random_r``
state per stream, seeded ``seed + b``, for the batched ones.  A draw is
``u = (float)r / (float)RAND_MAX`` exactly as lal_sampling.h:116 writes it.
"""
from __future__ import annotations

import ctypes as C
import ctypes.util
import dataclasses
from typing import Optional

import numpy as np

ROW_BLOCK = 1024          # LM-head rows generated per independent RNG block
RAND_MAX = 2147483647


@dataclasses.dataclass(frozen=True)
class TailConfig:
    name: str
    vocab: int
    n_embd: int
    streams: int
    top_k: int
    hist: int
    steps: int
    temperature: float            # single value, or lower bound of a U(lo, hi)
    temperature_hi: Optional[float] = None
    rep_penalty: float = 1.1
    hidden_std: float = 1.0
    outlier_frac: float = 0.0
    outlier_mult: float = 1.0
    w_std: float = 0.015
    dup_row_frac: float = 0.0
    hist_repeat_frac: float = 0.0
    draws: str = "rand"           # "rand" (one glibc stream) or "random_r" (per stream)
    seed: int = 0

    def with_(self, **kw) -> "TailConfig":
        return dataclasses.replace(self, **kw)


CONFIGS = {
    "c1_gpt2": TailConfig("c1_gpt2", 50257, 768, 1, 40, 64, 256, 0.8,
                          outlier_frac=0.01, outlier_mult=8.0, w_std=0.02, seed=0),
    "c2_qwen": TailConfig("c2_qwen", 152064, 3584, 1, 40, 256, 512, 0.7,
                          outlier_frac=0.005, outlier_mult=16.0, seed=0),
    "c3_batch": TailConfig("c3_batch", 152064, 3584, 64, 50, 256, 256, 0.5, 1.0,
                           outlier_frac=0.005, outlier_mult=16.0, draws="random_r",
                           seed=1000),
    "c4_dense": TailConfig("c4_dense", 152064, 3584, 256, 40, 0, 64, 0.7,
                           outlier_frac=0.005, outlier_mult=16.0, draws="random_r",
                           seed=2000),
    "c5_stress": TailConfig("c5_stress", 152064, 3584, 8, 1024, 4096, 128, 0.7,
                            rep_penalty=1.3, hidden_std=4.0, dup_row_frac=0.05,
                            hist_repeat_frac=0.30, draws="random_r", seed=3000),
}


def _gen(cfg: TailConfig, purpose: int, index: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(np.random.SeedSequence(
        [cfg.seed & 0xFFFFFFFF, cfg.vocab, cfg.n_embd, purpose, index])))


def _w_block(cfg: TailConfig, j: int) -> np.ndarray:
    """fp32 rows [j*ROW_BLOCK, ...) of the LM head, duplicates applied."""
    r0 = j * ROW_BLOCK
    n = min(ROW_BLOCK, cfg.vocab - r0)
    g = _gen(cfg, 1, j)
    w = g.standard_normal((n, cfg.n_embd), dtype=np.float32)
    w *= np.float32(cfg.w_std)
    if cfg.dup_row_frac > 0 and n > 1:
        # Duplicate 5% of rows bit-for-bit from another row of the same block,
        # so exact logit ties appear (within and across CTA slices).
        nd = max(1, int(round(cfg.dup_row_frac * n)))
        dst = g.choice(n, size=nd, replace=False)
        src = g.integers(0, n, size=nd)
        for a, b in zip(dst, src):
            if a != b:
                w[a] = w[b]
    return w


def lm_head_f32(cfg: TailConfig, r0: int = 0, r1: Optional[int] = None) -> np.ndarray:
    """fp32 LM-head rows [r0, r1) (~N(0, w_std)), shape [r1-r0, d]."""
    r1 = cfg.vocab if r1 is None else r1
    out = np.empty((r1 - r0, cfg.n_embd), np.float32)
    for j in range(r0 // ROW_BLOCK, (r1 - 1) // ROW_BLOCK + 1):
        b0 = j * ROW_BLOCK
        blk = _w_block(cfg, j)
        lo, hi = max(r0, b0), min(r1, b0 + blk.shape[0])
        out[lo - r0:hi - r0] = blk[lo - b0:hi - b0]
    return out


def hidden(cfg: TailConfig, step: int, streams: Optional[int] = None) -> np.ndarray:
    """fp32 hidden [B, d] for one decode step: N(0, hidden_std) with outliers."""
    B = cfg.streams if streams is None else streams
    g = _gen(cfg, 2, step)
    h = g.standard_normal((B, cfg.n_embd), dtype=np.float32)
    h *= np.float32(cfg.hidden_std)
    if cfg.outlier_frac > 0:
        k = max(1, int(round(cfg.outlier_frac * cfg.n_embd)))
        for b in range(B):
            idx = g.choice(cfg.n_embd, size=k, replace=False)
            h[b, idx] *= np.float32(cfg.outlier_mult)
    return h


def history(cfg: TailConfig, stream: int) -> np.ndarray:
    """Initial penalty history of one stream (uniform ids; with repeats)."""
    if cfg.hist <= 0:
        return np.zeros(0, np.int32)
    g = _gen(cfg, 3, stream)
    ids = g.integers(0, cfg.vocab, size=cfg.hist).astype(np.int32)
    if cfg.hist_repeat_frac > 0:
        rep = g.random(cfg.hist) < cfg.hist_repeat_frac
        rep[0] = False
        for i in np.nonzero(rep)[0]:
            ids[i] = ids[g.integers(0, i)]
    return ids


def temperatures(cfg: TailConfig) -> np.ndarray:
    if cfg.temperature_hi is None:
        return np.full(cfg.streams, cfg.temperature, np.float32)
    g = _gen(cfg, 4, 0)
    return g.uniform(cfg.temperature, cfg.temperature_hi, cfg.streams).astype(np.float32)


# ---- glibc draws ------------------------------------------------------------------

_libc = C.CDLL(ctypes.util.find_library("c"), use_errno=True)
_libc.rand.restype = C.c_int
_libc.srand.argtypes = [C.c_uint]


class _RandomData(C.Structure):
    # struct random_data from <stdlib.h> (glibc, LP64).
    _fields_ = [("fptr", C.c_void_p), ("rptr", C.c_void_p), ("state", C.c_void_p),
                ("rand_type", C.c_int), ("rand_deg", C.c_int), ("rand_sep", C.c_int),
                ("end_ptr", C.c_void_p)]


_libc.initstate_r.argtypes = [C.c_uint, C.c_char_p, C.c_size_t, C.POINTER(_RandomData)]
_libc.random_r.argtypes = [C.POINTER(_RandomData), C.POINTER(C.c_int32)]


def u_from_rand(r: int) -> np.float32:
    """(float)r / (float)RAND_MAX, as lal_sampling.h:116 computes it."""
    return np.float32(np.float32(r) / np.float32(RAND_MAX))


class GlibcStream:
    """One glibc generator: the process-global rand() or a private random_r."""

    def __init__(self, seed: int, private: bool):
        self.private = private
        if private:
            self._buf = C.create_string_buffer(128)
            self._rd = _RandomData()
            if _libc.initstate_r(C.c_uint(seed), self._buf, 128, C.byref(self._rd)) != 0:
                raise OSError("initstate_r failed")
        else:
            _libc.srand(C.c_uint(seed))

    def next_int(self) -> int:
        if self.private:
            out = C.c_int32()
            _libc.random_r(C.byref(self._rd), C.byref(out))
            return int(out.value)
        return int(_libc.rand())

    def next_u(self) -> np.float32:
        return u_from_rand(self.next_int())


class Draws:
    """Per-stream draw sources of a config (global rand() or random_r per stream)."""

    def __init__(self, cfg: TailConfig, streams: Optional[int] = None):
        B = cfg.streams if streams is None else streams
        if cfg.draws == "rand":
            g = GlibcStream(cfg.seed, private=False)
            self.streams = [g] * B
        else:
            self.streams = [GlibcStream(cfg.seed + b, private=True) for b in range(B)]

    def u(self, b: int) -> np.float32:
        return self.streams[b].next_u()
