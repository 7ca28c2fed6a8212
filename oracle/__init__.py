"""CPU checkers for the LAL decode tail -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py``
import this package, and only as the checker: the product library
``lal_b200/liblal_tail.so`` never loads it.

Two libraries are wrapped:

* ``port()``  -- ``oracle/liblal_oracle.so``, this repository's C restatement
  (``oracle/lal_oracle.c``), each function citing the reference lines it
  follows;
* ``ref()``   -- ``oracle/_ref/liblal_ref.so``, the reference's own C compiled
  from its sources by ``oracle/Makefile`` (``ref_harness.c``).  It exists only
  where it was built; it travels to the GPU box as a built file.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "liblal_oracle.so")
REF_GPT2_SO = os.path.join(HERE, "_ref", "liblal_ref_gpt2.so")
REF_SO = os.path.join(HERE, "_ref", "liblal_ref.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")


class SampleInfo(C.Structure):
    """Mirror of ``orc_sample_info`` (oracle/lal_oracle.h)."""
    _fields_ = [("threshold", C.c_float), ("max_l", C.c_float), ("sum", C.c_float),
                ("r", C.c_float), ("n_cand", C.c_int), ("greedy", C.c_int),
                ("drew", C.c_int)]


DECODE_FN = C.CFUNCTYPE(C.c_int, C.c_int, C.c_char_p, C.c_int)
FILTER_FN = C.CFUNCTYPE(C.c_int, C.POINTER(C.c_int), C.c_int, C.c_int,
                        C.POINTER(C.c_int), C.c_int, DECODE_FN)
DRAW_FN = C.CFUNCTYPE(C.c_float, C.c_void_p)


def build(force: bool = False) -> None:
    """Compile the restatement (and the reference harness when its sources exist)."""
    env = dict(os.environ)
    env.setdefault("HOSTCC", "gcc")
    if force:
        subprocess.run(["make", "-s", "-C", HERE, "clean"], check=True, env=env)
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True, env=env)


_port = None
_ref = None


def port():
    """ctypes handle of the C restatement, signatures set."""
    global _port
    if _port is None:
        if not os.path.exists(PORT_SO):
            build()
        lib = C.CDLL(PORT_SO)
        lib.orc_rms_norm.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_float]
        lib.orc_gpt2_quantize_x.restype = C.c_float
        lib.orc_gpt2_quantize_x.argtypes = [_f32p, _i8p, C.c_int]
        lib.orc_gpt2_lm_head.restype = C.c_int
        lib.orc_gpt2_lm_head.argtypes = [_f32p, _f32p, _i8p, _f32p, C.c_int, C.c_int, _i32p]
        lib.orc_gpt2_sample.restype = C.c_int
        lib.orc_gpt2_sample.argtypes = [_f32p, C.c_int, C.c_float, C.c_int, C.c_float,
                                        C.c_void_p, C.c_int, C.c_float, C.POINTER(SampleInfo)]
        lib.orc_gpt2_sample_p.restype = C.c_int
        lib.orc_gpt2_sample_p.argtypes = [_f32p, C.c_int, C.c_float, C.c_int, C.c_float,
                                          C.c_float, C.c_void_p, C.c_int, C.c_float,
                                          C.POINTER(SampleInfo)]
        lib.orc_gpt2_sample_f.restype = C.c_int
        lib.orc_gpt2_sample_f.argtypes = [_f32p, C.c_int, C.c_float, C.c_int, C.c_float,
                                          C.c_float, C.c_void_p, C.c_int, C.c_void_p,
                                          C.c_void_p, C.c_float, C.POINTER(SampleInfo)]
        lib.orc_quantize_x_int8.restype = C.c_float
        lib.orc_quantize_x_int8.argtypes = [_f32p, _i8p, C.c_int]
        lib.orc_compute_abs_xq.argtypes = [_i8p, _u8p, C.c_int]
        lib.orc_lm_head_int8_range.argtypes = [_f32p, _i8p, C.c_float, _i8p, _f32p,
                                               C.c_int, C.c_int, C.c_int]
        lib.orc_lm_head_int8_range_abs_8row.argtypes = [_f32p, _i8p, C.c_float, _i8p, _f32p,
                                                        C.c_int, C.c_int, C.c_int]
        lib.orc_lm_head_dots.argtypes = [_i32p, _i8p, _i8p, C.c_int, C.c_int, C.c_int]
        lib.orc_lm_head_multi.argtypes = [_f32p, _i8p, _f32p, _i8p, _f32p, C.c_int, C.c_int,
                                          C.c_int]
        lib.orc_quantize_q8_per_row.argtypes = [_f32p, _i8p, _f32p, C.c_int, C.c_int]
        lib.orc_quantize_q8_rows.argtypes = [_f32p, _i8p, _f32p, C.c_int, C.c_int]
        lib.orc_sample_token.restype = C.c_int
        lib.orc_sample_token.argtypes = [_f32p, C.c_int, C.c_float, C.c_int, C.c_float,
                                         C.c_void_p, C.c_int, C.c_float,
                                         C.POINTER(SampleInfo)]
        lib.orc_sample_token_filtered.restype = C.c_int
        lib.orc_sample_token_filtered.argtypes = [_f32p, C.c_int, C.c_float, C.c_int,
                                                  C.c_float, C.c_void_p, C.c_int,
                                                  C.c_void_p, C.c_void_p, C.c_void_p,
                                                  C.c_void_p, C.POINTER(SampleInfo)]
        lib.orc_recent_push.argtypes = [_i32p, C.POINTER(C.c_int), C.c_int, C.c_int]
        lib.orc_expf_batch.argtypes = [_f32p, _f32p, C.c_long]
        lib.orc_tail_step.restype = C.c_int
        lib.orc_tail_step.argtypes = [_f32p, C.c_int, _i8p, _f32p, C.c_int, C.c_float,
                                      C.c_int, C.c_float, _i32p, C.POINTER(C.c_int),
                                      C.c_int, C.c_float, C.c_int, C.c_void_p,
                                      C.POINTER(SampleInfo)]
        _port = lib
    return _port


def have_ref() -> bool:
    return os.path.exists(REF_SO)


def ref():
    """ctypes handle of the reference's own compiled C (oracle/_ref)."""
    global _ref
    if _ref is None:
        if not have_ref():
            raise FileNotFoundError(f"{REF_SO} not built (needs the reference sources)")
        lib = C.CDLL(REF_SO)
        lib.ref_vocab_max.restype = C.c_int
        lib.ref_xq_max.restype = C.c_int
        lib.ref_rms_norm.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_float]
        lib.ref_quantize_x_int8.restype = C.c_float
        lib.ref_quantize_x_int8.argtypes = [_f32p, _i8p, C.c_int]
        lib.ref_compute_abs_xq.argtypes = [_i8p, _u8p, C.c_int]
        for name in ("ref_lm_head_int8_range",):
            getattr(lib, name).argtypes = [_f32p, _i8p, C.c_float, _i8p, _f32p,
                                           C.c_int, C.c_int, C.c_int]
        for name in ("ref_lm_head_int8_range_abs", "ref_lm_head_int8_range_abs_8row"):
            getattr(lib, name).argtypes = [_f32p, _i8p, _u8p, C.c_float, _i8p, _f32p,
                                           C.c_int, C.c_int, C.c_int]
        lib.ref_lm_head_omp.argtypes = [_f32p, _i8p, _u8p, C.c_float, _i8p, _f32p,
                                        C.c_int, C.c_int, C.c_int]
        lib.ref_quantize_q8_per_row.argtypes = [_f32p, _i8p, _f32p, C.c_int, C.c_int]
        lib.ref_sample_token.restype = C.c_int
        lib.ref_sample_token.argtypes = [_f32p, C.c_int, C.c_float, C.c_int, C.c_float,
                                         C.c_void_p, C.c_int]
        lib.ref_sample_token_filtered.restype = C.c_int
        lib.ref_sample_token_filtered.argtypes = [_f32p, C.c_int, C.c_float, C.c_int,
                                                  C.c_float, C.c_void_p, C.c_int]
        lib.ref_set_filter.argtypes = [C.c_void_p]
        lib.ref_srand.argtypes = [C.c_uint]
        lib.ref_rand.restype = C.c_int
        lib.ref_tail_step.restype = C.c_int
        lib.ref_tail_step.argtypes = [_f32p, _i8p, _u8p, _f32p, _i8p, _f32p, C.c_int,
                                      C.c_int, C.c_float, C.c_int, C.c_float, _i32p,
                                      C.POINTER(C.c_int), C.c_int, C.c_int, C.c_int]
        _ref = lib
    return _ref


_ref_gpt2 = None


def have_ref_gpt2() -> bool:
    return os.path.exists(REF_GPT2_SO)


def ref_gpt2():
    """ctypes handle of the GPT-2 server's own LM-head code (oracle/_ref)."""
    global _ref_gpt2
    if _ref_gpt2 is None:
        if not have_ref_gpt2():
            raise FileNotFoundError(f"{REF_GPT2_SO} not built (needs the reference sources)")
        lib = C.CDLL(REF_GPT2_SO)
        lib.ref_gpt2_vocab.restype = C.c_int
        lib.ref_gpt2_n_embd.restype = C.c_int
        lib.ref_gpt2_quantize_x.restype = C.c_float
        lib.ref_gpt2_quantize_x.argtypes = [_f32p, _i8p, C.c_int]
        lib.ref_gpt2_lm_head.argtypes = [_f32p, _f32p, _i8p, _f32p, C.c_int]
        _ref_gpt2 = lib
    return _ref_gpt2


def gpt2_quantize_x(x: np.ndarray, lib: str = "port"):
    """lm_head_quantize_x (gpt2_server.c:1982-1998): (scale, xq)."""
    x = np.ascontiguousarray(x, np.float32)
    xq = np.zeros(x.size, np.int8)
    fn = port().orc_gpt2_quantize_x if lib == "port" else ref_gpt2().ref_gpt2_quantize_x
    return np.float32(fn(x, xq, x.size)), xq


def gpt2_lm_head(x: np.ndarray, wq: np.ndarray, sw: np.ndarray, lib: str = "port",
                 n_threads: int = 1):
    """lm_head_int8_parallel (gpt2_server.c:2125-2214): the logits of every
    row, the 512 kept by the server's heap re-scored in float.  The port also
    returns the kept rows (heap order)."""
    x = np.ascontiguousarray(x, np.float32)
    wq = np.ascontiguousarray(wq, np.int8)
    sw = np.ascontiguousarray(sw, np.float32)
    V, d = wq.shape
    logits = np.zeros(V, np.float32)
    if lib == "port":
        kept = np.zeros(512, np.int32)
        n = port().orc_gpt2_lm_head(logits, x, wq.reshape(-1), sw, V, d, kept)
        return logits, kept[:n].copy()
    R = ref_gpt2()
    if (V, d) != (R.ref_gpt2_vocab(), R.ref_gpt2_n_embd()):
        raise ValueError("the GPT-2 server is compiled for V=50257, d=768")
    R.ref_gpt2_lm_head(logits, x, wq.reshape(-1), sw, n_threads)
    return logits, None


def gpt2_sample(logits, temperature, top_k, rep_penalty, recent, u, top_p=0.0, filt=None,
                decode=None):
    """gpt2_server.c:2862-3013 (top-p branch when 0 < top_p < 1; the level-2
    filter hook when filt is given) on a copy: (token, info, penalised
    logits)."""
    lg = np.ascontiguousarray(logits, np.float32).copy()
    rec = None if recent is None or len(recent) == 0 else np.ascontiguousarray(recent, np.int32)
    info = SampleInfo()
    if filt is None and decode is None:
        tok = port().orc_gpt2_sample_p(lg, lg.size, np.float32(temperature), int(top_k),
                                       np.float32(top_p), np.float32(rep_penalty), _ptr(rec),
                                       0 if rec is None else rec.size, np.float32(u),
                                       C.byref(info))
        return tok, info, lg
    cf = FILTER_FN(filt) if filt is not None else None
    cd = DECODE_FN(decode) if decode is not None else None
    tok = port().orc_gpt2_sample_f(lg, lg.size, np.float32(temperature), int(top_k),
                                   np.float32(top_p), np.float32(rep_penalty), _ptr(rec),
                                   0 if rec is None else rec.size,
                                   C.cast(cf, C.c_void_p) if cf else None,
                                   C.cast(cd, C.c_void_p) if cd else None, np.float32(u),
                                   C.byref(info))
    return tok, info, lg


class Gpt2PortLoop:
    """The restated GPT-2 server tail of one stream: LM head with re-score,
    sampler, then the recent-token ring (gpt2_server.c:3347-3348 as a FIFO of
    hist_cap)."""

    def __init__(self, wq, sw, hist0, hist_cap, temperature, top_k, rep_penalty, top_p=0.0,
                 filt=None):
        self.top_p = top_p
        self.filt = filt
        self.wq = np.ascontiguousarray(wq, np.int8)
        self.sw = np.ascontiguousarray(sw, np.float32)
        self.cap = max(1, hist_cap)
        self.rec = np.zeros(self.cap, np.int32)
        self.rec[:len(hist0)] = hist0
        self.n = C.c_int(len(hist0))
        self.T, self.k, self.p = temperature, top_k, rep_penalty
        self.logits = None
        self.kept = None

    def step(self, x, u):
        logits, self.kept = gpt2_lm_head(x, self.wq, self.sw)
        tok, info, self.logits = gpt2_sample(logits, self.T, self.k, self.p,
                                             self.rec[:self.n.value], u, self.top_p,
                                             filt=self.filt)
        port().orc_recent_push(self.rec, C.byref(self.n), self.cap, int(tok))
        return tok, info

    def history(self):
        return self.rec[:self.n.value].copy()


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


# ---- convenience wrappers (numpy in, numpy out) --------------------------------

def rms_norm(x: np.ndarray, w: np.ndarray, eps: float = 1e-6, lib: str = "port"):
    """The final RMSNorm (runtime/lal_simd_optim.h:32-58) of one vector whose
    length is a multiple of 8."""
    x = np.ascontiguousarray(x, np.float32)
    if x.size % 8 != 0 or x.size == 0:
        raise ValueError("rms_norm: the length must be a positive multiple of 8")
    w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    (port().orc_rms_norm if lib == "port" else ref().ref_rms_norm)(out, x, w, x.size, eps)
    return out


def quantize_x(x: np.ndarray, lib: str = "port"):
    x = np.ascontiguousarray(x, np.float32)
    n = x.shape[-1]
    if lib == "ref":
        xq = np.zeros(max(32, -(-n // 32) * 32), np.int8)
        s = ref().ref_quantize_x_int8(x, xq, n)
        return np.float32(s), xq[:n].copy()
    xq = np.zeros(n, np.int8)
    s = port().orc_quantize_x_int8(x, xq, n)
    return np.float32(s), xq


def quantize_rows(W: np.ndarray, lib: str = "port"):
    W = np.ascontiguousarray(W, np.float32)
    V, d = W.shape
    q = np.empty((V, d), np.int8)
    s = np.empty(V, np.float32)
    if lib == "ref":
        ref().ref_quantize_q8_per_row(W.reshape(-1), q.reshape(-1), s, d, V)
    else:
        port().orc_quantize_q8_rows(W.reshape(-1), q.reshape(-1), s, d, V)
    return q, s


def lm_head(xq, sx, wq, sw, v0=0, v1=None, lib: str = "port"):
    V, d = wq.shape
    v1 = V if v1 is None else v1
    logits = np.zeros(V, np.float32)
    xq = np.ascontiguousarray(xq, np.int8)
    if lib == "ref":
        pad = max(32, -(-d // 32) * 32)
        xqp = np.zeros(pad, np.int8); xqp[:d] = xq
        ref().ref_lm_head_int8_range(logits, xqp, np.float32(sx), wq.reshape(-1), sw,
                                     v0, v1, d)
    else:
        port().orc_lm_head_int8_range(logits, xq, np.float32(sx), wq.reshape(-1), sw,
                                      v0, v1, d)
    return logits


def lm_head_8row(xq, sx, wq, sw, v0=0, v1=None):
    """The 8-row form (restated), including its dropped column tail."""
    V, d = wq.shape
    v1 = V if v1 is None else v1
    logits = np.zeros(V, np.float32)
    port().orc_lm_head_int8_range_abs_8row(logits, np.ascontiguousarray(xq, np.int8),
                                           np.float32(sx), wq.reshape(-1), sw, v0, v1, d)
    return logits


def lm_head_dots(xq, wq, v0=0, v1=None):
    V, d = wq.shape
    v1 = V if v1 is None else v1
    dots = np.zeros(v1 - v0, np.int32)
    port().orc_lm_head_dots(dots, np.ascontiguousarray(xq, np.int8), wq.reshape(-1), v0, v1, d)
    return dots


def sample(logits, temperature, top_k, rep_penalty, recent, u):
    """lal_sampling.h semantics (restated); returns (token, mutated logits, info)."""
    lg = np.array(logits, np.float32, copy=True)
    rec = None if recent is None else np.ascontiguousarray(recent, np.int32)
    info = SampleInfo()
    tok = port().orc_sample_token(lg, lg.size, np.float32(temperature), int(top_k),
                                  np.float32(rep_penalty), _ptr(rec),
                                  0 if rec is None else rec.size, np.float32(u),
                                  C.byref(info))
    return tok, lg, info


def sample_filtered(logits, temperature, top_k, rep_penalty, recent, draw, filt=None,
                    decode=None):
    """qwen7b_server.c lal_sample_token_filtered semantics (restated).

    ``draw`` is a Python callable returning u; it is called only where the
    reference calls rand()."""
    lg = np.array(logits, np.float32, copy=True)
    rec = None if recent is None else np.ascontiguousarray(recent, np.int32)
    info = SampleInfo()
    cdraw = DRAW_FN(lambda _ctx: float(draw()))
    cf = FILTER_FN(filt) if filt is not None else None
    cd = DECODE_FN(decode) if decode is not None else None
    tok = port().orc_sample_token_filtered(
        lg, lg.size, np.float32(temperature), int(top_k), np.float32(rep_penalty),
        _ptr(rec), 0 if rec is None else rec.size,
        C.cast(cf, C.c_void_p) if cf else None, C.cast(cd, C.c_void_p) if cd else None,
        C.cast(cdraw, C.c_void_p), None, C.byref(info))
    return tok, lg, info


def expf(x: np.ndarray) -> np.ndarray:
    """glibc expf, element-wise."""
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    port().orc_expf_batch(x, y, x.size)
    return y


class PortLoop:
    """The restated decode tail of one stream (qwen7b_server.c:829-850)."""

    def __init__(self, wq, sw, hist0, hist_cap, temperature, top_k, rep_penalty, variant):
        self.wq = np.ascontiguousarray(wq, np.int8)
        self.sw = np.ascontiguousarray(sw, np.float32)
        self.V, self.d = self.wq.shape
        self.cap = max(1, hist_cap)
        self.rec = np.zeros(self.cap, np.int32)
        self.rec[:len(hist0)] = hist0
        self.n = C.c_int(len(hist0))
        self.T, self.k, self.p, self.variant = temperature, top_k, rep_penalty, variant
        self.logits = np.zeros(self.V, np.float32)

    def step(self, hidden, u):
        info = SampleInfo()
        tok = port().orc_tail_step(np.ascontiguousarray(hidden, np.float32), self.d,
                                   self.wq.reshape(-1), self.sw, self.V, np.float32(self.T),
                                   int(self.k), np.float32(self.p), self.rec, C.byref(self.n),
                                   self.cap, np.float32(u), int(self.variant),
                                   self.logits.ctypes.data_as(C.c_void_p), C.byref(info))
        return tok, info

    def history(self):
        return self.rec[:self.n.value].copy()


def lm_head_multi(xq, sx, wq, sw):
    """Restated logits of B quantized vectors at once: [B, V]."""
    xq = np.ascontiguousarray(xq, np.int8)
    B, d = xq.shape
    V = wq.shape[0]
    out = np.empty((B, V), np.float32)
    port().orc_lm_head_multi(out.reshape(-1), xq.reshape(-1), np.ascontiguousarray(sx, np.float32),
                             np.ascontiguousarray(wq).reshape(-1),
                             np.ascontiguousarray(sw, np.float32), V, d, B)
    return out


class PortBatch:
    """B independent restated decode tails sharing one LM head (a batched
    step is B streams, each its own history, temperature, top-k and draws):
    per stream the quantizer, the 1-row LM head (computed for all streams in
    one pass), lal_sampling.h's sampler (uncapped heap) or the server's, and
    the history ring."""

    def __init__(self, wq, sw, hists, hist_cap, temps, top_ks, rep_penalty, variant):
        self.wq = np.ascontiguousarray(wq, np.int8)
        self.sw = np.ascontiguousarray(sw, np.float32)
        self.cap = max(1, hist_cap)
        self.push = hist_cap > 0
        self.recs, self.ns = [], []
        for h in hists:
            r = np.zeros(self.cap, np.int32)
            r[:len(h)] = h
            self.recs.append(r)
            self.ns.append(C.c_int(len(h)))
        self.T = [float(x) for x in temps]
        self.k = [int(x) for x in top_ks]
        self.p, self.variant = rep_penalty, variant

    def step(self, hidden, u):
        B = len(self.recs)
        q = [quantize_x(hidden[b]) for b in range(B)]
        lg = lm_head_multi(np.stack([x for _, x in q]), np.array([s for s, _ in q], np.float32),
                           self.wq, self.sw)
        toks = []
        for b in range(B):
            rec = self.recs[b][:self.ns[b].value]
            if self.variant == 1:
                tok, _, _ = sample_filtered(lg[b], self.T[b], self.k[b], self.p, rec,
                                            draw=lambda ub=u[b]: ub)
            else:
                tok, _, _ = sample(lg[b], self.T[b], self.k[b], self.p,
                                   rec if rec.size else None, u[b])
            if self.push:
                port().orc_recent_push(self.recs[b], C.byref(self.ns[b]), self.cap, int(tok))
            toks.append(tok)
        return np.array(toks, np.int32)

    def history(self, b):
        return self.recs[b][:self.ns[b].value].copy()


def ref_sample(logits, temperature, top_k, rep_penalty, recent, filtered=False):
    """The reference's own sampler; draws from the process's glibc rand()."""
    lg = np.array(logits, np.float32, copy=True)
    rec = None if recent is None else np.ascontiguousarray(recent, np.int32)
    fn = ref().ref_sample_token_filtered if filtered else ref().ref_sample_token
    tok = fn(lg, lg.size, np.float32(temperature), int(top_k), np.float32(rep_penalty),
             _ptr(rec), 0 if rec is None else rec.size)
    return tok, lg
