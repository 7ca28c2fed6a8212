"""lal_b200 -- the LAL decode tail on B200 (sm_100a), Python host mirror.

The product is ``lal_b200/liblal_tail.so`` (C ABI in ``include/lal_tail.h``).
This module binds it with ctypes and mirrors the reference's interface for
the path, with the reference's names:

* ``quantize_x_int8``      runtime/lal_q8_kernel.h:375  lal_quantize_x_int8
* ``compute_abs_xq``       runtime/lal_q8_kernel.h:450  lal_compute_abs_xq
* ``lm_head_int8_range``   runtime/lal_q8_kernel.h:463  lal_lm_head_int8_range
* ``quantize_q8_per_row``  runtime/lal_q8_kernel.h:357  lal_quantize_q8_per_row
* ``sample_token``         runtime/lal_sampling.h:46    lal_sample_token
* ``sample_token_filtered`` tools/server/qwen7b_server.c:219 (with the level-2
  filter hook of qwen7b_server.c:175-186)
* ``DecodeTail``           the fused tail replacing qwen7b_server.c:829-850

Everything computes on the GPU.  There is no CPU fallback: importing works
without a GPU (so the library can be inspected), but every compute call
raises ``LalTailError`` when the CUDA library or a GPU is unavailable.
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Callable, Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblal_tail.so")

LAL_SAMPLER_LIBRARY = 0
LAL_SAMPLER_SERVER = 1
LAL_SAMPLER_GPT2 = 2

ERRORS = {0: "OK", 1: "ERR_ARG", 2: "ERR_CUDA", 3: "ERR_NOMEM", 4: "ERR_TIMEOUT",
          5: "ERR_CAPACITY", 6: "ERR_STATE", 7: "ERR_COMM", 8: "ERR_UNSUPPORTED"}


class LalTailError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


class TailConfig(C.Structure):
    """Mirror of lal_tail_config."""
    _fields_ = [("vocab_size", C.c_int), ("n_embd", C.c_int), ("max_streams", C.c_int),
                ("max_top_k", C.c_int), ("history_cap", C.c_int), ("sampler", C.c_int),
                ("device", C.c_int), ("shard_rank", C.c_int), ("shard_count", C.c_int)]


class TailDiag(C.Structure):
    """Mirror of lal_tail_diag."""
    _fields_ = [("threshold", C.c_float), ("max_l", C.c_float), ("sum", C.c_float),
                ("r", C.c_float), ("n_cand", C.c_int), ("greedy", C.c_int),
                ("drew", C.c_int), ("token", C.c_int)]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


class Gpq8Tensor(C.Structure):
    """Mirror of ``lal_gpq8_tensor`` (include/lal_tail.h)."""
    _fields_ = [("ndim", C.c_int), ("shape", C.c_int * 4), ("qtype", C.c_int),
                ("data_offset", C.c_uint64), ("data_len", C.c_uint64), ("n_scale", C.c_int),
                ("scale_offset", C.c_uint64)]


class RecentTokens(C.Structure):
    """Mirror of LalRecentTokens (runtime/lal_sampling.h:128-131)."""
    _fields_ = [("tokens", C.c_int * 256), ("n", C.c_int)]


DECODE_FN = C.CFUNCTYPE(C.c_int, C.c_int, C.c_char_p, C.c_int)
FILTER_FN = C.CFUNCTYPE(C.c_int, C.POINTER(C.c_int), C.c_int, C.c_int,
                        C.POINTER(C.c_int), C.c_int, DECODE_FN)
DRAW_FN = C.CFUNCTYPE(C.c_float, C.c_void_p)

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_vp = C.c_void_p
_ip = C.c_int
_fp = C.c_float

# name -> (restype, argtypes); every symbol of include/lal_tail.h
SIGNATURES = {
    "lal_tail_last_error": (C.c_char_p, []),
    "lal_tail_version": (C.c_char_p, []),
    "lal_quantize_x_int8": (C.c_float, [_f32p, _i8p, _ip]),
    "lal_compute_abs_xq": (None, [_i8p, _u8p, _ip]),
    "lal_lm_head_int8_range": (None, [_f32p, _i8p, _fp, _i8p, _f32p, _ip, _ip, _ip]),
    "lal_lm_head_int8_range_abs": (None, [_f32p, _i8p, _u8p, _fp, _i8p, _f32p, _ip, _ip, _ip]),
    "lal_lm_head_int8_range_abs_8row": (None, [_f32p, _i8p, _u8p, _fp, _i8p, _f32p, _ip, _ip,
                                               _ip]),
    "lal_quantize_q8_per_row": (None, [_f32p, _i8p, _f32p, _ip, _ip]),
    "lal_sample_token": (C.c_int, [_f32p, _ip, _fp, _ip, _fp, _vp, _ip]),
    "lal_recent_push": (None, [C.POINTER(RecentTokens), _ip]),
    "lal_tail_quantize_x_int8": (C.c_int, [_f32p, _i8p, _ip, C.POINTER(C.c_float)]),
    "lal_tail_compute_abs_xq": (C.c_int, [_i8p, _u8p, _ip]),
    "lal_tail_lm_head_int8_range": (C.c_int, [_f32p, _i8p, _fp, _i8p, _f32p, _ip, _ip, _ip]),
    "lal_tail_quantize_q8_per_row": (C.c_int, [_f32p, _i8p, _f32p, _ip, _ip]),
    "lal_tail_sample_token": (C.c_int, [_f32p, _ip, _fp, _ip, _fp, _vp, _ip, _fp,
                                        C.POINTER(C.c_int)]),
    "lal_tail_sample_token_filtered": (C.c_int, [_f32p, _ip, _fp, _ip, _fp, _vp, _ip, _vp,
                                                 _vp, _vp, _vp, C.POINTER(C.c_int)]),
    "lal_tail_lm_head_register": (C.c_int, [_i8p, _f32p, _ip, _ip]),
    "lal_tail_lm_head_forget": (C.c_int, [_vp]),
    "lal_tail_create": (C.c_int, [C.POINTER(TailConfig), C.POINTER(_vp)]),
    "lal_tail_destroy": (C.c_int, [_vp]),
    "lal_tail_shard_rows": (C.c_int, [_vp, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "lal_tail_load_lm_head_q8": (C.c_int, [_vp, _i8p, _f32p]),
    "lal_tail_load_lm_head_f32": (C.c_int, [_vp, _f32p, _ip, _ip]),
    "lal_tail_read_lm_head": (C.c_int, [_vp, _vp, _vp]),
    "lal_tail_set_sampling": (C.c_int, [_vp, _ip, _f32p, _i32p, _f32p]),
    "lal_tail_set_history": (C.c_int, [_vp, _ip, _vp, _ip]),
    "lal_tail_get_history": (C.c_int, [_vp, _ip, _vp, C.POINTER(C.c_int)]),
    "lal_tail_step": (C.c_int, [_vp, _vp, _ip, _vp, _vp]),
    "lal_tail_step_device": (C.c_int, [_vp, _vp, _ip, _vp, _vp]),
    "lal_tail_sync": (C.c_int, [_vp]),
    "lal_tail_stage_inputs": (C.c_int, [_vp, _f32p, _ip, _f32p]),
    "lal_tail_fetch_tokens": (C.c_int, [_vp, _ip, _i32p]),
    "lal_tail_shard_select": (C.c_int, [_vp, _vp, _ip]),
    "lal_tail_exchange_buffers": (C.c_int, [_vp, _ip, C.POINTER(_vp), C.POINTER(_vp),
                                            C.POINTER(C.c_size_t)]),
    "lal_tail_shard_merge": (C.c_int, [_vp, _ip, _vp, _vp]),
    "lal_tail_exchange_handle": (C.c_int, [_vp, _vp]),
    "lal_tail_connect_peers": (C.c_int, [_vp, _vp]),
    "lal_tail_disconnect_peers": (C.c_int, [_vp]),
    "lal_tail_set_filter": (C.c_int, [_vp, _vp, _vp, _vp, _vp]),
    "lal_tail_set_final_norm": (C.c_int, [_vp, _vp, C.c_float]),
    "lal_tail_set_lm_head_copies": (C.c_int, [_vp, _ip]),
    "lal_tail_step_kind": (C.c_int, [_vp, _ip]),
    "lal_tail_set_top_p": (C.c_int, [_vp, C.c_float]),
    "lal_tail_gpq8_find": (C.c_int, [_vp, C.c_size_t, C.c_char_p, C.POINTER(Gpq8Tensor)]),
    "lal_tail_load_lm_head_gpq8": (C.c_int, [_vp, _vp, C.c_size_t, C.c_char_p]),
    "lal_tail_sample_token_noalloc": (C.c_int, [_vp, _ip, _fp, _ip, _fp, _vp, _ip, _fp, _vp,
                                                C.POINTER(C.c_int)]),
    "lal_tail_get_diag": (C.c_int, [_vp, _ip, C.POINTER(TailDiag)]),
    "lal_tail_get_logits": (C.c_int, [_vp, _ip, _f32p]),
    "lal_tail_device_buffers": (C.c_int, [_vp, C.POINTER(_vp), C.POINTER(_vp), C.POINTER(_vp)]),
    "lal_tail_get_stream": (C.c_int, [_vp, C.POINTER(_vp)]),
    "lal_tail_set_timing": (C.c_int, [_vp, _ip]),
    "lal_tail_kernel_time": (C.c_int, [_vp, C.POINTER(C.c_double), C.POINTER(C.c_int)]),
    "lal_tail_debug_expf": (C.c_int, [_f32p, _f32p, _ip]),
    "lal_tail_debug_phases": (C.c_int, [_vp, _ip]),
    "lal_tail_debug_phase_read": (C.c_int, [_vp, _vp, _ip, C.POINTER(C.c_int)]),
}

_lib = None


def lib():
    """The loaded liblal_tail.so (signatures set).  Raises if it was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise LalTailError(2, f"{LIB_PATH} is missing: run __graft_entry__.build()")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


_step = None


def _step_fn():
    """lal_tail_step bound once (the per-token call)."""
    global _step
    if _step is None:
        _step = lib().lal_tail_step
    return _step


def _check(rc: int):
    if rc != 0:
        raise LalTailError(rc, lib().lal_tail_last_error().decode(errors="replace"))


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


# ---- reference-named functions ------------------------------------------------------

def quantize_x_int8(x: np.ndarray):
    """lal_quantize_x_int8: returns (scale, xq)."""
    x = np.ascontiguousarray(x, np.float32)
    xq = np.empty(x.size, np.int8)
    s = C.c_float()
    _check(lib().lal_tail_quantize_x_int8(x, xq, x.size, C.byref(s)))
    return np.float32(s.value), xq


def compute_abs_xq(xq: np.ndarray) -> np.ndarray:
    xq = np.ascontiguousarray(xq, np.int8)
    ax = np.empty(xq.size, np.uint8)
    _check(lib().lal_tail_compute_abs_xq(xq, ax, xq.size))
    return ax


def lm_head_int8_range(logits: np.ndarray, xq: np.ndarray, scale_x: float,
                       wte_q: np.ndarray, scale_w: np.ndarray, v_start: int, v_end: int):
    """lal_lm_head_int8_range: fills logits[v_start:v_end] in place."""
    n_embd = wte_q.shape[1]
    _check(lib().lal_tail_lm_head_int8_range(logits, np.ascontiguousarray(xq, np.int8),
                                             np.float32(scale_x), wte_q.reshape(-1), scale_w,
                                             v_start, v_end, n_embd))
    return logits


def lm_head_forget(wte_q: np.ndarray):
    _check(lib().lal_tail_lm_head_forget(wte_q.ctypes.data_as(C.c_void_p)))


def quantize_q8_per_row(W: np.ndarray):
    """lal_quantize_q8_per_row on the GPU: returns (q8 [V,d], scale [V])."""
    W = np.ascontiguousarray(W, np.float32)
    V, d = W.shape
    q = np.empty((V, d), np.int8)
    s = np.empty(V, np.float32)
    _check(lib().lal_tail_quantize_q8_per_row(W.reshape(-1), q.reshape(-1), s, d, V))
    return q, s


def sample_token(logits: np.ndarray, temperature: float, top_k: int, rep_penalty: float,
                 recent: Optional[np.ndarray], u: float) -> int:
    """lal_sample_token with the draw u given; mutates logits like the reference."""
    rec = None if recent is None else np.ascontiguousarray(recent, np.int32)
    tok = C.c_int()
    _check(lib().lal_tail_sample_token(logits, logits.size, np.float32(temperature),
                                       int(top_k), np.float32(rep_penalty), _ptr(rec),
                                       0 if rec is None else rec.size, np.float32(u),
                                       C.byref(tok)))
    return tok.value


def sample_token_filtered(logits: np.ndarray, temperature: float, top_k: int,
                          rep_penalty: float, recent: Optional[np.ndarray],
                          draw: Callable[[], float], filt=None, decode=None) -> int:
    """qwen7b_server.c lal_sample_token_filtered; draw() is called only where
    the reference calls rand()."""
    rec = None if recent is None else np.ascontiguousarray(recent, np.int32)
    cdraw = DRAW_FN(lambda _ctx: float(draw()))
    cf = FILTER_FN(filt) if filt is not None else None
    cd = DECODE_FN(decode) if decode is not None else None
    tok = C.c_int()
    _check(lib().lal_tail_sample_token_filtered(
        logits, logits.size, np.float32(temperature), int(top_k), np.float32(rep_penalty),
        _ptr(rec), 0 if rec is None else rec.size,
        C.cast(cf, C.c_void_p) if cf else None, C.cast(cd, C.c_void_p) if cd else None,
        C.cast(cdraw, C.c_void_p), None, C.byref(tok)))
    return tok.value


def gpq8_find(blob: bytes, key: str) -> dict:
    """Locate a tensor in a GPQ8 blob (host only, no GPU)."""
    e = Gpq8Tensor()
    buf = C.create_string_buffer(blob, len(blob))
    _check(lib().lal_tail_gpq8_find(buf, len(blob), key.encode(), C.byref(e)))
    return {"ndim": e.ndim, "shape": list(e.shape)[:e.ndim], "qtype": e.qtype,
            "data_offset": e.data_offset, "data_len": e.data_len, "n_scale": e.n_scale,
            "scale_offset": e.scale_offset}


def debug_expf(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    _check(lib().lal_tail_debug_expf(x, y, x.size))
    return y


# ---- the fused decode tail -----------------------------------------------------------

class DecodeTail:
    """One GPU's fused decode tail (a vocab slice when shard_count > 1)."""

    def __init__(self, vocab_size: int, n_embd: int, max_streams: int = 1,
                 max_top_k: int = 64, history_cap: int = 256,
                 sampler: int = LAL_SAMPLER_LIBRARY, device: int = -1,
                 shard_rank: int = 0, shard_count: int = 1):
        self.cfg = TailConfig(vocab_size, n_embd, max_streams, max_top_k, history_cap,
                              sampler, device, shard_rank, shard_count)
        h = C.c_void_p()
        _check(lib().lal_tail_create(C.byref(self.cfg), C.byref(h)))
        self.h = h
        r0, n = C.c_int(), C.c_int()
        _check(lib().lal_tail_shard_rows(self.h, C.byref(r0), C.byref(n)))
        self.row0, self.n_rows = r0.value, n.value

    def close(self):
        if getattr(self, "h", None):
            lib().lal_tail_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def load_lm_head_q8(self, wte_q_rows: np.ndarray, scale_w_rows: np.ndarray):
        _check(lib().lal_tail_load_lm_head_q8(self.h, np.ascontiguousarray(wte_q_rows).reshape(-1),
                                              np.ascontiguousarray(scale_w_rows, np.float32)))

    def load_lm_head_f32(self, W_rows: np.ndarray, row_begin: int = 0):
        W_rows = np.ascontiguousarray(W_rows, np.float32)
        _check(lib().lal_tail_load_lm_head_f32(self.h, W_rows.reshape(-1), row_begin,
                                               W_rows.shape[0]))

    def load_lm_head_gpq8(self, blob: bytes, key: Optional[str] = None):
        """This slice of a [V, d] tensor of a GPQ8 blob (F32: quantized on the GPU)."""
        buf = C.create_string_buffer(blob, len(blob))
        _check(lib().lal_tail_load_lm_head_gpq8(self.h, buf, len(blob),
                                                key.encode() if key else None))

    def read_lm_head(self):
        q = np.empty((self.n_rows, self.cfg.n_embd), np.int8)
        s = np.empty(self.n_rows, np.float32)
        _check(lib().lal_tail_read_lm_head(self.h, _ptr(q), _ptr(s)))
        return q, s

    def set_sampling(self, temperature: Sequence[float], top_k: Sequence[int],
                     rep_penalty: Sequence[float]):
        t = np.ascontiguousarray(temperature, np.float32)
        k = np.ascontiguousarray(top_k, np.int32)
        p = np.ascontiguousarray(rep_penalty, np.float32)
        _check(lib().lal_tail_set_sampling(self.h, t.size, t, k, p))

    def set_history(self, stream: int, recent: Optional[np.ndarray]):
        rec = np.zeros(0, np.int32) if recent is None else np.ascontiguousarray(recent, np.int32)
        _check(lib().lal_tail_set_history(self.h, stream, _ptr(rec), rec.size))

    def get_history(self, stream: int) -> np.ndarray:
        out = np.zeros(max(1, self.cfg.history_cap), np.int32)
        n = C.c_int()
        _check(lib().lal_tail_get_history(self.h, stream, _ptr(out), C.byref(n)))
        return out[:n.value].copy()

    def step(self, hidden: np.ndarray, u: np.ndarray) -> np.ndarray:
        """One decode step from host arrays (hidden [B, d] or [d], u [B])."""
        if not (isinstance(hidden, np.ndarray) and hidden.dtype == np.float32
                and hidden.flags.c_contiguous):
            hidden = np.ascontiguousarray(hidden, np.float32)
        if not (isinstance(u, np.ndarray) and u.dtype == np.float32 and u.flags.c_contiguous):
            u = np.ascontiguousarray(u, np.float32)
        B = 1 if hidden.ndim == 1 else hidden.shape[0]
        if hidden.size != B * self.cfg.n_embd:
            raise ValueError(f"hidden: {hidden.size} values for {B} x {self.cfg.n_embd}")
        if u.size < B:
            raise ValueError(f"u: {u.size} draws for {B} streams")
        tok = np.empty(B, np.int32)
        # raw pointers: the arrays are checked above, the call is per token
        rc = _step_fn()(self.h, hidden.__array_interface__["data"][0], B,
                        u.__array_interface__["data"][0], tok.__array_interface__["data"][0])
        if rc:
            _check(rc)
        return tok

    def diag(self, stream: int = 0) -> dict:
        d = TailDiag()
        _check(lib().lal_tail_get_diag(self.h, stream, C.byref(d)))
        return d.as_dict()

    def logits(self, stream: int = 0) -> np.ndarray:
        out = np.empty(self.n_rows, np.float32)
        _check(lib().lal_tail_get_logits(self.h, stream, out))
        return out

    def set_timing(self, on: bool):
        _check(lib().lal_tail_set_timing(self.h, 1 if on else 0))

    def kernel_time(self):
        ms, n = C.c_double(), C.c_int()
        _check(lib().lal_tail_kernel_time(self.h, C.byref(ms), C.byref(n)))
        return ms.value, n.value

    def device_buffers(self):
        a, b, c = C.c_void_p(), C.c_void_p(), C.c_void_p()
        _check(lib().lal_tail_device_buffers(self.h, C.byref(a), C.byref(b), C.byref(c)))
        return a.value, b.value, c.value

    def debug_phases(self, on: bool):
        _check(lib().lal_tail_debug_phases(self.h, 1 if on else 0))

    def phase_times(self, merge: bool = False):
        """(per-CTA stamps [grid, 8], last-CTA stamps [8]) in ns, relative to
        the earliest CTA start, of the last launch (0 where not written);
        with merge=True also the peer merge's stamps [8]."""
        g = C.c_int()
        _check(lib().lal_tail_debug_phase_read(self.h, None, 0, C.byref(g)))
        out = np.zeros((g.value + 2) * 8, np.uint64)
        _check(lib().lal_tail_debug_phase_read(self.h, _ptr(out), out.size, C.byref(g)))
        st = out.reshape(g.value + 2, 8).astype(np.int64)
        t0 = st[:-2, 0].min()
        rel = np.where(st > 0, st - t0, 0)
        if merge:
            return rel[:-2], rel[-2], rel[-1]
        return rel[:-2], rel[-2]

    def stream(self) -> int:
        s = C.c_void_p()
        _check(lib().lal_tail_get_stream(self.h, C.byref(s)))
        return s.value or 0

    def step_device(self, d_hidden: int, n_streams: int, d_u: int, d_tokens: int):
        _check(lib().lal_tail_step_device(self.h, d_hidden, n_streams, d_u, d_tokens))

    def sync(self):
        _check(lib().lal_tail_sync(self.h))

    # ---- host staging and the vocab-sharded step ----
    def stage_inputs(self, hidden: np.ndarray, u: np.ndarray) -> int:
        hidden = np.ascontiguousarray(hidden, np.float32)
        B = 1 if hidden.ndim == 1 else hidden.shape[0]
        u = np.ascontiguousarray(u, np.float32).reshape(-1)
        _check(lib().lal_tail_stage_inputs(self.h, hidden.reshape(-1), B, u))
        return B

    def fetch_tokens(self, n_streams: int) -> np.ndarray:
        tok = np.empty(n_streams, np.int32)
        _check(lib().lal_tail_fetch_tokens(self.h, n_streams, tok))
        return tok

    def shard_select(self, d_hidden: int, n_streams: int):
        _check(lib().lal_tail_shard_select(self.h, d_hidden, n_streams))

    def exchange_buffers(self, n_streams: int):
        """(send pointer, receive pointer, bytes per rank) of the sharded step."""
        a, b, n = C.c_void_p(), C.c_void_p(), C.c_size_t()
        _check(lib().lal_tail_exchange_buffers(self.h, n_streams, C.byref(a), C.byref(b),
                                               C.byref(n)))
        return a.value, b.value, n.value

    def shard_merge(self, n_streams: int, d_u: int, d_tokens: int):
        _check(lib().lal_tail_shard_merge(self.h, n_streams, d_u, d_tokens))

    def exchange_handle(self) -> bytes:
        """IPC handle (64 bytes) of this rank's peer-exchange receive buffer."""
        buf = C.create_string_buffer(64)
        _check(lib().lal_tail_exchange_handle(self.h, buf))
        return buf.raw

    def connect_peers(self, handles):
        """handles: every rank's exchange_handle(), in rank order."""
        blob = b"".join(handles)
        if len(blob) != 64 * self.cfg.shard_count:
            raise ValueError("one 64-byte handle per rank expected")
        buf = C.create_string_buffer(blob, len(blob))
        _check(lib().lal_tail_connect_peers(self.h, buf))

    def disconnect_peers(self):
        _check(lib().lal_tail_disconnect_peers(self.h))

    def set_top_p(self, top_p: float):
        """The GPT-2 server's nucleus step (gpt2_server.c:2895-2960), after
        top-k; 0 switches it off.  LAL_SAMPLER_GPT2 contexts only."""
        _check(lib().lal_tail_set_top_p(self.h, C.c_float(top_p)))

    STEP_KINDS = {0: "per_stream", 1: "batched", 2: "gpt2"}

    def step_kind(self, n_streams: int) -> str:
        """'per_stream' (one fused launch a stream), 'batched' (quantize, one
        tcgen05 GEMM pass, a select CTA a stream) or 'gpt2' (the GPT-2
        server's tail)."""
        k = lib().lal_tail_step_kind(self.h, int(n_streams))
        if k < 0:
            _check(-k)
        return self.STEP_KINDS[k]

    def set_lm_head_copies(self, copies: int):
        """Measurement aid: single-stream steps use `copies` identical device
        copies of this slice's LM head in turn, so that a slice smaller than
        L2 is read from HBM at every step (results do not change)."""
        _check(lib().lal_tail_set_lm_head_copies(self.h, int(copies)))

    def set_final_norm(self, norm_w: Optional[np.ndarray], eps: float = 1e-6):
        """Fuse the model's final RMSNorm into the step (qwen7b_server.c:820):
        later steps take the residual stream x and quantize (x * inv_rms) * w.
        None switches it off."""
        if norm_w is None:
            _check(lib().lal_tail_set_final_norm(self.h, None, C.c_float(0.0)))
            return
        w = np.ascontiguousarray(norm_w, np.float32)
        if w.size != self.cfg.n_embd:
            raise ValueError(f"norm weights: {w.size} values for n_embd {self.cfg.n_embd}")
        _check(lib().lal_tail_set_final_norm(self.h, _ptr(w), C.c_float(eps)))

    def set_filter(self, filt=None, draw: Optional[Callable[[], float]] = None, decode=None):
        """Level-2 filter hook for step(): filt(keep, n_vocab, last, recent,
        n_recent, decode) edits the keep mask; draw() is called only where the
        server calls rand().  set_filter() with no arguments switches it off."""
        self._filter_refs = (
            FILTER_FN(filt) if filt is not None else None,
            DECODE_FN(decode) if decode is not None else None,
            DRAW_FN(lambda _ctx: float(draw())) if draw is not None else None)
        cf, cd, cw = self._filter_refs
        _check(lib().lal_tail_set_filter(
            self.h, C.cast(cf, C.c_void_p) if cf else None, C.cast(cd, C.c_void_p) if cd else None,
            C.cast(cw, C.c_void_p) if cw else None, None))
