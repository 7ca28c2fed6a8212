"""lal_tail_sample_token_noalloc (device logits, static scratch, no
allocation) against the existing entry lal_tail_sample_token (host logits,
buffers grown on demand): the same token and the same penalised logits, bit
for bit, on two calls in a row with different shapes and parameters.  Named
to be collected last, so it runs both after the other GPU tests and alone in
a fresh process (``pytest tests/test_zz_no_alloc.py``)."""
import ctypes as C

import numpy as np
import pytest

import lal_b200 as L

pytestmark = pytest.mark.gpu


def _case(seed, V, T, k, pen, n_hist, u):
    rng = np.random.default_rng(seed)
    logits = (rng.standard_normal(V) * 3.0).astype(np.float32)
    recent = rng.integers(0, V, size=n_hist).astype(np.int32)
    return logits, recent, T, k, pen, np.float32(u)


def _existing(logits, recent, T, k, pen, u):
    lg = logits.copy()
    tok = C.c_int(-1)
    rc = L.lib().lal_tail_sample_token(lg, lg.size, np.float32(T), k, np.float32(pen),
                                       recent.ctypes.data if recent.size else None,
                                       recent.size, u, C.byref(tok))
    assert rc == 0, L.lib().lal_tail_last_error()
    return tok.value, lg


def _noalloc(logits, recent, T, k, pen, u):
    import torch
    d_lg = torch.from_numpy(logits.copy()).to("cuda:0")
    d_rec = torch.from_numpy(recent.copy()).to("cuda:0") if recent.size else None
    torch.cuda.synchronize()
    tok = C.c_int(-1)
    rc = L.lib().lal_tail_sample_token_noalloc(
        d_lg.data_ptr(), logits.size, np.float32(T), k, np.float32(pen),
        d_rec.data_ptr() if d_rec is not None else None, recent.size, u, None, C.byref(tok))
    assert rc == 0, L.lib().lal_tail_last_error()
    return tok.value, d_lg.cpu().numpy()


def test_noalloc_matches_existing_on_two_calls_in_a_row():
    cases = [
        _case(11, 152064, 0.7, 40, 1.1, 256, 0.4172),   # Qwen vocab, small-k select
        _case(12, 50257, 0.8, 1024, 1.3, 64, 0.9031),   # GPT-2 vocab, large-k select
    ]
    got = [_noalloc(*c) for c in cases]          # two no-alloc calls in a row
    want = [_existing(*c) for c in cases]
    for (tg, lg), (tw, lw) in zip(got, want):
        assert tg == tw
        np.testing.assert_array_equal(lg.view(np.int32), lw.view(np.int32))
    # and interleaved with the existing entry, then greedy
    g = _case(13, 152064, 0.0, 40, 1.1, 256, 0.5)
    assert _noalloc(*g)[0] == _existing(*g)[0]
    assert _noalloc(*cases[0])[0] == want[0][0]


def test_noalloc_rejects_vocab_above_its_limit():
    tok = C.c_int(-1)
    dummy = C.c_void_p(16)  # never dereferenced: the size check comes first
    rc = L.lib().lal_tail_sample_token_noalloc(dummy, (1 << 18) + 1, np.float32(0.7), 40,
                                               np.float32(1.1), None, 0, np.float32(0.5),
                                               None, C.byref(tok))
    assert rc == 1  # LAL_TAIL_ERR_ARG
    assert b"static scratch limit" in L.lib().lal_tail_last_error()
