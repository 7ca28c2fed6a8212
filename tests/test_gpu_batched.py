"""GPU parity of the batched step (B >= 2 streams: one pass over the LM head
on the tcgen05 tensor cores, then one select/draw CTA per stream).

Logits are compared bit for bit with the reference's expression
(scale_x*scale_w[v])*(float)dot; the int32 dots are exact, so the GEMM must
reproduce them exactly whatever the tile split (odd V, d not a multiple of the
128-byte K box).  Tokens and per-step intermediates are compared with one
oracle decode loop per stream.  The full-size C3 (B=64) and C4 (B=256) steps
check every stream's logits against a float64 BLAS product (exact here:
|dot| < 2^26) and every stream's token against the oracle sampler.
"""
import numpy as np
import pytest

import lal_b200 as L
import oracle
from conftest import bits
from lal_b200 import synth

pytestmark = pytest.mark.gpu


def _tail(cfg, q, s, B, variant=0, max_top_k=None):
    t = L.DecodeTail(cfg.vocab, cfg.n_embd, max_streams=B,
                     max_top_k=max_top_k or max(cfg.top_k, 1), history_cap=cfg.hist,
                     sampler=variant)
    t.load_lm_head_q8(q, s)
    return t


def _exact_logits(h, q, s):
    """[B, V] logits of the reference expression via float64 dots."""
    B = h.shape[0]
    xq = np.empty((B, q.shape[1]), np.int8)
    sx = np.empty(B, np.float32)
    for b in range(B):
        sx[b], xq[b] = oracle.quantize_x(h[b])
    dots = (xq.astype(np.float64) @ q.astype(np.float64).T).astype(np.int64)
    assert np.abs(dots).max() < (1 << 31)
    return (sx[:, None] * s[None, :]).astype(np.float32) * dots.astype(np.float32)


@pytest.mark.parametrize("V,d,B", [(20000, 768, 5), (1531, 200, 3), (12345, 3584, 33),
                                   (777, 128, 2)])
def test_batched_logits_bit_exact(V, d, B):
    cfg = synth.CONFIGS["c3_batch"].with_(vocab=V, n_embd=d, streams=B, hist=0, steps=1)
    W = synth.lm_head_f32(cfg)
    q, s = oracle.quantize_rows(W, "port")
    t = _tail(cfg, q, s, B)
    temps = synth.temperatures(cfg)[:B]
    t.set_sampling(temps, [cfg.top_k] * B, [1.0] * B)
    h = synth.hidden(cfg, 0, B)
    u = np.full(B, 0.5, np.float32)
    t.step(h, u)
    want = _exact_logits(h, q, s)
    for b in range(B):
        np.testing.assert_array_equal(bits(t.logits(b)), bits(want[b]), err_msg=f"stream {b}")
    t.close()


@pytest.mark.parametrize("variant", [0, 1])
@pytest.mark.parametrize("vocab,top_k,hist", [(9000, 50, 256), (40000, 20, 64)])
def test_batched_decode_loops_match_oracle(variant, vocab, top_k, hist):
    """B = 6 streams, per-stream temperature and history, 6 steps.  The
    first shape is too small for the group bound (k + history ids above an
    eighth of the 32-row groups: full histogram pass), the second takes it."""
    base = synth.CONFIGS["c3_batch"]
    B = 6
    cfg = base.with_(vocab=vocab, n_embd=512, streams=B, steps=6, top_k=top_k, hist=hist)
    W = synth.lm_head_f32(cfg)
    q, s = oracle.quantize_rows(W, "port")
    temps = synth.temperatures(cfg)[:B]
    t = _tail(cfg, q, s, B, variant)
    t.set_sampling(temps, [cfg.top_k] * B, [cfg.rep_penalty] * B)
    ports = []
    for b in range(B):
        hb = synth.history(cfg, b)
        t.set_history(b, hb)
        ports.append(oracle.PortLoop(q, s, hb, cfg.hist, float(temps[b]), cfg.top_k,
                                     cfg.rep_penalty, variant))
    draws = synth.Draws(cfg, B)
    for step in range(cfg.steps):
        h = synth.hidden(cfg, step, B)
        u = np.array([draws.u(b) for b in range(B)], np.float32)
        toks = t.step(h, u)
        for b in range(B):
            ptok, info = ports[b].step(h[b], u[b])
            d = t.diag(b)
            assert int(toks[b]) == ptok, (variant, step, b)
            assert d["threshold"] == info.threshold
            assert bits(d["sum"]) == bits(info.sum)
            assert d["n_cand"] == info.n_cand
            if step == 0:
                np.testing.assert_array_equal(bits(t.logits(b)), bits(ports[b].logits))
    for b in range(B):
        np.testing.assert_array_equal(t.get_history(b), ports[b].history())
    t.close()


def test_batched_greedy_and_topk_mix():
    """Greedy and sampled streams in one step; k above a slice of the
    histogram; a stream without history."""
    cfg = synth.CONFIGS["c3_batch"].with_(vocab=30011, n_embd=256, streams=4, steps=3)
    W = synth.lm_head_f32(cfg)
    q, s = oracle.quantize_rows(W, "port")
    t = _tail(cfg, q, s, 4, max_top_k=1024)
    temps = [0.0, 0.8, 1.0, 0.6]
    ks = [40, 1024, 7, 0]
    pens = [1.1, 1.3, 1.0, 1.2]
    t.set_sampling(temps, ks, pens)
    ports = []
    for b in range(4):
        hb = synth.history(cfg, b) if b != 2 else np.zeros(0, np.int32)
        t.set_history(b, hb)
        ports.append(oracle.PortLoop(q, s, hb, cfg.hist, temps[b], ks[b], pens[b], 0))
    rng = np.random.default_rng(9)
    for step in range(cfg.steps):
        h = synth.hidden(cfg, step, 4)
        u = rng.random(4).astype(np.float32)
        toks = t.step(h, u)
        for b in range(4):
            assert int(toks[b]) == ports[b].step(h[b], u[b])[0], (step, b)
    t.close()


def _full_size_step(cfg, B, ks, temps, steps):
    W = synth.lm_head_f32(cfg)
    q, s = oracle.quantize_rows(W, "port")
    del W
    t = _tail(cfg, q, s, B, max_top_k=max(max(ks), 1))
    t.set_sampling(temps, ks, [cfg.rep_penalty] * B)
    hists = []
    for b in range(B):
        hb = synth.history(cfg, b) if cfg.hist else np.zeros(0, np.int32)
        t.set_history(b, hb)
        hists.append(list(hb))
    draws = synth.Draws(cfg, B)
    for step in range(steps):
        h = synth.hidden(cfg, step, B)
        u = np.array([draws.u(b) for b in range(B)], np.float32)
        toks = t.step(h, u)
        want = _exact_logits(h, q, s)
        for b in range(B):
            rec = np.array(hists[b], np.int32) if hists[b] else None
            ptok, plog, info = oracle.sample(want[b], temps[b], ks[b], cfg.rep_penalty, rec, u[b])
            assert int(toks[b]) == ptok, (step, b)
            if b % 17 == 0:
                np.testing.assert_array_equal(bits(t.logits(b)), bits(plog))
            if cfg.hist:
                hists[b].append(ptok)
                if len(hists[b]) > cfg.hist:
                    hists[b].pop(0)
    t.close()


@pytest.mark.slow
def test_full_size_c3_batch64():
    cfg = synth.CONFIGS["c3_batch"]
    B = cfg.streams
    _full_size_step(cfg, B, [cfg.top_k] * B, [float(x) for x in synth.temperatures(cfg)], 2)


@pytest.mark.slow
def test_full_size_c4_dense256_greedy_and_topk():
    cfg = synth.CONFIGS["c4_dense"]
    B = cfg.streams
    temps = [0.0 if b % 2 == 0 else 0.8 for b in range(B)]
    _full_size_step(cfg, B, [cfg.top_k] * B, temps, 1)
