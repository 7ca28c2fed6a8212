"""GPU parity of the fused decode tail (lal_tail_step through the C ABI):
token sequences of whole decode loops against the reference's golden tokens
and the oracle, per-step intermediates bit-exact, and full-size Qwen steps."""
import numpy as np
import pytest

import cases
import lal_b200 as L
import oracle
from conftest import bits
from lal_b200 import synth

pytestmark = pytest.mark.gpu


def make_tail(cfg, variant, W=None, q=None, s=None, streams=1, max_top_k=None):
    t = L.DecodeTail(cfg.vocab, cfg.n_embd, max_streams=streams,
                     max_top_k=max_top_k or max(cfg.top_k, 1), history_cap=cfg.hist,
                     sampler=variant)
    if q is not None:
        t.load_lm_head_q8(q, s)
    else:
        t.load_lm_head_f32(W)
    return t


@pytest.mark.parametrize("name", ["tiny_lib", "tiny_srv", "odd_shape", "c5_like", "c1_gpt2"])
def test_decode_loop_tokens_match_reference(golden, name):
    spec = cases.loop_cases()[name]
    cfg, W, hist0 = cases.loop_inputs(spec)
    t = make_tail(cfg, spec["variant"], W=W)
    # the device quantizer reproduces lal_quantize_q8_per_row bit for bit
    q_dev, s_dev = t.read_lm_head()
    q, s = oracle.quantize_rows(W, "port")
    np.testing.assert_array_equal(q_dev, q)
    np.testing.assert_array_equal(bits(s_dev), bits(s))
    t.set_sampling([cfg.temperature], [cfg.top_k], [cfg.rep_penalty])
    t.set_history(0, hist0)
    port = oracle.PortLoop(q, s, hist0, cfg.hist, cfg.temperature, cfg.top_k,
                           cfg.rep_penalty, spec["variant"])
    g = synth.GlibcStream(cfg.seed, private=False)
    toks = []
    for step in range(cfg.steps):
        h = synth.hidden(cfg, step)
        u = g.next_u()
        tok = int(t.step(h, np.array([u], np.float32))[0])
        ptok, info = port.step(h[0], u)
        d = t.diag(0)
        assert tok == ptok, (name, step)
        # intermediates, bit for bit
        assert bits(d["threshold"]) == bits(info.threshold) or d["threshold"] == info.threshold
        assert bits(d["max_l"]) == bits(info.max_l)
        assert bits(d["sum"]) == bits(info.sum), (name, step)
        assert d["n_cand"] == info.n_cand
        if step == 0:
            np.testing.assert_array_equal(bits(t.logits(0)), bits(port.logits))
        toks.append(tok)
    np.testing.assert_array_equal(np.array(toks, np.int32), golden[f"loop_{name}_tokens"])
    np.testing.assert_array_equal(t.get_history(0), port.history())
    t.close()


def test_greedy_and_tied_maxima():
    """Greedy (k<=0 or T<=0) returns the lowest index among equal maxima,
    even when they sit in different CTA slices."""
    V, d = 20000, 64
    rng = np.random.default_rng(2)
    cfg = synth.CONFIGS["c1_gpt2"].with_(vocab=V, n_embd=d, hist=0, top_k=1)
    W = (rng.standard_normal((V, d)) * 0.02).astype(np.float32)
    for r in (777, 5000, 19999):
        W[r] = W[123]            # identical rows -> identical logits
    x = np.zeros((1, d), np.float32)
    q, s = oracle.quantize_rows(W, "port")
    for variant in (L.LAL_SAMPLER_LIBRARY, L.LAL_SAMPLER_SERVER):
        t = make_tail(cfg, variant, q=q, s=s, max_top_k=8)
        t.set_sampling([0.0], [40], [1.1])
        for trial in range(5):
            x = rng.standard_normal((1, d)).astype(np.float32)
            tok = int(t.step(x, np.array([0.5], np.float32))[0])
            sx, xq = oracle.quantize_x(x[0], "port")
            lg = oracle.lm_head(xq, sx, q, s)
            assert tok == int(np.argmax(lg))
        t.close()


def test_full_size_qwen_steps_match_oracle():
    """C2 shape (V=152064, d=3584, 545 MB int8): a few fused steps, bit-exact
    logits and identical tokens against the restatement."""
    cfg = synth.CONFIGS["c2_qwen"]
    W = synth.lm_head_f32(cfg)
    t = make_tail(cfg, L.LAL_SAMPLER_LIBRARY, W=W)
    q, s = t.read_lm_head()
    qo, so = oracle.quantize_rows(W[:4096], "port")
    np.testing.assert_array_equal(q[:4096], qo)
    del W
    hist0 = synth.history(cfg, 0)
    t.set_sampling([cfg.temperature], [cfg.top_k], [cfg.rep_penalty])
    t.set_history(0, hist0)
    port = oracle.PortLoop(q, s, hist0, cfg.hist, cfg.temperature, cfg.top_k,
                           cfg.rep_penalty, 0)
    g = synth.GlibcStream(cfg.seed, private=False)
    for step in range(3):
        h = synth.hidden(cfg, step)
        u = g.next_u()
        tok = int(t.step(h, np.array([u], np.float32))[0])
        ptok, info = port.step(h[0], u)
        assert tok == ptok
        assert bits(t.diag(0)["sum"]) == bits(info.sum)
        if step == 0:
            np.testing.assert_array_equal(bits(t.logits(0)), bits(port.logits))
    t.close()


def test_stress_k1024_with_duplicate_rows():
    """k = 1024, p = 1.3 over a 4096-id history with repeats, 5% duplicated
    rows (exact ties), heavy-tailed logits: tokens equal the uncapped oracle."""
    base = synth.CONFIGS["c5_stress"]
    cfg = base.with_(vocab=60000, n_embd=512, steps=6)
    W = synth.lm_head_f32(cfg)
    q, s = oracle.quantize_rows(W, "port")
    for variant in (0, 1):
        t = make_tail(cfg, variant, q=q, s=s)
        hist0 = synth.history(cfg, 0)
        t.set_sampling([cfg.temperature], [cfg.top_k], [cfg.rep_penalty])
        t.set_history(0, hist0)
        port = oracle.PortLoop(q, s, hist0, cfg.hist, cfg.temperature, cfg.top_k,
                               cfg.rep_penalty, variant)
        draws = synth.Draws(cfg, 1)
        for step in range(cfg.steps):
            h = synth.hidden(cfg, step, 1)
            u = draws.u(0)
            tok = int(t.step(h, np.array([u], np.float32))[0])
            ptok, info = port.step(h[0], u)
            assert tok == ptok, (variant, step)
            assert t.diag(0)["n_cand"] == info.n_cand
        t.close()


def test_multi_stream_context_runs_streams_independently():
    """B streams in one context, each with its own history and temperature,
    equal B single-stream oracle loops."""
    base = synth.CONFIGS["c3_batch"]
    cfg = base.with_(vocab=8000, n_embd=256, streams=4, steps=5)
    W = synth.lm_head_f32(cfg)
    q, s = oracle.quantize_rows(W, "port")
    temps = synth.temperatures(cfg)[:4]
    t = make_tail(cfg, 0, q=q, s=s, streams=4)
    t.set_sampling(temps, [cfg.top_k] * 4, [cfg.rep_penalty] * 4)
    ports = []
    for b in range(4):
        hb = synth.history(cfg, b)
        t.set_history(b, hb)
        ports.append(oracle.PortLoop(q, s, hb, cfg.hist, float(temps[b]), cfg.top_k,
                                     cfg.rep_penalty, 0))
    draws = synth.Draws(cfg, 4)
    for step in range(cfg.steps):
        h = synth.hidden(cfg, step, 4)
        u = np.array([draws.u(b) for b in range(4)], np.float32)
        toks = t.step(h, u)
        for b in range(4):
            assert int(toks[b]) == ports[b].step(h[b], u[b])[0], (step, b)
    t.close()


def test_lm_head_copies_and_partial_streams_keep_results():
    """Steps that rotate over identical device copies of the LM head
    (lal_tail_set_lm_head_copies, the bench's way past L2) and steps of fewer
    streams than the context holds return the oracle's tokens."""
    spec = cases.loop_cases()["tiny_lib"]
    cfg, W, hist0 = cases.loop_inputs(spec)
    q, s = oracle.quantize_rows(W, "port")
    t = make_tail(cfg, 0, q=q, s=s, streams=3)
    t.set_lm_head_copies(3)
    t.set_sampling([cfg.temperature] * 3, [cfg.top_k] * 3, [cfg.rep_penalty] * 3)
    t.set_history(0, hist0)
    port = oracle.PortLoop(q, s, hist0, cfg.hist, cfg.temperature, cfg.top_k,
                           cfg.rep_penalty, 0)
    g = synth.GlibcStream(cfg.seed, private=False)
    for step in range(7):
        h = synth.hidden(cfg, step)
        u = g.next_u()
        tok = int(t.step(h, np.array([u], np.float32))[0])   # 1 of 3 streams
        assert tok == port.step(h[0], u)[0], step
    np.testing.assert_array_equal(t.get_history(0), port.history())
    t.set_lm_head_copies(1)
    t.close()
