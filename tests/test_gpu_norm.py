"""GPU parity of the final RMSNorm fused into the tail's prologue
(lal_tail_set_final_norm; runtime/lal_simd_optim.h:32-58 as called at
tools/server/qwen7b_server.c:820): the step takes the residual stream x, and
its logits, diagnostics and tokens equal the oracle's RMSNorm -> tail step,
bit for bit, in the per-stream, batched and sharded-emulation forms."""
import numpy as np
import pytest

import lal_b200 as L
import oracle
from conftest import bits
from lal_b200 import synth

pytestmark = pytest.mark.gpu


def residual(cfg, step, rng):
    """A pre-norm residual stream: the synthetic hidden scaled up, so that
    the norm changes the quantized vector."""
    return (synth.hidden(cfg, step)[0] * np.float32(rng.uniform(2.0, 40.0))).astype(np.float32)


@pytest.mark.parametrize("name,variant", [("c1_gpt2", L.LAL_SAMPLER_LIBRARY),
                                          ("c2_qwen", L.LAL_SAMPLER_SERVER)])
def test_fused_norm_matches_oracle(name, variant):
    cfg = synth.CONFIGS[name].with_(vocab=9001, hist=64)
    W = synth.lm_head_f32(cfg)
    rng = np.random.default_rng(11)
    w = (1.0 + 0.2 * rng.standard_normal(cfg.n_embd)).astype(np.float32)
    t = L.DecodeTail(cfg.vocab, cfg.n_embd, max_top_k=cfg.top_k, history_cap=cfg.hist,
                     sampler=variant)
    t.load_lm_head_f32(W)
    q, s = t.read_lm_head()
    hist0 = synth.history(cfg, 0)
    t.set_sampling([cfg.temperature], [cfg.top_k], [cfg.rep_penalty])
    t.set_history(0, hist0)
    t.set_final_norm(w, 1e-6)
    port = oracle.PortLoop(q, s, hist0, cfg.hist, cfg.temperature, cfg.top_k,
                           cfg.rep_penalty, variant)
    g = synth.GlibcStream(cfg.seed, private=False)
    for step in range(12):
        x = residual(cfg, step, rng)
        u = g.next_u()
        tok = int(t.step(x[None, :], np.array([u], np.float32))[0])
        ptok, info = port.step(oracle.rms_norm(x, w, 1e-6), u)
        assert tok == ptok, step
        d = t.diag(0)
        assert bits(d["sum"]) == bits(info.sum), step
        assert d["n_cand"] == info.n_cand
        np.testing.assert_array_equal(bits(t.logits(0)), bits(port.logits))
    # switched off: the hidden is quantized as given again
    t.set_final_norm(None)
    h = synth.hidden(cfg, 99)
    u = g.next_u()
    tok = int(t.step(h, np.array([u], np.float32))[0])
    ptok, _ = port.step(h[0], u)
    assert tok == ptok
    t.close()


def test_batched_norm_matches_oracle():
    """B >= 2 takes the quantize -> tensor-core GEMM -> select path; the norm
    runs in its quantize kernel."""
    B = 6
    cfg = synth.CONFIGS["c3_batch"].with_(vocab=12007, hist=32, streams=B)
    W = synth.lm_head_f32(cfg)
    rng = np.random.default_rng(5)
    w = (1.0 + 0.3 * rng.standard_normal(cfg.n_embd)).astype(np.float32)
    t = L.DecodeTail(cfg.vocab, cfg.n_embd, max_streams=B, max_top_k=cfg.top_k,
                     history_cap=cfg.hist)
    t.load_lm_head_f32(W)
    q, s = t.read_lm_head()
    temps = [0.5 + 0.1 * b for b in range(B)]
    t.set_sampling(temps, [cfg.top_k] * B, [cfg.rep_penalty] * B)
    ports = []
    for b in range(B):
        h0 = synth.history(cfg, b)
        t.set_history(b, h0)
        ports.append(oracle.PortLoop(q, s, h0, cfg.hist, temps[b], cfg.top_k,
                                     cfg.rep_penalty, L.LAL_SAMPLER_LIBRARY))
    t.set_final_norm(w, 1e-5)
    for step in range(4):
        x = np.stack([residual(cfg, step * B + b, rng) for b in range(B)])
        u = rng.random(B).astype(np.float32)
        toks = t.step(x, u)
        for b in range(B):
            ptok, info = ports[b].step(oracle.rms_norm(x[b], w, 1e-5), u[b])
            assert int(toks[b]) == ptok, (step, b)
            assert bits(t.diag(b)["sum"]) == bits(info.sum)
    t.close()


def test_norm_rejects_bad_arguments():
    cfg = synth.CONFIGS["c1_gpt2"].with_(vocab=4000, hist=8)
    t = L.DecodeTail(cfg.vocab, cfg.n_embd, max_top_k=cfg.top_k, history_cap=cfg.hist)
    with pytest.raises(ValueError):
        t.set_final_norm(np.ones(cfg.n_embd + 1, np.float32))
    with pytest.raises(L.LalTailError):
        t.set_final_norm(np.ones(cfg.n_embd, np.float32), float("nan"))
    t.close()
    # wider than the prologue holds, or not a multiple of 8 (the reference's
    # scalar tail loop would run): refused
    for d in (4104, 100):
        other = L.DecodeTail(4000, d, max_top_k=8, history_cap=8)
        with pytest.raises(L.LalTailError):
            other.set_final_norm(np.ones(d, np.float32))
        other.close()
