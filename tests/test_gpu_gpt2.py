"""GPU parity of the GPT-2 server's tail as a second drop-in (a context with
LAL_SAMPLER_GPT2; tools/server/gpt2_server.c:1982-2214 and 2862-3013):
tokens, diagnostics, the re-scored and penalised logits and the history,
bit for bit against the oracle's restatement (whose LM head is pinned to the
server's own compiled code by tests/test_oracle.py)."""
import numpy as np
import pytest

import cases
import lal_b200 as L
import oracle
from conftest import bits
from lal_b200 import synth

pytestmark = pytest.mark.gpu


def gpt2_tail(q, s, cfg, max_top_k=40):
    t = L.DecodeTail(cfg.vocab, cfg.n_embd, max_top_k=max_top_k, history_cap=cfg.hist,
                     sampler=L.LAL_SAMPLER_GPT2)
    t.load_lm_head_q8(q, s)
    return t


def draws(n, seed):
    """(rand() % 1000000) / 1e6, as the server draws; one exact zero."""
    g = np.random.default_rng(seed)
    u = (g.integers(0, 1000000, n) / np.float32(1e6)).astype(np.float32)
    u[min(3, n - 1)] = 0.0
    return u


def test_gpt2_decode_loop_matches_oracle():
    cfg = synth.CONFIGS["c1_gpt2"]
    W = synth.lm_head_f32(cfg)
    q, s = oracle.quantize_rows(W, "port")
    hist0 = synth.history(cfg, 0)
    t = gpt2_tail(q, s, cfg)
    t.set_sampling([cfg.temperature], [cfg.top_k], [cfg.rep_penalty])
    t.set_history(0, hist0)
    port = oracle.Gpt2PortLoop(q, s, hist0, cfg.hist, cfg.temperature, cfg.top_k,
                               cfg.rep_penalty)
    us = draws(16, 4)
    for step in range(16):
        x = synth.hidden(cfg, step)
        tok = int(t.step(x, us[step:step + 1])[0])
        ptok, info = port.step(x[0], us[step])
        assert tok == ptok, step
        d = t.diag(0)
        assert bits(d["sum"]) == bits(info.sum) and d["n_cand"] == info.n_cand, step
        assert bits(d["threshold"]) == bits(info.threshold)
        np.testing.assert_array_equal(bits(t.logits(0)), bits(port.logits))
    np.testing.assert_array_equal(t.get_history(0), port.history())
    # greedy: argmax of the re-scored logits, no penalty
    t.set_sampling([0.0], [cfg.top_k], [cfg.rep_penalty])
    port.T = 0.0
    for step in range(3):
        x = synth.hidden(cfg, 100 + step)
        tok = int(t.step(x, np.zeros(1, np.float32))[0])
        ptok, _ = port.step(x[0], 0.0)
        assert tok == ptok
        np.testing.assert_array_equal(bits(t.logits(0)), bits(port.logits))
    t.close()


def test_gpt2_boundary_ties_replay_the_heap():
    """21 rows tie at the 512th largest int8 logit: the kernel replays the
    server's heap to re-score the same 8 of them."""
    cfg = synth.CONFIGS["c1_gpt2"].with_(hist=8)
    for name, q, s, x in cases.gpt2_lm_inputs():
        t = gpt2_tail(q, s, cfg, max_top_k=50)
        t.set_sampling([0.9], [50], [1.0])
        t.set_history(0, np.zeros(0, np.int32))
        port = oracle.Gpt2PortLoop(q, s, [], cfg.hist, 0.9, 50, 1.0)
        tok = int(t.step(x[None, :], np.array([0.25], np.float32))[0])
        ptok, _ = port.step(x, np.float32(0.25))
        assert tok == ptok, name
        np.testing.assert_array_equal(bits(t.logits(0)), bits(port.logits), err_msg=name)
        t.close()


def test_gpt2_small_vocab_rescore_all_rows():
    """Fewer rows than the re-score window: every row is re-scored."""
    cfg = synth.CONFIGS["c1_gpt2"].with_(vocab=300, hist=16)
    rng = np.random.default_rng(9)
    W = (rng.standard_normal((cfg.vocab, cfg.n_embd)) * 0.02).astype(np.float32)
    q, s = oracle.quantize_rows(W, "port")
    t = gpt2_tail(q, s, cfg)
    t.set_sampling([0.8], [40], [1.1])
    hist0 = rng.integers(0, cfg.vocab, 16).astype(np.int32)
    t.set_history(0, hist0)
    port = oracle.Gpt2PortLoop(q, s, hist0, cfg.hist, 0.8, 40, 1.1)
    for step, u in enumerate(draws(6, 2)):
        x = rng.standard_normal((1, cfg.n_embd)).astype(np.float32)
        assert int(t.step(x, np.array([u], np.float32))[0]) == port.step(x[0], u)[0], step
        np.testing.assert_array_equal(bits(t.logits(0)), bits(port.logits))
    t.close()


def test_gpt2_context_limits():
    with pytest.raises(L.LalTailError):
        L.DecodeTail(1000, 100, max_top_k=8, history_cap=8, sampler=L.LAL_SAMPLER_GPT2)


@pytest.mark.parametrize("kind", ["crowded_bin", "mass_ties"])
def test_gpt2_crowded_boundary_bin(kind):
    """More than 4096 logits in the 12-bit bin that holds the 512th largest:
    the select's radix path.  crowded_bin: nearly equal rows (distinct
    values, the rows at or above T are exactly 512); mass_ties: 6000 identical
    rows tie across the boundary (the heap replay decides which are kept)."""
    cfg = synth.CONFIGS["c1_gpt2"].with_(hist=8)
    V, d = cfg.vocab, cfg.n_embd
    rng = np.random.default_rng(21 if kind == "crowded_bin" else 22)
    base = rng.standard_normal(d).astype(np.float32)
    if kind == "crowded_bin":
        W = (base[None, :] + 0.002 * rng.standard_normal((V, d))).astype(np.float32)
    else:
        W = (0.05 * rng.standard_normal((V, d))).astype(np.float32)
        W[rng.choice(V, 6000, replace=False)] = base * 0.05
    q, s = oracle.quantize_rows(W * 0.02, "port")
    x = (base * 3.0).astype(np.float32)
    lg = oracle.gpt2_lm_head(x, q, s)[0]
    sx, xq = oracle.gpt2_quantize_x(x, "port")
    plain = (sx * s) * (q.astype(np.int32) @ xq.astype(np.int32)).astype(np.float32)
    key = plain.view(np.uint32)
    key = np.where(key >> 31 == 1, ~key, key | 0x80000000).astype(np.uint32)
    T = np.sort(key)[::-1][511]
    assert (key >> 20 == T >> 20).sum() > 4096, "the case must crowd the boundary bin"
    assert ((key >= T).sum() == 512) == (kind == "crowded_bin")
    t = gpt2_tail(q, s, cfg)
    t.set_sampling([0.8], [40], [1.0])
    t.set_history(0, np.zeros(0, np.int32))
    port = oracle.Gpt2PortLoop(q, s, [], cfg.hist, 0.8, 40, 1.0)
    tok = int(t.step(x[None, :], np.array([0.4], np.float32))[0])
    ptok, _ = port.step(x, np.float32(0.4))
    assert tok == ptok
    np.testing.assert_array_equal(bits(t.logits(0)), bits(port.logits))
    t.close()


@pytest.mark.parametrize("top_p", [0.3, 0.9])
def test_gpt2_top_p_loop_matches_oracle(top_p):
    """The server's nucleus step after top-k (gpt2_server.c:2895-2960):
    tokens, kept count, sums and history of a C1 loop against the
    restatement of that branch."""
    cfg = synth.CONFIGS["c1_gpt2"]
    W = synth.lm_head_f32(cfg)
    q, s = oracle.quantize_rows(W, "port")
    hist0 = synth.history(cfg, 0)
    t = gpt2_tail(q, s, cfg)
    t.set_top_p(top_p)
    t.set_sampling([cfg.temperature], [cfg.top_k], [cfg.rep_penalty])
    t.set_history(0, hist0)
    port = oracle.Gpt2PortLoop(q, s, hist0, cfg.hist, cfg.temperature, cfg.top_k,
                               cfg.rep_penalty, top_p=top_p)
    us = draws(12, 9)
    kept = []
    for step in range(12):
        x = synth.hidden(cfg, step)
        tok = int(t.step(x, us[step:step + 1])[0])
        ptok, info = port.step(x[0], us[step])
        assert tok == ptok, (top_p, step)
        d = t.diag(0)
        assert d["n_cand"] == info.n_cand and bits(d["sum"]) == bits(info.sum), (top_p, step)
        kept.append(info.n_cand)
    assert min(kept) < cfg.top_k  # the nucleus really cut the pool
    np.testing.assert_array_equal(t.get_history(0), port.history())
    t.close()


def test_gpt2_top_p_over_an_all_tied_vocabulary():
    """An all-zero hidden vector: every row's logit is 0.0 (the re-scored rows
    too), so the top-k pool is the whole vocabulary at one probability and the
    nucleus keeps its first rows by index -- the select's wide path."""
    cfg = synth.CONFIGS["c1_gpt2"]
    W = synth.lm_head_f32(cfg)
    q, s = oracle.quantize_rows(W, "port")
    t = gpt2_tail(q, s, cfg)
    t.set_sampling([cfg.temperature], [cfg.top_k], [cfg.rep_penalty])
    t.set_history(0, np.zeros(0, np.int32))
    x = np.zeros((1, cfg.n_embd), np.float32)
    for top_p in (0.0, 0.25, 0.75):
        t.set_top_p(top_p)
        port = oracle.Gpt2PortLoop(q, s, np.zeros(0, np.int32), cfg.hist, cfg.temperature,
                                   cfg.top_k, cfg.rep_penalty, top_p=top_p)
        for u in (0.1, 0.6, 0.999):
            t.set_history(0, np.zeros(0, np.int32))
            port.n.value = 0
            tok = int(t.step(x, np.array([u], np.float32))[0])
            ptok, info = port.step(x[0], np.float32(u))
            assert tok == ptok, (top_p, u)
            assert t.diag(0)["n_cand"] == info.n_cand, (top_p, u)
    t.close()


def _drop_last_and_even(keep, n_vocab, last, recent, n_recent, decode):
    """The reference's test filter (tests/verify_qwen7b_lal.c:45-67): drops
    the last token and every even row."""
    ks = np.ctypeslib.as_array(keep, shape=(n_vocab,))
    dropped = int(ks[::2].sum())
    ks[::2] = 0
    if 0 <= last < n_vocab and ks[last]:
        ks[last] = 0
        dropped += 1
    return dropped


def _ban_all(keep, n_vocab, last, recent, n_recent, decode):
    np.ctypeslib.as_array(keep, shape=(n_vocab,))[:] = 0
    return n_vocab


def _add_rows(keep, n_vocab, last, recent, n_recent, decode):
    """A filter that also keeps rows outside the top-k pool: the server's
    softmax then runs over them too (gpt2_server.c:2981-2994)."""
    ks = np.ctypeslib.as_array(keep, shape=(n_vocab,))
    ks[7] = 1
    ks[n_vocab - 3] = 1
    return 0


@pytest.mark.parametrize("top_p", [0.0, 0.9])
def test_gpt2_filter_hook_loop_matches_oracle(top_p):
    """The GPT-2 server's level-2 filter call (gpt2_server.c:2962-2978) inside
    the GPT-2 context (lal_tail_set_filter): a C1 loop whose filter drops the
    last token and every even row, one step where it empties the mask (the
    top-k pool is restored), one where it adds rows, greedy steps (no
    filter): tokens and history against the restatement."""
    cfg = synth.CONFIGS["c1_gpt2"]
    W = synth.lm_head_f32(cfg)
    q, s = oracle.quantize_rows(W, "port")
    hist0 = synth.history(cfg, 0)
    t = gpt2_tail(q, s, cfg)
    t.set_top_p(top_p)
    t.set_history(0, hist0)
    port = oracle.Gpt2PortLoop(q, s, hist0, cfg.hist, cfg.temperature, cfg.top_k,
                               cfg.rep_penalty, top_p=top_p)
    us = draws(12, 21)
    for step in range(12):
        filt = {4: _ban_all, 7: _add_rows}.get(step, _drop_last_and_even)
        temp = 0.0 if step == 9 else cfg.temperature
        t.set_sampling([temp], [cfg.top_k], [cfg.rep_penalty])
        port.T = temp
        t.set_filter(filt)
        port.filt = filt
        x = synth.hidden(cfg, step)
        tok = int(t.step(x, us[step:step + 1])[0])
        ptok, info = port.step(x[0], us[step])
        assert tok == ptok, (top_p, step)
        if filt is _drop_last_and_even and temp > 0:
            assert tok % 2 == 1 or us[step] == 0.0
        np.testing.assert_array_equal(bits(t.logits(0)), bits(port.logits), err_msg=str(step))
    np.testing.assert_array_equal(t.get_history(0), port.history())
    t.set_filter(None)
    t.close()
