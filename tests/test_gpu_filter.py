"""The level-2 filter hook inside the fused context (lal_tail_set_filter):
a decode loop of the server sampler with a filter that drops the last token
and every even candidate (the contract of tests/verify_qwen7b_lal.c:45-67 in
the reference), one step where the filter empties the mask (the server
restores it), and greedy steps (no filter).  Tokens, the history and the
number of rand() draws consumed equal the oracle's
lal_sample_token_filtered loop."""
import numpy as np
import pytest

import cases
import lal_b200 as L
import oracle
from lal_b200 import synth

pytestmark = pytest.mark.gpu


def _drop_last_and_even(keep, n_vocab, last, recent, n_recent, decode):
    dropped = 0
    for v in range(n_vocab):
        if keep[v] and (v == last or v % 2 == 0):
            keep[v] = 0
            dropped += 1
    return dropped


def _ban_all(keep, n_vocab, last, recent, n_recent, decode):
    for v in range(n_vocab):
        keep[v] = 0
    return n_vocab


@pytest.mark.parametrize("temperature", [0.8, 0.0])
def test_fused_filter_loop_matches_oracle(temperature):
    spec = cases.loop_cases()["tiny_srv"]
    cfg, W, hist0 = cases.loop_inputs(spec)
    q, s = oracle.quantize_rows(W, "port")
    t = L.DecodeTail(cfg.vocab, cfg.n_embd, max_streams=1, max_top_k=cfg.top_k,
                     history_cap=cfg.hist, sampler=L.LAL_SAMPLER_SERVER)
    t.load_lm_head_q8(q, s)
    t.set_sampling([temperature], [cfg.top_k], [cfg.rep_penalty])
    t.set_history(0, hist0)
    g_gpu = synth.GlibcStream(77, private=True)
    g_orc = synth.GlibcStream(77, private=True)
    hist = list(hist0)
    for step in range(16):
        filt = _ban_all if step == 5 else _drop_last_and_even
        t.set_filter(filt, draw=g_gpu.next_u)
        h = synth.hidden(cfg, step)
        tok = int(t.step(h, np.array([0.0], np.float32))[0])
        sx, xq = oracle.quantize_x(h[0], "port")
        lg = oracle.lm_head(xq, sx, q, s)
        want, _, _ = oracle.sample_filtered(lg, temperature, cfg.top_k, cfg.rep_penalty,
                                            np.array(hist, np.int32), draw=g_orc.next_u,
                                            filt=filt)
        assert tok == want, (temperature, step)
        if temperature > 0 and filt is _drop_last_and_even:
            assert tok % 2 == 1 and tok != hist[-1]
        hist.append(tok)
        if len(hist) > cfg.hist:
            hist.pop(0)
    # the same number of rand() draws were consumed on both sides
    assert g_gpu.next_int() == g_orc.next_int()
    np.testing.assert_array_equal(t.get_history(0), np.array(hist, np.int32))
    t.set_filter()
    t.close()


def test_filter_needs_the_server_sampler():
    t = L.DecodeTail(1000, 128, max_streams=1, max_top_k=8, history_cap=4,
                     sampler=L.LAL_SAMPLER_LIBRARY)
    with pytest.raises(L.LalTailError) as ei:
        t.set_filter(_drop_last_and_even)
    assert ei.value.code == 8
    t.close()
