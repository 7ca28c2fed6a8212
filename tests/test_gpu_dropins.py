"""GPU parity of the reference-named drop-ins (through the C ABI) with the
golden vectors produced by the reference's own C and with the oracle."""
import threading

import numpy as np
import pytest

import cases
import lal_b200 as L
import oracle
from conftest import bits
from lal_b200 import synth

pytestmark = pytest.mark.gpu


def test_quantize_x(golden):
    for i, x in enumerate(cases.quantize_x_inputs()):
        s, xq = L.quantize_x_int8(x)
        assert bits(s) == bits(golden[f"qx{i}_scale"]), i
        np.testing.assert_array_equal(xq, golden[f"qx{i}_xq"])


def test_compute_abs_xq():
    xq = np.arange(-127, 128, dtype=np.int8)
    np.testing.assert_array_equal(L.compute_abs_xq(xq), np.abs(xq.astype(np.int16)).astype(np.uint8))


def test_quantize_q8_per_row(golden):
    for i, (W, x, ranges) in enumerate(cases.lm_head_inputs()):
        q, s = L.quantize_q8_per_row(W)
        qo, so = oracle.quantize_rows(W, "port")
        np.testing.assert_array_equal(q, qo)
        np.testing.assert_array_equal(bits(s), bits(golden[f"lm{i}_s"]))
    # a larger random case with exact .5 products and zero rows
    rng = np.random.default_rng(1)
    W = (rng.standard_normal((3000, 777)) * 0.02).astype(np.float32)
    W[10] = 0
    W[11, :] = np.float32(0.5) * np.arange(777, dtype=np.float32) / 776 * 127 / 63.5
    q, s = L.quantize_q8_per_row(W)
    qo, so = oracle.quantize_rows(W, "port")
    np.testing.assert_array_equal(q, qo)
    np.testing.assert_array_equal(bits(s), bits(so))


def test_lm_head_ranges(golden):
    for i, (W, x, ranges) in enumerate(cases.lm_head_inputs()):
        q, s = oracle.quantize_rows(W, "port")
        sx, xq = oracle.quantize_x(x, "port")
        V = q.shape[0]
        for j, (v0, v1) in enumerate(ranges):
            lg = np.zeros(V, np.float32)
            L.lm_head_int8_range(lg, xq, sx, q, s, v0, v1)
            np.testing.assert_array_equal(bits(lg), bits(golden[f"lm{i}_r{j}"]))
        L.lm_head_forget(q)


def test_lm_head_8row_reproduces_the_dropped_column_tail(golden):
    import ctypes as C
    for i, (W, x, ranges) in enumerate(cases.lm_head_inputs()):
        q, s = oracle.quantize_rows(W, "port")
        sx, xq = oracle.quantize_x(x, "port")
        V, d = q.shape
        ax = np.abs(xq.astype(np.int16)).astype(np.uint8)
        for j, (v0, v1) in enumerate(ranges):
            lg = np.zeros(V, np.float32)
            L.lib().lal_lm_head_int8_range_abs_8row(lg, xq, ax, np.float32(sx), q.reshape(-1),
                                                    s, v0, v1, d)
            np.testing.assert_array_equal(bits(lg), bits(golden[f"lm{i}_r{j}_8row"]))
        L.lm_head_forget(q)


def test_lm_head_concurrent_threads_like_the_server():
    """qwen7b_server.c:833-845 calls the range kernel from OpenMP threads on
    disjoint vocab slices of one shared logits array."""
    cfg = synth.CONFIGS["c1_gpt2"]
    W = synth.lm_head_f32(cfg, 0, 20011)
    q, s = oracle.quantize_rows(W, "port")
    sx, xq = oracle.quantize_x(synth.hidden(cfg, 0)[0], "port")
    V = q.shape[0]
    ref = oracle.lm_head(xq, sx, q, s)
    lg = np.zeros(V, np.float32)
    n = 4
    per = (V + n - 1) // n
    errs = []

    def work(t):
        try:
            L.lm_head_int8_range(lg, xq, sx, q, s, t * per, min(V, (t + 1) * per))
        except Exception as e:  # pragma: no cover
            errs.append(e)

    th = [threading.Thread(target=work, args=(t,)) for t in range(n)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    assert not errs
    np.testing.assert_array_equal(bits(lg), bits(ref))
    L.lm_head_forget(q)


def test_sample_token_library_form(golden):
    n = 0
    for i, c in enumerate(cases.sampler_cases()):
        key = f"s{i}_lib_tok"
        if key not in golden.files:
            continue
        lg = cases.sampler_logits(c)
        rec = cases.sampler_recent(c)
        g = synth.GlibcStream(c["seed"], private=False)
        greedy = c["temperature"] <= 0 or c["top_k"] <= 0
        u = 0.0 if greedy else g.next_u()
        mut = lg.copy()
        tok = L.sample_token(mut, c["temperature"], c["top_k"], c["penalty"], rec, u)
        assert tok == int(golden[key]), (i, c)
        idx = golden[f"s{i}_lib_mut_idx"]
        np.testing.assert_array_equal(np.nonzero(bits(mut) != bits(lg))[0], idx)
        np.testing.assert_array_equal(bits(mut[idx]), bits(golden[f"s{i}_lib_mut_val"]))
        assert g.next_int() == int(golden[f"s{i}_lib_next_rand"])
        n += 1
    assert n >= 15


def test_sample_token_server_form(golden):
    for i, c in enumerate(cases.sampler_cases()):
        lg = cases.sampler_logits(c)
        rec = cases.sampler_recent(c)
        g = synth.GlibcStream(c["seed"], private=False)
        mut = lg.copy()
        tok = L.sample_token_filtered(mut, c["temperature"], c["top_k"], c["penalty"], rec,
                                      draw=g.next_u)
        assert tok == int(golden[f"s{i}_srv_tok"]), (i, c)
        idx = golden[f"s{i}_srv_mut_idx"]
        np.testing.assert_array_equal(np.nonzero(bits(mut) != bits(lg))[0], idx)
        assert g.next_int() == int(golden[f"s{i}_srv_next_rand"])


def test_level2_filter_hook_matches_oracle():
    """A filter that drops the last token and every even candidate
    (the contract of tests/verify_qwen7b_lal.c:45-67)."""
    import ctypes as C

    def filt(keep, n_vocab, last, recent, n_recent, decode):
        dropped = 0
        for v in range(n_vocab):
            if keep[v] and (v == last or v % 2 == 0):
                keep[v] = 0
                dropped += 1
        return dropped

    def ban_all(keep, n_vocab, last, recent, n_recent, decode):
        for v in range(n_vocab):
            keep[v] = 0
        return n_vocab

    rng = np.random.default_rng(9)
    for trial in range(6):
        V = 700
        lg = (rng.standard_normal(V) * 3).astype(np.float32)
        rec = rng.integers(0, V, size=30).astype(np.int32)
        f = ban_all if trial == 5 else filt
        g1 = synth.GlibcStream(50 + trial, private=False)
        mut = lg.copy()
        t_gpu = L.sample_token_filtered(mut, 0.8, 40, 1.1, rec, draw=g1.next_u, filt=f)
        n1 = g1.next_int()
        g2 = synth.GlibcStream(50 + trial, private=False)
        t_orc, _, _ = oracle.sample_filtered(lg, 0.8, 40, 1.1, rec, draw=g2.next_u, filt=f)
        n2 = g2.next_int()
        assert t_gpu == t_orc and n1 == n2, trial
        if f is filt:
            assert t_gpu % 2 == 1 and t_gpu != rec[-1]


def test_large_k_sampler_against_oracle():
    """k = 1024 and heavy ties: beyond the reference's static heaps, so the
    uncapped restatement is the checker."""
    rng = np.random.default_rng(4)
    for V, k in ((152064, 1024), (50257, 200), (9000, 3000)):
        lg = np.round(rng.standard_normal(V) * 3, 1).astype(np.float32)
        rec = rng.integers(0, V, size=500).astype(np.int32)
        u = np.float32(rng.random())
        mut = lg.copy()
        tok = L.sample_token(mut, 0.7, k, 1.3, rec, u)
        t2, m2, info = oracle.sample(lg, 0.7, k, 1.3, rec, u)
        assert tok == t2, (V, k)
        np.testing.assert_array_equal(bits(mut), bits(m2))
