"""The CPU restatement (oracle/lal_oracle.c) against the golden vectors made by
the reference's own C, and -- where oracle/_ref was built from the reference
sources -- against that build on fresh random cases.  Pins the oracle before
the GPU suite trusts it."""
import hashlib

import numpy as np
import pytest

import cases
import oracle
from conftest import bits
from lal_b200 import synth


def h(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()[:16]


def test_quantize_x_matches_golden(golden, golden_meta):
    for i, x in enumerate(cases.quantize_x_inputs()):
        assert h(x) == golden_meta["hashes"][f"qx{i}"], "input generator drifted"
        s, xq = oracle.quantize_x(x, "port")
        assert bits(s) == bits(golden[f"qx{i}_scale"])
        np.testing.assert_array_equal(xq, golden[f"qx{i}_xq"])


def test_lm_head_and_row_quantizer_match_golden(golden, golden_meta):
    for i, (W, x, ranges) in enumerate(cases.lm_head_inputs()):
        assert h(W) + h(x) == golden_meta["hashes"][f"lm{i}"]
        q, s = oracle.quantize_rows(W, "port")
        assert h(q) == golden_meta["hashes"][f"lm{i}_q"]
        np.testing.assert_array_equal(bits(s), bits(golden[f"lm{i}_s"]))
        sx, xq = oracle.quantize_x(x, "port")
        for j, (v0, v1) in enumerate(ranges):
            lg = oracle.lm_head(xq, sx, q, s, v0, v1)
            np.testing.assert_array_equal(bits(lg), bits(golden[f"lm{i}_r{j}"]))
            lg8 = oracle.lm_head_8row(xq, sx, q, s, v0, v1)
            np.testing.assert_array_equal(bits(lg8), bits(golden[f"lm{i}_r{j}_8row"]))


def test_8row_quirk_is_real(golden):
    """d=100 is not a multiple of 32: the reference's 8-row form differs."""
    i = 2
    assert not np.array_equal(bits(golden[f"lm{i}_r0"]), bits(golden[f"lm{i}_r0_8row"]))


@pytest.mark.parametrize("variant", ["lib", "srv"])
def test_samplers_match_golden(golden, golden_meta, variant):
    n = 0
    for i, c in enumerate(cases.sampler_cases()):
        key = f"s{i}_{variant}_tok"
        if key not in golden.files:
            continue
        lg = cases.sampler_logits(c)
        rec = cases.sampler_recent(c)
        assert h(lg) + h(rec) == golden_meta["hashes"][f"s{i}"]
        g = synth.GlibcStream(c["seed"], private=False)
        if variant == "lib":
            greedy = c["temperature"] <= 0 or c["top_k"] <= 0
            u = 0.0 if greedy else g.next_u()
            tok, mut, info = oracle.sample(lg, c["temperature"], c["top_k"], c["penalty"], rec, u)
        else:
            tok, mut, info = oracle.sample_filtered(lg, c["temperature"], c["top_k"],
                                                    c["penalty"], rec, draw=g.next_u)
        assert tok == int(golden[key]), (i, c)
        idx = golden[f"s{i}_{variant}_mut_idx"]
        changed = np.nonzero(bits(mut) != bits(lg))[0]
        np.testing.assert_array_equal(changed, idx)
        np.testing.assert_array_equal(bits(mut[idx]), bits(golden[f"s{i}_{variant}_mut_val"]))
        # the same number of rand() draws was consumed
        assert g.next_int() == int(golden[f"s{i}_{variant}_next_rand"])
        n += 1
    assert n >= 15


@pytest.mark.parametrize("name", ["tiny_lib", "tiny_srv", "odd_shape", "c5_like", "c1_gpt2"])
def test_decode_loops_match_golden(golden, name):
    spec = cases.loop_cases()[name]
    cfg, W, hist0 = cases.loop_inputs(spec)
    q, s = oracle.quantize_rows(W, "port")
    loop = oracle.PortLoop(q, s, hist0, cfg.hist, cfg.temperature, cfg.top_k, cfg.rep_penalty,
                           spec["variant"])
    g = synth.GlibcStream(cfg.seed, private=False)
    toks = []
    for step in range(cfg.steps):
        tok, info = loop.step(synth.hidden(cfg, step)[0], g.next_u())
        toks.append(tok)
    np.testing.assert_array_equal(np.array(toks, np.int32), golden[f"loop_{name}_tokens"])


@pytest.mark.skipif(not oracle.have_ref(), reason="oracle/_ref not built (no reference checkout)")
def test_port_matches_reference_on_random_cases():
    R = oracle.ref()
    rng = np.random.default_rng(7)
    for trial in range(150):
        V = int(rng.integers(2, 2500))
        k = int(rng.integers(1, 65))
        T = float(rng.uniform(0.2, 2.0)) if trial % 9 else 0.0
        lg = (rng.standard_normal(V) * 3).astype(np.float32)
        if trial % 4 == 0:
            lg = np.round(lg).astype(np.float32)
        rec = rng.integers(-2, V + 2, size=int(rng.integers(0, 400))).astype(np.int32)
        p = float(rng.choice([1.0, 1.1, 1.3]))
        for filt in (False, True):
            R.ref_srand(trial)
            tr, lr = oracle.ref_sample(lg, T, k, p, rec, filtered=filt)
            g = synth.GlibcStream(trial, private=False)
            if filt:
                tp, lp, _ = oracle.sample_filtered(lg, T, k, p, rec, draw=g.next_u)
            else:
                u = g.next_u() if (T > 0 and k > 0) else 0.0
                tp, lp, _ = oracle.sample(lg, T, k, p, rec, u)
            assert tr == tp, (trial, filt)
            np.testing.assert_array_equal(bits(lr), bits(lp))


@pytest.mark.skipif(not oracle.have_ref(), reason="oracle/_ref not built (no reference checkout)")
def test_port_quantizers_match_reference_on_random_rows():
    rng = np.random.default_rng(3)
    for d in (16, 96, 768, 1000):
        W = (rng.standard_normal((50, d)) * rng.uniform(1e-3, 3)).astype(np.float32)
        qa, sa = oracle.quantize_rows(W, "ref")
        qb, sb = oracle.quantize_rows(W, "port")
        np.testing.assert_array_equal(qa, qb)
        np.testing.assert_array_equal(bits(sa), bits(sb))
        for n in (d, d - 3 if d > 3 else d):
            x = (rng.standard_normal(n) * 5).astype(np.float32)
            s1, x1 = oracle.quantize_x(x, "ref")
            s2, x2 = oracle.quantize_x(x, "port")
            assert bits(s1) == bits(s2)
            np.testing.assert_array_equal(x1, x2)


def test_uncapped_heap_defines_large_k():
    """k beyond the reference's static heaps (64 / 512) is defined in the
    restatement: its threshold is the k-th largest value with multiplicity."""
    rng = np.random.default_rng(5)
    lg = np.round(rng.standard_normal(5000) * 2).astype(np.float32)
    for k in (65, 513, 1024, 4999):
        tok, mut, info = oracle.sample(lg, 0.7, k, 1.0, None, 0.5)
        assert info.threshold == np.sort(lg)[::-1][k - 1]
        assert info.n_cand == int((lg >= info.threshold).sum())


def test_rms_norm_matches_golden(golden, golden_meta):
    for i, (x, w, eps) in enumerate(cases.rms_norm_inputs()):
        assert h(x) + h(w) == golden_meta["hashes"][f"rn{i}"], "input generator drifted"
        np.testing.assert_array_equal(bits(oracle.rms_norm(x, w, float(eps), "port")),
                                      bits(golden[f"rn{i}"]))


@pytest.mark.skipif(not oracle.have_ref(), reason="oracle/_ref not built")
def test_rms_norm_port_matches_reference_on_random_vectors():
    """Fresh vectors of lengths that are multiples of 8."""
    g = np.random.default_rng(3)
    for trial in range(200):
        n = int(g.choice([8, 16, 776, 768, 3584, 1000, 4096]))
        x = (g.standard_normal(n) * g.uniform(0.01, 50)).astype(np.float32)
        w = (1 + 0.2 * g.standard_normal(n)).astype(np.float32)
        np.testing.assert_array_equal(bits(oracle.rms_norm(x, w, 1e-6, "port")),
                                      bits(oracle.rms_norm(x, w, 1e-6, "ref")))


def test_gpt2_lm_head_matches_golden(golden, golden_meta):
    """The GPT-2 server's int8 LM head and float re-score: every logit, and
    which rows the heap re-scored -- including 21 rows tied at the 512th
    place, of which the server's heap history keeps 8."""
    for name, q, s, x in cases.gpt2_lm_inputs():
        assert h(q) + h(s) + h(x) == golden_meta["hashes"][f"g2_{name}_in"]
        sx, xq = oracle.gpt2_quantize_x(x, "port")
        assert bits(sx) == bits(golden[f"g2_{name}_sx"])
        np.testing.assert_array_equal(xq, golden[f"g2_{name}_xq"])
        logits, kept = oracle.gpt2_lm_head(x, q, s, "port")
        assert h(logits) == golden_meta["hashes"][f"g2_{name}_logits"], name
        rows = golden[f"g2_{name}_rescored_rows"]
        assert set(rows.tolist()) <= set(kept.tolist())
        np.testing.assert_array_equal(bits(logits[rows]), bits(golden[f"g2_{name}_rescored_vals"]))


@pytest.mark.skipif(not oracle.have_ref_gpt2(), reason="oracle/_ref not built")
def test_gpt2_quantizer_matches_reference_on_random_vectors():
    g = np.random.default_rng(17)
    for trial in range(50):
        x = (g.standard_normal(768) * g.uniform(1e-9, 30)).astype(np.float32)
        if trial % 5 == 0:
            x[g.integers(768)] = np.nan
        sp, qp = oracle.gpt2_quantize_x(x, "port")
        sr, qr = oracle.gpt2_quantize_x(x, "ref")
        assert bits(sp) == bits(sr)
        np.testing.assert_array_equal(qp, qr)


def test_gpt2_sampler_is_the_library_sampler_but_at_r_zero():
    """gpt2_server.c:2862-3013 restated: its k passes of find-max-and-mask and
    its kept-row softmax give the library sampler's token (pinned against the
    reference above) for every draw but r == 0, where its running sum stops
    at row 0."""
    g = np.random.default_rng(8)
    for trial in range(60):
        V = int(g.integers(50, 3000))
        logits = (g.standard_normal(V) * 3).astype(np.float32)
        if trial % 4 == 0:
            logits[g.integers(V, size=V // 5)] = logits[0]   # ties
        T = float(g.choice([0.0, 0.7, 1.3]))
        k = int(g.choice([0, 1, 5, 40, 64]))
        rec = g.integers(0, V, size=int(g.integers(0, 30))).astype(np.int32)
        u = np.float32(g.integers(0, 1000000) / 1e6)
        tg, ig, lg = oracle.gpt2_sample(logits, T, k, 1.1, rec, u)
        tl, ll, il = oracle.sample(logits, T, k, 1.1, rec, u)
        if not ig.greedy and ig.r == 0.0:
            assert tg == 0
        else:
            assert tg == tl, trial
        np.testing.assert_array_equal(bits(lg), bits(ll))
        if not ig.greedy:
            assert bits(ig.sum) == bits(il.sum) and ig.n_cand == il.n_cand
    # a zero draw
    lg = np.array([1.0, 5.0, 4.0, -2.0], np.float32)
    assert oracle.gpt2_sample(lg, 0.8, 2, 1.0, None, 0.0)[0] == 0
    assert oracle.sample(lg, 0.8, 2, 1.0, None, 0.0)[0] == 1


@pytest.mark.skipif(not oracle.have_ref(), reason="oracle/_ref not built (no reference checkout)")
def test_port_matches_reference_on_exact_ties():
    """Every logit 0.0 (an all-zero hidden) and 300 rows tied at the 40th
    place: the candidate set is the whole vocabulary, or k + 300 rows; the
    restatement returns the reference's token for both samplers and many
    draws (the GPU's wide path is checked against the same reference)."""
    rng = np.random.default_rng(21)
    V = 152064
    zero = np.zeros(V, np.float32)
    tied = rng.standard_normal(V).astype(np.float32)
    order = np.argsort(-tied, kind="stable")
    rows = rng.choice(order[60:], size=300, replace=False)
    tied[rows] = tied[order[39]]
    rec = rng.integers(0, V, size=200).astype(np.int32)
    R = oracle.ref()
    for lg in (zero, tied):
        for seed in range(6):
            for temp in (0.7, 0.0):
                R.ref_srand(seed)
                want, want_lg = oracle.ref_sample(lg, temp, 40, 1.1, rec)
                u = synth.GlibcStream(seed, private=False).next_u()
                got, got_lg, info = oracle.sample(lg, temp, 40, 1.1, rec, u)
                assert got == want, (seed, temp)
                if temp > 0:  # (the penalty may move a tied or a top row)
                    assert info.n_cand == V if lg is zero else info.n_cand >= 300
                np.testing.assert_array_equal(bits(got_lg), bits(want_lg))
                R.ref_srand(seed)
                want_s, _ = oracle.ref_sample(lg, temp, 40, 1.1, rec, filtered=True)
                g = synth.GlibcStream(seed, private=False)
                got_s, _, _ = oracle.sample_filtered(lg, temp, 40, 1.1, rec, draw=g.next_u)
                assert got_s == want_s, (seed, temp)


@pytest.mark.skipif(not oracle.have_ref(), reason="oracle/_ref not built (no reference checkout)")
def test_port_matches_reference_at_extreme_temperatures_and_scales():
    """Temperatures from 1e-3 (every weight but the largest underflows to 0 or a
    subnormal) to 1e3 (all weights near 1), and logits from 1e-30 to 1e30 in
    magnitude: the restatement's weights, sums and draws are the reference's
    (runtime/lal_sampling.h:106-124), for both samplers."""
    R = oracle.ref()
    rng = np.random.default_rng(99)
    trial = 0
    for scale in (1e-30, 1e-3, 1.0, 1e4, 1e30):
        for T in (1e-3, 0.05, 0.7, 30.0, 1e3):
            V = int(rng.integers(50, 3000))
            k = int(rng.integers(1, 65))
            lg = (rng.standard_normal(V) * scale).astype(np.float32)
            rec = rng.integers(0, V, size=64).astype(np.int32)
            for filt in (False, True):
                R.ref_srand(trial)
                tr, lr = oracle.ref_sample(lg, T, k, 1.1, rec, filtered=filt)
                g = synth.GlibcStream(trial, private=False)
                if filt:
                    tp, lp, _ = oracle.sample_filtered(lg, T, k, 1.1, rec, draw=g.next_u)
                else:
                    tp, lp, _ = oracle.sample(lg, T, k, 1.1, rec, g.next_u())
                assert tr == tp, (scale, T, filt)
                np.testing.assert_array_equal(bits(lr), bits(lp))
            trial += 1
