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
