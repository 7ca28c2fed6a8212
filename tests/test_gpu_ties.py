"""GPU parity when the candidate set is large: exact ties at the threshold.

An all-zero hidden vector quantizes to zeros, so every logit is 0.0: T = 0 is
the k-th largest and every row of the vocabulary is a candidate.  LM-head
rows duplicated bit for bit give logits that tie exactly; 300 of them at the
k-th place, spread over one CTA's slice of rows, crowd that CTA's slot of the
small-k select.  The reference returns a token for both
(runtime/lal_sampling.h:70-124, tools/server/qwen7b_server.c:219-295: every
row with l >= T is a candidate).  Each case runs through the drop-in
lal_sample_token, the fused step, a 2-shard emulated step and a B=4 batched
step, against the reference's own compiled C (oracle/_ref) on the same inputs
and the same glibc draws.
"""
import ctypes as C

import numpy as np
import pytest

import lal_b200 as L
import oracle
from conftest import bits
from lal_b200 import synth

pytestmark = pytest.mark.gpu

K, TEMP, PEN, CAP = 40, 0.7, 1.1, 64
SEEDS = (0, 7, 1234)


@pytest.fixture(scope="module", autouse=True)
def _need_ref():
    if not oracle.have_ref():
        pytest.skip("oracle/_ref (the reference's compiled C) is not built")


def ref_tail(q, s, h, hist, variant, seed, temp=TEMP, k=K):
    """The reference's tail step (qwen7b_server.c:829-850) on the same inputs:
    (token, penalised logits, history after the push); its rand() draws after
    srand(seed)."""
    R = oracle.ref()
    V, d = q.shape
    pad = max(32, -(-d // 32) * 32)
    xq = np.zeros(pad, np.int8)
    ax = np.zeros(pad, np.uint8)
    lg = np.zeros(V, np.float32)
    rec = np.zeros(CAP, np.int32)
    rec[:len(hist)] = hist
    n = C.c_int(len(hist))
    R.ref_srand(seed)
    tok = R.ref_tail_step(np.ascontiguousarray(h, np.float32), xq, ax, lg,
                          np.ascontiguousarray(q).reshape(-1), np.ascontiguousarray(s), V, d,
                          np.float32(temp), k, np.float32(PEN), rec, C.byref(n), CAP, 8,
                          variant)
    assert tok >= 0
    return int(tok), lg, rec[:n.value].copy()


def draw_u(seed):
    return synth.GlibcStream(seed, private=False).next_u()


def cta_slice(V, cta, grid=148):
    return V * cta // grid, V * (cta + 1) // grid


def head(V, d, seed=3):
    cfg = synth.CONFIGS["c2_qwen"].with_(vocab=V, n_embd=d, seed=seed)
    return oracle.quantize_rows(synth.lm_head_f32(cfg), "port"), cfg


def penalised(q, s, h, hist):
    sx, xq = oracle.quantize_x(h, "port")
    lg = oracle.lm_head(xq, sx, q, s)
    for t in hist:
        lg[t] = lg[t] / np.float32(PEN) if lg[t] > 0 else lg[t] * np.float32(PEN)
    return lg


def tie_head(q, s, h, hist, n_dup=300, cta=5, k=K):
    """Copy the row at the k-th place (after the penalty) into n_dup rows
    spread over CTA `cta`'s slice: k - 1 rows stay above T and 1 + n_dup rows
    tie at T."""
    V = q.shape[0]
    lg = penalised(q, s, h, hist)
    order = np.argsort(-lg, kind="stable")
    star = int(order[k - 1])
    assert star not in set(hist.tolist())
    lo, hi = cta_slice(V, cta)
    busy = set(hist.tolist()) | set(order[:k + 8].tolist())
    pool = np.array([r for r in range(lo, hi) if r not in busy], np.int64)
    rng = np.random.default_rng(11)
    dup = np.sort(rng.choice(pool, size=n_dup, replace=False))
    q2, s2 = q.copy(), s.copy()
    q2[dup] = q[star]
    s2[dup] = s[star]
    lg2 = penalised(q2, s2, h, hist)
    assert np.sum(lg2 > lg2[star]) == k - 1 and np.sum(lg2 == lg2[star]) == n_dup + 1
    return q2, s2


def cases_for(V, d):
    (q, s), cfg = head(V, d)
    rng = np.random.default_rng(5)
    hist = rng.integers(0, V, size=CAP - 8).astype(np.int32)
    h = synth.hidden(cfg, 0)[0]
    q2, s2 = tie_head(q, s, h, hist)
    zero = np.zeros(d, np.float32)
    return {"zero": (q, s, zero, hist), "dup300": (q2, s2, h, hist)}


@pytest.fixture(scope="module")
def small():
    return cases_for(60000, 512)


# ---- the drop-in sampler --------------------------------------------------------

@pytest.mark.parametrize("kind", ["zero", "dup300"])
def test_dropin_sampler_ties(small, kind):
    q, s, h, hist = small[kind]
    sx, xq = oracle.quantize_x(h, "port")
    lg = oracle.lm_head(xq, sx, q, s)
    for seed in SEEDS:
        for temp, k in ((TEMP, K), (0.0, K)):
            # library form
            R = oracle.ref()
            R.ref_srand(seed)
            want, want_lg = oracle.ref_sample(lg, temp, k, PEN, hist)
            mut = lg.copy()
            got = L.sample_token(mut, temp, k, PEN, hist, draw_u(seed))
            assert got == want, (kind, seed, temp)
            np.testing.assert_array_equal(bits(mut), bits(want_lg))
            # server form
            R.ref_srand(seed)
            want_s, _ = oracle.ref_sample(lg, temp, k, PEN, hist, filtered=True)
            g = synth.GlibcStream(seed, private=False)
            got_s = L.sample_token_filtered(lg.copy(), temp, k, PEN, hist, draw=g.next_u)
            assert got_s == want_s, (kind, seed, temp)
    # the restatement's intermediates for the first seed
    u = draw_u(SEEDS[0])
    tok, _, info = oracle.sample(lg, TEMP, K, PEN, hist, u)
    if kind == "zero":
        assert info.n_cand == lg.size and info.threshold == 0.0
    else:
        assert info.n_cand == K + 300


# ---- the fused step -------------------------------------------------------------

def fused(q, s, variant, streams=1, **kw):
    V, d = q.shape
    t = L.DecodeTail(V, d, max_streams=streams, max_top_k=64, history_cap=CAP, sampler=variant,
                     **kw)
    if "shard_count" in kw:
        t.load_lm_head_q8(q[t.row0:t.row0 + t.n_rows], s[t.row0:t.row0 + t.n_rows])
    else:
        t.load_lm_head_q8(q, s)
    return t


@pytest.mark.parametrize("variant", [L.LAL_SAMPLER_LIBRARY, L.LAL_SAMPLER_SERVER])
@pytest.mark.parametrize("kind", ["zero", "dup300"])
def test_fused_step_ties(small, kind, variant):
    q, s, h, hist = small[kind]
    t = fused(q, s, variant)
    for temp in (TEMP, 0.0):
        t.set_sampling([temp], [K], [PEN])
        for seed in SEEDS:
            t.set_history(0, hist)
            want, want_lg, want_hist = ref_tail(q, s, h, hist, variant, seed, temp=temp)
            got = int(t.step(h[None, :], np.array([draw_u(seed)], np.float32))[0])
            assert got == want, (kind, variant, temp, seed)
            np.testing.assert_array_equal(t.get_history(0), want_hist)
            np.testing.assert_array_equal(bits(t.logits(0)), bits(want_lg))
            if temp > 0 and variant == L.LAL_SAMPLER_LIBRARY:
                _, _, info = oracle.sample(want_lg, temp, K, 1.0, None, draw_u(seed))
                d = t.diag(0)
                assert d["n_cand"] == info.n_cand
                assert bits(d["sum"]) == bits(info.sum) and bits(d["r"]) == bits(info.r)
    # a normal step right after: the fast path again, same answer as the reference
    t.set_sampling([TEMP], [K], [PEN])
    t.set_history(0, hist)
    hn = synth.hidden(synth.CONFIGS["c2_qwen"].with_(vocab=q.shape[0], n_embd=q.shape[1]), 3)[0]
    want, _, _ = ref_tail(q, s, hn, hist, variant, 99)
    assert int(t.step(hn[None, :], np.array([draw_u(99)], np.float32))[0]) == want
    t.close()


# ---- the vocab-sharded step, two shards emulated on one GPU ----------------------

def sharded_step(tails, h, u):
    import torch
    from lal_b200.sharded import _DeviceBytes
    n = 1 if h.ndim == 1 else h.shape[0]
    for t in tails:
        t.stage_inputs(h, u)
        t.shard_select(t.device_buffers()[0], n)
    torch.cuda.synchronize()
    views = []
    for t in tails:
        send, recv, nb = t.exchange_buffers(n)
        views.append((torch.as_tensor(_DeviceBytes(send, nb), device="cuda:0"),
                      torch.as_tensor(_DeviceBytes(recv, nb * len(tails)), device="cuda:0"), nb))
    for dst in views:
        for r, src in enumerate(views):
            dst[1][r * src[2]:(r + 1) * src[2]].copy_(src[0][:src[2]])
    torch.cuda.synchronize()
    for t in tails:
        _, d_u, d_tok = t.device_buffers()
        t.shard_merge(n, d_u, d_tok)
    return [t.fetch_tokens(n) for t in tails]


@pytest.mark.parametrize("variant", [L.LAL_SAMPLER_LIBRARY, L.LAL_SAMPLER_SERVER])
@pytest.mark.parametrize("kind", ["zero", "dup300"])
def test_sharded_step_ties(small, kind, variant):
    q, s, h, hist = small[kind]
    tails = [fused(q, s, variant, shard_rank=r, shard_count=2, device=0) for r in range(2)]
    for temp in (TEMP, 0.0):
        for seed in SEEDS:
            for t in tails:
                t.set_sampling([temp], [K], [PEN])
                t.set_history(0, hist)
            want, _, want_hist = ref_tail(q, s, h, hist, variant, seed, temp=temp)
            per = sharded_step(tails, h[None, :], np.array([draw_u(seed)], np.float32))
            for r, tk in enumerate(per):
                assert int(tk[0]) == want, (kind, variant, temp, seed, r)
                np.testing.assert_array_equal(tails[r].get_history(0), want_hist)
    for t in tails:
        t.close()


# ---- the batched step (tensor-core GEMM, per-stream select) ---------------------

@pytest.mark.parametrize("variant", [L.LAL_SAMPLER_LIBRARY, L.LAL_SAMPLER_SERVER])
def test_batched_step_ties(small, variant):
    q, s, h_dup, hist = small["dup300"]
    d = q.shape[1]
    hn = synth.hidden(synth.CONFIGS["c2_qwen"].with_(vocab=q.shape[0], n_embd=d), 5)[0]
    H = np.stack([np.zeros(d, np.float32), h_dup, hn, np.zeros(d, np.float32)])
    temps = [TEMP, TEMP, 0.9, 0.0]
    hists = [hist, hist, hist[::-1].copy(), hist[:10].copy()]
    t = fused(q, s, variant, streams=4)
    t.set_sampling(temps, [K] * 4, [PEN] * 4)
    for seed in SEEDS:
        for b in range(4):
            t.set_history(b, hists[b])
        seeds = [seed + 17 * b for b in range(4)]
        u = np.array([draw_u(x) for x in seeds], np.float32)
        got = t.step(H, u)
        for b in range(4):
            want, _, want_hist = ref_tail(q, s, H[b], hists[b], variant, seeds[b], temp=temps[b])
            assert int(got[b]) == want, (variant, seed, b)
            np.testing.assert_array_equal(t.get_history(b), want_hist)
    t.close()


# ---- the same at the C2 shape ----------------------------------------------------

@pytest.mark.slow
def test_c2_shape_ties_every_path():
    """V=152064, d=3584 (545 MB): the zero hidden and 300 tied rows at the
    40th place, through the drop-in, the fused step, two emulated shards and a
    B=4 batched step, both samplers."""
    cs = cases_for(152064, 3584)
    for kind in ("zero", "dup300"):
        q, s, h, hist = cs[kind]
        sx, xq = oracle.quantize_x(h, "port")
        lg = oracle.lm_head(xq, sx, q, s)
        for variant in (L.LAL_SAMPLER_LIBRARY, L.LAL_SAMPLER_SERVER):
            seed = 42 + variant
            want, want_lg, want_hist = ref_tail(q, s, h, hist, variant, seed)
            # drop-in
            mut = lg.copy()
            if variant == L.LAL_SAMPLER_LIBRARY:
                got = L.sample_token(mut, TEMP, K, PEN, hist, draw_u(seed))
                np.testing.assert_array_equal(bits(mut), bits(want_lg))
            else:
                g = synth.GlibcStream(seed, private=False)
                got = L.sample_token_filtered(mut, TEMP, K, PEN, hist, draw=g.next_u)
            assert got == want, ("dropin", kind, variant)
            # fused
            t = fused(q, s, variant, streams=4)
            t.set_sampling([TEMP] * 4, [K] * 4, [PEN] * 4)
            t.set_history(0, hist)
            got = int(t.step(h[None, :], np.array([draw_u(seed)], np.float32))[0])
            assert got == want, ("fused", kind, variant)
            np.testing.assert_array_equal(t.get_history(0), want_hist)
            # batched: the case in every stream
            for b in range(4):
                t.set_history(b, hist)
            toks = t.step(np.stack([h] * 4), np.array([draw_u(seed)] * 4, np.float32))
            assert all(int(x) == want for x in toks), ("batched", kind, variant)
            t.close()
            # two shards
            tails = [fused(q, s, variant, shard_rank=r, shard_count=2, device=0)
                     for r in range(2)]
            for tt in tails:
                tt.set_sampling([TEMP], [K], [PEN])
                tt.set_history(0, hist)
            per = sharded_step(tails, h[None, :], np.array([draw_u(seed)], np.float32))
            assert all(int(p[0]) == want for p in per), ("sharded", kind, variant)
            for tt in tails:
                tt.close()
