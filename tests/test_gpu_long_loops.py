"""Every BASELINE configuration at its stated shape and step count on the GPU
(through the C ABI), against the reference: token ids of every step, and the
final histories.

- C2 (Qwen B=1, 512 steps) and C1 (GPT-2 shape, 256 steps): the reference's
  own compiled tail (oracle/_ref, qwen7b_server.c:829-850) drawing from glibc
  rand() after srand(seed), and the GPU given the same draws.
- C3 (B=64, 32 steps), C4 (B=256, 8 iterations, greedy and k=40) and C5 (B=8,
  k=1024, H=4096, 30% repeated history ids, 5% duplicated LM-head rows, 128
  steps; also as 8 shards emulated on one GPU): the restatement, per stream
  with its own random_r draws -- the reference's heap holds k <= 64
  (runtime/lal_sampling.h:74), and its sampler draws from the one global
  rand().  The restatement is pinned to the reference in test_oracle.py.
"""
import ctypes as C

import numpy as np
import pytest

import lal_b200 as L
import oracle
from lal_b200 import synth

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


def gpu_tail(cfg, streams=None, **kw):
    B = cfg.streams if streams is None else streams
    t = L.DecodeTail(cfg.vocab, cfg.n_embd, max_streams=B, max_top_k=max(cfg.top_k, 1),
                     history_cap=cfg.hist, device=0, **kw)
    for r in range(0, t.n_rows, 8192):
        n = min(8192, t.n_rows - r)
        t.load_lm_head_f32(synth.lm_head_f32(cfg, t.row0 + r, t.row0 + r + n), r)
    return t


def ref_loop(cfg, q, s, variant=0):
    """The reference's tail over cfg.steps steps: (tokens, final history)."""
    R = oracle.ref()
    V, d = cfg.vocab, cfg.n_embd
    pad = max(32, -(-d // 32) * 32)
    xq, ax = np.zeros(pad, np.int8), np.zeros(pad, np.uint8)
    logits = np.zeros(V, np.float32)
    cap = max(1, cfg.hist)
    h0 = synth.history(cfg, 0)
    rec = np.zeros(cap, np.int32)
    rec[:h0.size] = h0
    n = C.c_int(h0.size)
    R.ref_srand(cfg.seed)
    toks = []
    for step in range(cfg.steps):
        tok = R.ref_tail_step(synth.hidden(cfg, step)[0], xq, ax, logits, q.reshape(-1), s, V,
                              d, np.float32(cfg.temperature), cfg.top_k,
                              np.float32(cfg.rep_penalty), rec, C.byref(n), cap, 16, variant)
        assert tok >= 0
        toks.append(tok)
    return np.array(toks, np.int32), rec[:n.value].copy()


@pytest.mark.parametrize("name", ["c2_qwen", "c1_gpt2"])
def test_single_stream_full_length_loop_matches_reference(name):
    if not oracle.have_ref():
        pytest.skip("oracle/_ref not built")
    cfg = synth.CONFIGS[name]
    assert cfg.steps == {"c2_qwen": 512, "c1_gpt2": 256}[name]
    t = gpu_tail(cfg)
    q, s = t.read_lm_head()
    want, want_hist = ref_loop(cfg, q, s)
    t.set_sampling([cfg.temperature], [cfg.top_k], [cfg.rep_penalty])
    t.set_history(0, synth.history(cfg, 0))
    g = synth.GlibcStream(cfg.seed, private=False)
    got = np.array([int(t.step(synth.hidden(cfg, step), np.array([g.next_u()], np.float32))[0])
                    for step in range(cfg.steps)], np.int32)
    first_bad = np.nonzero(got != want)[0]
    assert first_bad.size == 0, f"{name}: first differing step {first_bad[:1]}"
    np.testing.assert_array_equal(t.get_history(0), want_hist)
    t.close()


def batched_loop(cfg, steps, t_list, temps, top_ks, variant=0):
    """Run `steps` batched steps on the GPU context(s) in t_list (one context,
    or the shards of an emulated sharded step) against PortBatch."""
    B = cfg.streams
    t0 = t_list[0]
    q, s = t0.read_lm_head()
    hists = [synth.history(cfg, b) for b in range(B)]
    port = oracle.PortBatch(q, s, hists, cfg.hist, temps, top_ks, cfg.rep_penalty, variant)
    for t in t_list:
        t.set_sampling(temps, top_ks, [cfg.rep_penalty] * B)
        for b in range(B):
            t.set_history(b, hists[b])
    draws = synth.Draws(cfg)
    return port, draws


@pytest.mark.parametrize("name,steps", [("c3_batch", 32), ("c5_stress", 128)])
def test_batched_full_size_loop_matches_restatement(name, steps):
    cfg = synth.CONFIGS[name]
    B = cfg.streams
    t = gpu_tail(cfg)
    assert t.step_kind(B) == "batched"
    temps = synth.temperatures(cfg)
    port, draws = batched_loop(cfg, steps, [t], temps, [cfg.top_k] * B)
    for step in range(steps):
        h = synth.hidden(cfg, step)
        u = np.array([draws.u(b) for b in range(B)], np.float32)
        got = t.step(h, u)
        want = port.step(h, u)
        assert np.array_equal(got, want), (name, step, np.nonzero(got != want)[0][:4])
    for b in range(B):
        np.testing.assert_array_equal(t.get_history(b), port.history(b))
    t.close()


def test_c4_dense_256_streams_greedy_and_top40():
    """C4: 256 streams, 8 iterations; even streams greedy, odd ones k=40."""
    cfg = synth.CONFIGS["c4_dense"]
    B = cfg.streams
    t = gpu_tail(cfg)
    assert t.step_kind(B) == "batched"
    temps = [0.0 if b % 2 == 0 else cfg.temperature for b in range(B)]
    port, draws = batched_loop(cfg, 8, [t], temps, [cfg.top_k] * B)
    for step in range(8):
        h = synth.hidden(cfg, step)
        u = np.array([draws.u(b) for b in range(B)], np.float32)
        got = t.step(h, u)
        want = port.step(h, u)
        assert np.array_equal(got, want), (step, np.nonzero(got != want)[0][:4])
    t.close()


def test_c5_eight_emulated_shards_128_steps():
    """C5 as 8 vocab shards on one GPU (contexts shard r of 8; the records'
    all-gather done by device copies): every shard returns the restated
    unsharded tokens on all 8 streams for 128 steps."""
    import torch
    from lal_b200.sharded import _DeviceBytes
    cfg = synth.CONFIGS["c5_stress"]
    B, N = cfg.streams, 8
    tails = [gpu_tail(cfg, shard_rank=r, shard_count=N) for r in range(N)]
    qs = [t.read_lm_head() for t in tails]
    q = np.concatenate([x for x, _ in qs])
    s = np.concatenate([y for _, y in qs])
    temps = synth.temperatures(cfg)
    hists = [synth.history(cfg, b) for b in range(B)]
    port = oracle.PortBatch(q, s, hists, cfg.hist, temps, [cfg.top_k] * B, cfg.rep_penalty, 0)
    for t in tails:
        t.set_sampling(temps, [cfg.top_k] * B, [cfg.rep_penalty] * B)
        for b in range(B):
            t.set_history(b, hists[b])
    views = []
    for t in tails:
        send, recv, nb = t.exchange_buffers(B)
        views.append((torch.as_tensor(_DeviceBytes(send, nb), device="cuda:0"),
                      torch.as_tensor(_DeviceBytes(recv, nb * N), device="cuda:0"), nb))
    draws = synth.Draws(cfg)
    for step in range(cfg.steps):
        h = synth.hidden(cfg, step)
        u = np.array([draws.u(b) for b in range(B)], np.float32)
        for t in tails:
            t.stage_inputs(h, u)
            t.shard_select(t.device_buffers()[0], B)
        torch.cuda.synchronize()
        for dst in views:
            for r, src in enumerate(views):
                dst[1][r * src[2]:(r + 1) * src[2]].copy_(src[0][:src[2]])
        torch.cuda.synchronize()
        for t in tails:
            _, d_u, d_tok = t.device_buffers()
            t.shard_merge(B, d_u, d_tok)
        want = port.step(h, u)
        for r, t in enumerate(tails):
            got = t.fetch_tokens(B)
            assert np.array_equal(got, want), (step, r, np.nonzero(got != want)[0][:4])
    for t in tails:
        for b in range(B):
            np.testing.assert_array_equal(t.get_history(b), port.history(b))
        t.close()
