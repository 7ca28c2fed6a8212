"""GPU parity of the vocab-sharded step.

Emulated on one GPU: N contexts (shard r of N, each with its own slice of
the LM head) run lal_tail_shard_select, the records are all-gathered with
device copies between the contexts' exchange buffers (no kernel waits on
another), and every context runs lal_tail_shard_merge.  Every shard must
return the unsharded step's token (the reference's golden decode-loop tokens
and the oracle's per-step intermediates, bit for bit), and the same token on
every shard.  With two or more GPUs, the same loop runs over NCCL through
lal_b200.sharded.ShardedDecodeTail, one process per GPU.
"""
import os
import socket

import numpy as np
import pytest

import cases
import lal_b200 as L
import oracle
from conftest import bits
from lal_b200 import synth

pytestmark = pytest.mark.gpu


def _tails(cfg, variant, q, s, n_shards, streams=1, max_top_k=None):
    tails = []
    for r in range(n_shards):
        t = L.DecodeTail(cfg.vocab, cfg.n_embd, max_streams=streams,
                         max_top_k=max_top_k or max(cfg.top_k, 1), history_cap=cfg.hist,
                         sampler=variant, device=0, shard_rank=r, shard_count=n_shards)
        t.load_lm_head_q8(q[t.row0:t.row0 + t.n_rows], s[t.row0:t.row0 + t.n_rows])
        tails.append(t)
    return tails


def _views(t, n):
    import torch
    from lal_b200.sharded import _DeviceBytes
    send, recv, nb = t.exchange_buffers(n)
    vs = torch.as_tensor(_DeviceBytes(send, nb), device="cuda:0")
    vr = torch.as_tensor(_DeviceBytes(recv, nb * t.cfg.shard_count), device="cuda:0")
    return vs, vr, nb


def _step(tails, h, u):
    """One emulated sharded step; returns each shard's tokens (or raises the
    first shard's error after every shard has run)."""
    import torch
    n = 1 if h.ndim == 1 else h.shape[0]
    for t in tails:
        t.stage_inputs(h, u)
        d_hid, _, _ = t.device_buffers()
        t.shard_select(d_hid, n)
    torch.cuda.synchronize()  # every context's stream (errors surface at the merge)
    views = [_views(t, n) for t in tails]
    for dst in views:
        for r, src in enumerate(views):
            nb = src[2]
            dst[1][r * nb:(r + 1) * nb].copy_(src[0][:nb])
    torch.cuda.synchronize()
    for t in tails:
        _, d_u, d_tok = t.device_buffers()
        t.shard_merge(n, d_u, d_tok)
    out, err = [], None
    for t in tails:
        try:
            out.append(t.fetch_tokens(n))
        except L.LalTailError as e:
            err = err or e
    if err is not None:
        raise err
    return out


@pytest.mark.parametrize("n_shards", [2, 3, 8])
@pytest.mark.parametrize("name", ["tiny_lib", "tiny_srv", "odd_shape", "c5_like", "c1_gpt2"])
def test_sharded_loop_matches_reference(golden, name, n_shards):
    spec = cases.loop_cases()[name]
    cfg, W, hist0 = cases.loop_inputs(spec)
    q, s = oracle.quantize_rows(W, "port")
    tails = _tails(cfg, spec["variant"], q, s, n_shards)
    for t in tails:
        t.set_sampling([cfg.temperature], [cfg.top_k], [cfg.rep_penalty])
        t.set_history(0, hist0)
    port = oracle.PortLoop(q, s, hist0, cfg.hist, cfg.temperature, cfg.top_k,
                           cfg.rep_penalty, spec["variant"])
    g = synth.GlibcStream(cfg.seed, private=False)
    toks = []
    for step in range(cfg.steps):
        h = synth.hidden(cfg, step)
        u = g.next_u()
        per = _step(tails, h, np.array([u], np.float32))
        ptok, info = port.step(h[0], u)
        for r, tk in enumerate(per):
            assert int(tk[0]) == ptok, (name, n_shards, step, r)
            d = tails[r].diag(0)
            assert d["threshold"] == info.threshold
            assert bits(d["max_l"]) == bits(info.max_l)
            assert bits(d["sum"]) == bits(info.sum), (name, step, r)
            assert d["n_cand"] == info.n_cand
        if step == 0:
            lg = np.concatenate([t.logits(0) for t in tails])
            np.testing.assert_array_equal(bits(lg), bits(port.logits))
        toks.append(ptok)
    np.testing.assert_array_equal(np.array(toks, np.int32), golden[f"loop_{name}_tokens"])
    for t in tails:
        np.testing.assert_array_equal(t.get_history(0), port.history())
        t.close()


def test_sharded_greedy_ties_across_shards():
    """Equal maxima in different slices: the lowest index wins on every shard."""
    V, d = 20000, 64
    rng = np.random.default_rng(4)
    cfg = synth.CONFIGS["c1_gpt2"].with_(vocab=V, n_embd=d, hist=0, top_k=1)
    W = (rng.standard_normal((V, d)) * 0.02).astype(np.float32)
    for r in (9000, 14999, 19999):
        W[r] = W[7001]
    q, s = oracle.quantize_rows(W, "port")
    for variant in (L.LAL_SAMPLER_LIBRARY, L.LAL_SAMPLER_SERVER):
        tails = _tails(cfg, variant, q, s, 4, max_top_k=8)
        for t in tails:
            t.set_sampling([0.0], [40], [1.1])
        for trial in range(6):
            x = rng.standard_normal((1, d)).astype(np.float32)
            per = _step(tails, x, np.array([0.5], np.float32))
            sx, xq = oracle.quantize_x(x[0], "port")
            want = int(np.argmax(oracle.lm_head(xq, sx, q, s)))
            assert all(int(p[0]) == want for p in per)
        for t in tails:
            t.close()


def test_sharded_stress_k1024_duplicate_rows():
    """k = 1024 over 4 slices (the grid-histogram select inside each), 5%
    duplicated rows, a 4096-id history: tokens equal the uncapped oracle."""
    base = synth.CONFIGS["c5_stress"]
    cfg = base.with_(vocab=60000, n_embd=512, steps=5)
    W = synth.lm_head_f32(cfg)
    q, s = oracle.quantize_rows(W, "port")
    for variant in (0, 1):
        tails = _tails(cfg, variant, q, s, 4)
        hist0 = synth.history(cfg, 0)
        for t in tails:
            t.set_sampling([cfg.temperature], [cfg.top_k], [cfg.rep_penalty])
            t.set_history(0, hist0)
        port = oracle.PortLoop(q, s, hist0, cfg.hist, cfg.temperature, cfg.top_k,
                               cfg.rep_penalty, variant)
        draws = synth.Draws(cfg, 1)
        for step in range(cfg.steps):
            h = synth.hidden(cfg, step, 1)
            u = draws.u(0)
            per = _step(tails, h, np.array([u], np.float32))
            ptok, info = port.step(h[0], u)
            assert all(int(p[0]) == ptok for p in per), (variant, step)
            assert tails[0].diag(0)["n_cand"] == info.n_cand
        for t in tails:
            t.close()


def test_sharded_multi_stream():
    """B = 3 streams over 2 slices, per-stream temperature and history."""
    base = synth.CONFIGS["c3_batch"]
    cfg = base.with_(vocab=8000, n_embd=256, streams=3, steps=4)
    W = synth.lm_head_f32(cfg)
    q, s = oracle.quantize_rows(W, "port")
    temps = synth.temperatures(cfg)[:3]
    tails = _tails(cfg, 0, q, s, 2, streams=3)
    ports = []
    for t in tails:
        t.set_sampling(temps, [cfg.top_k] * 3, [cfg.rep_penalty] * 3)
    for b in range(3):
        hb = synth.history(cfg, b)
        for t in tails:
            t.set_history(b, hb)
        ports.append(oracle.PortLoop(q, s, hb, cfg.hist, float(temps[b]), cfg.top_k,
                                     cfg.rep_penalty, 0))
    draws = synth.Draws(cfg, 3)
    for step in range(cfg.steps):
        h = synth.hidden(cfg, step, 3)
        u = np.array([draws.u(b) for b in range(3)], np.float32)
        per = _step(tails, h, u)
        for b in range(3):
            want = ports[b].step(h[b], u[b])[0]
            assert all(int(p[b]) == want for p in per), (step, b)
    for t in tails:
        t.close()


def test_sharded_tie_set_larger_than_a_record():
    """A tie set larger than a record (an all-zero hidden: every logit 0)
    goes out in the record's wide form; every shard returns the unsharded
    step's token and pushes it, and the next step runs the list form."""
    spec = cases.loop_cases()["tiny_lib"]
    cfg, W, hist0 = cases.loop_inputs(spec)
    q, s = oracle.quantize_rows(W, "port")
    tails = _tails(cfg, 0, q, s, 2)
    port = oracle.PortLoop(q, s, hist0, cfg.hist, cfg.temperature, cfg.top_k,
                           cfg.rep_penalty, 0)
    for t in tails:
        t.set_sampling([cfg.temperature], [cfg.top_k], [cfg.rep_penalty])
        t.set_history(0, hist0)
    for step, h in enumerate((np.zeros((1, cfg.n_embd), np.float32), synth.hidden(cfg, 0))):
        u = np.float32(0.3 + 0.2 * step)
        per = _step(tails, h, np.array([u], np.float32))
        want, info = port.step(h[0], u)
        for r, t in enumerate(tails):
            assert int(per[r][0]) == want, (step, r)
            assert t.diag(0)["n_cand"] == info.n_cand
            np.testing.assert_array_equal(t.get_history(0), port.history())
    for t in tails:
        t.close()


# ---- real ranks over NCCL (two or more GPUs) ----------------------------------

def _nccl_worker(rank, world, port, out_dir, p2p):
    import datetime

    import torch
    import torch.distributed as dist

    from lal_b200.sharded import ShardedDecodeTail
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    spec = cases.loop_cases()["c1_gpt2"]
    cfg, W, hist0 = cases.loop_inputs(spec)
    q, s = oracle.quantize_rows(W, "port")
    st = ShardedDecodeTail(cfg.vocab, cfg.n_embd, device=rank, max_top_k=cfg.top_k,
                           history_cap=cfg.hist, sampler=spec["variant"], p2p=p2p)
    assert st.p2p == p2p
    st.load_lm_head_q8(q[st.row0:st.row0 + st.n_rows], s[st.row0:st.row0 + st.n_rows])
    st.set_sampling([cfg.temperature], [cfg.top_k], [cfg.rep_penalty])
    st.set_history(0, hist0)
    g = synth.GlibcStream(cfg.seed, private=False)
    toks = []
    for step in range(cfg.steps):
        h = synth.hidden(cfg, step)
        toks.append(int(st.step(h, np.array([g.next_u()], np.float32))[0]))
    hist = st.get_history(0)
    st.close()
    dist.destroy_process_group()
    np.save(os.path.join(out_dir, f"tok{rank}.npy"), np.array(toks, np.int32))
    np.save(os.path.join(out_dir, f"hist{rank}.npy"), hist)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.parametrize("p2p", [False, True])
def test_nccl_ranks_match_reference(golden, tmp_path, p2p):
    """Two processes, one GPU each: the all-gather path (p2p=False) and the
    single-kernel peer exchange (p2p=True) both reproduce the reference's
    golden decode loop on every rank."""
    import torch
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("one GPU: the multi-GPU paths run under a multi-GPU call")
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_nccl_worker, args=(world, _free_port(), str(tmp_path), p2p),
                       nprocs=world, join=True, start_method="spawn")
    want = golden["loop_c1_gpt2_tokens"]
    for r in range(world):
        np.testing.assert_array_equal(np.load(tmp_path / f"tok{r}.npy"), want)
    np.testing.assert_array_equal(np.load(tmp_path / "hist0.npy"),
                                  np.load(tmp_path / f"hist{world - 1}.npy"))


def _wide_worker(rank, world, port, out_dir, p2p):
    """Steps whose tie set outgrows a record (all-zero hidden vectors: every
    logit 0.0) between normal ones, on real ranks: the record's wide form
    through the peer exchange (p2p) or the NCCL all-gather."""
    import datetime

    import torch
    import torch.distributed as dist

    from lal_b200.sharded import ShardedDecodeTail
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    spec = cases.loop_cases()["c1_gpt2"]
    cfg, W, hist0 = cases.loop_inputs(spec)
    q, s = oracle.quantize_rows(W, "port")
    st = ShardedDecodeTail(cfg.vocab, cfg.n_embd, device=rank, max_top_k=cfg.top_k,
                           history_cap=cfg.hist, sampler=0, p2p=p2p)
    st.load_lm_head_q8(q[st.row0:st.row0 + st.n_rows], s[st.row0:st.row0 + st.n_rows])
    st.set_sampling([cfg.temperature], [cfg.top_k], [cfg.rep_penalty])
    st.set_history(0, hist0)
    port = oracle.PortLoop(q, s, hist0, cfg.hist, cfg.temperature, cfg.top_k,
                           cfg.rep_penalty, 0)
    got, want = [], []
    for step in range(6):
        h = (np.zeros((1, cfg.n_embd), np.float32) if step % 2 == 0
             else synth.hidden(cfg, step))
        u = np.float32(0.15 + 0.13 * step)
        got.append(int(st.step(h, np.array([u], np.float32))[0]))
        want.append(port.step(h[0], u)[0])
    hist = st.get_history(0)
    st.close()
    dist.destroy_process_group()
    np.save(os.path.join(out_dir, f"w{rank}.npy"), np.array([got, want], np.int32))
    np.save(os.path.join(out_dir, f"wh{rank}.npy"), np.stack([hist, port.history()]))


@pytest.mark.parametrize("p2p", [False, True])
def test_ranks_exchange_wide_records(tmp_path, p2p):
    """Two processes, one GPU each: all-zero hidden vectors (every logit tied
    at 0.0) between normal steps return the oracle's tokens on both ranks."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("one GPU: the multi-GPU paths run under a multi-GPU call")
    import torch.multiprocessing as mp
    mp.start_processes(_wide_worker, args=(2, _free_port(), str(tmp_path), p2p), nprocs=2,
                       join=True, start_method="spawn")
    for r in range(2):
        got, want = np.load(tmp_path / f"w{r}.npy")
        np.testing.assert_array_equal(got, want)
        h = np.load(tmp_path / f"wh{r}.npy")
        np.testing.assert_array_equal(h[0], h[1])


def _p2p_timeout_worker(rank, world, port, out_dir):
    import datetime

    import torch
    import torch.distributed as dist

    from lal_b200.sharded import ShardedDecodeTail
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    spec = cases.loop_cases()["tiny_lib"]
    cfg, W, hist0 = cases.loop_inputs(spec)
    q, s = oracle.quantize_rows(W, "port")
    st = ShardedDecodeTail(cfg.vocab, cfg.n_embd, device=rank, max_top_k=cfg.top_k,
                           history_cap=cfg.hist, sampler=0, p2p=True)
    st.load_lm_head_q8(q[st.row0:st.row0 + st.n_rows], s[st.row0:st.row0 + st.n_rows])
    st.set_sampling([cfg.temperature], [cfg.top_k], [cfg.rep_penalty])
    st.set_history(0, hist0)
    h = synth.hidden(cfg, 0)
    u = np.array([0.25], np.float32)
    code = 0
    if rank == 0:
        # rank 1 never steps: the bounded peer wait runs out (2 s)
        try:
            st.step(h, u)
        except L.LalTailError as e:
            code = e.code
    dist.barrier()
    # both ranks reconnect (fresh sequence numbers) and step together
    handles = [None] * world
    dist.all_gather_object(handles, st.tail.exchange_handle())
    st.tail.connect_peers(handles)
    dist.barrier()
    tok = int(st.step(h, u)[0])
    hist = st.get_history(0)
    st.close()
    dist.destroy_process_group()
    np.save(os.path.join(out_dir, f"r{rank}.npy"), np.array([code, tok, hist.size], np.int64))


def test_p2p_wait_times_out_then_recovers(tmp_path):
    """A rank that does not step: the other rank's bounded wait ends with
    LAL_TAIL_ERR_TIMEOUT (no token pushed); after reconnecting, both ranks
    step together and agree."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("one GPU: the peer exchange runs under a multi-GPU call")
    import torch.multiprocessing as mp
    mp.start_processes(_p2p_timeout_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2,
                       join=True, start_method="spawn")
    r0 = np.load(tmp_path / "r0.npy")
    r1 = np.load(tmp_path / "r1.npy")
    assert r0[0] == 4          # LAL_TAIL_ERR_TIMEOUT on the rank that stepped alone
    assert r0[1] == r1[1]      # then the same token on both ranks
    spec = cases.loop_cases()["tiny_lib"]
    assert r0[2] == r1[2] == min(spec["hist"], cases.loop_inputs(spec)[2].size + 1)
