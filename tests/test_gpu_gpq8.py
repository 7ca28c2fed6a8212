"""Loading the LM head from a GPQ8 blob (lal_tail_load_lm_head_gpq8): an F32
lm_head.weight is quantized on the GPU exactly as the server's
lal_quantize_q8_per_row does at load (checked against the reference's own
compiled quantizer where it was built, else the restatement); a Q8 tensor is
taken as it is; sharded contexts each load their own rows."""
import numpy as np
import pytest

import lal_b200 as L
import oracle
from gpq8_blob import gpq8_blob

pytestmark = pytest.mark.gpu


def _model(V, d, seed=1):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((V, d)) * 0.02).astype(np.float32)
    W[rng.integers(0, V, 50), rng.integers(0, d, 50)] *= 20.0
    emb = rng.standard_normal((11, d)).astype(np.float32)
    return W, emb


def test_f32_lm_head_is_quantized_like_the_server():
    V, d = 5003, 200
    W, emb = _model(V, d)
    blob = gpq8_blob([("model.embed_tokens.weight", emb, None), ("lm_head.weight", W, None)])
    t = L.DecodeTail(V, d, max_streams=1, max_top_k=40, history_cap=16)
    t.load_lm_head_gpq8(blob)
    q, s = t.read_lm_head()
    which = "ref" if oracle.have_ref() else "port"
    qo, so = oracle.quantize_rows(W, which)
    np.testing.assert_array_equal(q, qo)
    np.testing.assert_array_equal(s.view(np.int32), so.view(np.int32))
    t.close()


def test_q8_lm_head_and_sharded_slices():
    V, d = 4099, 256
    W, emb = _model(V, d, 2)
    qo, so = oracle.quantize_rows(W, "port")
    blob = gpq8_blob([("lm_head.weight", qo, so), ("model.embed_tokens.weight", emb, None)])
    parts_q, parts_s = [], []
    for r in range(3):
        t = L.DecodeTail(V, d, max_streams=1, max_top_k=40, history_cap=16, shard_rank=r,
                         shard_count=3)
        t.load_lm_head_gpq8(blob)
        q, s = t.read_lm_head()
        parts_q.append(q)
        parts_s.append(s)
        t.close()
    np.testing.assert_array_equal(np.concatenate(parts_q), qo)
    np.testing.assert_array_equal(np.concatenate(parts_s).view(np.int32), so.view(np.int32))


def test_wrong_shape_is_rejected():
    V, d = 1000, 128
    W, emb = _model(V + 1, d, 3)
    blob = gpq8_blob([("lm_head.weight", W, None)])
    t = L.DecodeTail(V, d, max_streams=1, max_top_k=40, history_cap=16)
    with pytest.raises(L.LalTailError) as ei:
        t.load_lm_head_gpq8(blob)
    assert ei.value.code == 1
    t.close()
