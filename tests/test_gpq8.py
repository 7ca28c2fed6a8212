"""GPQ8 tensor directory (lal_tail_gpq8_find): host-only parsing of the
Qwen-7B server's weight format, including malformed blobs (no GPU needed)."""
import numpy as np
import pytest

import lal_b200 as L
from gpq8_blob import gpq8_blob


def _blob():
    rng = np.random.default_rng(0)
    emb = rng.standard_normal((5, 8)).astype(np.float32)
    head = rng.standard_normal((7, 8)).astype(np.float32)
    q = rng.integers(-127, 128, size=(3, 8)).astype(np.int8)
    s = rng.random(3).astype(np.float32)
    return gpq8_blob([("model.embed_tokens.weight", emb, None), ("lm_head.weight", head, None),
                      ("layer.q8", q, s)]), emb, head, q, s


def test_find_tensors():
    blob, emb, head, q, s = _blob()
    e = L.gpq8_find(blob, "lm_head.weight")
    assert e["ndim"] == 2 and e["shape"] == [7, 8] and e["qtype"] == 0 and e["n_scale"] == 0
    got = np.frombuffer(blob, np.float32, count=56, offset=e["data_offset"]).reshape(7, 8)
    np.testing.assert_array_equal(got, head)
    e = L.gpq8_find(blob, "layer.q8")
    assert e["qtype"] == 1 and e["n_scale"] == 3 and e["data_len"] == 24
    np.testing.assert_array_equal(
        np.frombuffer(blob, np.int8, count=24, offset=e["data_offset"]).reshape(3, 8), q)
    np.testing.assert_array_equal(np.frombuffer(blob, np.float32, count=3,
                                                offset=e["scale_offset"]), s)


@pytest.mark.parametrize("mutate", ["magic", "truncate", "missing", "ndim", "klen"])
def test_malformed_blobs_are_rejected(mutate):
    blob, *_ = _blob()
    key = "lm_head.weight"
    if mutate == "magic":
        blob = b"GPQ9" + blob[4:]
    elif mutate == "truncate":
        blob = blob[:len(blob) // 2]
    elif mutate == "missing":
        key = "no.such.tensor"
    elif mutate == "ndim":
        # the first tensor's ndim (after magic, count, key length, key) set to 9
        at = 4 + 4 + 4 + len("model.embed_tokens.weight")
        blob = blob[:at] + (9).to_bytes(4, "little") + blob[at + 4:]
    elif mutate == "klen":
        blob = blob[:8] + (100000).to_bytes(4, "little") + blob[12:]
    with pytest.raises(L.LalTailError) as ei:
        L.gpq8_find(blob, key)
    assert ei.value.code == 1
