"""CPU oracle pieces of the decoder: embedding (embedding.rs KATs), the greedy
pick (model.rs:325-337: f32::total_cmp maximum, the last among equals) and
the bf16 rounding helper the composition uses."""
import numpy as np
import pytest

import oracle as orc


def test_embedding_kats(kats):
    for c in kats["embedding"]:
        out = orc.embedding(c["table"], c["ids"], c["vocab"], c["hidden"])
        assert np.allclose(out.reshape(-1), np.float32(c["out"])), c["name"]


def test_embedding_error_kats(kats):
    for c in kats["embedding_errors"]:
        if c["error"] == "LengthMismatch" and c["argument"] == "output":
            continue  # the host restatement allocates its output
        with pytest.raises(ValueError, match=c["error"]):
            orc.embedding(np.zeros(c["table_len"]), c["ids"], c["vocab"], c["hidden"])


def test_argmax_total_order_and_ties():
    assert orc.argmax_total([1.0, 3.0, 3.0, -1.0]) == 2          # last of equal maxima
    assert orc.argmax_total([-0.0, 0.0]) == 1                    # +0 > -0 under total_cmp
    assert orc.argmax_total([0.0, -0.0]) == 0
    assert orc.argmax_total([np.inf, np.nan]) == 1               # +NaN is the greatest
    assert orc.argmax_total([-np.nan, -np.inf]) == 1             # -NaN is the least
    assert orc.argmax_total(np.float32([-5, -2, -3])) == 1


def test_bf16_rounding_matches_torch():
    import torch

    x = np.random.default_rng(0).standard_normal(10000).astype(np.float32) * 100
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(orc._bf16(x), ref)
