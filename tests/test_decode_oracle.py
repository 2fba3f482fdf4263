"""The FP64 decode-graph oracle (oracle/decode.c) pinned to the reference's
own scalar oracle: the golden logits that rucin93/qwen-mlx-runner's
scripts/make_fixture.py computes for its tiny hybrid models (three DeltaNet
layers and one attention layer, packed Q4/g32 with BF16 or F16 metadata).
Also the synthetic generator's determinism and distributions."""
import numpy as np
import pytest

import oracle
from _model_util import GOLDEN, golden, tiny_oracle


@pytest.mark.parametrize("fixture", ["tiny-bf16", "tiny-q4"])
def test_decode_oracle_reproduces_reference_golden_logits(fixture):
    path = GOLDEN / fixture
    o, cfg = tiny_oracle(path, context=8)
    tokens, want = golden(path)
    for repetition in range(2):
        o.reset()
        for i, tok in enumerate(tokens):
            got = o.forward(tok)
            assert o.position == i + 1
            # Same FP64 math in a different order than the Python scalar oracle.
            np.testing.assert_allclose(got, want[i], rtol=0, atol=1e-12, err_msg=f"{fixture} rep {repetition} token {i}")


def test_decode_oracle_rejects_vocabulary_and_context_overflow():
    o, cfg = tiny_oracle(GOLDEN / "tiny-bf16", context=3)
    with pytest.raises(ValueError):
        o.forward(cfg["vocab"])
    for _ in range(3):
        o.forward(3)
    with pytest.raises(ValueError):
        o.forward(3)
    assert o.position == 3


def test_synthetic_generator_is_deterministic_and_has_the_benchmark_distribution():
    a = oracle.synth_matrix(7, 123, 64, 512)
    b = oracle.synth_matrix(7, 123, 64, 512)
    c = oracle.synth_matrix(7, 124, 64, 512)
    for k in ("weight", "scales", "biases"):
        assert np.array_equal(a[k], b[k])
    assert not np.array_equal(a["weight"], c["weight"])
    nib = ((a["weight"][..., None] >> (4 * np.arange(8, dtype=np.uint32))) & 15).ravel()
    assert abs(nib.mean() - 7.5) < 0.1
    s = (a["scales"].astype(np.uint32) << 16).view(np.float32)
    bias = (a["biases"].astype(np.uint32) << 16).view(np.float32)
    assert s.min() >= 0.0019 and s.max() <= 0.0201
    noise = bias + 8 * s
    assert abs(noise.mean()) < 2e-4 and 0.7e-3 < noise.std() < 1.3e-3
