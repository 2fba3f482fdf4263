"""The decode engine on the GPU against the reference's golden logits and the
FP64 decode-graph oracle.

* The reference's tiny hybrid checkpoints (three DeltaNet layers, one gated
  attention layer; packed Q4/g32 with BF16 or F16 metadata) load through the
  C++ loader and reproduce the golden logits of the reference's scalar oracle
  (scripts/make_fixture.py) within the reference's own test tolerance
  (tests/bf16_inference.rs: 2e-3 + 2e-3|want|) and a tighter FP32 bound,
  across resets (tests/inference.rs:97-137); out-of-vocabulary tokens and a
  full context are rejected before any launch.
* A synthetic model with the same layer graph at widths the tensor-core
  kernel takes (so the fused RMSNorm / residual epilogues, the fused mixers
  and the graph replays all run) matches the FP64 oracle's logits and
  produces identical greedy token ids.
"""
import numpy as np
import pytest

import oracle
import qmr
from qmr import engine as qeng
from qmr._lib import QmrError
from _model_util import GOLDEN, golden, tiny_oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fixture", ["tiny-bf16", "tiny-q4"])
def test_tiny_checkpoints_match_reference_golden_logits(cuda, fixture):
    path = GOLDEN / fixture
    tokens, want = golden(path)
    eng = qmr.Engine.load(path, 8)
    try:
        for repetition in range(2):
            eng.reset()
            for i, tok in enumerate(tokens):
                got, nxt = eng.forward(tok)
                assert np.all(np.isfinite(got))
                # The reference's own tolerance for these fixtures ...
                assert np.all(np.abs(got - want[i]) < 2e-3 + 2e-3 * np.abs(want[i])), (fixture, repetition, i)
                # ... and the FP32 pipeline's: far inside it.
                assert np.max(np.abs(got - want[i])) < 1e-4, (fixture, i, np.max(np.abs(got - want[i])))
                assert nxt == oracle.argmax_f32(got)
                assert eng.position == i + 1
    finally:
        eng.close()


def test_tiny_engine_rejects_vocabulary_and_context_overflow(cuda):
    eng = qmr.Engine.load(GOLDEN / "tiny-bf16", 8)
    try:
        with pytest.raises(QmrError):
            eng.forward(64)
        for _ in range(8):
            eng.forward(3, logits=False)
        with pytest.raises(QmrError):
            eng.forward(3)
        assert eng.position == 8
        eng.reset()
        assert eng.position == 0
        with pytest.raises(QmrError):
            eng.generate([3, 4, 5], 7)  # 3 + 7 - 1 > 8
    finally:
        eng.close()


def test_metadata_compaction_stats_follow_the_metadata_mode(cuda):
    """Engine::metadata_stats (tests/bf16_inference.rs:11-16): 33 matrices and
    3288 * 2 bytes saved for tiny-bf16 in bf16 mode, none in f32 mode."""
    try:
        qmr.lib().qmr_set_modes(None, b"bf16", None, None)
        eng = qmr.Engine.load(GOLDEN / "tiny-bf16", 8)
        assert eng.metadata_stats() == (33, 3288 * 2)
        tokens, want = golden(GOLDEN / "tiny-bf16")
        got, _ = eng.forward(tokens[0])
        assert np.max(np.abs(got - want[0])) < 1e-4
        eng.close()
        qmr.lib().qmr_set_modes(None, b"f32", None, None)
        eng = qmr.Engine.load(GOLDEN / "tiny-bf16", 8)
        assert eng.metadata_stats() == (0, 0)
        assert eng.mlp_r2_eligible_matrices() == 0  # not the 17408x5120 MLP shapes
        eng.close()
    finally:
        qmr.lib().qmr_set_modes(None, b"f32", None, None)


def test_generate_equals_step_by_step_forward(cuda):
    path = GOLDEN / "tiny-q4"
    eng = qmr.Engine.load(path, 16)
    try:
        prompt = [3, 8, 4]
        toks, pre_ms, dec_ms = eng.generate(prompt, 6)
        assert eng.position == len(prompt) + 6 - 1
        assert pre_ms > 0 and dec_ms > 0
        eng.reset()
        ref = []
        nxt = None
        for t in prompt:
            _, nxt = eng.forward(t)
        ref.append(nxt)
        for _ in range(5):
            _, nxt = eng.forward(nxt)
            ref.append(nxt)
        assert toks == ref
        # and the FP64 oracle's greedy continuation
        o, _ = tiny_oracle(path, context=16)
        seq = []
        for t in prompt:
            lg = o.forward(t)
        seq.append(oracle.argmax_f64(lg))
        for _ in range(5):
            lg = o.forward(seq[-1])
            seq.append(oracle.argmax_f64(lg))
        assert toks == seq
    finally:
        eng.close()


def small_config():
    """The layer graph at small widths the tensor-core kernel takes (hidden and
    every matrix width a multiple of 512 columns)."""
    return dict(hidden=1024, inter=2048, layers=4, heads=4, kv_heads=2, head_dim=128, vocab=4096, lin_key_heads=2,
                lin_value_heads=4, lin_key_dim=128, lin_value_dim=128, conv_width=4, rotary_dim=32, eps=1e-6,
                theta=1e7, is_attn=[False, False, False, True])


def synthetic_oracle(cfg, seed, context):
    o = oracle.DecodeOracle(dict(cfg, context=context))
    H, F = cfg["hidden"], cfg["inter"]
    KD, VD = cfg["lin_key_heads"] * cfg["lin_key_dim"], cfg["lin_value_heads"] * cfg["lin_value_dim"]
    QD, KVD = cfg["heads"] * cfg["head_dim"], cfg["kv_heads"] * cfg["head_dim"]
    o.set_synth(-1, "embed", seed, qeng.MID_EMBED, cfg["vocab"], H)
    o.set_synth(-1, "head", seed, qeng.MID_HEAD, cfg["vocab"], H)
    keep = [np.ones(H, np.float32), np.ones(cfg["lin_value_dim"], np.float32), np.ones(cfg["head_dim"], np.float32),
            np.full((2 * KD + VD) * cfg["conv_width"], 0.1, np.float32), np.zeros(cfg["lin_value_heads"], np.float32)]
    o.set_vector(-1, None, keep[0])
    for l, att in enumerate(cfg["is_attn"]):
        mid = lambda s: qeng.synthetic_mid(l, s)  # noqa: E731
        o.set_vector(l, "input_norm", keep[0])
        o.set_vector(l, "post_norm", keep[0])
        o.set_synth(l, "gate", seed, mid("gate"), F, H)
        o.set_synth(l, "up", seed, mid("up"), F, H)
        o.set_synth(l, "down", seed, mid("down"), H, F)
        if att:
            o.set_synth(l, "q", seed, mid("q"), 2 * QD, H)
            o.set_synth(l, "k", seed, mid("k"), KVD, H)
            o.set_synth(l, "v", seed, mid("v"), KVD, H)
            o.set_synth(l, "o", seed, mid("o"), H, QD)
            o.set_vector(l, "q_norm", keep[2])
            o.set_vector(l, "k_norm", keep[2])
        else:
            o.set_synth(l, "qkv", seed, mid("qkv"), 2 * KD + VD, H)
            o.set_synth(l, "z", seed, mid("z"), VD, H)
            o.set_synth(l, "a", seed, mid("a"), cfg["lin_value_heads"], H)
            o.set_synth(l, "b", seed, mid("b"), cfg["lin_value_heads"], H)
            o.set_synth(l, "out", seed, mid("out"), H, VD)
            o.set_vector(l, "conv", keep[3])
            o.set_vector(l, "A_log", keep[4])
            o.set_vector(l, "dt_bias", keep[4])
            o.set_vector(l, "delta_norm", keep[1])
    o._keep += keep
    return o


def prompt_tokens(seed, n, vocab):
    from qmr import synth
    return [int(v % vocab) for v in synth.splitmix64(seed, n)]


def test_synthetic_engine_matches_fp64_oracle_logits_and_greedy_ids(cuda):
    cfg, seed, context = small_config(), 11, 96
    eng = qmr.Engine.synthetic(cfg, seed, context)
    o = synthetic_oracle(cfg, seed, context)
    try:
        with_head, without = eng.step_launches()
        # embed + per layer (fused in-proj, mixer, out + residual, gate/up, down + residual) + head + advance
        assert with_head == 1 + 9 * cfg["layers"] + 2 + 1 and without == with_head - 2
        prompt = prompt_tokens(5, 40, cfg["vocab"])
        worst = 0.0
        for i, t in enumerate(prompt):
            got, nxt = eng.forward(t)
            want = o.forward(t)
            scale = np.max(np.abs(want))
            err = np.max(np.abs(got - want))
            worst = max(worst, err / scale)
            # FP32 activations through 4 layers of 1024-2048 wide products.
            assert err <= 1e-4 * scale, (i, err, scale)
            wi = oracle.argmax_f64(want)
            top2 = np.sort(want)[-2:]
            if top2[1] - top2[0] > 2e-4 * scale:
                assert nxt == wi, (i, nxt, wi)
        # Greedy continuation on the device equals the oracle's.
        toks, _, _ = eng.generate([prompt[-1]], 16)
        seq, cur = [], prompt[-1]
        for _ in range(16):
            cur = oracle.argmax_f64(o.forward(cur))
            seq.append(cur)
        assert toks == seq
        assert qmr.ops.device_error() == 0
    finally:
        eng.close()
