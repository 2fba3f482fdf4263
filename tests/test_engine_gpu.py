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


@pytest.mark.parametrize("model", ["tiny-q4", "small"])
def test_prefill_blocks_equal_single_steps(cuda, model):
    """generate() runs a long prompt's positions in blocks of 3 through the
    batched path; the greedy tokens and the recurrent state after them (the
    next step's logits, bit for bit) equal those of one forward per token."""
    if model == "tiny-q4":
        make = lambda: qmr.Engine.load(GOLDEN / "tiny-q4", 32)  # noqa: E731
        vocab = 64
    else:
        make = lambda: qmr.Engine.synthetic(small_config(), 17, 64)  # noqa: E731
        vocab = small_config()["vocab"]
    prompt = prompt_tokens(23, 11, vocab)  # 10 positions before the last: 3 blocks and 1 single step
    eng = make()
    try:
        toks, _, _ = eng.generate(prompt, 4)
        assert eng.position == len(prompt) + 4 - 1
        lg_blocks, _ = eng.forward(toks[-1])
        eng.reset()
        ref = []
        for t in prompt:
            _, nxt = eng.forward(t)
        ref.append(nxt)
        for _ in range(3):
            _, nxt = eng.forward(nxt)
            ref.append(nxt)
        assert toks == ref
        lg_steps, _ = eng.forward(ref[-1])
        assert np.array_equal(lg_blocks.view(np.uint32), lg_steps.view(np.uint32))
        assert qmr.ops.device_error() == 0
    finally:
        eng.close()


def small_config():
    """The layer graph at small widths the tensor-core kernel takes (hidden and
    every matrix width a multiple of 512 columns)."""
    return dict(hidden=1024, inter=2048, layers=4, heads=4, kv_heads=2, head_dim=128, vocab=4096, lin_key_heads=2,
                lin_value_heads=4, lin_key_dim=128, lin_value_dim=128, conv_width=4, rotary_dim=32, eps=1e-6,
                theta=1e7, is_attn=[False, False, False, True])


def synthetic_oracle(cfg, seed, context):
    return oracle.synthetic_decode_oracle(cfg, seed, context, qeng.synthetic_mid, qeng.MID_EMBED, qeng.MID_HEAD)


def prompt_tokens(seed, n, vocab):
    from qmr import synth
    return [int(v % vocab) for v in synth.splitmix64(seed, n)]


def test_synthetic_engine_matches_fp64_oracle_logits_and_greedy_ids(cuda):
    cfg, seed, context = small_config(), 11, 96
    eng = qmr.Engine.synthetic(cfg, seed, context)
    o = synthetic_oracle(cfg, seed, context)
    try:
        with_head, without = eng.step_launches()
        # embed + per layer (in-proj, mixer, out + residual, gate/up, down + residual) + head
        # + advance: every matrix one streaming kernel that builds its own activation image
        assert with_head == 1 + 5 * cfg["layers"] + 1 + 1 and without == with_head - 1
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


def test_qwen27b_shaped_synthetic_model_gives_the_oracle_greedy_ids(cuda):
    """Config 4's model (64 layers, 3:1 DeltaNet : attention, hidden 5120, MLP
    17408, vocabulary 152064, distinct seeded Q4/g64 weights per matrix) on a
    short window: the last prompt token's logits against the FP64 oracle, and
    the greedy continuation identical to the oracle's."""
    import os
    cfg = qeng.qwen27b_config()
    seed, context = 2026, 64
    oracle.set_threads(len(os.sched_getaffinity(0)))
    eng = qmr.Engine.synthetic(cfg, seed, context)
    o = synthetic_oracle(cfg, seed, context)
    try:
        assert eng.mlp_r2_eligible_matrices() == (192 if "gemv=aligned" in modes() else 0)
        prompt = prompt_tokens(7, 3, cfg["vocab"])
        toks, _, _ = eng.generate(prompt, 3)
        seq = []
        for i, t in enumerate(prompt):
            want = o.forward(t)
        seq.append(oracle.argmax_f64(want))
        eng.reset()
        for t in prompt:
            got, nxt = eng.forward(t)
        scale = np.max(np.abs(want))
        err = np.max(np.abs(got - want))
        assert err <= 1e-3 * scale, (err, scale)
        assert nxt == seq[0]
        for _ in range(2):
            seq.append(oracle.argmax_f64(o.forward(seq[-1])))
        assert toks == seq, (toks, seq)
        assert qmr.ops.device_error() == 0
    finally:
        eng.close()


def modes():
    import ctypes
    buf = ctypes.create_string_buffer(256)
    qmr.lib().qmr_get_modes(buf, 256)
    return buf.value.decode()
