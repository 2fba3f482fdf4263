"""MTP-style block verification on the GPU (the reference's
src/engine/block.rs verify_block / commit_block_prefix, restated from its
tests/block_inference.rs), and the device-resident greedy verification loop.

* Blocks of width 1..4 over the golden tokens give the same logits as
  sequential steps (and the reference's golden logits) for every row.
* Every rollback prefix (keep = 0..width) continues exactly like a fresh
  causal run of the kept tokens; a second transaction does not retain the
  first one's snapshots; a pending block forbids other steps; invalid blocks
  fail without changing state.
* Greedy rounds with drafts equal to the greedy continuation accept every
  draft; with wrong drafts none; both emit the plain greedy tokens.
"""
import numpy as np
import pytest

import qmr
from qmr._lib import QmrError
from _model_util import GOLDEN, golden

pytestmark = pytest.mark.gpu


def near(a, b, what, tol=1e-4):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    assert a.shape == b.shape, what
    err = np.max(np.abs(a - b)) if a.size else 0.0
    assert err <= tol, (what, err)


@pytest.mark.parametrize("fixture", ["tiny-bf16", "tiny-q4"])
def test_block_widths_match_sequential_and_golden_logits(cuda, fixture):
    path = GOLDEN / fixture
    tokens, want = golden(path)
    seq = qmr.Engine.load(path, 32)
    blk = qmr.Engine.load(path, 32)
    try:
        for width in range(1, 5):
            seq.reset()
            blk.reset()
            for ci in range(0, len(tokens), width):
                chunk = tokens[ci:ci + width]
                lg, am = blk.verify_block(chunk)
                assert blk.position == ci + len(chunk)
                for i, tok in enumerate(chunk):
                    s_lg, s_next = seq.forward(tok)
                    near(lg[i], want[ci + i], f"golden w{width} {ci + i}")
                    # the same kernels and summation order as single steps
                    assert np.array_equal(lg[i].view(np.uint32), s_lg.view(np.uint32)), (width, ci + i)
                    assert am[i] == s_next
                blk.commit_block_prefix(len(chunk))
    finally:
        seq.close()
        blk.close()


def test_every_rollback_prefix_matches_fresh_causal_continuation(cuda):
    path = GOLDEN / "tiny-q4"
    ref = qmr.Engine.load(path, 64)
    blk = qmr.Engine.load(path, 64)
    try:
        for width in range(1, 5):
            for keep in range(width + 1):
                ref.reset()
                blk.reset()
                for t in (5, 9, 13):
                    ref.forward(t)
                    blk.forward(t)
                cands = [7, 21, 4, 30][:width]
                blk.verify_block(cands)
                with pytest.raises(QmrError):
                    blk.forward(2)  # pending block forbids a normal forward
                with pytest.raises(QmrError):
                    blk.verify_block([2])
                with pytest.raises(QmrError):
                    blk.commit_block_prefix(width + 1)
                assert blk.position == 3 + width
                blk.commit_block_prefix(keep)
                assert blk.position == 3 + keep
                with pytest.raises(QmrError):
                    blk.commit_block_prefix(0)  # commit consumes the transaction
                for t in cands[:keep]:
                    ref.forward(t)
                for t in (31, 11, 19):
                    near(blk.forward(t)[0], ref.forward(t)[0], f"rollback w{width} keep{keep}", tol=0)
                blk.verify_block([8, 17, 22])
                blk.commit_block_prefix(1)
                ref.forward(8)
                near(blk.forward(14)[0], ref.forward(14)[0], "second rollback", tol=0)
    finally:
        ref.close()
        blk.close()


def test_invalid_blocks_fail_without_changing_state(cuda):
    path = GOLDEN / "tiny-q4"
    eng = qmr.Engine.load(path, 8)
    ref = qmr.Engine.load(path, 8)
    try:
        eng.forward(5)
        ref.forward(5)
        for bad in ([], [1, 2, 3, 4, 5], [6, 64], [2**32 - 1]):
            with pytest.raises((QmrError, OverflowError, ValueError)):
                eng.verify_block(bad)
            assert eng.position == 1
        with pytest.raises(QmrError):
            eng.commit_block_prefix(1)  # nothing pending
        for t in (6, 7, 8, 9, 10):
            eng.forward(t)
        with pytest.raises(QmrError):
            eng.verify_block([2, 3, 4])  # 6 + 3 > 8
        assert eng.position == 6
        for t in (6, 7, 8, 9, 10):
            ref.forward(t)
        near(eng.forward(11)[0], ref.forward(11)[0], "after rejected blocks", tol=0)
    finally:
        eng.close()
        ref.close()


@pytest.mark.parametrize("block", [2, 3, 4])
def test_greedy_verification_rounds_emit_the_plain_greedy_tokens(cuda, block):
    from test_engine_gpu import small_config
    cfg = small_config()
    eng = qmr.Engine.synthetic(cfg, 13, 128)
    try:
        prompt = [17, 3001, 42, 977, 5]
        plain, _, _ = eng.generate(prompt, 24)
        eng.reset()
        table = [0] * 128
        for k, t in enumerate(plain):
            table[len(prompt) + k] = t
        toks, rounds, acc, _, _ = eng.mtp_generate(prompt, 24, block, table)
        assert toks == plain
        assert acc == rounds * (block - 1)  # every draft accepted
        assert rounds == -(-(24 - 1) // block)
        eng.reset()
        wrong = [(t + 1) % cfg["vocab"] for t in table]
        toks, rounds, acc, _, _ = eng.mtp_generate(prompt, 24, block, wrong)
        assert toks == plain
        assert acc == 0 and rounds == 23
        assert qmr.ops.device_error() == 0
    finally:
        eng.close()
