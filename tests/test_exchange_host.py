"""Argument checks of the sharded exchange entry points (include/qmr.h),
on the CPU: every malformed exchange is rejected with a clear error before
anything touches a device."""
import ctypes

import pytest

from qmr import _lib

ALIGNED = 1 << 20  # a 16-byte aligned address that is never dereferenced: the checks fail first


def _exchange(world=2, rank=0, total=64, base=0, head=False, fill=True):
    ex = _lib.QmrExchange()
    ex.world, ex.rank, ex.total_rows, ex.row_base = world, rank, total, base
    if fill:
        for r in range(min(world, _lib.QMR_MAX_RANKS)):
            ex.flags[r] = ALIGNED
            if head:
                ex.keys[r] = ALIGNED
            else:
                ex.out[r] = ALIGNED
        ex.epoch = ALIGNED
    return ex


def _rc(ex, rows=32, cols=512, batch=3):
    L = _lib.lib()
    return L.qmr_matmul_affine_exchange(ALIGNED, ALIGNED, ALIGNED, ALIGNED, rows, cols, 4, 64, batch, 1,
                                        ctypes.byref(ex), None)


@pytest.mark.parametrize("kw", [dict(world=1), dict(world=9), dict(rank=2), dict(fill=False)])
def test_malformed_exchanges_are_rejected(kw):
    assert _rc(_exchange(**kw)) == _lib.QMR_EINVAL


def test_shard_past_the_full_output_is_rejected():
    assert _rc(_exchange(total=64, base=48), rows=32) == _lib.QMR_ERANGE


def test_wait_needs_an_exchange_and_a_valid_batch():
    L = _lib.lib()
    assert L.qmr_exchange_wait(None, 3, None, None, None) == _lib.QMR_EINVAL
    assert L.qmr_exchange_wait(ctypes.byref(_exchange()), 5, None, None, None) == _lib.QMR_EINVAL


def test_head_exchange_needs_key_arrays():
    L = _lib.lib()
    ex = _exchange(head=False)  # outputs but no key arrays
    rc = L.qmr_head_argmax_exchange(ALIGNED, ALIGNED, ALIGNED, ALIGNED, ALIGNED, 32, 512, 4, 64, 3, 1,
                                    ctypes.byref(ex), None)
    assert rc == _lib.QMR_EINVAL
