"""CPU stand-ins for the qmr.ops kernels, built on the FP64 oracle.

Test infrastructure only: they let the sharded host logic of qmr.parallel
run on gloo ranks without a GPU.  Same call signatures as qmr.ops."""
import dataclasses

import numpy as np
import torch

import oracle


@dataclasses.dataclass
class CpuMatrix:
    weight: np.ndarray
    scales: np.ndarray
    biases: np.ndarray
    rows: int
    cols: int
    bits: int
    group: int

    def shard(self, r0, r1):
        return CpuMatrix(self.weight[r0:r1], self.scales[r0:r1], self.biases[r0:r1], r1 - r0, self.cols, self.bits,
                         self.group)


def _mm(m, x, batch):
    want, _ = oracle.matmul_f64(m.weight, m.scales, m.biases, x.numpy().reshape(batch, m.cols), m.rows, m.cols,
                                m.bits, m.group, batch=batch)
    return want  # float64 [batch, rows]


def total_order_key(v):
    u = np.asarray(v, np.float32).view(np.uint32).astype(np.uint64)
    return np.where(u & 0x80000000, u ^ 0xFFFFFFFF, u | 0x80000000)


class CpuOps:
    @staticmethod
    def matmul_affine(m, x, y, batch):
        y.copy_(torch.from_numpy(_mm(m, x, batch).astype(np.float32).ravel()))

    @staticmethod
    def gateup_swiglu(g, u, x, act, batch):
        gg, uu = _mm(g, x, batch), _mm(u, x, batch)
        act.copy_(torch.from_numpy((gg / (1.0 + np.exp(-gg)) * uu).astype(np.float32).ravel()))

    @staticmethod
    def head_argmax(m, x, logits, idx, batch, best_key=None, row_base=0):
        lg = _mm(m, x, batch).astype(np.float32)
        logits.copy_(torch.from_numpy(lg.ravel()))
        keys = (total_order_key(lg) << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - (np.uint64(row_base) +
                                                                                  np.arange(m.rows, dtype=np.uint64)))
        best = keys.max(axis=1)
        idx.copy_(torch.from_numpy((0xFFFFFFFF - (best & 0xFFFFFFFF)).astype(np.int32)))
        if best_key is not None:
            best_key.copy_(torch.from_numpy(best.view(np.int64)))
