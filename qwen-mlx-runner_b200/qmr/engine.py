"""Python mirror of the decode engine and the checkpoint loader (include/qmr.h,
"checkpoints and the decode engine").

Names follow the reference's own types (rucin93/qwen-mlx-runner v0.7.3):
`Checkpoint` (src/weights.rs), `Engine` with load / synthetic_qwen27b /
forward / reset / mlp_r2_eligible_matrices / metadata_stats
(src/engine.rs, src/engine/synthetic.rs).  Everything runs in libqmr: the
C++ loader, the C++ engine and its CUDA kernels; these classes pass pointers
and convert results.
"""
from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence

import numpy as np

from . import _lib
from ._lib import QmrModelConfig, check

# Matrix slots of the synthetic generator's matrix ids (layer * 16 + slot + 1;
# embedding 0x100000, head 0x100001), shared with the test oracle.
SLOTS = {"qkv": 0, "z": 1, "a": 2, "b": 3, "out": 4, "q": 5, "k": 6, "v": 7, "o": 8, "gate": 9, "up": 10,
         "down": 11}
MID_EMBED, MID_HEAD = 0x100000, 0x100001


def synthetic_mid(layer: int, slot: str) -> int:
    return layer * 16 + SLOTS[slot] + 1


def qwen27b_config(layers: int = 64, vocab: int = 152064) -> dict:
    """The 27B-shaped hybrid of the synthetic benchmark (src/engine/synthetic.rs:93-131,
    vocabulary 152064): hidden 5120, MLP 17408, DeltaNet 16 key / 48 value heads x 128,
    attention 24 q / 4 KV heads x 256 with rotary factor 0.25 and theta 1e7, every
    fourth layer attention."""
    return dict(hidden=5120, inter=17408, layers=layers, heads=24, kv_heads=4, head_dim=256, vocab=vocab,
                lin_key_heads=16, lin_value_heads=48, lin_key_dim=128, lin_value_dim=128, conv_width=4,
                rotary_dim=64, eps=1e-6, theta=1e7, is_attn=[(i + 1) % 4 == 0 for i in range(layers)])


def to_struct(cfg: dict) -> QmrModelConfig:
    c = QmrModelConfig()
    c.hidden_size, c.intermediate_size, c.num_layers = cfg["hidden"], cfg["inter"], cfg["layers"]
    c.num_heads, c.num_kv_heads, c.head_dim, c.vocab_size = cfg["heads"], cfg["kv_heads"], cfg["head_dim"], cfg["vocab"]
    c.linear_key_heads, c.linear_value_heads = cfg["lin_key_heads"], cfg["lin_value_heads"]
    c.linear_key_dim, c.linear_value_dim, c.conv_width = cfg["lin_key_dim"], cfg["lin_value_dim"], cfg["conv_width"]
    c.rotary_dim, c.rms_eps, c.rope_theta = cfg["rotary_dim"], cfg["eps"], cfg["theta"]
    for i, a in enumerate(cfg["is_attn"]):
        c.is_attention[i] = 1 if a else 0
    return c


def from_struct(c: QmrModelConfig) -> dict:
    n = c.num_layers
    return dict(hidden=c.hidden_size, inter=c.intermediate_size, layers=n, heads=c.num_heads,
                kv_heads=c.num_kv_heads, head_dim=c.head_dim, vocab=c.vocab_size, lin_key_heads=c.linear_key_heads,
                lin_value_heads=c.linear_value_heads, lin_key_dim=c.linear_key_dim, lin_value_dim=c.linear_value_dim,
                conv_width=c.conv_width, rotary_dim=c.rotary_dim, eps=float(c.rms_eps), theta=float(c.rope_theta),
                is_attn=[bool(c.is_attention[i]) for i in range(n)])


class Checkpoint:
    """Checkpoint (src/weights.rs): config, packed matrices and vectors of an
    MLX/safetensors checkpoint directory, read by libqmr's C++ loader."""

    def __init__(self, directory):
        self._h = ctypes.c_void_p()
        check(_lib.lib().qmr_checkpoint_open(str(directory).encode(), ctypes.byref(self._h)))

    def close(self):
        if self._h:
            _lib.lib().qmr_checkpoint_close(self._h)
            self._h = ctypes.c_void_p()

    __del__ = close

    def config(self):
        c = QmrModelConfig()
        maxpos, tied = ctypes.c_uint32(), ctypes.c_int()
        check(_lib.lib().qmr_checkpoint_config(self._h, ctypes.byref(c), ctypes.byref(maxpos), ctypes.byref(tied)))
        d = from_struct(c)
        d["max_position"] = maxpos.value
        d["tied"] = bool(tied.value)
        return d

    def matrix(self, name: str):
        """MatrixData::Packed: dict(rows, cols, bits, group, weight u32 [rows, cols*bits/32],
        scales/biases f32 [rows, cols/group])."""
        L = _lib.lib()
        r, c, b, g = (ctypes.c_uint32() for _ in range(4))
        check(L.qmr_checkpoint_matrix(self._h, name.encode(), ctypes.byref(r), ctypes.byref(c), ctypes.byref(b),
                                      ctypes.byref(g), None, None, None))
        rows, cols, bits, group = r.value, c.value, b.value, g.value
        w = np.empty((rows, cols * bits // 32), dtype=np.uint32)
        s = np.empty((rows, cols // group), dtype=np.float32)
        bb = np.empty((rows, cols // group), dtype=np.float32)
        check(L.qmr_checkpoint_matrix(self._h, name.encode(), None, None, None, None, w.ctypes.data, s.ctypes.data,
                                      bb.ctypes.data))
        return dict(rows=rows, cols=cols, bits=bits, group=group, weight=w, scales=s, biases=bb)

    def vector(self, name: str) -> np.ndarray:
        L = _lib.lib()
        n = ctypes.c_uint64()
        check(L.qmr_checkpoint_vector(self._h, name.encode(), None, 0, ctypes.byref(n)))
        out = np.empty(n.value, dtype=np.float32)
        check(L.qmr_checkpoint_vector(self._h, name.encode(), out.ctypes.data, out.size, ctypes.byref(n)))
        return out


class Engine:
    """The decode engine (src/engine.rs Engine) on the current CUDA device."""

    def __init__(self, handle: ctypes.c_void_p):
        self._h = handle
        c = QmrModelConfig()
        ctx = ctypes.c_uint32()
        check(_lib.lib().qmr_model_config(self._h, ctypes.byref(c), ctypes.byref(ctx)))
        self.config = from_struct(c)
        self.context = ctx.value

    @classmethod
    def load(cls, directory, context: int) -> "Engine":
        """Engine::load (src/engine.rs:276-446)."""
        h = ctypes.c_void_p()
        check(_lib.lib().qmr_model_load(str(directory).encode(), context, ctypes.byref(h)))
        return cls(h)

    @classmethod
    def synthetic(cls, cfg: dict, seed: int, context: int) -> "Engine":
        """Engine::synthetic_qwen27b (src/engine/synthetic.rs:92-281) with distinct
        seeded weights per matrix (see qwen27b_config for the benchmark shape)."""
        h = ctypes.c_void_p()
        s = to_struct(cfg)
        check(_lib.lib().qmr_model_synthetic(ctypes.byref(s), seed, context, ctypes.byref(h)))
        return cls(h)

    @classmethod
    def synthetic_sharded(cls, cfg: dict, seed: int, context: int, group=None) -> "Engine":
        """The synthetic model split over the ranks of a torch.distributed
        group, one process per GPU (tensor-parallel decode, include/qmr.h
        "tensor-parallel decode"): every rank calls this together; the IPC
        handles of the ranks' exchange memory travel through
        all_gather_object.  Afterwards every rank makes the same calls and
        gets the same tokens; logits are the rank's vocabulary rows."""
        import torch.distributed as dist
        L = _lib.lib()
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        h = ctypes.c_void_p()
        s = to_struct(cfg)
        check(L.qmr_model_synthetic_sharded(ctypes.byref(s), seed, context, world, rank, ctypes.byref(h)))
        eng = cls(h)
        eng._group, eng._sharded = group, world > 1
        if world > 1:
            mine = ctypes.create_string_buffer(_lib.QMR_IPC_HANDLE_BYTES)
            check(L.qmr_model_exchange_handle(h, mine))
            handles = [None] * world
            dist.all_gather_object(handles, mine.raw, group=group)
            dist.barrier(group)
            allh = ctypes.create_string_buffer(b"".join(handles), world * _lib.QMR_IPC_HANDLE_BYTES)
            check(L.qmr_model_exchange_open(h, allh))
        return eng

    @property
    def shard(self):
        """(world, rank, first vocabulary row, vocabulary rows) of this rank."""
        a, b, c, d = (ctypes.c_uint32() for _ in range(4))
        check(_lib.lib().qmr_model_shard(self._h, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c), ctypes.byref(d)))
        return a.value, b.value, c.value, d.value

    def close(self):
        """Free the model.  A sharded model's peers may still be writing into
        its exchange memory until they finish their last step, so its ranks
        synchronise (device, then a barrier of its group) first."""
        if getattr(self, "_h", None):
            if getattr(self, "_sharded", False):
                import torch
                import torch.distributed as dist
                torch.cuda.synchronize()
                dist.barrier(self._group)
            _lib.lib().qmr_model_free(self._h)
            self._h = None

    def __del__(self):
        if getattr(self, "_h", None):
            _lib.lib().qmr_model_free(self._h)
            self._h = None

    def reset(self) -> None:
        check(_lib.lib().qmr_model_reset(self._h))

    @property
    def position(self) -> int:
        p = ctypes.c_uint32()
        check(_lib.lib().qmr_model_position(self._h, ctypes.byref(p)))
        return p.value

    def forward(self, token: int, logits: bool = True):
        """Engine::forward: (logits f32 [vocab] or None, greedy next token);
        a sharded model returns its vocabulary rows."""
        out = np.empty(self.shard[3], dtype=np.float32) if logits else None
        nxt = ctypes.c_int32()
        check(_lib.lib().qmr_model_forward(self._h, token, out.ctypes.data if logits else None, ctypes.byref(nxt)))
        return out, nxt.value

    def generate(self, prompt: Sequence[int], max_new: int):
        """Prefill `prompt`, then greedy-decode `max_new` tokens on the device.
        Returns (tokens, prefill_ms, decode_ms)."""
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = np.empty(max_new, dtype=np.uint32)
        pre, dec = ctypes.c_double(), ctypes.c_double()
        check(_lib.lib().qmr_model_generate(self._h, p.ctypes.data, p.size, max_new, out.ctypes.data,
                                            ctypes.byref(pre), ctypes.byref(dec)))
        return out.tolist(), pre.value, dec.value

    def verify_block(self, tokens: Sequence[int], logits: bool = True):
        """Engine::verify_block (src/engine/block.rs:296-333): (logits [n, vocab] or
        None, greedy argmax per row); the state stays tentative until commit_block_prefix."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        n = t.size
        lg = np.empty((n, self.shard[3]), dtype=np.float32) if logits else None
        am = np.empty(n, dtype=np.int32)
        check(_lib.lib().qmr_model_verify_block(self._h, t.ctypes.data, n, lg.ctypes.data if logits else None,
                                                am.ctypes.data))
        return lg, am.tolist()

    def commit_block_prefix(self, consumed: int) -> None:
        """Engine::commit_block_prefix (src/engine/block.rs:335-390)."""
        check(_lib.lib().qmr_model_commit_block(self._h, consumed))

    def mtp_generate(self, prompt: Sequence[int], max_new: int, block: int, drafts: Sequence[int]):
        """Greedy decoding in verification rounds of `block` inputs with drafts
        from a per-position table.  Returns (tokens, rounds, accepted drafts,
        prefill_ms, decode_ms)."""
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        d = np.ascontiguousarray(drafts, dtype=np.uint32)
        out = np.empty(max_new, dtype=np.uint32)
        r, a = ctypes.c_uint32(), ctypes.c_uint32()
        pre, dec = ctypes.c_double(), ctypes.c_double()
        check(_lib.lib().qmr_model_mtp_generate(self._h, p.ctypes.data, p.size, block, max_new, d.ctypes.data, d.size,
                                                out.ctypes.data, ctypes.byref(r), ctypes.byref(a),
                                                ctypes.byref(pre), ctypes.byref(dec)))
        return out.tolist(), r.value, a.value, pre.value, dec.value

    def mlp_r2_eligible_matrices(self) -> int:
        n = ctypes.c_uint32()
        check(_lib.lib().qmr_model_mlp_r2_eligible(self._h, ctypes.byref(n)))
        return n.value

    def metadata_stats(self):
        a, b = ctypes.c_uint64(), ctypes.c_uint64()
        check(_lib.lib().qmr_model_metadata_stats(self._h, ctypes.byref(a), ctypes.byref(b)))
        return a.value, b.value

    def step_launches(self):
        """(kernels per step with the head, without it)."""
        a, b = ctypes.c_uint32(), ctypes.c_uint32()
        check(_lib.lib().qmr_model_step_launches(self._h, ctypes.byref(a), ctypes.byref(b)))
        return a.value, b.value
