"""Restatement of the reference's snapshot format and its take / restore
(xigh/herbert-jit-bf16 src/jit/model.rs:100-326, 675-857), over numpy arrays.

TEST INFRASTRUCTURE ONLY: the parity checker of ``hb_snapshot_take`` /
``hb_snapshot_restore`` (byte-identical images, identical restored state).

A ``Runner`` holds one sequence's state as the reference's Runner does on
x86 (no R16 copies, model.rs:552): one bf16 KV buffer with the layer at
``kv_offsets[l]`` laid out [K|V][kv_heads][kv_reserve][head_dim], the DeltaNet
conv and recurrent states (f32), the last token's bf16 logits and ``pos``.
"""
from __future__ import annotations

import struct

import numpy as np

SNAPSHOT_FORMAT = 1                 # model.rs:103
MAX_BLOCK_SNAPSHOT = 64 << 30       # model.rs:108


class Runner:
    """The state a snapshot carries (model.rs:329-396, offsets :545-559)."""

    def __init__(self, kv_heads, kv_reserve, head_dims, conv_len=0, recurrent_len=0,
                 logits_len=16):
        self.kv_heads, self.kv_reserve = kv_heads, kv_reserve
        self.kv_strides = [kv_reserve * h for h in head_dims]   # 0: a layer without cache
        self.kv_offsets = [0]
        for st in self.kv_strides:
            self.kv_offsets.append(self.kv_offsets[-1] + 2 * kv_heads * st)
        self.n_layers = len(head_dims)
        self.kv = np.zeros(self.kv_offsets[-1], np.uint16)
        self.dn_conv = np.zeros(conv_len, np.float32)
        self.dn_recurrent = np.zeros(recurrent_len, np.float32)
        self.logits = np.zeros(logits_len, np.uint16)
        self.pos = 0

    def layer_head_dim(self, l):  # model.rs:701-704
        return 0 if self.kv_strides[l] == 0 else self.kv_strides[l] // self.kv_reserve


class Instantaneous:
    """A frozen state (model.rs:205-221)."""

    def __init__(self, kv_offsets, snap_offsets, snap_positions, kv, dn_conv, dn_recurrent,
                 logits, pos=0, is_filled=False):
        self.kv_offsets, self.snap_offsets = list(kv_offsets), list(snap_offsets)
        self.snap_positions = list(snap_positions)
        self.kv, self.dn_conv, self.dn_recurrent, self.logits = kv, dn_conv, dn_recurrent, logits
        self.pos, self.is_filled = pos, is_filled

    def restorable_at(self, p):  # model.rs:321-323
        return self.is_filled and p <= self.pos and (p == self.pos or self.dn_recurrent.size == 0)


def snapshot_reserve(r: Runner, max_positions: int) -> Instantaneous:
    """model.rs:675-699: per layer min(kv_reserve, max_positions) positions."""
    snap_offsets, snap_positions, total = [0], [], 0
    for l in range(r.n_layers):
        cap = 0 if r.kv_strides[l] == 0 else min(r.kv_reserve, max_positions)
        snap_positions.append(cap)
        total += 2 * r.kv_heads * cap * r.layer_head_dim(l)
        snap_offsets.append(total)
    return Instantaneous(r.kv_offsets, snap_offsets, snap_positions, np.zeros(total, np.uint16),
                         np.zeros_like(r.dn_conv), np.zeros_like(r.dn_recurrent),
                         np.zeros_like(r.logits))


def _compatible(r: Runner, s: Instantaneous):  # model.rs:709-723
    if (s.kv_offsets != r.kv_offsets or s.dn_conv.size != r.dn_conv.size
            or s.dn_recurrent.size != r.dn_recurrent.size or s.logits.size != r.logits.size):
        raise ValueError("the snapshot has been reserved for a different Runner geometry")


def snapshot_take(r: Runner, s: Instantaneous) -> None:
    """model.rs:732-774: the first pos positions of every head, keys then values."""
    _compatible(r, s)
    s.is_filled = False
    for l in range(r.n_layers):
        st = r.kv_strides[l]
        if st == 0:
            continue
        hd, used = r.layer_head_dim(l), r.pos
        if used > s.snap_positions[l]:
            raise ValueError(f"layer {l} holds {used} positions, the slot buffer holds "
                             f"{s.snap_positions[l]}")
        snap_st = s.snap_positions[l] * hd
        src_at, dst_at = r.kv_offsets[l], s.snap_offsets[l]
        for half in range(2):
            src0 = src_at + half * r.kv_heads * st
            dst0 = dst_at + half * r.kv_heads * snap_st
            for h in range(r.kv_heads):
                n = used * hd
                s.kv[dst0 + h * snap_st:dst0 + h * snap_st + n] = r.kv[src0 + h * st:src0 + h * st + n]
    s.dn_conv[:] = r.dn_conv
    s.dn_recurrent[:] = r.dn_recurrent
    s.logits[:] = r.logits
    s.pos = r.pos
    s.is_filled = True


def restore_from(r: Runner, s: Instantaneous, p: int) -> None:
    """model.rs:786-857 (without the R16 copies of AArch64): the first p
    positions of every head, the states, the logits; pos = p."""
    _compatible(r, s)
    if not s.is_filled:
        raise ValueError("restoration refused: snapshot is empty")
    if p > s.pos:
        raise ValueError(f"restoration refused: p={p} beyond snapshot ({s.pos} positions)")
    if p < s.pos and r.dn_recurrent.size:
        raise ValueError("restoration refused: the recurrent state does not revert")
    for l in range(r.n_layers):
        st = r.kv_strides[l]
        if st == 0:
            continue
        hd = r.layer_head_dim(l)
        snap_st = s.snap_positions[l] * hd
        dst_at, src_at = r.kv_offsets[l], s.snap_offsets[l]
        for half in range(2):
            dst0 = dst_at + half * r.kv_heads * st
            src0 = src_at + half * r.kv_heads * snap_st
            for h in range(r.kv_heads):
                n = p * hd
                r.kv[dst0 + h * st:dst0 + h * st + n] = s.kv[src0 + h * snap_st:src0 + h * snap_st + n]
    r.dn_conv[:] = s.dn_conv
    r.dn_recurrent[:] = s.dn_recurrent
    r.logits[:] = s.logits
    r.pos = p


def write_to(s: Instantaneous) -> bytes:
    """model.rs:270-287: version, then every block with its u64 length."""
    if not s.is_filled:
        raise ValueError("empty snapshot: nothing to write")
    out = [struct.pack("<I", SNAPSHOT_FORMAT)]
    for v in (s.kv_offsets, s.snap_offsets, s.snap_positions):
        out.append(struct.pack("<Q", len(v)) + np.asarray(v, "<u8").tobytes())
    for a, dt in ((s.kv, "<u2"), (s.logits, "<u2"), (s.dn_conv, "<f4"), (s.dn_recurrent, "<f4")):
        out.append(struct.pack("<Q", a.size) + np.asarray(a, dt).tobytes())
    out.append(struct.pack("<Q", s.pos))
    return b"".join(out)


def read(b: bytes) -> Instantaneous:
    """model.rs:291-316: every length bounded (64 GiB); truncation refused."""
    at = 0

    def take(n):
        nonlocal at
        if at + n > len(b):
            raise ValueError("snapshot image truncated")
        v = b[at:at + n]
        at += n
        return v

    if struct.unpack("<I", take(4))[0] != SNAPSHOT_FORMAT:
        raise ValueError("snapshot of another version of format")

    def block(elem, dt):
        n = struct.unpack("<Q", take(8))[0]
        if n * elem > MAX_BLOCK_SNAPSHOT:
            raise ValueError(f"block of {n} elements: beyond the ceiling")
        return np.frombuffer(take(n * elem), dt).copy()

    kv_offsets = [int(x) for x in block(8, "<u8")]
    snap_offsets = [int(x) for x in block(8, "<u8")]
    snap_positions = [int(x) for x in block(8, "<u8")]
    kv, logits = block(2, "<u2"), block(2, "<u2")
    conv, rec = block(4, "<f4"), block(4, "<f4")
    pos = struct.unpack("<Q", take(8))[0]
    return Instantaneous(kv_offsets, snap_offsets, snap_positions, kv, conv, rec, logits, pos,
                         True)


def seeded_runner(kv_heads, kv_reserve, head_dims, conv_len, recurrent_len, logits_len, pos,
                  seed):
    """A Runner whose every buffer holds seeded values (bits, not meaning)."""
    r = Runner(kv_heads, kv_reserve, head_dims, conv_len, recurrent_len, logits_len)
    rng = np.random.default_rng(seed)
    r.kv[:] = rng.integers(0, 1 << 16, r.kv.size, dtype=np.uint16)
    r.dn_conv[:] = rng.standard_normal(conv_len, dtype=np.float32)
    r.dn_recurrent[:] = rng.standard_normal(recurrent_len, dtype=np.float32)
    r.logits[:] = rng.integers(0, 1 << 16, logits_len, dtype=np.uint16)
    r.pos = pos
    return r


def image_c(r: Runner, max_positions: int, out=None):
    """The same image as write_to(snapshot_take(reserve(max_positions))), made by
    the oracle's C restatement (memcpy per head, as the reference copies).
    With `out` (a uint8 array of the image's size, reserved once as the
    reference reserves its slot) the image is written there and `out` is
    returned; else a new bytes object."""
    import ctypes
    import oracle as O
    L = O.lib()
    fn = L.orc_snapshot_image
    fn.restype = ctypes.c_longlong
    u16, f32 = ctypes.POINTER(ctypes.c_uint16), ctypes.POINTER(ctypes.c_float)
    offs = np.asarray(r.kv_offsets, np.int64)
    args = [r.kv.ctypes.data_as(u16), offs.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)),
            ctypes.c_size_t(r.n_layers), ctypes.c_size_t(r.kv_heads),
            ctypes.c_size_t(r.kv_reserve), ctypes.c_size_t(max_positions), ctypes.c_size_t(r.pos),
            r.dn_conv.ctypes.data_as(f32), ctypes.c_size_t(r.dn_conv.size),
            r.dn_recurrent.ctypes.data_as(f32), ctypes.c_size_t(r.dn_recurrent.size),
            r.logits.ctypes.data_as(u16), ctypes.c_size_t(r.logits.size)]
    if out is not None:
        if fn(*args, out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8))) < 0:
            raise ValueError("the state holds more positions than the slot")
        return out
    n = fn(*args, None)
    if n < 0:
        raise ValueError("the state holds more positions than the slot")
    buf = np.empty(n, np.uint8)
    fn(*args, buf.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)))
    return buf.tobytes()
