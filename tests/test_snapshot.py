"""Snapshot / restore of a sequence's device state in the reference's
Instantaneous format (src/jit/model.rs:100-326, 675-857).

CPU: the oracle's format round-trips, matches the committed golden image and
its hand-decoded header; the C ABI sizes images as the oracle writes them,
reads their position, and refuses bad images and requests before any copy.
GPU: ``hb_snapshot_take`` writes the oracle's bytes from device buffers,
``hb_snapshot_restore`` gives the oracle's restored state, images cross
between the two in both directions.
"""
import ctypes
import os
import struct

import numpy as np
import pytest

import herbert_b200 as hb
import snapshot as S

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "snapshot_hybrid.bin")

GEOMETRIES = {
    # name: (kv_heads, kv_reserve, head_dims per layer, conv_len, recurrent_len, logits_len)
    "hybrid": (2, 40, [0, 0, 0, 64, 0, 0, 0, 64], 6 * 96 * 4, 6 * 2 * 16 * 16, 48),
    "attention_only": (4, 33, [32, 32, 128], 0, 0, 32),
    "no_cache": (1, 8, [0, 0], 16, 64, 16),
}


def _runner(name, pos, seed=0x5A7):
    kvh, res, hds, conv, rec, lg = GEOMETRIES[name]
    return S.seeded_runner(kvh, res, hds, conv, rec, lg, pos, seed)


def _geo(r):
    return hb.Geometry(r.kv_offsets, r.kv_heads, r.kv_reserve, r.dn_conv.size, r.dn_recurrent.size,
                       r.logits.size)


def _oracle_image(r, max_positions):
    s = S.snapshot_reserve(r, max_positions)
    S.snapshot_take(r, s)
    return S.write_to(s)


# ----------------------------------------------------------------- CPU only

@pytest.mark.parametrize("name", sorted(GEOMETRIES))
def test_oracle_round_trip(name):
    r = _runner(name, 17)
    img = _oracle_image(r, 25)
    s = S.read(img)
    assert S.write_to(s) == img
    fresh = S.Runner(r.kv_heads, r.kv_reserve, [r.layer_head_dim(l) for l in range(r.n_layers)],
                     r.dn_conv.size, r.dn_recurrent.size, r.logits.size)
    S.restore_from(fresh, s, 17)
    for l in range(r.n_layers):
        st, hd = r.kv_strides[l], r.layer_head_dim(l)
        for half in range(2):
            for h in range(r.kv_heads):
                a = r.kv_offsets[l] + (half * r.kv_heads + h) * st
                assert np.array_equal(fresh.kv[a:a + 17 * hd], r.kv[a:a + 17 * hd])
    assert np.array_equal(fresh.dn_recurrent, r.dn_recurrent) and fresh.pos == 17


@pytest.mark.parametrize("name", sorted(GEOMETRIES))
@pytest.mark.parametrize("pos,max_positions", [(17, 25), (0, 5), (8, 1000)])
def test_oracle_c_image_equals_the_restatement(name, pos, max_positions):
    pos = min(pos, GEOMETRIES[name][1])
    r = _runner(name, pos)
    want = _oracle_image(r, max_positions)
    assert S.image_c(r, max_positions) == want
    slot = np.full(len(want), 0xCD, np.uint8)   # a reused slot is fully rewritten
    assert S.image_c(r, max_positions, out=slot).tobytes() == want


def test_oracle_refusals():
    r = _runner("hybrid", 30)
    s = S.snapshot_reserve(r, 20)
    with pytest.raises(ValueError, match="slot buffer"):
        S.snapshot_take(r, s)
    r.pos = 12
    S.snapshot_take(r, s)
    with pytest.raises(ValueError, match="does not revert"):
        S.restore_from(r, s, 11)
    with pytest.raises(ValueError, match="beyond"):
        S.restore_from(r, s, 13)
    img = bytearray(S.write_to(s))
    img[0] = 2
    with pytest.raises(ValueError, match="version"):
        S.read(bytes(img))
    with pytest.raises(ValueError, match="truncated"):
        S.read(S.write_to(s)[:-3])


def test_golden_image_and_its_header():
    img = open(GOLDEN, "rb").read()
    r = _runner("hybrid", 21, seed=0x60D4)
    assert _oracle_image(r, 32) == img
    # hand-decoded: version 1; 9 kv_offsets, the first two zero (layers
    # without cache), the fourth layer at 0 and 2*2*40*64 = 10240 elements
    assert struct.unpack_from("<I", img, 0) == (1,)
    assert struct.unpack_from("<Q", img, 4) == (9,)
    assert struct.unpack_from("<9Q", img, 12) == (0, 0, 0, 0, 10240, 10240, 10240, 10240, 20480)
    # snap_offsets: 2*2*32*64 = 8192 per owning layer
    assert struct.unpack_from("<Q9Q", img, 84) == (9, 0, 0, 0, 0, 8192, 8192, 8192, 8192, 16384)
    assert struct.unpack_from("<Q8Q", img, 164) == (8, 0, 0, 0, 32, 0, 0, 0, 32)
    assert struct.unpack_from("<Q", img, len(img) - 8) == (21,)
    assert hb.snapshot_info(np.frombuffer(img, np.uint8)) == (21, False)


@pytest.mark.parametrize("name", sorted(GEOMETRIES))
@pytest.mark.parametrize("max_positions", [0, 7, 33, 1000])
def test_abi_sizes_images_as_the_oracle_writes_them(name, max_positions):
    r = _runner(name, 0)
    assert hb.snapshot_bytes(_geo(r), max_positions) == len(_oracle_image(r, max_positions))


def test_abi_info():
    r = _runner("attention_only", 9)
    assert hb.snapshot_info(np.frombuffer(_oracle_image(r, 20), np.uint8)) == (9, True)
    with pytest.raises(hb.HBError):
        hb.snapshot_info(np.frombuffer(_oracle_image(r, 20)[:-1], np.uint8))


def _restore_status(geo, img, p):
    bufs = hb.StateBuffers(kv=256, dn_conv=256, dn_recurrent=256, logits=256)
    a = np.frombuffer(img, np.uint8)
    return hb.lib().hb_snapshot_restore(ctypes.byref(geo.c), ctypes.byref(bufs),
                                        ctypes.c_void_p(a.ctypes.data), a.size, p, None)


def test_abi_refusals_happen_before_any_copy():
    # fake device pointers: every case must be refused by the host checks;
    # never run where a GPU could receive a copy
    import torch
    if torch.cuda.is_available():
        pytest.skip("fake-pointer refusals run on hosts without a GPU only")
    r = _runner("hybrid", 12)
    geo = _geo(r)
    img = _oracle_image(r, 20)
    assert _restore_status(geo, img, 13) == hb.HB_ERR_ARG          # beyond the snapshot
    assert _restore_status(geo, img, 11) == hb.HB_ERR_ARG          # recurrent state
    assert "does not revert" in hb.last_error()
    assert _restore_status(geo, b"\x02" + img[1:], 12) == hb.HB_ERR_ARG
    assert "version" in hb.last_error()
    assert _restore_status(geo, img[:100], 12) == hb.HB_ERR_ARG    # truncated
    bad = bytearray(img)
    struct.pack_into("<Q", bad, 84, 1 << 40)                     # a corrupted length
    assert _restore_status(geo, bytes(bad), 12) == hb.HB_ERR_ARG
    assert "ceiling" in hb.last_error() or "truncated" in hb.last_error()
    bad = bytearray(img)
    struct.pack_into("<Q", bad, 164 + 8 * 4, 33)                 # slot capacity / offsets disagree
    assert _restore_status(geo, bytes(bad), 12) == hb.HB_ERR_ARG
    other = hb.Geometry(r.kv_offsets, r.kv_heads, r.kv_reserve, r.dn_conv.size + 4,
                        r.dn_recurrent.size, r.logits.size)
    assert _restore_status(other, img, 12) == hb.HB_DECLINE_GEOMETRY
    # take: a state longer than the slot is refused, nothing copied
    bufs = hb.StateBuffers(kv=256, dn_conv=256, dn_recurrent=256, logits=256)
    out = np.zeros(hb.snapshot_bytes(geo, 10), np.uint8)
    rc = hb.lib().hb_snapshot_take(ctypes.byref(geo.c), ctypes.byref(bufs), 12, 10,
                                   ctypes.c_void_p(out.ctypes.data), out.size, None)
    assert rc == hb.HB_ERR_ARG and "slot buffer" in hb.last_error()
    small = np.zeros(hb.snapshot_bytes(geo, 20) - 1, np.uint8)
    rc = hb.lib().hb_snapshot_take(ctypes.byref(geo.c), ctypes.byref(bufs), 12, 20,
                                   ctypes.c_void_p(small.ctypes.data), small.size, None)
    assert rc == hb.HB_ERR_ARG
    bad_geo = hb.Geometry([0, 100], 2, 40)
    assert hb.snapshot_bytes(bad_geo, 10) == 0


# ---------------------------------------------------------------------- GPU

def _device_state(r):
    import torch
    dev = lambda a: torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a.copy()).cuda()  # noqa: E731
    return dev(r.kv.copy()), dev(r.dn_conv), dev(r.dn_recurrent), dev(r.logits.copy())


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(GEOMETRIES))
@pytest.mark.parametrize("pos,max_positions", [(17, 25), (0, 5), (33, 33), (8, 1000)])
def test_take_writes_the_oracle_bytes(name, pos, max_positions):
    import torch
    kvh, res, hds, conv, rec, lg = GEOMETRIES[name]
    pos = min(pos, res)
    r = _runner(name, pos)
    want = _oracle_image(r, max_positions)
    state = _device_state(r)
    image = torch.full((hb.snapshot_bytes(_geo(r), max_positions),), 0xAB,
                       dtype=torch.uint8).pin_memory()
    hb.snapshot_take(_geo(r), *state, image, pos=pos, max_positions=max_positions)
    torch.cuda.synchronize()
    assert image.numpy().tobytes() == want


@pytest.mark.gpu
@pytest.mark.parametrize("name,p", [("hybrid", 21), ("attention_only", 21), ("attention_only", 6),
                                    ("attention_only", 0), ("no_cache", 21)])
def test_restore_gives_the_oracle_state(name, p):
    import torch
    r = _runner(name, 21)
    img = _oracle_image(r, 30)                      # a file the reference would write
    target = _runner(name, 3, seed=0xBEEF)          # whatever the device held before
    state = _device_state(target)
    hb.snapshot_restore(_geo(r), *state, np.frombuffer(img, np.uint8), p=p)
    torch.cuda.synchronize()
    S.restore_from(target, S.read(img), p)
    kv, conv, rec, lg = (t.cpu().numpy() for t in state)
    assert np.array_equal(kv.view(np.uint16), target.kv)
    assert np.array_equal(conv.view(np.uint32), target.dn_conv.view(np.uint32))
    assert np.array_equal(rec.view(np.uint32), target.dn_recurrent.view(np.uint32))
    assert np.array_equal(lg.view(np.uint16), target.logits)


@pytest.mark.gpu
def test_device_round_trip_through_a_pinned_image():
    import torch
    r = _runner("hybrid", 40)
    src = _device_state(r)
    geo = _geo(r)
    image = torch.empty(hb.snapshot_bytes(geo, 40), dtype=torch.uint8).pin_memory()
    hb.snapshot_take(geo, *src, image, pos=40, max_positions=40)
    torch.cuda.synchronize()
    dst = tuple(torch.zeros_like(t) for t in src)
    hb.snapshot_restore(geo, *dst, image, p=40)
    torch.cuda.synchronize()
    for a, b in zip(src, dst):
        assert torch.equal(a, b)
    assert hb.snapshot_info(image) == (40, False)


def test_corrupted_images_are_refused_never_crash():
    # A file from disk may be truncated or damaged anywhere: parsing must end
    # in a named status.  Fake device pointers: skipped where a GPU could
    # receive a copy (an image damaged only in its payload passes validation).
    import torch
    if torch.cuda.is_available():
        pytest.skip("fake-pointer refusals run on hosts without a GPU only")
    r = _runner("hybrid", 12)
    geo = _geo(r)
    img = _oracle_image(r, 20)
    head = 4 + 8 * (1 + 9) + 8 * (1 + 9) + 8 * (1 + 8) + 8   # through the kv length field
    rng = np.random.default_rng(0xF022)
    allowed = {hb.HB_OK, hb.HB_ERR_ARG, hb.HB_DECLINE_GEOMETRY, hb.HB_ERR_CUDA}
    for trial in range(400):
        b = bytearray(img)
        kind = trial % 4
        if kind == 0:                                   # truncated anywhere
            b = b[:int(rng.integers(0, len(b)))]
        elif kind == 1:                                 # a byte of the header flipped
            i = int(rng.integers(0, head))
            b[i] ^= int(rng.integers(1, 256))
        elif kind == 2:                                 # a hostile 64-bit field
            i = 4 + 8 * int(rng.integers(0, (head - 4) // 8))
            hostile = [0, 1, 2**31, 2**40, 2**63, 2**64 - 1]
            struct.pack_into("<Q", b, i, hostile[int(rng.integers(0, len(hostile)))])
        else:                                           # the trailing pos field
            struct.pack_into("<Q", b, len(b) - 8, int(rng.integers(0, 2**63)))
        data = bytes(b) if b else b"\0"
        a = np.frombuffer(data, np.uint8)
        pos, below = ctypes.c_int64(0), ctypes.c_int32(0)
        st = hb.lib().hb_snapshot_info(ctypes.c_void_p(a.ctypes.data), len(b), ctypes.byref(pos),
                                       ctypes.byref(below))
        assert st in (hb.HB_OK, hb.HB_ERR_ARG)
        st = _restore_status(geo, data[:len(b)] if b else b"", 12)
        assert st in allowed, (trial, st)
        if kind in (0, 1, 2) and st == hb.HB_OK:
            raise AssertionError(f"trial {trial}: a damaged header was accepted")
