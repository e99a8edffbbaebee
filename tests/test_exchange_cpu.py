"""Host side of the peer exchange: the arena layout through the C ABI (no GPU
needed) and the peer-group structure the bindings pass."""

import ctypes

from gaussian_splats_b200 import native


def _layout(n, world):
    out = native.ExchangeLayout()
    status = native.lib().gs_exchange_layout_for(n, world, ctypes.byref(out))
    return status, out


def test_arena_layout_is_aligned_and_sized():
    for n in (0, 1, 1000, 1_000_003):
        status, lay = _layout(n, 4)
        assert status == 0
        offsets = [lay.grad_projected, lay.counts, lay.record, lay.gathered, lay.bytes]
        assert all(o % 256 == 0 for o in offsets)
        assert lay.grad_projected >= 256  # the header comes first
        assert lay.counts >= lay.grad_projected + 36 * n
        assert lay.record >= lay.counts + 4 * n
        assert lay.gathered >= lay.record + 4 * native.VIEW_RECORD_WORDS
        assert lay.bytes >= lay.gathered + 4 * native.VIEW_RECORD_WORDS * native.GS_MAX_PEERS


def test_layout_rejects_bad_groups():
    assert _layout(10, 0)[0] != 0
    assert _layout(10, native.GS_MAX_PEERS + 1)[0] != 0
    assert _layout(-1, 2)[0] != 0


def test_peer_group_struct_matches_the_header():
    # int32 rank, int32 world, then GS_MAX_PEERS pointers
    assert ctypes.sizeof(native.PeerGroup) == 8 + 8 * native.GS_MAX_PEERS
    assert ctypes.sizeof(native.ExchangeLayout) == 5 * 8


def test_shard_layout_follows_the_plain_arena():
    lib = native.lib()
    for n, world, k in ((1_000_000, 8, 16), (60_000, 2, 16), (7, 3, 1), (0, 4, 25)):
        base = _layout(n, world)[1]
        out = native.ShardLayout()
        assert lib.gs_exchange_shard_layout(n, world, k, ctypes.byref(out)) == 0
        rows = -(-n // world)
        rows = -(-rows // 64) * 64  # shards start on 16-byte boundaries of every array
        assert out.rows == rows
        offsets = [out.rotation, out.color, out.mean, out.scale, out.opacity, out.bytes]
        assert all(o % 256 == 0 for o in offsets)
        assert out.rotation >= base.bytes  # the shard follows the plain arena
        assert out.color >= out.rotation + 16 * rows
        assert out.mean >= out.color + 12 * k * rows
        assert out.scale >= out.mean + 12 * rows
        assert out.opacity >= out.scale + 12 * rows
        assert out.bytes >= out.opacity + 4 * rows
    out = native.ShardLayout()
    assert lib.gs_exchange_shard_layout(10, 2, 26, ctypes.byref(out)) != 0
    assert lib.gs_exchange_shard_layout(10, native.GS_MAX_PEERS + 1, 16, ctypes.byref(out)) != 0
