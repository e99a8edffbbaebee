"""The peer exchange's handshake on one GPU, with the "peer" a second buffer of
this GPU: the publish step passes when the peer's flag is set and copies the
peer's view record, and its bounded wait gives up -- reporting GS_ERR_TIMEOUT
instead of hanging -- when nothing ever sets the flag. No second kernel waits
on this one: the flag is either set beforehand or never."""

import ctypes

import pytest
import torch

from gaussian_splats_b200 import native

pytestmark = pytest.mark.gpu

READY = 2  # int64 index of ready[0] in the arena header: epoch, error+pad, ready[8], done[8]


def _arenas(n):
    lay = native.ExchangeLayout()
    native.check(native.lib().gs_exchange_layout_for(n, 2, ctypes.byref(lay)), "layout")
    arenas = [torch.zeros(int(lay.bytes), dtype=torch.uint8, device="cuda") for _ in range(2)]
    assert all(a.data_ptr() % 256 == 0 for a in arenas)
    group = native.PeerGroup(0, 2, (ctypes.c_void_p * native.GS_MAX_PEERS)(
        *[a.data_ptr() for a in arenas], *[None] * (native.GS_MAX_PEERS - 2)))
    return lay, arenas, group


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def test_publish_passes_when_the_peer_has_published():
    n = 1000
    lay, (mine, peer), group = _arenas(n)
    lib = native.lib()
    record = torch.arange(native.VIEW_RECORD_WORDS, dtype=torch.int32, device="cuda") + 100
    peer[lay.record:lay.record + 4 * native.VIEW_RECORD_WORDS].view(torch.int32).copy_(record)
    mine.view(torch.int64)[READY + 1] = 1  # the peer (rank 1) published epoch 1
    ref = ctypes.byref(group)
    native.check(lib.gs_exchange_begin(ref, _stream()), "begin")
    native.check(lib.gs_exchange_publish(ref, n, _stream()), "publish")
    native.check(lib.gs_exchange_finish(ref, _stream()), "finish")
    assert lib.gs_exchange_status(ref, _stream()) == 0
    header_mine, header_peer = mine.view(torch.int64), peer.view(torch.int64)
    assert int(header_mine[0]) == 1  # this rank's epoch
    assert int(header_peer[READY + 0]) == 1  # published to the peer
    assert int(header_peer[READY + 8 + 0]) == 1  # done, to the peer
    gathered = mine[lay.gathered:lay.gathered + 8 * native.VIEW_RECORD_WORDS].view(torch.int32)
    assert torch.equal(gathered[native.VIEW_RECORD_WORDS:2 * native.VIEW_RECORD_WORDS], record)


def test_publish_reports_a_peer_that_never_arrives():
    n = 1000
    _, (mine, _), group = _arenas(n)
    lib = native.lib()
    ref = ctypes.byref(group)
    native.check(lib.gs_exchange_publish(ref, n, _stream()), "publish")  # waits about a second
    assert lib.gs_exchange_status(ref, _stream()) == -6  # GS_ERR_TIMEOUT
    # the context stays usable
    x = torch.ones(4, device="cuda")
    assert float(x.sum()) == 4.0
