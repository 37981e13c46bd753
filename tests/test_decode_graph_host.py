"""Host logic of DeviceRingHeads (no GPU): the per-replay advance of each
layer's state, the re-upload of the device heads after eager calls moved a
window, the rejection of a changed history and of a partial window, and the
host state a recording puts back.  Fake layers stand in for M12LayerRuntime;
the device heads are a CPU tensor here."""
import types

import pytest
import torch

from helpers import pkg


def _layer(i, valid_len=1000, head=5, R=512, S=64, nb=16):
    cfg = types.SimpleNamespace(recent_tokens=R, sink_tokens=S, check_finite_outputs=True)
    return types.SimpleNamespace(
        layer_id=i, cfg=cfg, device=torch.device("cpu"), _fast_ok=True, record_q=False, record_ids=False,
        _k_store=object(), _dargs=object(), valid_len=valid_len, nblocks_filled=nb, _ring_head=head,
        _ids_view="ids", _last_ids_dev=None, _last_ids_host=[1], timings={}, _ring_dev_ptr=0,
        _out_override=None)


def test_heads_advance_wrap_and_resync():
    dg = pkg().decode_graph
    layers = [_layer(0, head=510), _layer(1, head=3, R=64)]
    h = dg.DeviceRingHeads(layers)
    assert h._ring[:, 0].tolist() == [510, 3] and h._ring[:, 1].tolist() == [0, 0]
    for _ in range(3):
        h.before_replay()
        h.after_replay()
    assert [rt._ring_head for rt in layers] == [1, 6]  # 510 -> 511 -> 0 -> 1 (R 512)
    assert [rt.valid_len for rt in layers] == [1003, 1003]
    assert layers[0]._last_ids_dev == "ids" and layers[0]._last_ids_host is None
    # an eager decode moved layer 1's window: the next replay re-uploads the heads
    layers[1]._ring_head = 7
    h._ring.zero_()
    h.before_replay()
    assert h._ring[:, 0].tolist() == [1, 7]
    # a history change invalidates the recording
    layers[0].nblocks_filled += 1
    with pytest.raises(RuntimeError):
        h.before_replay()


def test_recording_restores_host_state_and_rejects_partial_window():
    dg = pkg().decode_graph
    layers = [_layer(0)]
    h = dg.DeviceRingHeads(layers)
    with h.recording():
        assert layers[0]._ring_dev_ptr == h._ring[0].data_ptr()
        assert layers[0].cfg.check_finite_outputs is False
        layers[0].valid_len += 1
        layers[0]._ring_head += 1
    assert layers[0]._ring_dev_ptr == 0 and layers[0].cfg.check_finite_outputs is True
    assert layers[0].valid_len == 1000 and layers[0]._ring_head == 5
    with pytest.raises(AssertionError):
        dg.DeviceRingHeads([_layer(0, valid_len=400)])  # window not full yet
    with pytest.raises(AssertionError):
        dg.DeviceRingHeads([_layer(0, valid_len=30, R=16)])  # sink not full yet
