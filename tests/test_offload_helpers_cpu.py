"""CPU tests of the host helpers around the offloaded experts: page-locking
(``pin_experts``, bin/offload.py:664-699) and sizing the device cache from
free device memory (``size_cache_to_free_vram``, bin/offload.py:611-661).

No GPU: a fake model in the reference's layout
(``model.backbone.model.layers[i].mlp.experts``), ``Tensor.pin_memory`` /
``is_pinned`` and ``torch.cuda.mem_get_info`` stubbed, and
``devcache.init_dev_cache`` replaced by a recorder.
"""
from types import SimpleNamespace

import pytest
import torch

from drama3_offloading_b200 import devcache, offload, synth

H, I, E = 256, 128, 4          # one expert: 2*128*256 + 256*128 + 4*(2*2 + 2*1) = 98,328 B
EXPERT = 2 * I * H + H * I + 4 * (2 * I // 128) * (H // 128) + 4 * (H // 128) * (I // 128)


def _store(seed):
    return synth.make_experts(E, H, I, seed=seed, device="cpu", style="test")


def _model(n_layers, resident=()):
    """Fake model: layer i has host experts, except those in ``resident``
    (experts on a GPU-like device) and the last layer, which has no experts
    (a dense layer)."""
    layers = []
    for i in range(n_layers):
        ex = _store(i)
        if i in resident:
            ex = SimpleNamespace(num_experts=E, w13_weight=SimpleNamespace(
                device=torch.device("meta")))
        layers.append(SimpleNamespace(mlp=SimpleNamespace(experts=ex)))
    layers.append(SimpleNamespace(mlp=SimpleNamespace()))
    return SimpleNamespace(backbone=SimpleNamespace(model=SimpleNamespace(layers=layers)))


@pytest.fixture
def fake_pinning(monkeypatch):
    """pin_memory() returns a copy marked pinned; is_pinned() reads the mark."""
    pinned = set()

    def pin_memory(self):
        c = self.clone()
        pinned.add(c.data_ptr())
        return c

    monkeypatch.setattr(torch.Tensor, "pin_memory", pin_memory)
    monkeypatch.setattr(torch.Tensor, "is_pinned", lambda self: self.data_ptr() in pinned)
    return pinned


def test_bytes_per_expert_measures_the_store():
    assert offload.bytes_per_expert(_store(0)) == EXPERT
    full = synth.HostExperts(1, torch.empty(1, 1024, 2048, dtype=torch.float8_e4m3fn),
                             torch.empty(1, 2048, 512, dtype=torch.float8_e4m3fn),
                             torch.empty(1, 8, 16), torch.empty(1, 16, 4))
    assert offload.bytes_per_expert(full) == offload.EXPERT_BYTES == 3_146_496


def test_offloaded_stores_skips_dense_and_resident_layers():
    m = _model(4, resident=(1,))
    stores = offload.offloaded_stores(m)
    assert len(stores) == 3
    layers = m.backbone.model.layers
    assert [id(s) for s in stores] == [id(layers[i].mlp.experts) for i in (0, 2, 3)]
    # an iterable of stores is taken as it is (host stores only)
    assert offload.offloaded_stores(stores) == stores


def test_pin_experts_pins_each_buffer_once(fake_pinning):
    m = _model(3)
    stores = offload.offloaded_stores(m)
    before = {n: getattr(stores[0], n).clone() for n in devcache._BUFFERS}
    # one buffer already page-locked: it is left alone and not counted
    already = stores[1].w2_weight.pin_memory()
    stores[1].w2_weight = already
    gib, secs = offload.pin_experts(m, torch.device("cpu"))
    want = 3 * E * EXPERT - already.numel()
    assert gib == pytest.approx(want / 2**30)
    assert secs >= 0
    for ex in stores:
        for n in devcache._BUFFERS:
            assert getattr(ex, n).is_pinned()
    assert stores[1].w2_weight is already
    for n, t in before.items():  # contents unchanged
        assert torch.equal(getattr(stores[0], n).view(torch.uint8), t.view(torch.uint8))
    # a second call finds nothing to do
    gib2, _ = offload.pin_experts(m)
    assert gib2 == 0.0


@pytest.fixture
def fake_device(monkeypatch):
    """mem_get_info -> (free, total); init_dev_cache records its calls."""
    state = {"free": 0, "calls": [], "emptied": 0}
    monkeypatch.setattr(torch.cuda, "synchronize", lambda device=None: None)

    def empty_cache():
        state["emptied"] += 1

    monkeypatch.setattr(torch.cuda, "empty_cache", empty_cache)
    monkeypatch.setattr(torch.cuda, "mem_get_info",
                        lambda device=None: (state["free"], 180 << 30))
    monkeypatch.setattr(devcache, "init_dev_cache",
                        lambda ex, device, capacity, policy=None:
                        state["calls"].append((id(ex), capacity)))
    return state


GiB = 1 << 30


def test_size_cache_splits_free_memory_over_layers(fake_device):
    m = _model(4, resident=(2,))                 # 3 offloaded layers
    reserve = int((2.0 + offload.ACTIVATION_HEADROOM_GIB) * GiB)
    fake_device["free"] = reserve + 3 * EXPERT * 3 + 17   # 3 slots per layer and change
    cap = offload.size_cache_to_free_vram(m, "cpu", cap_per_layer=256)
    assert cap == 3
    assert fake_device["emptied"] == 1
    stores = offload.offloaded_stores(m)
    assert fake_device["calls"] == [(id(s), 3) for s in stores]


def test_size_cache_clamps_to_cap_and_expert_count(fake_device):
    m = _model(2)
    fake_device["free"] = 100 * GiB
    assert offload.size_cache_to_free_vram(m, "cpu", cap_per_layer=256) == E
    fake_device["calls"].clear()
    assert offload.size_cache_to_free_vram(m, "cpu", cap_per_layer=2) == 2
    assert all(c == 2 for _, c in fake_device["calls"])


def test_size_cache_zero_when_reserve_not_covered(fake_device):
    m = _model(2)
    fake_device["free"] = int(3.5 * GiB) + 2 * EXPERT - 1   # one byte short of a slot row
    assert offload.size_cache_to_free_vram(m, "cpu", leave_free_gib=2.0) == 0
    assert fake_device["calls"] == []
    fake_device["free"] = GiB                                 # below the reserve itself
    assert offload.size_cache_to_free_vram(m, "cpu") == 0
    # a model with no offloaded experts asks for nothing
    assert offload.size_cache_to_free_vram(_model(0), "cpu") == 0
