"""Host side of failure detection, without a GPU: the in-kernel status word
(``fqkv_device_status``) is turned into an exception that names the cause, and
reading it resets it.  A fake of the native call stands in for the library;
the GPU side (bounded waits that end with these codes) is covered by
``test_failure_gpu.py``."""
from __future__ import annotations

import pytest
import torch


class _FakeLib:
    def __init__(self, code: int):
        self.code = code
        self.clears = []

    def fqkv_device_status(self, out, clear):
        out._obj.value = self.code
        self.clears.append(clear)
        if clear:
            self.code = 0
        return 0


class _NoGuard:
    def __init__(self, dev):
        pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


@pytest.mark.parametrize("code,cause", [(64, "tensor-parallel peer"), (61, "wait for a KV tile"),
                                        (62, "free pipeline stage"), (63, "drain"), (99, "unknown code")])
def test_check_device_status_names_the_cause_and_resets(fqkv, monkeypatch, code, cause):
    fake = _FakeLib(code)
    monkeypatch.setattr(fqkv.ops._native, "lib", lambda: fake)
    monkeypatch.setattr(fqkv.ops, "_DeviceGuard", _NoGuard)
    dev = torch.device("cuda", 0)
    with pytest.raises(RuntimeError, match=cause) as e:
        fqkv.ops.check_device_status(dev, "decode step")
    assert f"device status {code}" in str(e.value)
    fqkv.ops.check_device_status(dev, "decode step")      # reset by the first read: no error now
    assert fake.clears == [1, 1]


def test_device_status_can_read_without_reset(fqkv, monkeypatch):
    fake = _FakeLib(64)
    monkeypatch.setattr(fqkv.ops._native, "lib", lambda: fake)
    monkeypatch.setattr(fqkv.ops, "_DeviceGuard", _NoGuard)
    dev = torch.device("cuda", 0)
    assert fqkv.ops.device_status(dev, clear=False) == 64
    assert fqkv.ops.device_status(dev, clear=True) == 64
    assert fqkv.ops.device_status(dev) == 0
