"""Host side of the failure path for the tensor-parallel layer, without a GPU.

When a bounded wait on the device gives up (an NVLS barrier whose peers never
arrived, a GEMM pipeline wait), the kernel records a code in the library's
device error word and the NVLS reduction skips its work. The host learns of
it through `zcutlass_b200.tp.check_device_error`, which bench.py calls after
its timed steps: it must raise for any recorded code and for an unreadable
word, and stay quiet when the word is clear. The device word is replaced here
by a fake reader, so nothing touches a GPU.
"""

from __future__ import annotations

import pytest

from zcutlass_b200 import _native, tp


def _fake_reader(values):
    calls = []

    def device_error(clear=False):
        calls.append(clear)
        return values.pop(0)

    return device_error, calls


def test_clear_word_passes(monkeypatch):
    reader, calls = _fake_reader([0])
    monkeypatch.setattr(_native, "device_error", reader)
    tp.check_device_error()
    assert calls == [True]  # the check clears the word it read


def test_barrier_timeout_code_raises(monkeypatch):
    code = (16 << 4) | 1  # the NVLS barrier before a reduction gave up waiting
    reader, _ = _fake_reader([code])
    monkeypatch.setattr(_native, "device_error", reader)
    with pytest.raises(RuntimeError, match=r"0x101 \(site 16, role 1\)"):
        tp.check_device_error()


def test_unreadable_word_raises(monkeypatch):
    reader, _ = _fake_reader([-1])
    monkeypatch.setattr(_native, "device_error", reader)
    with pytest.raises(RuntimeError, match="unreadable"):
        tp.check_device_error()
