"""The numpy entry points' device-copy cache of weight arrays, on the CPU: the
upload is replaced by a stand-in object, so the test needs no GPU. It checks
the cache's rules: one upload per buffer, the same object found without its
key, views sharing the copy, invalidate() after an in-place change, and the
copy dropped when the array is freed."""

import gc

import numpy as np
import pytest

from quartz_b200 import _host


class _Copy:
    """Stands in for the device tensor: remembers what was uploaded."""

    def __init__(self, a):
        self.a = np.array(a, copy=True)

    def to(self, device, non_blocking=False):
        return self

    def numel(self):
        return self.a.size

    def element_size(self):
        return self.a.itemsize


class _Torch:
    uploads = 0

    @classmethod
    def from_numpy(cls, a):
        cls.uploads += 1
        return _Copy(a)

    @staticmethod
    def device(*args):
        return args


@pytest.fixture
def fake_upload(monkeypatch):
    _Torch.uploads = 0
    monkeypatch.setattr(_host, "torch", _Torch)
    _host.invalidate()
    yield _Torch
    _host.invalidate()


def test_one_upload_per_buffer_and_identity_hits(fake_upload):
    q = np.arange(64, dtype=np.int8).reshape(8, 8)
    t = _host.resident(q, 0)
    assert fake_upload.uploads == 1
    assert _host.resident(q, 0) is t           # same object: found by identity
    v = q[:]                                    # another object over the same buffer
    assert _host.resident(v, 0) is t
    assert fake_upload.uploads == 1
    assert _host.resident(q, 1) is not t        # another device: its own copy
    assert _host.resident(q, 0) is t            # and the first one is still there
    assert fake_upload.uploads == 2


def test_invalidate_after_in_place_change(fake_upload):
    q = np.zeros((4, 16), dtype=np.int8)
    t = _host.resident(q, 0)
    q[0, 0] = 7
    _host.invalidate(q)
    t2 = _host.resident(q, 0)
    assert t2 is not t and t2.a[0, 0] == 7
    assert _host.resident(q, 0) is t2


def test_copy_dropped_when_the_array_is_freed(fake_upload):
    q = np.ones((32, 32), dtype=np.int8)
    _host.resident(q, 0)
    before = _host.cached_bytes()
    ident = id(q)
    del q
    gc.collect()
    assert _host.cached_bytes() == before - 32 * 32
    assert ident not in _host._fast
