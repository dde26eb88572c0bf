"""Host logic of the NVSwitch exchange on CPU (no GPU): multicast address
arithmetic, and NvlsGradientSum's contract with a stand-in exchange that
records what it is given."""
import types

import pytest
import torch

from xsimgs_b200 import exchange as E


def _handle(mc, bufs, rank=0):
    return types.SimpleNamespace(multicast_ptr=mc, buffer_ptrs=bufs, rank=rank)


class _Tensor:
    def __init__(self, ptr):
        self._p = ptr

    def data_ptr(self):
        return self._p


def test_multicast_address_follows_the_tensor_offset():
    # the tensor starts 256 bytes into rank 1's buffer: the multicast address too
    h = _handle(0x7000_0000, [0x1000_0000, 0x2000_0000], rank=1)
    assert E._multicast_address(_Tensor(0x2000_0100), h) == 0x7000_0100
    with pytest.raises(RuntimeError, match="multicast"):
        E._multicast_address(_Tensor(0x2000_0000), _handle(0, [0, 0x2000_0000], rank=1))
    with pytest.raises(RuntimeError, match="16-byte"):
        E._multicast_address(_Tensor(0x2000_0104), h)
    assert [E._pad4(n) for n in (0, 1, 4, 5, 11)] == [0, 4, 4, 8, 12]


class _FakeExchange:
    defer_views = False
    pending_views = None

    def __init__(self):
        self.calls = []

    def exchange(self, tensors, d=None, small=None):
        self.calls.append(([t.clone() for t in tensors], d, small))
        for t in tensors:
            t.mul_(2.0)  # as if a second rank held the same gradients
        return None, None


def test_gradient_sum_zero_fills_and_sums_in_place():
    a = torch.ones(3, requires_grad=True)
    b = torch.ones(2, 2, requires_grad=True)
    a.grad = torch.full((3,), 1.5)
    ex = _FakeExchange()
    red = E.NvlsGradientSum([a, b], ex)
    assert red.wait() == 1
    (sent, d, small), = ex.calls
    assert d is None and small is None
    assert torch.equal(sent[0], torch.full((3,), 1.5)) and torch.equal(sent[1], torch.zeros(2, 2))
    assert torch.equal(a.grad, torch.full((3,), 3.0)) and torch.equal(b.grad, torch.zeros(2, 2))
    assert ex.defer_views is False


def test_gradient_sum_with_sh_leaf_requires_the_views():
    means = torch.zeros(4, 3, requires_grad=True)
    sh = torch.zeros(4, 16, 3, requires_grad=True)
    ex = _FakeExchange()
    red = E.NvlsGradientSum([means], ex, sh_leaf=sh)
    assert ex.defer_views is True  # MultiViewSH leaves its view gradients to wait()
    with pytest.raises(RuntimeError, match="view gradients"):
        red.wait()
