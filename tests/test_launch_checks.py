"""Host-side launch validation (OMNI_DEVICE_CHECKS) and the pinned staging ring."""
import pytest
import torch

from sglang_omni_b200.ops import _check
from sglang_omni_b200.utils.staging import PinnedRing


def test_check_paged_rejects_out_of_pool_pages():
    bt = torch.tensor([[1, 2, 0], [3, 99, 0]], dtype=torch.int32)
    kl = torch.tensor([100, 70], dtype=torch.int32)
    _check.check_paged("t", bt[:1], kl[:1], 8)
    with pytest.raises(_check.LaunchCheckError, match="block_table\\[1\\] = 99"):
        _check.check_paged("t", bt, kl, 8)


def test_check_paged_rejects_context_beyond_table():
    bt = torch.tensor([[1, 2]], dtype=torch.int32)
    with pytest.raises(_check.LaunchCheckError, match="needs 3 pages"):
        _check.check_paged("t", bt, torch.tensor([129], dtype=torch.int32), 8)


def test_check_tiles_and_ranges():
    cu = torch.tensor([0, 3, 70], dtype=torch.int32)
    _check.check_tiles("t", torch.tensor([0, 1, 1], dtype=torch.int32), torch.tensor([0, 0, 64], dtype=torch.int32), cu)
    with pytest.raises(_check.LaunchCheckError):
        _check.check_tiles("t", torch.tensor([0, 1], dtype=torch.int32), torch.tensor([5, 0], dtype=torch.int32), cu)
    _check.check_range("t", "slots", torch.tensor([-1, 0, 127]), 0, 128, allow=-1)
    with pytest.raises(_check.LaunchCheckError, match="slots\\[1\\] = 128"):
        _check.check_range("t", "slots", torch.tensor([-1, 128]), 0, 128, allow=-1)
    with pytest.raises(_check.LaunchCheckError):
        _check.check_offsets("t", torch.tensor([0, 5, 3], dtype=torch.int32), 10)


def test_pinned_ring_round_robin():
    r = PinnedRing(8, torch.int32, n=2, cuda=False)
    a = r.next()
    a.fill_(1)
    dst = torch.zeros(8, dtype=torch.int32)
    r.upload(dst, 4)
    assert dst.tolist() == [1, 1, 1, 1, 0, 0, 0, 0]
    b = r.next()
    assert b.data_ptr() != a.data_ptr()
    assert r.next().data_ptr() == a.data_ptr()
