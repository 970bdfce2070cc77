"""Known-answer tests of the reference's allocator, run on the oracle and on the product.

Each scenario and its expected values come from the reference's own suite
(agentrl tests/test_paged_kv.py:15-74).  ``impl`` is either the oracle
restatement or the product allocator (C++ via libpkv_b200, host only).
"""

from __future__ import annotations

import pytest

from oracle.allocator import OracleAllocator


def _product(total, bs):
    from randomrepo_b200 import PagedKVAllocator

    return PagedKVAllocator(total_blocks=total, block_size_tokens=bs)


IMPLS = {"oracle": lambda total, bs: OracleAllocator(total, bs), "product": _product}


@pytest.fixture(params=sorted(IMPLS))
def make(request):
    return IMPLS[request.param]


def test_reserves_and_releases_blocks(make):  # test_paged_kv.py:15-27
    allocator = make(4, 2)
    first = allocator.reserve(sequence_id=7, token_count=3)
    assert first.physical_blocks == (0, 1)
    assert allocator.used_block_count == 2
    assert allocator.free_block_count == 2
    allocator.release(7)
    assert allocator.used_block_count == 0
    assert allocator.free_block_count == 4


def test_reuses_freed_blocks_deterministically(make):  # test_paged_kv.py:30-40
    allocator = make(4, 2)
    allocator.reserve(sequence_id=1, token_count=2)
    allocator.reserve(sequence_id=2, token_count=2)
    allocator.release(1)
    reused = allocator.reserve(sequence_id=3, token_count=2)
    assert reused.physical_blocks == (0,)
    assert allocator.block_reuse_count == 1


def test_grows_across_block_boundaries(make):  # test_paged_kv.py:43-51
    allocator = make(5, 2)
    allocator.reserve(sequence_id=4, token_count=2)
    grown = allocator.append_tokens(sequence_id=4, token_count=3)
    assert grown.token_count == 5
    assert grown.physical_blocks == (0, 1, 2)
    assert allocator.logical_to_physical(4, 2) == 2


def test_tracks_high_watermark_and_pressure(make):  # test_paged_kv.py:54-66
    allocator = make(4, 2)
    allocator.reserve(sequence_id=1, token_count=4)
    allocator.reserve(sequence_id=2, token_count=1)
    allocator.release(2)
    metrics = allocator.metrics()
    assert metrics["paged_kv_used_block_count"] == 2.0
    assert metrics["paged_kv_free_block_count"] == 2.0
    assert metrics["paged_kv_allocator_occupancy"] == 0.5
    assert metrics["paged_kv_max_blocks_in_use"] == 3.0


def test_raises_when_out_of_blocks(make):  # test_paged_kv.py:69-74
    allocator = make(1, 2)
    allocator.reserve(sequence_id=1, token_count=2)
    with pytest.raises(RuntimeError, match="out of free blocks"):
        allocator.append_tokens(sequence_id=1, token_count=1)


@pytest.mark.parametrize("total,bs,msg", [(0, 2, "total_blocks must be > 0."), (4, 0, "block_size_tokens must be > 0.")])
def test_constructor_validation(make, total, bs, msg):  # paged_kv.py:35-38
    with pytest.raises(ValueError) as err:
        make(total, bs)
    assert str(err.value) == msg


def test_error_types_and_messages(make):  # paged_kv.py:81-84,96-99,117-118,125-126
    allocator = make(8, 2)
    allocator.reserve(1, 3)
    with pytest.raises(ValueError, match="sequence_id 1 is already allocated."):
        allocator.reserve(1, 1)
    with pytest.raises(ValueError, match="token_count must be >= 0."):
        allocator.reserve(2, -1)
    with pytest.raises(ValueError, match="token_count must be >= 0."):
        allocator.append_tokens(1, -1)
    with pytest.raises(KeyError) as err:
        allocator.append_tokens(99, 1)
    assert str(err.value) == "'Unknown sequence_id 99.'"
    with pytest.raises(KeyError):
        allocator.release(99)
    with pytest.raises(ValueError, match="logical_block_index must be >= 0."):
        allocator.logical_to_physical(1, -1)
    with pytest.raises(KeyError) as err:
        allocator.logical_to_physical(99, 0)
    assert str(err.value) == "99"
    with pytest.raises(IndexError):
        allocator.logical_to_physical(1, 5)
    with pytest.raises(KeyError):
        allocator.view(99)
    assert allocator.has_sequence(1) and not allocator.has_sequence(99)


def test_zero_token_sequences(make):  # paged_kv.py:100-101,169-171
    allocator = make(4, 16)
    view = allocator.reserve(3, 0)
    assert view.physical_blocks == () and view.logical_block_count == 0
    assert allocator.append_tokens(3, 0).physical_blocks == ()
    assert allocator.append_tokens(3, 1).physical_blocks == (0,)
    assert allocator.metrics()["paged_kv_resident_sequences"] == 1.0
