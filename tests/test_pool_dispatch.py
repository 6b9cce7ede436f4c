"""The engine pool's shard dispatcher on fake host workers (no GPU).

The pool deals pages round-robin to one worker thread per device and gathers
the results in page order; a worker that misses the call's deadline has its
pages dealt again to the workers that answered, and one that fails with a
device error is left out of the call.  Here the workers are host threads that
sleep or raise on command, so stalls and failures are made on the host, with
no device involved.
"""

import pytest

import ppocr_b200 as P


def test_round_robin_in_page_order():
    owner, values = P.selftest_dispatch(4, 10, timeout_ms=2000)
    assert values == [i * 10 for i in range(10)]
    assert owner == [i % 4 for i in range(10)]


def test_no_deadline_waits_for_slow_worker():
    owner, values = P.selftest_dispatch(3, 7, stall=[1], stall_ms=150, timeout_ms=0)
    assert values == [i * 10 for i in range(7)]
    assert owner == [i % 3 for i in range(7)]


def test_late_worker_shard_is_requeued():
    owner, values = P.selftest_dispatch(4, 13, stall=[1], stall_ms=600, timeout_ms=100)
    assert values == [i * 10 for i in range(13)]
    assert 1 not in owner
    assert set(owner) == {0, 2, 3}
    # The first round's shards stay where they were dealt.
    for i in range(13):
        if i % 4 != 1:
            assert owner[i] == i % 4


def test_two_late_workers():
    owner, values = P.selftest_dispatch(5, 20, stall=[0, 3], stall_ms=500, timeout_ms=100)
    assert values == [i * 10 for i in range(20)]
    assert set(owner) <= {1, 2, 4}


def test_failed_worker_is_left_out():
    owner, values = P.selftest_dispatch(4, 9, fail=[0, 2], timeout_ms=2000)
    assert values == [i * 10 for i in range(9)]
    assert set(owner) <= {1, 3}


def test_failure_and_stall_together():
    owner, values = P.selftest_dispatch(3, 8, stall=[0], fail=[1], stall_ms=500, timeout_ms=100)
    assert values == [i * 10 for i in range(8)]
    assert owner == [2] * 8


def test_every_worker_late_is_a_gpu_error():
    with pytest.raises(P.GpuError, match="no device answered"):
        P.selftest_dispatch(2, 4, stall=[0, 1], stall_ms=400, timeout_ms=50)


def test_every_worker_failed_reports_the_device_error():
    with pytest.raises(P.GpuError, match="fake device"):
        P.selftest_dispatch(3, 5, fail=[0, 1, 2], timeout_ms=1000)


def test_more_workers_than_items_and_empty_calls():
    owner, values = P.selftest_dispatch(8, 3, timeout_ms=1000)
    assert values == [0, 10, 20] and owner == [0, 1, 2]
    assert P.selftest_dispatch(4, 0) == ([], [])


def test_invalid_worker_counts():
    with pytest.raises(P.InvalidInput):
        P.selftest_dispatch(0, 3)
    with pytest.raises(P.InvalidInput):
        P.selftest_dispatch(33, 3)
