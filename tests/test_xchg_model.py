"""The fused combine's protocol (model in tests/xchg_model.py) under random
interleavings: the output rank takes every sender's words of every call exactly
once and never words of another call, a sender never overwrites words still
unread, and no schedule deadlocks; senders run at most one call ahead."""

import pytest

import xchg_model as XM


@pytest.mark.parametrize("world,dst", [(2, 0), (2, 1), (4, 0), (8, 3)])
def test_protocol_delivers_every_call_once(world, dst):
    for seed in range(40):
        u = XM.run(world, dst, calls=12, seed=seed)
        want = [(i, s) for i in range(1, 13) for s in range(world) if s != dst]
        assert [(i, s) for i, s, _ in u.got] == want
        for i, s, d in u.got:
            assert d == (XM.Unit.data(i, s, 0), XM.Unit.data(i, s, 1))


def test_model_catches_a_sender_that_skips_the_ack_wait():
    caught = 0
    for seed in range(40):
        try:
            XM.run(2, 0, calls=12, seed=seed, ack_wait=False)
        except AssertionError:
            caught += 1
    assert caught > 0
