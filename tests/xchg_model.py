"""Interleaving model of the fused rank combine's protocol for one finalize
unit (qmesh-afd-tp3_b200/csrc/qx_decode_tc.cu finalize_unit; buffer layout in
csrc/qx_xchg.cuh): test infrastructure only.

A sender's call i: wait until its ack >= i - 2, store its two receive words of
parity i & 1 (each {data, i}, two separate stores), bump its call counter. The
output rank's call i: for each sender, poll both words of parity i & 1 until
both carry i, read their data; then store an ack of i into each sender's buffer
(one store per sender). Every step is atomic; the scheduler interleaves the
ranks' steps at random.
"""

from __future__ import annotations

import random


class Unit:
    def __init__(self, world: int, dst: int):
        self.world, self.dst = world, dst
        self.senders = [r for r in range(world) if r != dst]
        self.words = {(p, r, w): (0, 0) for p in (0, 1) for r in self.senders for w in (0, 1)}  # (flag, data)
        self.ack = {r: 0 for r in self.senders}         # in the sender's buffer, written by the output rank
        self.read_upto = {r: 0 for r in self.senders}   # calls the output rank has fully read from r
        self.sent = {r: 0 for r in self.senders}        # sender progress: calls whose words are stored
        self.got = []                                   # (call, sender, data) read by the output rank

    @staticmethod
    def data(call: int, sender: int, word: int) -> int:
        return call * 1000 + sender * 10 + word


def run(world: int, dst: int, calls: int, seed: int, max_steps: int = 200000, ack_wait: bool = True) -> Unit:
    """Run `calls` calls of every rank under one random schedule; `ack_wait=False`
    plants a mistake (senders skip the acknowledgement wait)."""
    rng = random.Random(seed)
    u = Unit(world, dst)
    # per-rank program counters: (call, phase, index)
    pc = {r: [1, 0, 0] for r in range(world)}
    pending = {}                                        # output rank: words seen for the current call
    for _ in range(max_steps):
        live = [r for r in range(world) if pc[r][0] <= calls]
        if not live:
            return u
        r = rng.choice(live)
        i, phase, idx = pc[r]
        p = i & 1
        if r != dst:
            if phase == 0:                              # wait for the ack of this parity's last use
                if u.ack[r] >= i - 2 or not ack_wait:
                    pc[r][1] = 1
            elif phase in (1, 2):                       # the two word stores
                w = phase - 1
                assert u.read_upto[r] >= i - 2, "a sender overwrote words the output rank had not read"
                u.words[(p, r, w)] = (i, Unit.data(i, r, w))
                pc[r][1] += 1
                if w == 1:
                    u.sent[r] = i
                    pc[r] = [i + 1, 0, 0]
        else:
            if phase == 0:                              # poll sender idx's two words
                s = u.senders[idx]
                a, b = u.words[(p, s, 0)], u.words[(p, s, 1)]
                if a[0] == i and b[0] == i:
                    assert a[1] == Unit.data(i, s, 0) and b[1] == Unit.data(i, s, 1)
                    pending[s] = (a[1], b[1])
                    u.read_upto[s] = i
                    if idx + 1 < len(u.senders):
                        pc[r][2] += 1
                    else:
                        pc[r][1], pc[r][2] = 1, 0
                else:                                   # still the parity's previous call (or nothing yet)
                    assert a[0] in (0, i - 2, i) and b[0] in (0, i - 2, i)
            else:                                       # one ack store per sender
                s = u.senders[idx]
                u.ack[s] = i
                u.got.append((i, s, pending[s]))
                if idx + 1 < len(u.senders):
                    pc[r][2] += 1
                else:
                    pending.clear()
                    pc[r] = [i + 1, 0, 0]
    raise AssertionError("no progress: the protocol deadlocked")
