"""Graph-captured multi-layer driver (qmesh_b200.driver): per-(layer, width)
graph replays equal direct slice calls bit for bit at exact and bucketed widths
and on the eager path; a round graph serves every layer once its cell is
published; a layer whose inputs never arrive times out (bounded device wait),
is reported, and the next round on the same context is correct."""

import pytest
import torch

import helpers as H

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def setup(cuda_ready):
    from qmesh_b200.arena import Arena
    dev = cuda_ready
    layers = [H.small_layer(40 + i, 8, inter=256) for i in range(3)]
    ar = Arena(dev, 3, 8, 0, 256, layout="tc")
    for li, layer in enumerate(layers):
        ar.load_layer(li, layer)
    return dev, ar


def _inputs(rows, seed, dev):
    ids, tw = H.random_routing(rows, 8, seed)
    _, q, inv = H.activations(rows, seed)
    return q.to(dev), inv.to(dev), ids.to(dev), tw.to(dev)


def _direct(ar, li, q, inv, ids, tw):
    from qmesh_b200.expert_slice import expert_slice
    return expert_slice(ar, li, q, ids, tw, x_scale=inv)


@pytest.mark.parametrize("rows", [6, 5, 16, 23])
def test_graph_replay_matches_direct_call(setup, rows):
    from qmesh_b200.driver import LayerDriver
    dev, ar = setup
    drv = LayerDriver(ar)
    for step, li in enumerate([0, 2, 0, 1]):
        q, inv, ids, tw = _inputs(rows, 100 * rows + step, dev)
        got = drv.step(li, q, inv, ids, tw).clone()
        want = _direct(ar, li, q, inv, ids, tw)
        torch.cuda.synchronize()
        assert torch.equal(got, want), f"rows {rows} layer {li} step {step}"
    assert (rows > 16) == (len(drv.graphs) == 0)


def test_round_graph_and_a_lost_layer(setup):
    from qmesh_b200.driver import LayerDriver
    dev, ar = setup
    drv = LayerDriver(ar, spin_timeout_ms=50)
    drv.capture_round(6)
    for rnd, lost in ((1, None), (2, 1), (3, None)):
        ins = [_inputs(6, 1000 * rnd + li, dev) for li in range(3)]
        drv.reset_status()
        for li in range(3):
            if li != lost:
                drv.stage_layer(li, *ins[li], seq=rnd)
        drv.replay_round(rnd)
        torch.cuda.synchronize()
        assert drv.round_timeouts() == (lost is not None), f"round {rnd}"
        for li in range(3):
            if li == lost:
                continue
            want = _direct(ar, li, *ins[li])
            torch.cuda.synchronize()
            assert torch.equal(drv.slots[li].out, want), f"round {rnd} layer {li}"
