"""Host logic of the hot-expert replica plan (CPU): the slot map it hands the
exchange, and the rank loads it reaches on a skewed (Zipf) expert load."""

import numpy as np
import pytest

from nki_moe_b200.ep_peer import plan_expert_replicas


def _zipf_load(E=128, tokens=16384, top_k=8, s=1.2, seed=0):
    rng = np.random.default_rng(seed)
    p = 1.0 / np.arange(1, E + 1) ** s
    p /= p.sum()
    load = np.zeros(E)
    load[rng.permutation(E)] = p * tokens * top_k
    return np.minimum(load, tokens)  # an expert takes a token at most once


def _rank_loads(load, P, per_rank, holders):
    rl = np.zeros(P)
    for e, h in enumerate(holders):
        for v in h:
            rl[v // per_rank] += load[e] / len(h)
    return rl


@pytest.mark.parametrize("P", [1, 2, 4, 8])
@pytest.mark.parametrize("extra", [0, 1, 2, 4])
def test_plan_slot_map_is_consistent(P, extra):
    E = 128
    load = _zipf_load(E)
    slot_experts, holders = plan_expert_replicas(load, P, extra)
    el, per_rank = E // P, E // P + extra
    assert len(slot_experts) == P and all(len(se) == per_rank for se in slot_experts)
    assert len(holders) == E
    for e, h in enumerate(holders):
        assert h[0] == (e // el) * per_rank + e % el  # the owner's own slot first
        ranks = [v // per_rank for v in h]
        assert len(set(ranks)) == len(ranks)  # at most one copy per rank
        for v in h:
            assert 0 <= v < P * per_rank and slot_experts[v // per_rank][v % per_rank] == e
    for r in range(P):  # the own experts keep their slots
        assert slot_experts[r][:el] == list(range(r * el, (r + 1) * el))
    if extra == 0 or P == 1:
        assert all(len(h) == 1 for h in holders)


@pytest.mark.parametrize("P,extra,bound", [(2, 2, 1.05), (4, 2, 1.10), (8, 2, 1.10), (8, 4, 1.03)])
def test_plan_balances_a_zipf_load(P, extra, bound):
    E = 128
    load = _zipf_load(E)
    _, h0 = plan_expert_replicas(load, P, 0)
    slot_experts, holders = plan_expert_replicas(load, P, extra)
    before = _rank_loads(load, P, E // P, h0)
    after = _rank_loads(load, P, E // P + extra, holders)
    assert np.isclose(after.sum(), load.sum())  # every row still goes somewhere
    assert after.max() <= before.max()
    assert after.max() / after.mean() < bound, (before.max() / before.mean(), after.max() / after.mean())


def test_plan_is_deterministic_and_leaves_a_uniform_load_alone():
    load = _zipf_load(seed=5)
    assert plan_expert_replicas(load, 8, 3) == plan_expert_replicas(list(load), 8, 3)
    _, holders = plan_expert_replicas(np.full(128, 64.0), 8, 4)
    assert all(len(h) == 1 for h in holders)  # nothing to gain: no copies


def test_plan_rejects_bad_shapes():
    with pytest.raises(ValueError):
        plan_expert_replicas(np.ones(10), 4, 1)
    with pytest.raises(ValueError):
        plan_expert_replicas(np.ones(8), 4, -1)
