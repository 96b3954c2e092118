"""Expert placement with replicated hot experts (mail_b200.ep.ExpertPlacement):
the virtual expert space the exchange runs in, on CPU."""
import numpy as np
import pytest
import torch

from mail_b200.ep import ExpertPlacement, hot_experts


@pytest.mark.parametrize("E,W,rep", [(8, 2, ()), (8, 2, (5,)), (64, 8, (3, 17, 60)), (6, 3, (0, 1, 2, 3, 4, 5))])
def test_virtual_ids(E, W, rep):
    EL = E // W
    for r in range(W):
        p = ExpertPlacement(E, W, r, rep)
        ELv = EL + len(rep)
        assert p.EL_virtual == ELv and p.E_virtual == W * ELv
        ids = torch.tensor([list(range(E)) + [-1, E, E + 7]], dtype=torch.int32)
        v = p.remap(ids)[0].tolist() if rep else None
        for e in range(E):
            if not rep:
                continue
            if e in rep:  # served here, as this rank's replica j
                assert v[e] == r * ELv + EL + list(rep).index(e)
            else:  # served by its owner, at its local index
                owner = e // EL
                assert v[e] == owner * ELv + e - owner * EL
        if rep:
            assert v[E:] == [-1, -1, -1]
            # every virtual id is owned by exactly one rank's range, and no two
            # global ids share one
            assert len(set(v[:E])) == E


def test_no_replicas_is_the_identity():
    p = ExpertPlacement(8, 2, 1)
    ids = torch.tensor([[0, 7], [-1, 3]], dtype=torch.int32)
    assert p.remap(ids) is ids and p.E_virtual == 8 and p.EL_virtual == 4


def test_local_weights_append_replicas_in_order():
    E, W, H, I = 8, 2, 16, 8
    rng = np.random.default_rng(0)
    w13 = torch.from_numpy(rng.standard_normal((E, H, 2 * I), dtype=np.float32))
    w2 = torch.from_numpy(rng.standard_normal((E, I, H), dtype=np.float32))
    p = ExpertPlacement(E, W, 1, (6, 0))
    a13, a2, _ = p.local_weights(w13[4:], w2[4:], None, ([6, 0], w13[[6, 0]], w2[[6, 0]]))
    assert a13.shape == (6, H, 2 * I) and a2.shape == (6, I, H)
    assert torch.equal(a13[:4], w13[4:]) and torch.equal(a13[4], w13[6]) and torch.equal(a13[5], w13[0])
    assert a13.transpose(1, 2).is_contiguous()  # K-major storage
    with pytest.raises(ValueError):
        p.local_weights(w13[4:], w2[4:], None, ([0, 6], w13[[0, 6]], w2[[0, 6]]))  # wrong order
    with pytest.raises(ValueError):
        ExpertPlacement(E, W, 0, (3, 3))


def test_hot_experts_picks_the_largest_counts():
    assert hot_experts(torch.tensor([5, 9, 9, 0, 12]), 3) == [4, 1, 2]


def _max_load(C, rep):
    W, E = C.shape
    EL = E // W
    load = np.zeros(W, np.int64)
    for e in range(E):
        if e in rep:
            load += C[:, e]
        else:
            load[e // EL] += C[:, e].sum()
    return int(load.max())


def test_plan_replicas_lowers_the_largest_load_greedily():
    from mail_b200.ep import plan_replicas
    rng = np.random.default_rng(3)
    for W, E in ((2, 8), (4, 16), (8, 64)):
        C = rng.integers(0, 50, size=(W, E))
        C[:, 5] += 2000  # a hot expert, owned by rank 5 // (E // W)
        rep = plan_replicas(torch.from_numpy(C), 4)
        assert 5 in rep
        base = _max_load(C, [])
        prev = base
        for i in range(len(rep)):  # each added replica lowers the largest load, and is the best single choice
            m = _max_load(C, rep[:i + 1])
            assert m < prev
            others = [e for e in range(E) if e not in rep[:i]]
            assert m == min(_max_load(C, rep[:i] + [e]) for e in others)
            prev = m


def test_plan_replicas_stops_when_balanced():
    from mail_b200.ep import plan_replicas
    C = torch.full((4, 8), 10)
    assert plan_replicas(C, 3) == []
