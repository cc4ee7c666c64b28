"""Optimizer math and state files (reference: flodl/src/nn/optim/*.rs tests)."""
import io

import pytest
import torch

from flodl_b200.optim import (SGD, Adagrad, Adam, AdamW, CosineScheduler, CyclicLR, ExponentialLR,
                              MultiStepLR, NAdam, OneCycleLR, PlateauScheduler, RAdam, RMSprop,
                              StepDecay, WarmupScheduler, migrate_optim_state_file)

CASES = [
    (lambda p: SGD(p, 0.1, momentum=0.9, weight_decay=1e-3), lambda p: torch.optim.SGD(p, 0.1, momentum=0.9, weight_decay=1e-3)),
    (lambda p: SGD(p, 0.1, momentum=0.9, nesterov=True), lambda p: torch.optim.SGD(p, 0.1, momentum=0.9, nesterov=True)),
    (lambda p: Adam(p, 1e-2, weight_decay=1e-2), lambda p: torch.optim.Adam(p, 1e-2, weight_decay=1e-2)),
    (lambda p: AdamW(p, 1e-2, 0.1), lambda p: torch.optim.AdamW(p, 1e-2, weight_decay=0.1)),
    (lambda p: RMSprop(p, 1e-2, momentum=0.5), lambda p: torch.optim.RMSprop(p, 1e-2, momentum=0.5)),
    (lambda p: Adagrad(p, 1e-1), lambda p: torch.optim.Adagrad(p, 1e-1)),
    (lambda p: RAdam(p, 1e-2), lambda p: torch.optim.RAdam(p, 1e-2)),
    (lambda p: NAdam(p, 1e-2), lambda p: torch.optim.NAdam(p, 1e-2)),
]


@pytest.mark.parametrize("mk,mk_ref", CASES)
def test_matches_torch(mk, mk_ref):
    torch.manual_seed(0)
    w = torch.randn(5, 3)
    p1 = torch.nn.Parameter(w.clone())
    p2 = torch.nn.Parameter(w.clone())
    o1, o2 = mk([p1]), mk_ref([p2])
    for i in range(8):
        g = torch.randn(5, 3)
        p1.grad = g.clone()
        p2.grad = g.clone()
        o1.step()
        o2.step()
    torch.testing.assert_close(p1.detach(), p2.detach(), rtol=1e-5, atol=1e-6)


def test_lr_and_groups():
    a, b = torch.nn.Parameter(torch.ones(2)), torch.nn.Parameter(torch.ones(2))
    o = SGD([{"params": [a], "lr": 0.1}, {"params": [b], "lr": 0.5}], 0.1)
    assert o.lr() == 0.1
    o.set_group_lr(1, 0.2)
    o.scale_lr(0.5)
    assert [g.lr for g in o.groups] == [0.05, 0.1]
    a.grad = torch.ones(2)
    b.grad = torch.ones(2)
    o.step()
    torch.testing.assert_close(a.detach(), torch.full((2,), 0.95))
    torch.testing.assert_close(b.detach(), torch.full((2,), 0.9))


@pytest.mark.parametrize("cls", [Adam, AdamW, SGD, RMSprop, Adagrad])
def test_state_file_roundtrip(tmp_path, cls):
    torch.manual_seed(0)
    p = torch.nn.Parameter(torch.randn(4))
    kw = {"momentum": 0.9} if cls is SGD else {}
    o = cls([p], 0.01, **kw)
    for _ in range(3):
        p.grad = torch.randn(4)
        o.step()
    path = str(tmp_path / "o.optim")
    o.save_state_file(path)
    raw = open(path, "rb").read()
    assert raw[:4] == b"FDLO"
    p2 = torch.nn.Parameter(p.detach().clone())
    o2 = cls([p2], 0.5, **kw)
    o2.load_state_file(path)
    assert o2.lr() == pytest.approx(0.01)
    g = torch.randn(4)
    p.grad, p2.grad = g.clone(), g.clone()
    o.step()
    o2.step()
    torch.testing.assert_close(p.detach(), p2.detach())
    with pytest.raises(ValueError, match="written by"):
        other = (SGD if cls is not SGD else Adam)([p2], 0.1)
        other.load_state_file(path)


def test_reset_state_and_migrate(tmp_path):
    p = torch.nn.Parameter(torch.randn(3))
    o = Adam([p], 0.1)
    p.grad = torch.ones(3)
    o.step()
    o.reset_state()
    assert not o.state
    path = str(tmp_path / "old.optim")
    buf = io.BytesIO()
    o.save_state(buf)
    open(path, "wb").write(buf.getvalue())
    migrate_optim_state_file(path, path + ".new", "Adam")
    o.load_state_file(path + ".new")


def test_schedulers():
    assert StepDecay(1.0, 10, 0.5).lr(25) == 0.25
    c = CosineScheduler(1.0, 0.0, 100)
    assert c.lr(0) == 1.0 and abs(c.lr(100)) < 1e-12 and abs(c.lr(50) - 0.5) < 1e-12
    w = WarmupScheduler(c, 1.0, 10)
    assert w.lr(0) == pytest.approx(0.1) and w.lr(10) == 1.0
    assert ExponentialLR(1.0, 0.9).lr(2) == pytest.approx(0.81)
    assert MultiStepLR(1.0, [5, 10], 0.1).lr(10) == pytest.approx(0.01)
    oc = OneCycleLR(1.0, 100)
    assert oc.lr(0) == pytest.approx(0.04) and oc.lr(30) == pytest.approx(1.0)
    cy = CyclicLR(0.1, 1.0, 10)
    assert cy.lr(10) == pytest.approx(1.0) and cy.lr(20) == pytest.approx(0.1)
    pl = PlateauScheduler(1.0, 2, 0.5, 0.1)
    for m in [1.0, 1.0, 1.0]:
        lr = pl.observe(m)
    assert lr == 0.5
    with pytest.raises(ValueError):
        StepDecay(1.0, 0, 0.5)


def test_adopted_arena_gets_fused_state():
    """An arena handed over by the cluster trainer (parameters moved into a
    peer-shared region) gets the optimizer's fused state like one the
    optimizer built itself."""
    from flodl_b200.optim import SGD, AdamW
    from flodl_b200.utils.arena import ParamArena

    ps = [torch.nn.Parameter(torch.randn(10, 3)), torch.nn.Parameter(torch.randn(7))]
    sgd = SGD(ps, lr=0.1, momentum=0.9)
    g = sgd.groups[0]
    arena = ParamArena(g.params)
    sgd.adopt_arena(g, arena)
    assert g.arena is arena and g.buf is not None and g.buf.numel() == arena.numel
    buf = g.buf
    sgd.adopt_arena(g, ParamArena(g.params))  # a later move keeps the state
    assert g.buf is buf
    adam = AdamW(ps, lr=1e-3)
    ga = adam.groups[0]
    adam.adopt_arena(ga, arena)
    assert ga.m.numel() == arena.numel and ga.v.numel() == arena.numel
