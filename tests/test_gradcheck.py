"""Finite-difference gradient checks (float64, CPU) through the graph runtime
and this package's own module compositions (reference: the autograd
`numerical_grad` checks, autograd/tests.rs)."""
import pytest
import torch
from torch.autograd import gradcheck

from flodl_b200.graph import FlowBuilder, MergeOp, SoftmaxRouter
from flodl_b200.nn import GELU, LayerNorm, Linear, RMSNorm, Tanh
from flodl_b200.nn import loss as L


def _double(m):
    for p in m.parameters():
        p.data = p.data.double()
    return m


def _check(fn, *shapes):
    torch.manual_seed(0)
    xs = [torch.randn(*s, dtype=torch.float64, requires_grad=True) for s in shapes]
    assert gradcheck(fn, xs, eps=1e-6, atol=1e-5, rtol=1e-4)


def test_graph_residual_split_merge():
    g = _double(FlowBuilder.from_(Linear(5, 6)).through(Tanh()).also(Linear(6, 6))
                .split([Linear(6, 4), Linear(6, 4)]).merge(MergeOp.MEAN).build())
    _check(lambda x: g(x), (3, 5))


def test_graph_loop_bptt():
    body = Linear(4, 4)
    g = _double(FlowBuilder.from_(Linear(3, 4)).loop_body(body).for_n(3).through(Tanh()).build())
    _check(lambda x: g(x), (2, 3))


def test_graph_soft_gate():
    g = _double(FlowBuilder.new().gate(SoftmaxRouter(4, 2), [Linear(4, 4), Linear(4, 4)]).build())
    _check(lambda x: g(x), (3, 4))


def test_norms():
    ln, rms = _double(LayerNorm(7)), _double(RMSNorm(7))
    _check(lambda x: ln(x), (3, 7))
    _check(lambda x: rms(x), (3, 7))


@pytest.mark.parametrize("name", ["mse_loss", "l1_loss", "smooth_l1_loss", "bce_with_logits_loss",
                                  "kl_div_loss", "poisson_nll_loss"])
def test_losses(name):
    fn = getattr(L, name)
    t = torch.rand(4, 3, dtype=torch.float64)
    if name == "kl_div_loss":
        _check(lambda x: fn(torch.log_softmax(x, -1), torch.softmax(t, -1)), (4, 3))
    else:
        _check(lambda x: fn(x, t), (4, 3))


def test_cross_entropy_with_label_smoothing_and_focal():
    y = torch.tensor([0, 2, 1, 2])
    _check(lambda x: L.cross_entropy_loss(x, y, label_smoothing=0.1), (4, 3))
    _check(lambda x: L.focal_loss(x, y), (4, 3))


def test_gelu_module():
    act = GELU()
    _check(lambda x: act(x), (5, 4))


def test_focal_reduces_to_scaled_cross_entropy_at_gamma_zero():
    x = torch.randn(6, 4, dtype=torch.float64)
    y = torch.tensor([0, 3, 1, 2, 2, 0])
    torch.testing.assert_close(L.focal_loss(x, y, alpha=0.25, gamma=0.0),
                               0.25 * torch.nn.functional.cross_entropy(x, y))
    t = torch.rand(4, 3, dtype=torch.float64)
    _check(lambda z: L.focal_loss(z, t), (4, 3))  # binary form
