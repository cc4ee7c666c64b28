"""Fused whole-model training ops against the composed fp32 PyTorch path.

The CUDA ``loss()`` of TransformerLM and BertForMaskedLM runs one fused
autograd function built from the sm_100a kernels (bf16 operands, f32
accumulation). The same module on the CPU composes plain PyTorch ops in fp32;
that is the oracle here: same weights, same batch, loss and every parameter
gradient compared (gradients by relative Frobenius error, since bf16 operands
make single elements noisy).
"""
import copy

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


def _compare(model_gpu, model_cpu, loss_gpu, loss_cpu, loss_tol, grad_tol):
    assert abs(loss_gpu.item() - loss_cpu.item()) < loss_tol, (loss_gpu.item(), loss_cpu.item())
    gp = dict(model_gpu.named_parameters())
    worst = []
    for name, pc in model_cpu.named_parameters():
        pg = gp[name]
        if pc.grad is None:
            assert pg.grad is None or pg.grad.abs().max().item() == 0.0, name
            continue
        assert pg.grad is not None, f"{name}: no gradient from the fused op"
        r = _rel(pg.grad.cpu(), pc.grad)
        worst.append((r, name))
        assert r < grad_tol, f"{name}: relative gradient error {r:.3e}"
    return max(worst)


@pytest.mark.parametrize("S,causal", [(128, True), (200, True), (96, False)])
def test_transformer_lm_fused_matches_fp32(S, causal):
    from flodl_b200.models import TransformerLM

    torch.manual_seed(0)
    cpu = TransformerLM(vocab_size=256, d_model=256, n_layers=2, n_heads=4, d_ff=1024,
                        max_seq=256, causal=causal)
    gpu = copy.deepcopy(cpu)
    gpu.move_to_device(torch.device("cuda"))
    ids = torch.randint(0, 256, (3, S))
    tgt = torch.randint(0, 256, (3, S))
    lc = cpu.loss(ids, tgt)
    lc.backward()
    lg = gpu.loss(ids.cuda(), tgt.cuda())
    lg.backward()
    torch.cuda.synchronize()
    _compare(gpu, cpu, lg, lc, loss_tol=2e-2, grad_tol=4e-2)


def test_transformer_lm_bench_width_matches_fp32():
    """The benchmarked LM width (6 layers, d512, 8 heads, d_ff 2048, S 256)
    against the fp32 CPU model: loss and every parameter gradient."""
    from flodl_b200.models import TransformerLM

    torch.manual_seed(0)
    cpu = TransformerLM(vocab_size=256, d_model=512, n_layers=6, n_heads=8, d_ff=2048,
                        max_seq=256, causal=True)
    gpu = copy.deepcopy(cpu)
    gpu.move_to_device(torch.device("cuda"))
    ids = torch.randint(0, 256, (4, 256))
    tgt = torch.randint(0, 256, (4, 256))
    lc = cpu.loss(ids, tgt)
    lc.backward()
    lg = gpu.loss(ids.cuda(), tgt.cuda())
    lg.backward()
    torch.cuda.synchronize()
    _compare(gpu, cpu, lg, lc, loss_tol=2e-2, grad_tol=5e-2)


def test_bert_mlm_fused_matches_fp32():
    from flodl_b200.models.bert import BertConfig, BertForMaskedLM

    torch.manual_seed(0)
    cfg = BertConfig(vocab_size=1000, hidden_size=256, num_hidden_layers=2,
                     num_attention_heads=4, intermediate_size=1024, max_position_embeddings=128)
    cpu = BertForMaskedLM(cfg)
    gpu = copy.deepcopy(cpu)
    gpu.move_to_device(torch.device("cuda"))
    B, S = 4, 128
    ids = torch.randint(0, 1000, (B, S))
    tt = torch.randint(0, 2, (B, S))
    labels = torch.full((B, S), -100)
    sel = torch.rand(B, S) < 0.15
    labels[sel] = ids[sel]
    mask = torch.ones(B, S, dtype=torch.int64)
    mask[1, 100:] = 0
    mask[3, 64:] = 0
    lc = cpu.loss(ids, labels, tt, mask)
    lc.backward()
    lg = gpu.loss(ids.cuda(), labels.cuda(), tt.cuda(), mask.cuda())
    lg.backward()
    torch.cuda.synchronize()
    _compare(gpu, cpu, lg, lc, loss_tol=3e-2, grad_tol=5e-2)
