"""Fused training step of a pre-LN transformer stack (embedding -> blocks ->
final LN -> vocabulary head -> softmax cross-entropy) as ONE autograd op.

Reference composition (per block, flodl's MultiheadAttention + Linear +
LayerNorm + GELU, flodl/src/nn/attention.rs, benchmarks/src/tier1/transformer.rs):

    x  = x + proj(attn(qkv(ln1(x))))
    x  = x + fc2(gelu(fc1(ln2(x))))

What is fused on sm_100a (per block, forward 7 kernels, backward 13):
* LayerNorm writes its output in bf16 straight into the next GEMM's operand.
* qkv/proj/fc1/fc2 GEMM epilogues add the bias, apply GELU (keeping GELU'
  of the pre-activation in bf16 for the backward), and add the f32 residual
  stream.
* Flash attention reads Q/K/V from the packed qkv buffer and writes [T, C].
* Backward: the fc2 dgrad epilogue multiplies by the stored GELU'; LayerNorm backward adds the
  skip-path gradient, writes the f32 residual gradient AND its bf16 copy, and
  accumulates dgamma/dbeta plus the bias gradient (column sum) of the Linear
  whose output fed that residual stream; weight gradients accumulate in f32
  directly into ``param.grad`` with split-K tcgen05 GEMMs.
* Cross-entropy computes the loss and the logits gradient in one pass; the
  upstream loss gradient is folded into the head GEMMs as a device scalar.

After each block's backward the gradient-ready listeners fire for its
parameters, which is where a DDP bucket reducer launches its fused
all-reduce+optimizer kernel on the communication stream while backward
continues on the compute stream.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch

from ._common import C, bf16_shadow, grad_buffer, grad_ready, splitk_for
from .attention import attn_bwd_packed, attn_fwd_packed


class WgradLane:
    """Weight-gradient GEMMs on a second stream. They read activations and
    output gradients that are already final and write only parameter
    gradients, so they run beside the input-gradient chain (whose kernels
    leave SMs idle in their last wave) instead of in series with it. Inputs
    read on the lane are kept referenced until ``join`` (after which the main
    stream is ordered behind the lane), so the caching allocator cannot hand
    their memory to a later kernel while the lane still reads it. Used as is
    inside CUDA-graph capture: the lane forks from and joins the capturing
    stream."""

    _streams = {}

    def __init__(self, dev):
        self.enabled = dev.type == "cuda"
        self.keep = []
        if self.enabled:
            self.main = torch.cuda.current_stream(dev)
            s = WgradLane._streams.get(dev.index)
            if s is None:
                s = WgradLane._streams[dev.index] = torch.cuda.Stream(dev)
            self.side = s

    def wgrad(self, dy16, x16, w, alpha_t=None):
        if not self.enabled:
            return _wgrad(dy16, x16, w, alpha_t)
        self.side.wait_stream(self.main)
        with torch.cuda.stream(self.side):
            _wgrad(dy16, x16, w, alpha_t)
        self.keep += [dy16, x16]

    def ready(self, params):
        """Gradient-ready listeners for ``params``: issued on the lane after it
        has caught up with the main stream, so a listener that orders its
        collective after the current stream sees every gradient complete."""
        if not self.enabled:
            for t in params:
                grad_ready(t)
            return
        self.side.wait_stream(self.main)
        with torch.cuda.stream(self.side):
            for t in params:
                grad_ready(t)

    def join(self):
        if self.enabled:
            self.main.wait_stream(self.side)
        self.keep = []


def _wgrad(dy16, x16, w, alpha_t=None):
    """w.grad += dy16^T @ x16 (f32, split-K accumulate)."""
    T, N = dy16.shape
    K = x16.shape[1]
    C().gemm(dy16, x16, grad_buffer(w), N, K, T, True, True, flags=C().EPI_ACCUMULATE,
             k_splits=splitk_for(N, K, T), alpha_t=alpha_t)


def _empty(shape, dtype, dev):
    return torch.empty(shape, dtype=dtype, device=dev)


class BlockParams:
    """Handles to one block's parameters (views of the module's tensors)."""

    __slots__ = ("ln1_w", "ln1_b", "wqkv", "bqkv", "wo", "bo", "ln2_w", "ln2_b", "w1", "b1",
                 "w2", "b2", "eps")

    def __init__(self, blk):
        self.ln1_w, self.ln1_b = blk.ln1.weight, blk.ln1.bias
        self.wqkv, self.bqkv = blk.qkv.weight, blk.qkv.bias
        self.wo, self.bo = blk.proj.weight, blk.proj.bias
        self.ln2_w, self.ln2_b = blk.ln2.weight, blk.ln2.bias
        self.w1, self.b1 = blk.fc1.weight, blk.fc1.bias
        self.w2, self.b2 = blk.fc2.weight, blk.fc2.bias
        self.eps = blk.ln1.eps

    def all(self):
        return [self.ln1_w, self.ln1_b, self.wqkv, self.bqkv, self.wo, self.bo, self.ln2_w,
                self.ln2_b, self.w1, self.b1, self.w2, self.b2]


def block_forward(x, p: BlockParams, B, S, H, causal, key_pad=None):
    """x f32 [T, C] -> (x3 f32 [T, C], saved tuple)."""
    K = C()
    T, Cd = x.shape
    dev = x.device
    mean1, rstd1 = _empty(T, torch.float32, dev), _empty(T, torch.float32, dev)
    h1 = _empty((T, Cd), torch.bfloat16, dev)
    K.ln_fwd(x, p.ln1_w.detach(), p.ln1_b.detach(), h1, None, mean1, rstd1, p.eps)
    qkv = _empty((T, 3 * Cd), torch.bfloat16, dev)
    K.gemm(h1, bf16_shadow(p.wqkv), qkv, T, 3 * Cd, Cd, False, False, bias=p.bqkv.detach())
    attn, lse = attn_fwd_packed(qkv, B, S, H, causal, key_pad)
    x2 = _empty((T, Cd), torch.float32, dev)
    K.gemm(attn, bf16_shadow(p.wo), x2, T, Cd, Cd, False, False, bias=p.bo.detach(), residual=x)
    mean2, rstd2 = _empty(T, torch.float32, dev), _empty(T, torch.float32, dev)
    h2 = _empty((T, Cd), torch.bfloat16, dev)
    K.ln_fwd(x2, p.ln2_w.detach(), p.ln2_b.detach(), h2, None, mean2, rstd2, p.eps)
    F4 = p.w1.shape[0]
    a = _empty((T, F4), torch.bfloat16, dev)
    pre = _empty((T, F4), torch.bfloat16, dev)  # GELU'(fc1 pre-activation), kept for backward
    K.gemm(h2, bf16_shadow(p.w1), a, T, F4, Cd, False, False, bias=p.b1.detach(), aux=pre,
           flags=K.EPI_GELU)
    x3 = _empty((T, Cd), torch.float32, dev)
    K.gemm(a, bf16_shadow(p.w2), x3, T, Cd, F4, False, False, bias=p.b2.detach(), residual=x2)
    saved = (x, mean1, rstd1, h1, qkv, attn, lse, x2, mean2, rstd2, h2, pre, a)
    return x3, saved


def block_backward(dx3, dx3_16, p: BlockParams, saved, B, S, H, causal, prev_bias_grad,
                   key_pad=None, lane=None):
    """Given the f32 gradient of the block output (and its bf16 copy), returns
    (dx f32, dx bf16). ``prev_bias_grad`` receives the column sum of dx (the
    bias gradient of the previous block's fc2), or None. With ``lane`` the
    weight-gradient GEMMs run on its stream."""
    K = C()
    wg = lane.wgrad if lane is not None else _wgrad
    x, mean1, rstd1, h1, qkv, attn, lse, x2, mean2, rstd2, h2, pre, a = saved
    T, Cd = x.shape
    F4 = p.w1.shape[0]
    dev = x.device
    # fc2
    wg(dx3_16, a, p.w2)
    da = _empty((T, F4), torch.bfloat16, dev)
    # da = (dy W2) * GELU'; the epilogue also adds column sums of da to fc1's bias gradient
    K.gemm(dx3_16, bf16_shadow(p.w2), da, T, F4, Cd, False, True, aux=pre, flags=K.EPI_DGELU,
           colsum=grad_buffer(p.b1))
    # fc1
    wg(da, h2, p.w1)
    dh2 = _empty((T, Cd), torch.bfloat16, dev)
    K.gemm(da, bf16_shadow(p.w1), dh2, T, Cd, F4, False, True)
    # ln2 (+ skip path), bias grad of proj
    dx2 = _empty((T, Cd), torch.float32, dev)
    dx2_16 = _empty((T, Cd), torch.bfloat16, dev)
    K.ln_bwd(dh2, x2, mean2, rstd2, p.ln2_w.detach(), dx3, dx2, dx2_16, grad_buffer(p.ln2_w),
             grad_buffer(p.ln2_b), grad_buffer(p.bo))
    # attention output projection
    wg(dx2_16, attn, p.wo)
    dattn = _empty((T, Cd), torch.bfloat16, dev)
    K.gemm(dx2_16, bf16_shadow(p.wo), dattn, T, Cd, Cd, False, True)
    dqkv = attn_bwd_packed(dattn, qkv, attn, lse, B, S, H, causal, key_pad,
                           bias_grad=grad_buffer(p.bqkv))
    wg(dqkv, h1, p.wqkv)
    dh1 = _empty((T, Cd), torch.bfloat16, dev)
    K.gemm(dqkv, bf16_shadow(p.wqkv), dh1, T, Cd, 3 * Cd, False, True)
    dx = _empty((T, Cd), torch.float32, dev)
    dx16 = _empty((T, Cd), torch.bfloat16, dev)
    K.ln_bwd(dh1, x, mean1, rstd1, p.ln1_w.detach(), dx2, dx, dx16, grad_buffer(p.ln1_w),
             grad_buffer(p.ln1_b), prev_bias_grad)
    return dx, dx16


class _LMTrainFn(torch.autograd.Function):
    """ids [B, S] int64, targets [B, S] int64 -> mean loss (0-d f32)."""

    @staticmethod
    def forward(ctx, anchor, model, ids, targets):
        K = C()
        B, S = ids.shape
        T = B * S
        H = model.num_heads
        dev = ids.device
        Cd = model.d_model
        ids_f = ids.reshape(-1).contiguous()
        x = _empty((T, Cd), torch.float32, dev)
        pos = model.pos_emb.detach()[:S].contiguous()
        K.embed_fwd(ids_f, model.tok_emb.weight.detach(), pos, None, None, x, None, S)
        blocks = [BlockParams(b) for b in model.blocks]
        saved = []
        for p in blocks:
            x, sv = block_forward(x, p, B, S, H, model.causal)
            saved.append(sv)
        # final LN + head + CE
        meanf, rstdf = _empty(T, torch.float32, dev), _empty(T, torch.float32, dev)
        hf = _empty((T, Cd), torch.bfloat16, dev)
        K.ln_fwd(x, model.ln_f.weight.detach(), model.ln_f.bias.detach(), hf, None, meanf, rstdf,
                 model.ln_f.eps)
        V = model.vocab_size
        logits = _empty((T, V), torch.bfloat16, dev)
        K.gemm(hf, bf16_shadow(model.head.weight), logits, T, V, Cd, False, False,
               bias=model.head.bias.detach())
        loss = torch.zeros((), device=dev, dtype=torch.float32)
        inv = _empty((), torch.float32, dev)
        dlogits = torch.empty_like(logits)
        K.softmax_ce(logits, targets.reshape(-1).contiguous(), loss, inv, dlogits, -100, 0.0)
        ctx.model = model
        ctx.blocks = blocks
        ctx.saved_blocks = saved
        ctx.misc = (ids_f, x, meanf, rstdf, hf, dlogits, B, S)
        return loss

    @staticmethod
    def backward(ctx, g):
        K = C()
        model = ctx.model
        ids_f, xL, meanf, rstdf, hf, dlogits, B, S = ctx.misc
        T, Cd = xL.shape
        dev = xL.device
        H = model.num_heads
        g = g.detach().reshape(()).float().contiguous()
        # head
        head = model.head
        lane = WgradLane(dev)
        lane.wgrad(dlogits, hf, head.weight, alpha_t=g)
        K.colsum(dlogits, grad_buffer(head.bias), g)
        dhf = _empty((T, Cd), torch.bfloat16, dev)
        K.gemm(dlogits, bf16_shadow(head.weight), dhf, T, Cd, model.vocab_size, False, True,
               alpha_t=g)
        dx = _empty((T, Cd), torch.float32, dev)
        dx16 = _empty((T, Cd), torch.bfloat16, dev)
        blocks = ctx.blocks
        last_b2 = grad_buffer(blocks[-1].b2) if blocks else None
        K.ln_bwd(dhf, xL, meanf, rstdf, model.ln_f.weight.detach(), None, dx, dx16,
                 grad_buffer(model.ln_f.weight), grad_buffer(model.ln_f.bias), last_b2)
        lane.ready((head.weight, head.bias, model.ln_f.weight, model.ln_f.bias))
        for li in range(len(blocks) - 1, -1, -1):
            p = blocks[li]
            prev_b2 = grad_buffer(blocks[li - 1].b2) if li > 0 else None
            dx, dx16 = block_backward(dx, dx16, p, ctx.saved_blocks[li], B, S, H, model.causal,
                                      prev_b2, lane=lane)
            ctx.saved_blocks[li] = None
            lane.ready(p.all())
        # embeddings
        tokw = model.tok_emb.weight
        V = tokw.shape[0]
        if V <= 4096:
            onehot = _empty((T, V), torch.bfloat16, dev)
            K.onehot_bf16(ids_f, onehot)
            K.gemm(onehot, dx16, grad_buffer(tokw), V, Cd, T, True, True,
                   flags=K.EPI_ACCUMULATE, k_splits=splitk_for(V, Cd, T))
        else:
            K.embed_bwd_atomic(ids_f, dx, grad_buffer(tokw))
        K.pos_grad(dx, grad_buffer(model.pos_emb), B, S)
        lane.join()
        grad_ready(tokw)
        grad_ready(model.pos_emb)
        ctx.saved_blocks = None
        return None, None, None, None


def lm_train_loss(model, ids: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """Fused forward of the whole LM; ``loss.backward()`` runs the fused backward."""
    anchor = model._grad_anchor
    return _LMTrainFn.apply(anchor, model, ids, targets)
