"""Fused training step of a post-LayerNorm encoder (BERT) with a masked-LM head.

Reference composition (HF BERT; flodl-hf/src/models/bert.rs):

    x1 = LN1(x + dense_o(attn(qkv(x))))
    x2 = LN2(x1 + dense_2(gelu(dense_1(x1))))

Per block on sm_100a: qkv GEMM (+bias) -> flash attention with the key
padding mask -> output GEMM with bias + residual epilogue (f32) -> LayerNorm
writing both the f32 residual and the bf16 GEMM operand -> FFN GEMMs (GELU /
residual epilogues) -> LayerNorm. Backward mirrors it; LayerNorm backward runs
in "pre-add" mode (it normalises dy + skip-gradient, the post-LN rule) and
accumulates the previous Linear's bias gradient. The MLM head runs only on
the masked rows (gathered once), with the decoder tied to the word embedding
table through its bf16 shadow; the tied gradient accumulates into the same
f32 buffer as the embedding-lookup gradient.
"""
from __future__ import annotations

import torch

from ._common import C, bf16_shadow, grad_buffer, grad_ready, splitk_for
from .attention import attn_bwd_packed, attn_fwd_packed
from .transformer import WgradLane, _empty, _wgrad


class PostBlockParams:
    __slots__ = ("wqkv", "bqkv", "wo", "bo", "ln1_w", "ln1_b", "w1", "b1", "w2", "b2", "eps", "_ln2")

    def __init__(self, layer):
        a = layer.attention
        self.wqkv, self.bqkv = a.self.qkv.weight, a.self.qkv.bias
        self.wo, self.bo = a.output.dense.weight, a.output.dense.bias
        self.ln1_w, self.ln1_b = a.output.LayerNorm.weight, a.output.LayerNorm.bias
        self.w1, self.b1 = layer.intermediate.dense.weight, layer.intermediate.dense.bias
        self.w2, self.b2 = layer.output.dense.weight, layer.output.dense.bias
        self.eps = a.output.LayerNorm.eps
        self._ln2 = layer.output.LayerNorm

    def all(self):
        return [self.wqkv, self.bqkv, self.wo, self.bo, self.ln1_w, self.ln1_b, self.w1, self.b1,
                self.w2, self.b2, self._ln2.weight, self._ln2.bias]


def post_block_forward(x, x16, p: PostBlockParams, B, S, H, key_pad):
    K = C()
    T, Cd = x.shape
    dev = x.device
    qkv = _empty((T, 3 * Cd), torch.bfloat16, dev)
    K.gemm(x16, bf16_shadow(p.wqkv), qkv, T, 3 * Cd, Cd, False, False, bias=p.bqkv.detach())
    attn, lse = attn_fwd_packed(qkv, B, S, H, False, key_pad)
    y1 = _empty((T, Cd), torch.float32, dev)
    K.gemm(attn, bf16_shadow(p.wo), y1, T, Cd, Cd, False, False, bias=p.bo.detach(), residual=x)
    m1, r1 = _empty(T, torch.float32, dev), _empty(T, torch.float32, dev)
    x1 = _empty((T, Cd), torch.float32, dev)
    x1_16 = _empty((T, Cd), torch.bfloat16, dev)
    K.ln_fwd(y1, p.ln1_w.detach(), p.ln1_b.detach(), x1_16, x1, m1, r1, p.eps)
    F4 = p.w1.shape[0]
    a = _empty((T, F4), torch.bfloat16, dev)
    pre = _empty((T, F4), torch.bfloat16, dev)  # GELU'(fc1 pre-activation), kept for backward
    K.gemm(x1_16, bf16_shadow(p.w1), a, T, F4, Cd, False, False, bias=p.b1.detach(), aux=pre,
           flags=K.EPI_GELU)
    y2 = _empty((T, Cd), torch.float32, dev)
    K.gemm(a, bf16_shadow(p.w2), y2, T, Cd, F4, False, False, bias=p.b2.detach(), residual=x1)
    m2, r2 = _empty(T, torch.float32, dev), _empty(T, torch.float32, dev)
    x2 = _empty((T, Cd), torch.float32, dev)
    x2_16 = _empty((T, Cd), torch.bfloat16, dev)
    ln2 = p._ln2
    K.ln_fwd(y2, ln2.weight.detach(), ln2.bias.detach(), x2_16, x2, m2, r2, ln2.eps)
    saved = (x16, qkv, attn, lse, y1, m1, r1, x1_16, a, pre, y2, m2, r2)
    return x2, x2_16, saved


def post_block_backward(g2, g2_16, extra16, p: PostBlockParams, saved, B, S, H, key_pad,
                        lane=None):
    """g2: f32 skip-path gradient of the block output, extra16: bf16 GEMM-path
    gradient of the block output (or None). Returns (g_in f32, g_in_extra bf16)
    for the previous block. With ``lane`` the weight-gradient GEMMs run on its
    stream."""
    K = C()
    wg = lane.wgrad if lane is not None else _wgrad
    x16, qkv, attn, lse, y1, m1, r1, x1_16, a, pre, y2, m2, r2 = saved
    T, Cd = y1.shape
    dev = y1.device
    F4 = p.w1.shape[0]
    ln2 = p._ln2
    # LN2 backward of (extra16 + g2) -> dy2 (f32 + bf16), dgamma2/dbeta2, b2 grad
    dy2 = _empty((T, Cd), torch.float32, dev)
    dy2_16 = _empty((T, Cd), torch.bfloat16, dev)
    if extra16 is None:
        K.ln_bwd(g2_16, y2, m2, r2, ln2.weight.detach(), None, dy2, dy2_16, grad_buffer(ln2.weight),
                 grad_buffer(ln2.bias), grad_buffer(p.b2))
    else:
        K.ln_bwd(extra16, y2, m2, r2, ln2.weight.detach(), g2, dy2, dy2_16, grad_buffer(ln2.weight),
                 grad_buffer(ln2.bias), grad_buffer(p.b2), True)
    # FFN
    wg(dy2_16, a, p.w2)
    da = _empty((T, F4), torch.bfloat16, dev)
    # da = (dy W2) * GELU'; the epilogue also adds column sums of da to fc1's bias gradient
    K.gemm(dy2_16, bf16_shadow(p.w2), da, T, F4, Cd, False, True, aux=pre, flags=K.EPI_DGELU,
           colsum=grad_buffer(p.b1))
    wg(da, x1_16, p.w1)
    dx1 = _empty((T, Cd), torch.bfloat16, dev)
    K.gemm(da, bf16_shadow(p.w1), dx1, T, Cd, F4, False, True)
    # LN1 backward of (dx1 + dy2) -> dy1, bo grad
    dy1 = _empty((T, Cd), torch.float32, dev)
    dy1_16 = _empty((T, Cd), torch.bfloat16, dev)
    K.ln_bwd(dx1, y1, m1, r1, p.ln1_w.detach(), dy2, dy1, dy1_16, grad_buffer(p.ln1_w),
             grad_buffer(p.ln1_b), grad_buffer(p.bo), True)
    # attention
    wg(dy1_16, attn, p.wo)
    dattn = _empty((T, Cd), torch.bfloat16, dev)
    K.gemm(dy1_16, bf16_shadow(p.wo), dattn, T, Cd, Cd, False, True)
    dqkv = attn_bwd_packed(dattn, qkv, attn, lse, B, S, H, False, key_pad,
                           bias_grad=grad_buffer(p.bqkv))
    wg(dqkv, x16, p.wqkv)
    dxq = _empty((T, Cd), torch.bfloat16, dev)
    K.gemm(dqkv, bf16_shadow(p.wqkv), dxq, T, Cd, 3 * Cd, False, True)
    return dy1, dxq  # skip-path gradient (f32) and GEMM-path gradient (bf16) of the block input


class _BertMLMTrainFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, anchor, model, ids, labels, token_type_ids, attention_mask, masked_rows):
        K = C()
        cfg = model.config
        B, S = ids.shape
        T, Cd, H = B * S, cfg.hidden_size, cfg.num_attention_heads
        dev = ids.device
        emb = model.bert.embeddings
        ids_f = ids.reshape(-1).contiguous()
        tt = (token_type_ids if token_type_ids is not None else torch.zeros_like(ids)).reshape(-1).contiguous()
        key_pad = None if attention_mask is None else (attention_mask == 0).contiguous()
        e = _empty((T, Cd), torch.float32, dev)
        K.embed_fwd(ids_f, emb.word_embeddings.weight.detach(), emb.position_embeddings.weight.detach()[:S].contiguous(),
                    tt, emb.token_type_embeddings.weight.detach(), e, None, S)
        me, re_ = _empty(T, torch.float32, dev), _empty(T, torch.float32, dev)
        x = _empty((T, Cd), torch.float32, dev)
        x16 = _empty((T, Cd), torch.bfloat16, dev)
        K.ln_fwd(e, emb.LayerNorm.weight.detach(), emb.LayerNorm.bias.detach(), x16, x, me, re_,
                 emb.LayerNorm.eps)
        blocks = [PostBlockParams(l) for l in model.bert.encoder.layer]
        saved = []
        for p in blocks:
            x, x16, sv = post_block_forward(x, x16, p, B, S, H, key_pad)
            saved.append(sv)
        # MLM head on the masked rows
        lab = labels.reshape(-1)
        if masked_rows is None:
            sel = (lab != -100).nonzero(as_tuple=True)[0]  # host sync for the count
            Tm = int(sel.numel())
            lab_sel = lab.index_select(0, sel).contiguous()
        else:
            # fixed row budget: no host sync, so the step can be graph-captured.
            # Padding rows point at row 0 and carry label -100 (ignored); masked
            # rows beyond the budget are dropped.
            Tm = int(masked_rows)
            keep = lab != -100
            sel = torch.nonzero_static(keep, size=Tm, fill_value=0).reshape(-1)
            valid = torch.arange(Tm, device=dev) < keep.sum()
            lab_sel = torch.where(valid, lab.index_select(0, sel),
                                  torch.full_like(sel, -100)).contiguous()
        head = model.cls
        hm16 = x16.index_select(0, sel)
        t = _empty((Tm, Cd), torch.bfloat16, dev)
        tpre = _empty((Tm, Cd), torch.bfloat16, dev)
        K.gemm(hm16, bf16_shadow(head.transform_dense.weight), t, Tm, Cd, Cd, False, False,
               bias=head.transform_dense.bias.detach(), aux=tpre, flags=K.EPI_GELU)
        mt, rt = _empty(Tm, torch.float32, dev), _empty(Tm, torch.float32, dev)
        tl16 = _empty((Tm, Cd), torch.bfloat16, dev)
        K.ln_fwd(t, head.transform_LayerNorm.weight.detach(), head.transform_LayerNorm.bias.detach(),
                 tl16, None, mt, rt, head.transform_LayerNorm.eps)
        V = cfg.vocab_size
        Vp = (V + 7) // 8 * 8  # 16-byte row pitch for the TMA-fed GEMMs
        logits = _empty((Tm, Vp), torch.bfloat16, dev)[:, :V]
        K.gemm(tl16, bf16_shadow(head.decoder_weight), logits, Tm, V, Cd, False, False,
               bias=head.bias.detach())
        loss = torch.zeros((), device=dev, dtype=torch.float32)
        inv = _empty((), torch.float32, dev)
        dlogits = _empty((Tm, Vp), torch.bfloat16, dev)[:, :V]
        K.softmax_ce(logits, lab_sel, loss, inv, dlogits, -100, 0.0)
        ctx.model = model
        ctx.blocks = blocks
        ctx.saved_blocks = saved
        ctx.misc = (ids_f, tt, key_pad, e, me, re_, sel, hm16, t, tpre, mt, rt, tl16, dlogits, B, S)
        return loss

    @staticmethod
    def backward(ctx, g):
        K = C()
        model = ctx.model
        cfg = model.config
        ids_f, tt, key_pad, e, me, re_, sel, hm16, t, tpre, mt, rt, tl16, dlogits, B, S = ctx.misc
        T, Cd, H = B * S, cfg.hidden_size, cfg.num_attention_heads
        dev = e.device
        Tm = int(sel.numel())
        g = g.detach().reshape(()).float().contiguous()
        head = model.cls
        emb = model.bert.embeddings
        wemb = emb.word_embeddings.weight
        # decoder (tied to the word embeddings)
        _wgrad(dlogits, tl16, wemb, alpha_t=g)
        K.colsum(dlogits, grad_buffer(head.bias), g)
        dtl = _empty((Tm, Cd), torch.bfloat16, dev)
        K.gemm(dlogits, bf16_shadow(wemb), dtl, Tm, Cd, cfg.vocab_size, False, True, alpha_t=g)
        # transform LayerNorm + GELU + dense
        dt = _empty((Tm, Cd), torch.bfloat16, dev)
        K.ln_bwd(dtl, t, mt, rt, head.transform_LayerNorm.weight.detach(), None, None, dt,
                 grad_buffer(head.transform_LayerNorm.weight), grad_buffer(head.transform_LayerNorm.bias),
                 None)
        dtp = _empty((Tm, Cd), torch.bfloat16, dev)
        K.mul_bf16(dt, tpre, dtp)  # tpre holds GELU' of the transform
        K.colsum(dtp, grad_buffer(head.transform_dense.bias))
        _wgrad(dtp, hm16, head.transform_dense.weight)
        dhm = _empty((Tm, Cd), torch.bfloat16, dev)
        K.gemm(dtp, bf16_shadow(head.transform_dense.weight), dhm, Tm, Cd, Cd, False, True)
        for p in (head.bias, head.transform_dense.weight, head.transform_dense.bias,
                  head.transform_LayerNorm.weight, head.transform_LayerNorm.bias):
            grad_ready(p)
        # scatter the head gradient back into the last block's output rows
        gx16 = torch.zeros((T, Cd), dtype=torch.bfloat16, device=dev)
        gx16.index_copy_(0, sel, dhm)
        gskip = torch.zeros((T, Cd), dtype=torch.float32, device=dev)
        extra = gx16
        blocks = ctx.blocks
        lane = WgradLane(dev)
        for li in range(len(blocks) - 1, -1, -1):
            p = blocks[li]
            gskip, extra = post_block_backward(gskip, None, extra, p, ctx.saved_blocks[li], B, S, H,
                                               key_pad, lane=lane)
            ctx.saved_blocks[li] = None
            lane.ready(p.all())
        # the word-embedding gradient below also receives the tied decoder's
        # weight gradient (main stream): the lane is joined first
        lane.join()
        # embedding LayerNorm (input grad = skip + GEMM path) and the three tables
        de = _empty((T, Cd), torch.float32, dev)
        K.ln_bwd(extra, e, me, re_, emb.LayerNorm.weight.detach(), gskip, de, None,
                 grad_buffer(emb.LayerNorm.weight), grad_buffer(emb.LayerNorm.bias), None, True)
        K.embed_bwd_atomic(ids_f, de, grad_buffer(wemb))
        K.embed_bwd_atomic(tt, de, grad_buffer(emb.token_type_embeddings.weight))
        pos = grad_buffer(emb.position_embeddings.weight)
        K.pos_grad(de, pos[:S], B, S)
        for q in (wemb, emb.token_type_embeddings.weight, emb.position_embeddings.weight,
                  emb.LayerNorm.weight, emb.LayerNorm.bias):
            grad_ready(q)
        ctx.saved_blocks = None
        return None, None, None, None, None, None, None


def bert_mlm_train_loss(model, ids, labels, token_type_ids=None, attention_mask=None,
                        masked_rows=None):
    """Mean MLM loss over positions whose label is not -100. ``masked_rows``
    (optional) fixes the number of head rows so no host sync is needed."""
    return _BertMLMTrainFn.apply(model._grad_anchor, model, ids, labels, token_type_ids,
                                 attention_mask, masked_rows)
