"""Fused training step of a CIFAR ResNet (conv/BN/ReLU basic blocks) as ONE
autograd op on sm_100a.

Reference composition (ddp-bench/src/models/resnet.rs, He et al. 2015):

    x   = relu(bn(conv3x3(img)))
    per block: out = relu(bn2(conv2(relu(bn1(conv1(x))))) + shortcut(x)),
               shortcut = bn(conv1x1, stride s) when the shape changes, else x
    logits = fc(avgpool(x))

On CUDA every activation is NHWC bf16 (the 3-channel input is padded to 8
channels). A convolution is im2col -> tcgen05 GEMM, with columns ordered
(kh, kw, ci) so that gathers move 16-byte vectors; one launch packs every
convolution weight into that order (bf16) at the start of the step. Its
backward is a dgrad GEMM + col2im gather (which also adds the shortcut
gradient) and a split-K weight-gradient GEMM that reuses the forward's column
buffer, accumulating in packed order; one launch unpacks all of them into the
OIHW ``param.grad`` at the end of backward.

Batch norm statistics (per-channel sum and sum of squares) are added by the
convolution GEMM's epilogue (kept in registers per CTA, one atomic per column
and CTA); one apply kernel derives mean / rstd, updates the running
statistics, adds the shortcut and applies the ReLU; its backward
applies the ReLU mask of the block output and hands the masked gradient to
the shortcut path in the same pass. Gradients accumulate in f32 straight into
``param.grad``; gradient-ready listeners (the DDP bucket hooks) fire per
batch-norm layer and, for the convolutions, after the final unpack.
"""
from __future__ import annotations

import torch

import os

from ._common import C, bf16_shadow, grad_buffer, grad_ready, splitk_for
from .transformer import _empty

# batch-norm statistics summed in the convolution GEMM's epilogue (no separate
# statistics pass); FLODL_BN_FUSED_STATS=0 keeps the statistics kernel
FUSED_BN_STATS = os.environ.get("FLODL_BN_FUSED_STATS", "1") != "0"
# batch-norm backward sums (sum dz, sum dz * xhat) added up by the col2im that
# produces dz, with FLODL_BN_FUSED_BWD=1. Off by default: on B200 the block
# reduction and ticket of the fused col2im cost more than the re-read of dz
# they save (col2im + separate reduction: 1.725 ms per ResNet-20 step; fused:
# 1.801 ms).
FUSED_BN_BWD = os.environ.get("FLODL_BN_FUSED_BWD", "0") == "1"


def _bn_bwd_fusable(c):
    return FUSED_BN_BWD and c % 8 == 0 and 256 % (c // 8) == 0


def _ws(bn, dev):
    ws = getattr(bn, "_flodl_bn_ws", None)
    C_ = bn.num_features
    if ws is None or ws.device != dev:
        ws = torch.zeros(2 * C_ + 1, device=dev, dtype=torch.float32)  # sums + ticket
        bn._flodl_bn_ws = ws
        bn._flodl_bn_sums = torch.zeros(2 * C_, device=dev, dtype=torch.float32)
    return ws, bn._flodl_bn_sums


class _ConvPlan:
    """Per-model table of the convolutions: packed bf16 weights (column order
    (kh, kw, ci), input channels padded to a multiple of 8), packed-order f32
    weight-gradient accumulators, and the device table that packs / unpacks
    them all in one launch each."""

    def __init__(self, convs, dev):
        import struct

        K_ = C()
        self.convs = convs
        recs = []
        self.max_elems = 0
        for c in convs:
            c.packed = torch.empty(c.cout, c.K, device=dev, dtype=torch.bfloat16)
            c.gacc = torch.zeros(c.cout, c.K, device=dev, dtype=torch.float32)
            g = grad_buffer(c.w)
            recs.append(struct.pack("<QQQQiiii", c.w.data_ptr(), c.packed.data_ptr(),
                                    c.gacc.data_ptr(), g.data_ptr(), c.cout, c.cin, c.cin_pad, c.k))
            self.max_elems = max(self.max_elems, c.cout * c.K)
        raw = b"".join(recs)
        assert len(raw) == len(convs) * K_.CONV_PACK_ENTRY_BYTES
        self.table = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(dev)
        self.sig = self.signature(convs)

    @staticmethod
    def signature(convs):
        return tuple((c.w.data_ptr(), c.w.grad.data_ptr() if c.w.grad is not None else 0)
                     for c in convs)

    def pack(self):
        C().pack_conv_weights(self.table, len(self.convs), self.max_elems)

    def unpack(self):
        C().unpack_conv_grads(self.table, len(self.convs), self.max_elems)
        for c in self.convs:
            grad_ready(c.w)


class _Conv:
    """One convolution of the fused op (geometry, packed weight, gradient buffer)."""

    def __init__(self, conv):
        self.mod = conv
        self.w = conv.weight
        self.cout, self.cin, self.k, _ = conv.weight.shape
        self.cin_pad = (self.cin + 7) // 8 * 8
        self.s = conv.stride[0]
        self.p = conv.padding[0]
        self.K = self.cin_pad * self.k * self.k
        self.packed = None
        self.gacc = None

    def out_hw(self, H, W):
        return (H + 2 * self.p - self.k) // self.s + 1, (W + 2 * self.p - self.k) // self.s + 1

    def forward(self, x, bn=None):
        """x NHWC bf16 -> (y [M, Cout] bf16, cols [M, K], (N, Ho, Wo)). With
        ``bn`` (the batch norm that follows) the GEMM epilogue also adds the
        output's per-channel sums and sums of squares into its workspace."""
        N, H, W, _ = x.shape
        Ho, Wo = self.out_hw(H, W)
        M = N * Ho * Wo
        K_ = C()
        if self.k == 1 and self.s == 1:
            cols = x.view(M, self.K)
        else:
            cols = _empty((M, self.K), torch.bfloat16, x.device)
            K_.im2col(x, cols, self.k, self.s, self.p)
        y = _empty((M, self.cout), torch.bfloat16, x.device)
        if bn is not None and FUSED_BN_STATS:
            ws, _ = _ws(bn.mod, x.device)
            K_.gemm(cols, self.packed, y, M, self.cout, self.K, False, False,
                    colsum=ws[:self.cout], colsumsq=ws[self.cout:2 * self.cout])
        else:
            K_.gemm(cols, self.packed, y, M, self.cout, self.K, False, False)
        return y, cols, (N, Ho, Wo)

    def backward(self, dy, cols, x_shape, add=None, mask=None, need_dx=True, bn=None):
        """dy [M, Cout] bf16 -> dx NHWC bf16 (+ add, * [mask > 0]); the weight
        gradient accumulates (packed order) into self.gacc. ``bn`` = (batch
        norm, its input, mean, rstd) when dx is that batch norm's output
        gradient: the col2im pass also reduces its backward sums."""
        K_ = C()
        M = dy.shape[0]
        K_.gemm(dy, cols, self.gacc, self.cout, self.K, M, True, True, flags=K_.EPI_ACCUMULATE,
                k_splits=splitk_for(self.cout, self.K, M))
        if not need_dx:
            return None
        dcols = _empty((M, self.K), torch.bfloat16, dy.device)
        K_.gemm(dy, self.packed, dcols, M, self.K, self.cout, False, True)
        dx = _empty(x_shape, torch.bfloat16, dy.device)
        if bn is not None:
            bno, y, mean, rstd = bn
            ws, sums = _ws(bno.mod, dy.device)
            K_.col2im_bn(dcols, dx, self.k, self.s, self.p, add, mask, y, mean, rstd,
                         grad_buffer(bno.mod.weight), grad_buffer(bno.mod.bias), sums, ws)
        else:
            K_.col2im(dcols, dx, self.k, self.s, self.p, add, mask)
        return dx


def _plan(model, parts, dev):
    stem_c, blocks = parts
    convs = [stem_c]
    for b in blocks:
        convs += [b.conv1, b.conv2] + ([b.ds[0]] if b.ds is not None else [])
    plan = getattr(model, "_flodl_conv_plan", None)
    if plan is not None and len(plan.convs) == len(convs):
        for c, old in zip(convs, plan.convs):
            c.packed, c.gacc = old.packed, old.gacc
        if _ConvPlan.signature(convs) == plan.sig:
            plan.convs = convs
            return plan
    plan = _ConvPlan(convs, dev)
    model._flodl_conv_plan = plan
    return plan


class _BN:
    def __init__(self, bn):
        self.mod = bn
        self.c = bn.num_features

    def forward(self, y, identity=None, relu=True, training=True):
        K_ = C()
        dev = y.device
        mean = _empty(self.c, torch.float32, dev)
        rstd = _empty(self.c, torch.float32, dev)
        ws, _ = _ws(self.mod, dev)
        b = self.mod
        out = torch.empty_like(y)
        if FUSED_BN_STATS:
            # the convolution's GEMM epilogue left sum / sum of squares in ws
            K_.bn_apply_sums(y, ws, mean, rstd, b.running_mean if training else None,
                             b.running_var if training else None, b.weight.detach(),
                             b.bias.detach(), identity, relu, out, b.eps, b.momentum)
            return out, mean, rstd
        K_.bn_stats(y, mean, rstd, b.running_mean if training else None,
                    b.running_var if training else None, ws, b.eps, b.momentum)
        K_.bn_apply(y, mean, rstd, b.weight.detach(), b.bias.detach(), identity, relu, out)
        return out, mean, rstd

    def backward(self, dy, ymask, y, mean, rstd, want_dz=False):
        K_ = C()
        b = self.mod
        ws, sums = _ws(b, dy.device)
        dx = torch.empty_like(y)
        dz = torch.empty_like(y) if want_dz else None
        K_.bn_bwd(dy, ymask, y, mean, rstd, b.weight.detach(), grad_buffer(b.weight),
                  grad_buffer(b.bias), sums, ws, dx, dz)
        grad_ready(b.weight)
        grad_ready(b.bias)
        return dx, dz

    def backward_apply(self, dz, y, mean, rstd):
        """Input gradient from sums that the producer of dz reduced (dgamma
        and dbeta are already accumulated)."""
        b = self.mod
        _, sums = _ws(b, dz.device)
        dx = torch.empty_like(y)
        C().bn_bwd_apply(dz, None, y, mean, rstd, b.weight.detach(), sums, dx)
        grad_ready(b.weight)
        grad_ready(b.bias)
        return dx


class _Block:
    def __init__(self, blk):
        self.conv1, self.bn1 = _Conv(blk.conv1), _BN(blk.bn1)
        self.conv2, self.bn2 = _Conv(blk.conv2), _BN(blk.bn2)
        self.ds = (_Conv(blk.downsample_conv), _BN(blk.downsample_bn)) if blk.downsample_conv is not None else None

    def forward(self, x):
        y1, cols1, (N, Ho, Wo) = self.conv1.forward(x, self.bn1)
        a1, m1, r1 = self.bn1.forward(y1)
        a1 = a1.view(N, Ho, Wo, -1)
        y2, cols2, _ = self.conv2.forward(a1, self.bn2)
        if self.ds is not None:
            yd, colsd, _ = self.ds[0].forward(x, self.ds[1])
            ident, md, rd = self.ds[1].forward(yd, relu=False)
            dsv = (yd, colsd, md, rd)
        else:
            ident = x.view(y2.shape)
            dsv = None
        out, m2, r2 = self.bn2.forward(y2, identity=ident, relu=True)
        saved = (x, cols1, y1, m1, r1, a1, cols2, y2, m2, r2, out, dsv)
        return out.view(N, Ho, Wo, -1), saved

    def backward(self, dout, saved, reduced=False, prev=None):
        """Gradient of the block input. ``reduced``: dout is already masked by
        the output ReLU and bn2's backward sums are reduced. ``prev`` = (batch
        norm, input, mean, rstd) of the batch norm whose ReLU output is this
        block's input: the returned gradient is then masked by that ReLU with
        the batch norm's sums reduced in the same pass."""
        x, cols1, y1, m1, r1, a1, cols2, y2, m2, r2, out, dsv = saved
        if reduced:
            dz = dout.view(y2.shape)
            dy2 = self.bn2.backward_apply(dz, y2, m2, r2)
        else:
            dy2, dz = self.bn2.backward(dout.view(y2.shape), out, y2, m2, r2, want_dz=True)
        if _bn_bwd_fusable(self.bn1.c):
            da1 = self.conv2.backward(dy2, cols2, a1.shape, mask=a1, bn=(self.bn1, y1, m1, r1))
            dy1 = self.bn1.backward_apply(da1.view(y1.shape), y1, m1, r1)
        else:
            da1 = self.conv2.backward(dy2, cols2, a1.shape, mask=a1)
            dy1, _ = self.bn1.backward(da1.view(y1.shape), None, y1, m1, r1)
        if dsv is not None:
            yd, colsd, md, rd = dsv
            dyd, _ = self.ds[1].backward(dz, None, yd, md, rd)
            add = self.ds[0].backward(dyd, colsd, x.shape)
        else:
            add = dz
        if prev is not None:
            return self.conv1.backward(dy1, cols1, x.shape, add=add, mask=x, bn=prev)
        return self.conv1.backward(dy1, cols1, x.shape, add=add)


class _ResNetTrainFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, anchor, model, images, targets):
        K_ = C()
        dev = images.device
        N, Cin, H, W = images.shape
        stem_c, stem_bn = _Conv(model.conv1), _BN(model.bn1)
        blocks = [_Block(b) for layer in (model.layer1, model.layer2, model.layer3) for b in layer]
        plan = _plan(model, (stem_c, blocks), dev)
        plan.pack()
        x = _empty((N, H, W, stem_c.cin_pad), torch.bfloat16, dev)
        K_.nchw_to_nhwc(images.float().contiguous(), x)
        y0, cols0, (_, Ho, Wo) = stem_c.forward(x, stem_bn)
        x0, m0, r0 = stem_bn.forward(y0)
        h = x0.view(N, Ho, Wo, -1)
        saved = []
        for b in blocks:
            h, sv = b.forward(h)
            saved.append(sv)
        Cf = h.shape[-1]
        pooled = _empty((N, Cf), torch.bfloat16, dev)
        K_.avgpool_fwd(h, pooled)
        ncls = model.fc.weight.shape[0]
        ldl = (ncls + 7) // 8 * 8
        logits_buf = _empty((N, ldl), torch.bfloat16, dev)
        logits = logits_buf[:, :ncls]
        K_.gemm(pooled, bf16_shadow(model.fc.weight), logits, N, ncls, Cf, False, False,
                bias=model.fc.bias.detach())
        loss = torch.zeros((), device=dev, dtype=torch.float32)
        inv = _empty((), torch.float32, dev)
        dl_buf = _empty((N, ldl), torch.bfloat16, dev)
        dlogits = dl_buf[:, :ncls]
        K_.softmax_ce(logits, targets.reshape(-1).contiguous(), loss, inv, dlogits, -100, 0.0)
        ctx.model = model
        ctx.parts = (stem_c, stem_bn, blocks, plan)
        ctx.saved_blocks = saved
        ctx.misc = (x.shape, cols0, y0, m0, r0, x0, h.shape, pooled, dlogits)
        return loss

    @staticmethod
    def backward(ctx, g):
        K_ = C()
        model = ctx.model
        stem_c, stem_bn, blocks, plan = ctx.parts
        x_shape, cols0, y0, m0, r0, x0, h_shape, pooled, dlogits = ctx.misc
        g = g.detach().reshape(()).float().contiguous()
        N, Cf = pooled.shape
        ncls = dlogits.shape[1]
        fc = model.fc
        # fc: dW += dlogits^T pooled (scaled by the upstream scalar), db, d pooled
        K_.gemm(dlogits, pooled, grad_buffer(fc.weight), ncls, Cf, N, True, True,
                flags=K_.EPI_ACCUMULATE, alpha_t=g)
        K_.colsum(dlogits, grad_buffer(fc.bias), g)
        grad_ready(fc.weight)
        grad_ready(fc.bias)
        dpooled = _empty((N, Cf), torch.bfloat16, pooled.device)
        K_.gemm(dlogits, bf16_shadow(fc.weight), dpooled, N, Cf, ncls, False, True, alpha_t=g)
        dh = _empty(h_shape, torch.bfloat16, pooled.device)
        K_.avgpool_bwd(dpooled, dh)
        saved = ctx.saved_blocks
        # the batch norm feeding each block's input: the stem's, then bn2 of
        # the block before
        prevs = [(stem_bn, y0, m0, r0)] + [(b.bn2, sv[7], sv[8], sv[9])
                                           for b, sv in zip(blocks[:-1], saved[:-1])]
        reduced = False
        for i in reversed(range(len(blocks))):
            prev = prevs[i] if _bn_bwd_fusable(prevs[i][0].c) else None
            dh = blocks[i].backward(dh, saved[i], reduced, prev)
            reduced = prev is not None
        if reduced:
            dy0 = stem_bn.backward_apply(dh.view(y0.shape), y0, m0, r0)
        else:
            dy0, _ = stem_bn.backward(dh.view(y0.shape), x0, y0, m0, r0)
        stem_c.backward(dy0, cols0, x_shape, need_dx=False)
        plan.unpack()  # packed-order conv gradients -> OIHW param.grad (+ grad-ready)
        ctx.saved_blocks = None
        return None, None, None, None


def resnet_train_loss(model, images: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """Mean cross-entropy of a CIFAR ResNet on ``images`` [N, 3, H, W] through
    the fused CUDA training op (training-mode batch norm)."""
    return _ResNetTrainFn.apply(model._grad_anchor, model, images, targets)
