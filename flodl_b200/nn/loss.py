"""Loss functions (flodl/src/nn/loss.rs). Cross-entropy runs the fused
softmax-CE kernel on CUDA; the others compose ATen ops."""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .. import ops


def mse_loss(pred, target):
    return F.mse_loss(pred, target)


def l1_loss(pred, target):
    return F.l1_loss(pred, target)


def smooth_l1_loss(pred, target, beta: float = 1.0):
    return F.smooth_l1_loss(pred, target, beta=beta)


def cross_entropy_loss(logits, target, ignore_index: int = -100, label_smoothing: float = 0.0):
    return ops.cross_entropy(logits, target, ignore_index, label_smoothing)


def nll_loss(log_probs, target, ignore_index: int = -100):
    return F.nll_loss(log_probs, target, ignore_index=ignore_index)


def bce_loss(pred, target):
    return F.binary_cross_entropy(pred, target)


def bce_with_logits_loss(logits, target, pos_weight=None):
    return F.binary_cross_entropy_with_logits(logits, target, pos_weight=pos_weight)


def kl_div_loss(log_pred, target, log_target: bool = False):
    return F.kl_div(log_pred, target, reduction="batchmean", log_target=log_target)


def ctc_loss(log_probs, targets, input_lengths, target_lengths, blank: int = 0):
    return F.ctc_loss(log_probs, targets, input_lengths, target_lengths, blank=blank)


def focal_loss(logits, target, alpha: float = 0.25, gamma: float = 2.0):
    """Focal loss (Lin et al. 2017). Class-index targets ``[N]`` with logits
    ``[N, C]`` (reference nn/loss.rs:174): mean of ``-alpha (1 - p_t)^gamma
    log p_t``; reduces to ``alpha`` x cross-entropy at ``gamma = 0``.
    Floating targets of the logits' shape select the binary form."""
    if not target.is_floating_point():
        log_p = torch.log_softmax(logits, dim=-1)
        log_pt = log_p.gather(-1, target.unsqueeze(-1)).squeeze(-1)
        pt = log_pt.exp()
        return (-alpha * (1 - pt) ** gamma * log_pt).mean()
    p = torch.sigmoid(logits)
    ce = F.binary_cross_entropy_with_logits(logits, target, reduction="none")
    p_t = p * target + (1 - p) * (1 - target)
    a_t = alpha * target + (1 - alpha) * (1 - target)
    return (a_t * (1 - p_t) ** gamma * ce).mean()


def triplet_margin_loss(anchor, positive, negative, margin: float = 1.0):
    return F.triplet_margin_loss(anchor, positive, negative, margin=margin)


def cosine_embedding_loss(x1, x2, y, margin: float = 0.0):
    return F.cosine_embedding_loss(x1, x2, y, margin=margin)


def hinge_embedding_loss(x, y, margin: float = 1.0):
    return F.hinge_embedding_loss(x, y, margin=margin)


def margin_ranking_loss(x1, x2, y, margin: float = 0.0):
    return F.margin_ranking_loss(x1, x2, y, margin=margin)


def poisson_nll_loss(log_input, target, log_input_flag: bool = True):
    return F.poisson_nll_loss(log_input, target, log_input=log_input_flag)
