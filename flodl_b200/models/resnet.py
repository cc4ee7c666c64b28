"""CIFAR ResNet-20 (He et al. 2015, option-B projection shortcuts).

Same module tree and parameter names as the reference benchmark model
(ddp-bench/src/models/resnet.rs:138-300): ``conv1``/``bn1`` stem, three
stages ``layer1..3`` of three ``BasicBlock`` (16/32/64 channels, the first
block of stages 2 and 3 with stride 2 and a 1x1 ``downsample_conv`` +
``downsample_bn`` shortcut), global average pooling and ``fc``.

``ResNet20.loss(images, targets)`` runs the fused sm_100a training op
(:mod:`flodl_b200.ops.resnet`) for CUDA inputs in training mode; otherwise it
composes the modules (PyTorch ops, the CPU oracle of the fused op).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .. import ops
from ..nn.layers import BatchNorm2d, Conv2d, Linear
from ..nn.module import Module


class BasicBlock(Module):
    NAME = "basic_block"

    def __init__(self, in_ch: int, out_ch: int, stride: int = 1, device=None):
        super().__init__()
        self.conv1 = Conv2d(in_ch, out_ch, 3, stride=stride, padding=1, bias=False, device=device)
        self.bn1 = BatchNorm2d(out_ch, device=device)
        self.conv2 = Conv2d(out_ch, out_ch, 3, padding=1, bias=False, device=device)
        self.bn2 = BatchNorm2d(out_ch, device=device)
        if stride != 1 or in_ch != out_ch:
            self.downsample_conv = Conv2d(in_ch, out_ch, 1, stride=stride, bias=False, device=device)
            self.downsample_bn = BatchNorm2d(out_ch, device=device)
        else:
            self.downsample_conv = None
            self.downsample_bn = None

    def forward(self, x):
        identity = x
        if self.downsample_conv is not None:
            identity = self.downsample_bn(self.downsample_conv(x))
        out = F.relu(self.bn1(self.conv1(x)))
        out = self.bn2(self.conv2(out))
        return F.relu(out + identity)


class ResNet20(Module):
    NAME = "resnet20"

    def __init__(self, num_classes: int = 10, device=None):
        super().__init__()
        self.conv1 = Conv2d(3, 16, 3, padding=1, bias=False, device=device)
        self.bn1 = BatchNorm2d(16, device=device)
        self.layer1 = torch.nn.ModuleList([BasicBlock(16, 16, 1, device) for _ in range(3)])
        self.layer2 = torch.nn.ModuleList([BasicBlock(16, 32, 2, device)] +
                                          [BasicBlock(32, 32, 1, device) for _ in range(2)])
        self.layer3 = torch.nn.ModuleList([BasicBlock(32, 64, 2, device)] +
                                          [BasicBlock(64, 64, 1, device) for _ in range(2)])
        self.fc = Linear(64, num_classes, device=device)
        dev = torch.device(device) if device is not None else torch.device("cpu")
        self._grad_anchor = torch.zeros((), device=dev, requires_grad=True)

    def move_to_device(self, device):
        super().move_to_device(device)
        self._grad_anchor = torch.zeros((), device=torch.device(device), requires_grad=True)
        return self

    def forward(self, x):
        x = F.relu(self.bn1(self.conv1(x)))
        for layer in (self.layer1, self.layer2, self.layer3):
            for b in layer:
                x = b(x)
        x = F.adaptive_avg_pool2d(x, 1).flatten(1)
        return self.fc(x)

    def loss(self, images, targets):
        """Mean cross-entropy (training-mode batch norm when ``self.training``)."""
        if images.is_cuda and self.training and torch.is_grad_enabled():
            return ops.resnet_train_loss(self, images, targets)
        return F.cross_entropy(self.forward(images).float(), targets)
