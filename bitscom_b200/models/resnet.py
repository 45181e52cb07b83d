"""ResNet models used by the DDP benchmarks.

* :func:`resnet18_cifar` — ResNet-18 for 32x32 inputs: 3x3 stride-1 stem, no
  max-pool, 10-way head (the benchmark config of the low-bit DDP runs).
* :func:`resnet50` — ImageNet-shape ResNet-50 (7x7 stem, bottleneck blocks).

The reference used torchvision's resnet50 (reference
benchmarks/multimodel_stochastic_e2e_curve.py:42-45).  These modules are plain
torch.nn (cuDNN convolutions); for B200 they are meant to run channels_last
under bf16 autocast, which maps every convolution onto the tensor cores.
"""

from __future__ import annotations

from typing import List, Type, Union

import torch
import torch.nn as nn


def _conv3x3(cin: int, cout: int, stride: int = 1) -> nn.Conv2d:
    return nn.Conv2d(cin, cout, 3, stride=stride, padding=1, bias=False)


class BasicBlock(nn.Module):
    expansion = 1

    def __init__(self, cin: int, width: int, stride: int = 1):
        super().__init__()
        self.conv1 = _conv3x3(cin, width, stride)
        self.bn1 = nn.BatchNorm2d(width)
        self.conv2 = _conv3x3(width, width)
        self.bn2 = nn.BatchNorm2d(width)
        self.relu = nn.ReLU(inplace=True)
        self.down = None
        if stride != 1 or cin != width:
            self.down = nn.Sequential(nn.Conv2d(cin, width, 1, stride=stride, bias=False), nn.BatchNorm2d(width))

    def forward(self, x):
        idt = x if self.down is None else self.down(x)
        y = self.relu(self.bn1(self.conv1(x)))
        y = self.bn2(self.conv2(y))
        return self.relu(y + idt)


class Bottleneck(nn.Module):
    expansion = 4

    def __init__(self, cin: int, width: int, stride: int = 1):
        super().__init__()
        cout = width * self.expansion
        self.conv1 = nn.Conv2d(cin, width, 1, bias=False)
        self.bn1 = nn.BatchNorm2d(width)
        self.conv2 = _conv3x3(width, width, stride)
        self.bn2 = nn.BatchNorm2d(width)
        self.conv3 = nn.Conv2d(width, cout, 1, bias=False)
        self.bn3 = nn.BatchNorm2d(cout)
        self.relu = nn.ReLU(inplace=True)
        self.down = None
        if stride != 1 or cin != cout:
            self.down = nn.Sequential(nn.Conv2d(cin, cout, 1, stride=stride, bias=False), nn.BatchNorm2d(cout))

    def forward(self, x):
        idt = x if self.down is None else self.down(x)
        y = self.relu(self.bn1(self.conv1(x)))
        y = self.relu(self.bn2(self.conv2(y)))
        y = self.bn3(self.conv3(y))
        return self.relu(y + idt)


class ResNet(nn.Module):
    def __init__(
        self,
        block: Type[Union[BasicBlock, Bottleneck]],
        layers: List[int],
        num_classes: int,
        cifar_stem: bool,
    ):
        super().__init__()
        self.cin = 64
        if cifar_stem:
            self.stem = nn.Sequential(_conv3x3(3, 64), nn.BatchNorm2d(64), nn.ReLU(inplace=True))
        else:
            self.stem = nn.Sequential(
                nn.Conv2d(3, 64, 7, stride=2, padding=3, bias=False),
                nn.BatchNorm2d(64),
                nn.ReLU(inplace=True),
                nn.MaxPool2d(3, stride=2, padding=1),
            )
        stages = []
        for i, (width, n) in enumerate(zip((64, 128, 256, 512), layers)):
            blocks = []
            for j in range(n):
                stride = 2 if (i > 0 and j == 0) else 1
                blocks.append(block(self.cin, width, stride))
                self.cin = width * block.expansion
            stages.append(nn.Sequential(*blocks))
        self.layers = nn.Sequential(*stages)
        self.pool = nn.AdaptiveAvgPool2d(1)
        self.fc = nn.Linear(self.cin, num_classes)
        for m in self.modules():
            if isinstance(m, nn.Conv2d):
                nn.init.kaiming_normal_(m.weight, mode="fan_out", nonlinearity="relu")
            elif isinstance(m, nn.BatchNorm2d):
                nn.init.ones_(m.weight)
                nn.init.zeros_(m.bias)

    def forward(self, x):
        x = self.layers(self.stem(x))
        return self.fc(torch.flatten(self.pool(x), 1))


def resnet18_cifar(num_classes: int = 10) -> ResNet:
    """ResNet-18, CIFAR stem (3x3 conv, stride 1, no max-pool)."""
    return ResNet(BasicBlock, [2, 2, 2, 2], num_classes, cifar_stem=True)


def resnet50(num_classes: int = 1000) -> ResNet:
    """ResNet-50, ImageNet stem."""
    return ResNet(Bottleneck, [3, 4, 6, 3], num_classes, cifar_stem=False)
