"""Small MLPs of the error-feedback and stochastic-rounding experiments.

* :class:`TinyMLP` — 64 -> 128 -> 128 -> 10 (reference
  benchmarks/error_feedback_comparison.py:73-88).
* :func:`tiny_mlp_sr` — 256 -> 512 -> 512 -> 10 (reference
  benchmarks/stochastic_rounding_e2e_curve.py:89-152).
"""

from __future__ import annotations

import torch
import torch.nn as nn


class TinyMLP(nn.Module):
    def __init__(self, in_dim: int = 64, hidden: int = 128, num_classes: int = 10):
        super().__init__()
        self.net = nn.Sequential(
            nn.Linear(in_dim, hidden),
            nn.ReLU(inplace=True),
            nn.Linear(hidden, hidden),
            nn.ReLU(inplace=True),
            nn.Linear(hidden, num_classes),
        )

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.net(x)


def tiny_mlp_sr() -> TinyMLP:
    return TinyMLP(256, 512, 10)


def toy_batch(batch: int, in_dim: int, num_classes: int, device, generator=None):
    """Synthetic, learnable classification batch: labels are the argmax of a
    fixed linear map of the inputs."""
    x = torch.randn(batch, in_dim, device=device, generator=generator)
    w = torch.linspace(-1.0, 1.0, in_dim, device=device).unsqueeze(1)
    w = w * torch.linspace(0.5, 1.5, num_classes, device=device).unsqueeze(0)
    y = torch.argmax(x @ w + torch.sin(x[:, :num_classes]), dim=1)
    return x, y
