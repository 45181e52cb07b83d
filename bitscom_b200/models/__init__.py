"""Model definitions used by the benchmarks and end-to-end tests."""

from .gpt2 import GPT2, GPT2Config, gpt2_medium, gpt2_small_test
from .mlp import TinyMLP, tiny_mlp_sr, toy_batch
from .resnet import resnet18_cifar, resnet50

__all__ = [
    "GPT2", "GPT2Config", "gpt2_medium", "gpt2_small_test",
    "TinyMLP", "tiny_mlp_sr", "toy_batch", "resnet18_cifar", "resnet50",
]
