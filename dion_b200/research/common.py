"""Shared pieces of the research harnesses: a bias-free 3-layer MLP, a
FashionMNIST-shaped dataset (real files when present, synthetic otherwise),
evaluation and the weight-direction cosine."""
from __future__ import annotations

import math
import os
from typing import Iterator, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

__all__ = ["MLP", "load_fmnist", "batches", "evaluate", "weight_cosines"]


class MLP(nn.Module):
    def __init__(self, hidden: int = 1024, d_in: int = 784, classes: int = 10):
        super().__init__()
        self.fc1 = nn.Linear(d_in, hidden, bias=False)
        self.fc2 = nn.Linear(hidden, hidden, bias=False)
        self.fc3 = nn.Linear(hidden, classes, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.fc3(torch.relu(self.fc2(torch.relu(self.fc1(x.view(x.size(0), -1))))))


def load_fmnist(data_dir: Optional[str] = "./data", seed: int = 0, n_train: int = 60000, n_test: int = 10000):
    """((x_train, y_train), (x_test, y_test), source); images normalised, [N, 784] fp32."""
    raw = os.path.join(data_dir or "", "FashionMNIST", "raw")
    if data_dir and os.path.isdir(raw):
        try:
            from torchvision import datasets

            tr = datasets.FashionMNIST(data_dir, train=True, download=False)
            te = datasets.FashionMNIST(data_dir, train=False, download=False)
            cv = lambda d: (((d.data.float() / 255.0 - 0.286) / 0.353).view(-1, 784), d.targets.clone())  # noqa: E731
            (xa, ya), (xb, yb) = cv(tr), cv(te)
            return (xa[:n_train], ya[:n_train]), (xb[:n_test], yb[:n_test]), "fashion_mnist"
        except Exception:  # noqa: BLE001
            pass
    g = torch.Generator().manual_seed(seed)
    templates = F.avg_pool2d(torch.rand(10, 1, 28, 28, generator=g), 5, 1, 2).view(10, 784)

    def make(n, off):
        gg = torch.Generator().manual_seed(seed + off)
        y = torch.randint(0, 10, (n,), generator=gg)
        x = templates[y] + 0.35 * torch.randn(n, 784, generator=gg)
        return (x - 0.5) / 0.35, y

    return make(n_train, 1), make(n_test, 2), "synthetic"


def batches(x: torch.Tensor, y: torch.Tensor, bs: int, seed: int) -> Iterator[Tuple[torch.Tensor, torch.Tensor]]:
    """Endless shuffled mini-batches (drop last)."""
    epoch = 0
    while True:
        perm = torch.randperm(x.size(0), generator=torch.Generator().manual_seed(seed * 1000 + epoch))
        for i in range(0, x.size(0) - bs + 1, bs):
            idx = perm[i:i + bs]
            yield x[idx], y[idx]
        epoch += 1


@torch.no_grad()
def evaluate(model: nn.Module, x: torch.Tensor, y: torch.Tensor, bs: int = 2048) -> Tuple[float, float, float]:
    model.eval()
    loss = correct = 0.0
    for i in range(0, x.size(0), bs):
        lo = model(x[i:i + bs])
        loss += float(F.cross_entropy(lo, y[i:i + bs], reduction="sum"))
        correct += float((lo.argmax(1) == y[i:i + bs]).sum())
    model.train()
    avg = loss / x.size(0)
    return avg, correct / x.size(0), math.exp(min(avg, 20))


def weight_cosines(a: nn.Module, b: nn.Module) -> dict:
    return {n: float(F.cosine_similarity(pa.detach().flatten(), pb.detach().flatten(), dim=0))
            for (n, pa), (_, pb) in zip(a.named_parameters(), b.named_parameters())}
