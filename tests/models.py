"""Small torch modules used by the planner and compile tests (same shapes of
computation as the reference's test modules and the benchmark workloads)."""

import torch
import torch.nn.functional as F
from torch import nn


class Attn(nn.Module):
    def __init__(self, scale=0.25):
        super().__init__()
        self.scale = scale

    def forward(self, q, k, v):
        s = torch.matmul(q, k.transpose(-2, -1)) * self.scale
        return torch.matmul(torch.softmax(s, dim=-1), v)


class Chain(nn.Module):
    def __init__(self):
        super().__init__()
        self.b = nn.Parameter(torch.randn(8, 16))

    def forward(self, x):
        return torch.exp(torch.relu(x * 2.0 + self.b) * 0.1)


class SoftmaxChain(nn.Module):
    def forward(self, x):
        return torch.relu(torch.softmax(x * 0.5, dim=-1))


class RowChain(nn.Module):
    def forward(self, x, bias):
        return torch.softmax(torch.relu(x * 0.5 + bias), dim=-1) * 2.0


class BroadcastChain(nn.Module):
    """y = relu((x + b) * s) * 0.5 + x with per-column b, s (the chain workload)."""

    def forward(self, x, b, s):
        return torch.relu((x + b) * s) * 0.5 + x


class BertBlock(nn.Module):
    """BERT-base-style encoder block: Linear/LayerNorm stay torch steps, attention
    fuses to fp_attention, bias+GELU and the two bias+residual adds fuse to chains."""

    def __init__(self, batch, seq, hidden=768, heads=12, ffn=3072):
        super().__init__()
        self.B, self.S, self.H, self.D = batch, seq, heads, hidden // heads
        self.q, self.k, self.v = (nn.Linear(hidden, hidden) for _ in range(3))
        self.o = nn.Linear(hidden, hidden)
        self.ln1, self.ln2 = nn.LayerNorm(hidden), nn.LayerNorm(hidden)
        self.fc1, self.fc2 = nn.Linear(hidden, ffn), nn.Linear(ffn, hidden)
        self.scale = self.D ** -0.5

    def forward(self, x):
        B, S, H, D = self.B, self.S, self.H, self.D
        q = self.q(x).view(B, S, H, D).transpose(1, 2)
        k = self.k(x).view(B, S, H, D).transpose(1, 2)
        v = self.v(x).view(B, S, H, D).transpose(1, 2)
        a = torch.matmul(torch.softmax(torch.matmul(q, k.transpose(-2, -1)) * self.scale, dim=-1), v)
        a = a.transpose(1, 2).reshape(B, S, H * D)
        h = self.ln1(x + self.o(a))
        f = F.gelu(self.fc1(h))
        return self.ln2(h + self.fc2(f))


def init_bert(m: nn.Module, seed: int = 0) -> nn.Module:
    """Weights ~ N(0, 0.02), biases 0 (the BERT-block workload's initialisation)."""
    g = torch.Generator().manual_seed(seed)
    for mod in m.modules():
        if isinstance(mod, nn.Linear):
            with torch.no_grad():
                mod.weight.copy_(torch.randn(mod.weight.shape, generator=g) * 0.02)
                mod.bias.zero_()
    return m
