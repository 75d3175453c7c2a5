"""Helpers of the CPU oracle: ulp distance and the seeded synthetic inputs of the benchmark
configurations.  Test infrastructure only."""

from __future__ import annotations

import torch


def bf16_ulp_diff(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Distance in units of bf16 ulps between two bf16 tensors (monotone integer mapping)."""
    def key(t):
        i = t.detach().cpu().contiguous().view(torch.int16).to(torch.int32)
        return torch.where(i < 0, -(i & 0x7FFF), i)
    return (key(a) - key(b)).abs()


def make_config_inputs(name: str, rows: int | None = None, device="cpu", seed: int = 0) -> dict:
    """Seeded synthetic inputs with the shapes and value distributions of the five benchmark
    configurations ("c1" .. "c5"); ``rows`` overrides M (for bounded CPU samples and small parity
    cases).  For "c4", pass name "c4:N" (e.g. "c4:4096")."""
    g = torch.Generator(device="cpu").manual_seed(seed)

    def randn(*shape):
        return torch.randn(*shape, generator=g, dtype=torch.float32)

    if name == "c1":
        M, N = rows or 4096, 4096
        return dict(x=randn(M, N).to(device), weight=(1 + 0.1 * randn(N)).to(device), eps=1e-6)
    if name == "c2":
        M, N = rows or 32768, 8192
        bf = torch.bfloat16
        return dict(x=randn(M, N).to(bf).to(device), residual=randn(M, N).to(bf).to(device),
                    weight=(1 + 0.1 * randn(N)).to(bf).to(device),
                    dout=randn(M, N).to(bf).to(device), eps=1e-6)
    if name == "c3":
        M, N = rows or 65536, 4096
        bf = torch.bfloat16
        return dict(x=(0.5 + randn(M, N)).to(bf).to(device),
                    weight=(1 + 0.1 * randn(N)).to(bf).to(device),
                    bias=(0.1 * randn(N)).to(bf).to(device),
                    dout=randn(M, N).to(bf).to(device), eps=1e-5)
    if name.startswith("c4"):
        N = int(name.split(":")[1]) if ":" in name else 4096
        M = rows or (2 ** 31) // N
        bf = torch.bfloat16
        return dict(x=(3 * randn(M, N)).to(bf).to(device), dy=randn(M, N).to(bf).to(device))
    if name == "c5":
        M, N = rows or 16384, 128256
        bf = torch.bfloat16
        target = torch.randint(0, N, (M,), generator=g, dtype=torch.int64)
        ignore = torch.rand(M, generator=g) < 0.05
        target[ignore] = -100
        return dict(x=(2 * randn(M, N)).to(bf).to(device), target=target.to(device),
                    ignore_index=-100)
    raise ValueError(f"unknown config {name}")
