"""Seeded synthetic inputs with the BASELINE configs' shapes and value
distributions (generated on the CPU with torch.Generator, then moved).

C1  W4A16 decode GEMV: x fp16 [M, 4096] ~ N(0,1); q ~ U{0..15} packed
    int32 [512, 11008]; fp16 scales [32, 11008] = |N(0,1)|*0.02 + 1e-3.
C2  W4A16 prefill GEMM bf16: x [4096, 4096]; N = 14336; bf16 scales.
C2' W8A16: int8 [N, K] ~ U{-127..127}; scales |N(0,1)|*0.01 [N].
"""
import torch

from .quant import pack_int4_gptq


def w4_inputs(M, N, K, group_size=128, dtype=torch.float16, seed=0, device="cpu", zeros=False):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(dtype)
    q = torch.randint(0, 16, (K, N), generator=g, dtype=torch.int32)
    scales = (torch.randn(K // group_size, N, generator=g).abs() * 0.02 + 1e-3).to(dtype)
    z = None
    if zeros:
        z = torch.rand(K // group_size, N, generator=g).mul(8.0).to(dtype)
    qw = pack_int4_gptq(q)
    out = dict(x=x, q=q, qweight=qw, scales=scales, zeros=z)
    return {k: (v.to(device) if isinstance(v, torch.Tensor) else v) for k, v in out.items()}


def w8_inputs(M, N, K, dtype=torch.bfloat16, seed=0, device="cpu", zeros=False):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(dtype)
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int32).to(torch.int8)
    scales = (torch.randn(N, generator=g).abs() * 0.01).to(dtype)
    z = torch.empty(N).uniform_(-1, 1, generator=g).to(dtype) if zeros else None
    out = dict(x=x, w=w, scales=scales, zeros=z)
    return {k: (v.to(device) if isinstance(v, torch.Tensor) else v) for k, v in out.items()}
