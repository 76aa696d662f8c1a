"""Parity of the tcgen05 prefill GEMMs (bf16, W8A16, W4A16) through the C ABI.

Floating-point kernels, compared with an fp32 torch reference of the same op
(dequantised weights exact in fp32); the BASELINE C2 shapes are checked on
sampled rows against the float64 CPU oracle.

Tolerances (rtol = atol = 1e-2):
  * bf16 GEMM and W8A16: element-wise |out - ref| <= 1e-2 + 1e-2 |ref|
    (int8 weights are exact in bf16; the channel scale is applied in fp32).
  * W4A16: the tensor-core operand is the bf16-rounded (q - 8) * s (12
    significant bits needed, 8 kept), so every output carries an absolute
    error ~ 2^-9 / sqrt(3) * rms(out) (rounding errors add like sqrt(K), as
    does rms(out)).  Asserted element-wise with atol in units of the output
    RMS: |out - ref| <= 1e-2 * (|ref| + rms(ref))."""
import numpy as np
import pytest
import torch

from oracle import quant as oq

pytestmark = pytest.mark.gpu


def _close(out, ref, tol=1e-2):
    out = out.float()
    ref = ref.float()
    err = (out - ref).abs()
    bound = tol + tol * ref.abs()
    assert bool((err <= bound).all()), f"max err {err.max().item():.4g}, worst ratio {(err / bound).max().item():.3g}"


def _close_w4(out, ref, tol=1e-2):
    out = out.float()
    ref = ref.float()
    err = (out - ref).abs()
    rms = ref.pow(2).mean().sqrt()
    bound = tol * (ref.abs() + rms)
    assert bool((err <= bound).all()), f"max err {err.max().item():.4g}, worst ratio {(err / bound).max().item():.3g}"


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 256), (512, 768, 1024), (1024, 2048, 512)])
def test_gemm_bf16(cuda, M, N, K):
    import b200kern as bk
    g = torch.Generator().manual_seed(M + N + K)
    x = torch.randn(M, K, generator=g).bfloat16().to(cuda)
    w = (torch.randn(N, K, generator=g) / K ** 0.5).bfloat16().to(cuda)
    out = bk.gemm_bf16(x, w)
    ref = x.float() @ w.float().t()
    _close(out, ref)


@pytest.mark.parametrize("M,N,K,G", [(128, 256, 128, 128), (256, 512, 512, 128), (384, 1024, 1024, 64),
                                     (256, 256, 2048, 256)])
def test_w4_gemm(cuda, M, N, K, G):
    import b200kern as bk
    from b200kern.synthetic import w4_inputs
    d = w4_inputs(M, N, K, group_size=G, dtype=torch.bfloat16, seed=M + K)
    out = bk.int4_matmul(d["x"].to(cuda), d["qweight"].to(cuda), d["scales"].to(cuda), group_size=G)
    wd = bk.int4_dequant(d["qweight"].to(cuda), d["scales"].to(cuda), None, G)
    ref = d["x"].to(cuda).float() @ wd
    _close_w4(out, ref)


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 512), (512, 1024, 1024)])
def test_w8_gemm(cuda, M, N, K):
    import b200kern as bk
    from b200kern.synthetic import w8_inputs
    d = w8_inputs(M, N, K, dtype=torch.bfloat16, seed=M + K)
    out = bk.int8_matmul(d["x"].to(cuda), d["w"].to(cuda), d["scales"].to(cuda))
    ref = d["x"].to(cuda).float() @ (d["w"].to(cuda).float() * d["scales"].to(cuda).float()[:, None]).t()
    _close(out, ref)


def test_w4_gemm_c2_sampled_rows(cuda):
    """BASELINE C2 (4096 x 4096 x 14336, G=128) vs the float64 oracle on 16 rows."""
    import b200kern as bk
    from b200kern.synthetic import w4_inputs
    d = w4_inputs(4096, 14336, 4096, group_size=128, dtype=torch.bfloat16, seed=0)
    out = bk.int4_matmul(d["x"].to(cuda), d["qweight"].to(cuda), d["scales"].to(cuda))
    rows = torch.arange(0, 4096, 257)[:16]
    ref = oq.int4_matmul(d["x"][rows].double().numpy(), d["q"].numpy(), d["scales"].double().numpy(), None, 128)
    _close_w4(out[rows].cpu(), torch.from_numpy(ref))


def test_w8_gemm_c2_sampled_rows(cuda):
    import b200kern as bk
    from b200kern.synthetic import w8_inputs
    d = w8_inputs(4096, 14336, 4096, dtype=torch.bfloat16, seed=0)
    out = bk.int8_matmul(d["x"].to(cuda), d["w"].to(cuda), d["scales"].to(cuda))
    rows = torch.arange(0, 4096, 257)[:16]
    ref = oq.int8_matmul(d["x"][rows].double().numpy(), d["w"].numpy(), d["scales"].double().numpy())
    _close(out[rows].cpu(), torch.from_numpy(ref))


def test_gemm_no_bounded_wait_ran_out(cuda):
    import ctypes
    from b200kern import _lib
    code = ctypes.c_uint(0)
    st = _lib.load().b2_device_error(torch.cuda.current_stream().cuda_stream, ctypes.byref(code))
    assert st == 0 and code.value == 0, hex(code.value)


# ---------------------------------------------------------------------------
# fp16 activations, asymmetric zeros, ragged M / N, the reference's fp32
# dtype and [N, K/2] layout on the GEMM path (M > 16).  The dequantised
# operand is rounded to the activation dtype (with zeros: fma(q, s, -z*s)
# or (w - z) rounded once), so these use the RMS-scaled bound.
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("zeros", [False, True])
@pytest.mark.parametrize("M,N,K,G", [(256, 512, 512, 128), (200, 264, 256, 64), (17, 1000, 1024, 128)])
def test_w4_gemm_variants(cuda, dtype, zeros, M, N, K, G):
    import b200kern as bk
    from b200kern.synthetic import w4_inputs
    d = w4_inputs(M, N, K, group_size=G, dtype=dtype, seed=M + N, zeros=zeros)
    z = None if d["zeros"] is None else d["zeros"].to(cuda)
    out = bk.int4_matmul(d["x"].to(cuda), d["qweight"].to(cuda), d["scales"].to(cuda), z, group_size=G)
    assert out.dtype == dtype and tuple(out.shape) == (M, N)
    wd = bk.int4_dequant(d["qweight"].to(cuda), d["scales"].to(cuda), z, G)
    ref = d["x"].to(cuda).float() @ wd
    _close_w4(out, ref)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("zeros", [False, True])
@pytest.mark.parametrize("M,N,K", [(256, 512, 512), (130, 72, 192)])
def test_w8_gemm_variants(cuda, dtype, zeros, M, N, K):
    import b200kern as bk
    from b200kern.synthetic import w8_inputs
    d = w8_inputs(M, N, K, dtype=dtype, seed=M + N, zeros=zeros)
    z = None if d["zeros"] is None else d["zeros"].to(cuda)
    out = bk.int8_matmul(d["x"].to(cuda), d["w"].to(cuda), d["scales"].to(cuda), z)
    assert out.dtype == dtype
    zf = 0.0 if z is None else z.float()[:, None]
    ref = d["x"].to(cuda).float() @ ((d["w"].to(cuda).float() - zf) * d["scales"].to(cuda).float()[:, None]).t()
    _close_w4(out, ref)


@pytest.mark.parametrize("M,N,K", [(200, 264, 128), (1, 8, 64), (333, 1000, 640)])
def test_gemm_bf16_ragged(cuda, M, N, K):
    import b200kern as bk
    g = torch.Generator().manual_seed(M * N)
    x = torch.randn(M, K, generator=g).bfloat16().to(cuda)
    w = (torch.randn(N, K, generator=g) / K ** 0.5).bfloat16().to(cuda)
    _close(bk.gemm_bf16(x, w), x.float() @ w.float().t())


def test_w4_gemm_reference_dtype_and_layout(cuda):
    """The reference's own buffers: fp32 input, uint8 [N, K/2] weight with
    low nibble = even k, fp32 scales / zeros [N, K/G], M = 64 rows (GEMM
    path), against the float64 oracle of _msl_templates.py:2716-2743."""
    import b200kern as bk
    g = torch.Generator().manual_seed(4242)
    M, N, K, G = 64, 768, 512, 128
    x = torch.randn(M, K, generator=g)
    q = torch.randint(0, 16, (N, K), generator=g, dtype=torch.int32)
    s = torch.rand(N, K // G, generator=g) * 0.05 + 0.01
    z = torch.randint(0, 16, (N, K // G), generator=g).float()
    w = bk.pack_int4_ref(q)
    out = bk.int4_matmul(x.to(cuda), w.to(cuda), s.to(cuda), z.to(cuda), group_size=G, layout="ref")
    assert out.dtype == torch.float32
    ref = oq.int4_matmul(x.double().numpy(), q.t().numpy(), s.t().double().numpy(), z.t().double().numpy(), G)
    _close_w4(out.cpu(), torch.from_numpy(ref))
