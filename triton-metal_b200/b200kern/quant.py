"""Weight-only quantized matmul ops (torch tensors in, torch tensors out).

These mirror the reference's INT4 / INT8 kernels:
  * int4_matmul  <- make_int4_matmul_kernel(group_size)
                    (triton_metal/codegen/_msl_templates.py:2682-2745)
  * int8_matmul  <- make_int8_matmul_kernel()
                    (triton_metal/codegen/_msl_templates.py:2630-2679)
The reference binds buffers in the order input, weight, output, scales,
zeros, M, N, K; these ops keep input, weight, scales, zeros in that order,
take the output as ``out=`` and read M, N, K from the shapes.

All compute runs in libb2.so on the caller's current CUDA stream.
"""
import torch

from . import _lib
from .errors import B2DtypeError, B2ShapeError

_DT = {torch.float16: 0, torch.bfloat16: 1}
_DTC = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}  # codes of the C ABI (fp32: reference dtype)
LAYOUT_GPTQ = "gptq"  # int32 [K/8, N], nibble j of a word holds k = 8*row + j
LAYOUT_REF = "ref"    # uint8 [N, K/2], low nibble = even k (the reference's)


def _stream():
    return _lib.current_stream()


def _check_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise B2ShapeError("b200kern ops take CUDA tensors (there is no CPU path)")


def _ptr(t):
    return None if t is None else t.data_ptr()


# --------------------------------------------------------------------------
# packing helpers (host-side layout conversion, plain torch)
# --------------------------------------------------------------------------
def pack_int4_gptq(q):
    """int [K, N] values 0..15 -> int32 [K/8, N]; nibble j of row r is k=8r+j."""
    K, N = q.shape
    if K % 8:
        raise B2ShapeError("K must be a multiple of 8")
    q = q.to(torch.int64).reshape(K // 8, 8, N)
    word = torch.zeros(K // 8, N, dtype=torch.int64, device=q.device)
    for j in range(8):
        word |= (q[:, j, :] & 0xF) << (4 * j)
    return (word - ((word >> 31) & 1) * (1 << 32)).to(torch.int32)


def unpack_int4_gptq(w):
    """int32 [K/8, N] -> int64 [K, N] nibble values 0..15."""
    w = w.to(torch.int64) & 0xFFFFFFFF
    parts = [(w >> (4 * j)) & 0xF for j in range(8)]
    return torch.stack(parts, dim=1).reshape(w.shape[0] * 8, w.shape[1])


def pack_int4_ref(q_nk):
    """int [N, K] values 0..15 -> uint8 [N, K/2], low nibble = even k
    (_msl_templates.py:2725-2732)."""
    q = q_nk.to(torch.int32)
    return ((q[:, 0::2] & 0xF) | ((q[:, 1::2] & 0xF) << 4)).to(torch.uint8)


# --------------------------------------------------------------------------
# ops
# --------------------------------------------------------------------------
def int4_matmul(input, weight, scales, zeros=None, group_size=128, layout=LAYOUT_GPTQ, out=None):
    """out[M, N] = input[M, K] @ ((q - z) * s), group-wise along K.

    layout="gptq": weight int32 [K/8, N]; scales (and zeros) [K/G, N].
    layout="ref":  weight uint8 [N, K/2] (the reference's buffer); scales
                   and zeros [N, K/G] as in _msl_templates.py:2693-2695.
                   Read natively by b2_int4_matmul_ref (no repack).
    zeros=None means the symmetric zero point 8.
    input fp16 / bf16 run the tensor-core kernels; fp32 input (the
    reference's dtype) runs with fp32 scales / zeros, the reference's fp32
    dequant (q - z) * s and fp32 products (no 16-bit rounding anywhere) and
    returns fp32.
    """
    # Common decode / prefill case, straight to the kernel with no conversion
    # or copy.  A decode step issues one of these per layer and the kernel
    # takes a few microseconds, so the argument checks run in C++ (_b2fast)
    # when it is built, else here reading each tensor attribute once.
    if zeros is None and layout == LAYOUT_GPTQ:
        fast = _lib.fast()
        if fast is not None:
            r = fast.int4_matmul(input, weight, scales, group_size, out)
            if r is not None:
                if r.__class__ is int:
                    _lib.check(r, "b2_int4_matmul")
                return r
    dti = input.dtype
    dt = _DT.get(dti)
    if (dt is not None and zeros is None and layout == LAYOUT_GPTQ and weight.dtype == torch.int32
            and scales.dtype == dti and input.is_cuda and weight.is_cuda and scales.is_cuda):
        ish, wsh = input.shape, weight.shape
        if (len(ish) == 2 and len(wsh) == 2 and input.is_contiguous() and weight.is_contiguous()
                and scales.is_contiguous()):
            M, K = ish
            N = wsh[1]
            if wsh[0] * 8 == K and K % group_size == 0 and scales.shape == (K // group_size, N):
                if (out is not None and out.dtype == dti and out.is_cuda and out.is_contiguous()
                        and out.shape == (M, N)):
                    res = out
                else:
                    res = torch.empty(M, N, dtype=dti, device=input.device)
                if M:
                    _lib.check(_lib.fn("b2_int4_matmul")(input.data_ptr(), weight.data_ptr(), res.data_ptr(),
                                                         scales.data_ptr(), None, M, N, K, group_size, dt,
                                                         _lib.current_stream()), "b2_int4_matmul")
                if out is not None and res is not out:
                    out.copy_(res)
                    return out
                return res
    _check_cuda(input, weight, scales, zeros)
    if input.dim() != 2:
        raise B2ShapeError(f"input must be [M, K], got {tuple(input.shape)}")
    M, K = input.shape
    if layout == LAYOUT_REF:
        if weight.dtype != torch.uint8 or weight.dim() != 2 or weight.shape[1] * 2 != K:
            raise B2ShapeError("ref layout weight must be uint8 [N, K/2]")
        N = weight.shape[0]
        if K % group_size or tuple(scales.shape) != (N, K // group_size):
            raise B2ShapeError(f"ref layout scales must be [N, K/G] = {(N, K // group_size)}")
        if zeros is not None and tuple(zeros.shape) != tuple(scales.shape):
            raise B2ShapeError("zeros must have the shape of scales")
        out_dtype = input.dtype
        cdt = input.dtype
        if cdt not in _DT and cdt != torch.float32:
            raise B2DtypeError(f"input dtype {input.dtype} unsupported (fp16, bf16, fp32)")
        x = input.to(cdt).contiguous()
        s = scales.to(cdt).contiguous()
        z = None if zeros is None else zeros.to(cdt).contiguous()
        res = torch.empty(M, N, dtype=cdt, device=input.device)
        if M:
            _lib.call("b2_int4_matmul_ref", _ptr(x), _ptr(weight.contiguous()), _ptr(res), _ptr(s), _ptr(z),
                      M, N, K, group_size, _DTC[cdt], _stream())
        res = res.to(out_dtype)
        if out is not None:
            out.copy_(res)
            return out
        return res
    elif layout != LAYOUT_GPTQ:
        raise B2ShapeError(f"unknown layout {layout!r}")
    if weight.dtype != torch.int32 or weight.dim() != 2 or weight.shape[0] * 8 != K:
        raise B2ShapeError(f"weight must be int32 [K/8, N] with K={K}, got {weight.dtype} {tuple(weight.shape)}")
    N = weight.shape[1]
    if K % group_size:
        raise B2ShapeError(f"group_size {group_size} must divide K={K}")
    if tuple(scales.shape) != (K // group_size, N):
        raise B2ShapeError(f"scales must be [K/G, N] = {(K // group_size, N)}, got {tuple(scales.shape)}")
    if zeros is not None and tuple(zeros.shape) != tuple(scales.shape):
        raise B2ShapeError("zeros must have the shape of scales")
    out_dtype = input.dtype
    cdt = input.dtype
    if cdt not in _DT and cdt != torch.float32:
        raise B2DtypeError(f"input dtype {input.dtype} unsupported (fp16, bf16, fp32)")
    x = input.to(cdt).contiguous()
    s = scales.to(cdt).contiguous()
    z = None if zeros is None else zeros.to(cdt).contiguous()
    w = weight.contiguous()
    if out is not None and (out.is_cuda and out.dtype == cdt and out.is_contiguous() and tuple(out.shape) == (M, N)):
        res = out
    else:
        res = torch.empty(M, N, dtype=cdt, device=input.device)
    if M == 0:
        return res.to(out_dtype)
    _lib.call("b2_int4_matmul", _ptr(x), _ptr(w), _ptr(res), _ptr(s), _ptr(z),
              M, N, K, group_size, _DTC[cdt], _stream())
    if res.dtype != out_dtype:
        res = res.to(out_dtype)
    if out is not None and res is not out:
        out.copy_(res)
        return out
    return res


def int4_dequant(weight, scales, zeros=None, group_size=128):
    """Exact fp32 dequantisation [K, N] of a GPTQ-layout int4 weight."""
    _check_cuda(weight, scales, zeros)
    K, N = weight.shape[0] * 8, weight.shape[1]
    if scales.dtype not in _DT:
        raise B2DtypeError("scales must be fp16 or bf16")
    out = torch.empty(K, N, dtype=torch.float32, device=weight.device)
    z = None if zeros is None else zeros.to(scales.dtype).contiguous()
    _lib.call("b2_int4_dequant", _ptr(weight.contiguous()), _ptr(scales.contiguous()), _ptr(z), _ptr(out),
              N, K, group_size, _DT[scales.dtype], _stream())
    return out


def int8_matmul(input, weight, scales, zeros=None, out=None):
    """out[M, N] = input[M, K] @ ((w8 - z) * s)^T with per-channel s, z [N].

    weight int8 [N, K] (the reference layout, _msl_templates.py:2640-2644).
    fp16 / bf16 input runs the tensor-core kernels; fp32 input runs the
    reference's fp32 arithmetic ((w - z) * s, fp32 products) and returns fp32.
    """
    _check_cuda(input, weight, scales, zeros)
    if input.dim() != 2 or weight.dim() != 2 or weight.dtype != torch.int8:
        raise B2ShapeError("int8_matmul takes input [M, K] and int8 weight [N, K]")
    M, K = input.shape
    N = weight.shape[0]
    if weight.shape[1] != K:
        raise B2ShapeError(f"weight K {weight.shape[1]} != input K {K}")
    if scales.numel() != N or (zeros is not None and zeros.numel() != N):
        raise B2ShapeError("scales / zeros must have N elements")
    out_dtype = input.dtype
    cdt = input.dtype
    if cdt not in _DT and cdt != torch.float32:
        raise B2DtypeError(f"input dtype {input.dtype} unsupported (fp16, bf16, fp32)")
    x = input.to(cdt).contiguous()
    s = scales.to(cdt).contiguous()
    z = None if zeros is None else zeros.to(cdt).contiguous()
    res = torch.empty(M, N, dtype=cdt, device=input.device)
    if M == 0:
        return res.to(out_dtype)
    _lib.call("b2_int8_matmul", _ptr(x), _ptr(weight.contiguous()), _ptr(res), _ptr(s), _ptr(z),
              M, N, K, _DTC[cdt], _stream())
    if res.dtype != out_dtype:
        res = res.to(out_dtype)
    if out is not None:
        out.copy_(res)
        return out
    return res


def gemm_bf16(x, w, out=None):
    """out[M, N] = x[M, K] @ w[N, K]^T on tcgen05 (bf16 in/out, fp32 accumulate).

    Needs N % 8 == 0 and K % 64 == 0 (any M)."""
    _check_cuda(x, w)
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or x.dim() != 2 or w.dim() != 2:
        raise B2DtypeError("gemm_bf16 takes bf16 x [M, K] and w [N, K]")
    M, K = x.shape
    N = w.shape[0]
    if w.shape[1] != K:
        raise B2ShapeError("K mismatch")
    res = (_lib.check_out(out, (M, N), torch.bfloat16, "gemm_bf16") if out is not None
           else torch.empty(M, N, dtype=torch.bfloat16, device=x.device))
    _lib.call("b2_gemm_bf16", _ptr(x.contiguous()), _ptr(w.contiguous()), _ptr(res), M, N, K, _stream())
    return res
