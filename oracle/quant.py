"""CPU oracle for the weight-only quantized matmuls (numpy).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference arm as the checker.  Never the product.

Restates the reference's arithmetic:
  * int4 unpack, reference layout uint8 [N, K/2]: even k in the low nibble,
    odd k in the high nibble  (triton_metal/codegen/_msl_templates.py:2723-2732)
  * int4 dequant w = (q - z) * s, group g = k / G
    (_msl_templates.py:2734-2737; reference CPU loop tests/test_emitter.py:6170-6185)
  * int8 dequant w = (w8 - z[n]) * s[n]  (_msl_templates.py:2668-2676;
    tests/test_emitter.py:6113-6124)
  * out = x @ W  accumulated in float64 here (the reference accumulates a
    Python float, i.e. float64, in its CPU loops).
The GPTQ layout int32 [K/8, N] (nibble j of a word = k % 8) is the
BASELINE layout of the decode/prefill configs.
"""
import numpy as np


def unpack_int4_ref(packed_nk2):
    """uint8 [N, K/2] -> int [N, K] nibble values (even k = low nibble)."""
    p = np.asarray(packed_nk2, dtype=np.uint8)
    lo = p & 0x0F
    hi = (p >> 4) & 0x0F
    out = np.empty((p.shape[0], p.shape[1] * 2), dtype=np.int64)
    out[:, 0::2] = lo
    out[:, 1::2] = hi
    return out


def pack_int4_ref(q_nk):
    q = np.asarray(q_nk, dtype=np.int64)
    return ((q[:, 0::2] & 0xF) | ((q[:, 1::2] & 0xF) << 4)).astype(np.uint8)


def unpack_int4_gptq(words_k8n):
    """int32 [K/8, N] -> int [K, N] nibble values."""
    w = np.asarray(words_k8n).astype(np.int64) & 0xFFFFFFFF
    k8, n = w.shape
    out = np.empty((k8, 8, n), dtype=np.int64)
    for j in range(8):
        out[:, j, :] = (w >> (4 * j)) & 0xF
    return out.reshape(k8 * 8, n)


def pack_int4_gptq(q_kn):
    q = np.asarray(q_kn, dtype=np.int64)
    k, n = q.shape
    q = q.reshape(k // 8, 8, n)
    w = np.zeros((k // 8, n), dtype=np.int64)
    for j in range(8):
        w |= (q[:, j, :] & 0xF) << (4 * j)
    return w.astype(np.uint32).view(np.int32)


def ref_to_gptq(packed_nk2):
    """Reference layout -> GPTQ layout (bit-exact repack)."""
    return pack_int4_gptq(unpack_int4_ref(packed_nk2).T)


def dequant_int4(q_kn, scales_gn, zeros_gn=None, group_size=128, dtype=np.float32):
    """W[k, n] = (q - z) * s with s/z [K/G, N]; z defaults to 8.

    In float32 the result is exact for fp16/bf16 scales: (q - z) is an
    integer in [-8, 15] (4 bits) and s has <= 11 significant bits.
    """
    q = np.asarray(q_kn, dtype=dtype)
    s = np.repeat(np.asarray(scales_gn, dtype=dtype), group_size, axis=0)
    z = 8.0 if zeros_gn is None else np.repeat(np.asarray(zeros_gn, dtype=dtype), group_size, axis=0)
    return ((q - z) * s).astype(dtype)


def int4_matmul(x_mk, q_kn, scales_gn, zeros_gn=None, group_size=128):
    """out[M, N] in float64 (reference CPU-loop precision)."""
    w = dequant_int4(q_kn, scales_gn, zeros_gn, group_size, dtype=np.float64)
    return np.asarray(x_mk, dtype=np.float64) @ w


def int4_matmul_ref_layout(x_mk, packed_nk2, scales_ng, zeros_ng, group_size):
    """The reference kernel's own signature and layouts (all fp32 buffers)."""
    q = unpack_int4_ref(packed_nk2).T
    return int4_matmul(x_mk, q, np.asarray(scales_ng).T, np.asarray(zeros_ng).T, group_size)


def int8_matmul(x_mk, w_nk, scales_n, zeros_n=None):
    w = np.asarray(w_nk, dtype=np.float64)
    z = 0.0 if zeros_n is None else np.asarray(zeros_n, dtype=np.float64)[:, None]
    wd = (w - z) * np.asarray(scales_n, dtype=np.float64)[:, None]
    return np.asarray(x_mk, dtype=np.float64) @ wd.T


def int4_matmul_fp32_torch(x, q_kn, scales, zeros=None, group_size=128, threads=None):
    """The reference's dequant-then-matmul in fp32 torch on the host cores
    (used as the timed CPU baseline; torch matmul uses all host threads)."""
    import torch
    if threads:
        torch.set_num_threads(threads)
    s = scales.float().repeat_interleave(group_size, dim=0)
    z = 8.0 if zeros is None else zeros.float().repeat_interleave(group_size, dim=0)
    w = (q_kn.float() - z) * s
    return x.float() @ w
