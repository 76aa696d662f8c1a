"""KDA chunked gated-delta-rule forward (torch in/out, libb2.so compute).

No reference counterpart (triton-metal has no KDA); the signature and the
[B, T, H, D] layout follow flash-linear-attention's naive_chunk_kda, the
library that defines the operator.
"""
import torch

from . import _lib
from .errors import B2DtypeError, B2ShapeError

_DT = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}


def workspace_size(B, T, H, Dk=128, Dv=128, chunk_size=64):
    """Bytes of device scratch kda_chunk_fwd needs for this shape."""
    return int(_lib.load().b2_kda_workspace_size(B, T, H, Dk, Dv, chunk_size))


def kernels_per_call():
    """Kernels one kda_chunk_fwd call launches."""
    return 2


def kda_chunk_fwd(q, k, v, g, beta, scale=None, initial_state=None, output_final_state=True, chunk_size=64,
                  out=None, workspace=None, final_state_out=None):
    """o[B,T,H,Dv], final state [B,H,Dk,Dv] (fp32) of the gated delta rule.

    q, k [B,T,H,Dk], v [B,T,H,Dv] and beta [B,T,H] share one dtype (bf16,
    fp16 or fp32); g [B,T,H,Dk] fp32 log-decay; initial_state fp32 or None.
    workspace: optional uint8 CUDA tensor of workspace_size(...) bytes;
    final_state_out: optional fp32 [B,H,Dk,Dv] tensor for the final state."""
    for t in (q, k, v, g, beta):
        if not t.is_cuda:
            raise B2ShapeError("b200kern ops take CUDA tensors (there is no CPU path)")
    if q.dtype not in _DT or k.dtype != q.dtype or v.dtype != q.dtype or beta.dtype != q.dtype:
        raise B2DtypeError("q, k, v, beta must share one dtype (bf16, fp16, fp32)")
    if g.dtype != torch.float32:
        raise B2DtypeError("g (log-decay) must be fp32")
    B, T, H, Dk = q.shape
    Dv = v.shape[-1]
    if tuple(k.shape) != (B, T, H, Dk) or tuple(g.shape) != (B, T, H, Dk) or tuple(v.shape[:3]) != (B, T, H) \
            or tuple(beta.shape) != (B, T, H):
        raise B2ShapeError("shapes must be q,k,g [B,T,H,Dk], v [B,T,H,Dv], beta [B,T,H]")
    scale = Dk ** -0.5 if scale is None else float(scale)
    q, k, v, g, beta = (t.contiguous() for t in (q, k, v, g, beta))
    o = (_lib.check_out(out, (B, T, H, Dv), q.dtype, "kda_chunk_fwd") if out is not None
         else torch.empty(B, T, H, Dv, dtype=q.dtype, device=q.device))
    s_out = None
    if output_final_state:
        s_out = final_state_out
        if s_out is None:
            s_out = torch.empty(B, H, Dk, Dv, dtype=torch.float32, device=q.device)
        elif (not s_out.is_cuda or s_out.dtype != torch.float32 or tuple(s_out.shape) != (B, H, Dk, Dv)
              or not s_out.is_contiguous()):
            raise B2ShapeError("final_state_out must be a contiguous fp32 [B, H, Dk, Dv] tensor")
    s0 = None
    if initial_state is not None:
        s0 = initial_state.to(torch.float32).contiguous()
    need = workspace_size(B, T, H, Dk, Dv, chunk_size)
    if need == 0:
        raise B2ShapeError(f"unsupported KDA shape T={T} chunk={chunk_size}")
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    p = lambda t: None if t is None else t.data_ptr()
    _lib.call("b2_kda_fwd", p(q), p(k), p(v), p(g), p(beta), p(s0), p(o), p(s_out), p(workspace),
              B, T, H, Dk, Dv, chunk_size, scale, _DT[q.dtype], torch.cuda.current_stream().cuda_stream)
    return o, s_out
