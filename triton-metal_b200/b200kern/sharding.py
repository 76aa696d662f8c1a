"""Natural sharding across the GPUs of one box (one process per GPU).

* Quantized matmuls shard over N (output columns): GPTQ int4 weights
  [K/8, N] and their scales [K/G, N] along dim 1, int8 weights [N, K] along
  dim 0.  x is replicated; each rank's output [M, N/P] is independent.  An
  all-gather (NCCL over NVLink on GPUs, gloo on CPU) rebuilds [M, N] only when
  the caller wants replicated output.
* Attention and KDA shard over whole heads.  For GQA, shards are groups of
  kv heads with their Hq/Hkv query heads, so no rank needs another's K/V.
No collective is needed in the data path.
"""
import torch


def shard_range(n, world, rank, align=1):
    """[start, stop) of rank's share of n items, in multiples of `align`."""
    if n % align:
        raise ValueError(f"{n} items not a multiple of the alignment {align}")
    units = n // align
    base, rem = divmod(units, world)
    start = rank * base + min(rank, rem)
    stop = start + base + (1 if rank < rem else 0)
    return start * align, stop * align


def shard_int4(qweight, scales, zeros=None, world=1, rank=0, align=8):
    a, b = shard_range(qweight.shape[1], world, rank, align)
    z = None if zeros is None else zeros[:, a:b].contiguous()
    return qweight[:, a:b].contiguous(), scales[:, a:b].contiguous(), z, (a, b)


def shard_int8(weight, scales, zeros=None, world=1, rank=0, align=8):
    a, b = shard_range(weight.shape[0], world, rank, align)
    z = None if zeros is None else zeros[a:b].contiguous()
    return weight[a:b].contiguous(), scales[a:b].contiguous(), z, (a, b)


def shard_heads(q, k, v, world=1, rank=0, head_dim=1):
    """Split [.., H, ..] tensors by kv-head groups along `head_dim`
    (1 for [B, H, S, D], 2 for [B, T, H, D])."""
    hq, hkv = q.shape[head_dim], k.shape[head_dim]
    a, b = shard_range(hkv, world, rank)
    rep = hq // hkv
    sl = lambda t, lo, hi: t.narrow(head_dim, lo, hi - lo).contiguous()
    return sl(q, a * rep, b * rep), sl(k, a, b), sl(v, a, b), (a, b)


def all_gather_columns(out_shard, group=None):
    """[M, N/P] per rank -> [M, N] on every rank (shards may differ in width)."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    widths = [torch.zeros(1, dtype=torch.int64, device=out_shard.device) for _ in range(world)]
    dist.all_gather(widths, torch.tensor([out_shard.shape[1]], device=out_shard.device), group=group)
    wmax = int(max(w.item() for w in widths))
    pad = torch.zeros(out_shard.shape[0], wmax, dtype=out_shard.dtype, device=out_shard.device)
    pad[:, : out_shard.shape[1]] = out_shard
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    return torch.cat([p[:, : int(w.item())] for p, w in zip(parts, widths)], dim=1)


def all_gather_columns_stacked(out_shard, out=None, group=None):
    """Equal-width column shards [M, N/P] -> [P, M, N/P] on every rank with one
    all_gather_into_tensor (NCCL over NVLink on GPUs), no padding or copy;
    columns_from_stacked() gives the [M, N] view when the caller needs it."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    if out is None:
        out = torch.empty((world,) + tuple(out_shard.shape), dtype=out_shard.dtype, device=out_shard.device)
    # the concatenated [P * M, N/P] form, accepted by every backend
    dist.all_gather_into_tensor(out.view(world * out_shard.shape[0], -1), out_shard.contiguous(), group=group)
    return out


def columns_from_stacked(stacked):
    """[P, M, N/P] -> [M, N] (column block r = rank r's shard)."""
    P, M, W = stacked.shape
    return stacked.permute(1, 0, 2).reshape(M, P * W)

