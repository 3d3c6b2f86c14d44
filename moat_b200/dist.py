"""Column sharding of M (and of heads for attention) across GPUs, one process per GPU.

The reference is single-device; this module adds the multi-GPU layout that
``BASELINE.json`` asks for. Each rank owns a group-aligned range of output columns
(whole 32-wide quantization groups, so every shard's q and scales are bit-identical
to the unsharded weight) re-packed as its own super-block stream, computes
``[N, M_r]`` with the local kernel, and the shards are joined with one all-gather
(NCCL over NVLink on GPUs; gloo in the CPU tests). Attention shards heads the same
way; no reduction crosses GPUs inside the softmax.
"""

from __future__ import annotations

from typing import Callable, List, Sequence, Tuple

GROUP = 32


def column_bounds(M: int, world: int, K: int | None = None, group: int = GROUP) -> List[Tuple[int, int]]:
    """Split M columns into ``world`` contiguous ranges of whole groups, as even as
    possible (the first ``groups % world`` ranks get one extra group)."""
    if M % group != 0:
        raise ValueError(f"M={M} is not a multiple of the group size {group}")
    if world < 1:
        raise ValueError("world must be >= 1")
    groups = M // group
    if groups < world:
        raise ValueError(f"cannot split {groups} groups over {world} ranks")
    base, rem = divmod(groups, world)
    out, c = [], 0
    for r in range(world):
        w = (base + (1 if r < rem else 0)) * group
        out.append((c, c + w))
        c += w
    if K is not None:
        for c0, c1 in out:
            if (K * (c1 - c0)) % 256 != 0:
                raise ValueError(f"shard [{c0},{c1}) x K={K} is not a whole number of super-blocks")
    return out


def head_bounds(H: int, world: int) -> List[Tuple[int, int]]:
    """Contiguous, as-even-as-possible head ranges."""
    if H < world:
        raise ValueError(f"cannot split {H} heads over {world} ranks")
    base, rem = divmod(H, world)
    out, h = [], 0
    for r in range(world):
        w = base + (1 if r < rem else 0)
        out.append((h, h + w))
        h += w
    return out


def gather_columns(local, bounds: Sequence[Tuple[int, int]], group=None):
    """All-gather column shards ``local [N, M_r]`` into ``[N, M]`` on every rank.

    Shards are padded to the widest one so one ``all_gather_into_tensor`` suffices.
    """
    import torch
    import torch.distributed as dist

    world = len(bounds)
    N = local.shape[0]
    wmax = max(c1 - c0 for c0, c1 in bounds)
    if local.shape[1] == wmax:
        send = local.contiguous()
    else:
        send = torch.zeros((N, wmax), dtype=local.dtype, device=local.device)
        send[:, :local.shape[1]] = local
    # flat [world * N, wmax] receive buffer: the layout every backend accepts
    recv = torch.empty((world * N, wmax), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(recv, send, group=group)
    recv = recv.view(world, N, wmax)
    M = bounds[-1][1]
    if all(c1 - c0 == wmax for c0, c1 in bounds):
        return recv.permute(1, 0, 2).reshape(N, M)
    out = torch.empty((N, M), dtype=local.dtype, device=local.device)
    for r, (c0, c1) in enumerate(bounds):
        out[:, c0:c1] = recv[r, :, :c1 - c0]
    return out


def gather_heads(local, bounds: Sequence[Tuple[int, int]], group=None):
    """All-gather head shards ``local [T, H_r, d]`` into ``[T, H, d]``."""
    import torch
    import torch.distributed as dist

    world = len(bounds)
    T, _, d = local.shape
    hmax = max(h1 - h0 for h0, h1 in bounds)
    send = local.contiguous()
    if local.shape[1] != hmax:
        send = torch.zeros((T, hmax, d), dtype=local.dtype, device=local.device)
        send[:, :local.shape[1]] = local
    recv = torch.empty((world * T, hmax, d), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(recv, send, group=group)
    recv = recv.view(world, T, hmax, d)
    H = bounds[-1][1]
    if all(h1 - h0 == hmax for h0, h1 in bounds):  # equal shards: one transposing copy
        return recv.transpose(0, 1).reshape(T, H, d)
    out = torch.empty((T, H, d), dtype=local.dtype, device=local.device)
    for r, (h0, h1) in enumerate(bounds):
        out[:, h0:h1] = recv[r, :, :h1 - h0]
    return out


class ColumnShardedGemm:
    """Column-parallel INT4 GEMM: this rank's [K, M_r] shard, local kernel, all-gather.

    ``superblocks`` is the full packed [K, M] weight (any device); only this rank's
    columns are kept (re-packed on the GPU, bit-identical). ``local_fn`` computes
    ``x [N, K] -> [N, M_r]`` for a shard stream; it defaults to the CUDA kernel.
    """

    def __init__(self, superblocks, K: int, M: int, rank: int, world: int, group=None,
                 local_fn: Callable | None = None):
        self.K, self.M, self.rank, self.world, self.group = K, M, rank, world, group
        self.bounds = column_bounds(M, world, K)
        self.c0, self.c1 = self.bounds[rank]
        if local_fn is None:
            from .dequant import extract_columns
            from .gemm import batched_gemm
            self.local_sb = extract_columns(superblocks, K, M, self.c0, self.c1)
            self._fn = lambda x: batched_gemm(x, self.local_sb, K, self.c1 - self.c0)
        else:
            self.local_sb = superblocks
            self._fn = local_fn

    def local(self, x):
        return self._fn(x)

    def __call__(self, x):
        return gather_columns(self.local(x), self.bounds, self.group)


class HeadShardedAttention:
    """Head-parallel LUT decode attention: this rank's heads, local kernel, all-gather."""

    def __init__(self, H: int, rank: int, world: int, group=None, local_fn: Callable | None = None):
        self.bounds = head_bounds(H, world)
        self.h0, self.h1 = self.bounds[rank]
        self.group = group
        if local_fn is None:
            from .attention import decode_attention
            local_fn = decode_attention
        self._fn = local_fn

    def __call__(self, q_local, k_local, v_local, exp_lut, scale=None):
        return gather_heads(self._fn(q_local, k_local, v_local, exp_lut, scale), self.bounds, self.group)
