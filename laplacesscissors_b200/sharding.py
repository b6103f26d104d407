"""Multi-GPU partitioning of readout validation (one process per GPU).

Validation rows are independent, so they shard by row with no data-path
collective; per-row results meet on every rank with one all-gather.  The vocab
can also be split: each rank then holds one block of lm_head rows, computes per
hidden row its best competitor key and (when it owns the target) the target
logit, and one max-reduction of the packed keys and of the target logits gives
the full-vocabulary margin and argmax.  Key packing and tie rules are those of
argmax / other / minimum_margin (src/diagnosis.rs:58-80, 490-492).

The collectives go through torch.distributed (NCCL between GPUs, gloo on CPU).
"""
from __future__ import annotations

import numpy as np


def row_shard(total: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [lo, hi) of `rank` when `total` rows split into `world` nearly equal
    contiguous shards (the first total % world shards hold one more row)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank out of range")
    base, extra = divmod(total, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def vocab_shard(vocab: int, world: int, rank: int) -> tuple[int, int]:
    """lm_head rows [v0, v1) held by `rank` (same split as rows)."""
    return row_shard(vocab, world, rank)


def _device_of(group):
    import torch
    import torch.distributed as dist
    return torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" else torch.device("cpu")


def gather_rows(parts: dict[str, np.ndarray], total: int, group=None) -> dict[str, np.ndarray]:
    """All-gathers per-row arrays computed on row shards (row_shard order) so every
    rank holds all `total` rows.  Arrays of one name share dtype on all ranks."""
    import torch
    import torch.distributed as dist
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    device = _device_of(group)
    sizes = [row_shard(total, world, r) for r in range(world)]
    width = max(hi - lo for lo, hi in sizes)
    out = {}
    for name in sorted(parts):
        local = np.ascontiguousarray(parts[name])
        lo, hi = sizes[rank]
        if local.shape[0] != hi - lo:
            raise ValueError(f"{name}: {local.shape[0]} rows on rank {rank}, expected {hi - lo}")
        raw = local.view(np.uint8).reshape(local.shape[0], -1)
        row_bytes = raw.shape[1]
        buf = np.zeros((width, row_bytes), dtype=np.uint8)
        buf[: raw.shape[0]] = raw
        send = torch.from_numpy(buf).to(device)
        recv = [torch.empty_like(send) for _ in range(world)]
        dist.all_gather(recv, send, group=group)
        rows = [recv[r].cpu().numpy()[: hi_r - lo_r] for r, (lo_r, hi_r) in enumerate(sizes)]
        out[name] = np.concatenate(rows, axis=0).reshape(-1).view(local.dtype).reshape((total,) + local.shape[1:])
    return out


def pack_key(value: np.ndarray, index: np.ndarray) -> np.ndarray:
    """(total-order f32 | ~index) as uint64: the larger key is the larger value,
    and on equal values the lower index (the first maximum)."""
    bits = np.ascontiguousarray(value, dtype=np.float32).view(np.uint32).astype(np.uint64)
    order = np.where(bits & 0x80000000, (~bits) & 0xFFFFFFFF, bits | 0x80000000).astype(np.uint64)
    return (order << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - index.astype(np.uint64))


def unpack_key(key: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    key = np.asarray(key, dtype=np.uint64)
    order = (key >> np.uint64(32)).astype(np.uint32)
    bits = np.where(order & 0x80000000, order & 0x7FFFFFFF, ~order).astype(np.uint32)
    index = (np.uint64(0xFFFFFFFF) - (key & np.uint64(0xFFFFFFFF))).astype(np.uint32)
    return bits.view(np.float32), index


def shard_partials(logits: np.ndarray, targets: np.ndarray, v0: int) -> tuple[np.ndarray, np.ndarray]:
    """Per-row partials of one vocab shard from its logits [rows, v1 - v0]: the
    packed key of the best column other than the target, and the target's logit
    (-inf when the target lies outside the shard)."""
    z = np.asarray(logits, dtype=np.float32)
    rows, width = z.shape
    local = targets.astype(np.int64) - v0
    inside = (local >= 0) & (local < width)
    masked = z.copy()
    masked[np.nonzero(inside)[0], local[inside]] = -np.inf
    idx = np.argmax(masked, axis=1)  # first maximum
    keys = pack_key(masked[np.arange(rows), idx], idx + v0)
    tl = np.full(rows, -np.inf, dtype=np.float32)
    tl[inside] = z[np.nonzero(inside)[0], local[inside]]
    return keys, tl


def pack_partials(keys: np.ndarray, target_logit: np.ndarray) -> np.ndarray:
    """The packed partials of lsx_readout_partials_device from (keys, target
    logits): int64 [2 n], the keys with their top bit flipped, then the target
    logits' total-order keys; an element-wise signed maximum merges shards."""
    k = (np.asarray(keys, dtype=np.uint64) ^ np.uint64(1 << 63)).view(np.int64)
    bits = np.ascontiguousarray(target_logit, dtype=np.float32).view(np.uint32).astype(np.uint64)
    order = np.where(bits & 0x80000000, (~bits) & 0xFFFFFFFF, bits | 0x80000000).astype(np.int64)
    return np.concatenate([k, order])


def unpack_partials(partials: np.ndarray, targets: np.ndarray):
    """(margin f64, first argmax u32, target logit f32) from merged packed partials."""
    p = np.asarray(partials, dtype=np.int64)
    n = p.size // 2
    other, other_idx = unpack_key(p[:n].view(np.uint64) ^ np.uint64(1 << 63))
    order = p[n:].astype(np.uint64)
    bits = np.where(order & 0x80000000, order & 0x7FFFFFFF, (~order) & 0xFFFFFFFF).astype(np.uint32)
    tl = bits.view(np.float32)
    tgt = np.asarray(targets, dtype=np.uint32)
    amax = np.where((tl > other) | ((tl == other) & (tgt < other_idx)), tgt, other_idx).astype(np.uint32)
    return tl.astype(np.float64) - other.astype(np.float64), amax, tl


def merge_partials_(keys, target_logit, group=None) -> None:
    """In-place max-merge of vocabulary-shard partials across `group`: `keys` is an
    int64 tensor holding the bits of the packed unsigned keys, `target_logit` f32.
    One all-reduce MAX over [keys | target logits] as signed int64: the keys with
    their sign bit flipped (so signed order is their unsigned order), the target
    logits as their f32 total-order keys (non-negative, so the maximum key is the
    maximum logit).  Runs on the tensors' device (NCCL for CUDA tensors, gloo on
    CPU) and on the current stream."""
    import torch
    import torch.distributed as dist
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return
    n = keys.numel()
    flip = torch.tensor(-(1 << 63), dtype=torch.int64, device=keys.device)
    bits = target_logit.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    order = torch.where(bits >= 0x80000000, bits ^ 0xFFFFFFFF, bits | 0x80000000)
    both = torch.cat([keys ^ flip, order])
    dist.all_reduce(both, op=dist.ReduceOp.MAX, group=group)
    keys.copy_(both[:n] ^ flip)
    order = both[n:]
    bits = torch.where(order >= 0x80000000, order & 0x7FFFFFFF, order ^ 0xFFFFFFFF)
    target_logit.copy_(bits.to(torch.int32).view(torch.float32))


def merge_vocab_partials(keys: np.ndarray, target_logit: np.ndarray, targets: np.ndarray, group=None):
    """Max-reduces the shards' packed competitor keys and target logits across the
    group and returns (margin f64, first argmax u32, target logit f32) per row."""
    import torch
    device = _device_of(group)
    k = torch.from_numpy(np.ascontiguousarray(keys, dtype=np.uint64).view(np.int64).copy()).to(device)
    t = torch.from_numpy(np.ascontiguousarray(target_logit, dtype=np.float32).copy()).to(device)
    merge_partials_(k, t, group)
    k = k.cpu().numpy().view(np.uint64)
    tl = t.cpu().numpy()
    other, other_idx = unpack_key(k)
    margin = tl.astype(np.float64) - other.astype(np.float64)
    tgt = np.asarray(targets, dtype=np.uint32)
    # the target is the argmax when it beats the best other, or ties it with a lower index
    amax = np.where((tl > other) | ((tl == other) & (tgt < other_idx)), tgt, other_idx).astype(np.uint32)
    return margin, amax, tl


def vocab_sharded_margin(gpu, weight_shard, bias_shard, vocab_offset: int, shard_vocab: int, width: int,
                         hidden_ptr: int, hidden_kind: int, rows: int, targets_ptr: int, rotation=None, group=None,
                         workspace=None, partials=None, outputs=None):
    """Readout validation with the lm_head split by rows across the ranks of
    `group` (one GPU per rank), on device-resident inputs.

    This rank holds lm_head rows [vocab_offset, vocab_offset + shard_vocab)
    (`weight_shard`, a BF16 Tensor) and scores every hidden row against them with
    lsx_readout_partials_device, which leaves the shard's per-row partials in one
    signed-orderable int64 buffer [2 x rows]; one NCCL all-reduce MAX of that
    buffer merges the shards, and lsx_readout_partials_merge_device turns the
    merged partials into margins and first argmaxes.  All work is ordered on the
    library's stream; nothing runs between the kernels and the collective.
    `hidden_ptr` / `targets_ptr` are device addresses ([rows, width] of
    `hidden_kind`; global target ids as u32).  `workspace`, `partials` (int64
    [2 * rows]) and `outputs` (margin f64, argmax int32, target logit f32, each
    [rows]) may be passed in to reuse buffers.  Returns the output tensors."""
    import ctypes as C

    import torch
    import torch.distributed as dist

    from ._lib import check, lib
    dev = torch.device("cuda", gpu.device)
    rot = rotation.handle if rotation is not None else None
    stream = torch.cuda.ExternalStream(gpu.stream(), device=dev)
    with torch.cuda.stream(stream):
        if workspace is None:
            workspace = torch.empty(lib.lsx_readout_workspace_bytes(shard_vocab, width, rows, rot),
                                    dtype=torch.uint8, device=dev)
        if partials is None:
            partials = torch.empty(2 * rows, dtype=torch.int64, device=dev)
        if outputs is None:
            outputs = (torch.empty(rows, dtype=torch.float64, device=dev),
                       torch.empty(rows, dtype=torch.int32, device=dev),
                       torch.empty(rows, dtype=torch.float32, device=dev))
        check(lib.lsx_readout_partials_device(gpu.handle, weight_shard.handle,
                                              bias_shard.handle if bias_shard else None, int(vocab_offset),
                                              int(shard_vocab), int(width), C.c_void_p(hidden_ptr), int(hidden_kind),
                                              int(rows), C.c_void_p(targets_ptr), rot,
                                              C.c_void_p(partials.data_ptr()), C.c_void_p(workspace.data_ptr()),
                                              workspace.numel()))
        if dist.is_initialized() and dist.get_world_size(group) > 1:
            dist.all_reduce(partials, op=dist.ReduceOp.MAX, group=group)
        margin, amax, tl = outputs
        check(lib.lsx_readout_partials_merge_device(gpu.handle, C.c_void_p(partials.data_ptr()),
                                                    C.c_void_p(targets_ptr), int(rows),
                                                    C.c_void_p(margin.data_ptr()), C.c_void_p(amax.data_ptr()),
                                                    C.c_void_p(tl.data_ptr())))
    return outputs
