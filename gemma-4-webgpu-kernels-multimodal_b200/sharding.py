"""Data-parallel placement of independent items (images, audio clips) on the
ranks of a job or the devices of a context.

The towers have no exchange step: every image and every clip is embedded
independently with the weights replicated per GPU (the reference runs one
item per call on one device, src/vision/index.ts:29-37 and
src/audio/index.ts:41-49).  So there is no collective on the data path;
ranks only agree on timing (max over ranks) and, when a caller wants the
embeddings in one place, gather them on the host.
"""
from typing import List, Sequence


def image_shard(n_items: int, world: int, rank: int) -> range:
    """Contiguous block of the n_items images owned by `rank` (block sizes
    differ by at most one)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(n_items, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def encoder_rows(samples: int, cap: int = 480000) -> int:
    """Audio encoder rows of a clip (computeGemma4AudioSoftTokenCount,
    src/preprocess/audio.ts:4-20): frames at hop 160 after 160 samples of
    left padding, then two stride-2 convs."""
    n = min(int(samples), cap)
    frames = (160 + n - 321) // 160 + 1 if 160 + n >= 321 else 0
    if frames == 0:
        return 0
    t0 = (frames - 1) // 2 + 1
    return (t0 - 1) // 2 + 1


def lpt_assign(rows: Sequence[int], world: int) -> List[List[int]]:
    """Length-balanced assignment of clips: longest first (stable) onto the
    least-loaded bin (lowest index on ties), load = encoder rows.  The same
    rule g4m_audio_embed_batch applies across the devices of a context."""
    order = sorted(range(len(rows)), key=lambda i: -rows[i])
    parts: List[List[int]] = [[] for _ in range(world)]
    load = [0] * world
    for i in order:
        g = min(range(world), key=lambda k: (load[k], k))
        parts[g].append(i)
        load[g] += rows[i]
    return parts


def max_over_ranks(value: float, dist=None, device=None) -> float:
    """Max of a per-rank number over the process group (the timing rule of a
    data-parallel job); the value itself without a group."""
    if dist is None or not dist.is_initialized():
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
