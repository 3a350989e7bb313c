"""Sharding the decode batch over GPUs (one process per GPU).

Decode shards by sequence with no reduction: each GPU owns the pages of its
sequences and attends them alone. The split restates the reference's work
split across threads (``_share``, ``paged_attn.mojo:788-816``) one level up:
contiguous sequence ranges balanced on cost = context + 16 (one 16-key unit
of fixed work per sequence), not on count.
"""


def balanced_ranges(lens, parts):
    """Contiguous [lo, hi) sequence ranges, one per part, covering all of
    ``lens`` and balanced on sum(len + 16): part p starts at the first sequence
    whose preceding cost reaches p/parts of the total (integer arithmetic)."""
    n = len(lens)
    cost = [max(0, int(x)) + 16 for x in lens]
    total = sum(cost)
    bounds = [0]
    cum, i = 0, 0
    for p in range(1, parts):
        target = p * total  # compare cum * parts against p * total
        while i < n and (cum + cost[i]) * parts <= target:
            cum += cost[i]
            i += 1
        # take the next sequence too if that lands closer to the target
        if i < n and abs((cum + cost[i]) * parts - target) < abs(cum * parts - target):
            cum += cost[i]
            i += 1
        bounds.append(max(i, bounds[-1]))
    bounds.append(n)
    return [(bounds[p], bounds[p + 1]) for p in range(parts)]


def gather_outputs(out_local, counts, group=None):
    """The optional collective: every rank's decode output rows gathered in
    sequence order on every rank ([sum(counts), ...]). Uneven shards are padded
    to the largest one for one all_gather_into_tensor, then unpadded; even ones
    go straight into the result."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    most = max(counts)
    if min(counts) == most and out_local.is_contiguous():
        # even shards: straight into the gathered tensor, nothing to pad or cut
        full = torch.empty((world * most,) + tuple(out_local.shape[1:]), dtype=out_local.dtype,
                           device=out_local.device)
        dist.all_gather_into_tensor(full, out_local, group=group)
        return full
    pad = torch.zeros((most,) + tuple(out_local.shape[1:]), dtype=out_local.dtype, device=out_local.device)
    pad[:out_local.shape[0]] = out_local
    full = torch.empty((world * most,) + tuple(out_local.shape[1:]), dtype=out_local.dtype,
                       device=out_local.device)
    dist.all_gather_into_tensor(full, pad, group=group)
    return torch.cat([full[r * most:r * most + counts[r]] for r in range(world)])
