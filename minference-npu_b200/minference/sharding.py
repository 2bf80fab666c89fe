"""Head-sharded execution across GPUs (one process per GPU).

Every MInference pattern is independent per head, index estimation
included, so a layer's heads split over the ranks with no exchange during
attention.  The only exchange is re-assembling the head outputs for
``o_proj``: an all-gather of each rank's ``[B, S, h_r, D]`` slice (NCCL over
NVLink/NVSwitch on B200; gloo works for CPU tests).

Two head maps:
  * contiguous (`head_range`): rank r takes a contiguous range;
  * cost-balanced (`balanced_head_map`): per-head costs from the pattern
    config (`head_cost`), assigned longest-first to the least-loaded rank
    with equal head counts per rank, so the layer time (set by the slowest
    rank) drops when the pattern mix is uneven across contiguous ranges.
    `gather_heads_mapped` re-assembles head order after the all-gather.

Heads differ in cost by ~30x between patterns, so whole heads cannot always
balance (13 vertical_and_slash heads over 8 ranks leave some rank with two).
Query tiles are independent in every pattern too, so `tile_partition` cuts
the layer's (head, 128-row tile) units into contiguous per-rank ranges of
equal modelled cost; a rank then runs row windows (``rows=``) of a few heads,
and `gather_row_ranges` re-assembles the ``[B, H, S, D]`` output, in which
each rank's range is one contiguous block of memory.

Without any collective for the data: `peer_addresses` opens the other
ranks' output buffers (CUDA IPC) so the attention kernels can store their
tiles into them directly (the ops' ``out_replicas=``).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

__all__ = ["head_range", "gather_heads", "head_cost", "balanced_head_map",
           "gather_heads_mapped", "o_proj_input_permutation", "gather_o_proj",
           "tile_costs", "tile_partition", "Piece", "unit_range_split", "gather_row_ranges",
           "peer_addresses", "close_peer_addresses"]


def head_range(num_heads: int, rank: int, world: int) -> range:
    """Contiguous heads of `rank`; the first num_heads % world ranks take one extra."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"bad rank/world {rank}/{world}")
    base, extra = divmod(num_heads, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def gather_heads(local_bshd: torch.Tensor, num_heads: int, group=None) -> torch.Tensor:
    """All-gather per-rank head slices ``[B, S, h_r, D]`` into ``[B, S, H, D]``.

    Equal shards use one ``all_gather_into_tensor`` (NCCL) into a rank-major
    buffer followed by a head-dim permute; uneven shards (or backends without
    the fused collective) fall back to ``all_gather`` of padded slices."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    B, S, h_local, D = local_bshd.shape
    sizes = [len(head_range(num_heads, r, world)) for r in range(world)]
    if sizes[rank] != h_local:
        raise ValueError(f"rank {rank} holds {h_local} heads, expected {sizes[rank]}")
    hmax = max(sizes)
    x = local_bshd.contiguous()
    if h_local < hmax:
        x = torch.cat([x, x.new_zeros(B, S, hmax - h_local, D)], dim=2)
    use_fused = dist.get_backend(group) == "nccl"
    if use_fused:
        buf = torch.empty((world,) + tuple(x.shape), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(buf, x, group=group)
        parts = list(buf.unbind(0))
    else:
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x, group=group)
    parts = [p[:, :, : sizes[r]] for r, p in enumerate(parts)]
    return torch.cat(parts, dim=2)


def head_cost(pattern, S: int) -> float:
    """Relative attention cost of one head: its visible (query, key) pairs.

    pattern: (type, v, s[, score]) as in the pattern JSON.  vertical_and_slash
    and dense count the causal triangle (at long contexts the VS set covers
    nearly all of it); block_sparse counts its selected 64x64 blocks;
    stream_llm counts sink plus window keys per query."""
    ty = pattern[0]
    causal = S * (S + 1) / 2.0
    if ty == "block_sparse":
        return min(causal, float(S) * 64.0 * max(1, int(pattern[1])))
    if ty == "stream_llm":
        return min(causal, float(S) * (int(pattern[1]) + int(pattern[2])))
    if ty in ("vertical_and_slash", "dense"):
        return causal
    raise ValueError(f"unknown pattern type {ty!r}")


def balanced_head_map(costs, world: int) -> list[list[int]]:
    """Heads per rank, each list ascending.  Requires len(costs) % world == 0
    (every rank holds the same number of heads, which keeps the fused
    equal-size all-gather).  Longest-processing-time-first: heads in
    decreasing cost go to the least-loaded rank that still has room; ties go
    to the lower rank, so the map is deterministic."""
    n = len(costs)
    if world <= 0 or n % world:
        raise ValueError(f"{n} heads do not split evenly over {world} ranks")
    per = n // world
    load = [0.0] * world
    ranks: list[list[int]] = [[] for _ in range(world)]
    for h in sorted(range(n), key=lambda i: (-costs[i], i)):
        r = min((r for r in range(world) if len(ranks[r]) < per), key=lambda r: (load[r], r))
        ranks[r].append(h)
        load[r] += costs[h]
    return [sorted(hs) for hs in ranks]


def gather_heads_mapped(local_bshd: torch.Tensor, head_map: list[list[int]],
                        group=None) -> torch.Tensor:
    """All-gather ``[B, S, h, D]`` slices whose heads are ``head_map[rank]``
    (equal sizes) and return ``[B, S, H, D]`` in global head order."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if len(head_map) != world:
        raise ValueError(f"head map has {len(head_map)} ranks, group has {world}")
    B, S, h_local, D = local_bshd.shape
    if len(head_map[rank]) != h_local:
        raise ValueError(f"rank {rank} holds {h_local} heads, map says {len(head_map[rank])}")
    x = local_bshd.contiguous()
    if dist.get_backend(group) == "nccl":
        buf = torch.empty((world,) + tuple(x.shape), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(buf, x, group=group)
        parts = list(buf.unbind(0))
    else:
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x, group=group)
    order = [h for hs in head_map for h in hs]  # head held at each gathered position
    inv = torch.empty(len(order), dtype=torch.long)
    inv[torch.tensor(order)] = torch.arange(len(order))
    return torch.cat(parts, dim=2).index_select(2, inv.to(x.device))


def o_proj_input_permutation(head_map: list[list[int]], head_dim: int) -> torch.Tensor:
    """Column order for o_proj's weight that consumes the rank-major gathered
    layout directly.

    After ``all_gather_into_tensor`` of equal slices, feature f of the
    gathered ``[B, S, H*D]`` row holds global feature perm[f].  Multiplying
    by ``W[:, perm]`` (permuted once, at load time) equals multiplying the
    head-ordered activations by W, so no per-layer re-ordering copy is needed."""
    order = [h for hs in head_map for h in hs]
    return torch.tensor([h * head_dim + d for h in order for d in range(head_dim)],
                        dtype=torch.long)


_comm_streams: dict[int, torch.cuda.Stream] = {}
_gather_bufs: dict[tuple, list[torch.Tensor]] = {}


def _comm_stream(device: torch.device) -> torch.cuda.Stream:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _comm_streams:
        _comm_streams[idx] = torch.cuda.Stream(device=idx)
    return _comm_streams[idx]


def gather_o_proj(local_bshd: torch.Tensor, weight_perm: torch.Tensor, bias=None, group=None,
                  chunks: int = 4) -> torch.Tensor:
    """o_proj of the all-gathered heads, with the gather overlapped.

    local_bshd: this rank's ``[B, S, h, D]`` head outputs (equal h on every
    rank).  weight_perm: o_proj's ``[hidden, H*D]`` weight with its input
    columns permuted by `o_proj_input_permutation` for the head map in use,
    so that rank r's slice of the gathered layout multiplies the column block
    ``weight_perm[:, r*h*D:(r+1)*h*D]``.  Returns ``[B, S, hidden]``, the same
    on every rank.

    The sequence is cut into `chunks` pieces.  With NCCL, the all-gather of
    piece c+1 runs on a side stream while the GEMMs of piece c run on the
    current stream, so the transfer hides behind o_proj.  Each piece's output
    is accumulated rank by rank (one addmm per rank) straight from the gather
    buffer, with no re-ordering copy.  The gather buffers are cached per
    shape and reused by the next call; calls on one device must not overlap.
    Other backends (gloo on CPU) run the pieces one after another."""
    world = dist.get_world_size(group)
    B, S, h, D = local_bshd.shape
    hd = h * D
    hidden = weight_perm.shape[0]
    x = local_bshd.contiguous()
    bounds = [S * i // chunks for i in range(chunks + 1)]
    out = torch.empty((B, S, hidden), dtype=x.dtype, device=x.device)
    wt = [weight_perm[:, r * hd:(r + 1) * hd].t() for r in range(world)]

    def project(parts, lo, hi):
        # out[:, lo:hi] = sum_r parts[r] @ W_r^T (+ bias)
        rows = B * (hi - lo)
        dst = out[:, lo:hi]
        acc = dst.reshape(rows, hidden) if B == 1 else torch.empty(rows, hidden, dtype=x.dtype,
                                                                     device=x.device)
        torch.matmul(parts[0].reshape(rows, hd), wt[0], out=acc)
        for r in range(1, world):
            acc.addmm_(parts[r].reshape(rows, hd), wt[r])
        if bias is not None:
            acc.add_(bias)
        if B != 1:
            dst.copy_(acc.view(B, hi - lo, hidden))

    nccl = dist.get_backend(group) == "nccl" and x.is_cuda
    if not nccl:
        for c in range(chunks):
            lo, hi = bounds[c], bounds[c + 1]
            piece = x[:, lo:hi].contiguous()
            parts = [torch.empty_like(piece) for _ in range(world)]
            dist.all_gather(parts, piece, group=group)
            project(parts, lo, hi)
        return out
    main = torch.cuda.current_stream(x.device)
    comm = _comm_stream(x.device)
    key = (x.device, world, B, S, h, D, x.dtype, chunks)
    if key not in _gather_bufs:
        _gather_bufs[key] = [torch.empty((world, B, bounds[c + 1] - bounds[c], h, D), dtype=x.dtype,
                                         device=x.device) for c in range(chunks)]
    bufs = _gather_bufs[key]
    # x is ready, and the previous call's GEMMs (which read bufs) have run.
    comm.wait_stream(main)
    events = []
    with torch.cuda.stream(comm):
        for c in range(chunks):
            lo, hi = bounds[c], bounds[c + 1]
            dist.all_gather_into_tensor(bufs[c], x[:, lo:hi].contiguous(), group=group)
            e = torch.cuda.Event()
            e.record(comm)
            events.append(e)
    for c in range(chunks):
        main.wait_event(events[c])
        project(bufs[c].unbind(0), bounds[c], bounds[c + 1])
    x.record_stream(comm)
    return out


# ---------------------------------------------------------------------------
# (head, query-tile) partition
# ---------------------------------------------------------------------------
TILE_ROWS = 128
# Cost model, in units of one 64-key step of a one-tile (M=128) attention
# entry, fitted to per-pattern timings of 8 heads x 64K on one B200
# (vertical_and_slash 0.84 ms, block_sparse 0.205 ms, stream_llm 0.048 ms
# per head): a tile's fixed cost (set-up, Q load, epilogue), the cost of a
# block_sparse split-tile step (two M=64 MMAs and a 128-row softmax), and
# the index estimation of a head, charged to its first tile.
TILE_OVERHEAD = 8.5
SPLIT_STEP = 1.25
HEAD_FIXED = {"vertical_and_slash": 9500.0, "block_sparse": 3000.0}


def tile_costs(pattern, S: int) -> list[float]:
    """Modelled cost of each 128-row query tile of one head: the 64-key
    blocks the attention kernel walks for it, plus a fixed per-tile cost
    (and the head's index estimation on its first tile).

    vertical_and_slash and dense walk the causal blocks (2t + 2 for tile t;
    at long contexts the VS set covers nearly all of them); block_sparse
    walks max over its two query blocks of min(top-k, causal blocks) split
    steps; stream_llm walks its sink and window blocks."""
    ty = pattern[0]
    T = -(-S // TILE_ROWS)
    out = []
    for t in range(T):
        causal = 2 * t + 2
        if ty in ("vertical_and_slash", "dense"):
            n = causal
        elif ty == "block_sparse":
            n = SPLIT_STEP * min(max(1, int(pattern[1])), causal)
        elif ty == "stream_llm":
            n_init, n_local = int(pattern[1]), int(pattern[2])
            n = min(causal, -(-n_init // 64) + -(-(n_local + TILE_ROWS) // 64) + 1)
        else:
            raise ValueError(f"unknown pattern type {ty!r}")
        out.append(n + TILE_OVERHEAD)
    if out:
        out[0] += HEAD_FIXED.get(ty, 0.0)
    return out


class Piece(tuple):
    """(slot, t0, t1): query tiles [t0, t1) of the head stored at position
    `slot` of the layer's head order (rows [128*t0, min(128*t1, S)))."""

    __slots__ = ()

    def __new__(cls, slot: int, t0: int, t1: int):
        return tuple.__new__(cls, (slot, t0, t1))

    slot = property(lambda self: self[0])
    t0 = property(lambda self: self[1])
    t1 = property(lambda self: self[2])

    def rows(self, S: int) -> tuple[int, int]:
        return self.t0 * TILE_ROWS, min(self.t1 * TILE_ROWS, S)


def tile_partition(patterns, S: int, world: int) -> list[list[Piece]]:
    """Split the layer into `world` contiguous ranges of (head, tile) units.

    Units are ordered head by head (in the order of `patterns`, one pattern
    tuple per head slot) and tile by tile inside a head, which is the memory
    order of a contiguous ``[1, H, S, D]`` output, so each rank's range is
    one contiguous block of it.  Rank r takes the units whose cost prefix
    midpoint falls in [r, r+1) * total / world.  Returns, per rank, its
    pieces in unit order."""
    if world <= 0:
        raise ValueError(f"bad world size {world}")
    costs = [tile_costs(p, S) for p in patterns]
    total = sum(sum(c) for c in costs)
    parts: list[list[Piece]] = [[] for _ in range(world)]
    acc = 0.0
    for slot, cs in enumerate(costs):
        cur_r, t_start = None, 0
        for t, c in enumerate(cs):
            r = min(world - 1, int((acc + c / 2) * world / total)) if total > 0 else 0
            acc += c
            if r != cur_r:
                if cur_r is not None:
                    parts[cur_r].append(Piece(slot, t_start, t))
                cur_r, t_start = r, t
        if cur_r is not None:
            parts[cur_r].append(Piece(slot, t_start, len(cs)))
    return parts


def unit_range_split(pieces: list[Piece], patterns, S: int, frac: float = 0.5):
    """Cut one rank's pieces (in unit order) where `frac` of their modelled
    cost is reached: returns (first, second) piece lists, a piece straddling
    the cut being split at a tile boundary."""
    costs = [tile_costs(patterns[p.slot], S) for p in pieces]
    total = sum(sum(c[p.t0:p.t1]) for p, c in zip(pieces, costs))
    target = frac * total
    first, second, acc = [], [], 0.0
    for p, c in zip(pieces, costs):
        if acc >= target:
            second.append(p)
            continue
        cut = p.t1
        for t in range(p.t0, p.t1):
            if acc >= target:
                cut = t
                break
            acc += c[t]
        if cut > p.t0:
            first.append(Piece(p.slot, p.t0, cut))
        if cut < p.t1:
            second.append(Piece(p.slot, cut, p.t1))
    return first, second


def _flat_span(pieces: list[Piece], S: int, D: int) -> tuple[int, int] | None:
    """Element span [lo, hi) of contiguous unit-ordered pieces inside a
    contiguous [1, H, S, D] buffer."""
    if not pieces:
        return None
    a, b = pieces[0], pieces[-1]
    lo = (a.slot * S + a.rows(S)[0]) * D
    hi = (b.slot * S + b.rows(S)[1]) * D
    return lo, hi


def gather_row_ranges(out: torch.Tensor, pieces_per_rank: list[list[Piece]], group=None):
    """In-place all-gather of row ranges: `out` is a contiguous ``[1, H, S, D]``
    tensor in which this rank has computed its pieces; afterwards every rank
    holds every rank's pieces.  Each rank's pieces must form one contiguous
    unit range (as `tile_partition` and `unit_range_split` produce).  With
    NCCL the exchange is one uneven all-gather whose outputs are the ranges
    themselves (no staging copy); other backends exchange the ranges with
    point-to-point sends and receives."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if out.dim() != 4 or out.shape[0] != 1 or not out.is_contiguous():
        raise ValueError("out must be a contiguous [1, H, S, D] tensor")
    _, H, S, D = out.shape
    flat = out.view(-1)
    spans = [_flat_span(p, S, D) for p in pieces_per_rank]
    if dist.get_backend(group) == "nccl":
        # uneven all-gather straight into the output (NCCL runs it as one
        # group of broadcasts, one per rank's range)
        parts = [flat[sp[0]:sp[1]] if sp else flat[:0] for sp in spans]
        dist.all_gather(parts, parts[rank], group=group)
        return out
    ops = []
    mine = spans[rank]
    for peer in range(world):
        if peer == rank:
            continue
        if mine is not None:
            ops.append(dist.P2POp(dist.isend, flat[mine[0]:mine[1]], peer, group))
        if spans[peer] is not None:
            lo, hi = spans[peer]
            ops.append(dist.P2POp(dist.irecv, flat[lo:hi], peer, group))
    if ops:
        for w in dist.batch_isend_irecv(ops):
            w.wait()
    return out


# ---------------------------------------------------------------------------
# Peer buffers (CUDA IPC) for output replicas
# ---------------------------------------------------------------------------
_opened: dict = {}


def _check(err, what):
    from cuda.bindings import runtime as rt

    if err != rt.cudaError_t.cudaSuccess:
        raise RuntimeError(f"{what} failed: {err}")


def peer_addresses(buf: torch.Tensor, group=None) -> list[int]:
    """Device addresses, valid on this process's GPU, of every rank's `buf`
    (rank order; this rank's entry is ``buf.data_ptr()``).

    Every rank passes its own tensor of the same shape (collective call).
    Each rank exports the CUDA IPC handle of the allocation holding its
    buffer, the handles and offsets are exchanged over the process group, and
    each peer's allocation is opened into this GPU's address space (reached
    over NVLink / NVSwitch).  The addresses serve as output replicas of the
    attention ops (``out_replicas=``), whose kernels then store each output
    tile into every rank's buffer.  Every rank must keep `buf` alive until all
    ranks have called `close_peer_addresses`."""
    from cuda.bindings import driver as cu
    from cuda.bindings import runtime as rt

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if not buf.is_cuda:
        raise ValueError("peer_addresses needs a CUDA tensor")
    dev = buf.device.index if buf.device.index is not None else torch.cuda.current_device()
    (err,) = rt.cudaSetDevice(dev)
    _check(err, f"cudaSetDevice({dev})")
    err, handle = rt.cudaIpcGetMemHandle(buf.data_ptr())
    _check(err, "cudaIpcGetMemHandle")
    err, base, _size = cu.cuMemGetAddressRange(cu.CUdeviceptr(buf.data_ptr()))
    if err != cu.CUresult.CUDA_SUCCESS:
        raise RuntimeError(f"cuMemGetAddressRange failed: {err}")
    off = buf.data_ptr() - int(base)
    infos = [None] * world
    dist.all_gather_object(infos, (bytes(handle.reserved), off), group=group)
    addrs = []
    for r, (h, o) in enumerate(infos):
        if r == rank:
            addrs.append(buf.data_ptr())
            continue
        key = (dev, h)
        if key not in _opened:
            hs = rt.cudaIpcMemHandle_t()
            hs.reserved = h
            err, ptr = rt.cudaIpcOpenMemHandle(hs, rt.cudaIpcMemLazyEnablePeerAccess)
            _check(err, f"cudaIpcOpenMemHandle (rank {r})")
            _opened[key] = int(ptr)
        addrs.append(_opened[key] + o)
    return addrs


def close_peer_addresses(group=None) -> None:
    """Unmap every peer allocation opened by `peer_addresses` (after this
    process's kernels that write them have finished), then wait for all
    ranks, so that no rank frees a buffer another still maps."""
    from cuda.bindings import runtime as rt

    torch.cuda.synchronize()
    for (dev, _), ptr in list(_opened.items()):
        (err,) = rt.cudaSetDevice(dev)
        _check(err, f"cudaSetDevice({dev})")
        (err,) = rt.cudaIpcCloseMemHandle(ptr)
        _check(err, "cudaIpcCloseMemHandle")
    _opened.clear()
    if dist.is_initialized():
        dist.barrier(group=group)
