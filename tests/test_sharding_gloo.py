"""Head sharding host logic on CPU with gloo, world_size 2 (and 3 for uneven shards).

Each rank computes its contiguous head range, produces per-head outputs
(a deterministic function of the global head id, standing in for the
attention of that head) and all-gathers them; every rank must end up with
the full [B, S, H, D] tensor in head order.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _head_output(h, B=1, S=16, D=8):
    g = torch.Generator().manual_seed(100 + h)
    return torch.randn(B, S, D, generator=g)


def _worker(rank, world, port, num_heads, q):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "minference-npu_b200"))
    import torch.distributed as dist

    from minference.sharding import gather_heads, head_range

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        hr = head_range(num_heads, rank, world)
        local = torch.stack([_head_output(h) for h in hr], dim=2)  # [B, S, h_r, D]
        full = gather_heads(local, num_heads)
        want = torch.stack([_head_output(h) for h in range(num_heads)], dim=2)
        q.put((rank, bool(torch.equal(full, want)), list(hr)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,num_heads", [(2, 32), (2, 5), (3, 32)])
def test_gather_heads_gloo(world, num_heads):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, num_heads, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    results = sorted(q.get(timeout=5) for _ in range(world))
    assert all(ok for _, ok, _ in results)
    covered = sorted(h for _, _, hs in results for h in hs)
    assert covered == list(range(num_heads))


def test_head_range_partition():
    from minference.sharding import head_range

    for H in (1, 7, 32):
        for G in (1, 2, 3, 4, 8):
            heads = [h for r in range(G) for h in head_range(H, r, G)]
            assert heads == list(range(H))
    with pytest.raises(ValueError):
        head_range(32, 2, 2)


def test_balanced_head_map_properties():
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "minference-npu_b200"))
    from minference.sharding import balanced_head_map, head_cost

    cycle = [("vertical_and_slash", 1000, 6096), ("block_sparse", 100, 0),
             ("vertical_and_slash", 1000, 6096), ("block_sparse", 100, 0), ("stream_llm", 128, 1024)]
    pats = [cycle[h % 5] for h in range(32)]
    costs = [head_cost(p, 65536) for p in pats]
    for world in (1, 2, 4, 8):
        m = balanced_head_map(costs, world)
        assert sorted(h for hs in m for h in hs) == list(range(32))
        assert all(len(hs) == 32 // world for hs in m)
        assert m == balanced_head_map(costs, world)  # deterministic
        bal = max(sum(costs[h] for h in hs) for hs in m)
        contig = max(sum(costs[h] for h in range(r * 32 // world, (r + 1) * 32 // world))
                     for r in range(world))
        assert bal <= contig + 1e-6
    # 8 ranks: the contiguous map puts 2 VS + 2 block_sparse heads on some ranks
    m8 = balanced_head_map(costs, 8)
    assert max(sum(costs[h] for h in hs) for hs in m8) < contig
    with pytest.raises(ValueError):
        balanced_head_map(costs[:5], 2)


def _worker_mapped(rank, world, port, head_map, q):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "minference-npu_b200"))
    import torch.distributed as dist

    from minference.sharding import gather_heads_mapped

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n = sum(len(hs) for hs in head_map)
        local = torch.stack([_head_output(h) for h in head_map[rank]], dim=2)
        full = gather_heads_mapped(local, head_map)
        want = torch.stack([_head_output(h) for h in range(n)], dim=2)
        q.put((rank, bool(torch.equal(full, want)), head_map[rank]))
    finally:
        dist.destroy_process_group()


def test_gather_heads_mapped_gloo():
    head_map = [[0, 3, 5, 6], [1, 2, 4, 7]]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_mapped, args=(r, 2, port, head_map, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(ok for _, ok, _ in res), res


def _worker_oproj(rank, world, port, q):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "minference-npu_b200"))
    import torch.distributed as dist

    from minference.sharding import gather_o_proj, o_proj_input_permutation

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        head_map = [[0, 3, 5, 6], [1, 2, 4, 7]]
        D, hidden = 8, 12
        g = torch.Generator().manual_seed(7)
        W = torch.randn(hidden, 8 * D, generator=g, dtype=torch.float64)
        bias = torch.randn(hidden, generator=g, dtype=torch.float64)
        heads = [_head_output(h).double() for h in range(8)]  # [B, S, D] each
        local = torch.stack([heads[h] for h in head_map[rank]], dim=2)
        wp = W[:, o_proj_input_permutation(head_map, D)]
        got = gather_o_proj(local, wp, bias, chunks=3)
        full = torch.stack(heads, dim=2).reshape(1, 16, 8 * D)  # head order
        want = full @ W.T + bias
        q.put((rank, bool(torch.allclose(got, want, atol=1e-10)), None))
    finally:
        dist.destroy_process_group()


def test_gather_o_proj_gloo():
    """Chunked gather + o_proj with a permuted weight equals o_proj of the
    head-ordered layer output."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_oproj, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(ok for _, ok, _ in res), res


CYCLE = [("vertical_and_slash", 1000, 6096), ("block_sparse", 100, 0),
         ("vertical_and_slash", 1000, 6096), ("block_sparse", 100, 0), ("stream_llm", 128, 1024)]


def _mixed_layout(n=32):
    pats = [CYCLE[h % 5] for h in range(n)]
    order = ("stream_llm", "block_sparse", "vertical_and_slash")
    return [pats[h] for h in sorted(range(n), key=lambda h: (order.index(pats[h][0]), h))]


def test_tile_partition_covers_and_balances():
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "minference-npu_b200"))
    from minference.sharding import (balanced_head_map, head_cost, tile_costs, tile_partition,
                                     unit_range_split)

    S = 65536
    pats = _mixed_layout()
    T = S // 128
    for world in (1, 2, 3, 4, 8):
        parts = tile_partition(pats, S, world)
        units = [(pc.slot, t) for pr in parts for pc in pr for t in range(pc.t0, pc.t1)]
        assert units == [(h, t) for h in range(32) for t in range(T)]  # contiguous, in order
        loads = [sum(sum(tile_costs(pats[pc.slot], S)[pc.t0:pc.t1]) for pc in pr) for pr in parts]
        assert max(loads) <= 1.01 * sum(loads) / world
        for pr in parts:
            a, b = unit_range_split(pr, pats, S)
            assert [(pc.slot, t) for pc in a + b for t in range(pc.t0, pc.t1)] == \
                [(pc.slot, t) for pc in pr for t in range(pc.t0, pc.t1)]
    # at 8 ranks whole heads cannot balance the 13 VS heads; tiles can
    costs = [head_cost(p, S) for p in pats]
    m8 = balanced_head_map(costs, 8)
    heads_max = max(sum(costs[h] for h in hs) for hs in m8) / (sum(costs) / 8)
    assert heads_max > 1.1


def _worker_rows(rank, world, port, S, q):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "minference-npu_b200"))
    import torch.distributed as dist

    from minference.sharding import gather_row_ranges, tile_partition, unit_range_split

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pats = _mixed_layout(10)
        H, D = len(pats), 4
        g = torch.Generator().manual_seed(5)
        want = torch.randn(1, H, S, D, generator=g)
        parts = tile_partition(pats, S, world)
        halves = [unit_range_split(pr, pats, S) for pr in parts]
        out = torch.zeros_like(want)
        ok = True
        for phase in (0, 1):
            for pc in halves[rank][phase]:  # "compute" this rank's rows
                r0, r1 = pc.rows(S)
                out[:, pc.slot, r0:r1] = want[:, pc.slot, r0:r1]
            gather_row_ranges(out, [h[phase] for h in halves])
            if phase == 0:  # after phase 0 every rank holds every first half
                for h in halves:
                    for pc in h[0]:
                        r0, r1 = pc.rows(S)
                        ok &= torch.equal(out[:, pc.slot, r0:r1], want[:, pc.slot, r0:r1])
        q.put((rank, bool(ok and torch.equal(out, want)), None))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,S", [(2, 1024), (3, 1000)])
def test_gather_row_ranges_gloo(world, S):
    """Each rank fills its (head, tile) pieces; the two-phase row-range
    exchange leaves every rank with the whole [1, H, S, D] output."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_rows, args=(r, world, port, S, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(ok for _, ok, _ in res), res
