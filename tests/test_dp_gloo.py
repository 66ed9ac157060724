"""Host logic of the data-parallel trainer on CPU: two gloo ranks, no GPU.

Checks the shard arithmetic, the view assignment, and that the collectives the trainer
issues on its padded storage (reduce-scatter of gradient rows into each rank's own slice,
all-gather of each rank's slice of a parameter array; in place over NCCL, from a copy here)
give the summed rows and the replicated arrays."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gs3d.dp import (CHUNKS, COLOUR_ROW, DENSE_ROW, GEOM_ROW, chunk_layout, exchange_factored_chunk,
                     exchange_next_colours_chunk, given_colour_row, shard_range, view_index)


def test_shard_ranges_partition_the_gaussians():
    for n in (1, 2, 7, 8, 9, 1000, 313_001):
        for world in (1, 2, 3, 4, 8):
            covered = []
            for r in range(world):
                S, lo, hi = shard_range(n, world, r)
                assert S * world >= n and (S - 1) * world < n or n < world
                covered.extend(range(lo, hi))
            assert covered == list(range(n)), (n, world)


def test_chunk_ownership_partitions_the_gaussians():
    """Rank r owns [c C + r S, c C + (r + 1) S) of every chunk c; together they cover [0, n)."""
    for chunks in sorted({1, 2, 3, 4, CHUNKS}):
        for n in (1, 5, 8, 9, 1000, 313_001):
            for world in (1, 2, 3, 8):
                S, C_ = chunk_layout(n, world, chunks)
                assert C_ == S * world and chunks * C_ >= n
                covered = []
                for c in range(chunks):
                    for r in range(world):
                        lo = c * C_ + r * S
                        covered.extend(range(min(lo, n), min(lo + S, n)))
                assert sorted(covered) == list(range(n)), (n, world, chunks)


def test_views_of_a_step_are_distinct():
    """The world x V views of a step are distinct cameras (batches up to #cameras), and
    consecutive steps walk the shared permutation without gaps."""
    perm = np.random.default_rng(0).permutation(256)
    for world in (1, 2, 4, 8):
        for V in (1, 4, 8, 16, 32):
            if world * V > 256:
                continue
            seen = []
            for step in range(300):
                views = [view_index(step, r, world, perm, 256, V, v) for r in range(world) for v in range(V)]
                assert len(set(views)) == world * V
                seen.extend(views)
            assert seen[:256] == [int(x) for x in perm] or world * V * 300 < 256


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        n = 11
        S, C_ = chunk_layout(n, world, CHUNKS)
        rows = CHUNKS * C_
        # each rank's dense rows: rank-dependent values, padding rows zero
        dense = torch.zeros((rows, DENSE_ROW))
        dense[:n] = torch.arange(n * DENSE_ROW, dtype=torch.float32).view(n, DENSE_ROW) * (rank + 1)
        total = sum(r + 1 for r in range(world))
        want = torch.zeros((rows, DENSE_ROW))
        want[:n] = torch.arange(n * DENSE_ROW, dtype=torch.float32).view(n, DENSE_ROW) * total
        ok_rs = True
        base = torch.full((rows, 4), -1.0)
        for c in range(CHUNKS):  # per chunk: reduce-scatter into the owners' sub-ranges
            flat = dense[c * C_:(c + 1) * C_].reshape(-1)
            per = S * DENSE_ROW
            dist.reduce_scatter_tensor(flat[rank * per:(rank + 1) * per], flat.clone(), op=dist.ReduceOp.SUM)
            lo = c * C_ + rank * S
            ok_rs = ok_rs and torch.equal(dense[lo:lo + S], want[lo:lo + S])
            base[lo:lo + S] = torch.arange(lo, lo + S, dtype=torch.float32)[:, None] + 0.5
        ok_ag = True
        for c in range(CHUNKS):  # per chunk: all-gather each owner's sub-range of a parameter array
            fb = base[c * C_:(c + 1) * C_].reshape(-1)
            per4 = fb.numel() // world
            dist.all_gather_into_tensor(fb, fb[rank * per4:(rank + 1) * per4].clone())
        ok_ag = torch.equal(base[:n], torch.arange(n, dtype=torch.float32)[:, None].expand(n, 4) + 0.5)
        q.put((rank, ok_rs, ok_ag))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e), None))


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_collectives_on_padded_storage(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok_rs, ok_ag in results:
        assert ok_rs is True and ok_ag is True, (rank, ok_rs, ok_ag)


def _factored_worker(rank, world, port, q, views=1):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        n = 13
        S, C_ = chunk_layout(n, world, CHUNKS)
        rows = CHUNKS * C_
        ar = torch.arange(n, dtype=torch.float32)
        geom = torch.zeros((rows, GEOM_ROW))
        geom[:n] = (ar[:, None] * GEOM_ROW + torch.arange(GEOM_ROW)) * (rank + 1)
        # one colour row per view (views == 1: the (rows, COLOUR_ROW) single-view layout)
        colour = torch.zeros((views, rows, COLOUR_ROW))
        for v in range(views):
            colour[v, :n] = ar[:, None] * 10 + torch.arange(COLOUR_ROW) + 1000 * rank + 100000 * v
        total = sum(r + 1 for r in range(world))
        want_geom = (ar[:, None] * GEOM_ROW + torch.arange(GEOM_ROW)) * total
        ok = True
        for c in range(CHUNKS):
            recv = torch.full((views, world, S, COLOUR_ROW), -7.0)
            for w in exchange_factored_chunk(geom, colour[0] if views == 1 else colour,
                                             recv[0] if views == 1 else recv, c, S, C_, rank,
                                             in_place=False):
                w.wait()
            lo = c * C_ + rank * S
            hi = min(lo + S, n)
            if lo < hi:
                ok = ok and torch.equal(geom[lo:hi], want_geom[lo:hi])
                for v in range(views):
                    for src in range(world):  # slot (v, src): rank src's view-v rows of this range
                        want = ar[lo:hi, None] * 10 + torch.arange(COLOUR_ROW) + 1000 * src + 100000 * v
                        ok = ok and torch.equal(recv[v, src, : hi - lo], want)
                        ok = ok and bool(torch.all(recv[v, src, hi - lo:] == 0))
        q.put((rank, ok))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e)))


@pytest.mark.parametrize("world, views", [(2, 1), (3, 1), (2, 3)])
def test_factored_exchange_on_padded_storage(world, views):
    """Geometry rows summed into each owner's sub-range; every view's colour rows of that
    sub-range delivered to the owner in (view, rank) order (the order the owner rebuilds the
    SH gradients in); padding rows arrive as zeros. views > 1: several views per rank."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_factored_worker, args=(r, world, port, q, views)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok in results:
        assert ok is True, (rank, ok)


def _colours_worker(rank, world, port, q, views):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        n = 17
        S, C_ = chunk_layout(n, world, CHUNKS)
        recv = torch.full((CHUNKS, world * views * S, 4), -1.0)
        for c in range(CHUNKS):
            # owner `rank`: slot r * V + v holds its sub-range's colours for view v of rank r,
            # encoded as gi * 1000 + r * 10 + v
            send = torch.full((world * views * S, 4), -2.0)
            for r in range(world):
                for v in range(views):
                    for i in range(S):
                        gi = c * C_ + rank * S + i
                        send[(r * views + v) * S + i] = gi * 1000 + r * 10 + v
            exchange_next_colours_chunk(send, recv[c]).wait()
        flat = recv.reshape(-1, 4)
        ok = all(bool(torch.all(flat[given_colour_row(gi, S, world, views, v)] == gi * 1000 + rank * 10 + v))
                 for gi in range(n) for v in range(views))
        q.put((rank, ok))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e)))


@pytest.mark.parametrize("world, views", [(2, 1), (3, 2)])
def test_next_colours_exchange_layout(world, views):
    """shard_sh: every owner's colours for view v of rank r reach rank r at the row
    gs3d_render_forward_given_colour reads for that Gaussian and view (given_colour_row)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_colours_worker, args=(r, world, port, q, views)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok in results:
        assert ok is True, (rank, ok)
