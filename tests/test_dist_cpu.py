"""Multi-rank host logic with 2 gloo ranks on CPU: sharding covers every unit
exactly once, times reduce to the slowest rank, checksums and row shards
(unequal ones too) gather in rank order, and a rank that raises does not leave its peer hanging (the process
group timeout ends the collective with an error)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from hybrid_model_mamba_xlstm_b200 import dist as D


def test_shard_range_partitions_units():
    for n in (0, 1, 7, 8, 64, 4096 * 8):
        for world in (1, 2, 3, 4, 8):
            spans = [D.shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        D.shard_range(4, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, mode):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    try:
        w, r, dev = D.init("gloo", timeout_s=10.0)
        assert (w, r) == (world, rank)
        if mode == "ok":
            t = D.max_over_ranks(1.5 + rank, w)
            a, b = D.shard_range(8, w, r)
            data = torch.arange(a, b, dtype=torch.float64)
            cs = D.gather_checksums(D.checksum(data), w)
            a7, b7 = D.shard_range(7, w, r)  # unequal shards (4 + 3 rows)
            full = D.gather_rows(torch.arange(a7 * 3, b7 * 3, dtype=torch.float32).view(-1, 3), 7, w)
            D.barrier(w)
            q.put((rank, t, cs.tolist(), full.tolist()))
        else:  # rank 1 fails before the collective; rank 0 must get an error, not hang
            if rank == 1:
                raise RuntimeError("planted failure on rank 1")
            try:
                D.max_over_ranks(1.0, w)
                q.put((rank, "no error"))
            except Exception as e:  # noqa: BLE001
                q.put((rank, "error:" + type(e).__name__))
    except RuntimeError as e:
        q.put((rank, "raised:" + str(e)))
    finally:
        try:
            D.finalize(world)
        except Exception:  # noqa: BLE001
            pass


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, mode)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    return sorted(out, key=lambda x: x[0])


def test_two_gloo_ranks_reduce_and_gather():
    out = _run("ok")
    for rank, t, cs, full in out:
        assert t == 2.5  # max of 1.5, 2.5
        assert cs[0][0] == sum(range(0, 4)) and cs[1][0] == sum(range(4, 8))
        assert full == torch.arange(21, dtype=torch.float32).view(7, 3).tolist()  # shards in rank order


def test_failed_rank_ends_peer_collective_with_error():
    out = _run("fail")
    assert out[1][1].startswith("raised:planted failure")
    assert out[0][1].startswith("error:")
