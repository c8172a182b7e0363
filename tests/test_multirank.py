"""Multi-rank host logic on CPU (gloo, world size 2): user sharding, stream
seeds independent of the rank count, the per-step gather of deltas, and a
rank that dies before the gather being reported to the survivor by the
process group's timeout (no GPU involved)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from provenloop_b200.multigpu import gather_rows, stream_seed, stream_seeds, user_block


def test_user_blocks_partition_everything():
    for n in (0, 1, 7, 256, 1000):
        for world in (1, 2, 3, 4, 8):
            blocks = [user_block(n, world, r) for r in range(world)]
            assert blocks[0][0] == 0 and blocks[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(blocks, blocks[1:]))
            sizes = [b - a for a, b in blocks]
            assert max(sizes) - min(sizes) <= 1


def test_stream_seeds_unique_and_rank_independent():
    n = 64
    s = {stream_seed(u, t, n) for u in range(n) for t in range(5)}
    assert len(s) == 5 * n
    # the owner rank does not enter the seed
    assert stream_seed(17, 3, n) == 1 + 3 * n + 17
    users = np.arange(5, 40, dtype=np.uint64)
    v = stream_seeds(users, 3, n)
    assert v.dtype == np.uint64 and v.tolist() == [stream_seed(int(u), 3, n) for u in users]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n_users, d, q, die):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    a, b = user_block(n_users, world, rank)
    # stand-in for a rank's decrypted deltas: a deterministic function of the user id
    rows = torch.tensor([[u * 1000 + j for j in range(d)] for u in range(a, b)], dtype=torch.float64)
    if die and rank == 1:
        os._exit(0)            # leaves between steps, with nothing in flight
    try:
        out = gather_rows(rows, world, rank)
        if rank == 0:
            q.put(("ok", torch.cat(out).numpy()))
    except Exception as e:   # the survivor learns of the dead peer from the collective
        q.put(("error", type(e).__name__))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


@pytest.mark.parametrize("die", [False, True])
def test_gloo_gather_and_dead_rank(die):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    n_users, d = 6, 4
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n_users, d, q, die)) for r in range(2)]
    for p in procs:
        p.start()
    kind, payload = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    if not die:
        assert kind == "ok"
        ref = np.array([[u * 1000 + j for j in range(d)] for u in range(n_users)], dtype=np.float64)
        assert np.array_equal(payload, ref)
    else:
        assert kind == "error"
