"""Multi-process host logic on CPU with the gloo backend (world size 2):
head sharding reproduces the single-process result, the Ulysses all-to-all
pair is an exact round trip, max-over-ranks timing, and a rank that fails
before a collective makes the other rank's collective end with an error
(host-side fault injection; no device is involved)."""
import datetime
import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "lightning-unified-video-editor-via-in-context-sparse-attention_b200")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    for p in (REPO, PKG):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    torch.set_num_threads(2)


def _worker_heads(rank, world, port, q):
    try:
        _init(rank, world, port)
        from in_context_sparse_attention import sharding
        from oracle import icsa_oracle as orc
        B, S, H, D, t = 1, 2048, 4, 64, 1024
        g = torch.Generator().manual_seed(0)
        x = [torch.randn(B, S, H, D, generator=g) for _ in range(3)]
        heads = sharding.head_range(H, rank, world)
        local = orc.editing_sparse_attention(*(y[:, :, heads.start:heads.stop].contiguous() for y in x), t).out
        full_from_shards = sharding.gather_heads(local)
        ref = orc.editing_sparse_attention(*x, t).out
        err = float((full_from_shards - ref).abs().max())
        slow = sharding.max_over_ranks(float(rank + 1))
        q.put((rank, err, slow))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e), None))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _worker_ulysses(rank, world, port, q):
    try:
        _init(rank, world, port)
        from in_context_sparse_attention import sharding
        B, S, H, D = 2, 96, 6, 8
        g = torch.Generator().manual_seed(1)
        full = torch.randn(B, S, H, D, generator=g)
        s = S // world
        mine = full[:, rank * s:(rank + 1) * s].contiguous()
        by_head = sharding.seq_to_heads(mine)
        hp = H // world
        want = full[:, :, rank * hp:(rank + 1) * hp]
        ok1 = torch.equal(by_head, want)
        back = sharding.heads_to_seq(by_head)
        ok2 = torch.equal(back, mine)
        q.put((rank, ok1 and ok2, None))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e), None))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _worker_fault(rank, world, port, q):
    try:
        _init(rank, world, port, timeout_s=5)
        if rank == 1:
            q.put((rank, "left before the collective", None))
            return  # the injected failure: never joins the all_reduce
        t = torch.ones(1)
        try:
            dist.all_reduce(t)
            q.put((rank, "collective completed unexpectedly", None))
        except Exception as e:  # noqa: BLE001
            q.put((rank, "error:" + type(e).__name__, None))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e), None))


def _run(target, world=2, timeout=180):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, a, b = q.get(timeout=timeout)
        res[r] = (a, b)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


def test_head_sharding_matches_single_process():
    res = _run(_worker_heads)
    for r in (0, 1):
        err, slow = res[r]
        assert isinstance(err, float), err
        assert err == 0.0
        assert slow == 2.0


def test_ulysses_all_to_all_round_trip():
    res = _run(_worker_ulysses)
    assert res[0][0] is True and res[1][0] is True, res


def test_missing_rank_ends_the_collective_with_an_error():
    res = _run(_worker_fault)
    assert res[1][0] == "left before the collective"
    assert str(res[0][0]).startswith("error:"), res


def test_head_range_rejects_uneven_splits():
    sys.path.insert(0, PKG)
    from in_context_sparse_attention import sharding
    assert list(sharding.head_range(40, 3, 8)) == [15, 16, 17, 18, 19]
    with pytest.raises(ValueError):
        sharding.head_range(40, 0, 3)
