"""The DiT's Ulysses path over NCCL on two GPUs (skipped with fewer): two
ranks with the B200 operations (fused passes, sparse attention kernels,
pooled bf16 q/k exchange) against one rank computing the same step alone.

The two runs differ only where cuBLAS blocks GEMMs of different heights
differently, so they agree as closely as two bf16 GEMM chains can; the
exchanges move bytes unchanged.  NVLS is off (NCCL_NVLS_ENABLE=0), and every
rank issues the same collectives in the same order."""
import datetime
import os
import socket
import sys

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "lightning-unified-video-editor-via-in-context-sparse-attention_b200")

TINY = dict(dim=256, ffn_dim=512, num_heads=2, num_layers=2, freq_dim=32, text_dim=64, text_len=16, in_dim=4,
            out_dim=4)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist
    try:
        for p in (REPO, PKG, os.path.join(REPO, "tests")):
            if p not in sys.path:
                sys.path.insert(0, p)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", rank))
        from wan_dit import WanDiT, WanDiTConfig
        cfg = WanDiTConfig(**TINY)
        g = torch.Generator().manual_seed(0)
        latent = torch.randn(cfg.in_dim, 4, 16, 34, generator=g)
        source = 0.8 * latent + 0.6 * torch.randn(latent.shape, generator=g)
        context = torch.randn(2, cfg.text_len, cfg.text_dim, generator=g)
        latent, source, context = latent.cuda(), source.cuda(), context.cuda()
        seq_len = 2 * 4 * 8 * 17 + 64            # 1152: whole 64-token blocks per rank
        solo = [dist.new_group([r]) for r in range(world)][rank]
        res = []
        for pooled in (True, False):
            a = WanDiT(cfg, seed=3, pooled_exchange=pooled).forward(latent, source, 500.0, context, seq_len)
            b = WanDiT(cfg, seed=3, group=solo).forward(latent, source, 500.0, context, seq_len)
            err = (a - b).abs().float()
            res.append((float(err.mean() / b.abs().mean()), float(err.max() / b.abs().max()),
                        bool(torch.isfinite(a).all())))
        torch.cuda.synchronize()
        dist.barrier()
        q.put((rank, res))
    except Exception as e:  # noqa: BLE001
        import traceback
        q.put((rank, repr(e) + traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_ulysses_step_on_two_gpus_equals_one_gpu(cuda_device):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    for rank, res in results:
        assert not isinstance(res, str), res
        for rel_mean, rel_max, finite in res:     # pooled bf16 q/k exchange, then f32
            print(f"rank {rank}: rel mean {rel_mean:.2e} rel max {rel_max:.2e}")
            assert finite and rel_mean <= 1e-2 and rel_max <= 0.15, (rank, rel_mean, rel_max)
