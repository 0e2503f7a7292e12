"""CPU checks of the Wan 2.2 DiT harness around the attention call
(wan_dit): rotary tables against the reference's own formulas, token
positions, and Ulysses sequence parallelism over two gloo ranks against one
rank, with the block math restated in torch (tests/_dit_reference.py)."""
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

from wan_dit import WanDiTConfig, head_dim_splits, rope_table, token_positions  # noqa: E402

from _dit_reference import reference_freqs, rope_apply_tokens  # noqa: E402

TINY = dict(dim=256, ffn_dim=512, num_heads=2, num_layers=2, freq_dim=32, text_dim=64, text_len=16, in_dim=4,
            out_dim=4)


def tiny_inputs(cfg, seed=0, grid=(4, 16, 34)):
    g = torch.Generator().manual_seed(seed)
    f, h, w = grid
    latent = torch.randn(cfg.in_dim, f, h, w, generator=g)
    source = 0.8 * latent + 0.6 * torch.randn(cfg.in_dim, f, h, w, generator=g)
    context = torch.randn(2, cfg.text_len, cfg.text_dim, generator=g)
    return latent, source, context


@pytest.mark.parametrize("D", [64, 128])
def test_rope_table_equals_reference_frequencies(D):
    ref = reference_freqs(D)
    tab = rope_table(D)
    assert tab.shape == (1024, D // 2, 2) and tab.dtype == torch.float64
    assert torch.equal(tab[..., 0], ref.real) and torch.equal(tab[..., 1], ref.imag)


def test_head_dim_splits_follow_the_reference():
    assert head_dim_splits(128) == (22, 43)
    assert head_dim_splits(64) == (12, 22)


def test_token_positions_cover_target_source_and_padding():
    pos = token_positions((2, 3, 4), (2, 3, 4), 64)
    assert pos.shape == (64, 4) and pos.dtype == torch.int32
    assert pos[:24, 3].all() and pos[24:48, 3].all() and not pos[48:, 3].any()
    assert pos[0].tolist() == [0, 0, 0, 1] and pos[23].tolist() == [1, 2, 3, 1]
    assert pos[24].tolist() == [0, 0, 0, 1] and pos[5].tolist() == [0, 1, 1, 1]
    with pytest.raises(ValueError):
        token_positions((2, 3, 4), (2, 3, 4), 40)


def test_rope_restatement_rotates_pairs_and_skips_padding():
    D = 128
    pos = token_positions((1, 2, 2), (1, 2, 2), 10)
    x = torch.randn(1, 10, 2, D)
    y = rope_apply_tokens(x, pos, reference_freqs(D))
    assert torch.equal(y[:, 8:], x[:, 8:])                       # padding: multiplied by ones
    # rotation keeps the norm of every complex pair
    nx = x[:, :8].reshape(1, 8, 2, D // 2, 2).norm(dim=-1)
    ny = y[:, :8].reshape(1, 8, 2, D // 2, 2).norm(dim=-1)
    assert torch.allclose(nx, ny, rtol=1e-5, atol=1e-6)


def test_default_config_is_the_a14b_expert():
    cfg = WanDiTConfig()
    assert (cfg.dim, cfg.ffn_dim, cfg.num_heads, cfg.num_layers, cfg.head_dim) == (5120, 13824, 40, 40, 128)
    assert (cfg.text_dim, cfg.text_len, cfg.freq_dim, cfg.patch_size) == (4096, 512, 256, (1, 2, 2))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker_ulysses_dit(rank, world, port, q):
    try:
        for p in (REPO, PKG, os.path.join(REPO, "tests")):
            if p not in sys.path:
                sys.path.insert(0, p)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
        torch.set_num_threads(2)
        from wan_dit import WanDiT, WanDiTConfig
        from _dit_reference import ReferenceOps
        cfg = WanDiTConfig(**TINY)
        latent, source, context = tiny_inputs(cfg)
        seq_len = 2 * 4 * 8 * 17 + 64          # 1152 tokens: target 544 | source 544 | 64 padding
        assert (seq_len // world) % 64 == 0     # whole 64-token blocks per rank: the pooled exchange applies
        solo = [dist.new_group([r]) for r in range(world)][rank]
        single = WanDiT(cfg, device="cpu", seed=3, ops=ReferenceOps(), group=solo)
        b = single.forward(latent, source, 500.0, context, seq_len)
        res = []
        for pipelined, pooled in ((True, True), (True, False), (False, False)):
            sharded = WanDiT(cfg, device="cpu", seed=3, ops=ReferenceOps(), pipelined=pipelined,
                             pooled_exchange=pooled)
            assert sharded.world == world and single.world == 1
            a = sharded.forward(latent, source, 500.0, context, seq_len)
            res.append((float((a - b).abs().max()), float(b.abs().max()), tuple(a.shape),
                        bool(torch.isfinite(a).all())))
        q.put((rank, res))
    except Exception as e:  # noqa: BLE001
        import traceback
        q.put((rank, repr(e) + traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_ulysses_step_on_two_ranks_equals_one_rank():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_ulysses_dit, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, res in results:
        assert not isinstance(res, str), res
        for err, scale, shape, finite in res:      # pipelined (pooled, f32), then one exchange per tensor
            assert shape == (2, 4, 4, 16, 34) and finite
            # the runs differ only in GEMM row blocking (bf16 outputs) and the
            # exchanges, which move bytes unchanged
            assert err <= 2e-2 * scale, (rank, err, scale)


def test_reference_block_statistics_follow_the_pool_stage_arithmetic():
    """The torch mirror of icsa_dit_norm_rope_pool (used by the CPU
    sequence-parallel test) writes the block statistics with the pool stage's
    arithmetic: bf16 block sums of the bf16 outputs (rows added in order in
    float32, rounded once), the float32 means of q and k, and for v the mean
    bf16(bf16(sum) / 64)."""
    from _dit_reference import ReferenceOps
    g = torch.Generator().manual_seed(4)
    s, H, D = 128, 2, 64
    C = H * D
    src = torch.randn(s, C, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(C, generator=g)).to(torch.bfloat16)
    q = torch.empty(1, 1, s, H, D, dtype=torch.bfloat16)
    v = torch.empty_like(q)
    qm, vm = (torch.empty(1, 1, H, s // 64, D) for _ in range(2))
    qs, vs = (torch.empty(1, 1, H, s // 64, D, dtype=torch.bfloat16) for _ in range(2))
    ReferenceOps().norm_rope_pool([(src, w, False, q), (src, None, False, v)], [qm, vm], rows_per_batch=s,
                                  eps=1e-6, sums=[qs, vs], bf16_mean=(False, True))
    for out, mean, sums, bf16_mean in ((q, qm, qs, False), (v, vm, vs, True)):
        x = out[0, 0].float()                                  # [s, H, D], the bf16 outputs
        acc = torch.zeros(s // 64, H, D)
        for r in range(64):
            acc = acc + x.view(s // 64, 64, H, D)[:, r]
        assert torch.equal(sums[0, 0], acc.to(torch.bfloat16).permute(1, 0, 2))
        if bf16_mean:
            want = (acc.to(torch.bfloat16).float() / 64.0).to(torch.bfloat16).float()
            assert torch.equal(mean[0, 0], want.permute(1, 0, 2))
    assert torch.equal(v[0, 0], src.view(s, H, D))             # v passes through
