"""GPU parity of the DiT harness's fused passes (libicsa.so, include/icsa_dit.h)
and of whole blocks against the reference's block math restated in torch
(tests/_dit_reference.py).

Tolerances: the fused passes round exactly where the reference rounds, so
they agree with the restatement except where a float32 row statistic
(mean, variance, mean square) summed in a different order moves a value
across a bf16 rounding boundary: such elements must stay within one bf16
unit (or 1e-6 where `n * scale + shift` cancels) and be rare.  The gate and
the residual update are elementwise with identical rounding and must agree
bit for bit.  Whole steps (two tiny blocks; one full-width block) are bf16
GEMM chains in which a last-bit change of q or k can flip a block
selection; they agree with the restated model within 1e-2 in mean-abs
(relative to the output's mean magnitude), 3e-2 at the 99.9th percentile
and 0.15 at the maximum (relative to its largest value)."""
import pytest
import torch

from _dit_reference import ReferenceOps

pytestmark = pytest.mark.gpu

TINY = dict(dim=256, ffn_dim=512, num_heads=2, num_layers=2, freq_dim=32, text_dim=64, text_len=16, in_dim=4,
            out_dim=4)


@pytest.fixture(scope="module")
def ops(cuda_device):
    from wan_dit._ops import CudaOps
    return CudaOps()


def bf16_ulps(a, b):
    """Distance in units of the bf16 spacing at |b|."""
    a, b = a.float(), b.float()
    ulp = torch.ldexp(torch.ones_like(b), (torch.frexp(b.abs().clamp_min(1e-30))[1] - 8))
    return (a - b).abs() / ulp


def assert_step_close(got, ref):
    """Whole-model outputs: bf16 GEMM chains plus the few selections that a
    last-bit change of q or k can flip; judged on the mean and on the tail."""
    err = (got - ref).abs().flatten().float()
    rel_mean = float(err.mean() / ref.abs().mean())
    rel_q999 = float(torch.quantile(err[:: max(1, err.numel() // 1000000)], 0.999) / ref.abs().max())
    rel_max = float(err.max() / ref.abs().max())
    print(f"step vs restated model: rel mean {rel_mean:.2e}, rel q99.9 {rel_q999:.2e}, rel max {rel_max:.2e}")
    assert rel_mean <= 1e-2 and rel_q999 <= 3e-2 and rel_max <= 0.15, (rel_mean, rel_q999, rel_max)


def assert_bf16_close(got, ref, max_ulps=1.0, max_frac=2e-3, atol=1e-6):
    """At most one bf16 unit apart, or `atol` apart where `n * scale + shift`
    cancels to a value much smaller than its terms (a float32 unit of the
    terms is then many bf16 units of the result); differences rare."""
    d = (got.float() - ref.float()).abs()
    u = bf16_ulps(got, ref)
    frac = float((d > 0).float().mean())
    bad = (u > max_ulps) & (d > atol)
    assert not bool(bad.any()) and frac <= max_frac, (float(u.max()), float(d.max()), frac)


@pytest.mark.parametrize("C,rows,xdt,round_norm", [(5120, 1031, torch.float32, False),
                                                    (5120, 512, torch.bfloat16, True),
                                                    (256, 300, torch.float32, False),
                                                    (6144, 64, torch.float32, False)])
def test_modulated_norm_matches_reference_math(ops, C, rows, xdt, round_norm):
    g = torch.Generator(device="cuda").manual_seed(C + rows)
    B = 2 if rows % 2 == 0 else 1
    x = (torch.randn(rows, C, generator=g, device="cuda") * 3 + 0.5).to(xdt)
    scale = 1 + 0.1 * torch.randn(B, C, generator=g, device="cuda")
    shift = 0.1 * torch.randn(B, C, generator=g, device="cuda")
    got = ops.modulated_norm(x, scale, shift, rows // B, 1e-6, round_norm)
    ref = ReferenceOps().modulated_norm(x, scale, shift, rows // B, 1e-6, round_norm)
    assert got.dtype == torch.bfloat16 and got.shape == (rows, C)
    atol = 1e-6
    if round_norm:
        # the normalised value is itself rounded to bf16 first: a flip there
        # moves the result by one bf16 unit of n times the scale
        n = torch.nn.functional.layer_norm(x.float(), (C,), eps=1e-6)
        per_row = scale[torch.arange(rows, device="cuda") // (rows // B)]
        atol = 1e-6 + 2.0 ** -6 * n.abs() * per_row.abs()
    assert_bf16_close(got, ref, atol=atol)


def test_affine_norm_shares_one_weight_row(ops):
    C, rows = 5120, 256
    x = torch.randn(rows, C, device="cuda")
    w = 1 + 0.1 * torch.randn(C, device="cuda")
    b = 0.1 * torch.randn(C, device="cuda")
    got = ops.modulated_norm(x, w, b, 128, 1e-6)
    ref = ReferenceOps().modulated_norm(x, w, b, 128, 1e-6)
    assert_bf16_close(got, ref)


@pytest.mark.parametrize("groups", [1, 2, 8])
def test_norm_rope_matches_reference_math_and_layout(ops, groups):
    from wan_dit import head_dim_splits, rope_table, token_positions
    B, H, D = 2, 40, 128
    C = H * D
    grid = (3, 8, 10)                       # 240 tokens per video
    S = 2 * 240 + 16
    s = S // groups
    rank = groups - 1                       # the last shard: source tokens and padding
    g = torch.Generator(device="cuda").manual_seed(groups)
    qkv = torch.randn(B * s, 3 * C + 8, generator=g, device="cuda").to(torch.bfloat16)
    wq = (1 + 0.1 * torch.randn(C, generator=g, device="cuda")).to(torch.bfloat16)
    wk = (1 + 0.1 * torch.randn(C, generator=g, device="cuda")).to(torch.bfloat16)
    table = rope_table(D).cuda()
    pos = token_positions(grid, grid, S).cuda()
    hp = H // groups
    outs = {}
    for name, impl in (("got", ops), ("ref", ReferenceOps())):
        q = torch.empty(B, groups, s, hp, D, device="cuda")
        k = torch.empty_like(q)
        v = torch.empty(B, groups, s, hp, D, dtype=torch.bfloat16, device="cuda")
        gate = torch.empty(B * s, dtype=torch.bfloat16, device="cuda")
        impl.norm_rope([(qkv[:, :C], wq, True, q), (qkv[:, C:2 * C], wk, True, k), (qkv[:, 2 * C:3 * C], None, False, v)],
                       rows_per_batch=s, eps=1e-6, token_offset=rank * s, table=table, token_pos=pos,
                       splits=head_dim_splits(D), gate=(qkv[:, 3 * C], gate))
        outs[name] = (q, k, v, gate)
    (q, k, v, gate), (rq, rk, rv, rgate) = outs["got"], outs["ref"]
    assert torch.equal(v, rv) and torch.equal(gate, rgate)
    for a, b in ((q, rq), (k, rk)):
        d = (a - b).abs()
        exact = float((d == 0).float().mean())
        # rotated bf16 values: a bf16 flip of the RMSNorm output moves a pair by about one bf16 unit
        assert exact >= 0.998 and float(d.max()) <= 2 ** -7 * float(b.abs().max()), (exact, float(d.max()))


def test_gated_residual_is_bit_exact(ops):
    rows, C, B = 512, 5120, 2
    x = torch.randn(rows, C, device="cuda")
    y = torch.randn(rows, 3 * C, device="cuda").to(torch.bfloat16)[:, C:2 * C]
    gate = torch.randn(B, C, device="cuda")
    a, b = x.clone(), x.clone()
    ops.gated_residual_(a, y, gate, rows // B)
    ReferenceOps().gated_residual_(b, y, gate, rows // B)
    assert torch.equal(a, b)
    ops.gated_residual_(a, y, None, rows // B)
    ReferenceOps().gated_residual_(b, y, None, rows // B)
    assert torch.equal(a, b)


def test_invalid_arguments_raise(ops):
    from in_context_sparse_attention._capi import IcsaError
    x = torch.randn(4, 100, device="cuda")          # C not a multiple of 8
    with pytest.raises(IcsaError):
        ops.modulated_norm(x, torch.ones(100, device="cuda"), torch.zeros(100, device="cuda"), 4, 1e-6)


def _tiny_inputs(cfg, grid=(4, 16, 34)):
    g = torch.Generator().manual_seed(0)
    latent = torch.randn(cfg.in_dim, *grid, generator=g)
    source = 0.8 * latent + 0.6 * torch.randn(cfg.in_dim, *grid, generator=g)
    context = torch.randn(2, cfg.text_len, cfg.text_dim, generator=g)
    return latent.cuda(), source.cuda(), context.cuda()


def test_tiny_dit_step_matches_reference_block_math(ops):
    """Two blocks with the product path (fused passes + sparse attention
    kernels) against the reference's math with the CPU oracle attention."""
    from wan_dit import WanDiT, WanDiTConfig
    cfg = WanDiTConfig(**TINY)
    latent, source, context = _tiny_inputs(cfg)
    seq_len = 2 * 4 * 8 * 17 + 32
    got = WanDiT(cfg, seed=3, ops=ops).forward(latent, source, 500.0, context, seq_len)
    ref = WanDiT(cfg, seed=3, ops=ReferenceOps()).forward(latent, source, 500.0, context, seq_len)
    assert got.shape == ref.shape == (2, 4, 4, 16, 34)
    assert_step_close(got, ref)


def test_full_width_block_matches_reference_block_math(ops):
    """One A14B-width block (C = 5120, 40 heads, FFN 13824) on a short
    sequence: the fused passes at full width against the reference's math,
    both using this package's attention so that only the elementwise chain
    is compared."""
    from wan_dit import WanDiT, WanDiTConfig
    cfg = WanDiTConfig(num_layers=1)
    grid = (2, 16, 32)                      # 256 tokens per video after 2x2 patches
    g = torch.Generator().manual_seed(1)
    latent = torch.randn(cfg.in_dim, 2, 32, 64, generator=g).cuda()
    source = (0.8 * latent.cpu() + 0.6 * torch.randn(latent.shape, generator=g)).cuda()
    context = torch.randn(2, cfg.text_len, cfg.text_dim, generator=g).cuda()
    seq_len = 2 * 2 * 16 * 32 + 64
    got = WanDiT(cfg, seed=5, ops=ops).forward(latent, source, 900.0, context, seq_len)
    ref = WanDiT(cfg, seed=5, ops=ReferenceOps(attention=ops.self_attention)).forward(
        latent, source, 900.0, context, seq_len)
    assert got.shape == (2, cfg.out_dim, 2, 32, 64) and bool(torch.isfinite(got).all())
    assert grid == (2, 16, 32)
    assert_step_close(got, ref)


@pytest.mark.parametrize("grid,S,t_aligned", [((4, 16, 32), 4096, True), ((3, 10, 17), 1024, False)])
def test_pooled_qk_give_the_f32_call_bit_for_bit(ops, grid, S, t_aligned):
    """The sequence-parallel exchange sends q and k as bf16 with the f32
    means of their 64-token blocks: the means equal those the pool stage
    takes of the f32 tensors, and the attention's output equals the f32
    call's bit for bit (aligned and unaligned t_seq_len).  With the v means
    and the bf16 block sums of q, k, v from the same producer pass, every
    pooled statistic equals the pool stage's, and the attention without its
    pooling pass still gives the same bits."""
    from wan_dit import head_dim_splits, rope_table, token_positions
    from _helpers import region
    from in_context_sparse_attention import editing_sparse_attention
    B, H, D = 1, 8, 128
    C = H * D
    t = grid[0] * grid[1] * grid[2]
    assert (t % 64 == 0) == t_aligned
    g = torch.Generator(device="cuda").manual_seed(11)
    qkv = torch.randn(B * S, 3 * C + 8, generator=g, device="cuda").to(torch.bfloat16)
    wq = (1 + 0.1 * torch.randn(C, generator=g, device="cuda")).to(torch.bfloat16)
    wk = (1 + 0.1 * torch.randn(C, generator=g, device="cuda")).to(torch.bfloat16)
    table, pos, splits = rope_table(D).cuda(), token_positions(grid, grid, S).cuda(), head_dim_splits(D)
    jobs = lambda q, k, v: [(qkv[:, :C], wq, True, q), (qkv[:, C:2 * C], wk, True, k),  # noqa: E731
                            (qkv[:, 2 * C:3 * C], None, False, v)]
    q32 = torch.empty(B, 1, S, H, D, device="cuda")
    k32 = torch.empty_like(q32)
    v_a = torch.empty(B, 1, S, H, D, dtype=torch.bfloat16, device="cuda")
    gate_a = torch.empty(B * S, dtype=torch.bfloat16, device="cuda")
    ops.norm_rope(jobs(q32, k32, v_a), rows_per_batch=S, eps=1e-6, table=table, token_pos=pos, splits=splits,
                  gate=(qkv[:, 3 * C], gate_a))
    qb, kb, v_b = (torch.empty(B, 1, S, H, D, dtype=torch.bfloat16, device="cuda") for _ in range(3))
    qm = torch.empty(B, 1, H, S // 64, D, device="cuda")
    km = torch.empty_like(qm)
    gate_b = torch.empty(B * S, dtype=torch.bfloat16, device="cuda")
    ops.norm_rope_pool(jobs(qb, kb, v_b), [qm, km, None], rows_per_batch=S, eps=1e-6, table=table, token_pos=pos,
                       splits=splits, gate=(qkv[:, 3 * C], gate_b))
    assert torch.equal(qb, q32.to(torch.bfloat16)) and torch.equal(kb, k32.to(torch.bfloat16))
    assert torch.equal(v_a, v_b) and torch.equal(gate_a, gate_b)
    # the means are the pool stage's means of the f32 tensors
    dbg = {}
    editing_sparse_attention(q32.view(B, S, H, D), k32.view(B, S, H, D), v_a.view(B, S, H, D), t, S - t, _debug=dbg)
    NB = S // 64
    assert torch.equal(qm.view(B, H, NB, D), region(dbg, "qmean", torch.float32, (B, H, NB, D)))
    assert torch.equal(km.view(B, H, NB, D), region(dbg, "kmean", torch.float32, (B, H, NB, D)))
    alpha = gate_a.view(B, S)
    out_a = ops.self_attention(q32.view(B, S, H, D), k32.view(B, S, H, D), v_a.view(B, S, H, D), alpha, t)
    out_b = ops.self_attention(qb.view(B, S, H, D), kb.view(B, S, H, D), v_b.view(B, S, H, D), alpha, t,
                               means=(qm.view(B, H, NB, D), km.view(B, H, NB, D)))
    assert torch.equal(out_a, out_b)
    # every block statistic of the pool stage from the producer pass: the
    # attention then skips its pooling pass and still gives the same bits
    stats = [torch.empty(B, 1, H, S // 64, D, device="cuda") for _ in range(3)]
    sums = [torch.empty(B, 1, H, S // 64, D, dtype=torch.bfloat16, device="cuda") for _ in range(3)]
    ops.norm_rope_pool(jobs(qb, kb, v_b), stats, rows_per_batch=S, eps=1e-6, table=table, token_pos=pos,
                       splits=splits, gate=(qkv[:, 3 * C], gate_b), sums=sums, bf16_mean=(False, False, True))
    assert torch.equal(stats[0], qm) and torch.equal(stats[1], km)
    for name, x, dt in (("vmean", stats[2], torch.float32), ("qsum", sums[0], torch.bfloat16),
                        ("ksum", sums[1], torch.bfloat16), ("vsum", sums[2], torch.bfloat16)):
        assert torch.equal(x.view(B, H, NB, D), region(dbg, name, dt, (B, H, NB, D))), name
    out_c = ops.self_attention(qb.view(B, S, H, D), kb.view(B, S, H, D), v_b.view(B, S, H, D), alpha, t,
                               means=tuple(x.view(B, H, NB, D) for x in stats + sums))
    assert torch.equal(out_a, out_c)


@pytest.mark.parametrize("shape", [
    # B, Lq, Lk, H, D, v taken from a k|v GEMM output (strided rows)
    (2, 4096, 512, 4, 128, True),    # the DiT's shape: 512 text tokens
    (2, 1000, 77, 3, 128, False),    # partial query and key blocks
    (1, 2048, 512, 2, 64, True),     # D = 64 (single-SM kernel)
])
def test_cross_attention_kernel_matches_fp32_attention(ops, shape):
    """icsa_dit_cross_attention (the dense tcgen05 attention kernel without
    order table, block table or residual) against softmax attention in fp32:
    max-abs <= 2e-2 and mean-abs <= 1e-3, the tolerance of the attention
    output in bf16."""
    B, Lq, Lk, H, D, strided = shape
    g = torch.Generator(device="cuda").manual_seed(Lq + Lk + D)
    q = torch.randn(B, Lq, H, D, device="cuda", generator=g).to(torch.bfloat16)
    if strided:
        kv = torch.randn(B * Lk, 2 * H * D, device="cuda", generator=g).to(torch.bfloat16)
        k = kv[:, :H * D].view(B, Lk, H, D)
        v = kv[:, H * D:].view(B, Lk, H, D)
        assert v.stride(1) == 2 * H * D
    else:
        k, v = (torch.randn(B, Lk, H, D, device="cuda", generator=g).to(torch.bfloat16) for _ in range(2))
    got = ops.cross_attention(q, k, v)
    torch.cuda.synchronize()
    ref = ReferenceOps.cross_attention(q, k, v)
    s = torch.einsum("blhd,bkhd->bhlk", q.float(), k.float()) / D ** 0.5
    exact = torch.einsum("bhlk,bkhd->blhd", s.softmax(-1), v.float())
    d = (got.float() - exact).abs()
    print(f"cross attention {shape}: max|d|={float(d.max()):.3e} mean|d|={float(d.mean()):.3e}")
    assert got.shape == (B, Lq, H, D) and got.dtype == torch.bfloat16
    assert float(d.max()) <= 2e-2 and float(d.mean()) <= 1e-3
    assert float((got.float() - ref.float()).abs().mean()) <= 1e-3


@pytest.mark.parametrize("shape", [
    # M, N, K, batches, gate, bias
    (512, 256, 128, 1, True, True),
    (1000, 768, 520, 2, True, True),     # partial row tile, K not a multiple of 64, two batches
    (777, 512, 256, 1, False, False),    # no gate (cross-attention o-projection), no bias
    (4096, 5120, 5120, 2, True, True),   # the DiT's o-projection shape on 32 rank-local tokens x 128
])
def test_linear_residual_matches_library_gemm_then_residual(ops, shape):
    """icsa_dit_linear_residual (tcgen05 GEMM with the residual update in its
    epilogue) against cuBLAS (F.linear, bf16 out) followed by the float32
    update.  The bf16 layer output can differ by one bf16 unit where the two
    float32 accumulations straddle a rounding boundary, so each element of x
    may differ by at most one unit of y times |gate| (plus the float32
    rounding of the sum), and such elements must be a small fraction."""
    M, N, K, nb, use_gate, use_bias = shape
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    a = (torch.randn(M, K, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) * K ** -0.5).to(torch.bfloat16)
    b = (torch.randn(N, device="cuda", generator=g) * 0.1).to(torch.bfloat16) if use_bias else None
    x0 = torch.randn(M, N, device="cuda", generator=g)
    gate = torch.randn(nb, N, device="cuda", generator=g) if use_gate else None
    rpb = -(-M // nb)
    got = ops.linear_residual_(x0.clone(), a, w, b, gate, rpb)
    y = torch.nn.functional.linear(a, w, b)
    ref = ReferenceOps().gated_residual_(x0.clone(), y, gate, rpb)
    torch.cuda.synchronize()
    gv = gate[torch.arange(M, device="cuda") // rpb] if use_gate else torch.ones(M, N, device="cuda")
    ulp = torch.ldexp(torch.ones_like(y.float()), torch.frexp(y.float().abs().clamp_min(1e-30))[1] - 8)
    bound = ulp * gv.abs() * 1.01 + ref.abs() * 2.0 ** -22 + 1e-30
    d = (got - ref).abs()
    frac = float((d > 0).float().mean())
    print(f"linear_residual {shape}: max|d|={float(d.max()):.3e} differing={frac:.4f}")
    assert bool((d <= bound).all()), float((d / bound).max())
    assert frac <= 0.05
