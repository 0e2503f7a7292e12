"""The CPU oracle against the fixtures recorded from the reference's own code
(tests/golden/make_golden.py).  CPU only."""
import os

import pytest
import torch

from in_context_sparse_attention import synthetic
from oracle import icsa_oracle as orc

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def checksum(t):
    t = t.double()
    return [float(t.sum()), float(t.abs().sum()), float((t * t).sum())]


def test_triton_interval_pin():
    """Exact + interval term == the reference Triton kernel (BN = 64, fp32)."""
    fx = torch.load(os.path.join(GOLDEN, "triton_interval_pin.pt"))
    B, H, TQ, TKV, D = fx["shape"]
    g = torch.Generator().manual_seed(fx["seed"])
    q = torch.randn(B, H, TQ, D, generator=g)
    k = torch.randn(B, H, TKV, D, generator=g)
    v = torch.randn(B, H, TKV, D, generator=g)
    for t, ref in zip((q, k, v), fx["input_checksums"]):
        assert checksum(t) == pytest.approx(ref, rel=1e-12), "random generator changed; regenerate fixtures"
    NQ, NKV = TQ // 64, TKV // 64
    mine = orc.sparse_kernel(q[0, 0].view(NQ, 64, D), k[0, 0], v[0, 0], fx["kc"][0, 0], fx["vc"][0, 0],
                             fx["idx"][0, 0], NKV, round_p_bf16=False)
    assert float((mine.reshape(TQ, D) - fx["out"][0, 0]).abs().max()) < 1e-6


def test_interval_terms_are_not_rescaled():
    """A chunk whose max exceeds the running max re-weights acc/l but not the
    earlier g terms (the reference's quirk): compare with a rescaled variant."""
    g = torch.Generator().manual_seed(0)
    D = 64
    q = torch.randn(1, 64, D, generator=g)
    k = torch.randn(256, D, generator=g) * 0.1
    v = torch.randn(256, D, generator=g)
    kc = k.view(4, 64, D).sum(1)
    vc = v.view(4, 64, D).sum(1)
    kc[3] = q[0, 0] * 400.0  # late block with a dominant mean score
    idx = torch.tensor([[0]])
    out = orc.sparse_kernel(q, k, v, kc, vc, idx, 4, round_p_bf16=False)
    assert torch.isfinite(out).all()


def test_config1_orchestration_matches_reference():
    """The oracle's own orchestration reproduces the reference's
    editing_sparse_attention on BASELINE configuration 1 (fp32)."""
    fx = torch.load(os.path.join(GOLDEN, "config1_reference.pt"))
    w = synthetic.CONFIG1
    q, k, v = synthetic.make_inputs(w)
    for t, ref in zip((q, k, v), fx["input_checksums"]):
        assert checksum(t) == pytest.approx(ref, rel=1e-12), "random generator changed; regenerate fixtures"
    o = orc.editing_sparse_attention(q, k, v, w.t_seq_len)
    c = o.counts
    assert c.topK == 8 and c.nkv == 72 and c.top_k == 4 and c.k_sparsity == 4
    assert torch.equal(o.sel, fx["sel"])
    assert torch.equal(o.order[..., :c.num_flat].sort(-1).values, fx["order"][..., :c.num_flat].sort(-1).values)
    torch.testing.assert_close(o.colsum.float(), fx["colsum"], rtol=1e-6, atol=1e-7)
    torch.testing.assert_close(o.sharp.float(), fx["sharp"], rtol=1e-6, atol=1e-7)
    assert float((o.out[:, ::13] - fx["out_rows"]).abs().max()) < 1e-6


def test_select_desc_ties_go_to_lower_index():
    keys = torch.tensor([[1.0, 3.0, 3.0, 2.0, 3.0, -0.0, 0.0]])
    assert orc.select_desc(keys, 7).tolist() == [[1, 2, 4, 3, 0, 5, 6]]


def test_counts_follow_reference_formulas():
    c = orc.Counts.make(1, 65536, 40, 128, 32768)
    assert (c.NB, c.n_t, c.n_s, c.topK, c.num_flat, c.k_sparsity, c.tkv, c.nkv, c.top_k) == \
        (1024, 512, 512, 64, 512, 32, 36864, 576, 36)
    c = orc.Counts.make(1, 151296, 40, 128, 75648)
    assert (c.NB, c.topK, c.tkv, c.nkv, c.top_k) == (2364, 147, 85056, 1329, 83)
