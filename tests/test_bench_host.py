"""CPU checks of the benchmark's definitions: the stage sweep covers BASELINE
configuration 4 with valid generator grids, and the algorithmic FLOP counts
that the roofline divides by are the ones quoted for the 480p call."""
import math

import bench
from in_context_sparse_attention import _capi, synthetic


def test_sweep_covers_configuration_4():
    assert sorted(2 * h for h in bench.SWEEP_GRIDS) == [8192, 16384, 32768, 65536, 131072]
    assert bench.SWEEP_FLAT == (0.0, 0.5, 1.0)
    assert bench.SWEEP_SRR == (0.0625, 0.125, 0.25)
    assert bench.SWEEP_BATCH == (1, 2)


def test_sweep_grids_fit_their_halves():
    for half, grid in bench.SWEEP_GRIDS.items():
        assert half % synthetic.BLOCK == 0
        n = math.prod(grid)
        # the generator fills the grid and pads the rest of the half with fresh rows
        assert half - synthetic.BLOCK < n <= half


def test_480p_attention_flops():
    p = _capi.problem(1, 65536, 40, 128, 32768)
    n_sparse = _capi.workspace_layout(p).n_sparse
    total, flat, sparse = bench.attention_flops(p, n_sparse)
    assert (p.num_flat, n_sparse, p.tkv, p.top_k, p.nkv) == (512, 512, 36864, 36, 576)
    assert flat == 4.0 * 40 * 32768 * 36864 * 128                      # 24.74 TFLOP
    assert sparse == 4.0 * 40 * 32768 * (36 * 64 + 576) * 128          # 1.93 TFLOP
    assert abs(total / 1e12 - 26.67) < 0.01
