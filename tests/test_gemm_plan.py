"""The GEMM template's launch plans on the CPU, for every BASELINE GEMM shape and the N-panel
each GPU gets at 2 / 4 / 8 GPUs: the module fits the SM (shared memory, TMEM, grid), the
grid covers the tiles, and tail K slices appear only past the last full wave and
account for every K block exactly once."""

import math

import pytest

from conftest import ROOT  # noqa: F401  (puts the package on sys.path)

SHAPES = [(8192, 8192, 8192), (4096, 14336, 4096), (2048, 2048, 2048), (512, 512, 512)]
SMS = 148
SMEM_MAX = 232448


def _panels():
    from baseline_configs import panel
    out = []
    for m, n, k in SHAPES:
        for world in (1, 2, 4, 8):
            n0, n1 = panel(n, 0, world)
            out.append((m, n1 - n0, k))
    return sorted(set(out))


@pytest.mark.parametrize("m,n,k", _panels())
@pytest.mark.parametrize("kind", ["bf16", "fp8"])
def test_plan_fits_and_covers(m, n, k, kind):
    from compiler import parse_launch
    from compiler.kernels.gemm import GemmConfig, choose_tiling, emit_gemm_module
    from compiler.kernels.quant import fp8_gemm_config
    if kind == "fp8":
        if (m, k) != (8192, 8192):
            pytest.skip("FP8 runs at 8192^3 and its panels only")
        cfg = fp8_gemm_config(m, n, k)
    else:
        cfg = GemmConfig(M=m, N=n, K=k, ab="bf16", c="bf16", name="k_plan", buffers=("a", "b", "c"),
                         **choose_tiling(m, n, 1))
    launch = parse_launch(emit_gemm_module(cfg))
    grid, smem = launch["grid"][0], launch["smem"]
    assert smem <= SMEM_MAX - 256, "the stage ring and staging exceed shared memory"
    assert cfg.BN * cfg.acc_bufs <= 512, "the TMEM accumulators exceed 512 columns"
    tm, tn = cfg.tiles
    tiles = tm * tn
    assert launch["tiles"] == tiles
    workers = SMS // 2 if cfg.pair else SMS
    if cfg.pair:
        assert launch["cluster"][0] == 2 and grid % 2 == 0
        assert grid // 2 == min(tiles, workers)
    else:
        assert grid <= SMS
    # tail slices: only past the last full wave, and the units count every K block once
    ts, tail_tiles = launch["tail_split"], launch["tail_tiles"]
    kblocks = math.ceil(k / cfg.BK)
    if ts > 1:
        full, rem = divmod(tiles, workers)
        assert full >= 1 and rem == tail_tiles and rem > 0
        assert kblocks % ts == 0
        units = (tiles - tail_tiles) + tail_tiles * ts
        assert (tiles - tail_tiles) * kblocks + tail_tiles * ts * (kblocks // ts) == tiles * kblocks
        assert units > tiles
        if k > 4096:
            assert ts <= 2, "8192-deep tiles are cut in two at most (measured)"
    else:
        assert tail_tiles == 0


def test_baseline_shapes_take_cta_pairs_and_small_ones_single_ctas():
    from compiler.kernels.gemm import choose_tiling
    for m, n, k in SHAPES[:3]:
        assert choose_tiling(m, n, 1)["pair"], (m, n, k)
    t = choose_tiling(512, 512, 1)
    assert not t["pair"] and t["BN"] == 64 and t["stages"] == 8
