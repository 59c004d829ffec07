"""CPU tests of the MoE tensor-parallel layout (128 experts, FFN 768,
TP=1/2/4/8): the uneven whole-group split, and that the rank shards of gate/up/down are
bit-exact slices whose partial block outputs sum to the unsharded output (oracle)."""
import numpy as np
import pytest


def test_group_split_uneven(vm):
    split = vm.distributed.group_split
    assert [split(12, 8, r) for r in range(8)] == [(0, 2), (2, 4), (4, 6), (6, 8), (8, 9), (9, 10), (10, 11),
                                                   (11, 12)]
    for world in (1, 2, 4, 8):
        parts = [split(12, world, r) for r in range(world)]
        assert parts[0][0] == 0 and parts[-1][1] == 12
        assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
        assert max(b - a for a, b in parts) - min(b - a for a, b in parts) <= 1


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_expert_partials_sum_to_full(vm, orc, world):
    """Per-rank partial outputs of the MoE FFN over the rank's intermediate slice (gate/up rows,
    down K columns at whole groups) add up to the full FFN output (fp64 oracle, 4-bit g64)."""
    rng = np.random.default_rng(world)
    E, D, F, gs, T, k = 4, 256, 768, 64, 3, 2
    mk = lambda n, kk, s: orc.quantize(orc.f32_to_bf16(rng.normal(0, 0.02, (E * n, kk)).astype(np.float32)),
                                       gs, 4)  # noqa: E731
    g = [a.reshape(E, F, -1) for a in mk(F, D, 1)]
    u = [a.reshape(E, F, -1) for a in mk(F, D, 2)]
    d = [a.reshape(E, D, -1) for a in mk(D, F, 3)]
    x = orc.f32_to_bf16(rng.normal(0, 1, (T, D)).astype(np.float32))
    inds = rng.integers(0, E, (T, k))
    full = orc.switch_glu(x, g, u, d, inds, gs, 4)
    acc = np.zeros_like(full)
    for r in range(world):
        g0, g1 = vm.distributed.group_split(F // gs, world, r)
        rs = slice(g0 * gs, g1 * gs)
        ws = slice(g0 * gs * 4 // 32, g1 * gs * 4 // 32)
        gr = [g[0][:, rs].copy(), g[1][:, rs].copy(), g[2][:, rs].copy()]
        ur = [u[0][:, rs].copy(), u[1][:, rs].copy(), u[2][:, rs].copy()]
        dr = [d[0][..., ws].copy(), d[1][..., g0:g1].copy(), d[2][..., g0:g1].copy()]
        acc += orc.switch_glu(x, gr, ur, dr, inds, gs, 4)
    # the activation is rounded to bf16 per element either way; only the K split of down differs
    assert np.abs(acc - full).max() <= 1e-3 * np.abs(full).max()
