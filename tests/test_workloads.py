"""Host logic: seeded generators, block-mask / BSR builders and shard planners (no GPU)."""
import torch

from periodicdent42_b200 import workloads as wl


def test_bsr_pattern_fixed_nnz_sorted_unique():
    crow, col = wl.bsr_pattern(64, 64, 16, torch.Generator().manual_seed(3))
    assert crow.tolist() == [16 * i for i in range(65)]
    for r in range(64):
        seg = col[crow[r]:crow[r + 1]]
        assert torch.all(seg[1:] > seg[:-1]) and seg.min() >= 0 and seg.max() < 64


def test_attention_mask_rows_follow_the_workload_rule():
    cfg = wl.AttnCfg(1, 2, 128 * 40, 128, 128, 4, 8, 4)
    rp, ci = wl.attn_mask_bsr(cfg)
    nqb = 40
    for p in range(2):
        for i in range(nqb):
            row = ci[rp[p * nqb + i]:rp[p * nqb + i + 1]].tolist()
            window = list(range(max(0, i - 3), i + 1))
            assert row == sorted(set(row)), "sorted, distinct"
            assert all(w in row for w in window)
            rnd = [c for c in row if c not in window]
            assert len(rnd) == min(8, max(0, i - 3))
            assert all(0 <= c <= i - 4 for c in rnd)
    # full workload: 1470 blocks per (b,h) pair
    assert sum(min(i + 1, 4) + min(8, max(0, i - 3)) for i in range(128)) == 1470


def test_attention_mask_is_seeded():
    cfg = wl.AttnCfg(1, 1, 128 * 24, 128, 128, 4, 8, 4)
    a = wl.attn_mask_bsr(cfg)
    b = wl.attn_mask_bsr(cfg)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_mask_to_bsr_matches_torch_to_sparse_bsr():
    g = torch.Generator().manual_seed(0)
    m = torch.rand(6, 5, generator=g) < 0.4
    crow, col = wl.mask_to_bsr(m)
    t = m.repeat_interleave(4, 0).repeat_interleave(4, 1).float().to_sparse_bsr((4, 4))
    assert torch.equal(crow, t.crow_indices()) and torch.equal(col, t.col_indices())


def test_dense_mask_diag_causal():
    bm = torch.tensor([[1, 0], [1, 1]], dtype=torch.bool)
    m = wl.dense_mask_from_blocks(bm, 4, True)
    assert m[0, 1] == False and m[1, 0] == True and m[5, 2] == True and m[5, 6] == False and m[6, 5] == True  # noqa: E712
    assert m[0, 4] == False  # noqa: E712  (block not in the mask)


def test_shard_ranges_partition_and_balance():
    for w, n in [([16] * 64, 8), ([1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12] * 5, 4), ([5], 3), ([0, 0, 9, 0], 2)]:
        rs = wl.shard_ranges(w, n)
        assert len(rs) == n and rs[0][0] == 0 and rs[-1][1] == len(w)
        assert all(rs[i][1] == rs[i + 1][0] for i in range(n - 1))
        loads = [sum(w[a:b]) for a, b in rs]
        assert max(loads) - min(loads) <= max(w)
    assert wl.shard_ranges([16] * 64, 8) == [(8 * i, 8 * i + 8) for i in range(8)]


def test_even_ranges_alignment():
    rs = wl.even_ranges(8192, 8, align=256)
    assert rs == [(1024 * i, 1024 * (i + 1)) for i in range(8)]
    rs = wl.even_ranges(237568, 3, align=64)
    assert rs[0][0] == 0 and rs[-1][1] == 237568 and all(a % 64 == 0 for a, _ in rs)


def test_quantize_e4m3_recipe():
    x = torch.tensor([[0.5, -2.0], [4.0, 1.0]])
    q, s = wl.quantize_e4m3(x)
    assert abs(s.item() - 4.0 / 448.0) < 1e-9
    assert q.float().abs().max().item() == 448.0


def test_dense_inputs_k_slice_is_a_prefix_distribution():
    cfg = wl.DenseCfg(64, 32, 4096, 1, "scaled_normal")
    A, Bt = wl.dense_inputs(cfg, "cpu", k_slice=256)
    assert A.shape == (64, 256) and Bt.shape == (32, 256) and A.dtype == torch.float16
    assert abs(A.float().std().item() - 4096 ** -0.25) < 0.02
