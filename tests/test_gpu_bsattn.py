"""Block-sparse attention forward through the C ABI vs the reference's torch path (SDPA with the dense
boolean mask) and the fp64 block-sparse restatement.

Tolerance: the output is bf16, whose own rounding already costs ~2e-3 normwise, so the 1e-3 fp64 bar
is applied above that floor: err_vs_fp64 <= max(1e-3, 1.25 * floor + 1e-3 ... ) is written below as
err <= floor + 1e-3, where floor = ||bf16(ref64) - ref64|| / ||ref64||. The kernel must also be at least
as close to fp64 as the reference's own bf16 SDPA path is (within 10 %)."""
import math

import pytest
import torch

from oracle import reference_path as ref
from periodicdent42_b200 import _capi
from periodicdent42_b200 import workloads as wl

pytestmark = pytest.mark.gpu


def _run(q, k, v, row_ptr, col_idx, scale, causal=True, bh=None):
    dev = torch.device("cuda", 0)
    O = torch.full_like(q, float("nan"), device=dev)
    b0, b1 = (0, q.shape[0] * q.shape[1]) if bh is None else bh
    _capi.bsattn_fwd_bf16(q.to(dev), k.to(dev), v.to(dev), O, row_ptr.to(torch.int32).to(dev),
                          col_idx.to(torch.int32).to(dev), scale, causal, b0, b1)
    torch.cuda.synchronize()
    return O.cpu()


def _check(O, q, k, v, rp, ci, scale, causal, nqb, pairs):
    B, H, S, D = q.shape
    for p in pairs:
        b, h = divmod(p, H)
        r0, r1 = p * nqb, (p + 1) * nqb
        ref64 = ref.attn_blocksparse_fp64(q[b, h], k[b, h], v[b, h], rp[r0:r1 + 1], ci[rp[r0]:rp[r1]], scale, causal)
        floor = ref.bf16_storage_floor(ref64)
        err = ref.normwise_rel_err(O[b, h], ref64)
        assert err <= floor + 1e-3, (p, err, floor)
        bm = wl.block_mask_dense(rp[r0:r1 + 1], ci[rp[r0]:rp[r1]], nqb, nqb)
        dm = wl.dense_mask_from_blocks(bm, 128, causal)
        sd = ref.attn_sdpa_ref(q[b, h][None, None], k[b, h][None, None], v[b, h][None, None], dm, scale)[0, 0]
        rows = dm.any(dim=1)
        err_sdpa = ref.normwise_rel_err(sd[rows], ref64[rows])
        assert err <= 1.1 * err_sdpa + 2e-4, (p, err, err_sdpa)


@pytest.mark.parametrize("B,H,S", [(1, 1, 256), (1, 2, 1024), (2, 2, 2048)])
def test_bsattn_config_mask(no_device_error, B, H, S):
    cfg = wl.AttnCfg(B, H, S, 128, 128, 4, 8, 4)
    q, k, v = wl.attn_inputs(cfg, "cpu")
    rp, ci = wl.attn_mask_bsr(cfg)
    scale = 1.0 / math.sqrt(128)
    O = _run(q, k, v, rp, ci, scale)
    assert torch.isfinite(O.float()).all()
    _check(O, q, k, v, rp, ci, scale, True, S // 128, range(B * H))


def test_bsattn_dense_noncausal(no_device_error):
    cfg = wl.AttnCfg(1, 2, 512, 128, 128, 4, 0, 7)
    q, k, v = wl.attn_inputs(cfg, "cpu")
    nqb = 4
    bm = torch.ones(nqb, nqb, dtype=torch.bool)
    crow, col = wl.mask_to_bsr(bm)
    rp = torch.cat([crow, crow[1:] + crow[-1]])
    ci = torch.cat([col, col])
    O = _run(q, k, v, rp, ci, 0.1, causal=False)
    _check(O, q, k, v, rp, ci, 0.1, False, nqb, range(2))


def test_bsattn_empty_rows_zero_and_bh_range(no_device_error):
    cfg = wl.AttnCfg(1, 3, 512, 128, 128, 4, 8, 9)
    q, k, v = wl.attn_inputs(cfg, "cpu")
    bm = torch.tensor([[1, 0, 0, 0], [0, 0, 0, 0], [1, 1, 1, 0], [0, 1, 0, 1]], dtype=torch.bool)
    crow, col = wl.mask_to_bsr(bm)
    rp = torch.cat([crow, crow[1:] + crow[-1], crow[1:] + 2 * crow[-1]])
    ci = torch.cat([col, col, col])
    dev = torch.device("cuda", 0)
    O = torch.full(q.shape, 3.0, dtype=torch.bfloat16, device=dev)
    _capi.bsattn_fwd_bf16(q.to(dev), k.to(dev), v.to(dev), O, rp.to(torch.int32).to(dev),
                          ci.to(torch.int32).to(dev), 0.088, True, 1, 2)
    torch.cuda.synchronize()
    O = O.cpu()
    assert torch.all(O[0, 0] == 3.0) and torch.all(O[0, 2] == 3.0)  # pairs outside [1,2) untouched
    assert torch.count_nonzero(O[0, 1, 128:256]) == 0  # empty mask row -> zeros
    _check(O, q, k, v, rp, ci, 0.088, True, 4, [1])


def test_bsattn_deterministic(no_device_error):
    cfg = wl.AttnCfg(1, 2, 1024, 128, 128, 4, 8, 4)
    q, k, v = wl.attn_inputs(cfg, "cpu")
    rp, ci = wl.attn_mask_bsr(cfg)
    a = _run(q, k, v, rp, ci, 0.0883)
    b = _run(q, k, v, rp, ci, 0.0883)
    assert torch.equal(a, b)


def test_bsattn_rejects_head_dim(cuda_dev):
    q = torch.zeros(1, 1, 128, 64, dtype=torch.bfloat16, device=cuda_dev)
    rp = torch.tensor([0, 1], dtype=torch.int32, device=cuda_dev)
    ci = torch.tensor([0], dtype=torch.int32, device=cuda_dev)
    with pytest.raises(_capi.BskError) as e:
        _capi.bsattn_fwd_bf16(q, q, q, torch.empty_like(q), rp, ci, 0.125)
    assert e.value.code == _capi.BSK_ERR_UNSUPPORTED
