"""Block-sparse attention forward through the C ABI vs the reference's torch path (SDPA with the dense
boolean mask) and the fp64 block-sparse restatement, for bf16 and fp16 and head dims 64 and 128.

Tolerance: the output is bf16 or fp16, whose own rounding already costs ~2e-3 (bf16) or ~3e-4 (fp16)
normwise, so the 1e-3 fp64 bar is applied above that floor: err <= floor + 1e-3, where
floor = ||round(ref64) - ref64|| / ||ref64|| in the output type. The kernel must also be at least as close
to fp64 as the reference's own SDPA path in the same type is (within 10 %, plus 2e-4)."""
import math

import pytest
import torch

from oracle import reference_path as ref
from periodicdent42_b200 import _capi
from periodicdent42_b200 import workloads as wl

pytestmark = pytest.mark.gpu


def _fwd(q):
    return _capi.bsattn_fwd_f16 if q.dtype == torch.float16 else _capi.bsattn_fwd_bf16


def _run(q, k, v, row_ptr, col_idx, scale, causal=True, bh=None):
    dev = torch.device("cuda", 0)
    O = torch.full_like(q, float("nan"), device=dev)
    b0, b1 = (0, q.shape[0] * q.shape[1]) if bh is None else bh
    _fwd(q)(q.to(dev), k.to(dev), v.to(dev), O, row_ptr.to(torch.int32).to(dev), col_idx.to(torch.int32).to(dev), scale,
            causal, b0, b1)
    torch.cuda.synchronize()
    return O.cpu()


def _check(O, q, k, v, rp, ci, scale, causal, nqb, pairs):
    B, H, S, D = q.shape
    for p in pairs:
        b, h = divmod(p, H)
        r0, r1 = p * nqb, (p + 1) * nqb
        ref64 = ref.attn_blocksparse_fp64(q[b, h], k[b, h], v[b, h], rp[r0:r1 + 1], ci[rp[r0]:rp[r1]], scale, causal)
        floor = ref.normwise_rel_err(ref64.to(O.dtype), ref64)
        err = ref.normwise_rel_err(O[b, h], ref64)
        assert err <= floor + 1e-3, (p, err, floor)
        bm = wl.block_mask_dense(rp[r0:r1 + 1], ci[rp[r0]:rp[r1]], nqb, nqb)
        dm = wl.dense_mask_from_blocks(bm, 128, causal)
        sd = ref.attn_sdpa_ref(q[b, h][None, None], k[b, h][None, None], v[b, h][None, None], dm, scale)[0, 0]
        rows = dm.any(dim=1)
        err_sdpa = ref.normwise_rel_err(sd[rows], ref64[rows])
        assert err <= 1.1 * err_sdpa + 2e-4, (p, err, err_sdpa)


_TYPES = [(torch.bfloat16, 128), (torch.bfloat16, 64), (torch.float16, 128), (torch.float16, 64)]


@pytest.mark.parametrize("dtype,D", _TYPES)
@pytest.mark.parametrize("B,H,S", [(1, 1, 256), (1, 2, 1024), (2, 2, 2048)])
def test_bsattn_config_mask(no_device_error, B, H, S, dtype, D):
    cfg = wl.AttnCfg(B, H, S, D, 128, 4, 8, 4)
    q, k, v = wl.attn_inputs(cfg, "cpu", dtype)
    rp, ci = wl.attn_mask_bsr(cfg)
    scale = 1.0 / math.sqrt(D)
    O = _run(q, k, v, rp, ci, scale)
    assert O.dtype == dtype and torch.isfinite(O.float()).all()
    _check(O, q, k, v, rp, ci, scale, True, S // 128, range(B * H))


@pytest.mark.parametrize("dtype,D", _TYPES)
def test_bsattn_dense_noncausal(no_device_error, dtype, D):
    cfg = wl.AttnCfg(1, 2, 512, D, 128, 4, 0, 7)
    q, k, v = wl.attn_inputs(cfg, "cpu", dtype)
    nqb = 4
    bm = torch.ones(nqb, nqb, dtype=torch.bool)
    crow, col = wl.mask_to_bsr(bm)
    rp = torch.cat([crow, crow[1:] + crow[-1]])
    ci = torch.cat([col, col])
    O = _run(q, k, v, rp, ci, 0.1, causal=False)
    _check(O, q, k, v, rp, ci, 0.1, False, nqb, range(2))


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float16, 64)])
def test_bsattn_empty_rows_zero_and_bh_range(no_device_error, dtype, D):
    cfg = wl.AttnCfg(1, 3, 512, D, 128, 4, 8, 9)
    q, k, v = wl.attn_inputs(cfg, "cpu", dtype)
    bm = torch.tensor([[1, 0, 0, 0], [0, 0, 0, 0], [1, 1, 1, 0], [0, 1, 0, 1]], dtype=torch.bool)
    crow, col = wl.mask_to_bsr(bm)
    rp = torch.cat([crow, crow[1:] + crow[-1], crow[1:] + 2 * crow[-1]])
    ci = torch.cat([col, col, col])
    dev = torch.device("cuda", 0)
    O = torch.full(q.shape, 3.0, dtype=dtype, device=dev)
    _fwd(q)(q.to(dev), k.to(dev), v.to(dev), O, rp.to(torch.int32).to(dev), ci.to(torch.int32).to(dev), 0.088, True, 1,
            2)
    torch.cuda.synchronize()
    O = O.cpu()
    assert torch.all(O[0, 0] == 3.0) and torch.all(O[0, 2] == 3.0)  # pairs outside [1,2) untouched
    assert torch.count_nonzero(O[0, 1, 128:256]) == 0  # empty mask row -> zeros
    _check(O, q, k, v, rp, ci, 0.088, True, 4, [1])


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float16, 64)])
def test_bsattn_deterministic(no_device_error, dtype, D):
    cfg = wl.AttnCfg(1, 2, 1024, D, 128, 4, 8, 4)
    q, k, v = wl.attn_inputs(cfg, "cpu", dtype)
    rp, ci = wl.attn_mask_bsr(cfg)
    a = _run(q, k, v, rp, ci, 0.0883)
    b = _run(q, k, v, rp, ci, 0.0883)
    assert torch.equal(a, b)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [32, 256])
def test_bsattn_rejects_head_dim(cuda_dev, dtype, D):
    q = torch.zeros(1, 1, 128, D, dtype=dtype, device=cuda_dev)
    rp = torch.tensor([0, 1], dtype=torch.int32, device=cuda_dev)
    ci = torch.tensor([0], dtype=torch.int32, device=cuda_dev)
    with pytest.raises(_capi.BskError) as e:
        _fwd(q)(q, q, q, torch.empty_like(q), rp, ci, 0.125)
    assert e.value.code == _capi.BSK_ERR_UNSUPPORTED


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float16, 64)])
def test_bsattn_output_16_byte_aligned_only(no_device_error, dtype, D):
    """O that starts 16 bytes past a 32-byte boundary (the ABI asks for 16-byte alignment only): the output warps
    fall back from 32-byte to 16-byte stores and the result is the same as into an aligned O."""
    cfg = wl.AttnCfg(1, 2, 1024, D, 128, 4, 8, 6)
    q, k, v = wl.attn_inputs(cfg, "cpu", dtype)
    rp, ci = wl.attn_mask_bsr(cfg)
    dev = torch.device("cuda", 0)
    big = torch.full((q.numel() + 64,), float("nan"), dtype=dtype, device=dev)
    off = (32 - big.data_ptr() % 32) // 2 + 8  # elements: 16 bytes past a 32-byte boundary
    O = big[off:off + q.numel()].view(q.shape)
    assert O.data_ptr() % 32 == 16
    _fwd(q)(q.to(dev), k.to(dev), v.to(dev), O, rp.to(torch.int32).to(dev), ci.to(torch.int32).to(dev), 0.0883, True,
            0, 2)
    torch.cuda.synchronize()
    assert torch.equal(O.cpu(), _run(q, k, v, rp, ci, 0.0883))
    assert torch.isnan(big[:off]).all() and torch.isnan(big[off + q.numel():]).all()  # nothing written outside O
