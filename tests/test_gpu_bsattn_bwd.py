"""Block-sparse attention backward (dQ, dK, dV) through the C ABI and autograd, against the oracle: torch
autograd of the dense-masked attention in fp64 on the CPU (the reference's torch path -- attention with the
block mask expanded -- differentiated). Also the forward's log-sum-exp, determinism, and the mask column lists.

Tolerance: the kernels round P and dS to the input type (bf16 / fp16) before the tensor-core products, as
FlashAttention-style backwards do; the bar is err <= 3 x (error of torch's own backward in the same low
precision) + 2e-3, normwise relative against fp64, per gradient."""
import math

import pytest
import torch

import periodicdent42_b200 as bsk
from oracle import reference_path as ref
from periodicdent42_b200 import _capi
from periodicdent42_b200 import workloads as wl

pytestmark = pytest.mark.gpu


def _dense_mask(rp, ci, B, H, nqb, causal):
    m = torch.zeros(B, H, nqb * 128, nqb * 128, dtype=torch.bool)
    for p in range(B * H):
        b, h = divmod(p, H)
        bm = wl.block_mask_dense(rp[p * nqb:(p + 1) * nqb + 1], ci[rp[p * nqb]:rp[(p + 1) * nqb]], nqb, nqb)
        m[b, h] = wl.dense_mask_from_blocks(bm, 128, causal)
    return m


def _attn(q, k, v, mask, scale):
    """softmax(scale q k^T on the mask) v with rows that attend nothing set to zero (as the kernel defines them),
    written so that such rows carry no NaN into the gradients."""
    s = (q @ k.transpose(-1, -2)) * scale
    rows = mask.any(dim=-1, keepdim=True)
    s = torch.where(rows, s.masked_fill(~mask, -math.inf), torch.zeros_like(s))
    p = torch.softmax(s, dim=-1) * rows
    return p @ v


def _grads(q, k, v, dO, mask, scale, dtype):
    qq, kk, vv = (t.detach().to(dtype).requires_grad_(True) for t in (q, k, v))
    out = _attn(qq, kk, vv, mask, scale)
    out.backward(dO.to(dtype))
    return out.detach(), qq.grad, kk.grad, vv.grad


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float16, 64), (torch.float16, 128),
                                     (torch.bfloat16, 64)])
@pytest.mark.parametrize("B,H,S,causal", [(1, 2, 512, True), (1, 1, 1024, True), (2, 1, 384, False)])
def test_bwd_matches_fp64_autograd(no_device_error, cuda_dev, dtype, D, B, H, S, causal):
    cfg = wl.AttnCfg(B, H, S, D, 128, 2, 2, 11 + S)
    q, k, v = wl.attn_inputs(cfg, "cpu", dtype)
    dO = torch.randn(B, H, S, D, generator=torch.Generator().manual_seed(5)).to(dtype)
    nqb = S // 128
    if causal:
        rp, ci = wl.attn_mask_bsr(cfg)
    else:  # a non-causal random block pattern with one empty block-row
        g = torch.Generator().manual_seed(S)
        bm = torch.rand(nqb, nqb, generator=g) < 0.6
        bm[1] = False
        crow, col = wl.mask_to_bsr(bm)
        rp = torch.cat([crow] + [crow[1:] + crow[-1] * i for i in range(1, B * H)])
        ci = col.repeat(B * H)
    scale = 1.0 / math.sqrt(D)
    mask = _dense_mask(rp, ci, B, H, nqb, causal)
    _, gq64, gk64, gv64 = _grads(q, k, v, dO, mask, scale, torch.float64)
    _, gq_lp, gk_lp, gv_lp = _grads(q, k, v, dO, mask, scale, dtype)  # torch's own path in the input type

    dev = cuda_dev
    Q, K, V = (t.to(dev) for t in (q, k, v))
    rpd, cid = rp.to(torch.int32).to(dev), ci.to(torch.int32).to(dev)
    O = torch.empty_like(Q)
    lse = torch.empty(B * H * S, dtype=torch.float32, device=dev)
    _capi.bsattn_fwd_ex(Q, K, V, O, lse, rpd, cid, scale, causal)
    col_ptr, row_idx = _capi.bsattn_mask_transpose(rpd, cid, B * H, nqb)
    dQ, dK, dV = torch.empty_like(Q), torch.empty_like(K), torch.empty_like(V)
    _capi.bsattn_bwd(dO.to(dev), Q, K, V, O, lse, dQ, dK, dV, rpd, cid, col_ptr, row_idx, scale, causal)
    torch.cuda.synchronize()
    for name, got, want, lp in (("dQ", dQ, gq64, gq_lp), ("dK", dK, gk64, gk_lp), ("dV", dV, gv64, gv_lp)):
        err = ref.normwise_rel_err(got.cpu(), want)
        base = ref.normwise_rel_err(lp, want)
        assert torch.isfinite(got.float()).all(), name
        assert err <= 3 * base + 2e-3, (name, err, base)


def test_forward_lse(no_device_error, cuda_dev):
    cfg = wl.AttnCfg(1, 2, 512, 128, 128, 2, 2, 3)
    q, k, v = wl.attn_inputs(cfg, "cpu")
    rp, ci = wl.attn_mask_bsr(cfg)
    scale = 1.0 / math.sqrt(128)
    mask = _dense_mask(rp, ci, 1, 2, 4, True)
    s = (q.double() @ k.double().transpose(-1, -2)) * scale
    want = torch.logsumexp(s.masked_fill(~mask, -math.inf), dim=-1).reshape(-1)
    Q, K, V = (t.to(cuda_dev) for t in (q, k, v))
    O = torch.empty_like(Q)
    lse = torch.empty(2 * 512, dtype=torch.float32, device=cuda_dev)
    _capi.bsattn_fwd_ex(Q, K, V, O, lse, rp.to(torch.int32).to(cuda_dev), ci.to(torch.int32).to(cuda_dev), scale, True)
    torch.cuda.synchronize()
    assert torch.allclose(lse.cpu().double(), want, atol=2e-3, rtol=0)


def test_mask_transpose(cuda_dev):
    cfg = wl.AttnCfg(2, 3, 1024, 128, 128, 3, 2, 8)
    rp, ci = wl.attn_mask_bsr(cfg)
    nqb = 8
    col_ptr, row_idx = _capi.bsattn_mask_transpose(rp.to(torch.int32).to(cuda_dev), ci.to(torch.int32).to(cuda_dev),
                                                   6, nqb)
    col_ptr, row_idx = col_ptr.cpu().tolist(), row_idx.cpu().tolist()
    rpl, cil = rp.tolist(), ci.tolist()
    for p in range(6):
        for j in range(nqb):
            want = [i for i in range(nqb) if j in cil[rpl[p * nqb + i]:rpl[p * nqb + i + 1]]]
            assert row_idx[col_ptr[p * nqb + j]:col_ptr[p * nqb + j + 1]] == want
    assert col_ptr[-1] == rpl[-1]


def test_autograd_and_determinism(no_device_error, cuda_dev):
    cfg = wl.AttnCfg(1, 2, 768, 128, 128, 2, 2, 6)
    q, k, v = wl.attn_inputs(cfg, "cpu")
    dO = torch.randn(1, 2, 768, 128, generator=torch.Generator().manual_seed(1)).bfloat16().to(cuda_dev)
    grads = []
    for _ in range(2):
        Q, K, V = (t.to(cuda_dev).requires_grad_(True) for t in (q, k, v))
        O = bsk.attention_forward(Q, K, V, causal=True)
        O.backward(dO)
        grads.append([t.grad.clone() for t in (Q, K, V)])
    for a, b in zip(*grads):
        assert torch.equal(a, b)
    mask = torch.ones(768, 768, dtype=torch.bool).tril()
    _, gq64, gk64, gv64 = _grads(q, k, v, dO.cpu(), mask, 1.0 / math.sqrt(128), torch.float64)
    for got, want in zip(grads[0], (gq64, gk64, gv64)):
        assert ref.normwise_rel_err(got.cpu(), want) <= 2e-2


@pytest.mark.parametrize("pairs,nqb,density", [(5, 40, 0.3), (2, 600, 0.02)])
def test_mask_transpose_random_masks(cuda_dev, pairs, nqb, density):
    """Random block masks through both transpose paths (shared-memory bit map for nqb <= 512, the serial kernel
    above): ascending query blocks per key block-column, col_ptr in row_ptr's numbering."""
    g = torch.Generator().manual_seed(nqb)
    rps, cis, base = [0], [], 0
    for p in range(pairs):
        m = torch.rand(nqb, nqb, generator=g) < density
        crow, col = wl.mask_to_bsr(m)
        rps.extend((crow[1:] + base).tolist())
        cis.extend(col.tolist())
        base += int(crow[-1])
    rp, ci = torch.tensor(rps, dtype=torch.int32), torch.tensor(cis, dtype=torch.int32)
    col_ptr, row_idx = _capi.bsattn_mask_transpose(rp.to(cuda_dev), ci.to(cuda_dev), pairs, nqb)
    col_ptr, row_idx = col_ptr.cpu().tolist(), row_idx.cpu().tolist()
    for p in range(pairs):
        cols = [[] for _ in range(nqb)]
        for i in range(nqb):
            for kb in cis[rps[p * nqb + i]:rps[p * nqb + i + 1]]:
                cols[kb].append(i)
        for j in range(nqb):
            assert row_idx[col_ptr[p * nqb + j]:col_ptr[p * nqb + j + 1]] == cols[j], (p, j)
    assert col_ptr[-1] == rps[-1]
