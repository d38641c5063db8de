"""Generates tests/golden/golden.npz: small known-answer cases produced by the REFERENCE's own code.

Run with REF_ROOT naming the reference checkout (required):
    REF_ROOT=<checkout> python tests/golden/make_golden.py
What each case comes from:
  * BSR index handling: the reference's ``convert_to_bsr`` (BlackwellSparseK/python/utils.py:10-57),
    imported from the reference checkout, applied to dense matrices whose block pattern our builders
    also produce -> crow/col/values the kernels' index handling must reproduce exactly.
  * BSR values: the reference's torch path torch.sparse.mm(A_bsr.float(), B.float()) (ops.py:117-120)
    and the reference's own compiled cpu_bsr (oracle/_ref, BlackwellSparseK/src/bsr_reference.cu:72-93).
  * dense GEMM: torch.matmul on fp32-upcast operands (the reference's dense baseline).
  * FP8 GEMM: torch._scaled_mm with per-tensor scales.
  * attention: F.scaled_dot_product_attention with the dense boolean mask expanded from a block mask.
The fixtures are then read by tests/test_golden.py without the reference present.
"""
from __future__ import annotations

import importlib.util
import math
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from periodicdent42_b200 import workloads as wl  # noqa: E402


def load_reference_utils():
    ref_root = os.environ.get("REF_ROOT")
    if not ref_root:
        raise SystemExit("set REF_ROOT to the reference checkout")
    path = os.path.join(ref_root, "BlackwellSparseK", "python", "utils.py")
    spec = importlib.util.spec_from_file_location("bsk_reference_utils", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main():
    ref_utils = load_reference_utils()
    out = {}

    # --- BSR via the reference's convert_to_bsr: 128x128 blocks, 4x6 block grid, 2 blocks per row
    g = torch.Generator().manual_seed(1234)
    crow, col = wl.bsr_pattern(4, 6, 2, g)
    vals = torch.randn(crow[-1].item(), 128, 128, generator=g).half()
    dense = torch.zeros(512, 768, dtype=torch.float16)
    for r in range(4):
        for j in range(crow[r].item(), crow[r + 1].item()):
            c = col[j].item()
            dense[r * 128:(r + 1) * 128, c * 128:(c + 1) * 128] = vals[j]
    A_bsr = ref_utils.convert_to_bsr(dense, block_size=128, sparsity_threshold=0.0)
    B = torch.randn(768, 128, generator=g).half()
    out["bsr_ref_crow"] = A_bsr.crow_indices().numpy()
    out["bsr_ref_col"] = A_bsr.col_indices().numpy()
    out["bsr_ref_vals"] = A_bsr.values().numpy()
    out["bsr_B"] = B.numpy()
    A32 = torch.sparse_bsr_tensor(A_bsr.crow_indices(), A_bsr.col_indices(), A_bsr.values().float(), size=(512, 768))
    out["bsr_C_sparse_mm"] = torch.sparse.mm(A32, B.float()).numpy()

    # --- the reference's own compiled cpu_bsr on a 128x64-block case (its fixed BM=128, BK=64)
    try:
        from oracle import build as obuild
        from oracle import cbsr

        obuild.build_ref()
        if cbsr.ref_available():
            rng = np.random.default_rng(42)
            M, N, K = 256, 192, 320
            rp, ci = [0], []
            for i in range(2):
                ci += sorted(rng.choice(5, size=2 + i, replace=False).tolist())
                rp.append(len(ci))
            Ab = rng.standard_normal((len(ci), 128, 64)).astype(np.float16)
            Bb = rng.standard_normal((K, N)).astype(np.float16)
            out["cpubsr_A"] = Ab
            out["cpubsr_rp"] = np.array(rp, np.int32)
            out["cpubsr_ci"] = np.array(ci, np.int32)
            out["cpubsr_B"] = Bb
            out["cpubsr_C"] = cbsr.ref_cpu_bsr(Ab, np.array(rp), np.array(ci), Bb, M, N, K)
    except Exception as e:  # noqa: BLE001
        print("cpu_bsr reference unavailable:", e)

    # --- dense GEMM: ragged shape, uniform[-1,1)
    g = torch.Generator().manual_seed(7)
    A = (torch.rand(200, 72, generator=g) * 2 - 1).half()
    Bt = (torch.rand(136, 72, generator=g) * 2 - 1).half()
    out["dense_A"] = A.numpy()
    out["dense_Bt"] = Bt.numpy()
    out["dense_C"] = torch.matmul(A.float(), Bt.float().t()).numpy()

    # --- FP8 GEMM
    g = torch.Generator().manual_seed(8)
    Aq, sa = wl.quantize_e4m3(torch.randn(64, 128, generator=g))
    Bqt, sb = wl.quantize_e4m3(torch.randn(96, 128, generator=g))
    D = torch._scaled_mm(Aq, Bqt.t(), scale_a=sa.reshape(()), scale_b=sb.reshape(()), out_dtype=torch.bfloat16)
    out["fp8_Aq_bits"] = Aq.view(torch.uint8).numpy()
    out["fp8_Bqt_bits"] = Bqt.view(torch.uint8).numpy()
    out["fp8_sa"] = sa.numpy()
    out["fp8_sb"] = sb.numpy()
    out["fp8_D_bits"] = D.view(torch.int16).numpy()

    # --- attention: one (b,h), S = 384, sliding window 2 + 1 random block (mask builder of the workload)
    cfg = wl.AttnCfg(1, 1, 384, 128, 128, 2, 1, 4)
    q, k, v = wl.attn_inputs(cfg, "cpu")
    rp, ci = wl.attn_mask_bsr(cfg)
    bm = wl.block_mask_dense(rp, ci, 3, 3)
    dm = wl.dense_mask_from_blocks(bm, 128, True)
    scale = 1.0 / math.sqrt(128)
    o = F.scaled_dot_product_attention(q.float(), k.float(), v.float(), attn_mask=dm, scale=scale)
    out["attn_q_bits"] = q.view(torch.int16).numpy()
    out["attn_k_bits"] = k.view(torch.int16).numpy()
    out["attn_v_bits"] = v.view(torch.int16).numpy()
    out["attn_rp"] = rp.numpy()
    out["attn_ci"] = ci.numpy()
    out["attn_O_sdpa_fp32"] = o.numpy()

    # --- index handling of the sliding-window workload at S=2048 (16 block-rows) for 2 pairs:
    # the reference's convert_to_bsr of the expanded mask == our direct BSR construction
    cfg = wl.AttnCfg(1, 2, 2048, 128, 128, 4, 8, 4)
    rp, ci = wl.attn_mask_bsr(cfg)
    crows, cols = [], []
    for p in range(2):
        bm = wl.block_mask_dense(rp[p * 16:(p + 1) * 16 + 1], ci[rp[p * 16]:rp[(p + 1) * 16]], 16, 16)
        expanded = bm.repeat_interleave(128, 0).repeat_interleave(128, 1).to(torch.float16)
        b = ref_utils.convert_to_bsr(expanded, block_size=128, sparsity_threshold=0.0)
        crows.append(b.crow_indices().numpy())
        cols.append(b.col_indices().numpy())
    out["mask_ref_crow"] = np.stack(crows)
    out["mask_ref_col"] = np.concatenate(cols)

    # --- the full BSR workload's index pattern (64 x 64 block grid, 16 per row, seed 3)
    crow, col = wl.bsr_pattern(64, 64, 16, torch.Generator().manual_seed(3))
    out["bsr_cfg_crow"] = crow.numpy()
    out["bsr_cfg_col"] = col.numpy()

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **out)
    print("wrote", os.path.join(HERE, "golden.npz"), sorted(out))


if __name__ == "__main__":
    main()
