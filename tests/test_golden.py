"""Pins the oracle and the host-side index handling against fixtures produced by the reference's own code
(tests/golden/make_golden.py): its convert_to_bsr, its torch path and its compiled cpu_bsr."""
import math
import os

import numpy as np
import pytest
import torch

from oracle import cbsr
from oracle import build as obuild
from oracle import reference_path as ref
from periodicdent42_b200 import workloads as wl

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))


def test_bsr_pattern_matches_reference_convert_to_bsr():
    crow, col = wl.bsr_pattern(4, 6, 2, torch.Generator().manual_seed(1234))
    assert np.array_equal(crow.numpy(), G["bsr_ref_crow"])
    assert np.array_equal(col.numpy(), G["bsr_ref_col"])


def test_bsr_oracle_matches_reference_sparse_mm():
    crow = torch.from_numpy(G["bsr_ref_crow"])
    col = torch.from_numpy(G["bsr_ref_col"])
    vals = torch.from_numpy(G["bsr_ref_vals"])
    B = torch.from_numpy(G["bsr_B"])
    C64 = ref.bsr_fp64(crow, col, vals, B, 512, 768)
    assert ref.normwise_rel_err(torch.from_numpy(G["bsr_C_sparse_mm"]), C64) < 1e-6
    # the reference torch path, re-run here, reproduces its own fixture
    C = ref.bsr_ref(crow, col, vals, B, 512, 768)
    assert ref.normwise_rel_err(C, torch.from_numpy(G["bsr_C_sparse_mm"])) < 1e-6


def test_c_restatement_bit_identical_to_reference_cpu_bsr_fixture():
    obuild.build_oracle()
    C = cbsr.oracle_cpu_bsr(G["cpubsr_A"], G["cpubsr_rp"], G["cpubsr_ci"], G["cpubsr_B"], 256, 192, 320, 128, 128, 64)
    assert np.array_equal(C.view(np.uint32), G["cpubsr_C"].view(np.uint32))


def test_numpy_restatement_matches_reference_cpu_bsr_fixture():
    C = ref.cpu_bsr_numpy(G["cpubsr_A"], G["cpubsr_rp"], G["cpubsr_ci"], G["cpubsr_B"], 256, 192, 320, 128, 128, 64)
    np.testing.assert_allclose(C, G["cpubsr_C"], rtol=1e-4, atol=1e-4)


@pytest.mark.skipif(not cbsr.ref_available(), reason="reference cpu_bsr not built here (oracle/build_ref.sh)")
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_c_restatement_bit_identical_to_reference_cpu_bsr_random(seed):
    obuild.build_oracle()
    rng = np.random.default_rng(seed)
    M, N, K = 128 * 3 - 40 * seed, 100 + 60 * seed, 64 * 5 - 24 * seed  # ragged edges included
    Mb, Kb = (M + 127) // 128, (K + 63) // 64
    rp, ci = [0], []
    for i in range(Mb):
        ci += sorted(rng.choice(Kb, size=rng.integers(0, Kb + 1), replace=False).tolist())
        rp.append(len(ci))
    A = rng.standard_normal((max(len(ci), 1), 128, 64)).astype(np.float16)
    B = rng.standard_normal((K, N)).astype(np.float16)
    c1 = cbsr.oracle_cpu_bsr(A, np.array(rp), np.array(ci), B, M, N, K, 128, 128, 64)
    c2 = cbsr.ref_cpu_bsr(A, np.array(rp), np.array(ci), B, M, N, K)
    assert np.array_equal(c1.view(np.uint32), c2.view(np.uint32))


def test_dense_reference_path_fixture():
    A = torch.from_numpy(G["dense_A"])
    Bt = torch.from_numpy(G["dense_Bt"])
    C = ref.dense_ref(A, Bt)
    np.testing.assert_allclose(C.numpy(), G["dense_C"], rtol=1e-5, atol=1e-5)
    assert ref.normwise_rel_err(torch.from_numpy(G["dense_C"]), ref.dense_fp64(A, Bt)) < 1e-6


def test_fp8_reference_path_fixture():
    Aq = torch.from_numpy(G["fp8_Aq_bits"]).view(torch.float8_e4m3fn)
    Bqt = torch.from_numpy(G["fp8_Bqt_bits"]).view(torch.float8_e4m3fn)
    sa, sb = torch.from_numpy(G["fp8_sa"]), torch.from_numpy(G["fp8_sb"])
    D_fix = torch.from_numpy(G["fp8_D_bits"]).view(torch.bfloat16)
    D = ref.fp8_ref(Aq, Bqt, sa, sb)
    assert ref.normwise_rel_err(D, D_fix) < 1e-3
    assert ref.normwise_rel_err(D_fix, ref.fp8_fp64(Aq, Bqt, sa, sb)) < 5e-3


def test_fp8_quantisation_recipe():
    g = torch.Generator().manual_seed(8)
    Aq, sa = wl.quantize_e4m3(torch.randn(64, 128, generator=g))
    assert np.array_equal(Aq.view(torch.uint8).numpy(), G["fp8_Aq_bits"])
    assert np.array_equal(sa.numpy(), G["fp8_sa"])


def test_attention_oracle_matches_reference_sdpa_fixture():
    q = torch.from_numpy(G["attn_q_bits"]).view(torch.bfloat16)
    k = torch.from_numpy(G["attn_k_bits"]).view(torch.bfloat16)
    v = torch.from_numpy(G["attn_v_bits"]).view(torch.bfloat16)
    rp = torch.from_numpy(G["attn_rp"])
    ci = torch.from_numpy(G["attn_ci"])
    cfg = wl.AttnCfg(1, 1, 384, 128, 128, 2, 1, 4)
    rp2, ci2 = wl.attn_mask_bsr(cfg)
    assert torch.equal(rp, rp2) and torch.equal(ci, ci2)
    o64 = ref.attn_blocksparse_fp64(q[0, 0], k[0, 0], v[0, 0], rp, ci, 1 / math.sqrt(128), True)
    assert ref.normwise_rel_err(torch.from_numpy(G["attn_O_sdpa_fp32"])[0, 0], o64) < 1e-5


def test_attention_mask_index_matches_reference_convert_to_bsr():
    cfg = wl.AttnCfg(1, 2, 2048, 128, 128, 4, 8, 4)
    rp, ci = wl.attn_mask_bsr(cfg)
    crows, cols = [], []
    for p in range(2):
        seg = rp[p * 16:(p + 1) * 16 + 1]
        crows.append((seg - seg[0]).numpy())
        cols.append(ci[seg[0]:seg[-1]].numpy())
    assert np.array_equal(np.stack(crows), G["mask_ref_crow"])
    assert np.array_equal(np.concatenate(cols), G["mask_ref_col"])


def test_bsr_workload_pattern_regression():
    crow, col = wl.bsr_pattern(64, 64, 16, torch.Generator().manual_seed(3))
    assert np.array_equal(crow.numpy(), G["bsr_cfg_crow"])
    assert np.array_equal(col.numpy(), G["bsr_cfg_col"])
