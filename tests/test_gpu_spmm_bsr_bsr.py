"""BSR x BSR SpMM (sparse B) through the C ABI, the reference-signature launcher and the public sparse_mm, against
the fp64 recompute of the dense operands (the oracle: A.to_dense() @ B.to_dense()).
Tolerance: normwise relative error <= 1e-3 against fp64 (the fp16 bar of the BSR path). Every case runs with B's
block map staged in shared memory and with the binary searches in global memory (BSK_BSRBSR_TABLE)."""
import ctypes

import pytest
import torch

import periodicdent42_b200 as bsk
from oracle import reference_path as ref
from periodicdent42_b200 import _capi
from periodicdent42_b200 import workloads as wl

pytestmark = pytest.mark.gpu
TOL = 1e-3


@pytest.fixture(autouse=True, params=["table", "search"])
def b_lookup(request, monkeypatch):
    monkeypatch.setenv("BSK_BSRBSR_TABLE", "1" if request.param == "table" else "0")
    return request.param


def _bsr(Mb, Kb, per_row, seed, dev):
    g = torch.Generator().manual_seed(seed)
    crow, col = wl.bsr_pattern(Mb, Kb, per_row, g)
    vals = torch.randn(int(crow[-1]), 128, 128, generator=g).half()
    return crow.to(torch.int32).to(dev), col.to(torch.int32).to(dev), vals.to(dev)


def _dense(crow, col, vals, M, K):
    return torch.sparse_bsr_tensor(crow.long().cpu(), col.long().cpu(), vals.cpu().float(), size=(M, K)).to_dense()


@pytest.mark.parametrize("Mb,Kb,Nb,a_per,b_per", [(4, 6, 4, 2, 1), (8, 8, 8, 3, 2), (6, 4, 3, 4, 1), (16, 16, 12, 5, 3),
                                                  (3, 5, 2, 5, 2), (2, 300, 2, 4, 1)])
def test_bsr_bsr_matches_dense_oracle(no_device_error, cuda_dev, Mb, Kb, Nb, a_per, b_per):
    M, K, N = Mb * 128, Kb * 128, Nb * 128
    arp, aci, av = _bsr(Mb, Kb, a_per, Mb * 7 + Kb, cuda_dev)
    brp, bci, bv = _bsr(Kb, Nb, b_per, Nb * 13 + Kb, cuda_dev)
    C = torch.full((M, N), float("nan"), device=cuda_dev)
    _capi.spmm_bsr_bsr_f16f32(arp, aci, av, brp, bci, bv, C, M, N, K)
    torch.cuda.synchronize()
    want = _dense(arp, aci, av, M, K).double() @ _dense(brp, bci, bv, K, N).double()
    assert torch.isfinite(C).all()
    err = ref.normwise_rel_err(C.cpu(), want)
    assert err <= TOL, err


def test_bsr_bsr_empty_rows_tiles_and_row_range(no_device_error, cuda_dev):
    """A block-row without blocks, an output tile with no contributing B blocks, a block-row range."""
    M, K, N = 512, 512, 768
    arp = torch.tensor([0, 2, 2, 3, 5], dtype=torch.int32, device=cuda_dev)  # block-row 1 empty
    aci = torch.tensor([0, 2, 1, 1, 3], dtype=torch.int32, device=cuda_dev)
    av = torch.randn(5, 128, 128, device=cuda_dev).half()
    # B: block-rows 0..3; only block columns 0, 1 and 5 used -> output tile of columns 256..511 is all zero
    brp = torch.tensor([0, 1, 2, 3, 4], dtype=torch.int32, device=cuda_dev)
    bci = torch.tensor([0, 5, 1, 0], dtype=torch.int32, device=cuda_dev)
    bv = torch.randn(4, 128, 128, device=cuda_dev).half()
    want = _dense(arp, aci, av, M, K).double() @ _dense(brp, bci, bv, K, N).double()
    C = torch.full((M, N), 5.0, device=cuda_dev)
    _capi.spmm_bsr_bsr_f16f32(arp, aci, av, brp, bci, bv, C, M, N, K, 1, 3)
    torch.cuda.synchronize()
    Cc = C.cpu()
    assert torch.all(Cc[:128] == 5.0) and torch.all(Cc[384:] == 5.0)  # rows outside [1, 3) untouched
    assert torch.count_nonzero(Cc[128:256]) == 0                        # empty block-row -> zeros
    assert torch.count_nonzero(Cc[128:384, 256:512]) == 0               # tile without B blocks -> zeros
    assert ref.normwise_rel_err(Cc[256:384], want[256:384]) <= TOL


def test_reference_launcher_routes_sparse_b(cuda_dev):
    Mb, Kb, Nb = 4, 4, 4
    M, K, N = Mb * 128, Kb * 128, Nb * 128
    arp, aci, av = _bsr(Mb, Kb, 2, 3, cuda_dev)
    brp, bci, bv = _bsr(Kb, Nb, 2, 4, cuda_dev)
    C = torch.zeros(M, N, device=cuda_dev)
    lib = _capi.lib()
    lib.launch_bsr_spmm_async(arp.data_ptr(), aci.data_ptr(), av.data_ptr(), Mb, Kb, aci.numel(), brp.data_ptr(),
                              bci.data_ptr(), bv.data_ptr(), Kb, Nb, bci.numel(), C.data_ptr(), M, N, K, N, 256, 128,
                              32, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert _capi.last_error() == ""
    want = _dense(arp, aci, av, M, K).double() @ _dense(brp, bci, bv, K, N).double()
    assert ref.normwise_rel_err(C.cpu(), want) <= TOL
    assert _capi.device_error() == 0


def test_public_sparse_mm_with_sparse_b(no_device_error, cuda_dev):
    Mb, Kb, Nb = 6, 8, 4
    M, K, N = Mb * 128, Kb * 128, Nb * 128
    arp, aci, av = _bsr(Mb, Kb, 3, 11, cuda_dev)
    brp, bci, bv = _bsr(Kb, Nb, 2, 12, cuda_dev)
    A = torch.sparse_bsr_tensor(arp.long(), aci.long(), av, size=(M, K))
    B = torch.sparse_bsr_tensor(brp.long(), bci.long(), bv, size=(K, N))
    C = bsk.sparse_mm(A, B)
    want = _dense(arp, aci, av, M, K).double() @ _dense(brp, bci, bv, K, N).double()
    assert ref.normwise_rel_err(C.cpu(), want) <= TOL
    # the same B as CSR (re-blocked on the device) gives the same product
    C2 = bsk.sparse_mm(A, B.to_dense().to_sparse_csr())
    assert torch.equal(C, C2)


def test_bsr_bsr_deterministic(no_device_error, cuda_dev):
    arp, aci, av = _bsr(8, 8, 3, 21, cuda_dev)
    brp, bci, bv = _bsr(8, 8, 3, 22, cuda_dev)
    outs = []
    for _ in range(2):
        C = torch.empty(1024, 1024, device=cuda_dev)
        _capi.spmm_bsr_bsr_f16f32(arp, aci, av, brp, bci, bv, C, 1024, 1024, 1024)
        outs.append(C.cpu())
    assert torch.equal(outs[0], outs[1])
