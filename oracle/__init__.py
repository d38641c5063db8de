"""Oracle for the BlackwellSparseK operator family -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline leg and ``--impl reference``) may
import, call, link or execute anything in this package, and only as the checker or as the timed CPU
baseline -- never as part of the product path, which has no CPU fallback.

Contents:
  reference_path.py  the reference's own torch CPU path for each operator (torch.matmul on fp32-upcast
                     operands, torch._scaled_mm, torch.sparse.mm on fp32 BSR, scaled_dot_product_attention
                     with a dense boolean mask), fp64 recomputes, and a block-sparse fp64 attention
                     restatement for shapes where a dense mask is too large.
  bsr_oracle.c       plain-C restatement of the reference's CPU BSR checker cpu_bsr
                     (BlackwellSparseK/src/bsr_reference.cu:72-93), same loop order and fp32 accumulation.
  build_ref.sh       compiles the reference's own cpu_bsr from its source into oracle/_ref/ (this
                     container only) so the restatement can be pinned bit-for-bit against it.

Pinning: the reference commits no golden vectors (its tests recompute with torch on the same seeded
inputs). The restatements here are pinned against (1) tests/golden/ fixtures produced by the reference's
torch path and by the reference's own Python ``convert_to_bsr`` (script: tests/golden/make_golden.py),
and (2) the reference's compiled cpu_bsr in oracle/_ref/.
"""
