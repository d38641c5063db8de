"""blackwellsparsek._C -- the reference's torch-extension module name (setup.py:18) bound to this build's
extension ``periodicdent42_b200._C`` (same ``sparse_mm_bsr`` signature, python/bsk_bindings.cpp:141-158, plus the
operators the reference never exposed). The module object itself is the extension: this file replaces its own
entry in ``sys.modules`` so that ``blackwellsparsek._C is periodicdent42_b200._C``."""
import sys

from periodicdent42_b200 import _C as _extension

sys.modules[__name__] = _extension
