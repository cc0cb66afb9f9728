"""The chunk kernels' product engine on its own (gdn2_selftest_engine): C = A B for 128 x 128 fp32
matrices through one K-loop of the engine every operator kernel uses (the CTA's warps stage each
K-slice into 128-byte-swizzled shared-memory tiles, one thread issues its tensor-core MMAs), with
A and B staged as K-major own-row, K-major coalesced or MN-major coalesced operands, in every
precision mode, against a float64 matmul.  Tolerances: 3-pass modes 1e-5 relative L2 (hi/lo splits carry
about 16 (bf16) or 22 (tf32) bits), 1-pass bf16 1e-2, 1-pass tf32 2e-3."""
import ctypes

import pytest
import torch

from atomic_gdn2 import _lib

pytestmark = pytest.mark.gpu
TOL = {0: 1e-5, 1: 1e-5, 2: 1e-2, 3: 2e-3}


@pytest.mark.parametrize("prec", [0, 1, 2, 3])
def test_engine_product_every_operand_kind(prec):
    lib = _lib.load()
    gen = torch.Generator(device="cuda").manual_seed(prec)
    A = torch.randn(128, 128, device="cuda", generator=gen)
    B = torch.randn(128, 128, device="cuda", generator=gen)
    At, Bt = A.t().contiguous(), B.t().contiguous()
    want = A.double() @ B.double()
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    for ak in range(3):
        for bk in range(3):
            C = torch.full((128, 128), float("nan"), device="cuda")
            rc = lib.gdn2_selftest_engine(p(A), p(At), p(B), p(Bt), p(C), prec, ak, bk, p(st), stream)
            assert rc == _lib.OK, (ak, bk, _lib.status_string(rc))
            torch.cuda.synchronize()
            assert int(st.item()) == 0, (ak, bk)
            err = float((C.double() - want).norm() / want.norm())
            assert err < TOL[prec], (prec, ak, bk, err)
