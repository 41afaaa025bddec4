"""The allocation-free dense GEMM entry point.

Some callers of this library may not allocate device memory themselves (an
application whose allocator owns the whole GPU, a plugin host that only
hands out its own buffers).  dsv4_b200_mxfp4_int8_dense_gemm_noalloc takes
its split-K workspace from a fixed array inside the library instead.  This
test calls it through the C ABI twice in a row and checks each result
bit-exactly against the regular entry point (which is given a workspace the
test allocates), plus its size rejection.  It lives in its own file so that
pytest collects it last.
"""

import numpy as np
import pytest
import torch

import gen_inputs as G
from oracle import mxfp4_int8_oracle as O

pytestmark = pytest.mark.gpu


def _case(m, n, k, seed):
    import dsv4_b200 as D
    w, s = G.make_random_packed_mxfp4(1, n, k, seed, exp_range=(-8, -4))
    b, sh, cs = D.remap_mxfp4_weight_for_int8(w.cuda(), s.cuda())
    x = G.randn_bf16((m, k), seed + 1).cuda()
    q, qs = D.quantize_per_token_int8(x)
    return q, qs, b[0], sh[0], cs[0]


@pytest.mark.parametrize("m,n,k", [(1, 4096, 1024), (16, 256, 1024), (128, 512, 512),
                                   (128, 4096, 7168)])  # the last: the largest size the array holds
def test_noalloc_matches_allocating_entry_twice(m, n, k):
    from dsv4_b200 import _native as N
    q, qs, b, sh, cs = _case(m, n, k, 500 + m)
    stream = torch.cuda.current_stream().cuda_stream
    ref = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    ld = (n + 31) // 32 * 32
    partial = torch.empty((4, m, ld), dtype=torch.int32, device="cuda")
    N.call("dsv4_b200_mxfp4_int8_dense_gemm", q.data_ptr(), qs.data_ptr(), m, k, b.data_ptr(),
           sh.data_ptr(), sh.shape[0], cs.data_ptr(), n, ref.data_ptr(), partial.data_ptr(), 4, ld,
           stream)
    for _ in range(2):
        out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        N.call("dsv4_b200_mxfp4_int8_dense_gemm_noalloc", q.data_ptr(), qs.data_ptr(), m, k,
               b.data_ptr(), sh.data_ptr(), sh.shape[0], cs.data_ptr(), n, out.data_ptr(), stream)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().view(torch.int16).numpy(),
                                      ref.cpu().view(torch.int16).numpy())


def test_noalloc_rejects_sizes_beyond_the_workspace():
    from dsv4_b200 import _native as N
    q, qs, b, sh, cs = _case(129, 256, 256, 7)
    out = torch.empty((129, 256), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match="fixed split-K workspace"):
        N.call("dsv4_b200_mxfp4_int8_dense_gemm_noalloc", q.data_ptr(), qs.data_ptr(), 129, 256,
               b.data_ptr(), sh.data_ptr(), sh.shape[0], cs.data_ptr(), 256, out.data_ptr(),
               torch.cuda.current_stream().cuda_stream)


def test_noalloc_rejects_n_beyond_the_workspace_at_m_128():
    """m = 128 with n = 4224: 4 * 128 * 4224 words exceed the 8 MiB array."""
    from dsv4_b200 import _native as N
    q, qs, b, sh, cs = _case(128, 4224, 256, 8)
    out = torch.empty((128, 4224), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match="fixed split-K workspace"):
        N.call("dsv4_b200_mxfp4_int8_dense_gemm_noalloc", q.data_ptr(), qs.data_ptr(), 128, 256,
               b.data_ptr(), sh.data_ptr(), sh.shape[0], cs.data_ptr(), 4224, out.data_ptr(),
               torch.cuda.current_stream().cuda_stream)
