"""Device-side errors reach the host (GPU).

The decode kernel checks every page id it loads against the storage's page count; an id
outside it is read as physical page 0 and recorded as error 2 in the workspace flag, and the
launch itself succeeds.  ``check_device_errors`` (and ``PagedRazorKVCache.check_errors``)
must raise it and clear the flag.  The case runs on the sm_100a decode kernel's shape (bf16,
head_dim 128, 16-token pages), whose producer performs that check before any copy, so the
bad id causes no out-of-range access.
"""

import numpy as np
import pytest
import torch

from oracle import razorkv_oracle as O
from razorkv_b200._lib import DeviceError
from razorkv_b200.kernels import check_device_errors, triton_paged_sparse_attention

pytestmark = pytest.mark.gpu


def _case(seed=0):
    g = torch.Generator().manual_seed(seed)
    B, H, Hkv, maxp, P, D = 2, 8, 2, 6, 16, 128
    q = torch.randn(B, H, 1, D, generator=g).to(torch.bfloat16)
    kp = torch.randn(B, Hkv, maxp, P, D, generator=g).to(torch.bfloat16)
    vp = torch.randn(B, Hkv, maxp, P, D, generator=g).to(torch.bfloat16)
    return q, kp, vp, maxp


def test_page_id_outside_the_storage_raises_on_check():
    q, kp, vp, maxp = _case()
    check_device_errors()   # start from clean flags
    good = torch.tensor([[0, 2, 4], [1, 3, 5]])
    bad = torch.tensor([[0, 2, 4], [1, 3, maxp]])
    with pytest.raises(IndexError):   # the operator's default host-side validation
        triton_paged_sparse_attention(q.cuda(), kp.cuda(), vp.cuda(), bad.cuda())
    out = triton_paged_sparse_attention(q.cuda(), kp.cuda(), vp.cuda(), bad.cuda(),
                                        validate=False)
    torch.cuda.synchronize()
    with pytest.raises(DeviceError) as e:
        check_device_errors()
    assert e.value.code == 2
    check_device_errors()   # cleared by the check
    # sequence 0 never touched the bad id; sequence 1 read page 0 in its place
    ref = O.paged_attention(q.float().numpy(), kp.float().numpy(), vp.float().numpy(),
                            np.array([[0, 2, 4], [1, 3, 0]]))
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=2e-2, rtol=1e-2)
    out2 = triton_paged_sparse_attention(q.cuda(), kp.cuda(), vp.cuda(), good.cuda())
    torch.cuda.synchronize()
    check_device_errors()   # a clean launch leaves no flag
    ref2 = O.paged_attention(q.float().numpy(), kp.float().numpy(), vp.float().numpy(),
                             good.numpy())
    np.testing.assert_allclose(out2.float().cpu().numpy(), ref2, atol=2e-2, rtol=1e-2)
