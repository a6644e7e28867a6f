"""qtb_attention_noalloc, the allocation-free variant of the standalone
attention stage, against the allocating entry point qtb_attention_host on the
same inputs: two calls in a row, each bit-identical to it (output and the
appended K/V pages); a request beyond the fixed scratch is refused before
anything runs.  Device buffers come from torch (plumbing only)."""
import ctypes as C

import numpy as np
import pytest

import qtts_b200 as Q
from test_gpu_kernels import make_attention_case

pytestmark = pytest.mark.gpu

_vp = C.c_void_p


def _noalloc():
    f = Q.lib().qtb_attention_noalloc
    f.argtypes = [_vp, C.c_int, C.c_int, C.c_int, C.c_int, _vp, _vp, C.c_float, _vp, _vp, C.c_int, _vp, _vp,
                  C.c_int, _vp, C.c_int, _vp, C.c_int, _vp, _vp]
    return f


# the second case sits at the limits (batch 4, n_kv 16, max_splits 16) with
# 1024 work items, more than the CTAs: the dynamic item order, whose counter
# lives in the shared scratch, runs through this entry point too
@pytest.mark.parametrize("pos,nh,nkv,n_pages,max_splits",
                         [([37, 200, 5], 16, 8, 40, 4), ([300, 511, 257, 400], 32, 16, 110, 16)])
def test_noalloc_attention_equals_allocating_entry_point(have_gpu, pos, nh, nkv, n_pages, max_splits):
    import torch
    rng = np.random.default_rng(21 + len(pos))
    eps = 1e-6
    qkv, kp, vp, pt, qn, kn, cs, sn = make_attention_case(rng, len(pos), pos, n_pages, nh=nh, nkv=nkv)
    kp_ref, vp_ref = kp.copy(), vp.copy()
    out_ref = Q.attention(qkv, nh, nkv, qn, kn, eps, cs, sn, kp_ref, vp_ref, pt, np.array(pos, np.int32), max_splits)

    dev = torch.device("cuda:0")

    def t(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(dev)

    d_qkv, d_qn, d_kn, d_cs, d_sn = t(qkv), t(qn), t(kn), t(cs), t(sn)
    d_kp, d_vp = t(kp.view(np.int16)), t(vp.view(np.int16))
    d_pt, d_pos = t(pt), t(np.array(pos, np.int32))
    d_out = torch.empty((len(pos), nh * 128), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    f = _noalloc()
    for call in range(2):
        d_out.fill_(float("nan"))
        rc = f(d_qkv.data_ptr(), len(pos), nh, nkv, 128, d_qn.data_ptr(), d_kn.data_ptr(), eps, d_cs.data_ptr(),
               d_sn.data_ptr(), cs.shape[0], d_kp.data_ptr(), d_vp.data_ptr(), n_pages, d_pt.data_ptr(),
               pt.shape[1], d_pos.data_ptr(), max_splits, d_out.data_ptr(), stream)
        assert rc == 0, (call, Q.lib().qtb_last_error())
        torch.cuda.synchronize(dev)
        assert np.array_equal(d_out.cpu().numpy(), out_ref), call
        # appending the same token again rewrites the same bytes
        assert np.array_equal(d_kp.cpu().numpy().view(np.uint16), kp_ref), call
        assert np.array_equal(d_vp.cpu().numpy().view(np.uint16), vp_ref), call

    # beyond the fixed scratch (batch > 4): refused, nothing written
    big = 5
    d_out2 = torch.full((big, nh * 128), 7.0, dtype=torch.float32, device=dev)
    rc = f(d_qkv.data_ptr(), big, nh, nkv, 128, d_qn.data_ptr(), d_kn.data_ptr(), eps, d_cs.data_ptr(),
           d_sn.data_ptr(), cs.shape[0], d_kp.data_ptr(), d_vp.data_ptr(), n_pages, d_pt.data_ptr(), pt.shape[1],
           d_pos.data_ptr(), max_splits, d_out2.data_ptr(), stream)
    assert rc == -1   # QTB_E_INVALID
    assert bool((d_out2 == 7.0).all())
