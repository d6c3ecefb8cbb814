"""The allocation-free decode entry point, called through the C ABI.

bpkv_page16_decode_noalloc serves callers that cannot allocate device memory
while they decode (a pool that already holds nearly all of HBM, an FFI host
without a device allocator, a loop that must avoid cudaMalloc's implicit
synchronisation).  Its scratch is a fixed 16 MiB device array inside the
library, so this test checks it against the workspace-taking entry point on
the same inputs, twice in a row (the array keeps the previous call's
contents), and that oversized shapes are refused.  The file name sorts last so
a run that stops at the first failure has already run every other test.
"""
import math

import numpy as np
import pytest
import torch

from oracle.page16 import page16_decode_reference
from tests.golden.inputs import page16_case

pytestmark = pytest.mark.gpu


def _call(fn_name, L, tensors, ws=None):
    q, k, v, bt, lens, out, lse = tensors
    args = [q.data_ptr(), k.data_ptr(), v.data_ptr(), bt.data_ptr(), lens.data_ptr(), out.data_ptr(),
            lse.data_ptr(), q.shape[0], q.shape[1], k.shape[2], q.shape[2], bt.shape[1], q.stride(0), q.stride(1),
            k.stride(0), bt.stride(0), 1.0 / math.sqrt(q.shape[2]), 2]
    if ws is not None:
        args += [ws.data_ptr(), ws.numel()]
    args.append(torch.cuda.current_stream().cuda_stream)
    return getattr(L, fn_name)(*args)


def _inputs(cuda, seed, lens, hq=32, hkv=8, d=128):
    q, k, v, bt, lens = page16_case(seed=seed, batch=len(lens), hq=hq, hkv=hkv, d=d, lens=lens, num_pages=600,
                                    scale_std=0.5)
    t = [torch.from_numpy(x).to(cuda, torch.bfloat16) for x in (q, k, v)]
    bt_d = torch.from_numpy(bt).to(cuda)
    lens_d = torch.from_numpy(lens).to(cuda)
    return t, bt_d, lens_d


def test_noalloc_matches_workspace_entry_point_twice(cuda):
    from unifiedkv_b200 import _lib
    L = _lib.load()
    assert L.bpkv_page16_decode_noalloc_max_scratch() == 16 << 20
    for call, (seed, lens) in enumerate([(11, (5, 300, 1000, 4000)), (12, (17, 2048, 3, 900, 77))]):
        (q, k, v), bt, ln = _inputs(cuda, seed, lens)
        B, hq, d = q.shape
        ref_out = torch.empty_like(q)
        ref_lse = torch.empty(B, hq, dtype=torch.float32, device=cuda)
        nbytes = L.bpkv_page16_decode_workspace_size(B, hq, 8, d, 2)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=cuda)
        assert _call("bpkv_page16_decode", L, (q, k, v, bt, ln, ref_out, ref_lse), ws) == 0
        out = torch.full_like(q, float("nan"))
        lse = torch.full((B, hq), float("nan"), dtype=torch.float32, device=cuda)
        rc = _call("bpkv_page16_decode_noalloc", L, (q, k, v, bt, ln, out, lse))
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        # same kernels and work split: the results agree to well within the
        # 2e-3 decode tolerance (they are in fact bitwise equal)
        assert (out.float() - ref_out.float()).abs().max().item() < 2e-3, call
        assert (lse - ref_lse).abs().max().item() < 1e-3, call
        # and both against the CPU oracle of the reference's gather-then-attention path
        o64 = page16_decode_reference(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                                      bt.cpu().numpy(), ln.cpu().numpy(), 1.0 / math.sqrt(d), hq // 8)
        assert np.abs(out.float().cpu().numpy() - o64).max() < 2e-3, call


def test_noalloc_rejects_oversized_scratch(cuda):
    from unifiedkv_b200 import _lib
    L = _lib.load()
    B, hq, d = 8192, 64, 256  # partial slots alone need ~560 MB > 16 MiB
    assert L.bpkv_page16_decode_workspace_size(B, hq, 8, d, 2) > L.bpkv_page16_decode_noalloc_max_scratch()
    dummy = torch.zeros(16, dtype=torch.bfloat16, device=cuda)
    rc = L.bpkv_page16_decode_noalloc(dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(),
                                      dummy.data_ptr(), dummy.data_ptr(), None, B, hq, 8, d, 1, hq * d, d,
                                      16 * 8 * d, 1, 0.1, 2, None)
    assert rc == _lib.BPKV_ERR_WORKSPACE and "exceeds_max" in _lib.last_error()
