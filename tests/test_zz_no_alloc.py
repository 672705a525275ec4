"""The allocation-free decode entry point, qfn_moe_decode_noalloc.

It serves callers that cannot allocate device memory when they run a decode
step (memory planned once up front, a foreign-language binding with no device
allocator, a loop that forbids allocator calls): instead of a caller h_buf it
uses a fixed 32 x 640-float device array inside the library.  This file runs
last (pytest collects it last) so that a failure here leaves every other
test already run; it passes alone in a fresh process too.
"""
import ctypes

import numpy as np
import pytest
import torch

import _lib
import synthetic
from conftest import rel_err

pytestmark = pytest.mark.gpu

FP32_GRADE = 5e-5   # the tolerance the decode parity tests use


def _call(name, table, sidx, s2, coef, x, out, h=None):
    L = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    args = [table.data_ptr(), table.shape[0], sidx.data_ptr(), s2.data_ptr(), coef.data_ptr(), x.data_ptr(),
            _lib.DTYPE_BF16 if x.dtype == torch.bfloat16 else _lib.DTYPE_F32]
    if name == "qfn_moe_decode":
        rc = L.qfn_moe_decode(*args, h.data_ptr(), out.data_ptr(), sidx.numel(), stream)
    else:
        rc = L.qfn_moe_decode_noalloc(*args, out.data_ptr(), sidx.numel(), stream)
    _lib.check(rc, name)


def test_noalloc_matches_allocating_entry_point_on_two_calls():
    dev = "cuda"
    table = torch.from_numpy(synthetic.make_blocks(16, seed=91)).to(dev)
    cases = []
    for seed, K, xdt in ((1, 10, torch.bfloat16), (2, 7, torch.float32)):
        rng = np.random.Generator(np.random.PCG64(seed))
        sidx = torch.from_numpy(rng.choice(16, size=K, replace=False).astype(np.int32)).to(dev)
        s2 = torch.from_numpy(synthetic.make_s2(K, seed=seed, spread=True)).to(dev)
        coef = torch.from_numpy(rng.random(K).astype(np.float32)).to(dev)
        x = synthetic.make_x(2560, seed=seed, dtype=xdt).to(dev)
        cases.append((sidx, s2, coef, x))
    # two calls in a row through the allocation-free entry point
    outs = []
    for sidx, s2, coef, x in cases:
        out = torch.empty(2560, device=dev)
        _call("qfn_moe_decode_noalloc", table, sidx, s2, coef, x, out)
        outs.append(out)
    torch.cuda.synchronize()
    for (sidx, s2, coef, x), got in zip(cases, outs):
        want = torch.empty(2560, device=dev)
        _call("qfn_moe_decode", table, sidx, s2, coef, x, want, h=torch.empty(sidx.numel(), 640, device=dev))
        torch.cuda.synchronize()
        assert rel_err(got.cpu().numpy(), want.cpu().numpy()) <= FP32_GRADE
    assert _lib.device_status(clear=True) == 0


def test_noalloc_rejects_k_beyond_the_scratch():
    fake = ctypes.c_void_p(0x10000)
    rc = _lib.lib().qfn_moe_decode_noalloc(fake, 1, fake, fake, fake, fake, 1, fake, 33, None)
    assert rc == 4 and b"static scratch" in _lib.lib().qfn_last_error()
