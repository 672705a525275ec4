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


def _cases(table_blocks, specs, dev="cuda"):
    cases = []
    for seed, K, xdt in specs:
        rng = np.random.Generator(np.random.PCG64(seed))
        sidx = torch.from_numpy(rng.choice(table_blocks, size=K, replace=K > table_blocks).astype(np.int32)).to(dev)
        s2 = torch.from_numpy(synthetic.make_s2(K, seed=seed, spread=True)).to(dev)
        coef = torch.from_numpy(rng.random(K).astype(np.float32)).to(dev)
        x = synthetic.make_x(2560, seed=seed, dtype=xdt).to(dev)
        cases.append((sidx, s2, coef, x))
    return cases


# K <= 10 runs the slice kernel; K = 16 and K = 32 (the whole extent of the
# scratch array) run the two-launch CUDA-core kernels, which pass h between
# their launches through the scratch.
@pytest.mark.parametrize("specs", [((1, 10, torch.bfloat16), (2, 7, torch.float32)),
                                   ((3, 16, torch.bfloat16), (4, 32, torch.float32))])
def test_noalloc_matches_allocating_entry_point_on_two_calls(specs):
    dev = "cuda"
    table = torch.from_numpy(synthetic.make_blocks(16, seed=91)).to(dev)
    cases = _cases(16, specs)
    # two calls in a row through the allocation-free entry point, queued on one
    # stream without a synchronisation between them: the second call's kernels
    # must not overwrite the shared scratch before the first call's have read it
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


def test_noalloc_back_to_back_mixed_paths_in_one_stream():
    """A K = 32 call (CUDA-core kernels, whole scratch) directly followed on the
    same stream by a K = 10 call (slice kernel) and another K = 32 call with
    other inputs: each result matches the allocating entry point."""
    dev = "cuda"
    table = torch.from_numpy(synthetic.make_blocks(16, seed=92)).to(dev)
    cases = _cases(16, ((11, 32, torch.bfloat16), (12, 10, torch.bfloat16), (13, 32, torch.float32)))
    outs = [torch.empty(2560, device=dev) for _ in cases]
    for (sidx, s2, coef, x), out in zip(cases, outs):
        _call("qfn_moe_decode_noalloc", table, sidx, s2, coef, x, out)
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
