"""The C-ABI library loads and exports every entry point include/qfn.h
declares; host-side argument validation returns status codes without a GPU."""
import ctypes
import os
import re

import pytest

import _lib
from conftest import REPO

HEADERS = [os.path.join(REPO, "include", f) for f in sorted(os.listdir(os.path.join(REPO, "include")))
           if f.endswith(".h")]


def declared():
    names = set()
    for h in HEADERS:
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names |= set(re.findall(r"\b(qfn_[a-z0-9_]+)\s*\(", src))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared()
    for must in ("qfn_moe_decode", "qfn_gemv_e4m3", "qfn_e4m3_rows_to_bf16", "qfn_deq", "qfn_block_deq", "qfn_version",
                 "qfn_strerror", "qfn_last_error"):
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_signatures_cover_compute_entry_points():
    compute = [n for n in declared() if n not in ("qfn_version", "qfn_strerror", "qfn_last_error")]
    assert sorted(compute) == sorted(_lib.SIGNATURES)


def test_version_and_strerror():
    lib = _lib.lib()
    assert lib.qfn_version() >= 100
    assert lib.qfn_strerror(0) == b"ok"
    assert lib.qfn_strerror(1) == b"invalid argument"
    assert lib.qfn_strerror(999) == b"unknown status"


def test_validation_rejects_bad_arguments_without_touching_a_device():
    lib = _lib.lib()
    # null pointers
    assert lib.qfn_moe_decode(None, 1, None, None, None, None, 1, None, None, 10, None) == 1
    assert lib.qfn_gemv_e4m3(None, None, None, None, 1, 16, 16, None) == 1
    assert lib.qfn_deq(None, None, ctypes.c_float(1.0), None, 1, 32, None) == 1
    assert b"null" in lib.qfn_last_error()
    fake = ctypes.c_void_p(0x10000)   # never dereferenced: validation fails first
    # K outside [1, 32]
    assert lib.qfn_moe_decode(fake, 1, fake, fake, fake, fake, 1, fake, fake, 33, None) == 4
    assert lib.qfn_moe_decode(fake, 1, fake, fake, fake, fake, 1, fake, fake, 0, None) == 4
    # n_blocks must be positive; x dtype code must be known
    assert lib.qfn_moe_decode(fake, 0, fake, fake, fake, fake, 1, fake, fake, 10, None) == 1
    assert lib.qfn_moe_decode(fake, 1, fake, fake, fake, fake, 7, fake, fake, 10, None) == 1
    # misaligned table
    odd = ctypes.c_void_p(0x10001)
    assert lib.qfn_moe_decode(odd, 1, fake, fake, fake, fake, 1, fake, fake, 10, None) == 2
    # variant selection
    assert lib.qfn_moe_decode_variant(fake, 1, fake, fake, fake, fake, 1, fake, fake, 10, 5, None) == 1
    assert lib.qfn_moe_decode_variant(fake, 1, fake, fake, fake, fake, 1, fake, fake, 11, 4, None) == 4
    assert lib.qfn_moe_decode_variant(fake, 1, fake, fake, fake, fake, 1, fake, fake, 11, 3, None) == 4
    assert lib.qfn_moe_decode_variant(fake, 1, fake, fake, fake, fake, 1, fake, fake, 11, 1, None) == 4
    assert lib.qfn_device_status(None, 0) == 1
    # GEMV: K % 16, dtype, alignment
    assert lib.qfn_gemv_e4m3(fake, fake, fake, fake, 1, 16, 24, None) == 4
    assert lib.qfn_gemv_e4m3(fake, fake, fake, fake, 5, 16, 32, None) == 1
    assert lib.qfn_gemv_e4m3(odd, fake, fake, fake, 1, 16, 32, None) == 2
    # FP8 linear layer (T > 1): nulls, sizes, K % 16, alignment
    ln = lambda q, x, T, N, K: lib.qfn_linear_e4m3(q, fake, x, fake, T, N, K, None)
    assert ln(None, fake, 4, 16, 32) == 1
    assert ln(fake, fake, 0, 16, 32) == 1
    assert ln(fake, fake, 4, 16, 24) == 4
    assert ln(odd, fake, 4, 16, 32) == 2
    assert ln(fake, odd, 4, 16, 32) == 2
    # deq: K % 32
    assert lib.qfn_deq(fake, fake, ctypes.c_float(1.0), fake, 4, 48, None) == 4
    # e4m3 rows -> bf16: nulls, sizes, K % 16, alignment
    assert lib.qfn_e4m3_rows_to_bf16(None, fake, fake, 4, 32, None) == 1
    assert lib.qfn_e4m3_rows_to_bf16(fake, fake, fake, 0, 32, None) == 1
    assert lib.qfn_e4m3_rows_to_bf16(fake, fake, fake, 4, 24, None) == 4
    assert lib.qfn_e4m3_rows_to_bf16(odd, fake, fake, 4, 32, None) == 2
    # fused router: nulls, n_experts % 4, topk range, s2_out without s2_layer, alignment
    r = lambda x, T, E, k, s2l, s2o: lib.qfn_moe_route(x, fake, T, E, k, 0, s2l, fake, fake, None, None, s2o, fake,
                                                         None)
    assert r(None, 1, 512, 10, None, None) == 1
    assert r(fake, 1, 510, 10, None, None) == 4
    assert r(fake, 1, 2048, 10, None, None) == 4
    assert r(fake, 1, 512, 33, None, None) == 4
    assert r(fake, 0, 512, 10, None, None) == 4
    assert r(fake, 1, 512, 10, None, fake) == 1
    assert r(odd, 1, 512, 10, None, None) == 2
    # shared expert (whole and halves): nulls, inter % 8 and range, T range, alignment
    sh = lambda x, I: lib.qfn_shared_expert(x, 1, fake, fake, fake, fake, I, None, fake, fake, fake, None)
    assert sh(None, 512) == 1
    assert sh(fake, 644) == 4
    assert sh(fake, 8192) == 4
    assert sh(odd, 512) == 2
    gu = lambda x, I: lib.qfn_shared_expert_gate_up(x, 1, fake, fake, fake, I, fake, fake, None)
    assert gu(None, 640) == 1
    assert gu(fake, 644) == 4
    assert gu(odd, 640) == 2
    dw = lambda wd, I, T: lib.qfn_shared_expert_down(wd, I, T, fake, fake, None, fake, None)
    assert dw(None, 640, 1) == 1
    assert dw(fake, 640, 0) == 4
    assert dw(odd, 640, 1) == 2
    # delta rule: nulls, head ratio, dk / dv
    dn = lambda H, Hk, dk, dv: lib.qfn_deltanet_step(fake, fake, fake, fake, fake, fake, fake, H, Hk, dk, dv, None)
    assert lib.qfn_deltanet_step(None, fake, fake, fake, fake, fake, fake, 4, 2, 128, 128, None) == 1
    assert dn(4, 3, 128, 128) == 1
    assert dn(4, 2, 96, 128) == 4
    assert dn(4, 2, 128, 100) == 4
    assert lib.qfn_set_prefill_sm_budget(-1) == 1
    # expert-parallel layer over NCCL: nulls (the communicator first), sizes, workspace query
    ep = lambda comm, T, nl: lib.qfn_moe_prefill_ep(fake, T, fake, 1, fake, 0, 10, fake, 8, 0, fake, nl, fake, 16,
                                                    comm, fake, fake, 1 << 20, None)
    assert ep(None, 4, 2) == 1
    assert ep(fake, 0, 2) == 1
    assert ep(fake, 4, 0) == 1
    assert lib.qfn_moe_prefill_ep_workspace(0, 10, 2, 2) == 0
    assert lib.qfn_moe_prefill_ep_workspace(64, 10, 2, 2) > lib.qfn_moe_prefill_workspace(128, 10, 2)
    assert lib.qfn_nccl_comm_init(None, 2, 0, fake) == 1
    assert lib.qfn_nccl_comm_destroy(None) == 1


def test_python_wrappers_reject_cpu_tensors():
    import torch
    import fp8gemv
    import qmoe
    q = torch.zeros(16, 32, dtype=torch.float8_e4m3fn)
    with pytest.raises(ValueError, match="CUDA"):
        fp8gemv.gemv(q, torch.ones(16), torch.zeros(32, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="CUDA"):
        fp8gemv.linear(torch.zeros(4, 32, dtype=torch.bfloat16), q, torch.ones(16, 1))
    with pytest.raises(ValueError, match="CUDA"):
        qmoe.moe_decode(torch.zeros(1, qmoe.BLOCK, dtype=torch.uint8), torch.zeros(1, dtype=torch.int32),
                        torch.zeros(1, 3), torch.zeros(1), torch.zeros(2560), torch.zeros(1, 640),
                        torch.zeros(1, 2560))
    with pytest.raises(NotImplementedError):
        qmoe.SWAP = True
        try:
            qmoe.deq(torch.zeros(2, 16, dtype=torch.uint8), torch.zeros(2, 2, dtype=torch.uint8), 1.0)
        finally:
            qmoe.SWAP = False


def test_reference_constants_kept():
    import qmoe
    assert (qmoe.HID, qmoe.INTER, qmoe.BLOCK) == (2560, 640, 2764800)
    assert (qmoe.O_GW, qmoe.O_UW, qmoe.O_DW, qmoe.O_GS, qmoe.O_US, qmoe.O_DS) == (
        0, 819200, 1638400, 2457600, 2560000, 2662400)
    assert (qmoe.KB_UP, qmoe.G_UP, qmoe.KB_DN, qmoe.G_DN) == (1280, 160, 320, 40)
    assert qmoe.E2M1.tolist() == [0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6]
    # the block layout adds up (repack_experts.py:12-19)
    sizes = [819200] * 3 + [102400] * 3
    assert sum(sizes) == qmoe.BLOCK and qmoe.BLOCK % 4096 == 0


def test_prefill_validation_and_workspace_size():
    lib = _lib.lib()
    fake = ctypes.c_void_p(0x10000)
    T, topk, E = 2048, 10, 512
    P = T * topk
    ws = lib.qfn_moe_prefill_workspace(T, topk, E)
    # pair arrays + f16 x rows + fp32 h + f16 hi/lo h dominate
    assert ws >= P * (2560 * 2 + 640 * 4 + 640 * 4)
    assert lib.qfn_moe_prefill_workspace(0, topk, E) == 0
    args = dict(x=fake, T=T, ti=fake, i64=1, tv=fake, tvd=1, topk=topk, table=fake, nb=24576, base=0, s2=fake,
                E=E, out=fake, ws=fake, wsb=ws)

    def call(**kw):
        a = dict(args, **kw)
        return lib.qfn_moe_prefill(a["x"], a["T"], a["ti"], a["i64"], a["tv"], a["tvd"], a["topk"], a["table"],
                                   a["nb"], a["base"], a["s2"], a["E"], a["out"], a["ws"], a["wsb"], None)

    assert call(T=0) == 0                        # nothing to do
    assert call(x=None) == 1                     # null pointer
    assert call(topk=33) == 1                    # topk outside [1, 32]
    assert call(E=1025) == 4                     # more experts than the routing kernel holds
    assert call(tvd=7) == 1                      # unknown tv dtype
    assert call(base=24576 - 100) == 1           # layer's experts past the end of the table
    assert call(wsb=ws - 1) == 5                 # workspace too small
    assert call(ws=ctypes.c_void_p(0x10010)) == 2  # workspace not 256-byte aligned


def test_torch_extension_registers_the_hot_path_operators():
    """libqfn_torch.so (the thin torch extension over the C ABI) loads on a
    machine without a GPU and registers the four operators; a CPU tensor is
    refused by the operator's own checks."""
    import torch
    ops = _lib.ops()
    for name in ("moe_decode", "moe_prefill", "gemv", "linear"):
        assert hasattr(ops, name), name
    schema = str(torch.ops.qfn.moe_decode.default._schema)
    assert "Tensor(a!) h_buf" in schema and "int variant" in schema
    with pytest.raises(ValueError, match="CUDA"):
        torch.ops.qfn.gemv(torch.zeros(16, 32, dtype=torch.uint8), torch.ones(16), torch.zeros(32, dtype=torch.bfloat16),
                           False)
