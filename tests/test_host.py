"""Host-side logic on CPU: generators, routing helper, expert-table indexing."""
import numpy as np
import torch

import oracle
import routing
import synthetic
from expert_table import ExpertTable


def test_make_blocks_deterministic_and_distributed():
    a = synthetic.make_blocks(2, seed=5)
    b = synthetic.make_blocks(2, seed=5)
    assert a.shape == (2, synthetic.BLOCK) and np.array_equal(a, b)
    sc = oracle.e4m3_decode_table()[a[:, synthetic.O_GS:]]
    assert sc.min() >= 2.0 ** -4 * 0.93 and sc.max() <= 4.0 * 1.07   # e4m3(2**U(-4,2))
    w = a[:, :synthetic.O_GS]
    assert abs(w.mean() - 127.5) < 1.0                                # uniform bytes


def test_route_matches_oracle_on_cpu_tensors():
    logits = synthetic.zipf_logits(32, seed=3)
    ti, tv = routing.route(torch.from_numpy(logits))
    oti, ocoef = oracle.route(logits)
    assert np.array_equal(ti.numpy(), oti)
    assert np.array_equal(tv.float().numpy(), ocoef)


def test_zipf_logits_skewed():
    l = synthetic.zipf_logits(2048, seed=1234)
    ti, _ = routing.route(torch.from_numpy(l))
    counts = np.bincount(ti.numpy().ravel(), minlength=512)
    assert counts.sum() == 20480
    assert counts.max() > 10 * np.median(counts)     # Zipf(1.1) popularity
    assert (counts > 0).sum() > 400


def test_expert_table_rows_and_protocol_without_gpu():
    t = ExpertTable(K=10, dev="cpu", n_layers=2, n_experts=8, allocate=False)
    assert t.row(1, 3) == 11
    ti = torch.tensor([1, 7, 0])
    assert t.sidx_from_device(1, ti).tolist() == [9, 15, 8]
    assert t.sidx_from_device(1, ti).dtype == torch.int32


def test_decode_args_device_side():
    s2 = torch.arange(2 * 4 * 3, dtype=torch.float32).view(2, 4, 3)
    ti = torch.tensor([3, 0])
    tv = torch.tensor([0.75, 0.25], dtype=torch.bfloat16)
    sidx, s2k, coef = routing.decode_args(ti, tv, 1, 4, s2)
    assert sidx.tolist() == [7, 4] and sidx.dtype == torch.int32
    assert torch.equal(s2k, s2[1, [3, 0]]) and coef.dtype == torch.float32
