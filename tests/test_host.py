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


def _write_repacked(tmp_path, n_layers, file_experts, seed):
    """A small experts.bin / experts_scal.npy in the repack_experts.py layout
    (block (L, e) at byte (L * file_experts + e) * BLOCK; scalars f32[L, E, 6])."""
    blocks = synthetic.make_blocks(n_layers * file_experts, seed=seed)
    path = tmp_path / "experts.bin"
    blocks.tofile(path)
    rng = np.random.Generator(np.random.PCG64(seed + 1))
    scal = rng.uniform(0.5, 2.0, size=(n_layers, file_experts, 6)).astype(np.float32) / 448.0
    np.save(tmp_path / "experts_scal.npy", scal)
    return blocks.reshape(n_layers, file_experts, -1), scal, str(path), str(tmp_path / "experts_scal.npy")


def test_expert_table_load_whole_file(tmp_path):
    blocks, scal, bin_path, scal_path = _write_repacked(tmp_path, 2, 3, seed=41)
    t = ExpertTable(K=2, dev="cpu", n_layers=2, n_experts=3).load(bin_path, scal_path, file_experts=3, chunk_blocks=2)
    assert np.array_equal(t.slots.numpy(), blocks.reshape(6, -1))
    assert np.array_equal(t.s2.numpy(), scal[..., :3])
    assert t.row(1, 2) == 5


def test_expert_table_load_expert_parallel_shard(tmp_path):
    """A shard of non-consecutive experts (a load-aware placement): table row
    L * n + i holds file block (L, experts[i]) and s2 follows the same order."""
    blocks, scal, bin_path, scal_path = _write_repacked(tmp_path, 2, 4, seed=42)
    experts = [3, 0]
    t = ExpertTable(K=2, dev="cpu", n_layers=2, n_experts=2).load(bin_path, scal_path, experts=experts, file_experts=4)
    for L in range(2):
        for i, e in enumerate(experts):
            assert np.array_equal(t.slots[t.row(L, i)].numpy(), blocks[L, e])
            assert np.array_equal(t.s2[L, i].numpy(), scal[L, e, :3])


def test_expert_table_load_rejects_short_file(tmp_path):
    import pytest
    _, _, bin_path, _ = _write_repacked(tmp_path, 1, 2, seed=43)
    t = ExpertTable(K=2, dev="cpu", n_layers=2, n_experts=2)
    with pytest.raises(ValueError):
        t.load(bin_path, file_experts=2)
