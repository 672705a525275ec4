"""HBM-resident expert table: the B200 replacement for ExpertCache.

The reference streams experts NVMe -> pinned-RAM LRU -> two GPU slot banks
(ExpertCache, qwen_engine.py:344-573) because 63 GiB do not fit in 8 GB.  On
a 180 GB B200 every block of every layer stays resident:

    slots  u8 [n_layers * n_experts, BLOCK]   block of (L, e) at row L*n_experts + e
    s2     f32[n_layers, n_experts, 3]        ws2 gate/up/down (experts_scal.npy[..., :3])

`moe_decode(table.slots, sidx, ...)` takes sidx = L*n_experts + e directly,
so a decode step moves no expert bytes over PCIe.  The ExpertCache call
protocol (start -> finish -> kernel -> done, plus speculate / prefetch /
drop_pf / prefill_batch) is kept so QwenEngine.moe runs unchanged; the
prefetch/speculation hooks have nothing left to do and return immediately.
"""
import collections
import os

import numpy as np
import torch

BLOCK = 2764800


class ExpertTable:
    PB = 32   # experts per prefill batch (ExpertCache.PB, qwen_engine.py:523)

    def __init__(self, K=10, dev="cuda", n_layers=48, n_experts=512, ram_gb=0.0, threads=0, pf=0, spec=0,
                 allocate=True):
        self.K, self.dev = K, torch.device(dev)
        self.n_layers, self.n_experts = n_layers, n_experts
        self.pf, self.spec = 0, 0
        self.slots = (torch.empty(n_layers * n_experts, BLOCK, dtype=torch.uint8, device=self.dev)
                      if allocate else None)
        self.s2 = torch.full((n_layers, n_experts, 3), 1.0 / 448.0, dtype=torch.float32, device=self.dev)
        # Pinned ring of per-layer sidx rows, as in ExpertCache (qwen_engine.py:362-363): a row is
        # rewritten only a whole token later, long after its copy completed.
        self._sidx_h = torch.empty(64, K, dtype=torch.int32).pin_memory() if self.dev.type == "cuda" else None
        self._sidx_d = torch.empty(64, K, dtype=torch.int32, device=self.dev)
        self.stat = collections.Counter()
        self.read_s = 0.0
        self.nread = 0

    @property
    def nbytes(self):
        return 0 if self.slots is None else self.slots.numel()

    def row(self, L, e):
        return L * self.n_experts + e

    def sidx(self, L, experts):
        """int32[K] device tensor of absolute block rows for `experts` (host ints) of layer L."""
        k = len(experts)
        r = self._sidx_h[L % 64, :k]
        r.copy_(torch.tensor([self.row(L, e) for e in experts], dtype=torch.int32))
        d = self._sidx_d[L % 64, :k]
        d.copy_(r, non_blocking=True)
        return d

    def sidx_from_device(self, L, ti):
        """Block rows from device expert ids (no host synchronisation)."""
        return (ti + L * self.n_experts).to(torch.int32)

    # ---- ExpertCache decode protocol (qwen_engine.py:412-468)
    def start(self, L, experts):
        self.stat["hbm_hit"] += len(experts)
        return L, self.sidx(L, experts)

    def finish(self, h):
        return h[1]

    def done(self, L):
        pass

    def speculate(self, L, cands):
        pass

    def prefetch(self, L, cands, protect=()):
        pass

    def drop_pf(self, L):
        pass

    # ---- prompt path (qwen_engine.py:525-553): device rows instead of pinned host rows
    def prefill_batch(self, L, experts):
        return [self.slots[self.row(L, e)] for e in experts]

    def block_host(self, L, e):
        return self.slots[self.row(L, e)].cpu()

    # ---- filling
    def fill_synthetic(self, seed=0, experts=None):
        """Synthetic blocks (config-0 distributions): row L * n_experts + i gets
        the block of (L, experts[i]) (default: the first n_experts), seeded per
        (layer, global expert) so that any process can regenerate it."""
        from synthetic import fill_table_gpu
        experts = list(range(self.n_experts)) if experts is None else list(experts)
        fill_table_gpu(self.slots, self.n_layers, experts, seed)
        return self

    def load(self, experts_bin, experts_scal=None, experts=None, file_experts=512, chunk_blocks=64):
        """Copy blocks of a repacked experts.bin and the ws2 of experts_scal.npy into the table.

        File layout (repack_experts.py:8-19): block (L, e) at byte
        (L * file_experts + e) * BLOCK, file_experts = 512 (NE, :11); scalars
        f32[L, file_experts, 6] with ws2 gate/up/down in [..., :3]
        (repack_experts.py:20-21, read as store.s2 at qwen_engine.py:370).
        `experts` lists the global expert ids this table holds, in table
        order (an expert-parallel shard; default: the first n_experts), so
        table row L * n_experts + i holds file block (L, experts[i]).  On a
        CUDA table, runs of consecutive file blocks are read through two
        pinned staging buffers: the disk read of one chunk overlaps the
        host->device copy of the previous one."""
        experts = list(range(self.n_experts)) if experts is None else [int(e) for e in experts]
        if len(experts) != self.n_experts or min(experts) < 0 or max(experts) >= file_experts:
            raise ValueError(f"experts must list {self.n_experts} ids in [0, {file_experts})")
        need = self.n_layers * file_experts * BLOCK
        size = os.path.getsize(experts_bin)
        if size < need:
            raise ValueError(f"{experts_bin} has {size} bytes, {self.n_layers} layers of {file_experts} "
                             f"experts need {need}")
        # (table row, file block, count) runs of consecutive blocks, at most chunk_blocks long
        runs = []
        for L in range(self.n_layers):
            i = 0
            while i < self.n_experts:
                j = i + 1
                while j < self.n_experts and j - i < chunk_blocks and experts[j] == experts[j - 1] + 1:
                    j += 1
                runs.append((L * self.n_experts + i, L * file_experts + experts[i], j - i))
                i = j
        cuda = self.slots.is_cuda
        if cuda:
            stage = [torch.empty(chunk_blocks * BLOCK, dtype=torch.uint8).pin_memory() for _ in range(2)]
            events = [None, None]
            side = torch.cuda.Stream(self.dev)
        with open(experts_bin, "rb", buffering=0) as f:
            for k, (row, fblk, n) in enumerate(runs):
                f.seek(fblk * BLOCK)
                if not cuda:
                    view = memoryview(self.slots[row:row + n].numpy()).cast("B")
                    got = f.readinto(view)
                else:
                    buf = stage[k % 2]
                    if events[k % 2] is not None:
                        events[k % 2].synchronize()
                    got = f.readinto(memoryview(buf.numpy())[: n * BLOCK])
                    with torch.cuda.stream(side):
                        self.slots[row:row + n].view(-1).copy_(buf[: n * BLOCK], non_blocking=True)
                        ev = torch.cuda.Event()
                        ev.record(side)
                    events[k % 2] = ev
                if got != n * BLOCK:
                    raise IOError(f"short read at file block {fblk}: {got} of {n * BLOCK} bytes")
        if cuda:
            side.synchronize()
        if experts_scal is not None:
            scal = np.load(experts_scal)
            if scal.ndim != 3 or scal.shape[0] < self.n_layers or scal.shape[1] != file_experts or scal.shape[2] < 3:
                raise ValueError(f"experts_scal must be f32[>={self.n_layers}, {file_experts}, 6], got {scal.shape}")
            sel = np.ascontiguousarray(scal[: self.n_layers][:, experts, :3], dtype=np.float32)
            self.s2.copy_(torch.from_numpy(sel))
        return self
