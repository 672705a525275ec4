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
    def fill_synthetic(self, seed=0):
        from synthetic import fill_blocks_gpu
        fill_blocks_gpu(self.slots, seed)
        return self

    def load(self, experts_bin, experts_scal=None, chunk_blocks=64):
        """Copy a repacked experts.bin (repack_experts.py layout, block (L,e) at
        byte (L*n_experts+e)*BLOCK) and experts_scal.npy f32[L,E,6] into HBM.
        Reads go through two pinned staging buffers so the disk read of chunk
        i+1 overlaps the host->device copy of chunk i."""
        n = self.slots.shape[0]
        need = n * BLOCK
        size = os.path.getsize(experts_bin)
        if size < need:
            raise ValueError(f"{experts_bin} has {size} bytes, the table needs {need}")
        stage = [torch.empty(chunk_blocks * BLOCK, dtype=torch.uint8).pin_memory() for _ in range(2)]
        events = [None, None]
        side = torch.cuda.Stream(self.dev)
        with open(experts_bin, "rb", buffering=0) as f:
            for i, b0 in enumerate(range(0, n, chunk_blocks)):
                b1 = min(n, b0 + chunk_blocks)
                buf = stage[i % 2]
                if events[i % 2] is not None:
                    events[i % 2].synchronize()
                view = memoryview(buf.numpy())[: (b1 - b0) * BLOCK]
                got = f.readinto(view)
                if got != (b1 - b0) * BLOCK:
                    raise IOError(f"short read at block {b0}: {got}")
                with torch.cuda.stream(side):
                    self.slots[b0:b1].view(-1).copy_(buf[: (b1 - b0) * BLOCK], non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(side)
                events[i % 2] = ev
        side.synchronize()
        if experts_scal is not None:
            scal = np.load(experts_scal)
            self.s2.copy_(torch.from_numpy(np.ascontiguousarray(scal[: self.n_layers, : self.n_experts, :3])))
        return self
