"""Column (output-feature) sharding of a packed MTC matrix over the GPUs of a node.

Each GPU keeps the column slice [cut_g, cut_g+1) of the stored (permuted)
matrix, cut on 32-column tile boundaries and balanced by payload bytes
(MTC-QT-P sorts columns by importance, so equal column counts would give
unequal bytes).  Every GPU receives the full activations, gathers X[:, pr]
and computes its slice of the permuted output; one all-gather over NCCL
(NVLink/NVSwitch) collects the slices, and one row-permute kernel writes the
original column order Y[:, pc].  For large M the rows go in two chunks: the
second chunk's GEMM (held to all but 16 SMs) runs while the first chunk is
all-gathered and assembled on a side stream.  No other communication: the reference has
no distributed path (it is a single-process Numba package), so this is the
B200-side scale-out of mtc_gemm (mtc/kernels/gemm.py:541-574 and the
gather/scatter of mtc/core/permutation.py:15-21).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import numpy as np

from .core import layout
from .kernels.gemm import MTCMatrix

TILE = layout.TILE


@dataclass
class ShardPlan:
    cuts: List[int]          # permuted column boundaries, len world + 1
    wmax: int                # widest slice (all-gather chunk width)
    pos: np.ndarray          # int32 [N]: original column j reads gathered position pos[j]

    @property
    def world(self) -> int:
        return len(self.cuts) - 1


def column_cuts(mat: MTCMatrix, world: int) -> List[int]:
    """Tile-aligned cuts of the stored columns with near-equal payload bytes."""
    K, N = mat.shape
    ntc = -(-N // TILE)
    if world > ntc:
        raise ValueError(f"{world} shards for {ntc} tile columns: use at most {ntc} GPUs for this matrix")
    ls = mat.leaf_set
    per_col = np.bincount((ls.col // TILE).astype(np.int64), weights=ls.payload_bytes.astype(np.float64),
                          minlength=ntc)
    # metadata per leaf counts too (scale + mode), so empty (P0) columns still cost something
    per_col += np.bincount((ls.col // TILE).astype(np.int64), minlength=ntc) * 3.0
    csum = np.concatenate([[0.0], np.cumsum(per_col)])
    cuts = [0]
    for g in range(1, world):
        target = csum[-1] * g / world
        c = int(np.searchsorted(csum, target))
        c = min(max(c, cuts[-1] + 1), ntc - (world - g))
        cuts.append(c)
    cuts.append(ntc)
    return [min(c * TILE, N) for c in cuts]


def plan_shards(mat: MTCMatrix, world: int) -> ShardPlan:
    cuts = column_cuts(mat, world)
    widths = np.diff(cuts)
    wmax = int(widths.max())
    K, N = mat.shape
    shard_of = np.searchsorted(np.asarray(cuts[1:]), np.arange(N), side="right")
    loc = np.arange(N) - np.asarray(cuts)[shard_of]
    gathered = (shard_of * wmax + loc).astype(np.int64)   # position of stored column n in the gathered row
    if mat.col_perm is None:
        pos = gathered
    else:
        inv = np.empty(N, dtype=np.int64)
        inv[np.asarray(mat.col_perm)] = np.arange(N)
        pos = gathered[inv]                                  # original column j = stored column inv[j]
    return ShardPlan(list(map(int, cuts)), wmax, pos.astype(np.int32))


def local_shard(mat: MTCMatrix, plan: ShardPlan, rank: int) -> MTCMatrix:
    """The stored-column slice of rank `rank` as a packed matrix of its own
    (shares the arena; output in slice-local stored order)."""
    n0, n1 = plan.cuts[rank], plan.cuts[rank + 1]
    ls = mat.leaf_set
    sel = (ls.col >= n0) & (ls.col < n1)
    if mat.is_quadtree:
        return MTCMatrix((mat.shape[0], n1 - n0), mat.block_size, mat.arena, ls.offset[sel].astype(np.uint32),
                         ls.mode[sel].copy(), ls.scale[sel].copy(), None, leaf_rows=ls.row[sel],
                         leaf_cols=ls.col[sel] - n0, leaf_sizes=ls.size[sel], sizes=mat.sizes,
                         row_perm=mat.row_perm, col_perm=None)
    bs = mat.block_size
    if n0 % bs or (n1 - n0) % bs and n1 != mat.shape[1]:
        raise ValueError("fixed-block matrices shard on block boundaries only")
    j0, j1 = n0 // bs, -(-n1 // bs)
    return MTCMatrix((mat.shape[0], n1 - n0), bs, mat.arena, np.ascontiguousarray(mat.offsets[:, j0:j1]),
                     np.ascontiguousarray(mat.precisions[:, j0:j1]), np.ascontiguousarray(mat.scales[:, j0:j1]),
                     None, row_perm=mat.row_perm, col_perm=None)


class ShardedMTCMatrix:
    """One rank's part of a column-sharded GEMM: ``matmul(X)`` returns the full
    Y = X @ W (original column order) on every rank."""

    def __init__(self, mat: MTCMatrix, group=None, device=None):
        import torch
        import torch.distributed as dist

        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = torch.device(device if device is not None else "cuda")
        self.plan = plan_shards(mat, self.world)
        self.local = local_shard(mat, self.plan, self.rank)
        self.N = mat.shape[1]
        self.stream = self.local.device_stream(self.device)
        self.pos = torch.from_numpy(self.plan.pos).to(self.device)
        self._buf = {}
        self.side = torch.cuda.Stream(self.device)
        self.pipeline_min_rows = 1024
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        self.limit_sms = max(2, sms - 16)  # 16 SMs left to the exchange while the prefill runs
        # "nccl": one all-gather per chunk (default); "copy": slices pushed
        # into the peers' symmetric-memory buffers by the copy engines
        self.transport = "nccl"
        self._calls = 0

    def _peer_buffers(self, M: int, idx: int):
        """[world][M][wmax] gather buffer in symmetric memory (every rank's
        slice lands in every rank's buffer) and the peers' views of it.  Calls
        alternate between two such buffers: a rank may push the next call's
        slices while a slower peer still assembles this call's."""
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        key = ("peer", M, idx)
        if key not in self._buf:
            wmax = self.plan.wmax
            buf = symm.empty(self.world, M, wmax, dtype=torch.float32, device=self.device)
            hdl = symm.rendezvous(buf, self.group if self.group is not None else dist.group.WORLD)
            peers = [buf if r == self.rank else hdl.get_buffer(r, (self.world, M, wmax), torch.float32)
                     for r in range(self.world)]
            self._buf[key] = (buf, peers, hdl, torch.zeros(1, dtype=torch.float32, device=self.device))
        return self._buf[key]

    def matmul(self, X, Y: Optional["torch.Tensor"] = None):
        import torch
        import torch.distributed as dist

        from . import _lib

        M = X.shape[0]
        w, wmax = self.local.shape[1], self.plan.wmax
        if Y is None:
            Y = torch.empty(M, self.N, dtype=torch.float32, device=self.device)
        lib = _lib.load()
        # Large M on several GPUs: two row chunks, the second chunk's GEMM
        # overlapping the first chunk's exchange and assembly on a side
        # stream.  The prefill then leaves 16 SMs to the exchange.
        chunks = [(0, M)]
        if self.world > 1 and M >= self.pipeline_min_rows:
            h = (M // 2 + 511) // 512 * 512
            chunks = [(0, h), (h, M)] if h < M else [(0, M)]
        peer = None
        if self.world > 1 and self.transport == "copy":
            try:
                peer = self._peer_buffers(M, self._calls & 1)
            except Exception:  # no symmetric memory here: exchange through NCCL instead
                self.transport = "nccl"
        if peer is None:
            key = (M, len(chunks))
            if key not in self._buf:
                self._buf[key] = (torch.zeros(M, wmax, dtype=torch.float32, device=self.device),
                                  [torch.empty(self.world, r1 - r0, wmax, dtype=torch.float32, device=self.device)
                                   for r0, r1 in chunks])
            part, gathered = self._buf[key]
        else:
            gbuf, peers, _, token = peer
            part = gbuf[self.rank]
        self._calls += 1
        main = torch.cuda.current_stream(self.device)
        self.stream.desc.max_sms = self.limit_sms if len(chunks) > 1 else 0
        for c, (r0, r1) in enumerate(chunks):
            self.stream.matmul(X[r0:r1], part[r0:r1, :w])
            done = torch.cuda.Event()
            done.record(main)
            side = self.side if (len(chunks) > 1 or peer is not None) else main
            rows = r1 - r0
            with torch.cuda.stream(side):
                side.wait_event(done)
                if self.world == 1:
                    src, seg_stride = part[r0:r1], rows * wmax
                elif peer is None:
                    work = dist.all_gather_into_tensor(gathered[c], part[r0:r1], group=self.group, async_op=True)
                    work.wait()
                    src, seg_stride = gathered[c], rows * wmax
                else:
                    # this rank's rows go straight into every peer's buffer
                    # (copy engines over NVLink, no SMs); a one-element
                    # all-reduce after the copies tells every rank that all
                    # slices of the chunk have landed in its own buffer
                    nbytes = rows * wmax * 4
                    for r in range(self.world):
                        if r != self.rank:
                            _lib.check(lib.mtc_copy_async(peers[r][self.rank, r0].data_ptr(),
                                                          part[r0].data_ptr(), nbytes, side.cuda_stream),
                                       "shard exchange")
                    work = dist.all_reduce(token, group=self.group, async_op=True)
                    work.wait()
                    src, seg_stride = gbuf[0, r0:], M * wmax
                _lib.check(lib.mtc_permute_rows(src.data_ptr(), seg_stride, wmax, self.world, wmax,
                                                self.pos.data_ptr(), self.N, rows, Y[r0:r1].data_ptr(), Y.stride(0),
                                                None, side.cuda_stream), "shard assembly")
        if side is not main:
            main.wait_stream(self.side)
        self.stream.desc.max_sms = 0
        return Y
