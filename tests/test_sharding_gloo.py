"""Column-sharded GEMM host logic on CPU ranks (gloo, world size 2).

Each rank packs the same MTC-QT-P matrix, takes its byte-balanced column
slice (tensorpack_b200.sharding), computes its slice of the permuted output
with the CPU oracle (standing in for the GPU kernel), all-gathers the slices
and assembles Y[:, pc] with the same position map the CUDA assembly kernel
uses.  The result must equal the unsharded product.
"""

import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, golden_dir, out_q):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, golden_dir)
    import torch
    import torch.distributed as dist

    import inputs
    from oracle import mtc_oracle as O
    from tensorpack_b200.kernels.gemm import MTCMatrix
    from tensorpack_b200.sharding import local_shard, plan_shards

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = np.load(os.path.join(golden_dir, "llm_like_256x512.npz"))
        W, _ = inputs.llm_like(256, 512, seed=1)
        sizes = tuple(int(s) for s in g["b4.25_inner_sizes"])
        inner = O.QuadtreeAllocation(sizes, {s: g[f"b4.25_inner_leaf_{s}"] for s in sizes},
                                     {s: g[f"b4.25_inner_modes_{s}"] for s in sizes},
                                     {s: g[f"b4.25_inner_scales_{s}"] for s in sizes}, None, 0)
        pr, pc = g["b4.25_row_perm"], g["b4.25_col_perm"]
        mat = MTCMatrix.from_qt_allocation(W, O.PermutedAllocation(inner, pr, pc, None, 0))
        plan = plan_shards(mat, world)
        shard = local_shard(mat, plan, rank)
        # slice of the stored matrix, rebuilt by the oracle from the shard's own leaves
        ls = shard.leaf_set
        Wp_slice = np.zeros(shard.shape, np.float32)
        for i in range(len(ls)):
            s, m = int(ls.size[i]), int(ls.mode[i])
            if m == 0:
                continue
            q = O.bitstream_unpack(shard.arena.raw_buffer, int(ls.offset[i]), s * s, m).reshape(s, s)
            Wp_slice[ls.row[i]:ls.row[i] + s, ls.col[i]:ls.col[i] + s] = q * np.float32(ls.scale[i])
        X = inputs.llm_activations(6, 256, seed=3, outlier_seed=1)
        part = np.zeros((6, plan.wmax), np.float64)
        part[:, :shard.shape[1]] = X[:, shard.row_perm].astype(np.float64) @ Wp_slice
        parts = [torch.zeros(6, plan.wmax, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(part))
        gathered = torch.stack(parts).numpy()                      # [world, M, wmax]
        rows = gathered.transpose(1, 0, 2).reshape(6, world * plan.wmax)
        Y = rows[:, plan.pos]                                       # the assembly kernel's formula
        ref = X.astype(np.float64) @ O.permuted_quadtree_dequant(W, pr, pc, inner.sizes, inner.leaf, inner.modes,
                                                                  inner.scales).astype(np.float64)
        err = float(np.abs(Y - ref).max() / np.abs(ref).max())
        widths = np.diff(plan.cuts)
        out_q.put((rank, err, list(plan.cuts), int(widths.min())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_column_sharded_gemm_on_gloo_ranks(golden_dir, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, golden_dir, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    res = sorted(q.get(timeout=10) for _ in range(world))
    for rank, err, cuts, wmin in res:
        assert err < 1e-12, (rank, err)
        assert cuts[0] == 0 and cuts[-1] == 512 and all(c % 32 == 0 for c in cuts)
        assert wmin > 0


def test_cuts_are_tile_aligned_and_byte_balanced(golden_dir):
    sys.path.insert(0, golden_dir)
    import inputs
    from oracle import mtc_oracle as O
    from tensorpack_b200.kernels.gemm import MTCMatrix
    from tensorpack_b200.sharding import column_cuts

    W, sizes, leaf, modes, scales = inputs.forced_mode_allocation(128, 1024, seed=2, p_split=0.5)
    mat = MTCMatrix.from_qt_allocation(W, O.QuadtreeAllocation(sizes, leaf, modes, scales, None, 0))
    ls = mat.leaf_set
    for world in (1, 2, 4, 8):
        cuts = column_cuts(mat, world)
        assert cuts[0] == 0 and cuts[-1] == 1024 and len(cuts) == world + 1
        assert all(c % 32 == 0 for c in cuts) and all(b > a for a, b in zip(cuts, cuts[1:]))
        load = [int(ls.payload_bytes[(ls.col >= a) & (ls.col < b)].sum()) for a, b in zip(cuts, cuts[1:])]
        assert max(load) <= 1.6 * (sum(load) / world) + 600, (world, load)
    with pytest.raises(ValueError):
        column_cuts(mat, 64)
