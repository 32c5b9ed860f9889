"""Column-sharded GEMM on two GPUs through the CUDA kernels and NCCL.

Each rank packs the same MTC-QT-P matrix, keeps its byte-balanced column
slice (tensorpack_b200.sharding), runs the decode (M <= 16) or prefill
kernel on it, all-gathers the permuted output slices over NCCL and assembles
Y[:, pc] with mtc_permute_rows; the exchange goes through NCCL or through
copy-engine copies into the peers' symmetric-memory buffers.  Every rank
must hold the full product:
within the GEMM tolerance of the oracle's fp64 product of the exact dequant.
The prefill result must also match the unsharded single-GPU result to
within the accumulation-order bound TOL_F16: each output tile sums the same
operands, but when the last wave of tiles is cut along K the cut depends on
the tile count, which differs between a slice and the whole matrix (the
decode splits K by the number of bands, so there too only the tolerance
applies).
Needs two GPUs; skipped otherwise.
"""

import datetime
import os
import socket
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, golden_dir, out_q, transport):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, golden_dir)
    import torch
    import torch.distributed as dist

    import inputs
    from oracle import mtc_oracle as O
    from tensorpack_b200.kernels.gemm import MTCMatrix
    from tensorpack_b200.sharding import ShardedMTCMatrix

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    res = []
    try:
        W, sizes, leaf, modes, scales = inputs.forced_mode_allocation(256, 1024, seed=11, p_split=0.4)
        rng = np.random.default_rng(5)
        pr, pc = rng.permutation(256), rng.permutation(1024)
        inner = O.QuadtreeAllocation(sizes, leaf, modes, scales, None, 0)
        mat = MTCMatrix.from_qt_allocation(W, O.PermutedAllocation(inner, pr, pc, None, 0))
        ref_w = O.permuted_quadtree_dequant(W, pr, pc, sizes, leaf, modes, scales).astype(np.float64)
        sh = ShardedMTCMatrix(mat, device=dev)
        sh.transport = transport
        full = mat.device_stream(dev)
        for M in (1, 16, 300, 1200):  # 1200: two row chunks, GEMM overlapping the first chunk's all-gather
            X = torch.from_numpy(inputs.llm_activations(M, 256, seed=M, outlier_seed=2)).to(dev)
            Y = sh.matmul(X)
            Y1 = torch.empty(M, 1024, dtype=torch.float32, device=dev)
            full.matmul(X, Y1)
            torch.cuda.synchronize(dev)
            sh.stream.check_status()
            full.check_status()
            ref = X.double().cpu().numpy() @ ref_w
            err = O.relative_frobenius_error(ref, Y.cpu().numpy())
            diff = float((Y.double() - Y1.double()).norm() / Y1.double().norm())
            res.append((M, err, diff))
        out_q.put((rank, res, list(sh.plan.cuts)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("transport", ["nccl", "copy"])
def test_sharded_gemm_on_two_gpus(golden_dir, transport):
    import torch
    import torch.multiprocessing as mp

    from test_gpu_parity import TOL_F16, TOL_REF

    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from tensorpack_b200 import build

    build.build()
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, golden_dir, q, transport)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    out = sorted(q.get(timeout=10) for _ in range(world))
    for rank, res, cuts in out:
        assert len(cuts) == world + 1 and cuts[0] == 0 and cuts[-1] == 1024
        for M, err, diff in res:
            assert err < TOL_REF, (rank, M, err)
            if M > 16:
                assert diff < TOL_F16, (rank, M, diff)
