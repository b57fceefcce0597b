"""Column-sharded GEMM with the output replicated on every rank, on 2 GPUs.

Each rank runs as its own process on its own GPU (gloo carries only the IPC
handles). Checks: every rank's replica equals an unsharded GEMM on that GPU bit
for bit; and a rank that never runs its step makes the other rank's bounded
completion wait expire with MMR_ERR_TIMEOUT while its context stays usable.
Skipped with fewer than 2 GPUs.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, scenario, q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    result = "error"
    try:
        from momiru_b200 import BoundGemm, DeviceBuffer, DeviceView, Epilogue, MatMulNode, rng
        from momiru_b200 import _abi, execution
        from momiru_b200.sharding import ReplicatedColumnGemm
        if scenario == "replicate_split":
            result = _replicate_split(rank, world)
            return
        m, k, n = 1000, 512, 1536 if scenario == "replicate" else 512
        a = rng.randu((m, k), 1)
        b = rng.randu((k, n), 2)
        bias = rng.randn((n,), 3, 0.1)
        node = MatMulNode(epilogue=Epilogue.BIAS_RELU)
        A, B, BIAS = DeviceView.from_host(a, rank), DeviceView.from_host(b, rank), DeviceView.from_host(bias, rank)
        out_t = torch.full((m, n), 7.0, dtype=torch.float32, device=f"cuda:{rank}")
        C = DeviceView.contiguous(DeviceBuffer.from_torch(out_t), (m, n))
        g = ReplicatedColumnGemm(node, A, B, C, BIAS, stream=torch.cuda.current_stream().cuda_stream)
        if scenario == "replicate":
            for _ in range(2):
                g.replay()
            g.quiesce_or_abort(30)
            dist.barrier()
            ref = DeviceView.empty((m, n), rank)
            with BoundGemm(node, A, B, ref, BIAS) as single:
                single.replay()
                single.quiesce_or_abort(30)
            same = np.array_equal(out_t.cpu().numpy().view(np.uint32), ref.to_host().view(np.uint32))
            result = "ok" if same else "mismatch"
        else:  # rank 1 never runs its step: rank 0's handshake must time out
            if rank == 0:
                g.replay()
                try:
                    g.quiesce_or_abort(30)
                    result = "no-timeout"
                except execution.QuiescenceTimeout:
                    # the context is still usable
                    x = DeviceView.from_host(np.eye(8, dtype=np.float32), rank)
                    y = execution.matmul(x, x, node=MatMulNode(math_mode=execution.KernelMathMode.Exact,
                                                               accuracy=execution.AccuracyContract.Exact))
                    result = "timeout" if np.array_equal(y.to_host(), np.eye(8, dtype=np.float32)) else "broken"
            else:
                result = "idle"
            dist.barrier()  # rank 1 keeps its replica mapped until rank 0 is done
        g.close()
    finally:
        q.put((rank, result))
        dist.destroy_process_group()


def _replicate_split(rank, world):
    """4096 x 2555 output, K = 640, 3xTF32 + bias + ReLU: each rank's column
    block has 80 tiles of 256 x 256, more than there are CTA pairs, so its
    tiles are split by k-blocks across pairs, and the ragged last columns go
    through the replica copy one by one. Checks: both replicas hold the same
    bytes, sampled rows match the oracle, and the padding columns of the
    replicas are untouched."""
    import hashlib

    import torch
    import torch.distributed as dist

    from momiru_b200 import DeviceBuffer, DeviceView, Epilogue, MatMulNode, rng
    from momiru_b200.sharding import ReplicatedColumnGemm
    from oracle import oracle as O
    m, k, n, n_phys = 4096, 640, 2555, 2560
    a = rng.randu((m, k), 31)
    b = rng.randu((k, n), 32)
    bias = rng.randn((n,), 33, 0.1)
    node = MatMulNode(epilogue=Epilogue.BIAS_RELU)
    b_phys = np.zeros((k, n_phys), np.float32)  # rows padded to 16 bytes
    b_phys[:, :n] = b
    A, BIAS = DeviceView.from_host(a, rank), DeviceView.from_host(bias, rank)
    B = DeviceView.from_host(b_phys, rank).narrow(1, 0, n)
    out_t = torch.full((m, n_phys), 7.0, dtype=torch.float32, device=f"cuda:{rank}")
    C = DeviceView.contiguous(DeviceBuffer.from_torch(out_t), (m, n_phys)).narrow(1, 0, n)
    g = ReplicatedColumnGemm(node, A, B, C, BIAS, stream=torch.cuda.current_stream().cuda_stream)
    for _ in range(3):
        g.replay()
    g.quiesce_or_abort(30)
    host = out_t.cpu().numpy()
    digest = hashlib.sha256(host.tobytes()).hexdigest()
    everyone = [None] * world
    dist.all_gather_object(everyone, digest)
    rows = np.random.default_rng(5).choice(m, 64, replace=False)
    ref = O.matmul(a, b, bias=bias, epilogue=O.EPI_BIAS_RELU, rows=rows)
    got = host[rows, :n].astype(np.float64)
    err = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    if len(set(everyone)) != 1:
        result = "replicas differ"
    elif not np.all(host[:, n:] == 7.0):
        result = "padding written"
    elif not err <= 1e-5:
        result = f"error {err:.3g}"
    else:
        result = "ok"
    dist.barrier()  # each rank keeps its replica mapped until both have checked
    g.close()
    return result


def _run(scenario):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, scenario, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    return res


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_replicated_column_shards_match_single_gpu():
    assert _run("replicate") == {0: "ok", 1: "ok"}


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_replicated_split_tiles_and_ragged_columns():
    assert _run("replicate_split") == {0: "ok", 1: "ok"}


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_missing_rank_times_out_with_context_usable():
    assert _run("missing") == {0: "timeout", 1: "idle"}
