"""The GEMM whose epilogue delivers its column shard into several gathered outputs
(mxfp6_gemm_gather): the building block of the fused all-gather of column-parallel shards.

On one GPU: two local destinations of pitch 2N, at column 0 or N, on every route and output
type; each must hold exactly the plain GEMM's D in its column range and keep its poison
elsewhere. A D assembled block by block from one-destination calls matches the oracle. Two
ranks (processes), on two GPUs (skipped with fewer) and both on one GPU: each rank writes its
shard into its own and its peer's gathered output through a CUDA IPC mapping; both ranks must
end with [D_0 | D_1]."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
TORCH_OUT = {0: torch.float32, 1: torch.float16, 2: torch.bfloat16}


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()


def _bits(t):
    return t.view(torch.int32) if t.element_size() == 4 else t.view(torch.int16)


# shapes routed to 128x128, 128x128 split 16, 128x256, the 256x256 pair, the pair split 8, and
# the pair with a stream-K tail
@pytest.mark.parametrize("ot", ["F32", "F16", "BF16"])
@pytest.mark.parametrize("M,N,K", [(640, 768, 1408), (256, 384, 32768), (2048, 2048, 1024), (2048, 2048, 2048),
                                   (1024, 512, 24576), (2304, 2560, 1024)])
@pytest.mark.parametrize("col0_blocks", [0, 1])
def test_two_local_destinations(lib, ot, M, N, K, col0_blocks):
    from gpu_helpers import DeviceOperands, run_gemm
    from mxfp6_b200.synth import make_operands
    ops = make_operands(M, N, K, kind="codes", seed=M + N + K)
    dev = DeviceOperands(ops)
    o = lib.OutType[ot]
    routed = run_gemm(dev, o)
    ldd, col0 = 2 * N, col0_blocks * N
    poison = 0x5A5A if o != lib.OutType.F32 else 0x5A5A5A5A
    outs = [torch.empty((M, ldd), dtype=TORCH_OUT[int(o)], device="cuda") for _ in range(2)]
    for t in outs:
        _bits(t).fill_(poison)
    wsb = lib.gemm_workspace_size(M, N, ops.Kp, o)
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device="cuda") if wsb else None
    lib.gemm_gather(o, M, N, ops.Kp, dev.A, dev.Bt, dev.sA, dev.sB, outs, ldd, col0, ops.row_bytes,
                    ops.row_bytes, ws, wsb)
    assert lib.last_error() == lib.OK, lib.last_error_string()
    torch.cuda.synchronize()
    assert lib.device_status() == 0
    for t in outs:
        t = t.cpu()
        assert torch.equal(_bits(t[:, col0:col0 + N].contiguous()), _bits(routed))
        other = t[:, N:] if col0 == 0 else t[:, :N]
        assert bool((_bits(other.contiguous()) == poison).all())


@pytest.mark.parametrize("M,N,K", [(512, 768, 1408), (2048, 2048, 2048), (1024, 512, 24576)])
def test_eight_local_destinations(lib, M, N, K):
    """The largest destination list (8): every destination holds exactly the plain GEMM's D, on
    the single-CTA, pair and split routes (the regrouping epilogue and the reduce pass)."""
    from gpu_helpers import DeviceOperands, run_gemm
    from mxfp6_b200.synth import make_operands
    ops = make_operands(M, N, K, kind="codes", seed=M + 3 * N + K)
    dev = DeviceOperands(ops)
    o = lib.OutType.BF16
    routed = run_gemm(dev, o)
    outs = [torch.full((M, N), 7.0, dtype=torch.bfloat16, device="cuda") for _ in range(8)]
    wsb = lib.gemm_workspace_size(M, N, ops.Kp, o)
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device="cuda") if wsb else None
    lib.gemm_gather(o, M, N, ops.Kp, dev.A, dev.Bt, dev.sA, dev.sB, outs, N, 0, ops.row_bytes, ops.row_bytes,
                    ws, wsb)
    assert lib.last_error() == lib.OK, lib.last_error_string()
    torch.cuda.synchronize()
    assert lib.device_status() == 0
    for t in outs:
        assert torch.equal(_bits(t.cpu()), _bits(routed))


@pytest.mark.parametrize("ot", ["F16", "BF16"])
def test_blocks_assembled_into_one_output(lib, oracle, ot):
    """The end-to-end pipeline's building block: D assembled from row chunks of A and row chunks
    of B^T (with their scale atoms), each block written by a one-destination gather call at its
    column offset of D; every block holds the oracle's values (its own route may split K)."""
    from gpu_helpers import DeviceOperands, check
    from mxfp6_b200.synth import make_operands
    M, N, K, ra, rc = 1024, 1024, 2048, 2, 4
    ops = make_operands(M, N, K, kind="codes", seed=77, exp_range=(116, 128))
    dev = DeviceOperands(ops)
    o = lib.OutType[ot]
    mc, nc = M // ra, N // rc
    sa_chunk = (mc // 128) * (ops.Kp // 128) * 512
    sb_chunk = (nc // 128) * (ops.Kp // 128) * 512
    D = torch.empty((M, N), dtype=TORCH_OUT[int(o)], device="cuda")
    _bits(D).fill_(0x5A5A)
    wsb = lib.gemm_workspace_size(mc, nc, ops.Kp, o)
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device="cuda") if wsb else None
    for i in range(ra):
        for j in range(rc):
            lib.gemm_gather(o, mc, nc, ops.Kp, dev.A[i * mc:], dev.Bt[j * nc:], dev.sA[i * sa_chunk:],
                            dev.sB[j * sb_chunk:], [D[i * mc:].data_ptr()], N, j * nc, ops.row_bytes, ops.row_bytes,
                            ws, wsb)
            assert lib.last_error() == lib.OK, lib.last_error_string()
    torch.cuda.synchronize()
    assert lib.device_status() == 0
    ref = oracle.gemm(ops.A, ops.sA, ops.Bt, ops.sB, ops.Kp)
    check(D.cpu(), ref, o, oracle, label=f"blocks {ra}x{rc} {ot}")


def _rank_main(rank, world, port, out_q, device=None, shape=(512, 768, 1920)):
    """One rank of the two-rank gather test (spawned process), on GPU `device` (default: its rank)."""
    try:
        sys.path.insert(0, os.path.join(os.path.dirname(HERE), "mxfp6-gemm_b200"))
        sys.path.insert(0, HERE)
        import torch.distributed as dist
        from datetime import timedelta
        import mxfp6_b200 as lib
        from mxfp6_b200.synth import make_operands
        from gpu_helpers import DeviceOperands, run_gemm
        torch.cuda.set_device(rank if device is None else device)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60))
        M, N, K = shape
        a = make_operands(M, 128, K, kind="codes", seed=11)
        b = make_operands(128, N, K, kind="codes", seed=20 + rank)
        from mxfp6_b200.synth import Operands
        ops = Operands(M, N, K, a.Kp, a.A, a.sA, b.Bt, b.sB)
        dev = DeviceOperands(ops)
        o = lib.OutType.BF16
        mine = run_gemm(dev, o)  # this rank's shard, plain GEMM
        gathered = torch.zeros((M, world * N), dtype=torch.bfloat16, device="cuda")
        h, off = lib.ipc_export(gathered)
        handles = [None] * world
        dist.all_gather_object(handles, (h, off))
        dsts, bases = [], []
        for r in range(world):
            if r == rank:
                dsts.append(gathered.data_ptr())
            else:
                base, ptr = lib.ipc_import(*handles[r])
                bases.append(base)
                dsts.append(ptr)
        dist.barrier()
        wsb = lib.gemm_workspace_size(M, N, ops.Kp, o)
        ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device="cuda")
        lib.gemm_gather(o, M, N, ops.Kp, dev.A, dev.Bt, dev.sA, dev.sB, dsts, world * N, rank * N, ops.row_bytes,
                        ops.row_bytes, ws, wsb)
        err = lib.last_error()
        torch.cuda.synchronize()
        status = lib.device_status()
        dist.barrier()  # every rank's stores into its peers have completed
        shards = [None] * world
        dist.all_gather_object(shards, mine.view(torch.int16).numpy())
        got = gathered.cpu().view(torch.int16).numpy()
        want = np.concatenate(shards, axis=1)
        ok = err == 0 and status == 0 and np.array_equal(got, want)
        dist.barrier()
        for base in bases:
            lib.ipc_close(base)
        dist.barrier()
        dist.destroy_process_group()
        out_q.put((rank, ok, f"err={err} status={status}"))
    except Exception as e:  # reported to the parent, never left hanging
        out_q.put((rank, False, repr(e)))


def _run_two_ranks(device=None, shape=(512, 768, 1920)):
    import socket
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q, device, shape)) for r in range(2)]
    for p in procs:
        p.start()
    results = []
    for _ in range(2):
        results.append(q.get(timeout=300))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert all(ok for _, ok, _ in results), results


def test_two_gpu_gather_over_ipc():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    _run_two_ranks()


@pytest.mark.parametrize("shape", [(512, 768, 1920), (4096, 3584, 1024)])
def test_two_process_gather_over_ipc_on_one_gpu(shape):
    """The same two-rank exchange with both ranks' processes on GPU 0: each maps the other's
    gathered output through CUDA IPC and the GEMM's epilogue stores into it, so the IPC-mapped
    destination path runs even where only one GPU is available. No kernel waits on the other
    rank (the host barrier orders them), so sharing the GPU is safe. Shapes on the 128 x 128
    route and on the CTA pair with a cut last wave."""
    _run_two_ranks(device=0, shape=shape)
