"""Row-sharded tensor parallelism on the GPU. One GPU: the TP kernel at world 1 equals the same TMA instance bit for
bit and counts its CTAs in; the bounded arrival wait gives up with an error status (a counter nothing increments)
and leaves the context usable. Two or more GPUs (skipped otherwise): two NCCL ranks, fused peer-store path and
NCCL all-gather baseline, both equal to the oracle and to each other bit for bit."""
import ctypes
import os
import socket

import numpy as np
import pytest
import torch

import oracle as O
from gpu_cases import bits, check, make

pytestmark = pytest.mark.gpu
TMA_MATH = {"bf16": 5, "fp8": 8, "int4": 7, "int4_asym": 7}


@pytest.fixture(scope="module")
def L():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from paia_gemv import load_lib
    return load_lib()


def _ptr(t):
    return None if t is None else t.data_ptr()


@pytest.mark.parametrize("kind", ["bf16", "fp8", "int4", "int4_asym"])
def test_tp_world1_matches_tma_instance(L, kind):
    N, K = 1000, 4096
    ops = make(kind, N, K, seed=21, with_bias=True)
    ref = torch.full((N,), float("nan"), dtype=torch.bfloat16, device="cuda")
    L.launch_ex(kind, 0, 2, 8, TMA_MATH[kind], 1, 0, 0, _ptr(ops.W), _ptr(ops.s), _ptr(ops.z), _ptr(ops.x),
                _ptr(ops.bias), ref.data_ptr(), N, K)
    y = torch.full((N,), float("nan"), dtype=torch.bfloat16, device="cuda")
    flag = torch.zeros(2, dtype=torch.int32, device="cuda")
    P = ctypes.c_void_p
    L.tp(kind, _ptr(ops.W), _ptr(ops.s), _ptr(ops.z), _ptr(ops.x), _ptr(ops.bias), (P * 1)(y.data_ptr()),
         (P * 1)(flag.data_ptr()), 1, 0, N, K)
    ctas = L.tp_ctas(kind, N, K)
    L.tp_wait(flag.data_ptr(), ctas)
    torch.cuda.synchronize()
    assert L.device_error(1) == 0
    assert flag.tolist() == [ctas, 1]
    assert np.array_equal(bits(y), bits(ref))
    check(ops, bits(y), ops.oracle(with_bias=True)[0], f"tp world 1 {kind}")


def test_tp_wait_gives_up_with_an_error_status(L):
    """A counter that nothing increments: the wait kernel returns after ~1 s, reports code 6, and the GPU keeps
    working (a GEMV right after it is still correct)."""
    L.device_error(1)
    flag = torch.zeros(2, dtype=torch.int32, device="cuda")
    L.tp_wait(flag.data_ptr(), 1)
    torch.cuda.synchronize()
    assert L.device_error(1) == 6
    ops = make("fp8", 300, 1024, seed=2)
    ops.nan_fill()
    ops.call(L, 0)
    torch.cuda.synchronize()
    check(ops, bits(ops.y), ops.oracle()[0], "fp8 after a timed-out wait")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _two_rank_worker(rank, world, port, kind, result):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from paia_gemv import load_lib, tp
    L = load_lib()
    N, K = 2048, 4096
    full = make(kind, N, K, seed=5)                    # same seed: identical operands on every rank
    r0, r1 = tp.shard_rows(N, world, rank)
    sl = lambda t: None if t is None else t[r0:r1].contiguous()   # noqa: E731
    g = tp.ShardedGemv(L, kind, sl(full.W), sl(full.s), sl(full.z), None, N, K)
    y_f = g.fused(full.x).clone()
    y_n = g.nccl(full.x).clone()
    y_f2 = g.fused(full.x).clone()                     # second epoch
    torch.cuda.synchronize()
    err = L.device_error(1)
    ok = err == 0 and np.array_equal(bits(y_f), bits(y_n)) and np.array_equal(bits(y_f2), bits(y_f))
    rel = None
    if ok and rank == 0:
        rel = O.rel_l2(bits(y_f), full.oracle()[0])     # bf16 bits against bf16 bits
        ok = rel <= 1e-3
    g.close()
    dist.destroy_process_group()
    result.put((rank, bool(ok), err, rel))


@pytest.mark.parametrize("kind", ["fp8", "int4_asym"])
def test_two_gpus_fused_equals_nccl_and_oracle(kind):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_rank_worker, args=(r, 2, port, kind, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(2))
    assert all(r[1] for r in res), res
