"""Host logic of the row-sharded tensor-parallel GEMV without a GPU: the partitioning rule, the arrival-counter
arithmetic, reassembly order (two gloo ranks computing their shards with the CPU oracle and all-gathering them must
give the full oracle, bit for bit), and failure propagation (a rank that dies before the exchange makes the other
rank's collective fail with an error instead of hanging)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from paia_gemv import tp


def test_shard_rows_cover_every_row_once():
    for N, world in ((128256, 8), (28672, 8), (28672, 4), (4096, 2), (16, 1)):
        seen = np.zeros(N, dtype=np.int32)
        last = 0
        for r in range(world):
            r0, r1 = tp.shard_rows(N, world, r)
            assert r0 == last and r1 - r0 == N // world
            seen[r0:r1] += 1
            last = r1
        assert last == N and np.all(seen == 1)
    with pytest.raises(ValueError):
        tp.shard_rows(1000, 3, 0)
    with pytest.raises(ValueError):
        tp.shard_rows(1024, 2, 2)


def test_expected_counts_wrap():
    """Per-source counts after e calls: e starts and e * ctas arrivals from every rank, uint32 wrapping; the device
    waits compare wrap-safely ((int32)(count - target) >= 0), so one call's step stays positive past the wrap."""
    blk = tp.expected_counts(1, 8, 148)
    assert blk[tp.EPOCH] == 1 and blk[tp.ARRIVE:tp.ARRIVE + 8] == [148] * 8 and blk[tp.READY:tp.READY + 8] == [1] * 8
    assert len(blk) == tp.COUNTER_WORDS and tp.ARRIVE + 8 <= tp.READY and tp.READY + 8 <= tp.COUNTER_WORDS
    e = 2 ** 32 // 148 + 3                              # past the uint32 wrap of the arrival counts
    v = tp.expected_counts(e, 8, 148)[tp.ARRIVE]
    assert v == (e * 148) % 2 ** 32
    prev = tp.expected_counts(e - 1, 8, 148)[tp.ARRIVE]
    assert np.int32(np.uint32(v) - np.uint32(prev)) == 148

def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _shard_worker(rank, world, port, kind, N, K, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(11)                    # same operands on every rank
    Wf = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    xb = O.f32_to_bf16(rng.standard_normal(K).astype(np.float32))
    r0, r1 = tp.shard_rows(N, world, rank)
    if kind == "fp8":
        q, sc = O.quantize_fp8_rowwise(Wf)
        yb, _ = O.gemv("fp8", xb, q=q[r0:r1], scale=sc[r0:r1])
    else:
        pk, sc, zr = O.quantize_int4_asym(Wf)
        yb, _ = O.gemv("int4_asym", xb, packed=pk[r0:r1], scales=sc[r0:r1], zeros=zr[r0:r1])
    mine = torch.from_numpy(yb.astype(np.int32))
    parts = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(parts, mine)
    if rank == 0:
        got = tp.assemble([p.numpy().astype(np.uint16) for p in parts])
        if kind == "fp8":
            want, _ = O.gemv("fp8", xb, q=q, scale=sc)
        else:
            want, _ = O.gemv("int4_asym", xb, packed=pk, scales=sc, zeros=zr)
        result.put(bool(np.array_equal(got, want)))
    dist.destroy_process_group()


@pytest.mark.parametrize("kind", ["fp8", "int4_asym"])
def test_two_gloo_ranks_reassemble_the_full_oracle(kind):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_shard_worker, args=(r, 2, port, kind, 96, 256, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert q.get(timeout=10) is True


def _failing_worker(rank, world, port, result):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(3)                                    # dies between steps, before the exchange
    try:
        t = torch.zeros(4)
        parts = [torch.empty(4) for _ in range(world)]
        dist.all_gather(parts, t)
        result.put("no error")
    except Exception as e:                             # noqa: BLE001 - any collective error is the expected outcome
        result.put("error: " + type(e).__name__)


def test_dead_rank_surfaces_as_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert procs[1].exitcode == 3
    msg = q.get(timeout=10)
    assert msg.startswith("error"), msg
