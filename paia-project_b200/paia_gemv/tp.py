"""Row-sharded tensor-parallel batch-1 GEMV (e.g. Llama-3.1-8B lm_head and gate_up over 2/4/8 GPUs).

W [N, K] is split into `world` contiguous row blocks of N / world rows; rank r holds rows [r N/world, (r+1) N/world)
with their scales / zeros / bias, and x is replicated. Two ways to assemble y [N] on every rank:

* `ShardedGemv.fused(x)`: one kernel per rank (paia_gemv_tp) whose epilogue stores each output straight into every
  rank's y over NVLink (peer pointers: CUDA IPC handles of the library's own allocations, exchanged through
  torch.distributed and mapped with paia_gemv_ipc_open). The ranks count in each other's counter blocks the calls
  they have started and the CTAs that have finished storing, per source rank; a CTA stores into a rank's y only once
  that rank has started the same call, and CTA 0 waits until every rank's CTAs are done, so y is complete on this
  rank when the launch ends (no second launch; the counts live in device memory, so captured CUDA graphs stay
  correct). Counts only grow: after call e, every per-source arrival count is e * ctas.
* `ShardedGemv.nccl(x)`: the baseline, the same kernel writing the local slice, then `all_gather_into_tensor`.

`shard_rows` and `assemble` hold the partitioning rule shared by both and by the CPU tests. One process per GPU,
`torch.distributed` for the plumbing (NCCL on GPUs, gloo in the CPU tests).
"""
import ctypes


def shard_rows(N, world, rank):
    """Rows [r0, r1) of rank `rank`: equal contiguous blocks (N must divide evenly: every rank launches the same grid,
    so each call adds the same count to every arrival counter)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if N % world:
        raise ValueError(f"N = {N} rows do not split evenly over {world} ranks")
    n = N // world
    return rank * n, (rank + 1) * n


def assemble(slices):
    """y from the per-rank slices, rank-major (what both the fused stores and all_gather produce)."""
    import numpy as np
    return np.concatenate([np.asarray(s) for s in slices])


class _CudaArray:
    """A raw device allocation seen by torch through __cuda_array_interface__ (no copy, no ownership)."""

    def __init__(self, ptr, n, typestr):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 3,
                                         "strides": None}


def _device_view(ptr, n, typestr, device):
    import torch
    return torch.as_tensor(_CudaArray(ptr, n, typestr), device=device)


# Counter block of one rank (uint32 words; kTpEpoch / kTpReaders / kTpComplete / kTpArrive / kTpReady in the kernel):
# calls completed here, CTAs here that have read the call count, complete-form calls, CTAs of each source rank done
# storing here (complete form), calls each source rank has started.
COUNTER_WORDS, EPOCH, READERS, COMPLETE, ARRIVE, READY = 32, 0, 4, 5, 8, 16


def expected_counts(epoch, world, ctas):
    """A rank's counter block after `epoch` completed complete-form calls (uint32, wraps): the epoch, ctas * epoch
    readers, ctas * epoch arrivals from every rank and epoch starts of every rank."""
    blk = [0] * COUNTER_WORDS
    blk[EPOCH] = epoch & 0xFFFFFFFF
    blk[READERS] = (epoch * ctas) & 0xFFFFFFFF
    blk[COMPLETE] = epoch & 0xFFFFFFFF
    for r in range(world):
        blk[ARRIVE + r] = (epoch * ctas) & 0xFFFFFFFF
        blk[READY + r] = epoch & 0xFFFFFFFF
    return blk


class TpBuffers:
    """Per-rank buffers of the fused path for a full output of N rows: this rank's full-size y and its
    [arrivals, epoch] counters (the library's own allocations, so their IPC handles name exactly these bytes), plus
    every peer's y and counters mapped into this process. Several ShardedGemv objects with the same N may share one
    set (their calls are stream-ordered on each rank and add the same count per call to every counter)."""

    def __init__(self, lib, N, device, group=None):
        import torch
        import torch.distributed as dist
        self.lib, self.N, self.group = lib, N, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("at most 8 ranks")
        self._y_mem = lib.tp_alloc(2 * N)
        self._f_mem = lib.tp_alloc(4 * COUNTER_WORDS)
        self.y = _device_view(self._y_mem, N, "<i2", device).view(torch.bfloat16)
        self.flag = _device_view(self._f_mem, COUNTER_WORDS, "<i4", device)
        torch.cuda.synchronize(device)
        mine = (lib.ipc_handle(self._y_mem), lib.ipc_handle(self._f_mem))
        gathered = [None] * self.world
        dist.all_gather_object(gathered, mine, group=group)
        self._opened = []
        y_ptrs, f_ptrs = [], []
        for r, (hy, hf) in enumerate(gathered):
            if r == self.rank:
                y_ptrs.append(self._y_mem)
                f_ptrs.append(self._f_mem)
            else:
                py, pf = lib.ipc_open(hy), lib.ipc_open(hf)
                self._opened += [py, pf]
                y_ptrs.append(py)
                f_ptrs.append(pf)
        P = ctypes.c_void_p
        self.y_ptrs = (P * self.world)(*y_ptrs)
        self.f_ptrs = (P * self.world)(*f_ptrs)
        dist.barrier(group=group)

    def reset(self):
        """Zero this rank's counters on every rank at once (collective): after a wait gave up (error 6 or 8) the counts
        are out of step."""
        import torch
        import torch.distributed as dist
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        self.flag.zero_()
        torch.cuda.synchronize()
        dist.barrier(group=self.group)

    def close(self):
        """Unmap the peers' buffers and free this rank's, once every rank is done with them."""
        import torch
        import torch.distributed as dist
        if self._y_mem is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for ptr in self._opened:
            self.lib.ipc_close(ptr)
        self._opened = []
        dist.barrier(group=self.group)
        for ptr in (self._y_mem, self._f_mem):
            self.lib.tp_free(ptr)
        self._y_mem = self._f_mem = None


class TpExchange:
    """The exchange block of every rank for deferred TP calls (paia_gemv_tp_deferred / paia_gemv_tp_exchange): this
    rank's block (the library's own allocation) and every peer's mapped in. `run()` publishes this rank's deferred
    stores and waits for every rank's; after it, the y of every deferred call issued before it is complete."""

    def __init__(self, lib, device, group=None):
        import torch
        import torch.distributed as dist
        self.lib, self.group = lib, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self._mem = lib.tp_alloc(4 * COUNTER_WORDS)
        self.flag = _device_view(self._mem, COUNTER_WORDS, "<i4", device)
        torch.cuda.synchronize(device)
        gathered = [None] * self.world
        dist.all_gather_object(gathered, lib.ipc_handle(self._mem), group=group)
        self._opened = []
        ptrs = []
        for r, h in enumerate(gathered):
            if r == self.rank:
                ptrs.append(self._mem)
            else:
                q = lib.ipc_open(h)
                self._opened.append(q)
                ptrs.append(q)
        self.ptrs = (ctypes.c_void_p * self.world)(*ptrs)
        dist.barrier(group=group)

    def run(self, stream=None):
        self.lib.tp_exchange(self.ptrs, self.world, self.rank, stream)

    def close(self):
        import torch
        import torch.distributed as dist
        if self._mem is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for q in self._opened:
            self.lib.ipc_close(q)
        self._opened = []
        dist.barrier(group=self.group)
        self.lib.tp_free(self._mem)
        self._mem = None


class ShardedGemv:
    """One rank's shard of a row-sharded GEMV. `Wq`, `s`, `z`, `bias` are this rank's rows (device tensors, formats as
    the per-format C-ABI calls); `N` is the full row count. `buffers`: a TpBuffers for N to share (else its own)."""

    # the TMA-fed instance paia_gemv_tp launches (same decode, same geometry, so the same bits per row)
    TMA_MATH = {"bf16": 5, "fp8": 8, "int4": 7, "int4_asym": 7}

    def __init__(self, lib, kind, Wq, s, z, bias, N, K, group=None, buffers=None):
        import torch
        import torch.distributed as dist
        self.lib, self.kind, self.N, self.K = lib, kind, N, K
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        r0, r1 = shard_rows(N, self.world, self.rank)
        self.N_local = r1 - r0
        if Wq.shape[0] != self.N_local:
            raise ValueError(f"rank {self.rank}: shard has {Wq.shape[0]} rows, expected {self.N_local}")
        self.Wq, self.s, self.z, self.bias = Wq, s, z, bias
        dev = Wq.device
        self._own = buffers is None
        self.buf = buffers if buffers is not None else TpBuffers(lib, N, dev, group)
        if self.buf.N != N:
            raise ValueError("shared TpBuffers were made for another N")
        self.y, self.flag = self.buf.y, self.buf.flag
        self.y_nccl = torch.empty(N, dtype=torch.bfloat16, device=dev)
        self.y_local = torch.empty(self.N_local, dtype=torch.bfloat16, device=dev)
        self.ctas = lib.tp_ctas(kind, self.N_local, K)

    def _ptrs(self):
        p = lambda t: t.data_ptr() if t is not None else None       # noqa: E731
        return p(self.Wq), p(self.s), p(self.z), p(self.bias)

    def deferred(self, x, stream=None):
        """The deferred form: this rank's outputs go into every rank's y, complete only after the next
        TpExchange.run() on every rank (at most one deferred call per buffer set between two exchanges)."""
        W, s, z, b = self._ptrs()
        self.lib.tp_deferred(self.kind, W, s, z, x.data_ptr(), b, self.buf.y_ptrs, self.buf.f_ptrs, self.world,
                             self.rank, self.N_local, self.K, stream)
        return self.y

    def fused(self, x, stream=None):
        """y on every rank through the peer-store epilogue; returns this rank's full y, complete in stream order once
        the launch ends. The same buffer serves every call: the next call's peer stores wait until this rank has
        started that call, so readers of y earlier in this rank's stream are safe."""
        W, s, z, b = self._ptrs()
        self.lib.tp(self.kind, W, s, z, x.data_ptr(), b, self.buf.y_ptrs, self.buf.f_ptrs, self.world, self.rank,
                    self.N_local, self.K, stream)
        return self.y

    def local(self, x, y_local, stream=None):
        """This rank's slice alone, with the kernel the fused path uses (no peer stores)."""
        W, s, z, b = self._ptrs()
        self.lib.launch_ex(self.kind, 0, 2, 8, self.TMA_MATH[self.kind], 1, 0, 0, W, s, z, x.data_ptr(), b,
                           y_local.data_ptr(), self.N_local, self.K, stream)

    def nccl(self, x, stream=None):
        """Baseline: the local slice, then NCCL all_gather_into_tensor on the same stream."""
        import torch.distributed as dist
        self.local(x, self.y_local, stream)
        dist.all_gather_into_tensor(self.y_nccl, self.y_local, group=self.group)
        return self.y_nccl

    def close(self):
        if self._own:
            self.buf.close()
