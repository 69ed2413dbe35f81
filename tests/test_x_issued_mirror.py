"""Mirror of the x-first handshake of the TMA kernel (paia-project_b200/csrc/gemv_tma.cuh, gemv_mma.cuh x_blocks /
x_blocks_all): the producer streams `pre` stages and then waits on the x_ready mbarrier, whose count is every consumer
thread (NC x 32). Each consumer thread arrives exactly once per launch - from the staging pass's hook right after its
first round of x loads is issued, or at once when it has no block to load, or directly when the CTA has no rows of
op 0. One arrival too few leaves the producer waiting until its bounded wait gives up; one too many completes the
phase early. Checked on the CPU for every staging pass form, thread count and K the kernels take."""
import pytest

XR = 4                                    # blocks per thread per round in stage_x


def hook_calls_x_blocks(n, nthr, R=XR):
    """x_blocks_t: a thread with no block calls the hook up front; one with blocks after its first round's loads."""
    calls = [0] * nthr
    for tid in range(nthr):
        if tid >= n:
            calls[tid] += 1
        i0, r = tid, 0
        while i0 < n:
            if r == 0:
                calls[tid] += 1
            i0 += R * nthr
            r += 1
    return calls


def hook_calls_x_blocks_all(n, nthr, R=XR):
    """x_blocks_all_t: every thread runs every round (i0 from 0), hook after round 0; none when n <= 0 (then up front)."""
    calls = [0] * nthr
    for tid in range(nthr):
        if n <= 0:
            calls[tid] += 1
        i0, r = 0, 0
        while i0 < n:
            if r == 0:
                calls[tid] += 1
            i0 += R * nthr
            r += 1
    return calls


def first_pass(fmt, dec, K):
    """(form, blocks) of stage_x's first pass over x, the one that carries the hook: BF16 copies the padded blocks
    (Kp / 8) in one x_blocks pass; FP8 (every decode) and INT4 DEC 1 / DEC 2 take the max over the K / 8 real blocks
    with x_blocks; INT4 DEC 0 stages through x_blocks_all over K / 8 blocks."""
    if fmt == "bf16":
        kp = (K + 31) // 32 * 32
        return "blocks", kp // 8
    if fmt.startswith("int4") and dec == 0:
        return "all", K // 8
    return "blocks", K // 8


CASES = [("bf16", 0), ("fp8", 0), ("fp8", 1), ("fp8", 2), ("fp8", 3), ("int4", 0), ("int4", 1), ("int4", 2),
         ("int4_asym", 0), ("int4_asym", 1), ("int4_asym", 2)]
KS = [128, 256, 384, 1024, 2048, 3584, 4096, 8192, 14336, 18944, 32768, 54016]


@pytest.mark.parametrize("fmt,dec", CASES)
@pytest.mark.parametrize("nc", [4, 8, 16])
def test_every_consumer_thread_arrives_once(fmt, dec, nc):
    nthr = nc * 32
    for K in KS:
        if fmt.startswith("int4") and K % 128:
            continue
        form, n = first_pass(fmt, dec, K)
        calls = (hook_calls_x_blocks if form == "blocks" else hook_calls_x_blocks_all)(n, nthr)
        assert calls == [1] * nthr, (fmt, dec, nc, K, calls.count(0), calls.count(2))


@pytest.mark.parametrize("xm", [1, 2, 8])
def test_batched_rows_arrive_once(xm):
    """Batched x stages every x row with its own pass; the hook arrives only from row 0's pass."""
    nthr, K = 256, 4096
    total = [0] * nthr
    for m in range(xm):
        calls = hook_calls_x_blocks(K // 8, nthr)
        total = [t + (c if m == 0 else 0) for t, c in zip(total, calls)]
    assert total == [1] * nthr


def test_pre_never_waits_past_the_ring():
    """pre: LaunchOpts 0 -> kTmaPreAuto (1 stage), k in 1..254 -> k - 1, 255 -> never; the kernel waits only for
    0 <= pre < ring (a pre at or past the ring would wait on x while every slot is already full - it never waits)."""
    kTmaPreAuto = 1

    def params_pre(opt):
        return kTmaPreAuto if opt == 0 else (-1 if opt >= 255 else opt - 1)

    def kernel_pre(p, st):
        return p if 0 <= p < st else -1

    for st in range(2, 17):
        assert kernel_pre(params_pre(0), st) == 1
        assert kernel_pre(params_pre(255), st) == -1
        assert kernel_pre(params_pre(1), st) == 0
        for opt in range(1, 255):
            k = kernel_pre(params_pre(opt), st)
            assert k == -1 or 0 <= k < st
