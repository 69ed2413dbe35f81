// Host-side launch machinery shared by the per-format translation units: variant tables, grid sizing, the K-split
// choice and the (optionally programmatic) launch. No allocation, no synchronisation, graph-capturable.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "gemv_kernel.cuh"

namespace pb2 {

using KernelFn = void (*)(const Params);

// One variant: the reference's (R, U, W, S, H) tuple and the kernel instance it maps to on B200.
//   R  rows per warp row-slot            U  16-byte steps per row in flight (x2 with double buffering)
//   W  warps per CTA                     S  BF16 only: 1 = mixed-precision bf16 FMA, 0 = fp32 conversion + FFMA
//   H  1 = launch with programmatic dependent launch (PDL) and leave room on each SM for the next kernel
struct Variant {
    int R, U, W, S, H;
    int math;                 // kernel family and dequantisation path (0/1 CUDA cores, 2-4 mma from registers,
                              // 5-7 TMA-fed mma; see gemv_kernel.cuh, gemv_mma.cuh, gemv_tma.cuh)
    KernelFn fn;
    size_t (*smem)(int K);    // dynamic shared memory bytes for a given K (kernels without a prep step)
    // TMA kernels: fills the stage geometry of p for the device's shared-memory capacity and returns the dynamic
    // shared memory bytes (0 if the shape cannot be staged); threads per CTA are (W + 1) * 32 (a producer warp).
    size_t (*prep)(Params& p, size_t cap);
};

// Launch-time knobs beyond the tuple (the _ex entry points); zero means "choose automatically".
struct LaunchOpts {
    int ks;                   // warps per row (power of two dividing W), 0 = auto
    int ctas_per_sm;          // 0 = auto (all resident CTAs)
    int ring = 0;             // TMA kernels: ring stages (0 = as many as fit, else 2..16)
    int share = 0;            // TMA kernels: size the CTA for 1/share of the SM's shared memory (0 = 1: all of it);
                              // share 2 with one CTA per SM leaves room for the next kernel's CTA under PDL
    int pre = 0;              // TMA kernels: 0 = auto; k in 1..254: k - 1 stages streamed before the producer waits
                              // for the consumers' x loads to be issued; 255: never wait (the whole ring first)
    int tensor_on = 0;        // TMA kernels: 1 = tiled tensor copies of full tiles (comparisons; slower, off by default)
};

int sm_count();                                              // current device, cached
int max_ctas_per_sm(KernelFn fn, int threads, size_t smem);  // occupancy, cached; 0 if it cannot launch
size_t sm_smem_bytes();                                      // shared memory per SM, less one CTA's reservation
size_t max_dyn_smem();                                       // opt-in shared memory per block, current device

inline int ilog2(int v) { int l = 0; while ((1 << (l + 1)) <= v) ++l; return l; }

// Warps per row: enough that every warp still has >= U steps of its row (K-split for long rows), and enough that the
// CTA's row slots are not left idle when a CTA owns few rows, but never more warps than 512-byte steps in a row.
inline int choose_ks(int nchunk, int rows_per_cta, int W, int R, int U) {
    const int steps = (nchunk + 31) / 32;
    int ks_k = 1;
    while (ks_k * 2 <= W && steps >= ks_k * 2 * U) ks_k *= 2;
    const int slots = (rows_per_cta + R - 1) / R;
    int nr = 1;
    while (nr * 2 <= W && nr * 2 <= slots) nr *= 2;
    const int ks_r = W / nr;
    int ks = ks_k > ks_r ? ks_k : ks_r;
    int cap = 1;
    while (cap * 2 <= W && cap * 2 <= steps) cap *= 2;
    return ks < cap ? ks : cap;
}

// A launch with its geometry fixed: the kernel's Params (stage geometry filled in), grid, block and shared memory.
struct Planned {
    Params p;
    size_t smem;
    long long G;
    int threads;
    bool pdl;
};

// Geometry of a launch of v on the current device: returns 0 and fills `out`, or -2 when the shape cannot run.
inline int plan_variant(const Variant& v, const Params& p_in, const LaunchOpts& o, Planned* out) {
    Params p = p_in;
    size_t smem;
    if (v.prep) {
        const int share = o.share > 0 ? o.share : 1;
        if (share > 4) return -2;
        size_t cap = sm_smem_bytes() / share - (share > 1 ? 1024 : 0);
        if (cap > max_dyn_smem()) cap = max_dyn_smem();
        p.ring = o.ring;
        p.pre = o.pre == 0 ? kTmaPreAuto : (o.pre >= 255 ? -1 : o.pre - 1);
        p.tensor_on = o.tensor_on;
        smem = v.prep(p, cap);
    } else {
        smem = v.smem(p.K);
    }
    if (smem == 0 || smem > max_dyn_smem()) return -2;
    const int threads = (v.prep ? v.W + 2 : v.W) * 32;     // TMA kernels: + producer and epilogue warps
    const int occ = max_ctas_per_sm(v.fn, threads, smem);
    if (occ <= 0) return -2;
    // Full occupancy by default: under PDL the next kernel's CTAs take the SM slots that this grid's CTAs free at
    // its tail (measured better than leaving half of each SM to the next kernel from the start).
    int per_sm = o.ctas_per_sm > 0 ? o.ctas_per_sm : occ;
    if (per_sm > occ) per_sm = occ;
    long long G = (long long)sm_count() * per_sm;
    if (G > p.N) G = p.N;
    const int rows_per_cta = (int)((p.N + G - 1) / G);
    int ks = 1;                                               // the tensor-core kernels split work themselves
    if (v.math < 2) {
        ks = o.ks > 0 ? o.ks : choose_ks(p.nchunk, rows_per_cta, v.W, v.R, v.U);
        if (ks > v.W || (v.W % ks) != 0 || (ks & (ks - 1)) != 0) return -2;
    }
    p.ks_log2 = ilog2(ks);
    p.host_ops = nullptr;                                     // host memory: never part of what the kernel sees
    out->p = p;
    out->smem = smem;
    out->G = G;
    out->threads = threads;
    out->pdl = v.H != 0;
    return 0;
}

// Layer mode (p.nops > 0) launches cooperatively: CTAs wait for every CTA's outputs of the previous op, so all of
// them must be resident at once. Otherwise programmatic dependent launch when the variant asks for it.
inline int launch_planned(KernelFn fn, const Planned& pl, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)pl.G);
    cfg.blockDim = dim3((unsigned)pl.threads);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    if (pl.p.nops > 0) {
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    } else if (pl.pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    const cudaError_t e = cudaLaunchKernelEx(&cfg, fn, pl.p);
    if (e != cudaSuccess) { (void)cudaGetLastError(); return (int)e; }
    return 0;
}

// grid_out != nullptr: plan only (no launch) and return the grid size in *grid_out.
inline int launch_variant(const Variant& v, const Params& p, const LaunchOpts& o, cudaStream_t st,
                          long long* grid_out = nullptr) {
    Planned pl;
    const int rc = plan_variant(v, p, o, &pl);
    if (rc) return rc;
    if (grid_out) {
        *grid_out = pl.G;
        return 0;
    }
    return launch_planned(v.fn, pl, st);
}

template <int F, int NW, int R>
size_t smem_of(int K) { return smem_bytes<F, NW, R>(K); }

// Table accessors, one translation unit per format (compiled in parallel).
const Variant* table_bf16(int* n);
const Variant* table_fp8(int* n);
const Variant* table_int4(int* n);
const Variant* table_int4a(int* n);
// Extra kernel instances reachable only through paia_gemv_launch_ex (tuning): same tuple space, other math paths.
const Variant* find_instance(int fmt, int R, int U, int W, int math);
const Variant* mma_instances(int fmt, int math, int* n);
const Variant* tma_instances(int fmt, int math, int* n);
const Variant* tma_public(int fmt, int* n);                  // the TMA variants appended to each format's table
const Variant* tma_rope(int fmt, int math);                 // the rotary-epilogue instance of (format, math)
int tma_device_error(int clear);
int launch_tp_exchange(unsigned int* const* flag_all, int world, int rank, cudaStream_t st);

}  // namespace pb2
