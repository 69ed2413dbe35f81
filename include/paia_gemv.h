/*
 * paia_gemv.h: C ABI of libpaia_gemv.so, the B200 (sm_100a) batch-1 decode GEMV family.
 *
 * y[N] = dequant(W)[N,K] . x[K] (+ bias), bf16 activations and outputs, fp32 accumulation. Pointers are device
 * pointers; `stream` is a cudaStream_t (NULL = legacy default stream). Every entry point launches asynchronously on
 * `stream`, allocates nothing and never synchronises (exceptions are noted at their declarations).
 * Return codes: 0 ok, -1 bad variant, -2 bad shape or alignment, >0 the cudaError_t of the launch.
 *
 * The entry points marked REF replace the reference's (Bejaine/PAIA-Project) symbols of the same name with identical
 * signatures, argument checks and return codes, so its ctypes loader (src/paia_gemv/loader.py:28-99) and harness
 * adapters (paia-bench/bench/ops/ours_bf16.py, ours_quant.py) load this library through $PAIA_GEMV_LIB unchanged.
 *
 * Formats (byte-identical to the reference's, src/paia_gemv/quant_host.h:1-13):
 *   BF16        W bf16 [N][K] row-major (nn.Linear layout), K % 8 == 0, W/x/y 16-byte aligned.
 *   FP8 W8A16   Wq e4m3fn bytes [N][K], scale fp32 [N] (row amax / 448), K % 16 == 0, Wq/x 16 B, scale 4 B, y 2 B.
 *   INT4 W4A16  Wq uint8 [N][K/2] (byte j: weight 2j in the low nibble, 2j+1 in the high nibble, zero point 8),
 *               scales fp16 [N][K/128], K % 128 == 0, Wq/x 16 B, scales/y 2 B.
 *   INT4 asym   Wq as INT4 (a little-endian int32 [N][K/8] with nibble j at bits 4j holding k = 8i + j is the same
 *               bytes), scales and zeros bf16 [N][K/128] each, w = (q - 8) * scale + zero
 *               (paia-bench/bench/ops/lib_quant.py:159-167, :227-231).
 * Additional limit of the B200 kernels: x is staged in shared memory, so K <= 98304 (else -2).
 *
 * Weights, scales, zeros and bias are read before the kernel waits on its predecessor when the variant launches with
 * programmatic dependent launch (H = 1): they must not be written by the kernel immediately before on the same stream.
 * x and y are only touched after that wait.
 */
#ifndef PAIA_GEMV_H
#define PAIA_GEMV_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* REF src/paia_gemv/gemv_bf16.cu:37. Number of BF16 variants. */
int paia_gemv_bf16_variant_count(void);
/* REF src/paia_gemv/gemv_bf16.cu:40-44. (R, U, W, S, H) of variant v; -1 if out of range. */
int paia_gemv_bf16_variant_info(int v, int* R, int* U, int* W, int* S, int* H);
/* REF src/paia_gemv/gemv_bf16.cu:48-53. y[N] = W[N,K] x[K]. */
int paia_gemv_bf16(const void* W, const void* x, void* y, int N, int K, int variant, void* stream);

/* REF src/paia_gemv/gemv_quant.cu:61-62. */
int paia_gemv_fp8_variant_count(void);
int paia_gemv_fp8_variant_info(int v, int* R, int* U, int* W, int* H);
/* REF src/paia_gemv/gemv_quant.cu:64-68. y = scale[n] * sum_k e4m3(Wq[n,k]) x[k]. */
int paia_gemv_fp8(const void* Wq, const void* scale, const void* x, void* y, int N, int K, int variant, void* stream);

/* REF src/paia_gemv/gemv_quant.cu:70-71. */
int paia_gemv_int4_variant_count(void);
int paia_gemv_int4_variant_info(int v, int* R, int* U, int* W, int* H);
/* REF src/paia_gemv/gemv_quant.cu:73-77. Fused INT4 W4A16 g128 (symmetric, fp16 scale). */
int paia_gemv_int4(const void* Wq, const void* scales, const void* x, void* y, int N, int K, int variant, void* stream);
/* REF src/paia_gemv/gemv_quant.cu:80-85. Naive control kernel (same result, deliberately slow). */
int paia_gemv_int4_naive(const void* Wq, const void* scales, const void* x, void* y, int N, int K, void* stream);
/* REF src/paia_gemv/gemv_quant.cu:88-97. Unfused control: dequantise into scratch_bf16 (2*N*K bytes, 16-byte
 * aligned, caller-owned), then the default BF16 GEMV variant. */
int paia_gemv_int4_unfused(const void* Wq, const void* scales, const void* x, void* y, void* scratch_bf16, int N, int K,
                           void* stream);

/* No reference counterpart. paia_gemv_int4_unfused for callers that cannot hand the library a scratch buffer: a
 * serving engine whose memory pool owns the whole HBM budget, a plain C host with no device allocator of its own, or
 * a latency-critical loop where cudaMalloc / cudaFree would synchronise the device. The bf16 dequantised weights go
 * to a file-scope device array of 16 Mi elements (32 MiB, held by every GPU that loads the library until the process
 * exits), so the call allocates nothing. N * K above 16777216 (e.g. more than 4096 x 4096) returns -2; other checks
 * and codes as paia_gemv_int4_unfused (a >0 cudaError_t also when the array's address cannot be looked up). The
 * array keeps the last call's contents; each call overwrites the N * K elements it reads, so nothing needs clearing.
 * Calls that overlap on the GPU (two streams, or two host threads) share the array and race. The first call on each
 * device does a set-up step: it looks the array's address up with a runtime call and caches it, so make that first
 * call before any stream capture; the cached address does not survive a cudaDeviceReset. */
int paia_gemv_int4_unfused_static(const void* Wq, const void* scales, const void* x, void* y, int N, int K,
                                  void* stream);

/* ---- Row-sharded tensor parallelism (no reference kernel; the outputs of a row-partitioned GEMV gathered) ----
 * Rank `rank` of `world` (<= 8) holds rows [rank N_local, (rank+1) N_local) of W (and their scales/zeros/bias) and
 * computes them with the TMA-fed kernel, storing every output to every rank's full-size y (world * N_local bf16;
 * y_all[r] = rank r's buffer as mapped in this process, e.g. through CUDA IPC) at rank * N_local + row.
 * flag_all[r] = rank r's counter block: 32 zero-initialised uint32 in rank r's memory, 16-byte aligned (word 0: calls
 * completed on r; words 8 + s: CTAs of rank s done storing into r; words 16 + s: calls rank s has started). Each call
 * tells every rank that this rank has started it; each CTA stores into a rank's y only once that rank has started the
 * same call (so a rank's readers of the previous y, earlier in its stream, are done), then counts itself in on every
 * rank with system-scope atomics; CTA 0 waits until all CTAs of every rank have counted in, so this rank's y is
 * complete when the launch ends (no separate wait; captured CUDA graphs stay correct, the counts live in device
 * memory). Both waits give up after ~1 s with error code 8 (start) or 6 (arrivals) in paia_gemv_device_error();
 * after that, zero every rank's counter block before the next call. Same argument checks and codes as the per-format
 * calls; -2 also for a bad world/rank/pointer or a shape the TMA kernel cannot stage. paia_gemv_tp_ctas gives the
 * CTAs of one launch (the same on every rank). */
int paia_gemv_tp(int kind, const void* Wq, const void* scales, const void* zeros, const void* x, const void* bias,
                 void* const* y_all, unsigned int* const* flag_all, int world, int rank, int N_local, int K,
                 void* stream);
int paia_gemv_tp_ctas(int kind, int N_local, int K);
/* Deferred form, for sequences of TP GEMVs: the kernel only stores its outputs into every rank's y (after the same start
 * handshake), with no arrival counts and no wait, and y is complete only after the next paia_gemv_tp_exchange on every
 * rank (its CTAs count themselves in on word 4 of this rank's block once they have read the call count, error 9 if
 * they do not within ~1 s). Between two exchanges each buffer set (y_all, flag_all) takes at most one call: a second
 * would overwrite y before it is published. paia_gemv_tp_exchange
 * (one small kernel, launched in stream order after the calls it publishes): a system-scope fence makes every store of
 * this rank's earlier kernels visible, the rank counts itself in on every rank's exchange block (xflag_all[r]), and it
 * waits (bounded, ~1 s, error 6) until every rank has done the same; after it, every y written by deferred calls
 * before it is complete on this rank. */
int paia_gemv_tp_deferred(int kind, const void* Wq, const void* scales, const void* zeros, const void* x,
                          const void* bias, void* const* y_all, unsigned int* const* flag_all, int world, int rank,
                          int N_local, int K, void* stream);
int paia_gemv_tp_exchange(unsigned int* const* xflag_all, int world, int rank, void* stream);
/* Setup of the buffers other ranks map: a zero-filled device allocation (cudaMalloc), its 64-byte CUDA IPC handle,
 * and the mapping of a peer's handle in this process (usable from kernels on the current device; peer access is
 * enabled lazily). Codes: 0, -2 bad argument, >0 cudaError_t. Not for use inside a captured stream. */
int paia_gemv_tp_alloc(size_t bytes, void** ptr);
int paia_gemv_tp_free(void* ptr);
int paia_gemv_ipc_handle(const void* ptr, void* handle64);
int paia_gemv_ipc_open(const void* handle64, void** ptr);
int paia_gemv_ipc_close(void* ptr);

/* ---- B200 additions (no reference kernel) ---- */

/* Library identification string. */
const char* paia_gemv_version(void);

/* Asymmetric INT4 g128 (replaces the tinygemm call of paia-bench/bench/ops/lib_quant.py:221 for this format, with
 * this repo's packing). It shares the INT4 variant tuples. */
int paia_gemv_int4_asym_variant_count(void);
int paia_gemv_int4_asym_variant_info(int v, int* R, int* U, int* W, int* H);
int paia_gemv_int4_asym(const void* Wq, const void* scales, const void* zeros, const void* x, void* y, int N, int K,
                        int variant, void* stream);

/* Fused bias epilogue, y = W x + bias (bias bf16 [N], 2-byte aligned, may be NULL), added in fp32 before the single
 * rounding to bf16. For the Qwen2.5 QKV projection, whose bias the reference harness ignores
 * (paia-bench/configs/shapes.yaml:7). */
int paia_gemv_bf16_bias(const void* W, const void* x, const void* bias, void* y, int N, int K, int variant,
                        void* stream);
int paia_gemv_fp8_bias(const void* Wq, const void* scale, const void* x, const void* bias, void* y, int N, int K,
                       int variant, void* stream);
int paia_gemv_int4_bias(const void* Wq, const void* scales, const void* x, const void* bias, void* y, int N, int K,
                        int variant, void* stream);
int paia_gemv_int4_asym_bias(const void* Wq, const void* scales, const void* zeros, const void* x, const void* bias,
                             void* y, int N, int K, int variant, void* stream);

/* How the B200 build interprets variant v of `kind` (0 bf16, 1 fp8, 2 int4, 3 int4_asym): R rows per warp slot,
 * U 16-byte steps per row in flight, W warps per CTA, S (bf16) mixed-precision FMA, H programmatic dependent launch,
 * KS warps per row (0 = chosen at launch from K and N), vec_bytes per load, math = dequantisation path. Extends the
 * tuple interface of src/paia_gemv/gemv_quant.cu:61-71. */
typedef struct paia_gemv_variant_ex { int R, U, W, S, H, KS, pdl, vec_bytes, math; } paia_gemv_variant_ex;
int paia_gemv_variant_info_ex(int kind, int v, paia_gemv_variant_ex* out);

/* Tuning entry point (the B200 analogue of the variant sweep of src/tools/dev_sweep_bf16.py): launch any compiled
 * kernel instance (R, U, W, math) of `kind` with explicit PDL (0/1), warps per row ks (0 = auto) and CTAs per SM
 * (0 = auto). TMA-fed instances (math >= 5): R = ring stages (<= 1: as many as fit) and ks = shared-memory share
 * (bits 0-7) | x-first knob (bits 8-15: 0 auto, k in 1..254 streams k - 1 weight stages before the producer
 * waits for the consumers' x loads, 255 streams the whole ring first) | full tiles as one tiled tensor copy per stage
 * instead of per-row bulk copies (bit 16; slower on every decode shape measured, kept for comparison).
 * s/z/bias as in the per-format entry points (unused ones may be NULL). -1 if no such instance exists. */
int paia_gemv_launch_ex(int kind, int R, int U, int W, int math, int pdl, int ks, int ctas_per_sm, const void* Wq,
                        const void* s, const void* z, const void* x, const void* bias, void* y, int N, int K,
                        void* stream);

/* No reference kernel (the QKV neighbour of the decode GEMV): y = RoPE(W x + bias) for a fused QKV
 * projection, the rotary embedding applied in the epilogue. Rows [0, rope_rows) are the q and k heads (head_dim rows
 * each) in pair-interleaved order - row 2i + h of a head holds dimension i + h head_dim / 2 (rope_pair_rows in
 * paia_gemv.quant permutes W, its scales / zeros and the bias once) - and rows past rope_rows (v) are as usual. The
 * epilogue rotates pair i of each head by pos * theta^(-2i / head_dim) (the rotate-half form) and stores every
 * dimension of every head at its natural row, so y is in the usual order. Same checks and codes as the per-format
 * calls; -2 also for odd N or head_dim, rope_rows not a multiple of head_dim, theta <= 0, pos < 0, or a shape the
 * TMA-fed kernel cannot stage. */
int paia_gemv_rope(int kind, const void* Wq, const void* scales, const void* zeros, const void* x, const void* bias,
                   void* y, int N, int K, int rope_rows, int head_dim, float pos, float theta, void* stream);

/* Batched x (M >= 1 activation rows; the reference kernels are M = 1 only, src/README.md:118):
 * Y[M, N] = X[M, K] . dequant(W)^T (+ bias on every row), x and y bf16 row-major (row m at x + m K, y + m N), same
 * weight formats, pointer rules and codes as the per-format calls (kind 0 bf16, 1 fp8, 2 int4, 3 int4_asym; scales /
 * zeros as there, NULL where unused). Up to 8 x rows ride in the columns of each tensor-core MMA, so a launch streams
 * the weights once for all of its rows; rows are grouped 8 (fewer when x of the group does not fit in shared memory
 * next to the weight ring) per launch. Decode per format: bf16 as is, fp8 e4m3 -> f16 with x scaled per row, int4 as
 * bf16 128 + n. */
int paia_gemv_batched(int kind, const void* Wq, const void* scales, const void* zeros, const void* x, const void* bias,
                      void* y, int M, int N, int K, void* stream);

/* One launch for a sequence of up to 6 GEMVs of one format (a decode layer's projections): a persistent grid, one CTA
 * per SM, streams the weights of op 0, 1, ... back to back, so op j + 1's weights are already in flight while op j
 * finishes. Op j's x is read only after every CTA has stored op j - 1's outputs, so x of op j may be the y of any
 * earlier op; y of op j must not overlap x of op j. Same decode and accuracy as the per-format calls, and the same
 * bits on every run of the same op list; a separate per-format call may differ in the last bits, because the stage
 * chunk (and with it the split of a row among warps) is chosen for the whole sequence. math 0 = the format's default decode (bf16 5, fp8 8, int4 / int4_asym 7, falling back to 5), else a TMA math
 * code of paia_gemv_launch_ex. `counters`: nops + 1 zero-initialised uint32 in device memory, 4-byte aligned,
 * used by one launch at a time; the kernel leaves them zero. A wait that gives up after ~2 s sets error code 7 in
 * paia_gemv_device_error(). No reference counterpart (the reference launches one kernel per GEMV,
 * src/paia_gemv/gemv_quant.cu:61-71). Codes: 0, -2 bad argument / shape the kernel cannot stage, >0 cudaError_t. */
typedef struct paia_gemv_op {
    const void* Wq;       /* weights in the format of `kind` */
    const void* scales;   /* fp8 float row scales, int4 fp16 / int4_asym bf16 group scales; NULL for bf16 */
    const void* zeros;    /* int4_asym bf16 group zeros; NULL otherwise */
    const void* x;        /* bf16 [K] */
    const void* bias;     /* bf16 [N] or NULL */
    void* y;              /* bf16 [N] */
    int N, K;
    int act;              /* 0: x as given; 1: x holds [gate | up] (2K bf16) and the op reads bf16(SiLU(gate) * up),
                             SiLU(v) = v / (1 + e^-v) in fp32 (the activation between gate_up and down, fused) */
} paia_gemv_op;
int paia_gemv_layer(int kind, int math, int nops, const paia_gemv_op* ops, unsigned int* counters, void* stream);

/* A plan: the same persistent launch for a longer sequence (up to 4096 ops, e.g. every GEMV of one decode token:
 * each layer's projections and the lm_head), its op table and counters in device memory owned by the plan.
 * paia_gemv_plan_create checks the ops as paia_gemv_layer does, chooses the geometry once, and allocates and fills
 * the device table (synchronous; not inside a captured stream); paia_gemv_plan_launch is one launch (capturable,
 * no allocation; launches of one plan must not overlap); paia_gemv_plan_destroy frees it. The plan belongs to the
 * device that was current at creation. No reference counterpart (its per-token GEMV cost is the sum of one launch
 * per GEMV over the layers plus the lm_head, paia-bench/bench/analyze_e4.py:177-192). */
typedef struct paia_gemv_plan paia_gemv_plan;
int paia_gemv_plan_create(int kind, int math, int nops, const paia_gemv_op* ops, paia_gemv_plan** plan);
int paia_gemv_plan_launch(const paia_gemv_plan* plan, void* stream);
int paia_gemv_plan_destroy(paia_gemv_plan* plan);

/* Device-side error word of the current device (0 = none), set by kernels whose bounded waits gave up; clear != 0
 * resets it. Synchronous. */
int paia_gemv_device_error(int clear);

#ifdef __cplusplus
}
#endif
#endif /* PAIA_GEMV_H */
