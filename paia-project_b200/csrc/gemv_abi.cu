// libpaia_gemv.so: the C ABI of the B200 decode GEMV family.
//
// The first group of symbols is the reference's ABI with identical names, signatures, argument checks and return
// codes (Bejaine/PAIA-Project src/paia_gemv/gemv_bf16.cu:35-55 and gemv_quant.cu:58-99), so the reference's ctypes
// loader (src/paia_gemv/loader.py) and its harness adapters load this library unchanged through $PAIA_GEMV_LIB.
// Return codes: 0 ok, -1 bad variant, -2 bad shape or alignment, >0 cudaError_t of the launch.
// The library allocates nothing, keeps no per-call state, never synchronises and launches on the caller's stream
// (CUDA-graph capturable). Its only static state is a per-device cache of SM counts and occupancies.
#include <cuda_runtime.h>
#include <stdint.h>
#include <cmath>
#include <cstring>
#include <mutex>
#include <unordered_map>
#include <vector>
#include "gemv_launch.cuh"
#include "paia_gemv.h"

namespace pb2 {
int launch_int4_naive(const void* Wq, const void* sc, const void* x, void* y, int N, int K, cudaStream_t st);
int launch_int4_dequant(const void* Wq, const void* sc, void* out, int N, int K, cudaStream_t st);
const Variant* extra_int4(int* n);
const Variant* extra_int4a(int* n);

// ------------------------------------------------------------------ per-device caches
namespace {
constexpr int kMaxDev = 64;
int g_sms[kMaxDev];
size_t g_smem_optin[kMaxDev];
size_t g_smem_sm[kMaxDev];
std::mutex g_mu;
struct OccKey {
    const void* fn; int dev; int threads; size_t smem;
    bool operator==(const OccKey& o) const { return fn == o.fn && dev == o.dev && threads == o.threads && smem == o.smem; }
};
struct OccHash {
    size_t operator()(const OccKey& k) const {
        return std::hash<const void*>()(k.fn) ^ (size_t)k.dev * 0x9E3779B97F4A7C15ull ^ (k.smem << 8) ^ (size_t)k.threads;
    }
};
std::unordered_map<OccKey, int, OccHash> g_occ;

int cur_dev() { int d = 0; cudaGetDevice(&d); return (d >= 0 && d < kMaxDev) ? d : 0; }
}  // namespace

int sm_count() {
    const int d = cur_dev();
    if (g_sms[d] == 0) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, d);
        g_sms[d] = v > 0 ? v : 1;
    }
    return g_sms[d];
}

size_t max_dyn_smem() {
    const int d = cur_dev();
    if (g_smem_optin[d] == 0) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, d);
        g_smem_optin[d] = v > 0 ? (size_t)v : 48 * 1024;
    }
    return g_smem_optin[d];
}

size_t sm_smem_bytes() {
    const int d = cur_dev();
    if (g_smem_sm[d] == 0) {
        int v = 0, r = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerMultiprocessor, d);
        cudaDeviceGetAttribute(&r, cudaDevAttrReservedSharedMemoryPerBlock, d);
        g_smem_sm[d] = v > r ? (size_t)(v - r) : max_dyn_smem();
    }
    return g_smem_sm[d];
}

int max_ctas_per_sm(KernelFn fn, int threads, size_t smem) {
    const OccKey key{(const void*)fn, cur_dev(), threads, smem};
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_occ.find(key);
    if (it != g_occ.end()) return it->second;
    if (smem > 48 * 1024) cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)max_dyn_smem());
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, threads, smem) != cudaSuccess) { (void)cudaGetLastError(); n = 0; }
    g_occ.emplace(key, n);
    return n;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against the driver library).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledFn encode_tiled() {
    static const EncodeTiledFn fn = []() -> EncodeTiledFn {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            (void)cudaGetLastError();
            return nullptr;
        }
        return reinterpret_cast<EncodeTiledFn>(f);
    }();
    return fn;
}

// W [N][rb bytes] as a 3-D uint8 tensor (64 bytes, rb / 64 pieces 64 bytes apart, N rows rb bytes apart) with a box of
// 64 x rs / 64 x 16: one copy lands 16 rows of a stage at row stride rs, x coordinate always 0. A piece past the
// row end reads zeros (out of bounds). 0 when the shape does not qualify or the driver refuses the map.
int encode_weight_map(Params& p) {
    const EncodeTiledFn fn = encode_tiled();
    const uint64_t rb = (uint64_t)p.nchunk * 16;
    if (!fn || p.N < 16 || rb % 64 || p.rs % 64 || p.rs / 64 > 256 || ((uintptr_t)p.W & 15)) return 0;
    const cuuint64_t dims[3] = {64, rb / 64, (cuuint64_t)p.N};
    const cuuint64_t strides[2] = {64, rb};
    const cuuint32_t box[3] = {64, (cuuint32_t)(p.rs / 64), 16};
    const cuuint32_t es[3] = {1, 1, 1};
    const CUresult r = fn(&p.tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t*>(p.W), dims, strides, box,
                          es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 1 : 0;
}

const Variant* find_instance(int fmt, int R, int U, int W, int math) {
    int n = 0;
    if (math >= 5) {                        // TMA-fed: R is the ring depth, a launch option
        const Variant* t = tma_instances(fmt, math, &n);
        for (int i = 0; i < n; ++i)
            if (t[i].U == U && t[i].W == W) return &t[i];
        return nullptr;
    }
    if (math >= 2) {
        const Variant* t = mma_instances(fmt, math, &n);
        for (int i = 0; i < n; ++i)
            if (t[i].U == U && t[i].W == W) return &t[i];
        return nullptr;
    }
    const Variant* tabs[2] = {nullptr, nullptr};
    int counts[2] = {0, 0};
    switch (fmt) {
        case kBF16: tabs[0] = table_bf16(&counts[0]); break;
        case kFP8: tabs[0] = table_fp8(&counts[0]); break;
        case kINT4: tabs[0] = table_int4(&counts[0]); tabs[1] = extra_int4(&counts[1]); break;
        case kINT4A: tabs[0] = table_int4a(&counts[0]); tabs[1] = extra_int4a(&counts[1]); break;
        default: return nullptr;
    }
    (void)n;
    for (int t = 0; t < 2; ++t)
        for (int i = 0; i < counts[t]; ++i) {
            const Variant& v = tabs[t][i];
            if (v.R == R && v.U == U && v.W == W && v.math == math) return &v;
        }
    return nullptr;
}

}  // namespace pb2

using namespace pb2;

namespace {
inline bool aligned(const void* p, unsigned a) { return (reinterpret_cast<uintptr_t>(p) & (uintptr_t)(a - 1)) == 0; }

// A format's public variant table: the reference's tuple grid (ids and order as the reference numbers them), then
// the TMA-fed B200 variants (R = 0). Built once.
struct PublicTable {
    std::vector<Variant> v[4];
    PublicTable() {
        for (int f = 0; f < 4; ++f) {
            int n = 0, m = 0;
            const Variant* t = f == kBF16 ? table_bf16(&n) : f == kFP8 ? table_fp8(&n) : f == kINT4 ? table_int4(&n)
                                                                                                  : table_int4a(&n);
            const Variant* e = tma_public(f, &m);
            v[f].assign(t, t + n);
            v[f].insert(v[f].end(), e, e + m);
        }
    }
};
const PublicTable& public_tables() {
    static const PublicTable t;
    return t;
}

const Variant* table_of(int fmt, int* n) {
    if (fmt < 0 || fmt > 3) { *n = 0; return nullptr; }
    const std::vector<Variant>& t = public_tables().v[fmt];
    *n = (int)t.size();
    return t.data();
}

// Shape and alignment contract of each format (the reference's checks, plus the bias and zero pointers).
int check_args(int fmt, const void* W, const void* s, const void* z, const void* x, const void* bias, const void* y,
               int N, int K) {
    if (N <= 0 || K <= 0) return -2;
    switch (fmt) {
        case kBF16:   // gemv_bf16.cu:49-51: K % 8, W/x/y 16-byte aligned
            if ((K & 7) || !aligned(W, 16) || !aligned(x, 16) || !aligned(y, 16)) return -2;
            break;
        case kFP8:    // gemv_quant.cu:66: K % 16, Wq/x 16 B, scale 4 B, y 2 B
            if ((K & 15) || !aligned(W, 16) || !aligned(x, 16) || !aligned(s, 4) || !aligned(y, 2)) return -2;
            break;
        case kINT4:   // gemv_quant.cu:75: K % 128, Wq/x 16 B, scales 2 B, y 2 B
            if ((K & 127) || !aligned(W, 16) || !aligned(x, 16) || !aligned(s, 2) || !aligned(y, 2)) return -2;
            break;
        case kINT4A:
            if ((K & 127) || !aligned(W, 16) || !aligned(x, 16) || !aligned(s, 2) || !aligned(z, 2) || !aligned(y, 2))
                return -2;
            break;
        default: return -2;
    }
    if (bias && !aligned(bias, 2)) return -2;
    return 0;
}

int row_bytes(int fmt, int K) { return fmt == kBF16 ? K * 2 : fmt == kFP8 ? K : K / 2; }

// The reference's op adapters use one default tuple per format unless a tuned entry names another
// (paia-bench/bench/ops/ours_bf16.py:22-29, ours_quant.py:19-26): BF16 (2,4,4,0,1), FP8 (2,2,4,0,1), INT4 (4,2,4,0,1);
// the asymmetric INT4 format uses the INT4 tuple.
bool is_default_tuple(int fmt, const Variant& v) {
    if (v.S != 0 || v.H != 1) return false;
    switch (fmt) {
        case kBF16: return v.R == 2 && v.U == 4 && v.W == 4;
        case kFP8: return v.R == 2 && v.U == 2 && v.W == 4;
        default: return v.R == 4 && v.U == 2 && v.W == 4;
    }
}

// B200 path behind the default tuples, chosen per shape from the kernel-family comparison on B200 (every real
// Llama-3.1-8B / Qwen2.5-7B shape, each format, alone and in decode-layer chains; `bench.py --families`):
//   * N <= 1024 (k/v projections): the tuple's own CUDA-core instance (it splits K across warps; 16-row tiles leave
//     most SMs with a single partial tile) - signalled by returning -2;
//   * otherwise the TMA-fed tensor-core kernel with the decode measured fastest (BF16 as is, FP8 e4m3 straight into
//     e4m3 MMA, INT4 through the integer MMA; 8 consumer warps, 2 steps per iteration, as deep a ring as fits).
//     (Alone, the register-fed kernel wins a few long-K INT4 shapes by up to 15%; inside the chained decode layer,
//     which is how the op runs, the TMA kernel is faster for every INT4 layer sequence measured.)
// Returns -2 when the chosen kernel cannot stage the shape (the caller then runs the tuple's own instance).
// pdl = false: the launch waits for the whole preceding grid (no programmatic dependent launch), for callers whose
// weights the preceding kernel writes.
int launch_b200_default(int fmt, const Params& p, cudaStream_t st, bool pdl = true) {
    if (p.N <= 1024) return -2;
    static const int maths[4][2] = {{5, 0}, {8, 5}, {7, 5}, {7, 5}};   // first choice, then a fallback (0: none)
    for (int k = 0; k < 2; ++k) {
        const int math = maths[fmt][k];
        if (!math) break;
        const Variant* inst = find_instance(fmt, 0, 2, 8, math);
        if (!inst) continue;
        Variant v = *inst;
        v.H = pdl ? 1 : 0;
        const LaunchOpts o{0, 0};
        const int rc = launch_variant(v, p, o, st);
        if (rc != -2) return rc;
    }
    return -2;
}

int run(int fmt, const void* W, const void* s, const void* z, const void* x, const void* bias, void* y, int N, int K,
        int variant, void* stream, const LaunchOpts* opts) {
    int n = 0;
    const Variant* tab = table_of(fmt, &n);
    if (variant < 0 || variant >= n) return -1;
    const int rc = check_args(fmt, W, s, z, x, bias, y, N, K);
    if (rc) return rc;
    Params p{};
    p.W = static_cast<const uint8_t*>(W);
    p.s = s;
    p.z = z;
    p.x = static_cast<const __nv_bfloat16*>(x);
    p.bias = static_cast<const __nv_bfloat16*>(bias);
    p.y = static_cast<__nv_bfloat16*>(y);
    p.N = N;
    p.K = K;
    p.nchunk = row_bytes(fmt, K) / 16;
    p.groups = K / 128;
    if (!opts && is_default_tuple(fmt, tab[variant])) {
        const int rc = launch_b200_default(fmt, p, static_cast<cudaStream_t>(stream));
        if (rc != -2) return rc;                         // else: the CUDA-core instance of the same tuple
    }
    const LaunchOpts none{0, 0};
    return launch_variant(tab[variant], p, opts ? *opts : none, static_cast<cudaStream_t>(stream));
}

int info4(int fmt, int v, int* R, int* U, int* W, int* H) {
    int n = 0;
    const Variant* t = table_of(fmt, &n);
    if (v < 0 || v >= n) return -1;
    *R = t[v].R; *U = t[v].U; *W = t[v].W; *H = t[v].H;
    return 0;
}

int default_bf16_variant() {   // (R, U, W, S, H) = (2, 4, 4, 0, 1), looked up by tuple as gemv_quant.cu:47-56 does
    int n = 0;
    const Variant* t = table_bf16(&n);
    for (int i = 0; i < n; ++i)
        if (t[i].R == 2 && t[i].U == 4 && t[i].W == 4 && t[i].S == 0 && t[i].H == 1) return i;
    return 0;
}

}  // namespace

namespace pb2tp {   // tensor-parallel helpers (named, outside the C linkage block: they hold a kernel)
// The TMA-fed kernel every TP launch uses (the only one with the peer-store epilogue): the format's default decode.
const Variant* tp_instance(int fmt, const Params& p, Variant* out) {
    static const int maths[4][2] = {{5, 0}, {8, 5}, {7, 5}, {7, 5}};
    for (int k = 0; k < 2; ++k) {
        const int math = maths[fmt][k];
        if (!math) break;
        const Variant* inst = find_instance(fmt, 0, 2, 8, math);
        if (!inst) continue;
        long long G = 0;
        *out = *inst;
        out->H = 1;
        const LaunchOpts o{0, 0};
        if (launch_variant(*out, p, o, nullptr, &G) == 0) return out;
    }
    return nullptr;
}

// The rotary-epilogue instance of the same decodes, in the same order (the first one whose plan fits).
const Variant* rope_instance(int fmt, const Params& p, Variant* out) {
    static const int maths[4][2] = {{5, 0}, {8, 5}, {7, 5}, {7, 5}};
    for (int k = 0; k < 2; ++k) {
        const int math = maths[fmt][k];
        if (!math) break;
        const Variant* inst = tma_rope(fmt, math);
        if (!inst) continue;
        long long G = 0;
        *out = *inst;
        const LaunchOpts o{0, 0};
        if (launch_variant(*out, p, o, nullptr, &G) == 0) return out;
    }
    return nullptr;
}

}  // namespace pb2tp


namespace {
// Checks the ops of a layer launch or plan and converts them to kernel descriptors; *maxN = the largest N.
int fill_ops(int kind, int nops, const paia_gemv_op* ops, pb2::GemvOp* out, int* maxN) {
    *maxN = 0;
    for (int j = 0; j < nops; ++j) {
        const paia_gemv_op& o = ops[j];
        const int rc = check_args(kind, o.Wq, o.scales, o.zeros, o.x, o.bias, o.y, o.N, o.K);
        if (rc) return rc;
        if (o.act != kActNone && o.act != kActSiluMul) return -2;
        const uintptr_t x0 = (uintptr_t)o.x, x1 = x0 + 2 * (size_t)o.K * (o.act == kActSiluMul ? 2 : 1);
        const uintptr_t y0 = (uintptr_t)o.y, y1 = y0 + 2 * (size_t)o.N;
        if (x0 < y1 && y0 < x1) return -2;                   // other CTAs store y while x is still being read
        GemvOp& g = out[j];
        g = GemvOp{};
        g.W = static_cast<const uint8_t*>(o.Wq);
        g.s = o.scales;
        g.z = o.zeros;
        g.x = static_cast<const __nv_bfloat16*>(o.x);
        g.bias = static_cast<const __nv_bfloat16*>(o.bias);
        g.y = static_cast<__nv_bfloat16*>(o.y);
        g.N = o.N;
        g.K = o.K;
        g.nchunk = row_bytes(kind, o.K) / 16;
        g.groups = o.K / 128;
        g.act = o.act;
        *maxN = o.N > *maxN ? o.N : *maxN;
    }
    return 0;
}

// The TMA instance of a layer launch and its geometry: math 0 = the format's default decode (then a fallback when it
// cannot stage the sequence), one CTA per SM so that every CTA is resident.
int plan_layer(int kind, int math, Params& p, const Variant** inst_out, Planned* pl) {
    static const int maths[4][2] = {{5, 0}, {8, 5}, {7, 5}, {7, 5}};
    const int first = math ? math : maths[kind][0], second = math ? 0 : maths[kind][1];
    for (int m : {first, second}) {
        if (m < 5) break;
        const Variant* inst = find_instance(kind, 0, 2, 8, m);
        if (!inst) return -2;
        const LaunchOpts o{0, 1};
        const int rc = plan_variant(*inst, p, o, pl);
        if (rc == 0) { *inst_out = inst; return 0; }
        if (rc != -2) return rc;
    }
    return -2;
}
}  // namespace

extern "C" {

// ------------------------------------------------------------------ the reference's ABI

int paia_gemv_bf16_variant_count(void) { int n = 0; table_of(kBF16, &n); return n; }

int paia_gemv_bf16_variant_info(int v, int* R, int* U, int* W, int* S, int* H) {
    int n = 0;
    const Variant* t = table_of(kBF16, &n);
    if (v < 0 || v >= n) return -1;
    *R = t[v].R; *U = t[v].U; *W = t[v].W; *S = t[v].S; *H = t[v].H;
    return 0;
}

int paia_gemv_bf16(const void* W, const void* x, void* y, int N, int K, int variant, void* stream) {
    return run(kBF16, W, nullptr, nullptr, x, nullptr, y, N, K, variant, stream, nullptr);
}

int paia_gemv_fp8_variant_count(void) { int n = 0; table_of(kFP8, &n); return n; }
int paia_gemv_fp8_variant_info(int v, int* R, int* U, int* W, int* H) { return info4(kFP8, v, R, U, W, H); }

int paia_gemv_fp8(const void* Wq, const void* scale, const void* x, void* y, int N, int K, int variant, void* stream) {
    return run(kFP8, Wq, scale, nullptr, x, nullptr, y, N, K, variant, stream, nullptr);
}

int paia_gemv_int4_variant_count(void) { int n = 0; table_of(kINT4, &n); return n; }
int paia_gemv_int4_variant_info(int v, int* R, int* U, int* W, int* H) { return info4(kINT4, v, R, U, W, H); }

int paia_gemv_int4(const void* Wq, const void* scales, const void* x, void* y, int N, int K, int variant, void* stream) {
    return run(kINT4, Wq, scales, nullptr, x, nullptr, y, N, K, variant, stream, nullptr);
}

int paia_gemv_int4_naive(const void* Wq, const void* scales, const void* x, void* y, int N, int K, void* stream) {
    if (check_args(kINT4, Wq, scales, nullptr, x, nullptr, y, N, K)) return -2;
    return launch_int4_naive(Wq, scales, x, y, N, K, static_cast<cudaStream_t>(stream));
}

int paia_gemv_int4_unfused(const void* Wq, const void* scales, const void* x, void* y, void* scratch_bf16, int N, int K,
                           void* stream) {
    // gemv_quant.cu:89: the reference checks Wq/x/scratch 16 B and scales 2 B; y is checked by the BF16 GEMV.
    if (N <= 0 || K <= 0 || (K & 127) || !aligned(Wq, 16) || !aligned(x, 16) || !aligned(scales, 2) ||
        !aligned(scratch_bf16, 16))
        return -2;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int rc = launch_int4_dequant(Wq, scales, scratch_bf16, N, K, st);
    if (rc) return rc;
    // The BF16 GEMV (the default tuple's path, as gemv_quant.cu:96 runs it) reads the scratch the dequantisation grid
    // has just written, so it is launched without programmatic dependent launch: its kernels start streaming W before
    // their grid-dependency wait, and only a full stream-order dependency makes the previous grid's writes visible.
    const int arc = check_args(kBF16, scratch_bf16, nullptr, nullptr, x, nullptr, y, N, K);
    if (arc) return arc;
    Params p{};
    p.W = static_cast<const uint8_t*>(scratch_bf16);
    p.x = static_cast<const __nv_bfloat16*>(x);
    p.y = static_cast<__nv_bfloat16*>(y);
    p.N = N;
    p.K = K;
    p.nchunk = row_bytes(kBF16, K) / 16;
    p.groups = K / 128;
    const int brc = launch_b200_default(kBF16, p, st, false);
    if (brc != -2) return brc;
    int n = 0;
    Variant v = table_bf16(&n)[default_bf16_variant()];
    v.H = 0;
    const LaunchOpts none{0, 0};
    return launch_variant(v, p, none, st);
}

// Unfused INT4 with library-owned scratch, for callers that cannot pass a scratch buffer (a memory pool that owns
// all of HBM, a C host without a device allocator, a loop where cudaMalloc / cudaFree would synchronise the device).
// The scratch is a file-scope device array (module-load storage, not an allocation in this call); its device
// address is looked up once per device with cudaGetSymbolAddress, with that device current, and cached (the cache
// does not survive cudaDeviceReset). Calls that overlap on the GPU (two streams, or two host threads) share the array
// and race; it keeps the last call's contents, and every call overwrites the N x K elements it reads. The first call
// on a device does the address lookup (a host-side runtime call), so it should come before any stream capture.
namespace {
constexpr size_t kStaticScratchElems = (size_t)16 << 20;       // 16 Mi bf16 = 32 MiB (e.g. N x K = 4096 x 4096)
static __device__ __align__(256) __nv_bfloat16 g_static_scratch[kStaticScratchElems];
void* g_static_scratch_addr[kMaxDev];
}  // namespace

int paia_gemv_int4_unfused_static(const void* Wq, const void* scales, const void* x, void* y, int N, int K,
                                  void* stream) {
    if (N <= 0 || K <= 0 || (size_t)N * (size_t)K > kStaticScratchElems) return -2;   // too big for the scratch
    const int d = cur_dev();
    void* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!g_static_scratch_addr[d]) {
            void* a = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&a, g_static_scratch);
            if (e != cudaSuccess || !a) {
                (void)cudaGetLastError();
                return e != cudaSuccess ? (int)e : (int)cudaErrorInvalidSymbol;
            }
            g_static_scratch_addr[d] = a;
        }
        scratch = g_static_scratch_addr[d];
    }
    return paia_gemv_int4_unfused(Wq, scales, x, y, scratch, N, K, stream);
}

// ------------------------------------------------------------------ row-sharded tensor parallelism

namespace {
int tp_launch(int kind, const void* Wq, const void* s, const void* z, const void* x, const void* bias,
              void* const* y_all, unsigned int* const* flag_all, int world, int rank, int N_local, int K,
              bool defer, void* stream) {
    if (kind < 0 || kind > 3 || world < 1 || world > 8 || rank < 0 || rank >= world || !y_all || !flag_all) return -2;
    for (int r = 0; r < world; ++r)
        if (!y_all[r] || !flag_all[r] || !aligned(y_all[r], 2) || !aligned(flag_all[r], 16)) return -2;
    const int rc = check_args(kind, Wq, s, z, x, bias, y_all[rank], N_local, K);
    if (rc) return rc;
    Params p{};
    p.W = static_cast<const uint8_t*>(Wq);
    p.s = s;
    p.z = z;
    p.x = static_cast<const __nv_bfloat16*>(x);
    p.bias = static_cast<const __nv_bfloat16*>(bias);
    p.y = static_cast<__nv_bfloat16*>(y_all[rank]) + (size_t)rank * N_local;
    p.N = N_local;
    p.K = K;
    p.nchunk = row_bytes(kind, K) / 16;
    p.groups = K / 128;
    p.tp_world = world;
    p.tp_rank = rank;
    p.tp_off = rank * N_local;
    p.tp_defer = defer ? 1 : 0;
    for (int r = 0; r < world; ++r) {
        p.tp_y[r] = static_cast<__nv_bfloat16*>(y_all[r]);
        p.tp_flag[r] = flag_all[r];
    }
    Variant v;
    if (!pb2tp::tp_instance(kind, p, &v)) return -2;
    const LaunchOpts o{0, 0};
    return launch_variant(v, p, o, static_cast<cudaStream_t>(stream));
}
}  // namespace

int paia_gemv_tp(int kind, const void* Wq, const void* s, const void* z, const void* x, const void* bias,
                 void* const* y_all, unsigned int* const* flag_all, int world, int rank, int N_local, int K,
                 void* stream) {
    return tp_launch(kind, Wq, s, z, x, bias, y_all, flag_all, world, rank, N_local, K, false, stream);
}

int paia_gemv_tp_deferred(int kind, const void* Wq, const void* s, const void* z, const void* x, const void* bias,
                          void* const* y_all, unsigned int* const* flag_all, int world, int rank, int N_local, int K,
                          void* stream) {
    return tp_launch(kind, Wq, s, z, x, bias, y_all, flag_all, world, rank, N_local, K, true, stream);
}

int paia_gemv_tp_exchange(unsigned int* const* xflag_all, int world, int rank, void* stream) {
    if (world < 1 || world > 8 || rank < 0 || rank >= world || !xflag_all) return -2;
    for (int r = 0; r < world; ++r)
        if (!xflag_all[r] || !aligned(xflag_all[r], 16)) return -2;
    return launch_tp_exchange(xflag_all, world, rank, static_cast<cudaStream_t>(stream));
}

// Buffers that other ranks map (full-size y and the arrival counters): plain device allocations, so that their
// CUDA IPC handles name exactly these bytes; zero-filled. Setup-time calls, never inside a GEMV.
int paia_gemv_tp_alloc(size_t bytes, void** ptr) {
    if (!ptr || bytes == 0) return -2;
    *ptr = nullptr;
    cudaError_t e = cudaMalloc(ptr, bytes);
    if (e == cudaSuccess) e = cudaMemset(*ptr, 0, bytes);
    if (e != cudaSuccess) { (void)cudaGetLastError(); return (int)e; }
    return 0;
}
int paia_gemv_tp_free(void* ptr) {
    const cudaError_t e = cudaFree(ptr);
    if (e != cudaSuccess) { (void)cudaGetLastError(); return (int)e; }
    return 0;
}
// 64-byte CUDA IPC handle of a paia_gemv_tp_alloc buffer, and its mapping in another process (peer access enabled
// lazily by the driver: the mapped pointer is usable from kernels on the calling process's current device).
int paia_gemv_ipc_handle(const void* ptr, void* handle64) {
    if (!ptr || !handle64) return -2;
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
    if (e != cudaSuccess) { (void)cudaGetLastError(); return (int)e; }
    static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
    memcpy(handle64, &h, sizeof(h));
    return 0;
}
int paia_gemv_ipc_open(const void* handle64, void** ptr) {
    if (!handle64 || !ptr) return -2;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle64, sizeof(h));
    *ptr = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) { (void)cudaGetLastError(); return (int)e; }
    return 0;
}
int paia_gemv_ipc_close(void* ptr) {
    const cudaError_t e = cudaIpcCloseMemHandle(ptr);
    if (e != cudaSuccess) { (void)cudaGetLastError(); return (int)e; }
    return 0;
}

int paia_gemv_tp_ctas(int kind, int N_local, int K) {
    if (kind < 0 || kind > 3 || N_local <= 0 || K <= 0) return -2;
    Params p{};
    p.N = N_local;
    p.K = K;
    p.nchunk = row_bytes(kind, K) / 16;
    p.groups = K / 128;
    Variant v;
    if (!pb2tp::tp_instance(kind, p, &v)) return -2;
    long long G = 0;
    const LaunchOpts o{0, 0};
    if (launch_variant(v, p, o, nullptr, &G)) return -2;
    return (int)G;
}

// ------------------------------------------------------------------ rotary embedding fused into the epilogue

int paia_gemv_rope(int kind, const void* Wq, const void* scales, const void* zeros, const void* x, const void* bias,
                   void* y, int N, int K, int rope_rows, int head_dim, float pos, float theta, void* stream) {
    if (kind < 0 || kind > 3) return -2;
    const int rc = check_args(kind, Wq, scales, zeros, x, bias, y, N, K);
    if (rc) return rc;
    if ((N & 1) || head_dim < 2 || (head_dim & 1) || rope_rows < 0 || rope_rows > N || rope_rows % head_dim ||
        !(theta > 0.f) || !(pos >= 0.f))
        return -2;
    Params p{};
    p.W = static_cast<const uint8_t*>(Wq);
    p.s = scales;
    p.z = zeros;
    p.x = static_cast<const __nv_bfloat16*>(x);
    p.bias = static_cast<const __nv_bfloat16*>(bias);
    p.y = static_cast<__nv_bfloat16*>(y);
    p.N = N;
    p.K = K;
    p.nchunk = row_bytes(kind, K) / 16;
    p.groups = K / 128;
    p.rope_rows = rope_rows;
    p.rope_hd = head_dim;
    p.rope_pos = pos;
    p.rope_log2_theta = log2f(theta);
    Variant v;
    if (!pb2tp::rope_instance(kind, p, &v)) return -2;        // the rotary instance of the format's default decode
    const LaunchOpts o{0, 0};
    return launch_variant(v, p, o, static_cast<cudaStream_t>(stream));
}

// ------------------------------------------------------------------ batched x (M > 1)

int paia_gemv_batched(int kind, const void* Wq, const void* scales, const void* zeros, const void* x, const void* bias,
                      void* y, int M, int N, int K, void* stream) {
    if (kind < 0 || kind > 3 || M < 1) return -2;
    const int rc = check_args(kind, Wq, scales, zeros, x, bias, y, N, K);
    if (rc) return rc;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const Variant* inst = find_instance(kind, 0, 2, 8, 9);
    if (!inst) return -2;
    int n = 0;
    const Variant* tab = table_of(kind, &n);
    int dflt = -1;                                             // the format's default tuple: rows no group can take
    for (int v = 0; v < n; ++v)
        if (is_default_tuple(kind, tab[v])) { dflt = v; break; }
    const auto* xb = static_cast<const __nv_bfloat16*>(x);
    auto* yb = static_cast<__nv_bfloat16*>(y);
    // groups of up to 8 x rows per launch, as many as fit next to the ring; each launch streams the weights once. A
    // group of one row takes the single-row path (its decodes are faster than the batched ones).
    for (int m0 = 0; m0 < M;) {
        int mg = M - m0 < 8 ? M - m0 : 8;
        Planned pl;
        int prc = -2;
        for (; mg >= 2; --mg) {
            Params p{};
            p.W = static_cast<const uint8_t*>(Wq);
            p.s = scales;
            p.z = zeros;
            p.x = xb + (size_t)m0 * K;
            p.bias = static_cast<const __nv_bfloat16*>(bias);
            p.y = yb + (size_t)m0 * N;
            p.N = N;
            p.K = K;
            p.nchunk = row_bytes(kind, K) / 16;
            p.groups = K / 128;
            p.xm = mg;
            p.ldx = K;
            p.ldy = N;
            const LaunchOpts o{0, 0};
            prc = plan_variant(*inst, p, o, &pl);
            if (prc != -2) break;
        }
        if (prc == 0) {
            const int lrc = launch_planned(inst->fn, pl, st);
            if (lrc) return lrc;
            m0 += mg;
            continue;
        }
        if (prc != -2 || dflt < 0) return prc;
        // one row (or rows that no batched launch can stage): the single-row path
        const int r = run(kind, Wq, scales, zeros, xb + (size_t)m0 * K, bias, yb + (size_t)m0 * N, N, K, dflt, stream,
                          nullptr);
        if (r) return r;
        m0 += 1;
    }
    return 0;
}

// ------------------------------------------------------------------ layer launch and plans


int paia_gemv_layer(int kind, int math, int nops, const paia_gemv_op* ops, unsigned int* counters, void* stream) {
    if (kind < 0 || kind > 3 || nops < 1 || nops > kMaxOps || !ops || !counters || !aligned(counters, 4)) return -2;
    Params p{};
    p.nops = nops;
    p.layer_done = counters;
    const int rc = fill_ops(kind, nops, ops, p.ops, &p.N);
    if (rc) return rc;
    const Variant* inst = nullptr;
    Planned pl;
    const int prc = plan_layer(kind, math, p, &inst, &pl);
    if (prc) return prc;
    return launch_planned(inst->fn, pl, static_cast<cudaStream_t>(stream));
}

struct paia_gemv_plan {
    KernelFn fn;
    Planned pl;
    void* dev_mem;            // op table, then nops + 1 counters
};

int paia_gemv_plan_create(int kind, int math, int nops, const paia_gemv_op* ops, paia_gemv_plan** out) {
    if (!out) return -2;
    *out = nullptr;
    if (kind < 0 || kind > 3 || nops < 1 || nops > kMaxPlanOps || !ops) return -2;
    std::vector<GemvOp> host((size_t)nops);
    Params p{};
    p.nops = nops;
    int rc = fill_ops(kind, nops, ops, host.data(), &p.N);
    if (rc) return rc;
    p.host_ops = host.data();
    const Variant* inst = nullptr;
    Planned pl;
    rc = plan_layer(kind, math, p, &inst, &pl);           // also fills every op's stages per row in `host`
    if (rc) return rc;
    const size_t table = (size_t)nops * sizeof(GemvOp), ctr = (size_t)(nops + 1) * sizeof(unsigned int);
    void* mem = nullptr;
    cudaError_t e = cudaMalloc(&mem, table + ctr);
    if (e == cudaSuccess) e = cudaMemcpy(mem, host.data(), table, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(static_cast<uint8_t*>(mem) + table, 0, ctr);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        if (mem) cudaFree(mem);
        return (int)e;
    }
    paia_gemv_plan* plan = new paia_gemv_plan;
    plan->fn = inst->fn;
    plan->pl = pl;
    plan->pl.p.op_table = static_cast<const GemvOp*>(mem);
    plan->pl.p.layer_done = reinterpret_cast<unsigned int*>(static_cast<uint8_t*>(mem) + table);
    plan->dev_mem = mem;
    *out = plan;
    return 0;
}

int paia_gemv_plan_launch(const paia_gemv_plan* plan, void* stream) {
    if (!plan) return -2;
    return launch_planned(plan->fn, plan->pl, static_cast<cudaStream_t>(stream));
}

int paia_gemv_plan_destroy(paia_gemv_plan* plan) {
    if (!plan) return 0;
    const cudaError_t e = cudaFree(plan->dev_mem);
    delete plan;
    if (e != cudaSuccess) { (void)cudaGetLastError(); return (int)e; }
    return 0;
}

// ------------------------------------------------------------------ B200 additions

const char* paia_gemv_version(void) { return "paia-gemv-b200 1.0 (sm_100a)"; }

int paia_gemv_int4_asym_variant_count(void) { int n = 0; table_of(kINT4A, &n); return n; }
int paia_gemv_int4_asym_variant_info(int v, int* R, int* U, int* W, int* H) { return info4(kINT4A, v, R, U, W, H); }

int paia_gemv_int4_asym(const void* Wq, const void* scales, const void* zeros, const void* x, void* y, int N, int K,
                        int variant, void* stream) {
    return run(kINT4A, Wq, scales, zeros, x, nullptr, y, N, K, variant, stream, nullptr);
}

int paia_gemv_bf16_bias(const void* W, const void* x, const void* bias, void* y, int N, int K, int variant,
                        void* stream) {
    return run(kBF16, W, nullptr, nullptr, x, bias, y, N, K, variant, stream, nullptr);
}

int paia_gemv_fp8_bias(const void* Wq, const void* scale, const void* x, const void* bias, void* y, int N, int K,
                       int variant, void* stream) {
    return run(kFP8, Wq, scale, nullptr, x, bias, y, N, K, variant, stream, nullptr);
}

int paia_gemv_int4_bias(const void* Wq, const void* scales, const void* x, const void* bias, void* y, int N, int K,
                        int variant, void* stream) {
    return run(kINT4, Wq, scales, nullptr, x, bias, y, N, K, variant, stream, nullptr);
}

int paia_gemv_int4_asym_bias(const void* Wq, const void* scales, const void* zeros, const void* x, const void* bias,
                             void* y, int N, int K, int variant, void* stream) {
    return run(kINT4A, Wq, scales, zeros, x, bias, y, N, K, variant, stream, nullptr);
}

// Variant details as the B200 build interprets them. kind: 0 bf16, 1 fp8, 2 int4, 3 int4_asym.
int paia_gemv_variant_info_ex(int kind, int v, paia_gemv_variant_ex* out) {
    int n = 0;
    const Variant* t = table_of(kind, &n);
    if (!t || v < 0 || v >= n || !out) return -1;
    *out = {t[v].R, t[v].U, t[v].W, t[v].S, t[v].H, 0, t[v].H, 16, t[v].math};
    return 0;
}

// Tuning entry point: any compiled instance (R, U, W, math) of a format with explicit K-split (ks, 0 = auto),
// CTAs per SM (0 = auto) and PDL (0/1). Pointers and bias as in the per-format entry points (s/z unused where the
// format has none). Same return codes; -1 when no such instance is compiled.
int paia_gemv_launch_ex(int kind, int R, int U, int W, int math, int pdl, int ks, int ctas_per_sm, const void* Wq,
                        const void* s, const void* z, const void* x, const void* bias, void* y, int N, int K,
                        void* stream) {
    const Variant* inst = find_instance(kind, R, U, W, math);
    if (!inst) return -1;
    const int rc = check_args(kind, Wq, s, z, x, bias, y, N, K);
    if (rc) return rc;
    Variant v = *inst;
    v.H = pdl ? 1 : 0;
    Params p{};
    p.W = static_cast<const uint8_t*>(Wq);
    p.s = s;
    p.z = z;
    p.x = static_cast<const __nv_bfloat16*>(x);
    p.bias = static_cast<const __nv_bfloat16*>(bias);
    p.y = static_cast<__nv_bfloat16*>(y);
    p.N = N;
    p.K = K;
    p.nchunk = row_bytes(kind, K) / 16;
    p.groups = K / 128;
    LaunchOpts o{ks, ctas_per_sm};
    if (math >= 5) {                        // TMA-fed kernels: R = ring stages (<= 1: auto), ks = shared-memory share
        o.ring = R <= 1 ? 0 : R;            // (bits 0-7), stages streamed before the x loads (bits 8-15, LaunchOpts),
        o.share = ks & 0xFF;                // tiled tensor copies of full tiles (bit 16)
        o.pre = (ks >> 8) & 0xFF;
        o.tensor_on = (ks >> 16) & 1;
        o.ks = 0;
    }
    return launch_variant(v, p, o, static_cast<cudaStream_t>(stream));
}

// Device-side error word of the current device (0 = none; the codes of the TMA-fed kernels' bounded waits, 6 and 8
// from the tensor-parallel exchange); clear != 0 resets it. Synchronous (a symbol copy).
int paia_gemv_device_error(int clear) { return tma_device_error(clear); }

}  // extern "C"
