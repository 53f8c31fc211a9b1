// w4a8_capi.cu -- the C ABI of libw4a8_b200.so (declared in include/w4a8_b200.h).
//
// Host-side work only: argument checks (the reference's TORCH_CHECKs,
// npu_ops/host/midgroup_w4a8_gemm.cpp:149-183), workspace carving, TMA
// descriptor encoding, tile / grid sizing, and the two launches of a linear
// call (quantiser, then the GEMM with programmatic dependent launch so its
// weight stream starts while the quantiser is still running).
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "w4a8_b200.h"
#include "w4a8_kernels.h"

using namespace w4a8;

namespace {

thread_local int g_last_cuda = 0;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
constexpr int kMaxDev = 64;
int g_sms[kMaxDev] = {0};
int g_major[kMaxDev] = {0};

int fail_cuda(cudaError_t e)
{
    g_last_cuda = static_cast<int>(e);
    return W4A8_ERR_CUDA;
}

int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
int64_t round_up(int64_t a, int64_t b) { return cdiv(a, b) * b; }

bool group_ok(int32_t gk) { return gk == 64 || gk == 128 || gk == 256 || gk == 1024; }

int64_t kpad_of(int64_t K, int32_t gk)
{
    const int64_t G = cdiv(K, gk);
    const int64_t stride = round_up(gk, 64);
    const int64_t last = K - (G - 1) * gk;
    return (G - 1) * stride + round_up(last, 64);
}

int device_info(int* sms)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail_cuda(e);
    if (dev < 0 || dev >= kMaxDev) return W4A8_ERR_DEVICE;
    if (g_sms[dev] == 0) {
        int n = 0, major = 0;
        if ((e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return fail_cuda(e);
        if ((e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess) return fail_cuda(e);
        g_major[dev] = major;
        g_sms[dev] = n;
    }
    if (g_major[dev] != 10) return W4A8_ERR_DEVICE;
    *sms = g_sms[dev];
    return W4A8_OK;
}

int get_encoder()
{
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    return g_encode ? W4A8_OK : W4A8_ERR_CUDA;
}

bool encode_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
               uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw)
{
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = g_encode(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Per-call geometry and the workspace carve-up.
struct Plan {
    int64_t M, N, K, Kpad, G;
    int gk, tt, n_wt, n_tt, upt, units, grid, kb_total;
    size_t off_as, off_aq, off_part, total;
    bool split;   // some output tile's units are divided between CTAs
};

// tt_cap bounds the token tile (the debug partials mode runs 16-token tiles).
// A smaller tile never needs more workspace than the tile chosen for M.
Plan compute_plan(int64_t M, int64_t N, int64_t K, int32_t gk, int sms, int tt_cap)
{
    Plan p{};
    p.M = M;
    p.N = N;
    p.K = K;
    p.gk = gk;
    p.G = cdiv(K, gk);
    p.Kpad = kpad_of(K, gk);
    p.tt = M <= 16 ? 16 : (M <= 32 ? 32 : (M <= 64 ? 64 : 128));
    p.tt = std::min(p.tt, tt_cap);
    p.n_wt = static_cast<int>(cdiv(N, 128));
    p.n_tt = static_cast<int>(cdiv(M, p.tt));
    p.kb_total = static_cast<int>(cdiv(p.Kpad, 256));
    // units per tile: stage_kblocks(tt) k-blocks (GK <= 256), one group for
    // GK = 1024 (the kernel's Cfg)
    const int ks = stage_kblocks(p.tt);
    p.upt = gk <= 256 ? static_cast<int>(cdiv(p.kb_total, ks)) : static_cast<int>(p.G);
    p.units = p.n_wt * p.n_tt * p.upt;
    p.grid = std::max(1, std::min(sms, p.units));
    p.split = false;
    for (int c = 1; c < p.grid && !p.split; ++c)
        p.split = (static_cast<int64_t>(c) * p.units / p.grid) % p.upt != 0;
    size_t off = 1024;                                                    // status word block
    p.off_as = off;                                                       // [n_tt][G][tt] fp32
    off += round_up(static_cast<int64_t>(p.n_tt) * p.G * p.tt * 4, 1024);
    p.off_aq = off;                                                       // [n_tt][kb_total][tt*256]
    off += round_up(static_cast<int64_t>(p.n_tt) * p.kb_total * p.tt * 256, 1024);
    p.off_part = off;
    off += static_cast<size_t>(2) * p.grid * p.tt * 128 * 4;
    p.total = round_up(off, 1024);
    return p;
}

// compute_plan behind a small per-thread cache: a serving loop calls the same
// few shapes over and over, and the plan's split test walks every CTA.
Plan make_plan(int64_t M, int64_t N, int64_t K, int32_t gk, int sms, int tt_cap = 128)
{
    struct Entry {
        int64_t M, N, K;
        int32_t gk;
        int sms, tt_cap;
        Plan plan;
    };
    constexpr int kEntries = 16;
    thread_local Entry cache[kEntries];
    thread_local int used = 0, next = 0;
    for (int i = 0; i < used; ++i) {
        const Entry& e = cache[i];
        if (e.M == M && e.N == N && e.K == K && e.gk == gk && e.sms == sms && e.tt_cap == tt_cap) return e.plan;
    }
    const Plan p = compute_plan(M, N, K, gk, sms, tt_cap);
    cache[next] = Entry{M, N, K, gk, sms, tt_cap, p};
    next = (next + 1) % kEntries;
    if (used < kEntries) ++used;
    return p;
}

bool aligned(const void* ptr, uintptr_t a) { return (reinterpret_cast<uintptr_t>(ptr) & (a - 1)) == 0; }

int check_common(int64_t M, int64_t N, int64_t K, int32_t gk)
{
    if (M < 0 || N <= 0 || K <= 0) return W4A8_ERR_INVALID;
    if (!group_ok(gk)) return W4A8_ERR_UNSUPPORTED;
    if (N % 8 != 0) return W4A8_ERR_INVALID;
    if (M > (int64_t(1) << 30) || K > (int64_t(1) << 30) || N > (int64_t(1) << 30)) return W4A8_ERR_INVALID;
    return W4A8_OK;
}

// Quantise x (or, with swiglu, bf16(silu(gate) * up) of x = [gate | up]) into
// the GEMM's operand order inside the workspace.
int run_quant_kernel_layout(const Plan& pl, const void* x, int64_t ldx, uint8_t* ws, cudaStream_t st,
                            bool swiglu = false)
{
    QuantParams q{};
    q.x = static_cast<const uint16_t*>(x);
    q.ldx = ldx;
    q.swiglu = swiglu ? 1 : 0;
    q.M = static_cast<int>(pl.M);
    q.K = static_cast<int>(pl.K);
    q.Kpad = static_cast<int>(pl.Kpad);
    q.G = static_cast<int>(pl.G);
    q.gk = pl.gk;
    q.rows = pl.n_tt * pl.tt;
    q.vec_ok = aligned(x, 16) && (pl.K % 8 == 0) && (ldx % 8 == 0);
    q.aq = reinterpret_cast<int8_t*>(ws + pl.off_aq);
    q.as = reinterpret_cast<float*>(ws + pl.off_as);
    q.tt = pl.tt;
    q.kb_total = pl.kb_total;
    const cudaError_t e = launch_quant_act(q, kOutKernel, st, true);
    return e == cudaSuccess ? W4A8_OK : fail_cuda(e);
}

// Encoded descriptors of one raw weight set.  Encoding tensor maps costs
// microseconds of host time per call, so recently used sets are kept (a
// serving loop calls the same few layers over and over).
struct MapKey {
    const void* w_packed;
    const void* w_scale;
    const void* w_zero;
    int64_t N, K;
    int gk, ws_dtype, gpu, dev;
    bool operator==(const MapKey& o) const { return std::memcmp(this, &o, sizeof(MapKey)) == 0; }
};

struct MapEntry {
    MapKey key;
    CUtensorMap maps[3];
    uint64_t stamp;
    bool used;
};

constexpr int kMapCache = 128;
MapEntry g_maps[kMapCache];
uint64_t g_map_clock = 0;
std::mutex g_map_mutex;

// Groups per GEMM unit (the scale / zero-point box height): the kernel's Cfg::GPU.
int groups_per_unit(const Plan& pl) { return pl.gk <= 256 ? stage_kblocks(pl.tt) * (256 / pl.gk) : 1; }

bool encode_maps(const Plan& pl, const void* w_packed, const void* w_scale, int32_t ws_dtype, const void* w_zero,
                 CUtensorMap* m)
{
    const int gpk = groups_per_unit(pl);
    return encode_2d(&m[0], CU_TENSOR_MAP_DATA_TYPE_UINT8, w_packed, pl.Kpad / 2, pl.N, pl.Kpad / 2, 128, 128,
                     CU_TENSOR_MAP_SWIZZLE_128B) &&
           (w_scale == nullptr ||   // the partials mode reads no scales
            encode_2d(&m[1],
                      ws_dtype == W4A8_DTYPE_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16,
                      w_scale, pl.N, pl.G, pl.N * (ws_dtype == W4A8_DTYPE_F32 ? 4 : 2), 128, gpk,
                      CU_TENSOR_MAP_SWIZZLE_NONE)) &&
           (w_zero == nullptr ||
            encode_2d(&m[2], CU_TENSOR_MAP_DATA_TYPE_UINT16, w_zero, pl.N, pl.G, pl.N * 2, 128, gpk,
                      CU_TENSOR_MAP_SWIZZLE_NONE));
}

bool cached_maps(const Plan& pl, const void* w_packed, const void* w_scale, int32_t ws_dtype, const void* w_zero,
                 GemmParams& g)
{
    MapKey k;
    std::memset(&k, 0, sizeof(k));
    k.w_packed = w_packed;
    k.w_scale = w_scale;
    k.w_zero = w_zero;
    k.ws_dtype = ws_dtype;
    k.gpu = groups_per_unit(pl);
    k.N = pl.N;
    k.K = pl.K;
    k.gk = pl.gk;
    cudaGetDevice(&k.dev);
    std::lock_guard<std::mutex> lock(g_map_mutex);
    int victim = 0;
    MapEntry* hit = nullptr;
    for (int i = 0; i < kMapCache && !hit; ++i) {
        if (g_maps[i].used && g_maps[i].key == k) hit = &g_maps[i];
        else if (g_maps[victim].used && (!g_maps[i].used || g_maps[i].stamp < g_maps[victim].stamp)) victim = i;
    }
    if (!hit) {
        MapEntry& e = g_maps[victim];
        std::memset(e.maps, 0, sizeof(e.maps));
        e.used = false;
        if (!encode_maps(pl, w_packed, w_scale, ws_dtype, w_zero, e.maps)) return false;
        e.key = k;
        e.used = true;
        hit = &e;
    }
    hit->stamp = ++g_map_clock;
    std::memcpy(&g.tm_w, &hit->maps[0], sizeof(CUtensorMap));
    std::memcpy(&g.tm_ws, &hit->maps[1], sizeof(CUtensorMap));
    std::memcpy(&g.tm_wz, &hit->maps[2], sizeof(CUtensorMap));
    return true;
}

// The weight operand of a call: the reference row-major layout, or a buffer
// made by w4a8_prepare_weights.
struct Weights {
    const void* w_packed;   // raw
    const void* w_scale;    // raw
    const void* w_zero;     // raw, or null
    const uint8_t* prepared;
    bool has_zero;          // prepared: zero points present
    int32_t ws_dtype;
};

// Tensor maps over activations (fused quantisation), keyed by (pointer, shape,
// stride, device): a serving loop reuses a few activation buffers, so most
// calls find their map here instead of encoding it again.
struct XMapKey {
    const void* x;
    int64_t M, K, ldx;
    int dev, pad;
    bool operator==(const XMapKey& o) const { return std::memcmp(this, &o, sizeof(XMapKey)) == 0; }
};

struct XMapEntry {
    XMapKey key;
    CUtensorMap map;
    uint64_t stamp;
    bool used;
};

constexpr int kXMapCache = 256;
XMapEntry g_xmaps[kXMapCache];
uint64_t g_xmap_clock = 0;

bool cached_x_map(const void* x, int64_t M, int64_t K, int64_t ldx, CUtensorMap* out)
{
    XMapKey k;
    std::memset(&k, 0, sizeof(k));
    k.x = x;
    k.M = M;
    k.K = K;
    k.ldx = ldx;
    cudaGetDevice(&k.dev);
    std::lock_guard<std::mutex> lock(g_map_mutex);
    int victim = 0;
    XMapEntry* hit = nullptr;
    for (int i = 0; i < kXMapCache && !hit; ++i) {
        if (g_xmaps[i].used && g_xmaps[i].key == k) hit = &g_xmaps[i];
        else if (g_xmaps[victim].used && (!g_xmaps[i].used || g_xmaps[i].stamp < g_xmaps[victim].stamp)) victim = i;
    }
    if (!hit) {
        XMapEntry& e = g_xmaps[victim];
        e.used = false;
        // box: 256 positions x 16 rows of bf16; rows >= M and positions >= K read as zero
        if (!encode_2d(&e.map, CU_TENSOR_MAP_DATA_TYPE_UINT16, x, static_cast<uint64_t>(K), static_cast<uint64_t>(M),
                       static_cast<uint64_t>(ldx) * 2, 256, 16, CU_TENSOR_MAP_SWIZZLE_NONE))
            return false;
        e.key = k;
        e.used = true;
        hit = &e;
    }
    hit->stamp = ++g_xmap_clock;
    std::memcpy(out, &hit->map, sizeof(CUtensorMap));
    return true;
}

// Library options (w4a8_set_options).
int g_options = 0;

// Whether a linear call quantises its activation inside the GEMM: only with
// W4A8_OPT_FUSED_QUANT set, and then for one 16-token tile (M <= 16), GK <= 256
// and an activation the 2-D tensor copies can read (16-byte aligned rows).
// Everything else runs the standalone quantiser first.
bool fused_quant_ok(const Plan& pl, const void* x, int64_t ldx, bool swiglu)
{
    return (g_options & W4A8_OPT_FUSED_QUANT) && !swiglu && pl.tt == 16 && pl.n_tt == 1 && pl.gk <= 256 &&
           aligned(x, 16) && ldx % 8 == 0;
}

int run_gemm(const Plan& pl, const Weights& w, void* out, int64_t ldy, bool partials, uint8_t* ws, cudaStream_t st,
             const void* fq_x = nullptr, int64_t fq_ldx = 0, const PushParams* push = nullptr)
{
    GemmParams g;
    std::memset(&g, 0, sizeof(g));
    if (push) g.push = *push;
    if (fq_x) {
        if (get_encoder() != W4A8_OK) return fail_cuda(cudaErrorNotSupported);
        if (!cached_x_map(fq_x, pl.M, pl.K, fq_ldx, &g.tm_x)) return W4A8_ERR_INVALID;
    }
    const bool asym = w.prepared ? w.has_zero : (w.w_zero != nullptr);
    if (w.prepared) {
        const PreparedLayout L = prepared_layout(pl.N, pl.G, pl.kb_total, w.ws_dtype == W4A8_DTYPE_F32 ? 4 : 2, asym);
        g.w_tiles = w.prepared + L.off_tiles;
        g.ws_tiles = w.prepared + L.off_ws;
        g.wz_tiles = asym ? w.prepared + L.off_wz : nullptr;
    } else {
        if (get_encoder() != W4A8_OK) return fail_cuda(cudaErrorNotSupported);
        if (!cached_maps(pl, w.w_packed, w.w_scale, w.ws_dtype, w.w_zero, g)) return W4A8_ERR_INVALID;
    }
    g.a_tiles = ws + pl.off_aq;
    g.as_tiles = reinterpret_cast<const float*>(ws + pl.off_as);
    g.out = out;
    g.partials = reinterpret_cast<float*>(ws + pl.off_part);
    g.status = reinterpret_cast<int*>(ws);
    g.M = static_cast<int>(pl.M);
    g.N = static_cast<int>(pl.N);
    g.Kpad = static_cast<int>(pl.Kpad);
    g.G = static_cast<int>(pl.G);
    g.ldy = ldy;
    g.n_wt = pl.n_wt;
    g.n_tt = pl.n_tt;
    g.units_per_tile = pl.upt;
    g.total_units = pl.units;
    g.kb_total = pl.kb_total;
    GemmConfig c{};
    c.tt = pl.tt;
    c.gk = pl.gk;
    c.asym = asym;
    c.ws_bf16 = w.ws_dtype != W4A8_DTYPE_F32;
    c.partials = partials;
    c.fq = fq_x != nullptr;
    cudaError_t e = launch_gemm(g, c, pl.grid, st, true);
    if (e != cudaSuccess) return fail_cuda(e);
    if (!partials && pl.split) e = launch_splitk_reduce(g, pl.tt, pl.grid, st);
    return e == cudaSuccess ? W4A8_OK : fail_cuda(e);
}

int check_weights(const void* w_packed, const void* w_scale, int32_t ws_dtype, const void* w_zero)
{
    if (!w_packed || !w_scale) return W4A8_ERR_INVALID;
    if (ws_dtype != W4A8_DTYPE_BF16 && ws_dtype != W4A8_DTYPE_F32) return W4A8_ERR_UNSUPPORTED;
    if (!aligned(w_packed, 16) || !aligned(w_scale, 16) || (w_zero && !aligned(w_zero, 16))) return W4A8_ERR_INVALID;
    return W4A8_OK;
}

// ---- fixed scratch for w4a8_linear_fixed_scratch ----
// One statically sized device array per device context (module data, not an
// allocation).  Its address is looked up with the device current and cached
// together with the id of the context it belongs to: a context made after a
// device reset loads the module again, so the array may move and its
// contents are gone, and the next call looks it up and clears it again.  The
// whole array is cleared on that first call per context, after which the
// kernels leave the status word at zero unless a wait runs out.
static __device__ __align__(256) uint8_t g_fixed_scratch[W4A8_FIXED_SCRATCH_BYTES];
uint8_t* g_fixed_ptr[kMaxDev];
unsigned long long g_fixed_ctx[kMaxDev];   // cuCtxGetId of the context g_fixed_ptr belongs to
std::mutex g_fixed_mutex;
PFN_cuCtxGetCurrent_v4000 g_ctx_current = nullptr;
PFN_cuCtxGetId_v12000 g_ctx_id = nullptr;
std::once_flag g_ctx_once;

// Id of the current context (unique for the life of the process).
int current_ctx_id(unsigned long long* id)
{
    std::call_once(g_ctx_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_ctx_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(fn);
        fn = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_ctx_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(fn);
    });
    if (!g_ctx_current || !g_ctx_id) return fail_cuda(cudaErrorNotSupported);
    CUcontext ctx = nullptr;
    if (g_ctx_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return fail_cuda(cudaErrorDeviceUninitialized);
    if (g_ctx_id(ctx, id) != CUDA_SUCCESS) return fail_cuda(cudaErrorDeviceUninitialized);
    return W4A8_OK;
}

// The array's address in the current context, or null when no call has
// looked it up there yet (caller holds g_fixed_mutex).
int fixed_scratch_cached(int* dev_out, unsigned long long* ctx_out, uint8_t** out)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail_cuda(e);
    if (dev < 0 || dev >= kMaxDev) return W4A8_ERR_DEVICE;
    unsigned long long ctx = 0;
    const int rc = current_ctx_id(&ctx);
    if (rc != W4A8_OK) return rc;
    *dev_out = dev;
    *ctx_out = ctx;
    *out = (g_fixed_ptr[dev] != nullptr && g_fixed_ctx[dev] == ctx) ? g_fixed_ptr[dev] : nullptr;
    return W4A8_OK;
}

int fixed_scratch(cudaStream_t st, uint8_t** out)
{
    std::lock_guard<std::mutex> lock(g_fixed_mutex);
    // The symbol lookup also makes the device's primary context current when
    // no call has done so yet, so it runs before the context is queried.
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_fixed_scratch);
    if (e != cudaSuccess) return fail_cuda(e);
    int dev = 0;
    unsigned long long ctx = 0;
    uint8_t* cur = nullptr;
    const int rc = fixed_scratch_cached(&dev, &ctx, &cur);
    if (rc != W4A8_OK) return rc;
    if (cur == nullptr) {
        if ((e = cudaMemsetAsync(ptr, 0, W4A8_FIXED_SCRATCH_BYTES, st)) != cudaSuccess) return fail_cuda(e);
        if ((e = cudaStreamSynchronize(st)) != cudaSuccess) return fail_cuda(e);
        g_fixed_ptr[dev] = static_cast<uint8_t*>(ptr);
        g_fixed_ctx[dev] = ctx;
        cur = g_fixed_ptr[dev];
    }
    *out = cur;
    return W4A8_OK;
}

// The launches of one linear call on a planned workspace: the GEMM with the
// quantiser fused in when the call allows it, else the standalone quantiser
// and then the GEMM.  Both give the same bits (same codes, scales and
// accumulation order).
int run_linear(const Plan& pl, const void* x, int64_t ldx, const Weights& w, void* y, int64_t ldy, uint8_t* ws,
               cudaStream_t st, bool swiglu)
{
    if (fused_quant_ok(pl, x, ldx, swiglu)) return run_gemm(pl, w, y, ldy, false, ws, st, x, ldx);
    const int rc = run_quant_kernel_layout(pl, x, ldx, ws, st, swiglu);
    if (rc != W4A8_OK) return rc;
    return run_gemm(pl, w, y, ldy, false, ws, st);
}

int linear_impl(const void* x, int64_t M, int64_t K, int64_t ldx, int64_t N, int32_t gk, const void* w_packed,
                const void* w_scale, int32_t ws_dtype, const void* w_zero, void* y, int64_t ldy, void* workspace,
                size_t workspace_bytes, void* stream, bool swiglu)
{
    int rc = check_common(M, N, K, gk);
    if (rc != W4A8_OK) return rc;
    if (M == 0) return W4A8_OK;
    if (!x || ldx < (swiglu ? 2 * K : K) || !aligned(x, 2)) return W4A8_ERR_INVALID;
    if ((rc = check_weights(w_packed, w_scale, ws_dtype, w_zero)) != W4A8_OK) return rc;
    if (!y || ldy < N || !aligned(y, 2)) return W4A8_ERR_INVALID;
    int sms = 0;
    if ((rc = device_info(&sms)) != W4A8_OK) return rc;
    const Plan pl = make_plan(M, N, K, gk, sms);
    if (!workspace || !aligned(workspace, 1024) || workspace_bytes < pl.total) return W4A8_ERR_WORKSPACE;
    const Weights w{w_packed, w_scale, w_zero, nullptr, false, ws_dtype};
    return run_linear(pl, x, ldx, w, y, ldy, static_cast<uint8_t*>(workspace), static_cast<cudaStream_t>(stream),
                      swiglu);
}

int linear_prepared_impl(const void* x, int64_t M, int64_t K, int64_t ldx, int64_t N, int32_t gk,
                         const void* prepared, int32_t ws_dtype, int32_t has_zero, void* y, int64_t ldy,
                         void* workspace, size_t workspace_bytes, void* stream, bool swiglu)
{
    int rc = check_common(M, N, K, gk);
    if (rc != W4A8_OK) return rc;
    if (M == 0) return W4A8_OK;
    if (!x || ldx < (swiglu ? 2 * K : K) || !aligned(x, 2)) return W4A8_ERR_INVALID;
    if (!prepared || !aligned(prepared, 256)) return W4A8_ERR_INVALID;
    if (ws_dtype != W4A8_DTYPE_BF16 && ws_dtype != W4A8_DTYPE_F32) return W4A8_ERR_UNSUPPORTED;
    if (!y || ldy < N || !aligned(y, 2)) return W4A8_ERR_INVALID;
    int sms = 0;
    if ((rc = device_info(&sms)) != W4A8_OK) return rc;
    const Plan pl = make_plan(M, N, K, gk, sms);
    if (!workspace || !aligned(workspace, 1024) || workspace_bytes < pl.total) return W4A8_ERR_WORKSPACE;
    const Weights w{nullptr, nullptr, nullptr, static_cast<const uint8_t*>(prepared), has_zero != 0, ws_dtype};
    return run_linear(pl, x, ldx, w, y, ldy, static_cast<uint8_t*>(workspace), static_cast<cudaStream_t>(stream),
                      swiglu);
}

}  // namespace

extern "C" {

int64_t w4a8_num_groups(int64_t K, int32_t gk) { return (K <= 0 || gk <= 0) ? 0 : cdiv(K, gk); }

int64_t w4a8_k_pad_elems(int64_t K, int32_t gk) { return (K <= 0 || gk <= 0) ? 0 : kpad_of(K, gk); }

int64_t w4a8_pad_rows(int64_t M)
{
    const int64_t t = M <= 16 ? 16 : (M <= 64 ? 64 : 128);
    return round_up(M, t);
}

size_t w4a8_linear_workspace_size(int64_t M, int64_t N, int64_t K, int32_t gk)
{
    if (check_common(M, N, K, gk) != W4A8_OK) return 0;
    int sms = 0;
    if (device_info(&sms) != W4A8_OK) sms = 148;
    return make_plan(std::max<int64_t>(M, 1), N, K, gk, sms).total;
}

size_t w4a8_midgroup_gemm_workspace_size(int64_t M, int64_t N, int64_t K, int32_t gk)
{
    return w4a8_linear_workspace_size(M, N, K, gk);
}

int w4a8_linear_quant(const void* x, int64_t M, int64_t K, int64_t ldx, int64_t N, int32_t gk, void* workspace,
                      size_t workspace_bytes, void* stream)
{
    int rc = check_common(M, N, K, gk);
    if (rc != W4A8_OK) return rc;
    if (M == 0) return W4A8_OK;
    if (!x || ldx < K || !aligned(x, 2)) return W4A8_ERR_INVALID;
    int sms = 0;
    if ((rc = device_info(&sms)) != W4A8_OK) return rc;
    const Plan pl = make_plan(M, N, K, gk, sms);
    if (!workspace || !aligned(workspace, 1024) || workspace_bytes < pl.total) return W4A8_ERR_WORKSPACE;
    return run_quant_kernel_layout(pl, x, ldx, static_cast<uint8_t*>(workspace), static_cast<cudaStream_t>(stream));
}

int w4a8_linear_gemm(int64_t M, int64_t K, int64_t N, int32_t gk, const void* w_packed, const void* w_scale,
                     int32_t ws_dtype, const void* w_zero, void* y, int64_t ldy, void* workspace,
                     size_t workspace_bytes, void* stream)
{
    int rc = check_common(M, N, K, gk);
    if (rc != W4A8_OK) return rc;
    if (M == 0) return W4A8_OK;
    if ((rc = check_weights(w_packed, w_scale, ws_dtype, w_zero)) != W4A8_OK) return rc;
    if (!y || ldy < N || !aligned(y, 2)) return W4A8_ERR_INVALID;
    int sms = 0;
    if ((rc = device_info(&sms)) != W4A8_OK) return rc;
    const Plan pl = make_plan(M, N, K, gk, sms);
    if (!workspace || !aligned(workspace, 1024) || workspace_bytes < pl.total) return W4A8_ERR_WORKSPACE;
    const Weights w{w_packed, w_scale, w_zero, nullptr, false, ws_dtype};
    return run_gemm(pl, w, y, ldy, false, static_cast<uint8_t*>(workspace), static_cast<cudaStream_t>(stream));
}

int w4a8_linear(const void* x, int64_t M, int64_t K, int64_t ldx, int64_t N, int32_t gk, const void* w_packed,
                const void* w_scale, int32_t ws_dtype, const void* w_zero, void* y, int64_t ldy, void* workspace,
                size_t workspace_bytes, void* stream)
{
    return linear_impl(x, M, K, ldx, N, gk, w_packed, w_scale, ws_dtype, w_zero, y, ldy, workspace,
                       workspace_bytes, stream, false);
}

int w4a8_linear_swiglu(const void* gu, int64_t M, int64_t K, int64_t ldx, int64_t N, int32_t gk,
                       const void* w_packed, const void* w_scale, int32_t ws_dtype, const void* w_zero, void* y,
                       int64_t ldy, void* workspace, size_t workspace_bytes, void* stream)
{
    return linear_impl(gu, M, K, ldx, N, gk, w_packed, w_scale, ws_dtype, w_zero, y, ldy, workspace,
                       workspace_bytes, stream, true);
}

int w4a8_linear_fixed_scratch(const void* x, int64_t M, int64_t K, int64_t ldx, int64_t N, int32_t gk,
                              const void* w_packed, const void* w_scale, int32_t ws_dtype, const void* w_zero, void* y,
                              int64_t ldy, void* stream)
{
    int rc = check_common(M, N, K, gk);
    if (rc != W4A8_OK) return rc;
    if (M == 0) return W4A8_OK;
    if (!x || ldx < K || !aligned(x, 2)) return W4A8_ERR_INVALID;
    if ((rc = check_weights(w_packed, w_scale, ws_dtype, w_zero)) != W4A8_OK) return rc;
    if (!y || ldy < N || !aligned(y, 2)) return W4A8_ERR_INVALID;
    int sms = 0;
    if ((rc = device_info(&sms)) != W4A8_OK) return rc;
    const Plan pl = make_plan(M, N, K, gk, sms);
    if (pl.total > W4A8_FIXED_SCRATCH_BYTES) return W4A8_ERR_WORKSPACE;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint8_t* ws = nullptr;
    if ((rc = fixed_scratch(st, &ws)) != W4A8_OK) return rc;
    const Weights w{w_packed, w_scale, w_zero, nullptr, false, ws_dtype};
    return run_linear(pl, x, ldx, w, y, ldy, ws, st, false);
}

int w4a8_fixed_scratch_status(int32_t reset, void* stream)
{
    uint8_t* ptr = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_fixed_mutex);
        int dev = 0;
        unsigned long long ctx = 0;
        const int rc = fixed_scratch_cached(&dev, &ctx, &ptr);
        if (rc != W4A8_OK) return rc;
    }
    if (ptr == nullptr) return W4A8_ERR_WORKSPACE;   // no call has run in this context
    return w4a8_workspace_status(ptr, reset, stream);
}

int w4a8_group_partials(const void* x, int64_t M, int64_t K, int64_t ldx, int64_t N, int32_t gk,
                        const void* w_packed, const void* w_zero, int32_t* partials, void* workspace,
                        size_t workspace_bytes, void* stream)
{
    int rc = check_common(M, N, K, gk);
    if (rc != W4A8_OK) return rc;
    if (M == 0) return W4A8_OK;
    if (!x || ldx < K || !aligned(x, 2) || !partials) return W4A8_ERR_INVALID;
    if (!w_packed || !aligned(w_packed, 16) || (w_zero && !aligned(w_zero, 16))) return W4A8_ERR_INVALID;
    int sms = 0;
    if ((rc = device_info(&sms)) != W4A8_OK) return rc;
    const Plan pl = make_plan(M, N, K, gk, sms, 16);
    if (!workspace || !aligned(workspace, 1024) || workspace_bytes < pl.total) return W4A8_ERR_WORKSPACE;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if ((rc = run_quant_kernel_layout(pl, x, ldx, ws, st)) != W4A8_OK) return rc;
    const Weights w{w_packed, nullptr, w_zero, nullptr, false, W4A8_DTYPE_F32};
    return run_gemm(pl, w, partials, N, true, ws, st);
}

int w4a8_quant_act(const void* x, int64_t M, int64_t K, int64_t ldx, int32_t gk, int8_t* a_q, void* a_scale,
                   int32_t scale_dtype, int32_t* a_ksum, void* stream)
{
    if (M < 0 || K <= 0 || !group_ok(gk)) return M < 0 || K <= 0 ? W4A8_ERR_INVALID : W4A8_ERR_UNSUPPORTED;
    if (M == 0) return W4A8_OK;
    if (!x || !a_q || !a_scale || ldx < K || !aligned(x, 2)) return W4A8_ERR_INVALID;
    if (scale_dtype != W4A8_DTYPE_BF16 && scale_dtype != W4A8_DTYPE_F32) return W4A8_ERR_UNSUPPORTED;
    int sms = 0;
    int rc = device_info(&sms);
    if (rc != W4A8_OK) return rc;
    QuantParams q{};
    q.x = static_cast<const uint16_t*>(x);
    q.ldx = ldx;
    q.M = static_cast<int>(M);
    q.K = static_cast<int>(K);
    q.Kpad = static_cast<int>(kpad_of(K, gk));
    q.G = static_cast<int>(cdiv(K, gk));
    q.gk = gk;
    q.rows = static_cast<int>(M);
    q.vec_ok = aligned(x, 16) && (K % 8 == 0) && (ldx % 8 == 0);
    q.q = a_q;
    q.scale = a_scale;
    q.scale_f32 = scale_dtype == W4A8_DTYPE_F32;
    q.ksum = a_ksum;
    const cudaError_t e = launch_quant_act(q, kOutPublic, static_cast<cudaStream_t>(stream), true);
    return e == cudaSuccess ? W4A8_OK : fail_cuda(e);
}

int w4a8_midgroup_quant_a(const void* x, int64_t M, int64_t K, int32_t gk, int64_t Mp, int8_t* a_hi, int8_t* a_lo,
                          void* a_scale, int32_t* a_ksum, void* stream)
{
    if (M < 0 || K <= 0 || Mp < M) return W4A8_ERR_INVALID;
    if (!group_ok(gk)) return W4A8_ERR_UNSUPPORTED;
    if (Mp == 0) return W4A8_OK;
    if (!x || !a_hi || !a_lo || !a_scale || !a_ksum || !aligned(x, 2)) return W4A8_ERR_INVALID;
    if (!aligned(a_hi, 4) || !aligned(a_lo, 4) || !aligned(a_scale, 2) || !aligned(a_ksum, 4)) return W4A8_ERR_INVALID;
    int sms = 0;
    int rc = device_info(&sms);
    if (rc != W4A8_OK) return rc;
    QuantParams q{};
    q.x = static_cast<const uint16_t*>(x);
    q.ldx = K;
    q.M = static_cast<int>(M);
    q.K = static_cast<int>(K);
    q.Kpad = static_cast<int>(kpad_of(K, gk));
    q.G = static_cast<int>(cdiv(K, gk));
    q.gk = gk;
    q.rows = static_cast<int>(Mp);
    q.vec_ok = aligned(x, 16) && (K % 8 == 0);
    q.a_hi = a_hi;
    q.a_lo = a_lo;
    q.a_scale = static_cast<uint16_t*>(a_scale);
    q.a_ksum = a_ksum;
    const cudaError_t e = launch_quant_act(q, kOutMsd, static_cast<cudaStream_t>(stream), true);
    return e == cudaSuccess ? W4A8_OK : fail_cuda(e);
}

int w4a8_midgroup_w4a8_gemm(const int8_t* a_hi, const int8_t* a_lo, const void* a_scale, const int32_t* a_ksum,
                            int64_t M, const int8_t* w_q, const void* w_scale, const int32_t* w_ksum,
                            const void* w_zero, int64_t N, int64_t K, int32_t gk, void* y, void* workspace,
                            size_t workspace_bytes, void* stream)
{
    (void)a_ksum;
    (void)w_ksum;
    int rc = check_common(M, N, K, gk);
    if (rc != W4A8_OK) return rc;
    if (M == 0) return W4A8_OK;
    if (!a_hi || !a_lo || !a_scale || !y || !aligned(a_hi, 4) || !aligned(a_lo, 4) || !aligned(a_scale, 2))
        return W4A8_ERR_INVALID;
    if ((rc = check_weights(w_q, w_scale, W4A8_DTYPE_BF16, w_zero)) != W4A8_OK) return rc;
    int sms = 0;
    if ((rc = device_info(&sms)) != W4A8_OK) return rc;
    const Plan pl = make_plan(M, N, K, gk, sms);
    if (!workspace || !aligned(workspace, 1024) || workspace_bytes < pl.total) return W4A8_ERR_WORKSPACE;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    MsdToKernelParams m{};
    m.a_hi = a_hi;
    m.a_lo = a_lo;
    m.a_scale = static_cast<const uint16_t*>(a_scale);
    m.scale_ld = static_cast<int>(M);
    m.M = static_cast<int>(M);
    m.Kpad = static_cast<int>(pl.Kpad);
    m.G = static_cast<int>(pl.G);
    m.gk = gk;
    m.rows = pl.n_tt * pl.tt;
    m.aq = reinterpret_cast<int8_t*>(ws + pl.off_aq);
    m.as = reinterpret_cast<float*>(ws + pl.off_as);
    m.tt = pl.tt;
    m.kb_total = pl.kb_total;
    cudaError_t e = launch_msd_to_kernel(m, st, true);
    if (e != cudaSuccess) return fail_cuda(e);
    const Weights w{w_q, w_scale, w_zero, nullptr, false, W4A8_DTYPE_BF16};
    return run_gemm(pl, w, y, N, false, ws, st);
}

size_t w4a8_prepared_weights_size(int64_t N, int64_t K, int32_t gk, int32_t ws_dtype, int32_t has_zero)
{
    if (N <= 0 || K <= 0 || !group_ok(gk) || N % 8 != 0) return 0;
    if (ws_dtype != W4A8_DTYPE_BF16 && ws_dtype != W4A8_DTYPE_F32) return 0;
    const int64_t Kpad = kpad_of(K, gk);
    return static_cast<size_t>(prepared_layout(N, cdiv(K, gk), static_cast<int>(cdiv(Kpad, 256)),
                                               ws_dtype == W4A8_DTYPE_F32 ? 4 : 2, has_zero != 0).total);
}

int w4a8_prepare_weights(const void* w_packed, const void* w_scale, int32_t ws_dtype, const void* w_zero, int64_t N,
                         int64_t K, int32_t gk, void* out, size_t out_bytes, void* stream)
{
    int rc = check_common(1, N, K, gk);
    if (rc != W4A8_OK) return rc;
    if ((rc = check_weights(w_packed, w_scale, ws_dtype, w_zero)) != W4A8_OK) return rc;
    const size_t need = w4a8_prepared_weights_size(N, K, gk, ws_dtype, w_zero != nullptr);
    if (!out || !aligned(out, 256) || out_bytes < need) return W4A8_ERR_INVALID;
    PrepareParams p{};
    p.w_packed = static_cast<const uint8_t*>(w_packed);
    p.w_scale = static_cast<const uint8_t*>(w_scale);
    p.w_zero = static_cast<const uint16_t*>(w_zero);
    p.out = static_cast<uint8_t*>(out);
    p.N = static_cast<int>(N);
    p.Kpad = static_cast<int>(kpad_of(K, gk));
    p.G = static_cast<int>(cdiv(K, gk));
    p.kb_total = static_cast<int>(cdiv(p.Kpad, 256));
    p.ws_elt = ws_dtype == W4A8_DTYPE_F32 ? 4 : 2;
    const cudaError_t e = launch_prepare_weights(p, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? W4A8_OK : fail_cuda(e);
}

int w4a8_linear_prepared(const void* x, int64_t M, int64_t K, int64_t ldx, int64_t N, int32_t gk, const void* prepared,
                         int32_t ws_dtype, int32_t has_zero, void* y, int64_t ldy, void* workspace,
                         size_t workspace_bytes, void* stream)
{
    return linear_prepared_impl(x, M, K, ldx, N, gk, prepared, ws_dtype, has_zero, y, ldy, workspace,
                                workspace_bytes, stream, false);
}

int w4a8_linear_prepared_swiglu(const void* gu, int64_t M, int64_t K, int64_t ldx, int64_t N, int32_t gk,
                                const void* prepared, int32_t ws_dtype, int32_t has_zero, void* y, int64_t ldy,
                                void* workspace, size_t workspace_bytes, void* stream)
{
    return linear_prepared_impl(gu, M, K, ldx, N, gk, prepared, ws_dtype, has_zero, y, ldy, workspace,
                                workspace_bytes, stream, true);
}

int w4a8_linear_prepared_allreduce(const void* x, int64_t M, int64_t K, int64_t ldx, int64_t N, int32_t gk,
                                   const void* prepared, int32_t ws_dtype, int32_t has_zero, int32_t act, void* y,
                                   void* workspace, size_t workspace_bytes, w4a8_ar* ar, void* stream)
{
    int rc = check_common(M, N, K, gk);
    if (rc != W4A8_OK) return rc;
    if (act != W4A8_ACT_NONE && act != W4A8_ACT_SWIGLU) return W4A8_ERR_UNSUPPORTED;
    if (!ar) return W4A8_ERR_INVALID;
    const bool swiglu = act == W4A8_ACT_SWIGLU;
    if (M == 0) return W4A8_OK;
    if (!x || ldx < (swiglu ? 2 * K : K) || !aligned(x, 2)) return W4A8_ERR_INVALID;
    if (!prepared || !aligned(prepared, 256)) return W4A8_ERR_INVALID;
    if (ws_dtype != W4A8_DTYPE_BF16 && ws_dtype != W4A8_DTYPE_F32) return W4A8_ERR_UNSUPPORTED;
    // y is the reduced [M, N] message: dense, 16-byte aligned, whole 8-element vectors
    if (!y || !aligned(y, 16) || (M * N) % 8 != 0) return W4A8_ERR_INVALID;
    PushParams pp;
    const bool pull = !(g_options & W4A8_OPT_AR_PUSH);
    if ((rc = ar_push_params(ar, static_cast<size_t>(M) * N * 2, pull, &pp)) != W4A8_OK) return rc;
    int sms = 0;
    if ((rc = device_info(&sms)) != W4A8_OK) return rc;
    const Plan pl = make_plan(M, N, K, gk, sms);
    if (!workspace || !aligned(workspace, 1024) || workspace_bytes < pl.total) return W4A8_ERR_WORKSPACE;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if ((rc = run_quant_kernel_layout(pl, x, ldx, ws, st, swiglu)) != W4A8_OK) return rc;
    const Weights w{nullptr, nullptr, nullptr, static_cast<const uint8_t*>(prepared), has_zero != 0, ws_dtype};
    if ((rc = run_gemm(pl, w, nullptr, N, false, ws, st, nullptr, 0, &pp)) != W4A8_OK) return rc;
    const cudaError_t e = ar_launch_reduce_pushed(ar, y, M * N, pull, st);
    return e == cudaSuccess ? W4A8_OK : fail_cuda(e);
}

int w4a8_linear_gemm_prepared(int64_t M, int64_t K, int64_t N, int32_t gk, const void* prepared, int32_t ws_dtype,
                              int32_t has_zero, void* y, int64_t ldy, void* workspace, size_t workspace_bytes,
                              void* stream)
{
    int rc = check_common(M, N, K, gk);
    if (rc != W4A8_OK) return rc;
    if (M == 0) return W4A8_OK;
    if (!prepared || !aligned(prepared, 256) || !y || ldy < N || !aligned(y, 2)) return W4A8_ERR_INVALID;
    if (ws_dtype != W4A8_DTYPE_BF16 && ws_dtype != W4A8_DTYPE_F32) return W4A8_ERR_UNSUPPORTED;
    int sms = 0;
    if ((rc = device_info(&sms)) != W4A8_OK) return rc;
    const Plan pl = make_plan(M, N, K, gk, sms);
    if (!workspace || !aligned(workspace, 1024) || workspace_bytes < pl.total) return W4A8_ERR_WORKSPACE;
    const Weights w{nullptr, nullptr, nullptr, static_cast<const uint8_t*>(prepared), has_zero != 0, ws_dtype};
    return run_gemm(pl, w, y, ldy, false, static_cast<uint8_t*>(workspace), static_cast<cudaStream_t>(stream));
}

int w4a8_workspace_status(void* workspace, int32_t reset, void* stream)
{
    if (!workspace) return W4A8_ERR_WORKSPACE;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    int v = 0;
    cudaError_t e = cudaMemcpyAsync(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return fail_cuda(e);
    if (reset && v != 0) {
        e = cudaMemsetAsync(workspace, 0, sizeof(int), st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) return fail_cuda(e);
    }
    return v;
}

const char* w4a8_status_string(int s)
{
    switch (s) {
        case W4A8_OK: return "ok";
        case W4A8_ERR_INVALID: return "invalid argument (shape, null or misaligned pointer)";
        case W4A8_ERR_UNSUPPORTED: return "unsupported group size or dtype";
        case W4A8_ERR_CUDA: return "CUDA call failed (see w4a8_last_cuda_error)";
        case W4A8_ERR_WORKSPACE: return "workspace missing, misaligned or too small";
        case W4A8_ERR_DEVICE: return "current device is not an sm_100 GPU";
        case W4A8_ERR_TIMEOUT: return "a device-side wait on a peer rank timed out";
        default: return s >= 0x100 ? "a kernel pipeline wait timed out" : "unknown status";
    }
}

int w4a8_last_cuda_error(void) { return g_last_cuda; }

int w4a8_build_arch(void) { return 100; }

int w4a8_set_options(int32_t flags)
{
    const int old = g_options;
    g_options = flags;
    return old;
}

}  // extern "C"
