// w4a8_allreduce.cu -- one-shot all-reduce for small bf16 messages over peer memory.
//
// The row-parallel layers of the tensor-parallel stack sum [M, hidden] bf16
// partials across ranks twice per layer.  At decode sizes (M <= 64: 10-640 KB)
// that is latency-bound, and a one-shot exchange over NVLink peer memory beats
// a ring: every rank pushes its message into every peer's buffer once, each
// rank sums the world messages it holds in fp32 in a fixed rank order (so all
// ranks hold identical bits) and writes its own output.  The reference does
// the same on its hardware with a peer-read kernel and device flags
// (npu_ops/kernel/peer_allreduce_f32.cpp:1-67, 127-270); writes are used here
// because NVLink stores are posted, while a remote load waits a round trip.
//
// Memory: each rank allocates one buffer holding two banks of `world` message
// slots (one per source rank) and a flag row per source rank and block; the
// buffers are mapped into every peer with CUDA IPC.  Plain loads and stores
// only (no multicast, no bulk copies).
//
// Per call and per block b (all ranks call in the same order with the same
// count; each block keeps its own call counter in device memory, so calls
// replay correctly inside CUDA graphs; every call runs all kMaxBlocks blocks,
// so the counters advance together):
//   1. store this rank's slice b into slot [bank seq & 1][my_rank] of every
//      rank's buffer (its own included);
//   2. store seq into flag[my_rank][b] of every rank with release semantics
//      (system scope);
//   3. wait (acquire) until every flag[src][b] in this rank's buffer reaches
//      seq -- bounded: after the time limit the block records an error in the
//      status word and returns without touching the output;
//   4. sum slice b of the `world` local slots of the bank in rank order, store bf16.
// Two banks make a closing barrier unnecessary: a rank writes bank s of a peer
// again only two calls later, after the next call's step 3 has shown that the
// peer has started that call, i.e. finished reading this one.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <new>

#include "w4a8_b200.h"
#include "w4a8_kernels.h"

namespace {

constexpr int kMaxRanks = 8;
constexpr int kMaxBlocks = 32;           // measured: 16 best at M = 1, 64 best at M = 64
constexpr int kThreads = 512;
constexpr uint64_t kWaitNs = 1000000000ull;      // 1 s per wait

struct Layout {
    size_t slot_bytes;     // one message slot (multiple of 256)
    size_t bank_bytes;     // kMaxRanks slots
    size_t off_flags;      // uint32 [kMaxRanks][kMaxBlocks] written by the source ranks
    size_t off_counter;    // uint32 [kMaxBlocks] calls made, per block (local)
    size_t off_status;     // int32
    size_t total;
};

Layout layout_for(size_t max_bytes, int world)
{
    Layout l;
    l.slot_bytes = (max_bytes + 255) / 256 * 256;
    l.bank_bytes = l.slot_bytes * world;
    l.off_flags = 2 * l.bank_bytes;
    l.off_counter = l.off_flags + sizeof(uint32_t) * kMaxRanks * kMaxBlocks;
    l.off_status = l.off_counter + sizeof(uint32_t) * kMaxBlocks;
    l.total = (l.off_status + 256 + 255) / 256 * 256;
    return l;
}

struct Params {
    uint8_t* base[kMaxRanks];      // every rank's buffer as mapped in this process (own included)
    const __nv_bfloat16* in;
    __nv_bfloat16* out;
    int64_t count;                 // elements
    int64_t per_block;             // elements per block (multiple of 8)
    size_t slot_bytes, bank_bytes;
    size_t off_flags, off_counter, off_status;
    int rank, world;
};

__device__ __forceinline__ uint64_t now_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void store_release_sys(uint32_t* p, uint32_t v)
{
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t load_acquire_sys(const uint32_t* p)
{
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

template <int W>
__global__ void __launch_bounds__(kThreads) allreduce_oneshot_bf16(const Params p)
{
    const int b = blockIdx.x;
    uint8_t* mine = p.base[p.rank];
    uint32_t* counter = reinterpret_cast<uint32_t*>(mine + p.off_counter) + b;
    __shared__ uint32_t s_seq;
    __shared__ int s_abort;
    if (threadIdx.x == 0) {
        s_seq = *counter + 1u;
        s_abort = 0;
    }
    __syncthreads();
    const uint32_t seq = s_seq;
    const size_t bank_off = (seq & 1u) * p.bank_bytes;
    const int64_t e0 = static_cast<int64_t>(b) * p.per_block < p.count ? static_cast<int64_t>(b) * p.per_block : p.count;
    const int64_t e1 = e0 + p.per_block < p.count ? e0 + p.per_block : p.count;   // e0 <= e1 <= count
    const int64_t v0 = e0 / 8, v1 = e1 / 8;                                        // 16-byte vectors

    // 1. push this rank's slice into slot [bank][rank] of every rank (posted stores)
    {
        const uint4* src = reinterpret_cast<const uint4*>(p.in);
        const size_t slot = bank_off + static_cast<size_t>(p.rank) * p.slot_bytes;
        for (int64_t i = v0 + threadIdx.x; i < v1; i += blockDim.x) {
            const uint4 v = src[i];
#pragma unroll
            for (int r = 0; r < W; ++r) reinterpret_cast<uint4*>(p.base[r] + slot)[i] = v;
        }
    }
    __syncthreads();
    // 2. publish: one release store per rank.  The CTA barrier above orders the
    //    block's data stores before the signalling thread's release (causality
    //    order is transitive across the barrier and the system-scope release),
    //    so no separate fence is needed; measured, a __threadfence_system()
    //    here cost ~3.5 us per call.
    if (threadIdx.x < W) {
        uint32_t* f = reinterpret_cast<uint32_t*>(p.base[threadIdx.x] + p.off_flags) + p.rank * kMaxBlocks + b;
        store_release_sys(f, seq);
    }
    // 3. every source's slice of this call has arrived here (bounded wait)
    if (threadIdx.x < W) {
        const uint32_t* f = reinterpret_cast<const uint32_t*>(mine + p.off_flags) + threadIdx.x * kMaxBlocks + b;
        const uint64_t t0 = now_ns();
        while (static_cast<int32_t>(load_acquire_sys(f) - seq) < 0) {
            if (now_ns() - t0 > kWaitNs) {
                atomicCAS(reinterpret_cast<int*>(mine + p.off_status), 0, 1);
                s_abort = 1;
                break;
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) *counter = seq;
    if (s_abort) return;
    // 4. fixed-order fp32 sum of the world local slots
    const uint8_t* bank = mine + bank_off;
    for (int64_t i = v0 + threadIdx.x; i < v1; i += blockDim.x) {
        uint4 v[W];
#pragma unroll
        for (int r = 0; r < W; ++r) v[r] = reinterpret_cast<const uint4*>(bank + static_cast<size_t>(r) * p.slot_bytes)[i];
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
        for (int r = 0; r < W; ++r) {
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[r]);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 f = __bfloat1622float2(h[j]);
                acc[2 * j] += f.x;
                acc[2 * j + 1] += f.y;
            }
        }
        uint4 o;
        __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
        for (int j = 0; j < 4; ++j) oh[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
        reinterpret_cast<uint4*>(p.out)[i] = o;
    }
}

// The reduction half of the fused row-parallel linear: the GEMM (and its
// stream-K fix-up) already stored this rank's message into slot [bank][rank]
// of every rank (PushParams), so the push pass of the one-shot kernel is gone.
// Per block b: wait for the pushing kernels to finish (programmatic dependent
// launch), make their peer stores visible system-wide, publish seq into
// flag[rank][b] of every rank, wait (bounded) for every source's flag, then sum
// slice b of the bank in rank order.  The same bank, flag and counter protocol
// as allreduce_oneshot_bf16, so pushed and ordinary calls can interleave.
// PULL: every rank's GEMM wrote only its own slot (locally), so the sum reads
// slot [bank][r] from rank r's buffer (peer loads) instead of from this rank's.
template <int W, bool PULL>
__global__ void __launch_bounds__(kThreads) allreduce_pushed_bf16(const Params p)
{
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int b = blockIdx.x;
    uint8_t* mine = p.base[p.rank];
    uint32_t* counter = reinterpret_cast<uint32_t*>(mine + p.off_counter) + b;
    __shared__ uint32_t s_seq;
    __shared__ int s_abort;
    if (threadIdx.x == 0) {
        s_seq = *counter + 1u;
        s_abort = 0;
    }
    __syncthreads();
    const uint32_t seq = s_seq;
    const size_t bank_off = (seq & 1u) * p.bank_bytes;
    const int64_t e0 = static_cast<int64_t>(b) * p.per_block < p.count ? static_cast<int64_t>(b) * p.per_block : p.count;
    const int64_t e1 = e0 + p.per_block < p.count ? e0 + p.per_block : p.count;
    const int64_t v0 = e0 / 8, v1 = e1 / 8;
    if (threadIdx.x < W) {
        // Push: the previous grids stored into peers' memory over NVLink; a
        // system-scope fence orders those stores before this release.  Pull:
        // the stores were local and had reached this GPU's L2 when the grid
        // completed, and peers read them there after acquiring the flag, so the
        // fence (several microseconds per call, measured) is not needed.
        if (!PULL) __threadfence_system();
        uint32_t* f = reinterpret_cast<uint32_t*>(p.base[threadIdx.x] + p.off_flags) + p.rank * kMaxBlocks + b;
        store_release_sys(f, seq);
        const uint32_t* g = reinterpret_cast<const uint32_t*>(mine + p.off_flags) + threadIdx.x * kMaxBlocks + b;
        const uint64_t t0 = now_ns();
        while (static_cast<int32_t>(load_acquire_sys(g) - seq) < 0) {
            if (now_ns() - t0 > kWaitNs) {
                atomicCAS(reinterpret_cast<int*>(mine + p.off_status), 0, 1);
                s_abort = 1;
                break;
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) *counter = seq;
    if (s_abort) return;
    for (int64_t i = v0 + threadIdx.x; i < v1; i += blockDim.x) {
        uint4 v[W];
#pragma unroll
        for (int r = 0; r < W; ++r) {
            const uint8_t* src = (PULL ? p.base[r] : mine) + bank_off + static_cast<size_t>(r) * p.slot_bytes;
            v[r] = PULL ? __ldcv(reinterpret_cast<const uint4*>(src) + i) : reinterpret_cast<const uint4*>(src)[i];
        }
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
        for (int r = 0; r < W; ++r) {
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[r]);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 f = __bfloat1622float2(h[j]);
                acc[2 * j] += f.x;
                acc[2 * j + 1] += f.y;
            }
        }
        uint4 o;
        __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
        for (int j = 0; j < 4; ++j) oh[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
        reinterpret_cast<uint4*>(p.out)[i] = o;
    }
}

}  // namespace

struct w4a8_ar {
    int rank = 0, world = 1, dev = 0;
    size_t max_bytes = 0;
    Layout lay{};
    uint8_t* local = nullptr;               // own allocation
    uint8_t* mapped[kMaxRanks] = {};        // peers' allocations opened here
    bool ipc[kMaxRanks] = {};               // mapped[r] came from cudaIpcOpenMemHandle
    bool opened = false;
};

namespace {

Params make_params(const w4a8_ar* h, const void* in, void* out, int64_t count)
{
    Params p{};
    for (int r = 0; r < h->world; ++r) p.base[r] = h->mapped[r];
    p.in = static_cast<const __nv_bfloat16*>(in);
    p.out = static_cast<__nv_bfloat16*>(out);
    p.count = count;
    // Always kMaxBlocks blocks (trailing slices may be empty): every block
    // then advances its call counter on every call, so all blocks of a call
    // share one sequence number and the slot parity alternates uniformly
    // whatever the message sizes of successive calls.
    p.per_block = ((count + kMaxBlocks - 1) / kMaxBlocks + 7) / 8 * 8;
    p.slot_bytes = h->lay.slot_bytes;
    p.bank_bytes = h->lay.bank_bytes;
    p.off_flags = h->lay.off_flags;
    p.off_counter = h->lay.off_counter;
    p.off_status = h->lay.off_status;
    p.rank = h->rank;
    p.world = h->world;
    return p;
}

}  // namespace

namespace w4a8 {

int ar_push_params(const w4a8_ar* h, size_t bytes, bool pull, PushParams* out)
{
    if (!h || !out || bytes > h->max_bytes || (h->world > 1 && !h->opened)) return W4A8_ERR_INVALID;
    PushParams q{};
    // pull: the GEMM writes only this rank's own slot (one destination, local)
    q.world = pull ? 1 : h->world;
    for (int r = 0; r < q.world; ++r) q.base[r] = pull ? h->local : h->mapped[r];
    q.counter = reinterpret_cast<const uint32_t*>(h->local + h->lay.off_counter);
    q.slot_bytes = h->lay.slot_bytes;
    q.bank_bytes = h->lay.bank_bytes;
    q.rank = h->rank;
    *out = q;
    return W4A8_OK;
}

cudaError_t ar_launch_reduce_pushed(w4a8_ar* h, void* out, int64_t count, bool pull, cudaStream_t st)
{
    const Params p = make_params(h, nullptr, out, count);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kMaxBlocks);
    cfg.blockDim = dim3(kThreads);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (pull) {
        switch (h->world) {
            case 1: return cudaLaunchKernelEx(&cfg, allreduce_pushed_bf16<1, true>, p);
            case 2: return cudaLaunchKernelEx(&cfg, allreduce_pushed_bf16<2, true>, p);
            case 3: return cudaLaunchKernelEx(&cfg, allreduce_pushed_bf16<3, true>, p);
            case 4: return cudaLaunchKernelEx(&cfg, allreduce_pushed_bf16<4, true>, p);
            case 5: return cudaLaunchKernelEx(&cfg, allreduce_pushed_bf16<5, true>, p);
            case 6: return cudaLaunchKernelEx(&cfg, allreduce_pushed_bf16<6, true>, p);
            case 7: return cudaLaunchKernelEx(&cfg, allreduce_pushed_bf16<7, true>, p);
            default: return cudaLaunchKernelEx(&cfg, allreduce_pushed_bf16<8, true>, p);
        }
    }
    switch (h->world) {
        case 1: return cudaLaunchKernelEx(&cfg, allreduce_pushed_bf16<1, false>, p);
        case 2: return cudaLaunchKernelEx(&cfg, allreduce_pushed_bf16<2, false>, p);
        case 3: return cudaLaunchKernelEx(&cfg, allreduce_pushed_bf16<3, false>, p);
        case 4: return cudaLaunchKernelEx(&cfg, allreduce_pushed_bf16<4, false>, p);
        case 5: return cudaLaunchKernelEx(&cfg, allreduce_pushed_bf16<5, false>, p);
        case 6: return cudaLaunchKernelEx(&cfg, allreduce_pushed_bf16<6, false>, p);
        case 7: return cudaLaunchKernelEx(&cfg, allreduce_pushed_bf16<7, false>, p);
        default: return cudaLaunchKernelEx(&cfg, allreduce_pushed_bf16<8, false>, p);
    }
}

}  // namespace w4a8

extern "C" {

size_t w4a8_ar_ipc_handle_size(void) { return sizeof(cudaIpcMemHandle_t); }

int w4a8_ar_create(int32_t rank, int32_t world, size_t max_bytes, w4a8_ar** out)
{
    if (!out || world < 1 || world > kMaxRanks || rank < 0 || rank >= world || max_bytes == 0 ||
        max_bytes % 16)
        return W4A8_ERR_INVALID;
    w4a8_ar* h = new (std::nothrow) w4a8_ar();
    if (!h) return W4A8_ERR_CUDA;
    h->rank = rank;
    h->world = world;
    h->max_bytes = max_bytes;
    h->lay = layout_for(max_bytes, world);
    if (cudaGetDevice(&h->dev) != cudaSuccess || cudaMalloc(&h->local, h->lay.total) != cudaSuccess ||
        cudaMemset(h->local, 0, h->lay.total) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        if (h->local) cudaFree(h->local);
        delete h;
        return W4A8_ERR_CUDA;
    }
    h->mapped[rank] = h->local;
    *out = h;
    return W4A8_OK;
}

int w4a8_ar_ipc_handle(w4a8_ar* h, void* handle_out)
{
    if (!h || !handle_out) return W4A8_ERR_INVALID;
    cudaIpcMemHandle_t m;
    if (cudaIpcGetMemHandle(&m, h->local) != cudaSuccess) return W4A8_ERR_CUDA;
    memcpy(handle_out, &m, sizeof(m));
    return W4A8_OK;
}

int w4a8_ar_open_peers(w4a8_ar* h, const void* handles)
{
    if (!h || (!handles && h->world > 1)) return W4A8_ERR_INVALID;
    if (h->opened) return W4A8_OK;
    for (int r = 0; r < h->world; ++r) {
        if (r == h->rank) continue;
        cudaIpcMemHandle_t m;
        memcpy(&m, static_cast<const uint8_t*>(handles) + r * sizeof(m), sizeof(m));
        void* p = nullptr;
        if (cudaIpcOpenMemHandle(&p, m, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return W4A8_ERR_CUDA;
        h->mapped[r] = static_cast<uint8_t*>(p);
        h->ipc[r] = true;
    }
    h->opened = true;
    return W4A8_OK;
}

int w4a8_ar_open_local(w4a8_ar* h, w4a8_ar* const* peers)
{
    if (!h || (!peers && h->world > 1)) return W4A8_ERR_INVALID;
    if (h->opened) return W4A8_OK;
    for (int r = 0; r < h->world; ++r) {
        if (r == h->rank) continue;
        const w4a8_ar* q = peers[r];
        if (!q || q->rank != r || q->world != h->world || q->max_bytes != h->max_bytes) return W4A8_ERR_INVALID;
        if (q->dev != h->dev) {
            int ok = 0;
            if (cudaDeviceCanAccessPeer(&ok, h->dev, q->dev) != cudaSuccess || !ok) return W4A8_ERR_CUDA;
            const cudaError_t e = cudaDeviceEnablePeerAccess(q->dev, 0);
            if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) return W4A8_ERR_CUDA;
            cudaGetLastError();
        }
        h->mapped[r] = q->local;
    }
    h->opened = true;
    return W4A8_OK;
}

size_t w4a8_ar_max_bytes(const w4a8_ar* h) { return h ? h->max_bytes : 0; }

int w4a8_ar_allreduce_bf16(w4a8_ar* h, const void* in, void* out, int64_t count, void* stream)
{
    if (!h || !in || !out || count < 0) return W4A8_ERR_INVALID;
    if (count == 0) return W4A8_OK;
    if (count % 8 || static_cast<size_t>(count) * 2 > h->max_bytes) return W4A8_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15) return W4A8_ERR_INVALID;
    if (h->world > 1 && !h->opened) return W4A8_ERR_INVALID;
    const Params p = make_params(h, in, out, count);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (h->world) {
        case 1: allreduce_oneshot_bf16<1><<<kMaxBlocks, kThreads, 0, st>>>(p); break;
        case 2: allreduce_oneshot_bf16<2><<<kMaxBlocks, kThreads, 0, st>>>(p); break;
        case 3: allreduce_oneshot_bf16<3><<<kMaxBlocks, kThreads, 0, st>>>(p); break;
        case 4: allreduce_oneshot_bf16<4><<<kMaxBlocks, kThreads, 0, st>>>(p); break;
        case 5: allreduce_oneshot_bf16<5><<<kMaxBlocks, kThreads, 0, st>>>(p); break;
        case 6: allreduce_oneshot_bf16<6><<<kMaxBlocks, kThreads, 0, st>>>(p); break;
        case 7: allreduce_oneshot_bf16<7><<<kMaxBlocks, kThreads, 0, st>>>(p); break;
        default: allreduce_oneshot_bf16<8><<<kMaxBlocks, kThreads, 0, st>>>(p); break;
    }
    return cudaGetLastError() == cudaSuccess ? W4A8_OK : W4A8_ERR_CUDA;
}

int w4a8_ar_status(w4a8_ar* h, int32_t reset)
{
    if (!h) return W4A8_ERR_INVALID;
    int v = 0;
    if (cudaMemcpy(&v, h->local + h->lay.off_status, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess)
        return W4A8_ERR_CUDA;
    if (reset && v) {
        const int z = 0;
        if (cudaMemcpy(h->local + h->lay.off_status, &z, sizeof(z), cudaMemcpyHostToDevice) != cudaSuccess)
            return W4A8_ERR_CUDA;
    }
    return v ? W4A8_ERR_TIMEOUT : W4A8_OK;
}

int w4a8_ar_destroy(w4a8_ar* h)
{
    if (!h) return W4A8_OK;
    cudaDeviceSynchronize();
    for (int r = 0; r < h->world; ++r)
        if (h->ipc[r]) cudaIpcCloseMemHandle(h->mapped[r]);
    cudaFree(h->local);
    delete h;
    cudaGetLastError();          // leave no error pending for the caller's next launch check
    return W4A8_OK;
}

}  // extern "C"
