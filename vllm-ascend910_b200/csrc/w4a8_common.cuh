// w4a8_common.cuh -- sm_100a building blocks shared by the W4A8 kernels:
// mbarriers with bounded waits, TMA tile loads, tcgen05 (TMEM alloc, MMA,
// commit, ld/st, fences) and programmatic dependent launch.
//
// Every wait in this library is bounded.  A wait that runs out sets the CTA's
// shared abort flag and a status word in global memory (read back by the host
// after the call), so a desynchronised pipeline ends with an error status
// instead of a hung GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace w4a8 {

// Status codes written to the device status word (host reads them back).
enum : int {
    kDevOk = 0,
    kDevTimeoutBase = 0x100,   // + role/wait id
};

// Wall-clock limit for any single wait (nanoseconds of %globaltimer).
constexpr uint64_t kWaitLimitNs = 2000000000ull;   // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31u; }
__device__ __forceinline__ uint32_t warp_id() { return threadIdx.x >> 5; }

__device__ __forceinline__ bool elect_one()
{
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "elect.sync _|P, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, P;\n\t}"
        : "=r"(pred));
    return pred != 0;
}

// ---------------------------------------------------------------- mbarrier

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, P;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with parity `parity`.  Returns false (after
// raising the CTA abort flag and recording `where` in *status) when the wait
// runs out, or when another role of the CTA has already aborted.  Inlined: an
// out-of-line call in the pipeline loops costs more than the wait itself.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int* status, int where)
{
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 63u) {
            if (*abort_flag) return false;
            if (global_timer_ns() - t0 > kWaitLimitNs) {
                *abort_flag = 1;
                atomicCAS(status, 0, kDevTimeoutBase + where);
                return false;
            }
        }
    }
}

// ---------------------------------------------------------------- TMA

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map)
{
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load (no multicast): box at (x = inner coordinate, y = row).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Same, with an L2 cache-eviction policy (createpolicy result).
__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, uint64_t* bar,
                                                 int32_t x, int32_t y, uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// 1-D bulk copy of `bytes` contiguous bytes (16-byte aligned, multiple of 16).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint64_t policy_evict_last()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// ---------------------------------------------------------------- PDL

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents()
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Pins a value in a register at this point of the program: arithmetic that
// depends only on the launch shape is then done before a following
// pdl_wait() (volatile asm statements keep their order) instead of after it.
__device__ __forceinline__ void pin(int& v) { asm volatile("" : "+r"(v)); }
__device__ __forceinline__ void pin(int64_t& v) { asm volatile("" : "+l"(v)); }

// ---------------------------------------------------------------- tcgen05

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Arrive on `bar` once every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc], int8 x int8 -> int32, one CTA.
__device__ __forceinline__ void tc_mma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Per-warpgroup register re-allocation (all 4 warps of a warpgroup execute the
// same instruction).  The block's launch allocation bounds the sum.
template <int N>
__device__ __forceinline__ void regs_dec() { asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N)); }
template <int N>
__device__ __forceinline__ void regs_inc() { asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N)); }

__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 16 consecutive 32-bit columns, one lane per thread of the warp.
__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&r)[16])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

// Orders later uses of tcgen05.ld destination registers after the
// tcgen05.wait::ld that precedes this call: the empty volatile asm is not moved
// across the wait, and every later read of r depends on its outputs.
__device__ __forceinline__ void reg_fence16(uint32_t (&r)[16])
{
    asm volatile("" : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
                 "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
                 "+r"(r[14]), "+r"(r[15]));
}

// 32 lanes x 8 / x 4 consecutive 32-bit columns (narrow token tiles).
__device__ __forceinline__ void tc_ld8(uint32_t taddr, uint32_t* r)
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}

__device__ __forceinline__ void tc_ld4(uint32_t taddr, uint32_t* r)
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
}

// reg_fence16 for 4 registers.
__device__ __forceinline__ void reg_fence4(uint32_t* r)
{
    asm volatile("" : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]));
}

__device__ __forceinline__ void tc_st8(uint32_t taddr, const uint32_t (&r)[8])
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
        : "memory");
}

// Shared-memory matrix descriptor for a K-major operand stored in the
// 128-byte-swizzled canonical layout (8 rows x 128 B atoms, atoms 1024 B apart).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr)
{
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);          // start address
    d |= static_cast<uint64_t>(1u) << 16;                        // leading byte offset (unused)
    d |= static_cast<uint64_t>(1024u >> 4) << 32;                // stride byte offset
    d |= static_cast<uint64_t>(1u) << 46;                        // descriptor version (sm_100)
    d |= static_cast<uint64_t>(2u) << 61;                        // layout: SWIZZLE_128B
    return d;
}

// Instruction descriptor: s8 x s8 -> s32, both operands K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_i8(uint32_t M, uint32_t N)
{
    return (2u << 4)             // D format: s32
           | (1u << 7)           // A: signed 8-bit
           | (1u << 10)          // B: signed 8-bit
           | ((N >> 3) << 17)    // N / 8
           | ((M >> 4) << 24);   // M / 16
}

// ---------------------------------------------------------------- packed fp32 pairs
// sm_100 executes two fp32 lanes per instruction on a 64-bit register pair.

// The pair (lo, hi) as one 64-bit register pair, formed inside PTX with
// mov.b64 {lo, hi}: the register allocator then places lo and hi in adjacent
// registers, with no shift-and-or of a C++ 64-bit expression to untangle.
__device__ __forceinline__ uint64_t pair2(float lo, float hi)
{
    uint64_t d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
    return d;
}

__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b)
{
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c)
{
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

// ---------------------------------------------------------------- misc

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b)
{
    return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// fp32 -> bf16 bits, round to nearest even (inputs here are finite).
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f)
{
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// Makes this thread's generic-proxy shared-memory writes visible to the async
// proxy (the tensor core's operand reads, bulk copies) before a barrier
// arrival hands the buffer over.
__device__ __forceinline__ void fence_proxy_async_smem()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- activation quantisation
// The reference's rule (fakequant_lab/quant.py:89-141), per (token, K-group):
//   s = bf16_rne(amax / 127) (IEEE division), bf16 tiny when that is 0
//   q = clamp(rint(x / s), -128, 127)        (IEEE division, half-even)

// Scale bits from the group's amax (quant.py:102-105).
__device__ __forceinline__ uint16_t act_scale_bits(float amax)
{
    uint16_t sb = f32_to_bf16_bits(__fdiv_rn(amax, 127.0f));
    if ((sb & 0x7FFFu) == 0) sb = 0x0080u;
    return sb;
}

// One code with the true division.
__device__ __forceinline__ int quant_exact(float xv, float s)
{
    float r = rintf(__fdiv_rn(xv, s));
    r = fminf(fmaxf(r, -128.0f), 127.0f);
    return static_cast<int>(r);
}

// One code without a division: y = x * (1/s), and the true division only
// when y is within 2^-11 of a half-integer.  For a normal s, x / s (x, s bf16)
// is either a half-integer or at least 1/1020 from every half-integer, while
// |y - x / s| <= 2^-16, so rint(y) equals rint(x / s) outside that window and
// every tie falls inside it; |x / s| < 127.5 because s = bf16(amax / 127), so
// the clamp cannot bind.  `rcp` = __frcp_rn(s); callers take quant_exact for
// the whole group when s is a bf16 subnormal (act_scale_fast false).
__device__ __forceinline__ int quant_fast(float xv, float s, float rcp)
{
    const float y = __fmul_rn(xv, rcp);
    const float n = rintf(y);
    if (fabsf(__fsub_rn(y, n)) > 0.49951171875f) return quant_exact(xv, s);
    return static_cast<int>(n);
}

__device__ __forceinline__ bool act_scale_fast(uint16_t sb) { return (sb & 0x7F80u) != 0; }

// 8 codes k0..k7 -> two words in the GEMM's operand order: k0 k2 k4 k6 | k1 k3 k5 k7.
__device__ __forceinline__ uint2 pack_operand_order(const int (&q)[8])
{
    const uint32_t lo = (q[0] & 0xFF) | ((q[2] & 0xFF) << 8) | ((q[4] & 0xFF) << 16) |
                        (static_cast<uint32_t>(q[6] & 0xFF) << 24);
    const uint32_t hi = (q[1] & 0xFF) | ((q[3] & 0xFF) << 8) | ((q[5] & 0xFF) << 16) |
                        (static_cast<uint32_t>(q[7] & 0xFF) << 24);
    return make_uint2(lo, hi);
}

// The stack's activation on one element: bf16(silu(g) * u) with
// silu(g) = g / (1 + exp(-g)) in fp32, as the reference computes it in torch
// (F.silu(g) * u, npu_ops/python/bench_decode_layer.py:81) before quantising.
__device__ __forceinline__ float swiglu_bf16(float g, float u)
{
    const float a = __fmul_rn(__fdiv_rn(g, 1.0f + expf(-g)), u);
    return bf16_bits_to_f32(f32_to_bf16_bits(a));
}

// 8 bf16 values (one 16-byte word) -> fp32.
__device__ __forceinline__ void unpack8_bf16(uint4 v, float (&x)[8])
{
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        x[2 * i] = __uint_as_float(w[i] << 16);
        x[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
}

}  // namespace w4a8
