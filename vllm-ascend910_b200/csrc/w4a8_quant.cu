// w4a8_quant.cu -- dynamic per-(token, K-group) int8 activation quantisation.
//
// Semantics are those of fakequant_lab/quant.py:89-141 (the reference's
// numerical definition, also implemented by npu_ops/kernel/midgroup_quant_a.inc):
//
//   amax  = max |x| over the group's real members           (fp32)
//   s     = bf16_rne(amax / 127)   (IEEE fp32 division)
//   s     = bf16 tiny               where s == 0
//   q     = clamp(rint(x / float(s)), -128, 127)   (IEEE fp32 division, half-even)
//   ksum  = -sum(q) over the group  (int32, negated as the reference's kernels expect)
//
// Layout: one thread owns 8 consecutive positions of the group-padded row
// (mg_kgeom.h: group g starts at g*GK, the last group is zero-padded to a
// multiple of 64), loads them with one 16-byte bf16 vector load when the row is
// aligned, and a group of GK/8 threads reduces its amax / sum with warp
// shuffles (plus a shared-memory step when a group spans several warps).
//
// Three output forms, selected at compile time:
//   kOutKernel  the GEMM's activation tiles: int8 codes in operand order (each
//               8 positions stored as k0 k2 k4 k6 k1 k3 k5 k7, matching the
//               nibble order the GEMM unpacks weights in) inside swizzled
//               [token tile][k-block] tiles, zero-filled past M and K, plus
//               fp32 scales [token tile][group][row]
//   kOutPublic  int8 codes [M, K] natural order + scales [G, M] (bf16 or fp32)
//               + negated sums [G, M]
//   kOutMsd     the reference op's four tensors: MSD int4 planes a_hi/a_lo
//               [Mp, Kpad/2], bf16 scales [G, Mp], negated sums [G, Mp]; rows
//               [M, Mp) encode q = 0 with scale = bf16 tiny
//               (npu_ops/host/midgroup_quant_a.cpp:40-78, midgroup_quant_a.inc:1-30)
#include "w4a8_common.cuh"
#include "w4a8_kernels.h"

namespace w4a8 {

namespace {

constexpr int kQThreads = 256;
constexpr int kQPos = kQThreads * 8;   // padded positions per block

__device__ __forceinline__ float warp_group_max(float v, int tpg)
{
    for (int o = (tpg < 32 ? tpg : 32) >> 1; o > 0; o >>= 1)
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ int warp_group_sum(int v, int tpg)
{
    for (int o = (tpg < 32 ? tpg : 32) >> 1; o > 0; o >>= 1)
        v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ void load8_bf16(const uint16_t* xr, int pos, int K, bool vec, float (&v)[8])
{
    if (vec && pos + 8 <= K) {
        unpack8_bf16(*reinterpret_cast<const uint4*>(xr + pos), v);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = pos + i < K ? bf16_bits_to_f32(xr[pos + i]) : 0.0f;
    }
}

template <int kOut>
__global__ void __launch_bounds__(kQThreads) quant_act_kernel(const QuantParams p)
{
    __shared__ float red_f[kQThreads / 32];
    __shared__ int red_i[kQThreads / 32];

    pdl_launch_dependents();

    const int row = blockIdx.y;
    const int tid = threadIdx.x;
    const int pos = (blockIdx.x * kQThreads + tid) * 8;   // padded position of element 0
    const int gk = p.gk;
    const int tpg = gk >> 3;                               // threads per group
    // the GEMM's tiles span whole k-blocks: positions up to kb_total*256 exist there
    const int span = (kOut == kOutKernel) ? p.kb_total * 256 : p.Kpad;
    const bool active = pos < span;
    const bool real_row = row < p.M;
    int g = pos / gk;
    // Output offsets depend on the launch shape only: the integer divisions run
    // before the wait for the kernel that produces x.
    int64_t a_off = 0, s_off = 0;
    if (kOut == kOutKernel) {
        a_off = gemm_act_tile_offset(row, pos, p.tt, p.kb_total);
        s_off = (static_cast<int64_t>(row / p.tt) * p.G + g) * p.tt + row % p.tt;
    }
    pin(g);
    pin(a_off);
    pin(s_off);
    pdl_wait();

    // ---- load 8 elements (positions >= K are the group pad: zero) ----
    float xv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) xv[i] = 0.0f;
    if (active && real_row && pos < p.Kpad) {
        const uint16_t* xr = p.x + static_cast<int64_t>(row) * p.ldx;
        load8_bf16(xr, pos, p.K, p.vec_ok, xv);
        if (p.swiglu) {
            float uv[8];
            load8_bf16(xr + p.K, pos, p.K, p.vec_ok, uv);
#pragma unroll
            for (int i = 0; i < 8; ++i) xv[i] = swiglu_bf16(xv[i], uv[i]);
        }
    }

    // ---- group amax ----
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(xv[i]));
    amax = warp_group_max(amax, tpg);
    if (tpg > 32) {
        if (lane_id() == 0) red_f[warp_id()] = amax;
        __syncthreads();
        const int w0 = (warp_id() / (tpg >> 5)) * (tpg >> 5);
        amax = 0.0f;
        for (int w = 0; w < (tpg >> 5); ++w) amax = fmaxf(amax, red_f[w0 + w]);
    }

    const uint16_t sb = act_scale_bits(amax);
    const float s = bf16_bits_to_f32(sb);

    int q[8];
    int qsum = 0;
    if (act_scale_fast(sb)) {
        const float rcp = __frcp_rn(s);
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = quant_fast(xv[i], s, rcp);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = quant_exact(xv[i], s);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) qsum += q[i];

    if (kOut != kOutKernel) {
        qsum = warp_group_sum(qsum, tpg);
        if (tpg > 32) {
            __syncthreads();   // red_f reads are done before red_i is reused
            if (lane_id() == 0) red_i[warp_id()] = qsum;
            __syncthreads();
            const int w0 = (warp_id() / (tpg >> 5)) * (tpg >> 5);
            qsum = 0;
            for (int w = 0; w < (tpg >> 5); ++w) qsum += red_i[w0 + w];
        }
    }
    if (!active) return;
    const bool leader = (pos % gk) == 0;

    if (kOut == kOutKernel) {
        // operand order: k0 k2 k4 k6 | k1 k3 k5 k7 (rows >= M and positions >= K are zero)
        *reinterpret_cast<uint2*>(p.aq + a_off) = pack_operand_order(q);
        if (leader && g < p.G) p.as[s_off] = real_row ? s : 0.0f;
    } else if (kOut == kOutPublic) {
        if (!real_row) return;
        int8_t* qr = p.q + static_cast<int64_t>(row) * p.K;
        if (pos + 8 <= p.K && (p.K & 7) == 0) {
            const uint32_t w0 = (q[0] & 0xFF) | ((q[1] & 0xFF) << 8) | ((q[2] & 0xFF) << 16) |
                                (static_cast<uint32_t>(q[3] & 0xFF) << 24);
            const uint32_t w1 = (q[4] & 0xFF) | ((q[5] & 0xFF) << 8) | ((q[6] & 0xFF) << 16) |
                                (static_cast<uint32_t>(q[7] & 0xFF) << 24);
            *reinterpret_cast<uint2*>(qr + pos) = make_uint2(w0, w1);
        } else {
            for (int i = 0; i < 8; ++i)
                if (pos + i < p.K) qr[pos + i] = static_cast<int8_t>(q[i]);
        }
        if (leader) {
            const int64_t o = static_cast<int64_t>(g) * p.M + row;
            if (p.scale_f32) reinterpret_cast<float*>(p.scale)[o] = s;
            else reinterpret_cast<uint16_t*>(p.scale)[o] = sb;
            if (p.ksum) p.ksum[o] = -qsum;
        }
    } else {   // kOutMsd
        uint32_t hw = 0, lw = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t hn = static_cast<uint32_t>(q[i] >> 4) & 0xFu;     // arithmetic shift
            const uint32_t ln = (static_cast<uint32_t>(q[i]) & 0xFu) ^ 0x8u;
            hw |= hn << (4 * i);
            lw |= ln << (4 * i);
        }
        const int64_t o = static_cast<int64_t>(row) * (p.Kpad / 2) + pos / 2;
        *reinterpret_cast<uint32_t*>(p.a_hi + o) = hw;
        *reinterpret_cast<uint32_t*>(p.a_lo + o) = lw;
        if (leader) {
            const int64_t so = static_cast<int64_t>(g) * p.rows + row;
            p.a_scale[so] = real_row ? sb : static_cast<uint16_t>(0x0080u);
            p.a_ksum[so] = real_row ? -qsum : 0;
        }
    }
}

// MSD planes (the reference op's a_hi / a_lo / bf16 a_scale) -> the GEMM's
// operand order and fp32 scales: q = 16*hi + lo + 8 (quant.py:221-223).
__global__ void __launch_bounds__(kQThreads) msd_to_kernel_kernel(const MsdToKernelParams p)
{
    pdl_launch_dependents();
    pdl_wait();
    const int row = blockIdx.y;
    const int pos = (blockIdx.x * kQThreads + threadIdx.x) * 8;
    const bool real_row = row < p.M;
    if (threadIdx.x == 0) {
        const int g0 = (blockIdx.x * kQPos) / p.gk;
        const int g1 = min(p.G, ((blockIdx.x + 1) * kQPos + p.gk - 1) / p.gk);
        for (int g = g0; g < g1; ++g)
            p.as[(static_cast<int64_t>(row / p.tt) * p.G + g) * p.tt + row % p.tt] =
                real_row ? bf16_bits_to_f32(p.a_scale[static_cast<int64_t>(g) * p.scale_ld + row]) : 0.0f;
    }
    if (pos >= p.kb_total * 256) return;
    int q[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (real_row && pos < p.Kpad) {
        const int64_t o = static_cast<int64_t>(row) * (p.Kpad / 2) + pos / 2;
        const uint32_t hw = *reinterpret_cast<const uint32_t*>(p.a_hi + o);
        const uint32_t lw = *reinterpret_cast<const uint32_t*>(p.a_lo + o);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int hn = static_cast<int>((hw >> (4 * i)) & 0xFu);
            const int ln = static_cast<int>((lw >> (4 * i)) & 0xFu);
            const int hv = (hn & 8) ? hn - 16 : hn;
            const int lv = (ln & 8) ? ln - 16 : ln;
            q[i] = 16 * hv + lv + 8;
        }
    }
    const uint32_t lo = (q[0] & 0xFF) | ((q[2] & 0xFF) << 8) | ((q[4] & 0xFF) << 16) |
                        (static_cast<uint32_t>(q[6] & 0xFF) << 24);
    const uint32_t hi = (q[1] & 0xFF) | ((q[3] & 0xFF) << 8) | ((q[5] & 0xFF) << 16) |
                        (static_cast<uint32_t>(q[7] & 0xFF) << 24);
    *reinterpret_cast<uint2*>(p.aq + gemm_act_tile_offset(row, pos, p.tt, p.kb_total)) = make_uint2(lo, hi);
}

template <typename Kern, typename Params>
cudaError_t launch_pdl(Kern kern, dim3 grid, dim3 block, const Params& prm, cudaStream_t stream,
                       bool pdl)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, prm);
}

}  // namespace

cudaError_t launch_quant_act(const QuantParams& p, int out_kind, cudaStream_t stream, bool pdl)
{
    const int span = out_kind == kOutKernel ? p.kb_total * 256 : p.Kpad;
    const dim3 grid((span + kQPos - 1) / kQPos, p.rows);
    const dim3 block(kQThreads);
    switch (out_kind) {
        case kOutKernel: return launch_pdl(quant_act_kernel<kOutKernel>, grid, block, p, stream, pdl);
        case kOutPublic: return launch_pdl(quant_act_kernel<kOutPublic>, grid, block, p, stream, pdl);
        default: return launch_pdl(quant_act_kernel<kOutMsd>, grid, block, p, stream, pdl);
    }
}

cudaError_t launch_msd_to_kernel(const MsdToKernelParams& p, cudaStream_t stream, bool pdl)
{
    const dim3 grid((p.kb_total * 256 + kQPos - 1) / kQPos, p.rows);
    return launch_pdl(msd_to_kernel_kernel, grid, dim3(kQThreads), p, stream, pdl);
}

}  // namespace w4a8
