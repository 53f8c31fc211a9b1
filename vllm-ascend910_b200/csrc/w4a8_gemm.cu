// w4a8_gemm.cu -- the mid-group W4A8 GEMM for sm_100a.
//
//   y[m, n] = sum_g  as[g, m] * ws[g, n] * P[g, m, n]
//   P[g, m, n] = sum_{k in g} A_q[m, k] * (W_q[n, k] - wz[g, n])        (int32, exact)
//
// which is the reference's mid-group GEMM (fakequant_lab/fake_linear.py:155-179,
// npu_ops/kernel/midgroup_w4a8_gemm.inc:1-60) computed without its MSD split:
// B200's tensor core multiplies int8 x int8 natively (tcgen05 kind::i8).
//
// Mapping onto the tensor core (one CTA per SM, persistent):
//   * MMA M = 128 weight rows (output channels), MMA N = TT tokens, K = 32/instr.
//   * A operand = weights.  Packed int4 rows arrive by TMA into shared memory;
//     four converter warps unpack them to int8 in registers and store them into
//     tensor memory (tcgen05.st), so converted weights never make a second trip
//     through shared memory.  Symmetric weights with GK <= 256 are unpacked as
//     16*w (a nibble shifted into the top of its byte: 3 logic ops per 8
//     weights); otherwise as the int8 value w - zero.
//   * B operand = int8 activations from the quantiser (already in the order the
//     unpack produces: k0 k2 k4 k6 k1 k3 k5 k7 per 8), TMA-loaded with 128-byte
//     swizzle.
//   * Each K-group accumulates into its own int32 TMEM region.  Regions are
//     handed to the epilogue through a ring of up to 8 accumulator slots (a
//     slot holds one K-unit's groups when the token tile is small, else one
//     group), so the MMA runs several groups ahead of the rescale instead of
//     waiting for it.  A group's first MMA overwrites its region (no clear).
//   * Epilogue warps: tcgen05.ld of each slot's partials, acc += P * (ws * as)
//     with packed f32x2 arithmetic in registers, bf16 store at tile end.  A
//     16-token tile rescales only the token columns the call has (4 or 8 per
//     thread at M <= 4 / 8; two warpgroups of 8 at M = 9..16).
//   * Work split: stream-K over (tile, K-unit) so every SM gets the same number
//     of weight bytes.  A tile split across CTAs leaves fp32 parts that a small
//     fix-up kernel (chained by programmatic dependent launch) sums in CTA
//     order, so the result does not depend on timing.
//   * Every mbarrier wait is bounded (w4a8_common.cuh).
#include "w4a8_common.cuh"
#include "w4a8_kernels.h"

namespace w4a8 {

namespace {

constexpr int kWTileBytes = 128 * 128;    // 128 weight rows x 128 B (256 int4)
constexpr int kNumPreWarps = 8;           // weight producer, 2 MMA issuers, activation producer, 4 converters
constexpr int kActProducerWarp = 3;
constexpr int kNumIssuers = 2;            // two threads issue the units' MMAs alternately
constexpr int kSmemBudget = 227 * 1024 - 1024;
constexpr int kBarBytes = 1024;

// wait-site ids for the status word
enum { kWProdEmpty = 1, kWActEmpty, kWProdSlot, kWConvFull, kWConvAEmpty, kWMmaFull, kWMmaAFull, kWMmaAccEmpty,
       kWEpiSlot, kWEpiAccFull, kWDrain, kWQuantSlot, kWQuantX, kWQuantAEmpty };

// FQ_: the activation is quantised inside the GEMM.  Warp 3 then streams the
// bf16 activation (2-D tensor copies into a staging ring) instead of codes,
// and four more warps quantise each stage straight into the MMA operand
// buffer and the unit's scale slot.  Built for one 16-token tile (decode),
// GK <= 256.
template <int TT_, int GK_, bool ASYM_, bool FQ_ = false, int E_ = 0>
struct Cfg {
    static constexpr int TT = TT_;
    static constexpr int GK = GK_;
    static constexpr bool ASYM = ASYM_;
    static constexpr bool FQ = FQ_;
    static_assert(!FQ || (TT == 16 && GK <= 256), "fused quantisation: 16-token tiles, GK <= 256");
    // Pipeline granularity.  Every hand-over between warps costs a few
    // hundred cycles of mbarrier latency, so 16-token tiles move two k-blocks
    // (32 KB of int4 weights) per stage.
    static constexpr int KS = stage_kblocks(TT);             // k-blocks per stage
    static constexpr int GPK = GK <= 256 ? 256 / GK : 1;     // groups per k-block
    static constexpr int UKB = GK <= 256 ? KS : GK / 256;    // k-blocks per unit (max)
    static constexpr int GPU = GK <= 256 ? KS * GPK : 1;     // groups per unit (max)
    static constexpr bool SYM16 = !ASYM && GK <= 256;
    static constexpr int E = E_ ? E_ : (TT <= 16 ? 1 : 2);   // epilogue warpgroups
    static constexpr int NC = TT / E;                        // accumulator columns per thread
    static constexpr int NCH = NC >= 16 ? NC / 16 : 1;       // 16-column TMEM chunks per thread
    static constexpr int NQW = FQ ? 4 : 0;                   // quantiser warps
    static constexpr int QWARP0 = kNumPreWarps + 4 * E;      // first quantiser warp
    static constexpr int THREADS = (kNumPreWarps + 4 * E + NQW) * 32;
    // TMEM: NA A buffers of KS x 64 columns (the stage's int8 weights), the
    // rest for accumulator slots of CG groups x TT columns.  Tiles of 32 to
    // 128 tokens keep two A buffers (128 columns), so their slots hold three
    // or more units (measured: 64-token tiles 2-4 % faster than with four
    // buffers; 32-token tiles with one-k-block units 3 % faster over the
    // four projections than with two-k-block units and two slots of slack).
    static constexpr int ABUF = KS * 64;
    static constexpr int NA = (TT <= 16 ? 256 : 128) / ABUF;
    static constexpr int ACC0 = NA * ABUF;
    static constexpr int ACC_COLS = 512 - ACC0;
    static constexpr int CG_FIT = ACC_COLS / (4 * TT);       // keeps >= 4 slots
    static constexpr int CG = GPU <= CG_FIT ? GPU : (CG_FIT >= 4 ? 4 : (CG_FIT >= 2 ? 2 : 1));
    static constexpr int TOTCH = CG * NCH;                   // 16-column chunks per slot and thread
    static constexpr int BCH = TOTCH < 2 ? TOTCH : 2;        // chunks per tcgen05.ld batch
    static constexpr int NB = TOTCH / BCH;                   // batches per slot
    // Releasing a slot before its rescale (measured): faster for 32-token
    // tiles, slower for 128-token tiles, neutral otherwise.
    static constexpr bool EARLY_RELEASE = TT == 32;
    static constexpr int NACC_FIT = ACC_COLS / (CG * TT);
    static constexpr int NACC = NACC_FIT > 8 ? 8 : NACC_FIT;           // accumulator slots
    __host__ __device__ static constexpr int r128(int x) { return (x + 127) / 128 * 128; }
    // Shared memory, in this order (tiles first: they need 1024-byte alignment):
    //   S_W weight stages     KS x 16 KB, released by the converters
    //   S_A activation stages KS x TT x 256 B, released by the MMA
    //   S_W zero-point rows   (asymmetric) the unit's GPU x 128 bf16, loaded with its first stage
    //   DS scale slots        one unit's [GPU][128] weight scales (sized for fp32) and
    //                         [GPU][TT] activation scales, filled by the activation
    //                         producer (FQ: weight scales by warp 3, activation
    //                         scales by the quantiser warps), released by the epilogue
    //   XS x stages           (FQ) KS boxes of TT rows x 256 bf16, filled by warp 3,
    //                         released by the quantiser warps
    //   barriers
    static constexpr int A_TILE = TT * 256;
    static constexpr int A_STAGE = KS * A_TILE;
    static constexpr int W_STAGE = KS * kWTileBytes;
    static constexpr int WZ_BYTES = ASYM ? GPU * 128 * 2 : 0;
    static constexpr int WZ_SLOT = r128(WZ_BYTES);
    static constexpr int SL_WS = GPU * 128 * 4;
    static constexpr int SL_AS = GPU * TT * 4;
    static constexpr int SLOT = r128(SL_WS) + r128(SL_AS);
    static constexpr int DS = FQ ? 6 : 8;
    static constexpr int S_A = FQ ? 2 : (TT <= 64 ? 4 : 3);
    static constexpr int X_BOX = TT * 512;                   // one 2-D copy: TT rows x 256 bf16
    static constexpr int X_STAGE = FQ ? KS * X_BOX : 0;
    static constexpr int XS = FQ ? 2 : 0;
    static constexpr int S_W_FIT = (kSmemBudget - kBarBytes - DS * SLOT - S_A * A_STAGE - XS * X_STAGE - (FQ ? 1024 : 0)) /
                                   (W_STAGE + WZ_SLOT);
    static constexpr int S_W = S_W_FIT > 16 ? 16 : S_W_FIT;
    // Two MMA issuers take alternate units only when every activation stage
    // and every TMEM weight buffer then has one issuer as its only consumer
    // (one stage per unit, even ring sizes).  An mbarrier wait matches a phase
    // by parity alone: an issuer that skipped the other issuer's rounds of a
    // shared stage would take the other's unfinished round r for its own round
    // r + 1 and multiply stale operands (seen as intermittently wrong token
    // columns with 128-token tiles, whose ring has 3 stages).  Otherwise one
    // issuer runs every unit.
    static constexpr bool TWO_ISSUERS = GK <= 256 && S_A % 2 == 0 && NA % 2 == 0;
    // With two issuers the accumulator slots are split between them too
    // (issuer i owns the slots i, i + 2, ...), so neither ever waits on a slot
    // phase of the other's: an issuer that only watched the other's slots
    // could fall two phases behind one of them once the epilogue outpaces the
    // MMA, and then wait for a phase that never comes.
    static constexpr int NRING = TWO_ISSUERS ? NACC / 2 : NACC;   // slots per issuer
    __host__ __device__ static constexpr int acc_slot(int i, int who) { return TWO_ISSUERS ? 2 * i + who : i; }
    static constexpr int OFF_A = S_W * W_STAGE;
    static constexpr int OFF_WZ = OFF_A + S_A * A_STAGE;
    static constexpr int OFF_SL = OFF_WZ + S_W * WZ_SLOT;
    static constexpr int OFF_X = (OFF_SL + DS * SLOT + 1023) / 1024 * 1024;
    static constexpr int BAR_OFF = FQ ? OFF_X + XS * X_STAGE : OFF_SL + DS * SLOT;
    static constexpr int SMEM = BAR_OFF + kBarBytes + 1024;  // + alignment slack
    static constexpr int TMEM_COLS = 512;
    static_assert(S_W >= 3 && S_A >= 2, "pipeline too shallow");
    static_assert(NACC >= 2, "need at least two accumulator slots");
    static_assert(!TWO_ISSUERS || (NACC % 2 == 0 && NRING >= 2), "two slots per issuer");
    static_assert(GPU % CG == 0, "slots split a unit evenly");
    static_assert(NC % 16 == 0 || NC == 8, "epilogue works in 16-column chunks (or 8 columns per thread)");
    static_assert(TOTCH % BCH == 0, "slots split into whole batches");
    static_assert(OFF_A % 1024 == 0 && OFF_WZ % 1024 == 0, "tile alignment");
    static_assert(SMEM <= 227 * 1024, "shared memory");
    static_assert(!FQ || (S_A >= 2 && XS >= 2), "fused quantisation rings");
    // Register split for the 64/128-token tiles (2 + E warpgroups): producers +
    // MMA issuers and converters give registers to the epilogue warpgroups,
    // which hold NC fp32 accumulators per thread.  The sum stays within the
    // launch allocation (__launch_bounds__(THREADS, 1): LAUNCH_REGS per thread);
    // the host also checks it against the compiled register count.
    static constexpr int NWG = 2 + E;
    static constexpr bool SPLIT_REGS = TT >= 64;
    static_assert(!(FQ && SPLIT_REGS), "the register split does not count quantiser warps");
    static constexpr int LAUNCH_REGS = (65536 / THREADS) / 8 * 8;
    static constexpr int REGS_PRE = 56;
    static constexpr int REGS_CONV = E <= 2 ? 80 : 72;
    static constexpr int REGS_EPI = ((NWG * LAUNCH_REGS - REGS_PRE - REGS_CONV) / E) / 8 * 8;
    static constexpr int REG_SUM = REGS_PRE + REGS_CONV + E * REGS_EPI;
    static_assert(!SPLIT_REGS || (REG_SUM <= NWG * LAUNCH_REGS && REGS_EPI <= 256 && REGS_EPI >= REGS_CONV),
                  "register split exceeds the launch allocation");
};

struct Bars {
    uint64_t wfull[16], wempty[16];     // weight tiles
    uint64_t afull[8], aempty[8];       // activation tiles
    uint64_t tfull[4], tempty[4];       // converted weights in TMEM
    uint64_t accfull[8], accempty[8];   // accumulator slots
    uint64_t sfull[8], sempty[8];       // scale slots
    uint64_t xfull[2], xempty[2];       // bf16 activation stages (fused quantisation)
    uint64_t drain[2];
    uint32_t tmem_base;
    int abort;
};

static_assert(sizeof(Bars) <= kBarBytes, "barrier block overflows its reservation");

struct Unit {
    int t, wt, tt, ut;
};

// Bounded wait taken by a whole warp; the verdict is made warp-uniform so the
// warp stays converged for the .sync.aligned tcgen05 instructions that follow.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int* status, int where)
{
    const bool ok = mbar_wait(bar, parity, abort_flag, status, where);
    return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ Unit unit_of(const GemmParams& p, int u)
{
    Unit r;
    r.t = u / p.units_per_tile;
    r.ut = u - r.t * p.units_per_tile;
    r.wt = r.t / p.n_tt;
    r.tt = r.t - r.wt * p.n_tt;
    return r;
}

// The unit after `r` (units run K-unit fastest, then token tile, then weight tile).
__device__ __forceinline__ void unit_next(const GemmParams& p, Unit& r)
{
    if (++r.ut == p.units_per_tile) {
        r.ut = 0;
        ++r.t;
        if (++r.tt == p.n_tt) {
            r.tt = 0;
            ++r.wt;
        }
    }
}

// A unit (the stream-K work item and the epilogue's step) is UKB k-blocks:
// one stage of KS k-blocks when GK <= 256, one GK = 1024 group otherwise.
template <class C>
__device__ __forceinline__ void unit_kblocks(const GemmParams& p, int ut, int& kb0, int& kb1)
{
    kb0 = ut * C::UKB;
    kb1 = min(kb0 + C::UKB, p.kb_total);
}

template <class C>
__device__ __forceinline__ void unit_groups(const GemmParams& p, int ut, int& g0, int& g1)
{
    g0 = ut * C::GPU;
    g1 = min(g0 + C::GPU, p.G);
}

__device__ __forceinline__ void cta_range(const GemmParams& p, int c, int C, int& u0, int& u1)
{
    u0 = static_cast<int>(static_cast<int64_t>(c) * p.total_units / C);
    u1 = static_cast<int>(static_cast<int64_t>(c + 1) * p.total_units / C);
}

// The CTA whose range holds unit u (inverse of cta_range).
__device__ __forceinline__ int cta_of_unit(const GemmParams& p, int u, int C)
{
    return static_cast<int>((static_cast<int64_t>(u + 1) * C - 1) / p.total_units);
}

struct R16 {
    uint32_t v[16];
};

// acc[16*i + j] += float(P_j) * (ws * as[j]) for one 16-column chunk.  The
// accumulator lives in packed fp32 pairs (acc2[k] = columns 2k, 2k+1) so the
// scale and accumulate steps are f32x2 instructions on register pairs.  r holds
// the int32 group partials P (|P| < 2^23, so the conversion is exact).
template <int NC>
__device__ __forceinline__ void rescale_chunk(uint64_t (&acc2)[NC / 2], int i, const R16& r, float wsv,
                                              const float* asg)
{
    const uint64_t ws2 = pair2(wsv, wsv);
#pragma unroll
    for (int j = 0; j < 16; j += 4) {
        const float4 a4 = *reinterpret_cast<const float4*>(asg + j);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t r0 = r.v[j + 2 * h], r1 = r.v[j + 2 * h + 1];
            const uint64_t f2 = pair2(__int2float_rn(static_cast<int>(r0)), __int2float_rn(static_cast<int>(r1)));
            const uint64_t c2 = f2_mul(ws2, h == 0 ? pair2(a4.x, a4.y) : pair2(a4.z, a4.w));
            uint64_t& a = acc2[8 * i + j / 2 + h];
            a = f2_fma(f2, c2, a);
        }
    }
}

// rescale_chunk for the first NV columns (NV a multiple of 4) of one group.
template <int NC, int NV>
__device__ __forceinline__ void rescale_cols(uint64_t (&acc2)[NC / 2], const uint32_t* r, float wsv, const float* asg)
{
    const uint64_t ws2 = pair2(wsv, wsv);
#pragma unroll
    for (int j = 0; j < NV; j += 4) {
        const float4 a4 = *reinterpret_cast<const float4*>(asg + j);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint64_t f2 = pair2(__int2float_rn(static_cast<int>(r[j + 2 * h])),
                                      __int2float_rn(static_cast<int>(r[j + 2 * h + 1])));
            const uint64_t c2 = f2_mul(ws2, h == 0 ? pair2(a4.x, a4.y) : pair2(a4.z, a4.w));
            uint64_t& a = acc2[j / 2 + h];
            a = f2_fma(f2, c2, a);
        }
    }
}

__device__ __forceinline__ float acc_at(const uint64_t* acc2, int j)
{
    return __uint_as_float(static_cast<uint32_t>(acc2[j >> 1] >> ((j & 1) * 32)));
}

// Debug output mode: the exact int32 partials of one 16-column chunk of group g.
template <bool SYM16>
__device__ __noinline__ void store_partials(const GemmParams& p, R16 r, int g, int m0, int n)
{
    if (n >= p.N) return;
    int* dst = reinterpret_cast<int*>(p.out) + (static_cast<int64_t>(g) * p.M + m0) * p.N + n;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        int P = static_cast<int>(r.v[j]);
        if (SYM16) P >>= 4;
        if (m0 + j < p.M) dst[static_cast<int64_t>(j) * p.N] = P;
    }
}

// The fused all-reduce's output path: element (m, n) of this rank's bf16 result
// goes to slot [bank][rank] of every rank's all-reduce buffer (a dense [M, N]
// message; plain stores, over NVLink for the peers).  The bank is the parity of
// the all-reduce call this result belongs to: the counter of completed calls
// plus one, read after the kernel's dependency wait (this thread reaches here
// only after that wait, through the pipeline's barriers).
__device__ __forceinline__ __nv_bfloat16* push_slot(const PushParams& pp, int r)
{
    const uint32_t seq = *reinterpret_cast<const volatile uint32_t*>(pp.counter) + 1u;
    return reinterpret_cast<__nv_bfloat16*>(pp.base[r] + (seq & 1u) * pp.bank_bytes +
                                            static_cast<size_t>(pp.rank) * pp.slot_bytes);
}

template <int NC, int NV>
__device__ __forceinline__ void push_tile(const GemmParams& p, int m0, int n, const uint64_t (&acc2)[NC / 2])
{
    if (n >= p.N) return;
    for (int r = 0; r < p.push.world; ++r) {
        __nv_bfloat16* dst = push_slot(p.push, r);
#pragma unroll
        for (int j = 0; j < NV; ++j)
            if (m0 + j < p.M) dst[static_cast<int64_t>(m0 + j) * p.N + n] = __float2bfloat16_rn(acc_at(acc2, j));
    }
}

// End of a CTA's share of one output tile: store the bf16 tile when the CTA
// computed all of it, else store its fp32 part for w4a8_splitk_reduce_kernel
// (which runs after the GEMM, so no fence or arrival count is needed here).
// Only the first NV columns hold results (the rest are past M).  PUSH: the
// fused all-reduce's instantiation, whose finished tiles go to the ranks'
// receive slots instead of y.
template <class C, int NV, bool PUSH>
__device__ __forceinline__ void flush_tile(const GemmParams& p, const Unit& un, int u0, int u1, int cta, int row,
                                           int col0, const uint64_t (&acc2)[C::NC / 2])
{
    constexpr int TT = C::TT, NC = C::NC;
    const int t = un.t;
    const int tfirst = t * p.units_per_tile, tlast = tfirst + p.units_per_tile - 1;
    const int n = un.wt * 128 + row;
    if (u0 <= tfirst && u1 - 1 >= tlast) {
        if constexpr (PUSH) {
            push_tile<NC, NV>(p, un.tt * TT + col0, n, acc2);
            return;
        }
        __nv_bfloat16* y = reinterpret_cast<__nv_bfloat16*>(p.out);
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int m = un.tt * TT + col0 + j;
            if (m < p.M && n < p.N) y[static_cast<int64_t>(m) * p.ldy + n] = __float2bfloat16_rn(acc_at(acc2, j));
        }
        return;
    }
    const int side = (t == u0 / p.units_per_tile) ? 0 : 1;
    float* mine = p.partials + static_cast<int64_t>(2 * cta + side) * (TT * 128);
#pragma unroll
    for (int j = 0; j < NV; ++j) __stcg(mine + (col0 + j) * 128 + row, acc_at(acc2, j));
}

// The epilogue warps' loop.  NV: token columns rescaled per thread -- all NC,
// or (16-token tiles of calls with at most 4 or 8 tokens) only the first NV:
// the MMA still multiplies 16 token columns (its smallest N at 128 rows), but
// the columns past M hold zeros and are neither rescaled nor stored.
template <class C, bool PART, int NV, bool PUSH>
__device__ __forceinline__ void epilogue_role(const GemmParams& p, Bars* bars, uint8_t* smem, uint32_t tbase,
                                              volatile int* abort_flag, int ws_bf16, int warp, int lane, int u0,
                                              int u1, int cta)
{
    constexpr int TT = C::TT;
    constexpr bool NARROW = NV < 16;     // one batch of x4 / x8 loads per slot
    static_assert(NV <= C::NC && (!NARROW || (C::TT == 16 && !PART && (NV == 4 || NV == 8))),
                  "narrow columns: 16-token tiles");
    auto slot_ws = [&](int s) { return smem + C::OFF_SL + s * C::SLOT; };
    auto slot_as = [&](int s) { return reinterpret_cast<float*>(slot_ws(s) + C::r128(C::SL_WS)); };
    const int ew = warp - kNumPreWarps;
    const int quarter = warp & 3;
    const int part = ew >> 2;
    const int row = quarter * 32 + lane;
    const int col0 = part * NV;                   // NV == NC unless the tile has fewer tokens
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    constexpr int NCH = C::NCH;

    tc_fence_before();
    __syncwarp();
    if (lane == 0)
        for (int b = 0; b < C::NACC; ++b) mbar_arrive(&bars->accempty[b]);
    __syncwarp();

    uint64_t acc2[C::NC / 2];
#pragma unroll
    for (int j = 0; j < C::NC / 2; ++j) acc2[j] = 0ull;
    // Accumulator slot ring position of the unit's issuer (sl, aph) and of the
    // other issuer (sl_o, aph_o): with two issuers units alternate between them
    // and each fills its own slots (Cfg::acc_slot), so the pair swaps per unit.
    int sl = 0, sl_o = 0, slot = 0;
    uint32_t aph = 0, aph_o = 0, slph = 0;
    bool ok = true;
    Unit un = unit_of(p, u0);
    for (int u = u0; ok && u < u1; ++u, unit_next(p, un)) {
        int g0, g1;
        unit_groups<C>(p, un.ut, g0, g1);
        const int who = C::TWO_ISSUERS ? (u - u0) & 1 : 0;
        if (!warp_wait(&bars->sfull[slot], slph, abort_flag, p.status, kWEpiSlot)) { ok = false; break; }
        const uint8_t* wsb = slot_ws(slot);
        const float* asb = slot_as(slot);
        // one accumulator slot holds CG groups: all of this unit's, or one
        for (int gs = g0; gs < g1; gs += C::CG) {
            const int ps = C::acc_slot(sl, who);
            if (!warp_wait(&bars->accfull[ps], aph, abort_flag, p.status, kWEpiAccFull)) { ok = false; break; }
            tc_fence_after();
            const uint32_t t_slot = tbase + lane_off + C::ACC0 + static_cast<uint32_t>(ps * C::CG * TT + col0);
            // this row's weight scale of each group in the slot, read once
            float wsv[C::CG];
            if (!PART) {
#pragma unroll
                for (int gi = 0; gi < C::CG; ++gi) {
                    const int gl = min(gs + gi, g1 - 1) - g0;
                    wsv[gi] = ws_bf16 ? bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(wsb)[gl * 128 + row])
                                      : reinterpret_cast<const float*>(wsb)[gl * 128 + row];
                    if (C::SYM16) wsv[gi] *= 0.0625f;   // the unpack carried weights as 16*w
                }
            }
            if constexpr (NARROW) {
                // every group of the slot in one batch of loads; the slot goes
                // back to the MMA as soon as the values are in registers
                uint32_t r[C::CG][NV];
#pragma unroll
                for (int gi = 0; gi < C::CG; ++gi) {
                    if constexpr (NV == 8)
                        tc_ld8(t_slot + gi * TT, r[gi]);
                    else
                        tc_ld4(t_slot + gi * TT, r[gi]);
                }
                tc_wait_ld();
#pragma unroll
                for (int gi = 0; gi < C::CG; ++gi)
#pragma unroll
                    for (int q = 0; q < NV; q += 4) reg_fence4(r[gi] + q);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars->accempty[ps]);
                __syncwarp();
#pragma unroll
                for (int gi = 0; gi < C::CG; ++gi)
                    if (gs + gi < g1) rescale_cols<C::NC, NV>(acc2, r[gi], wsv[gi], asb + (gs + gi - g0) * TT + col0);
            } else {
                // Batches of BCH chunks, software-pipelined: the next batch's
                // tcgen05.ld is in flight while this batch is rescaled.  With
                // EARLY_RELEASE the slot goes back to the MMA as soon as its last
                // batch is in registers, otherwise after the rescale.
                R16 r[2][C::BCH];
    #pragma unroll
                for (int q = 0; q < C::BCH; ++q)
                    tc_ld16(t_slot + (q / NCH) * TT + 16 * (q % NCH), r[0][q].v);
                tc_wait_ld();
    #pragma unroll
                for (int q = 0; q < C::BCH; ++q) reg_fence16(r[0][q].v);
    #pragma unroll
                for (int b = 0; b < C::NB; ++b) {
                    if (b + 1 < C::NB) {
    #pragma unroll
                        for (int q = 0; q < C::BCH; ++q) {
                            const int c = (b + 1) * C::BCH + q;
                            tc_ld16(t_slot + (c / NCH) * TT + 16 * (c % NCH), r[(b + 1) & 1][q].v);
                        }
                    } else if (C::EARLY_RELEASE) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&bars->accempty[ps]);
                        __syncwarp();
                    }
    #pragma unroll
                    for (int q = 0; q < C::BCH; ++q) {
                        const int c = b * C::BCH + q, gi = c / NCH, i = c % NCH;
                        const int g = gs + gi;
                        if (g >= g1) continue;
                        const int gl = g - g0;           // group index within the unit's scale entry
                        if (PART)
                            store_partials<C::SYM16>(p, r[b & 1][q], g, un.tt * TT + col0 + 16 * i, un.wt * 128 + row);
                        else
                            rescale_chunk<C::NC>(acc2, i, r[b & 1][q], wsv[gi], asb + gl * TT + col0 + 16 * i);
                    }
                    if (b + 1 < C::NB) {
                        tc_wait_ld();
    #pragma unroll
                        for (int q = 0; q < C::BCH; ++q) reg_fence16(r[(b + 1) & 1][q].v);
                    }
                }
                if (!C::EARLY_RELEASE) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&bars->accempty[ps]);
                    __syncwarp();
                }
            }
            if (++sl == C::NRING) { sl = 0; aph ^= 1; }
        }
        if (!ok) break;
        if (C::TWO_ISSUERS) {
            const int ts = sl;
            sl = sl_o;
            sl_o = ts;
            const uint32_t tp = aph;
            aph = aph_o;
            aph_o = tp;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->sempty[slot]);
        __syncwarp();
        if (++slot == C::DS) { slot = 0; slph ^= 1; }

        // ---- end of this CTA's share of tile t: store or hand over ----
        if (un.ut == p.units_per_tile - 1 || u == u1 - 1) {
            if (!PART) flush_tile<C, NV, PUSH>(p, un, u0, u1, cta, row, col0, acc2);
#pragma unroll
            for (int j = 0; j < C::NC / 2; ++j) acc2[j] = 0ull;
        }
    }
}

// PART: the debug mode that writes each group's exact int32 partials instead
// of y.  It is a separate instantiation (16-token tiles only) so the product
// epilogue carries no call and no second output path.
//
// NV: token columns the epilogue rescales (0: all of the tile).  A call of at
// most 4 or 8 tokens runs a 16-token instantiation with NV = 4 or 8; the
// variants are separate kernels so the common case carries no extra code.
template <int TT, int GK, bool ASYM, bool PART, bool FQ, int NV, int EPI, bool PUSH>
__global__ void __launch_bounds__(Cfg<TT, GK, ASYM, FQ, EPI>::THREADS, 1)
    w4a8_gemm_kernel(const __grid_constant__ GemmParams p, const int ws_bf16)
{
    using C = Cfg<TT, GK, ASYM, FQ, EPI>;
    static_assert(NV == 0 || (TT == 16 && !PART), "narrow epilogues: 16-token tiles");
    static_assert(C::NC >= 16 || !PART, "the partials mode stores 16-column chunks");
    static_assert(!(PART && FQ), "the partials mode reads codes from the standalone quantiser");
    extern __shared__ uint8_t smem_raw[];
    // Align by an offset from the __shared__ array itself: a pointer rebuilt from
    // an integer loses the address space, and every read through it would be a
    // generic load (the L1TEX path, behind the bulk copies) instead of ld.shared.
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    Bars* bars = reinterpret_cast<Bars*>(smem + C::BAR_OFF);

    const int warp = static_cast<int>(warp_id());
    const int lane = static_cast<int>(lane_id());
    const int nctas = static_cast<int>(gridDim.x);
    const int cta = static_cast<int>(blockIdx.x);
    int u0, u1;
    cta_range(p, cta, nctas, u0, u1);

    auto w_tile = [&](int s) { return smem + s * C::W_STAGE; };
    auto a_stage = [&](int s) { return smem + C::OFF_A + s * C::A_STAGE; };
    auto w_zero = [&](int s) { return smem + C::OFF_WZ + s * C::WZ_SLOT; };
    auto slot_ws = [&](int s) { return smem + C::OFF_SL + s * C::SLOT; };
    auto slot_as = [&](int s) { return reinterpret_cast<float*>(slot_ws(s) + C::r128(C::SL_WS)); };
    auto x_stage = [&](int s) { return smem + C::OFF_X + s * C::X_STAGE; };

    // ---------------------------------------------------------------- setup
    if (threadIdx.x == 0) {
        for (int i = 0; i < C::S_W; ++i) {
            mbar_init(&bars->wfull[i], 1);                  // weight producer (+ bytes)
            mbar_init(&bars->wempty[i], 4);                 // 4 converter warps
        }
        for (int i = 0; i < C::S_A; ++i) {
            mbar_init(&bars->afull[i], C::FQ ? C::NQW : 1); // activation producer (+ bytes) / quantiser warps
            mbar_init(&bars->aempty[i], 1);                 // the owning issuer's commit
        }
        for (int i = 0; i < C::XS; ++i) {
            mbar_init(&bars->xfull[i], 1);                  // warp 3 (+ bytes)
            mbar_init(&bars->xempty[i], C::NQW);            // quantiser warps
        }
        for (int i = 0; i < C::NA; ++i) {
            mbar_init(&bars->tfull[i], 4);
            mbar_init(&bars->tempty[i], 1);
        }
        for (int i = 0; i < C::NACC; ++i) {
            mbar_init(&bars->accfull[i], 1);
            mbar_init(&bars->accempty[i], 4 * C::E);
        }
        for (int i = 0; i < C::DS; ++i) {
            mbar_init(&bars->sfull[i], 1 + C::NQW);         // activation producer (+ bytes), quantiser warps
            mbar_init(&bars->sempty[i], 4 * C::E);          // epilogue warps
        }
        mbar_init(&bars->drain[0], 1);
        mbar_init(&bars->drain[1], 1);
        bars->abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(&bars->tmem_base, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = bars->tmem_base;
    volatile int* abort_flag = &bars->abort;
    const uint32_t ws_elt = ws_bf16 ? 2u : 4u;

    // With SPLIT_REGS each role re-sizes its warpgroup's registers first thing
    // in its branch (warps 0-3: producers + issuers, 4-7: converters, 8-15:
    // epilogue), so the compiler allocates each branch for its own budget.
    if (warp == 0 || warp == kActProducerWarp) {
        if (C::SPLIT_REGS) regs_dec<C::REGS_PRE>();
        // ============================================================ producers
        // Warp 0 streams weight tiles (and, asymmetric, the unit's zero points
        // with its first tile); it never waits for the epilogue nor for the
        // kernel that produced x.  Warp 3, after the programmatic dependency
        // resolves, streams activation tiles and fills each unit's scale slot
        // (weight and activation scales) for the epilogue.  Each copy is one
        // instruction.
        const bool wside = warp == 0;
        const bool prepared = p.w_tiles != nullptr;
        if (elect_one()) {
            if (wside && !prepared) {
                tma_prefetch_desc(&p.tm_w);
                if (C::ASYM) tma_prefetch_desc(&p.tm_wz);
            }
            if (!wside && !prepared && !PART) tma_prefetch_desc(&p.tm_ws);
            if (!wside && C::FQ) tma_prefetch_desc(&p.tm_x);
            if (!wside) pdl_wait();
            // Weights stream once when there is one token tile (decode): evict
            // them first.  With several token tiles a CTA re-reads its weight
            // tile once per token tile, so they must stay in L2.
            const uint64_t pol = (wside && p.n_tt == 1) ? policy_evict_first() : policy_evict_last();
            // warp 3's stage ring: activation codes, or (FQ) bf16 activation boxes
            const int ns = wside ? C::S_W : (C::FQ ? C::XS : C::S_A);
            uint64_t* fullb = wside ? bars->wfull : (C::FQ ? bars->xfull : bars->afull);
            uint64_t* emptyb = wside ? bars->wempty : (C::FQ ? bars->xempty : bars->aempty);
            int stage = 0, issued = 0, slot = 0, sissued = 0;
            uint32_t ph = 0, slph = 0;
            bool ok = true;
            Unit un = unit_of(p, u0);
            for (int u = u0; ok && u < u1; ++u, unit_next(p, un)) {
                int kb0, kb1, g0, g1;
                unit_kblocks<C>(p, un.ut, kb0, kb1);
                unit_groups<C>(p, un.ut, g0, g1);
                if (!wside) {
                    if (!mbar_wait(&bars->sempty[slot], slph ^ 1, abort_flag, p.status, kWProdSlot)) break;
                    if (PART) {
                        mbar_arrive(&bars->sfull[slot]);      // the partials mode reads no scales
                    } else {
                        const uint32_t ng = static_cast<uint32_t>(g1 - g0);
                        const uint32_t wsb = prepared ? ng * 128u * ws_elt : C::GPU * 128u * ws_elt;
                        // (FQ: the quantiser warps write the activation scales)
                        const uint32_t asb = C::FQ ? 0u : ng * static_cast<uint32_t>(C::TT * 4);
                        mbar_arrive_expect_tx(&bars->sfull[slot], wsb + asb);
                        if (prepared)
                            bulk_load(slot_ws(slot), p.ws_tiles + (static_cast<int64_t>(un.wt) * p.G + g0) * 128 * ws_elt,
                                      wsb, &bars->sfull[slot], pol);
                        else
                            tma_load_2d(slot_ws(slot), &p.tm_ws, &bars->sfull[slot], un.wt * 128, g0);
                        if (!C::FQ)
                            bulk_load(slot_as(slot), p.as_tiles + (static_cast<int64_t>(un.tt) * p.G + g0) * C::TT, asb,
                                      &bars->sfull[slot], pol);
                    }
                    ++sissued;
                    if (++slot == C::DS) { slot = 0; slph ^= 1; }
                }
                for (int kbs = kb0; kbs < kb1; kbs += C::KS) {
                    const int kn = min(C::KS, kb1 - kbs);       // k-blocks in this stage
                    if (!mbar_wait(&emptyb[stage], ph ^ 1, abort_flag, p.status, wside ? kWProdEmpty : kWActEmpty)) {
                        ok = false;
                        break;
                    }
                    if (wside) {
                        const bool zp = C::ASYM && kbs == kb0;
                        const uint32_t zb = zp ? (prepared ? static_cast<uint32_t>(g1 - g0) * 256u : C::GPU * 256u) : 0u;
                        mbar_arrive_expect_tx(&fullb[stage], static_cast<uint32_t>(kn) * kWTileBytes + zb);
                        if (prepared) {
                            bulk_load(w_tile(stage), p.w_tiles + (static_cast<int64_t>(un.wt) * p.kb_total + kbs) * kWTileBytes,
                                      static_cast<uint32_t>(kn) * kWTileBytes, &fullb[stage], pol);
                        } else {
                            for (int j = 0; j < kn; ++j)
                                tma_load_2d_hint(w_tile(stage) + j * kWTileBytes, &p.tm_w, &fullb[stage], (kbs + j) * 128,
                                                 un.wt * 128, pol);
                        }
                        if (zp) {
                            if (prepared)
                                bulk_load(w_zero(stage), p.wz_tiles + (static_cast<int64_t>(un.wt) * p.G + g0) * 256, zb,
                                          &fullb[stage], pol);
                            else
                                tma_load_2d(w_zero(stage), &p.tm_wz, &fullb[stage], un.wt * 128, g0);
                        }
                    } else if (C::FQ) {
                        // bf16 x: one TT-row x 256-position box per k-block (zeros past M and K)
                        mbar_arrive_expect_tx(&fullb[stage], static_cast<uint32_t>(kn * C::X_BOX));
                        for (int j = 0; j < kn; ++j)
                            tma_load_2d_hint(x_stage(stage) + j * C::X_BOX, &p.tm_x, &fullb[stage], (kbs + j) * 256,
                                             un.tt * C::TT, pol);
                    } else {
                        mbar_arrive_expect_tx(&fullb[stage], static_cast<uint32_t>(kn * C::A_TILE));
                        bulk_load(a_stage(stage), p.a_tiles + (static_cast<int64_t>(un.tt) * p.kb_total + kbs) * C::A_TILE,
                                  static_cast<uint32_t>(kn * C::A_TILE), &fullb[stage], pol);
                    }
                    ++issued;
                    if (++stage == ns) { stage = 0; ph ^= 1; }
                }
            }
            // The next kernels in the stream (fix-up, the next call's quantiser
            // and GEMM) may launch once every CTA's weight producer has issued
            // its last copy: they then prepare while this CTA drains its
            // pipeline.  Triggering at setup instead let those grids launch and
            // sit resident for the whole GEMM; that chain stalled a dependency
            // wait for seconds about once in 50,000 calls (measured), this
            // placement did not in 576,000.
            if (wside) pdl_launch_dependents();
            // Never leave with a copy in flight: wait (bounded) for the last
            // copy into each stage (copy i went to stage i % ns, phase i / ns).
            for (int i = issued > ns ? issued - ns : 0; i < issued; ++i)
                mbar_wait(&fullb[i % ns], static_cast<uint32_t>((i / ns) & 1), abort_flag, p.status, kWDrain);
            for (int i = sissued > C::DS ? sissued - C::DS : 0; i < sissued; ++i)
                mbar_wait(&bars->sfull[i % C::DS], static_cast<uint32_t>((i / C::DS) & 1), abort_flag, p.status, kWDrain);
        }
    } else if (warp <= kNumIssuers) {
        if (C::SPLIT_REGS) regs_dec<C::REGS_PRE>();
        // ============================================================ MMA issuers
        // With two issuers (Cfg::TWO_ISSUERS), issuer i owns the units u0 + i,
        // u0 + i + 2, ...: for those it waits for the stages, issues every MMA
        // and commits the stages' buffers and the unit's accumulator slots (from
        // its own share of the slots); for the other issuer's units it only
        // advances its stage ring positions.  Each
        // barrier hand-over costs a few hundred cycles, so splitting whole units
        // halves every issuer's share.  Otherwise issuer 0 owns every unit.
        const int me = warp - 1;
        if (elect_one() && (C::TWO_ISSUERS || me == 0)) {
            const uint32_t idesc = idesc_i8(128, TT);
            int sa = 0, ab = 0, sl = 0;
            uint32_t saph = 0, abph = 0, slph = 0;
            bool ok = true;
            Unit un = unit_of(p, u0);
            for (int u = u0; ok && u < u1; ++u, unit_next(p, un)) {
                int kb0, kb1, g0, g1;
                unit_kblocks<C>(p, un.ut, kb0, kb1);
                unit_groups<C>(p, un.ut, g0, g1);
                const bool mine = !C::TWO_ISSUERS || ((u - u0) & 1) == me;
                for (int kbs = kb0; kbs < kb1; kbs += C::KS) {
                    const int kn = min(C::KS, kb1 - kbs);
                    if (mine) {
                        if (!mbar_wait(&bars->afull[sa], saph, abort_flag, p.status, kWMmaFull)) { ok = false; break; }
                        if (!mbar_wait(&bars->tfull[ab], abph, abort_flag, p.status, kWMmaAFull)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t a_smem = smem_u32(a_stage(sa));
                        const uint32_t a_tmem = tbase + static_cast<uint32_t>(ab * C::ABUF);
                        if (C::GK <= 256 && g1 - g0 == C::GPU) {
                            // A whole unit: its slots, groups and K steps are compile-time
                            // constants, so the MMAs go out as one straight-line block.
                            // (An MMA issued from a runtime loop iteration costs the
                            // issuing thread ~250 cycles; unrolled ones ~17.)
#pragma unroll
                            for (int s = 0; s < C::GPU / C::CG; ++s) {
                                const int ps = C::acc_slot(sl, me);
                                if (!mbar_wait(&bars->accempty[ps], slph, abort_flag, p.status, kWMmaAccEmpty)) { ok = false; break; }
                                tc_fence_after();
                                const uint32_t d_slot = tbase + C::ACC0 + static_cast<uint32_t>(ps * C::CG * TT);
#pragma unroll
                                for (int gi = 0; gi < C::CG; ++gi) {
                                    const int gl = s * C::CG + gi;
                                    const int j = gl / C::GPK;                       // k-block within the stage
                                    const int s0 = (gl % C::GPK) * (C::GK / 32);     // first K step within it
#pragma unroll
                                    for (int t = 0; t < C::GK / 32; ++t) {
                                        const int ks = s0 + t;
                                        const uint64_t bd = smem_desc_sw128(a_smem + j * C::A_TILE + (ks >> 2) * (TT * 128) + (ks & 3) * 32);
                                        tc_mma_i8_ts(d_slot + gi * TT, a_tmem + j * 64 + ks * 8, bd, idesc, t == 0 ? 0u : 1u);
                                    }
                                }
                                tc_commit(&bars->accfull[ps]);
                                if (++sl == C::NRING) { sl = 0; slph ^= 1; }
                            }
                            if (!ok) break;
                        } else if (C::GK <= 256) {
                            // a ragged last unit: groups g0..g1, CG per accumulator slot
                            for (int g = g0; g < g1; ++g) {
                                const int gl = g - g0, gi = gl % C::CG;
                                const int ps = C::acc_slot(sl, me);
                                if (gi == 0) {
                                    if (!mbar_wait(&bars->accempty[ps], slph, abort_flag, p.status, kWMmaAccEmpty)) { ok = false; break; }
                                    tc_fence_after();
                                }
                                const uint32_t d_tmem = tbase + C::ACC0 + static_cast<uint32_t>((ps * C::CG + gi) * TT);
                                const int j = gl / C::GPK;                       // k-block within the stage
                                const int s0 = (gl % C::GPK) * (C::GK / 32);     // first K step within it
#pragma unroll
                                for (int t = 0; t < C::GK / 32; ++t) {
                                    const int ks = s0 + t;
                                    const uint64_t bd = smem_desc_sw128(a_smem + j * C::A_TILE + (ks >> 2) * (TT * 128) + (ks & 3) * 32);
                                    tc_mma_i8_ts(d_tmem, a_tmem + j * 64 + ks * 8, bd, idesc, t == 0 ? 0u : 1u);
                                }
                                if (gi == C::CG - 1 || g == g1 - 1) {
                                    tc_commit(&bars->accfull[ps]);
                                    if (++sl == C::NRING) { sl = 0; slph ^= 1; }
                                }
                            }
                            if (!ok) break;
                        } else {
                            // one GK = 1024 group spread over several stages
                            const bool first_stage = kbs == kb0, last_stage = kbs + kn >= kb1;
                            const int ps = C::acc_slot(sl, me);
                            if (first_stage) {
                                if (!mbar_wait(&bars->accempty[ps], slph, abort_flag, p.status, kWMmaAccEmpty)) { ok = false; break; }
                                tc_fence_after();
                            }
                            const uint32_t d_tmem = tbase + C::ACC0 + static_cast<uint32_t>(ps * TT);
                            for (int j = 0; j < kn; ++j) {
#pragma unroll
                                for (int ks = 0; ks < 8; ++ks) {
                                    const uint64_t bd = smem_desc_sw128(a_smem + j * C::A_TILE + (ks >> 2) * (TT * 128) + (ks & 3) * 32);
                                    tc_mma_i8_ts(d_tmem, a_tmem + j * 64 + ks * 8, bd, idesc,
                                                 (first_stage && j == 0 && ks == 0) ? 0u : 1u);
                                }
                            }
                            if (last_stage) {
                                tc_commit(&bars->accfull[ps]);
                                if (++sl == C::NRING) { sl = 0; slph ^= 1; }
                            }
                        }
                        tc_commit(&bars->tempty[ab]);
                        tc_commit(&bars->aempty[sa]);
                    }
                    if (++ab == C::NA) { ab = 0; abph ^= 1; }
                    if (++sa == C::S_A) { sa = 0; saph ^= 1; }
                }
            }
            // Wait for every MMA issued by this thread before TMEM can be released.
            tc_commit(&bars->drain[me]);
            mbar_wait(&bars->drain[me], 0, abort_flag, p.status, kWDrain);
        }
    } else if (warp < kNumPreWarps) {
        if (C::SPLIT_REGS) regs_dec<C::REGS_CONV>();
        // ============================================================ converters
        // Unpack one weight stage into a TMEM A buffer and hand the
        // shared-memory tiles straight back to the producer.
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
        int stage = 0, ab = 0;
        uint32_t sph = 0, abph = 0;
        bool ok = true;
        uint32_t bias[C::GPU];
#pragma unroll
        for (int i = 0; i < C::GPU; ++i) bias[i] = 0x78787878u;   // zero point 0
        Unit un = unit_of(p, u0);
        for (int u = u0; ok && u < u1; ++u, unit_next(p, un)) {
            int kb0, kb1;
            unit_kblocks<C>(p, un.ut, kb0, kb1);
            for (int kbs = kb0; kbs < kb1; kbs += C::KS) {
                const int kn = min(C::KS, kb1 - kbs);
                if (!warp_wait(&bars->wfull[stage], sph, abort_flag, p.status, kWConvFull)) { ok = false; break; }
                if (C::ASYM && kbs == kb0) {
                    const uint16_t* wz = reinterpret_cast<const uint16_t*>(w_zero(stage));
#pragma unroll
                    for (int i = 0; i < C::GPU; ++i) {
                        const int zu = static_cast<int>(bf16_bits_to_f32(wz[i * 128 + row])) + 8;
                        bias[i] = static_cast<uint32_t>((0x80 - zu) & 0xFF) * 0x01010101u;
                    }
                }
                if (!warp_wait(&bars->tempty[ab], abph ^ 1, abort_flag, p.status, kWConvAEmpty)) { ok = false; break; }
                tc_fence_after();
                const uint32_t a_tmem = tbase + lane_off + static_cast<uint32_t>(ab * C::ABUF);
#pragma unroll
                for (int j = 0; j < C::KS; ++j) {
                    if (j >= kn) break;
                    const uint8_t* wrow = w_tile(stage) + j * kWTileBytes + row * 128;
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        const uint4 v = *reinterpret_cast<const uint4*>(wrow + ((c ^ (row & 7)) << 4));
                        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
                        uint32_t o[8];
                        // chunk c holds K positions [32c, 32c+32) of k-block j
                        const uint32_t bz = bias[C::GK <= 256 ? j * C::GPK + (c * 32) / (C::GK <= 256 ? C::GK : 256) : 0];
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            if (C::SYM16) {
                                o[2 * q] = (w[q] << 4) & 0xF0F0F0F0u;       // 16 * even-k weights
                                o[2 * q + 1] = w[q] & 0xF0F0F0F0u;          // 16 * odd-k weights
                            } else {
                                const uint32_t x = w[q] ^ 0x88888888u;     // nibble + 8 in [0, 15]
                                o[2 * q] = ((x & 0x0F0F0F0Fu) + bz) ^ 0x80808080u;
                                o[2 * q + 1] = (((x >> 4) & 0x0F0F0F0Fu) + bz) ^ 0x80808080u;
                            }
                        }
                        tc_st8(a_tmem + j * 64 + c * 8, o);
                    }
                }
                tc_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&bars->tfull[ab]);
                    mbar_arrive(&bars->wempty[stage]);
                }
                __syncwarp();
                if (++ab == C::NA) { ab = 0; abph ^= 1; }
                if (++stage == C::S_W) { stage = 0; sph ^= 1; }
            }
        }
    } else if (C::FQ && warp >= C::QWARP0) {
        // ============================================================ quantiser (FQ)
        // Per stage: the bf16 boxes warp 3 staged -> per (row, group) amax over
        // the group's lanes -> scale (the reference's rule) -> int8 codes in
        // the MMA's operand order, written into the A stage; the unit's
        // activation scales go into its scale slot.  Work items are (row,
        // k-block) pairs: a warp takes one row's 256 positions, 8 per lane.
        const int qw = warp - C::QWARP0;
        const int Mr = min(p.M, TT);   // one token tile: rows >= Mr never hold data
        constexpr int TPG = C::GK / 8;                       // lanes per group
        // Rows >= Mr of every A stage are zero for the whole kernel (the MMA
        // multiplies them with the weights; the epilogue stores no such row).
        for (int idx = qw * 32 + lane; idx < C::S_A * C::KS * 2 * (TT - Mr) * 8; idx += C::NQW * 32) {
            const int c = idx & 7, rr = (idx >> 3) % (TT - Mr), h = ((idx >> 3) / (TT - Mr)) & 1;
            const int js = ((idx >> 3) / (TT - Mr)) >> 1;    // stage * KS + k-block
            *reinterpret_cast<uint4*>(a_stage(js / C::KS) + (js % C::KS) * C::A_TILE + h * (TT * 128) +
                                      (Mr + rr) * 128 + c * 16) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
        int xs = 0, stage = 0, slot = 0;
        uint32_t xph = 0, aph = 0, slph = 0;
        bool ok = true;
        Unit un = unit_of(p, u0);
        for (int u = u0; ok && u < u1; ++u, unit_next(p, un)) {
            int kb0, kb1, g0, g1;
            unit_kblocks<C>(p, un.ut, kb0, kb1);
            unit_groups<C>(p, un.ut, g0, g1);
            if (!warp_wait(&bars->sempty[slot], slph ^ 1, abort_flag, p.status, kWQuantSlot)) break;
            float* asl = slot_as(slot);
            for (int idx = qw * 32 + lane; idx < (g1 - g0) * (TT - Mr); idx += C::NQW * 32)
                asl[(idx / (TT - Mr)) * TT + Mr + idx % (TT - Mr)] = 0.0f;
            for (int kbs = kb0; kbs < kb1; kbs += C::KS) {
                const int kn = min(C::KS, kb1 - kbs);
                if (!warp_wait(&bars->xfull[xs], xph, abort_flag, p.status, kWQuantX)) { ok = false; break; }
                if (!warp_wait(&bars->aempty[stage], aph ^ 1, abort_flag, p.status, kWQuantAEmpty)) { ok = false; break; }
                const uint8_t* xsm = x_stage(xs);
                uint8_t* ast = a_stage(stage);
                for (int it = qw; it < Mr * kn; it += C::NQW) {
                    const int r = it % Mr, j = it / Mr;
                    float xv[8];
                    unpack8_bf16(*reinterpret_cast<const uint4*>(xsm + j * C::X_BOX + r * 512 + lane * 16), xv);
                    float amax = 0.0f;
#pragma unroll
                    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(xv[i]));
#pragma unroll
                    for (int o = TPG / 2; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
                    const uint16_t sb = act_scale_bits(amax);
                    const float sv = bf16_bits_to_f32(sb);
                    int q[8];
                    if (act_scale_fast(sb)) {
                        const float rcp = __frcp_rn(sv);
#pragma unroll
                        for (int i = 0; i < 8; ++i) q[i] = quant_fast(xv[i], sv, rcp);
                    } else {
#pragma unroll
                        for (int i = 0; i < 8; ++i) q[i] = quant_exact(xv[i], sv);
                    }
                    // lane l holds positions 8l..8l+7 of the k-block: half l/16, chunk (l%16)/2
                    *reinterpret_cast<uint2*>(ast + j * C::A_TILE + (lane >> 4) * (TT * 128) + r * 128 +
                                              ((((lane & 15) >> 1) ^ (r & 7)) << 4) + (lane & 1) * 8) =
                        pack_operand_order(q);
                    if ((lane & (TPG - 1)) == 0)
                        asl[((kbs - kb0 + j) * C::GPK + (lane * 8) / C::GK) * TT + r] = sv;
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&bars->afull[stage]);
                    mbar_arrive(&bars->xempty[xs]);
                }
                __syncwarp();
                if (++xs == C::XS) { xs = 0; xph ^= 1; }
                if (++stage == C::S_A) { stage = 0; aph ^= 1; }
            }
            if (!ok) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->sfull[slot]);
            __syncwarp();
            if (++slot == C::DS) { slot = 0; slph ^= 1; }
        }
    } else {
        if (C::SPLIT_REGS) regs_inc<C::REGS_EPI>();
        epilogue_role<C, PART, NV == 0 ? C::NC : NV, PUSH>(p, bars, smem, tbase, abort_flag, ws_bf16, warp, lane, u0,
                                                           u1, cta);
    }

    // ---------------------------------------------------------------- teardown
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tbase, C::TMEM_COLS);
    }
}

// Regroup raw weights into the prepared layout (one thread per 16-byte chunk
// of a tile, then per scale / zero element); rows past N and bytes past Kpad
// are written as zero.
__global__ void prepare_weights_kernel(const PrepareParams p)
{
    const int n_wt = (p.N + 127) / 128;
    const int64_t chunks = static_cast<int64_t>(n_wt) * p.kb_total * 128 * 8;
    const int64_t scal = static_cast<int64_t>(n_wt) * p.G * 128;
    const int rowb = p.Kpad / 2;
    const PreparedLayout L = prepared_layout(p.N, p.G, p.kb_total, p.ws_elt, p.w_zero != nullptr);
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < chunks + scal;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        if (i < chunks) {
            const int c = static_cast<int>(i & 7);
            const int r = static_cast<int>((i >> 3) & 127);
            const int64_t tile = i >> 10;                      // wt * kb_total + kb
            const int kb = static_cast<int>(tile % p.kb_total);
            const int wt = static_cast<int>(tile / p.kb_total);
            const int n = wt * 128 + r;
            const int byte = kb * 128 + c * 16;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (n < p.N && byte < rowb)
                v = *reinterpret_cast<const uint4*>(p.w_packed + static_cast<int64_t>(n) * rowb + byte);
            *reinterpret_cast<uint4*>(p.out + L.off_tiles + tile * 16384 + r * 128 + ((c ^ (r & 7)) << 4)) = v;
        } else {
            const int64_t j = i - chunks;                      // (wt * G + g) * 128 + r
            const int r = static_cast<int>(j & 127);
            const int64_t wg = j >> 7;
            const int g = static_cast<int>(wg % p.G);
            const int wt = static_cast<int>(wg / p.G);
            const int n = wt * 128 + r;
            const bool in = n < p.N;
            if (p.ws_elt == 4)
                reinterpret_cast<float*>(p.out + L.off_ws)[j] =
                    in ? reinterpret_cast<const float*>(p.w_scale)[static_cast<int64_t>(g) * p.N + n] : 0.0f;
            else
                reinterpret_cast<uint16_t*>(p.out + L.off_ws)[j] =
                    in ? reinterpret_cast<const uint16_t*>(p.w_scale)[static_cast<int64_t>(g) * p.N + n] : 0;
            if (p.w_zero)
                reinterpret_cast<uint16_t*>(p.out + L.off_wz)[j] =
                    in ? p.w_zero[static_cast<int64_t>(g) * p.N + n] : 0;
        }
    }
}

// Stream-K fix-up: one block per 16-token column chunk of an output tile
// (128 weight rows x TT tokens).
// A tile whose units were split across CTAs c_first..c_last is summed from
// their fp32 parts in CTA order (deterministic) and stored as bf16; tiles a
// single CTA finished were stored by the GEMM and are skipped.  Launched
// right after the GEMM as a programmatic dependent: it waits for the GEMM
// grid to complete, so every part is visible without fences.
//
// Which CTAs hold parts of a tile follows from the launch shape alone, so the
// integer divisions that find them run before the wait, while the GEMM is
// still streaming.  A CTA after the first one of a split tile starts its range
// inside the tile, so its part is in its first-tile slot (flush_tile's side 0);
// the first CTA's part is there only when its range starts with the tile.
template <int TT, bool PUSH>
__global__ void __launch_bounds__(128) splitk_reduce_kernel(const GemmParams p, const int nctas)
{
    pdl_launch_dependents();
    const int t = blockIdx.x;
    const int tfirst = t * p.units_per_tile, tlast = tfirst + p.units_per_tile - 1;
    int cf = cta_of_unit(p, tfirst, nctas), cl = cta_of_unit(p, tlast, nctas);
    if (cf == cl) return;
    int u0f, u1f;
    cta_range(p, cf, nctas, u0f, u1f);
    int side_f = u0f == tfirst ? 0 : 1;
    int wt = t / p.n_tt;
    pin(cf);
    pin(cl);
    pin(side_f);
    pin(wt);
    pdl_wait();
    const int tt = t - wt * p.n_tt;
    const int row = threadIdx.x;
    const int n = wt * 128 + row;
    __nv_bfloat16* y = reinterpret_cast<__nv_bfloat16*>(p.out);
    {
        const int c0 = blockIdx.y * 16;
        float sum[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) sum[j] = 0.0f;
        for (int c = cf; c <= cl; c += 4) {
            float v[4][16];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int cc = c + q;
                const bool valid = cc <= cl;
                const float* src = valid ? p.partials + static_cast<int64_t>(2 * cc + (cc == cf ? side_f : 0)) * (TT * 128)
                                         : p.partials;
#pragma unroll
                for (int j = 0; j < 16; ++j) v[q][j] = valid ? __ldcg(src + (c0 + j) * 128 + row) : 0.0f;
            }
#pragma unroll
            for (int q = 0; q < 4; ++q)
#pragma unroll
                for (int j = 0; j < 16; ++j) sum[j] += v[q][j];
        }
        if constexpr (PUSH) {
            if (n < p.N)
                for (int r = 0; r < p.push.world; ++r) {
                    __nv_bfloat16* dst = push_slot(p.push, r);
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int m = tt * TT + c0 + j;
                        if (m < p.M) dst[static_cast<int64_t>(m) * p.N + n] = __float2bfloat16_rn(sum[j]);
                    }
                }
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int m = tt * TT + c0 + j;
                if (m < p.M && n < p.N) y[static_cast<int64_t>(m) * p.ldy + n] = __float2bfloat16_rn(sum[j]);
            }
        }
    }
}

template <int TT, int GK, bool ASYM, bool PART, bool FQ = false, int NV = 0, int EPI = 0, bool PUSH = false>
cudaError_t launch_t(const GemmParams& p, int grid, cudaStream_t stream, bool pdl, int ws_bf16)
{
    using C = Cfg<TT, GK, ASYM, FQ, EPI>;
    auto kern = w4a8_gemm_kernel<TT, GK, ASYM, PART, FQ, NV, EPI, PUSH>;
    // The shared-memory opt-in is per device; set it once per device.
    static bool attr_done[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64 || !attr_done[dev]) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return e;
        if (C::SPLIT_REGS) {
            // setmaxnreg.inc waits for registers the other warpgroups released:
            // refuse a build whose launch allocation cannot cover the split.
            cudaFuncAttributes fa{};
            e = cudaFuncGetAttributes(&fa, kern);
            if (e != cudaSuccess) return e;
            if (static_cast<int64_t>(fa.numRegs) * C::THREADS < static_cast<int64_t>(C::REG_SUM) * 128)
                return cudaErrorInvalidConfiguration;
        }
        if (dev >= 0 && dev < 64) attr_done[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(C::THREADS);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, p, ws_bf16);
}

template <int TT, int GK>
cudaError_t launch_gk(const GemmParams& p, const GemmConfig& c, int grid, cudaStream_t s, bool pdl)
{
    if (c.partials) {
        // the debug partials mode exists for 16-token tiles only (the host plans it so)
        if constexpr (TT == 16)
            return c.asym ? launch_t<TT, GK, true, true>(p, grid, s, pdl, c.ws_bf16)
                          : launch_t<TT, GK, false, true>(p, grid, s, pdl, c.ws_bf16);
        else
            return cudaErrorInvalidValue;
    }
    if (p.push.world) {
        // the fused all-reduce's own instantiations (standalone quantiser, full epilogue)
        return c.asym ? launch_t<TT, GK, true, false, false, 0, 0, true>(p, grid, s, pdl, c.ws_bf16)
                      : launch_t<TT, GK, false, false, false, 0, 0, true>(p, grid, s, pdl, c.ws_bf16);
    }
    if (c.fq) {
        // fused quantisation exists for 16-token tiles and GK <= 256 (the host plans it so)
        if constexpr (TT == 16 && GK <= 256)
            return c.asym ? launch_t<TT, GK, true, false, true>(p, grid, s, pdl, c.ws_bf16)
                          : launch_t<TT, GK, false, false, true>(p, grid, s, pdl, c.ws_bf16);
        else
            return cudaErrorInvalidValue;
    }
    if constexpr (TT == 16) {
        // a call of at most 4 or 8 tokens: the epilogue rescales only those columns
        if (p.M <= 4)
            return c.asym ? launch_t<TT, GK, true, false, false, 4>(p, grid, s, pdl, c.ws_bf16)
                          : launch_t<TT, GK, false, false, false, 4>(p, grid, s, pdl, c.ws_bf16);
        if (p.M <= 8)
            return c.asym ? launch_t<TT, GK, true, false, false, 8>(p, grid, s, pdl, c.ws_bf16)
                          : launch_t<TT, GK, false, false, false, 8>(p, grid, s, pdl, c.ws_bf16);
        return c.asym ? launch_t<TT, GK, true, false, false, 8, 2>(p, grid, s, pdl, c.ws_bf16)
                      : launch_t<TT, GK, false, false, false, 8, 2>(p, grid, s, pdl, c.ws_bf16);
    }
    return c.asym ? launch_t<TT, GK, true, false>(p, grid, s, pdl, c.ws_bf16)
                  : launch_t<TT, GK, false, false>(p, grid, s, pdl, c.ws_bf16);
}

template <int TT>
cudaError_t launch_tt(const GemmParams& p, const GemmConfig& c, int grid, cudaStream_t s, bool pdl)
{
    switch (c.gk) {
        case 64: return launch_gk<TT, 64>(p, c, grid, s, pdl);
        case 128: return launch_gk<TT, 128>(p, c, grid, s, pdl);
        case 256: return launch_gk<TT, 256>(p, c, grid, s, pdl);
        case 1024: return launch_gk<TT, 1024>(p, c, grid, s, pdl);
        default: return cudaErrorInvalidValue;
    }
}

template <int TT>
size_t smem_tt(int gk, bool asym)
{
    switch (gk) {
        case 64: return asym ? Cfg<TT, 64, true>::SMEM : Cfg<TT, 64, false>::SMEM;
        case 128: return asym ? Cfg<TT, 128, true>::SMEM : Cfg<TT, 128, false>::SMEM;
        case 256: return asym ? Cfg<TT, 256, true>::SMEM : Cfg<TT, 256, false>::SMEM;
        default: return asym ? Cfg<TT, 1024, true>::SMEM : Cfg<TT, 1024, false>::SMEM;
    }
}

}  // namespace

cudaError_t launch_gemm(const GemmParams& p, const GemmConfig& c, int grid, cudaStream_t stream, bool pdl)
{
    switch (c.tt) {
        case 16: return launch_tt<16>(p, c, grid, stream, pdl);
        case 32: return launch_tt<32>(p, c, grid, stream, pdl);
        case 64: return launch_tt<64>(p, c, grid, stream, pdl);
        case 128: return launch_tt<128>(p, c, grid, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_splitk_reduce(const GemmParams& p, int tt, int grid, cudaStream_t stream)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.n_wt * p.n_tt, tt / 16);
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const bool push = p.push.world != 0;
    switch (tt) {
        case 16: return cudaLaunchKernelEx(&cfg, push ? splitk_reduce_kernel<16, true> : splitk_reduce_kernel<16, false>, p, grid);
        case 32: return cudaLaunchKernelEx(&cfg, push ? splitk_reduce_kernel<32, true> : splitk_reduce_kernel<32, false>, p, grid);
        case 64: return cudaLaunchKernelEx(&cfg, push ? splitk_reduce_kernel<64, true> : splitk_reduce_kernel<64, false>, p, grid);
        case 128:
            return cudaLaunchKernelEx(&cfg, push ? splitk_reduce_kernel<128, true> : splitk_reduce_kernel<128, false>, p, grid);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_prepare_weights(const PrepareParams& p, cudaStream_t stream)
{
    prepare_weights_kernel<<<148 * 8, 256, 0, stream>>>(p);
    return cudaGetLastError();
}

size_t gemm_smem_bytes(const GemmConfig& c)
{
    switch (c.tt) {
        case 16: return smem_tt<16>(c.gk, c.asym);
        case 32: return smem_tt<32>(c.gk, c.asym);
        case 64: return smem_tt<64>(c.gk, c.asym);
        default: return smem_tt<128>(c.gk, c.asym);
    }
}

}  // namespace w4a8
