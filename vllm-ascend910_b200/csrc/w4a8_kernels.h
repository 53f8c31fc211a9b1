// w4a8_kernels.h -- parameter blocks and launchers shared by the .cu files of
// libw4a8_b200.so (internal; the public C ABI is include/w4a8_b200.h).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace w4a8 {

enum QuantOutKind { kOutKernel = 0, kOutPublic = 1, kOutMsd = 2 };

struct QuantParams {
    const uint16_t* x;   // bf16 bits [M, ldx]
    int64_t ldx;
    int M, K, Kpad, G, gk;
    int swiglu;          // x holds [gate | up] ([M, 2K] within ldx): quantise bf16(silu(gate) * up)
    int rows;            // rows to emit: M, or Mp for the MSD form
    int vec_ok;          // 16-byte vector loads are legal for this x
    // kOutKernel: the GEMM's activation tiles (see gemm_act_tile_offset)
    int8_t* aq;          // [n_tt][kb_total][TT * 256] bytes, 128-byte swizzled
    float* as;           // [n_tt][G][TT]
    int tt, kb_total;
    // kOutPublic
    int8_t* q;           // [M, K]
    void* scale;         // [G, M] bf16 bits or fp32
    int scale_f32;
    int32_t* ksum;       // [G, M] or null
    // kOutMsd
    int8_t* a_hi;        // [rows, Kpad/2]
    int8_t* a_lo;
    uint16_t* a_scale;   // [G, rows]
    int32_t* a_ksum;     // [G, rows]
};

struct MsdToKernelParams {
    const int8_t* a_hi;      // [M, Kpad/2]
    const int8_t* a_lo;
    const uint16_t* a_scale; // [G, scale_ld] bf16 bits
    int scale_ld;
    int M, Kpad, G, gk;
    int rows;                // n_tt * tt: rows of the tile layout (>= M)
    int8_t* aq;              // activation tiles, as in QuantParams
    float* as;
    int tt, kb_total;
};

// Byte offset of activation code (row, padded position) inside the GEMM's
// activation tiles: tile (row / tt, pos / 256) holds tt rows x 256 codes as two
// halves of tt x 128 bytes, each in the 128-byte-swizzled order the MMA's
// shared-memory descriptor expects (16-byte chunk c of row r stored at chunk
// c ^ (r % 8)).  One 1-D bulk copy moves a tile.
__host__ __device__ inline int64_t gemm_act_tile_offset(int row, int pos, int tt, int kb_total)
{
    const int r = row % tt, t = row / tt, kb = pos >> 8, w = pos & 255;
    const int h = w >> 7, c = (w & 127) >> 4, b = w & 15;
    return (static_cast<int64_t>(t) * kb_total + kb) * (tt * 256) + h * (tt * 128) + r * 128 +
           ((c ^ (r & 7)) << 4) + b;
}

// Row-parallel output pushed to every rank (the fused GEMM + all-reduce): the
// bf16 result tile goes straight into slot [bank][rank] of every rank's
// one-shot all-reduce buffer instead of into y.  world == 0: no push.
struct PushParams {
    uint8_t* base[8];          // every rank's buffer as mapped in this process (own included)
    const uint32_t* counter;   // this rank's call counter of the all-reduce (block 0's)
    size_t slot_bytes, bank_bytes;
    int world, rank;
};

// The GEMM's view of one call.  Tensor maps are built on the host.
// k-blocks (256 K positions) per pipeline stage and stream-K unit when
// GK <= 256: two for 16-token tiles (32 KB of int4 weights per unit), one for
// wider tiles.  The host plan and the kernel's Cfg both take it from here.
__host__ __device__ constexpr int stage_kblocks(int tt) { return tt <= 16 ? 2 : 1; }

struct alignas(64) GemmParams {
    // raw (reference-layout) weights, read with 2-D tensor copies
    CUtensorMap tm_w;    // packed int4 weights [N, Kpad/2] bytes, box {128 B, 128 rows}, SW128
    CUtensorMap tm_ws;   // weight scales [G, N] (fp32 or bf16), box {128, GPK}
    CUtensorMap tm_wz;   // weight zero points [G, N] bf16, box {128, GPK} (asymmetric only)
    // prepared weights (w4a8_prepare_weights), read with 1-D bulk copies; null = raw path
    const uint8_t* w_tiles;   // [n_wt][kb_total][16384] swizzled packed int4 tiles
    const uint8_t* ws_tiles;  // [n_wt][G][128] scales (fp32 or bf16)
    const uint8_t* wz_tiles;  // [n_wt][G][128] bf16 zero points (asymmetric only)
    // activations from the quantiser, read with 1-D bulk copies
    const uint8_t* a_tiles;   // [n_tt][kb_total][TT * 256] (gemm_act_tile_offset)
    const float* as_tiles;    // [n_tt][G][TT]
    // fused quantisation (GemmConfig::fq): the bf16 activation itself, read with
    // 2-D tensor copies of 256 positions x TT rows (rows >= M and positions >= K
    // arrive as zeros) and quantised inside the GEMM
    CUtensorMap tm_x;    // x bf16 [M, K] (row stride ldx), box {256, TT}, no swizzle
    void* out;           // y bf16 [M, N] (row stride ldy), or int32 partials [G, M, N]
    float* partials;     // stream-K partial tiles: [2 * grid][TT][128] fp32
    int* status;         // device status word
    PushParams push;     // (fused all-reduce) where finished bf16 tiles go instead of out
    int M, N, Kpad, G;
    int64_t ldy;
    int n_wt, n_tt, units_per_tile, total_units, kb_total;
};

// Prepared weight layout: the packed int4 weights regrouped into one
// contiguous, pre-swizzled 16 KB tile per (128-row tile, 256-element k-block),
// followed by the scales and zero points regrouped per row tile.
struct PreparedLayout {
    int64_t off_tiles, off_ws, off_wz, total;
};

__host__ __device__ inline PreparedLayout prepared_layout(int64_t N, int64_t G, int kb_total, int ws_elt, bool zero)
{
    const int64_t n_wt = (N + 127) / 128;
    PreparedLayout L;
    L.off_tiles = 0;
    L.off_ws = n_wt * kb_total * 16384;
    L.off_wz = L.off_ws + ((n_wt * G * 128 * ws_elt + 255) / 256) * 256;
    L.total = L.off_wz + (zero ? ((n_wt * G * 128 * 2 + 255) / 256) * 256 : 0);
    return L;
}

struct PrepareParams {
    const uint8_t* w_packed;   // [N, Kpad/2]
    const uint8_t* w_scale;    // [G, N]
    const uint16_t* w_zero;    // [G, N] or null
    uint8_t* out;
    int N, Kpad, G, kb_total, ws_elt;
};

struct GemmConfig {
    int tt;        // token tile (MMA N): 16, 32, 64 or 128
    int gk;        // 64, 128, 256 or 1024
    bool asym;
    bool ws_bf16;
    bool partials; // debug mode: write int32 group partials instead of y
    bool fq;       // quantise the activation inside the GEMM (one token tile of 16, GK <= 256)
};

cudaError_t launch_quant_act(const QuantParams& p, int out_kind, cudaStream_t stream, bool pdl);
cudaError_t launch_prepare_weights(const PrepareParams& p, cudaStream_t stream);
cudaError_t launch_msd_to_kernel(const MsdToKernelParams& p, cudaStream_t stream, bool pdl);

// Launches the GEMM on `grid` persistent CTAs.  Returns cudaErrorInvalidValue
// for an unsupported configuration.
cudaError_t launch_gemm(const GemmParams& p, const GemmConfig& cfg, int grid, cudaStream_t stream,
                        bool pdl);
size_t gemm_smem_bytes(const GemmConfig& cfg);

// Sums the parts of output tiles split across GEMM CTAs (a programmatic
// dependent of the GEMM launched with the same parameters and grid).
cudaError_t launch_splitk_reduce(const GemmParams& p, int tt, int grid, cudaStream_t stream);

// The one-shot all-reduce's side of the fused row-parallel linear
// (w4a8_allreduce.cu): where a GEMM must push a message of `bytes`, and the
// reduction that follows the pushes (flags, bounded waits, rank-order sum).
}  // namespace w4a8
struct w4a8_ar;
namespace w4a8 {
// pull: the GEMM stores into this rank's own slot only and the reduction reads
// the peers' slots; otherwise the GEMM stores into every rank's slot.
int ar_push_params(const w4a8_ar* h, size_t bytes, bool pull, PushParams* out);
cudaError_t ar_launch_reduce_pushed(w4a8_ar* h, void* out, int64_t count, bool pull, cudaStream_t stream);

}  // namespace w4a8
