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
    int rows;            // rows to emit: M, or Mp for the MSD form
    int vec_ok;          // 16-byte vector loads are legal for this x
    // kOutKernel
    int8_t* aq;          // [M, Kpad] operand order
    float* as;           // [G, as_ld]
    int as_ld;
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
    int8_t* aq;              // [M, Kpad]
    float* as;               // [G, as_ld]
    int as_ld;
};

// The GEMM's view of one call.  Tensor maps are built on the host.
struct alignas(64) GemmParams {
    CUtensorMap tm_w;    // packed int4 weights [N, Kpad/2] bytes, box {128 B, 128 rows}, SW128
    CUtensorMap tm_a;    // int8 activations [M, Kpad] bytes, box {128 B, TT rows}, SW128
    CUtensorMap tm_ws;   // weight scales [G, N] (fp32 or bf16), box {128, GPK}
    CUtensorMap tm_wz;   // weight zero points [G, N] bf16, box {128, GPK} (asymmetric only)
    CUtensorMap tm_as;   // activation scales [G, M] fp32 (row stride as_ld), box {TT, GPK}
    void* out;           // y bf16 [M, N] (row stride ldy), or int32 partials [G, M, N]
    float* partials;     // stream-K partial tiles: [2 * grid][TT][128] fp32
    int* counters;       // [n_tiles] arrival counters, zero between calls
    int* status;         // device status word
    int M, N, Kpad, G;
    int64_t ldy;
    int n_wt, n_tt, units_per_tile, total_units, kb_total;
};

struct GemmConfig {
    int tt;        // token tile (MMA N): 16, 32, 64 or 128
    int gk;        // 64, 128, 256 or 1024
    bool asym;
    bool ws_bf16;
    bool partials; // debug mode: write int32 group partials instead of y
};

cudaError_t launch_quant_act(const QuantParams& p, int out_kind, cudaStream_t stream, bool pdl);
cudaError_t launch_msd_to_kernel(const MsdToKernelParams& p, cudaStream_t stream, bool pdl);

// Launches the GEMM on `grid` persistent CTAs.  Returns cudaErrorInvalidValue
// for an unsupported configuration.
cudaError_t launch_gemm(const GemmParams& p, const GemmConfig& cfg, int grid, cudaStream_t stream,
                        bool pdl);
size_t gemm_smem_bytes(const GemmConfig& cfg);

}  // namespace w4a8
