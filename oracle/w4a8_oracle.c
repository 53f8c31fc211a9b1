/*
 * w4a8_oracle.c -- CPU restatement of the reference's mid-group W4A8 path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the CUDA kernels are
 * compared against; nothing in the shipped library links, loads or calls it.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it.
 *
 * Every function restates one piece of the reference algorithm and cites the
 * reference file:line it follows (paths relative to the reference project):
 *
 *   group geometry ............ npu_ops/kernel/mg_kgeom.h:64-101
 *   activation quantiser ...... fakequant_lab/quant.py:89-141,153-173
 *                               (sym int8, bf16-rounded scale, true division,
 *                               round-half-even, clamp [-128,127])
 *   MSD planes ................ fakequant_lab/quant.py:204-218,
 *                               int4_cube_lab/host/gemm_ref.cpp:62-90,
 *                               npu_ops/kernel/midgroup_quant_a.inc:1-30 (pad rows)
 *   int4 packing .............. npu_ops/python/w4a8_ops.py:142-148,231-239,
 *                               int4_cube_lab/host/gemm_ref.cpp:42-60
 *   group partials ............ fakequant_lab/fake_linear.py:170-178 and the
 *                               definition form of gemm_ref.cpp:219-232
 *   fp32 rescale order ........ fakequant_lab/fake_linear.py:170-179
 *   exact float64 reference ... fakequant_lab/run_selftest.py:104-121
 *
 * Pinned against golden vectors produced by the reference's own Python code
 * (tests/golden/make_golden.py) and against the reference's C++ CPU GEMM
 * compiled from its own sources (oracle/Makefile, target `ref`).
 *
 * Build: gcc -O3 -fopenmp -shared -fPIC (oracle/Makefile).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_API __attribute__((visibility("default")))

/* ---- bf16 <-> fp32 (int4_cube_lab/host/bf16.h:9-27 semantics: RNE) ---- */

ORC_API float orc_bf16_to_f32(uint16_t b)
{
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

ORC_API uint16_t orc_f32_to_bf16(float f)
{
    uint32_t u;
    memcpy(&u, &f, sizeof u);
    if (isnan(f)) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

/* ---- ragged-K group geometry (mg_kgeom.h:64-101, w4a8_ops.py:157-178) ---- */

#define ORC_KALIGN 64 /* int4 fractal: 32 bytes = 64 elements (mg_kgeom.h:52) */

static int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

ORC_API int64_t orc_num_groups(int64_t K, int32_t gk) { return cdiv(K, gk); }

ORC_API int64_t orc_group_real(int64_t g, int64_t K, int32_t gk)
{
    int64_t G = cdiv(K, gk);
    return (g + 1 < G) ? gk : K - (G - 1) * (int64_t)gk;
}

ORC_API int64_t orc_group_stride(int32_t gk) { return cdiv(gk, ORC_KALIGN) * ORC_KALIGN; }

ORC_API int64_t orc_k_pad_elems(int64_t K, int32_t gk)
{
    int64_t G = cdiv(K, gk);
    return (G - 1) * orc_group_stride(gk) + cdiv(orc_group_real(G - 1, K, gk), ORC_KALIGN) * ORC_KALIGN;
}

/* ---- activation quantiser: quant.py:102-105 (scale), :138-141 (codes) ----
 *
 * One (row, group): amax over the REAL members, fp32 `amax / 127` rounded to
 * bf16 (RNE), bf16 zero replaced by bf16 tiny (quant.py:83-86), then
 * q = clamp(rint(x / float(scale)), -128, 127) with an IEEE fp32 division and
 * round-half-to-even.  ksum_neg = -sum(q) over the group (the negated row sum
 * the kernel consumes, midgroup_quant_a.inc:11). */
static void quant_group(const uint16_t* x, int64_t n, int8_t* q, uint16_t* scale_out,
                        int32_t* ksum_out)
{
    float amax = 0.0f;
    for (int64_t k = 0; k < n; ++k) {
        float v = fabsf(orc_bf16_to_f32(x[k]));
        if (v > amax) amax = v;
    }
    uint16_t sb = orc_f32_to_bf16(amax / 127.0f);
    if ((sb & 0x7FFFu) == 0) sb = 0x0080u; /* torch.finfo(bfloat16).tiny */
    const float s = orc_bf16_to_f32(sb);
    int32_t acc = 0;
    for (int64_t k = 0; k < n; ++k) {
        float r = nearbyintf(orc_bf16_to_f32(x[k]) / s);
        if (r > 127.0f) r = 127.0f;
        if (r < -128.0f) r = -128.0f;
        q[k] = (int8_t)r;
        acc += (int32_t)q[k];
    }
    *scale_out = sb;
    *ksum_out = -acc;
}

/* x: bf16 bits [M,K] (row stride ldx).  q: [M,K] natural order.
 * scale: bf16 bits [G,M] group-major.  ksum_neg: [G,M] (may be NULL). */
ORC_API void orc_quant_act(const uint16_t* x, int64_t M, int64_t K, int64_t ldx, int32_t gk,
                           int8_t* q, uint16_t* scale, int32_t* ksum_neg)
{
    const int64_t G = cdiv(K, gk);
#pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; ++m) {
        for (int64_t g = 0; g < G; ++g) {
            const int64_t real = orc_group_real(g, K, gk);
            uint16_t sb;
            int32_t ks;
            quant_group(x + m * ldx + g * gk, real, q + m * K + g * gk, &sb, &ks);
            scale[g * M + m] = sb;
            if (ksum_neg) ksum_neg[g * M + m] = ks;
        }
    }
}

/* ---- nibble helpers (gemm_ref.cpp:26-40, ragged_layout_test.cpp:33-39) ---- */

static void put_nibble(int8_t* out, int64_t pos, int v)
{
    uint8_t* b = (uint8_t*)out + (pos >> 1);
    const uint8_t nib = (uint8_t)v & 0x0Fu;
    if (pos & 1) *b = (uint8_t)((*b & 0x0Fu) | (nib << 4));
    else         *b = (uint8_t)((*b & 0xF0u) | nib);
}

static int get_nibble(const int8_t* p, int64_t pos)
{
    const uint8_t b = ((const uint8_t*)p)[pos >> 1];
    const uint8_t n = (pos & 1) ? (uint8_t)(b >> 4) : (uint8_t)(b & 0x0F);
    return (n & 8) ? (int)n - 16 : (int)n;
}

/* codes [rows,K] in [-8,7] -> packed [rows, Kpad/2], group g at element offset
 * g*ceil(gk/64)*64, even element in the LOW nibble, pad slots zero
 * (w4a8_ops.py:231-239, gemm_ref.cpp:42-60). */
ORC_API void orc_pack_int4_grouped(const int8_t* codes, int64_t rows, int64_t K, int32_t gk,
                                   int8_t* out)
{
    const int64_t G = cdiv(K, gk), Kpad = orc_k_pad_elems(K, gk), st = orc_group_stride(gk);
    memset(out, 0, (size_t)(rows * (Kpad / 2)));
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t g = 0; g < G; ++g) {
            const int64_t real = orc_group_real(g, K, gk);
            for (int64_t k = 0; k < real; ++k)
                put_nibble(out, r * Kpad + g * st + k, codes[r * K + g * gk + k]);
        }
}

ORC_API void orc_unpack_int4_grouped(const int8_t* packed, int64_t rows, int64_t K, int32_t gk,
                                     int8_t* codes)
{
    const int64_t G = cdiv(K, gk), Kpad = orc_k_pad_elems(K, gk), st = orc_group_stride(gk);
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t g = 0; g < G; ++g) {
            const int64_t real = orc_group_real(g, K, gk);
            for (int64_t k = 0; k < real; ++k)
                codes[r * K + g * gk + k] = (int8_t)get_nibble(packed, r * Kpad + g * st + k);
        }
}

/* ---- midgroup_quant_a outputs (the MSD planes) ----
 * hi = q >> 4, lo nibble = (q & 15) ^ 8, so q == 16*hi + lo_value + 8
 * (quant.py:204-218, gemm_ref.cpp:62-90).  Unwritten slots -- the group pad
 * and the rows [M, Mp) -- encode q = 0: hi 0x0, lo 0x8; rows [M, Mp) carry
 * scale = bf16 tiny and ksum 0 (midgroup_quant_a.inc:22-27). */
ORC_API void orc_midgroup_quant_a(const uint16_t* x, int64_t M, int64_t Mp, int64_t K, int32_t gk,
                                  int8_t* a_hi, int8_t* a_lo, uint16_t* a_scale, int32_t* a_ksum)
{
    const int64_t G = cdiv(K, gk), Kpad = orc_k_pad_elems(K, gk), st = orc_group_stride(gk);
    int8_t* q = (int8_t*)malloc((size_t)(M * K > 0 ? M * K : 1));
    uint16_t* s = (uint16_t*)malloc((size_t)(G * M > 0 ? G * M : 1) * sizeof(uint16_t));
    int32_t* ks = (int32_t*)malloc((size_t)(G * M > 0 ? G * M : 1) * sizeof(int32_t));
    orc_quant_act(x, M, K, K, gk, q, s, ks);
    memset(a_hi, 0x00, (size_t)(Mp * (Kpad / 2)));
    memset(a_lo, 0x88, (size_t)(Mp * (Kpad / 2)));
    for (int64_t m = 0; m < Mp; ++m)
        for (int64_t g = 0; g < G; ++g) {
            a_scale[g * Mp + m] = (m < M) ? s[g * M + m] : (uint16_t)0x0080u;
            a_ksum[g * Mp + m] = (m < M) ? ks[g * M + m] : 0;
            if (m >= M) continue;
            const int64_t real = orc_group_real(g, K, gk);
            for (int64_t k = 0; k < real; ++k) {
                const int8_t e = q[m * K + g * gk + k];
                put_nibble(a_hi, m * Kpad + g * st + k, (int8_t)(e >> 4));
                put_nibble(a_lo, m * Kpad + g * st + k, (int8_t)(e ^ 8));
            }
        }
    free(q);
    free(s);
    free(ks);
}

/* Rebuild int8 codes from MSD planes: a = 16*hi + lo + 8 (quant.py:221-223). */
ORC_API void orc_msd_recombine(const int8_t* a_hi, const int8_t* a_lo, int64_t rows, int64_t K,
                               int32_t gk, int8_t* q)
{
    const int64_t G = cdiv(K, gk), Kpad = orc_k_pad_elems(K, gk), st = orc_group_stride(gk);
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t g = 0; g < G; ++g) {
            const int64_t real = orc_group_real(g, K, gk);
            for (int64_t k = 0; k < real; ++k) {
                const int64_t pos = r * Kpad + g * st + k;
                q[r * K + g * gk + k] = (int8_t)(16 * get_nibble(a_hi, pos) + get_nibble(a_lo, pos) + 8);
            }
        }
}

/* ---- int32 group partials, definition form ----
 * P[g,m,n] = sum_{k in g} A[m,k] * (W[n,k] - wz[g,n])   (gemm_ref.cpp:219-232);
 * fake_linear.py:175-177 computes the same integer as A.W - wz * sum(A).
 * wz: [G,N] zero points (integers held in float), NULL = symmetric. */
ORC_API void orc_group_partials(const int8_t* qa, const int8_t* qw, const float* wz, int64_t M,
                                int64_t N, int64_t K, int32_t gk, int32_t* P)
{
    const int64_t G = cdiv(K, gk);
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        const int8_t* wrow = qw + n * K;
        for (int64_t g = 0; g < G; ++g) {
            const int64_t base = g * gk, real = orc_group_real(g, K, gk);
            const int32_t z = wz ? (int32_t)wz[g * N + n] : 0;
            for (int64_t m = 0; m < M; ++m) {
                const int8_t* arow = qa + m * K + base;
                int32_t dot = 0;
                for (int64_t k = 0; k < real; ++k)
                    dot += (int32_t)arow[k] * ((int32_t)wrow[base + k] - z);
                P[(g * M + m) * N + n] = dot;
            }
        }
    }
}

/* ---- fp32 GEMM in the reference oracle's order (fake_linear.py:170-179) ----
 * acc[m,n] = 0; for g: acc += partial * (as[g,m] * ws[g,n]) with the scale
 * product rounded to fp32 first and no fused multiply-add (the Makefile builds
 * with -ffp-contract=off).  as/ws: fp32 [G,M], [G,N] (the caller widens bf16
 * scales exactly). */
ORC_API void orc_gemm_kernel_order(const int8_t* qa, const float* as, const int8_t* qw,
                                   const float* ws, const float* wz, int64_t M, int64_t N,
                                   int64_t K, int32_t gk, float* y)
{
    const int64_t G = cdiv(K, gk);
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        const int8_t* wrow = qw + n * K;
        for (int64_t m = 0; m < M; ++m) {
            const int8_t* arow = qa + m * K;
            float acc = 0.0f;
            for (int64_t g = 0; g < G; ++g) {
                const int64_t base = g * gk, real = orc_group_real(g, K, gk);
                const int32_t z = wz ? (int32_t)wz[g * N + n] : 0;
                int32_t dot = 0;
                for (int64_t k = 0; k < real; ++k)
                    dot += (int32_t)arow[base + k] * ((int32_t)wrow[base + k] - z);
                const float c = as[g * M + m] * ws[g * N + n];
                const float t = (float)dot * c;
                acc = acc + t;
            }
            y[m * N + n] = acc;
        }
    }
}

/* ---- exact reference: integer sums, float64 rescale (run_selftest.py:104-121) ---- */
ORC_API void orc_gemm_f64(const int8_t* qa, const float* as, const int8_t* qw, const float* ws,
                          const float* wz, int64_t M, int64_t N, int64_t K, int32_t gk, double* y)
{
    const int64_t G = cdiv(K, gk);
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        const int8_t* wrow = qw + n * K;
        for (int64_t m = 0; m < M; ++m) {
            const int8_t* arow = qa + m * K;
            double acc = 0.0;
            for (int64_t g = 0; g < G; ++g) {
                const int64_t base = g * gk, real = orc_group_real(g, K, gk);
                const int32_t z = wz ? (int32_t)wz[g * N + n] : 0;
                int64_t dot = 0;
                for (int64_t k = 0; k < real; ++k)
                    dot += (int64_t)arow[base + k] * ((int64_t)wrow[base + k] - z);
                acc += (double)dot * ((double)as[g * M + m] * (double)ws[g * N + n]);
            }
            y[m * N + n] = acc;
        }
    }
}

/* bf16 RNE of a float array (the final `acc.to(x.dtype)` of fake_linear.py:149). */
ORC_API void orc_f32_to_bf16_array(const float* in, int64_t n, uint16_t* out)
{
    for (int64_t i = 0; i < n; ++i) out[i] = orc_f32_to_bf16(in[i]);
}

/* Threads of the OpenMP loops above (the process-wide setting: the reference
 * C++ GEMM linked into the same process shares it).  A launcher that exports
 * OMP_NUM_THREADS=1 to each rank (torchrun) would otherwise leave the CPU
 * baseline on one core. */
#ifdef _OPENMP
#include <omp.h>
#endif
ORC_API void orc_set_threads(int32_t n)
{
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
