/*
 * w4a8_b200.h -- C ABI of libw4a8_b200.so, the B200 (sm_100a) mid-group W4A8
 * linear layer.
 *
 * All tensor arguments are raw device pointers to densely packed row-major
 * arrays; bf16 values are 16-bit patterns.  `stream` is a cudaStream_t (NULL =
 * legacy default stream).  Every call is asynchronous on `stream`, allocates
 * no memory, and returns W4A8_OK or a negative status.  Asynchronous failures
 * inside a kernel (a pipeline wait that ran out) are recorded in the
 * workspace's status word: read it with w4a8_workspace_status().
 *
 * Layout conventions (the reference's; mg_kgeom.h in the reference project):
 *   G    = ceil(K / group_size)                       -- w4a8_num_groups()
 *   Kpad = group-padded row length (each group padded to 64 elements;
 *          only the last group can pad when group_size % 64 == 0)
 *   packed int4 weights: [N, Kpad/2] bytes, two codes per byte, even k in the
 *          low nibble, codes in [-8, 7]
 *   scales / zero points: group-major [G, N] (weights), [G, M] (activations)
 *   zero points: integers in code units held in bf16 (asymmetric weights)
 *
 * Each entry point cites the reference interface it replaces.
 */
#ifndef W4A8_B200_H
#define W4A8_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define W4A8_API __attribute__((visibility("default")))
#else
#define W4A8_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define W4A8_OK 0
#define W4A8_ERR_INVALID (-1)     /* bad shape, null or misaligned pointer       */
#define W4A8_ERR_UNSUPPORTED (-2) /* group size / dtype not built                */
#define W4A8_ERR_CUDA (-3)        /* a CUDA call failed: w4a8_last_cuda_error()  */
#define W4A8_ERR_WORKSPACE (-4)   /* workspace missing or smaller than required  */
#define W4A8_ERR_DEVICE (-5)      /* current device is not an sm_100 part         */
#define W4A8_ERR_TIMEOUT (-6)     /* a device-side wait on a peer ran out          */

#define W4A8_DTYPE_BF16 0
#define W4A8_DTYPE_F32 1

/* ---- geometry (npu_ops/python/w4a8_ops.py:63-82,160-178; mg_kgeom.h:64-101) ---- */
W4A8_API int64_t w4a8_num_groups(int64_t K, int32_t group_size);
W4A8_API int64_t w4a8_k_pad_elems(int64_t K, int32_t group_size);
/* Rows `midgroup_quant_a` emits for M rows: M rounded up to 16 / 64 / 128
 * (TileMFor, npu_ops/host/midgroup_quant_a.cpp:37). */
W4A8_API int64_t w4a8_pad_rows(int64_t M);

/* ---- fused linear: y = x @ W^T, activation quantised per (token, group) ----
 * Replaces MidGroupW4A8LinearMethod.apply's quant_a -> gemm pair
 * (npu_ops/python/midgroup_quant.py:163-178, w4a8_ops.py:243-252).
 *   x        bf16 [M, ldx] (ldx >= K)
 *   w_packed int8 [N, Kpad/2]            (16-byte aligned)
 *   w_scale  [G, N] bf16 or f32 (w_scale_dtype)
 *   w_zero   [G, N] bf16, or NULL for symmetric weights
 *   y        bf16 [M, ldy] (ldy >= N)
 * group_size in {64, 128, 256, 1024}; N % 8 == 0.
 * The workspace (w4a8_linear_workspace_size bytes, 1024-byte aligned) must be
 * zero-filled before its first use; calls leave it reusable.  Calls that share
 * a workspace must not overlap in time (use one workspace per stream). */
W4A8_API size_t w4a8_linear_workspace_size(int64_t M, int64_t N, int64_t K, int32_t group_size);
W4A8_API int w4a8_linear(const void* x, int64_t M, int64_t K, int64_t ldx, int64_t N, int32_t group_size,
                const void* w_packed, const void* w_scale, int32_t w_scale_dtype,
                const void* w_zero, void* y, int64_t ldy, void* workspace, size_t workspace_bytes,
                void* stream);

/* ---- the down projection with the SwiGLU activation applied to its input ----
 * y = bf16(silu(gate) * up) @ W^T for gu = [gate | up], bf16 [M, ldx] with
 * ldx >= 2K: gate = columns [0, K), up = columns [K, 2K) (vLLM's
 * MergedColumnParallelLinear output order).  silu(g) = g / (1 + exp(-g)) and
 * the product are computed in fp32 and rounded to bf16 before quantisation,
 * as the reference's layer does in torch before its quant op
 * (F.silu(g) * u in npu_ops/python/bench_decode_layer.py:81; torch_npu.npu_swiglu
 * in npu_ops/python/bench_decode_graph.py:64), so no [M, K] activation tensor
 * and no elementwise kernel sit between gate_up and down.  Otherwise as
 * w4a8_linear (same weights, workspace and rules; K is the down projection's). */
W4A8_API int w4a8_linear_swiglu(const void* gu, int64_t M, int64_t K, int64_t ldx, int64_t N, int32_t group_size,
                                const void* w_packed, const void* w_scale, int32_t w_scale_dtype,
                                const void* w_zero, void* y, int64_t ldy, void* workspace, size_t workspace_bytes,
                                void* stream);

/* The two halves of w4a8_linear, for callers that quantise once and reuse the
 * quantised activation, or time the GEMM alone.  w4a8_linear_gemm reads the
 * activation w4a8_linear_quant left in the same workspace (same M, K). */
W4A8_API int w4a8_linear_quant(const void* x, int64_t M, int64_t K, int64_t ldx, int64_t N,
                      int32_t group_size, void* workspace, size_t workspace_bytes, void* stream);
W4A8_API int w4a8_linear_gemm(int64_t M, int64_t K, int64_t N, int32_t group_size, const void* w_packed,
                     const void* w_scale, int32_t w_scale_dtype, const void* w_zero, void* y,
                     int64_t ldy, void* workspace, size_t workspace_bytes, void* stream);

/* ---- prepared weights: the fast path for weights that are used many times ----
 * One-time regrouping of the reference layout (packed int4 [N, Kpad/2], scales
 * and zero points [G, N]) into contiguous, pre-swizzled 16 KB tiles plus
 * per-row-tile scale rows, so each pipeline stage is filled by one bulk copy.
 * Plays the part of MidGroupW4A8LinearMethod.process_weights_after_loading
 * (npu_ops/python/midgroup_quant.py:148-161), which also re-lays scales once
 * after loading.  `prepared` must be 256-byte aligned. */
W4A8_API size_t w4a8_prepared_weights_size(int64_t N, int64_t K, int32_t group_size, int32_t w_scale_dtype,
                                           int32_t has_zero);
W4A8_API int w4a8_prepare_weights(const void* w_packed, const void* w_scale, int32_t w_scale_dtype,
                                  const void* w_zero, int64_t N, int64_t K, int32_t group_size, void* prepared,
                                  size_t prepared_bytes, void* stream);
/* w4a8_linear on prepared weights (same workspace rules). */
W4A8_API int w4a8_linear_prepared(const void* x, int64_t M, int64_t K, int64_t ldx, int64_t N, int32_t group_size,
                                  const void* prepared, int32_t w_scale_dtype, int32_t has_zero, void* y,
                                  int64_t ldy, void* workspace, size_t workspace_bytes, void* stream);
/* w4a8_linear_swiglu on prepared weights. */
W4A8_API int w4a8_linear_prepared_swiglu(const void* gu, int64_t M, int64_t K, int64_t ldx, int64_t N,
                                         int32_t group_size, const void* prepared, int32_t w_scale_dtype,
                                         int32_t has_zero, void* y, int64_t ldy, void* workspace,
                                         size_t workspace_bytes, void* stream);
/* The GEMM half of w4a8_linear_prepared (after w4a8_linear_quant on the same workspace). */
W4A8_API int w4a8_linear_gemm_prepared(int64_t M, int64_t K, int64_t N, int32_t group_size, const void* prepared,
                                       int32_t w_scale_dtype, int32_t has_zero, void* y, int64_t ldy,
                                       void* workspace, size_t workspace_bytes, void* stream);

/* ---- w4a8_linear without a caller-provided workspace ----
 * No counterpart in the reference.  Same arguments, checks and results as
 * w4a8_linear minus the workspace: its scratch is one fixed
 * W4A8_FIXED_SCRATCH_BYTES array of device memory per device, declared in the
 * library itself, so the call allocates nothing.  For callers that cannot
 * allocate device memory at the call site: foreign-language hosts that hold
 * no device allocator, and serving loops whose allocator must not be entered
 * (cudaMalloc synchronises the device; a caching allocator may be in a
 * no-growth phase).
 *   - Returns W4A8_ERR_WORKSPACE when the call would need more scratch than
 *     the array holds (16 MiB covers M <= 64 on 27648 x 7168 weights).
 *   - The first call on a device looks the array up, clears it and waits for
 *     the clear on `stream`: make that first call before any stream capture.
 *     The same happens again on the first call after the device's context
 *     was reset (the module, and with it the array, is loaded anew).
 *   - Every call on a device shares the one array: calls that overlap in time
 *     (different streams, threads) race on it and must be serialised by the
 *     caller.
 *   - A kernel wait that runs out is recorded in the array's status word:
 *     read (and clear) it with w4a8_fixed_scratch_status. */
#define W4A8_FIXED_SCRATCH_BYTES ((size_t)16 << 20)
W4A8_API int w4a8_linear_fixed_scratch(const void* x, int64_t M, int64_t K, int64_t ldx, int64_t N,
                                       int32_t group_size, const void* w_packed, const void* w_scale,
                                       int32_t w_scale_dtype, const void* w_zero, void* y, int64_t ldy,
                                       void* stream);
/* Status word of the current device's fixed scratch, as w4a8_workspace_status
 * returns it for a workspace (synchronises `stream`; reset != 0 clears it).
 * No counterpart in the reference.  W4A8_ERR_WORKSPACE when no
 * w4a8_linear_fixed_scratch call has run in the current context yet. */
W4A8_API int w4a8_fixed_scratch_status(int32_t reset, void* stream);

/* ---- activation quantiser (fakequant_lab/quant.py:89-141 semantics) ----
 *   a_q       int8 [M, K] natural order
 *   a_scale   [G, M] bf16 bits or f32 (scale_dtype)
 *   a_ksum    int32 [G, M] NEGATED per-group code sums, or NULL */
W4A8_API int w4a8_quant_act(const void* x, int64_t M, int64_t K, int64_t ldx, int32_t group_size,
                   int8_t* a_q, void* a_scale, int32_t scale_dtype, int32_t* a_ksum, void* stream);

/* ---- the reference op torch.ops.npu.midgroup_quant_a ----
 * (npu_ops/host/midgroup_quant_a.cpp:40-78; schema :87-90).  Emits Mp rows
 * (Mp >= M; rows [M, Mp) encode zero with scale = bf16 tiny):
 *   a_hi, a_lo int8 [Mp, Kpad/2]   MSD int4 planes: q = 16*hi + lo + 8
 *   a_scale    bf16 [G, Mp]
 *   a_ksum     int32 [G, Mp]       negated code sums */
W4A8_API int w4a8_midgroup_quant_a(const void* x, int64_t M, int64_t K, int32_t group_size, int64_t Mp,
                          int8_t* a_hi, int8_t* a_lo, void* a_scale, int32_t* a_ksum, void* stream);

/* ---- the reference op torch.ops.npu.midgroup_w4a8_gemm ----
 * (npu_ops/host/midgroup_w4a8_gemm.cpp:143-238; schema :249-250).  Computes the
 * definition form y = sum_g as*ws*sum_k A*(W - wz) from the MSD planes
 * (ReferenceMidGroupGemm, int4_cube_lab/host/gemm_ref.cpp:199-240); a_ksum and
 * w_ksum are the MSD bookkeeping of the reference kernel and are not needed by
 * this path (they may be NULL).  M = rows of a_hi; y bf16 [M, N].
 * Workspace: w4a8_midgroup_gemm_workspace_size bytes, zero-filled before first use. */
W4A8_API size_t w4a8_midgroup_gemm_workspace_size(int64_t M, int64_t N, int64_t K, int32_t group_size);
W4A8_API int w4a8_midgroup_w4a8_gemm(const int8_t* a_hi, const int8_t* a_lo, const void* a_scale,
                            const int32_t* a_ksum, int64_t M, const int8_t* w_q,
                            const void* w_scale, const int32_t* w_ksum, const void* w_zero,
                            int64_t N, int64_t K, int32_t group_size, void* y, void* workspace,
                            size_t workspace_bytes, void* stream);

/* ---- int32 per-group partials P[g, m, n] = sum_{k in g} A_q*(W - wz) ----
 * The exactness contract of the reference (fakequant_lab/run_selftest.py:104-141,
 * int4_cube_lab/host/ragged_layout_test.cpp:112-148), computed by the same
 * tensor-core path as w4a8_linear.  partials int32 [G, M, N].  Test-sized
 * problems; workspace as for w4a8_linear. */
W4A8_API int w4a8_group_partials(const void* x, int64_t M, int64_t K, int64_t ldx, int64_t N,
                        int32_t group_size, const void* w_packed, const void* w_zero,
                        int32_t* partials, void* workspace, size_t workspace_bytes, void* stream);

/* ---- one-shot all-reduce over peer memory (tensor-parallel row reductions) ----
 * Replaces the reference's peer-read all-reduce (npu_ops/kernel/peer_allreduce_f32.cpp:127-270,
 * driven from npu_ops/python/peer_allreduce.py) for small bf16 messages.  One
 * handle per rank and device; every rank of the group calls
 * w4a8_ar_allreduce_bf16 in the same order with the same count.
 *   create:     allocates one buffer of two message slots of max_bytes plus flags
 *               (max_bytes a multiple of 16); world <= 8.
 *   ipc_handle: this rank's CUDA IPC handle (w4a8_ar_ipc_handle_size() bytes);
 *   open_peers: `handles` = world handles concatenated in rank order (own ignored).
 *   allreduce:  out[i] = bf16(sum over ranks, in rank order, of in[i] in fp32);
 *               count a multiple of 8 elements, count * 2 <= max_bytes, in / out
 *               16-byte aligned, in == out allowed.  Graph-capturable.  A wait for
 *               a peer is bounded (1 s): on expiry the call leaves its output
 *               untouched and records the failure, which w4a8_ar_status returns
 *               as W4A8_ERR_TIMEOUT (after the stream's work is done).
 * This entry point allocates device memory in create (nothing at call time). */
typedef struct w4a8_ar w4a8_ar;
W4A8_API size_t w4a8_ar_ipc_handle_size(void);
W4A8_API int w4a8_ar_create(int32_t rank, int32_t world, size_t max_bytes, w4a8_ar** out);
W4A8_API int w4a8_ar_ipc_handle(w4a8_ar* h, void* handle_out);
W4A8_API int w4a8_ar_open_peers(w4a8_ar* h, const void* handles);
/* Same, for ranks driven from this process (peers[r] = rank r's handle, own
 * ignored; on other devices peer access is enabled). */
W4A8_API int w4a8_ar_open_local(w4a8_ar* h, w4a8_ar* const* peers);
W4A8_API size_t w4a8_ar_max_bytes(const w4a8_ar* h);
W4A8_API int w4a8_ar_allreduce_bf16(w4a8_ar* h, const void* in, void* out, int64_t count, void* stream);
W4A8_API int w4a8_ar_status(w4a8_ar* h, int32_t reset);
W4A8_API int w4a8_ar_destroy(w4a8_ar* h);

/* ---- row-parallel linear fused with its all-reduce (tensor parallelism) ----
 * y = sum over the ranks of ar's group, in rank order in fp32 and rounded once
 * to bf16, of this rank's w4a8_linear_prepared result (x: the rank's K shard;
 * act = W4A8_ACT_SWIGLU takes x = [gate | up] as w4a8_linear_prepared_swiglu).
 * Every rank calls it in the same order with the same M and N, like
 * w4a8_ar_allreduce_bf16; M * N * 2 <= w4a8_ar_max_bytes(ar), (M * N) % 8 == 0,
 * y dense [M, N] and 16-byte aligned.  The GEMM's epilogue (and its stream-K
 * fix-up, for output tiles split between CTAs) stores each finished bf16 tile
 * straight into this rank's receive slot of the all-reduce buffer, and one
 * reduction kernel then publishes this rank's flags, waits (bounded, 1 s) for
 * the others' and sums every rank's slot in place with peer loads: the
 * partial output's own buffer and the all-reduce's copy pass are gone
 * (W4A8_OPT_AR_PUSH: the epilogue stores into every rank's slot instead).  The same bits as w4a8_linear_prepared
 * followed by w4a8_ar_allreduce_bf16.  A wait that runs out leaves y
 * untouched and is reported by w4a8_ar_status.  Replaces the reference's
 * row-parallel GEMM + peer all-reduce pair, fused as its design notes
 * propose (MGCKPT/P6.5_TP.md:900-957; npu_ops/kernel/peer_allreduce_f32.cpp:127-270). */
#define W4A8_ACT_NONE 0
#define W4A8_ACT_SWIGLU 1
W4A8_API int w4a8_linear_prepared_allreduce(const void* x, int64_t M, int64_t K, int64_t ldx, int64_t N,
                                            int32_t group_size, const void* prepared, int32_t w_scale_dtype,
                                            int32_t has_zero, int32_t act, void* y, void* workspace,
                                            size_t workspace_bytes, w4a8_ar* ar, void* stream);

/* ---- status ---- */
/* Synchronises `stream` and returns the device status word of `workspace`
 * (0 = no kernel reported a failure; otherwise 0x100 + the id of the wait
 * that ran out).  reset != 0 clears it. */
W4A8_API int w4a8_workspace_status(void* workspace, int32_t reset, void* stream);
W4A8_API const char* w4a8_status_string(int status);
W4A8_API int w4a8_last_cuda_error(void);
/* Library build: returns the sm architecture it was compiled for (100). */
W4A8_API int w4a8_build_arch(void);

/* ---- options (process-wide; no counterpart in the reference) ----
 * W4A8_OPT_FUSED_QUANT: a linear call with M <= 16, group size <= 256 and
 * 16-byte aligned activation rows quantises its activation inside the GEMM
 * (four quantiser warps per CTA, the bf16 rows brought in by 2-D tensor
 * copies) instead of running the standalone quantiser kernel first.  Same
 * bits.  Off by default: every CTA quantises the activation slice of each
 * weight tile it visits, and measured on B200 the fused call is slower at
 * every decode size (e.g. gate_up M = 16: 183 us against 34 us per call).
 * W4A8_OPT_AR_PUSH: w4a8_linear_prepared_allreduce stores every output tile
 * into every rank's receive slot (posted peer stores from the GEMM epilogue)
 * instead of its own slot only, the peers then reading it (the default).
 * Returns the previous flags. */
#define W4A8_OPT_FUSED_QUANT 1
#define W4A8_OPT_AR_PUSH 2
W4A8_API int w4a8_set_options(int32_t flags);

#ifdef __cplusplus
}
#endif

#endif /* W4A8_B200_H */
