/*
 * triposplat_b200.h — C ABI of libtriposplat_b200.so, the B200 (sm_100a) implementation of
 * the TripoSplat flow-model hot path: NF24 int16 dequant GEMM, exact SDPA, and the
 * prologue / epilogue kernels around them.
 *
 * Drop-in contract.  Every function below that cites a reference file keeps that
 * function's name, argument list, argument meaning and status codes, so the reference's
 * ctypes bindings (scripts/native_linear_rnf8_avx512_patch.py:201-210,
 * scripts/native_sdpa_ctypes.py:14-20, the norm/GELU/SiLU/block/sampler patches) bind this
 * library unchanged.  Differences, all deliberate:
 *   - every float / code pointer is a CUDA device pointer (device, managed or mapped
 *     memory); a host-only pointer returns -9 instead of being dereferenced;
 *   - work is queued asynchronously on the calling thread's stream
 *     (triposplat_b200_set_stream, default: the legacy default stream); the call returns
 *     once the work is enqueued;
 *   - the trailing `threads` argument is accepted and ignored.
 *
 * Status codes: 0 ok; -1 null pointer; -2 bad dimension / stages; -3 bad range / bias
 * length; -4 alignment (range start/count not a multiple of 16, or an unaligned q/out
 * pointer for SDPA); -5 workspace allocation failed; -6 problem larger than a fixed scratch; -9 pointer not device-accessible;
 * -10 kernel launch failed; -11 an earlier kernel of this library gave up on a bounded
 * wait (see triposplat_b200_status); -12 no usable CUDA device.
 */
#ifndef TRIPOSPLAT_B200_H
#define TRIPOSPLAT_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- runtime controls --
 * No reference counterpart: the CPU library has no streams and a thread-local workspace. */

/* Stream (cudaStream_t) used by this thread's subsequent calls; NULL = legacy default. */
void triposplat_b200_set_stream(void* stream);
void* triposplat_b200_get_stream(void);
/* Non-zero once a kernel of this library recorded a bounded-wait timeout (host-mapped
 * status word, readable without synchronising); entry points then return -11. */
int triposplat_b200_status(void);
void triposplat_b200_clear_status(void);
/* Pre-size the library workspace of the current (device, stream), e.g. before capturing
 * the calls into a CUDA graph, so no call grows it later. */
int triposplat_b200_workspace_reserve(uint64_t bytes);
int triposplat_b200_workspace_stats(uint64_t* allocations, uint64_t* capacity_bytes);
void triposplat_b200_workspace_release(void);
int triposplat_b200_abi_version(void);
/* Text of the last CUDA launch / tensor-map error seen by this thread's calls. */
const char* triposplat_b200_last_error(void);
/* Number of kernels this library has launched in this process (all devices). */
uint64_t triposplat_b200_launch_count(void);
/* While enabled, every launch is bracketed by CUDA events on its stream. */
void triposplat_b200_profile_enable(int on);
/* Waits for the bracketed launches recorded so far and returns, per kernel family
 * (0 GEMM tensor-core, 1 GEMM activation split, 2 GEMM scalar tail, 3 SDPA attention,
 * 4 SDPA split, 5 elementwise, 6 multi-GPU peer barrier, 7 peer K / V gather and partial
 * reduction; n entries), the launch count and summed device ms. */
int triposplat_b200_profile_collect(uint64_t* launches, double* total_ms, int n);
/* Same; keep != 0 leaves the events registered (a captured CUDA graph records into them on
 * every replay, so each read reflects the latest replay). */
int triposplat_b200_profile_collect2(uint64_t* launches, double* total_ms, int n, int keep);

/* ---------------------------------------------------------------- NF24 GEMM ----------
 * Y[M, N] = X[M, K] . W + bias,  W[k, n] = scale[n] * (256*q01[k, n] + q2[k, n]).
 * For NF24: codes0_t = int16 q01 [K, N]; codes1_t = codes2_t = int8 q2 [K, N];
 * scales0 = scales1 = scales2 = scale [N]; codebook is not read (any non-null pointer);
 * stages must be 3.  X fp32 with row stride stride_x; out fp32 with row stride stride_out.
 * Work space (library-owned, per device and stream): the split activation, and from M = 2048
 * rows on (the tensor-core path) also a k-contiguous copy of the requested columns' codes,
 * 3 bytes per weight with K rounded up to 16, written by each call before its GEMM; the
 * result is the same bit for bit as without the copy. */

/* replaces scripts/gemm_nf24_i16_avx512.c:199-220 */
int triposplat_gemm_rnf8_avx512(const float* x, const uint8_t* codes0_t, const uint8_t* codes1_t,
                                const uint8_t* codes2_t, const float* scales0,
                                const float* scales1, const float* scales2,
                                const float* codebook, const float* bias, float* out, int M,
                                int K, int N, int stride_x, int stride_out, int threads,
                                int stages);

/* replaces scripts/gemm_nf24_i16_avx512.c:151-197; out is [M, output_count] */
int triposplat_gemm_rnf8_avx512_range(const float* x, const uint8_t* codes0_t,
                                      const uint8_t* codes1_t, const uint8_t* codes2_t,
                                      const float* scales0, const float* scales1,
                                      const float* scales2, const float* codebook,
                                      const float* bias, float* out, int M, int K, int N,
                                      int output_start, int output_count, int stride_x,
                                      int stride_out, int threads, int stages);

/* replaces scripts/gemm_nf24_i16_avx512_tail.c:8-49 (any N; reference operation order) */
int triposplat_gemm_rnf8_avx512_tail(const float* x, const uint8_t* codes0_t,
                                     const uint8_t* codes1_t, const uint8_t* codes2_t,
                                     const float* scales0, const float* scales1,
                                     const float* scales2, const float* codebook,
                                     const float* bias, float* out, int M, int K, int N,
                                     int stride_x, int stride_out, int threads, int stages);

/* No counterpart in the reference.  Same arguments and result as
 * triposplat_gemm_rnf8_avx512, for callers that cannot let a library allocate device
 * memory: hosts whose device memory belongs to their own allocator or to a fixed plan made
 * at start-up (a serving process that reserves the GPU's memory up front, an application
 * that must account for every byte it places on the device), and loops that cannot absorb
 * cudaMalloc's device-wide synchronisation.  It calls no allocator: its scratch is a fixed
 * 32 MiB __device__ array that every GPU loading the library holds until exit, so it
 * serves split activations of up to 32 MiB (triposplat_b200_split_bytes(M, K); e.g.
 * M <= 8184 at K = 1024), returns -6 beyond, and -4 unless N % 16 == 0 with 16-byte aligned
 * code planes and output (stride_out % 4 == 0).  All calls on a device share the scratch:
 * calls whose kernels may overlap on the GPU race, so order them on one stream.  Nothing
 * in the scratch needs to start at zero.  The first call on a device does its set-up —
 * resolves the scratch's device address and maps a static status word (cudaHostRegister
 * of a static page, not an allocation) for the kernels' bounded waits — so make that first
 * call before any stream capture.  A wait that gives up is reported by
 * triposplat_b200_status() as for every other entry point, also when this is the first
 * library call on the device. */
int triposplat_gemm_nf24_noalloc(const float* x, const uint8_t* codes0_t, const uint8_t* codes1_t,
                                 const uint8_t* codes2_t, const float* scales0,
                                 const float* scales1, const float* scales2,
                                 const float* codebook, const float* bias, float* out, int M,
                                 int K, int N, int stride_x, int stride_out, int threads,
                                 int stages);

/* No reference counterpart: fused B200 entry points.  Activations pass between kernels in
 * the GEMM's split format — fp16 hi/lo planes [M, Kp] plus one power-of-two scale per
 * row — in a caller buffer of triposplat_b200_split_bytes(M, K) bytes
 * (256-byte aligned), so LayerNorm / modulation / GELU / residual passes fold into the
 * kernels that produce or consume the activations. */
uint64_t triposplat_b200_split_bytes(int M, int K);
int triposplat_b200_split_f32(const float* x, int M, int K, int stride_x, void* split);
/* LayerNorm without affine, then (if shift and scale are non-null, [B, mod_ld] with
 * b = row / rows_per_batch) h*(1+scale[b])+shift[b], written as a split buffer. */
int triposplat_b200_ln_modulate_split(const float* x, int M, int C, float eps, const float* shift,
                                      const float* scale, int mod_ld, int rows_per_batch,
                                      void* split);
/* The same, and in the same pass the row scales of next_split (the split buffer of an
 * [M, next_K] activation) for a following triposplat_b200_gemm_nf24_split_nk mode 4: per
 * row 2^-s with GELU(h.W + b) * 2^s < 2^15 for any weight whose columns have euclidean
 * norm <= wnorm and any bias with |b| <= bmax (Cauchy-Schwarz on the row h as split).
 * next_split 256-byte aligned; its planes are written by that GEMM. */
int triposplat_b200_ln_modulate_split_bound(const float* x, int M, int C, float eps,
                                            const float* shift, const float* scale, int mod_ld,
                                            int rows_per_batch, void* split, void* next_split,
                                            int next_K, float wnorm, float bmax);
/* NF24 GEMM over a split buffer; mode 0 store, 1 GELU(tanh) store, 2 out += gate[b]*y
 * (gate [B, gate_ld], b = row / rows_per_batch), 3 out += y.  N % 16 == 0; out 16-byte
 * aligned with stride_out % 4 == 0 (the outputs leave through TMA stores). */
int triposplat_b200_gemm_nf24_split(const void* split, int M, int K, const int16_t* code01_t,
                                    const int8_t* q2_t, const float* scale, const float* bias,
                                    float* out, int N, int stride_out, int mode,
                                    const float* gate, int gate_ld, int rows_per_batch);
/* No reference counterpart: triposplat_b200_gemm_nf24_split restricted to the output columns
 * [start, start + count) of the N-column weight (out [M, count], stride_out per row): the
 * column windows a tensor-parallel rank computes.  start, count multiples of 16. */
int triposplat_b200_gemm_nf24_split_range(const void* split, int M, int K, const int16_t* code01_t,
                                          const int8_t* q2_t, const float* scale, const float* bias,
                                          float* out, int N, int start, int count, int stride_out,
                                          int mode, const float* gate, int gate_ld,
                                          int rows_per_batch);

/* No reference counterpart: copies a weight's reference-layout code planes (code01_t int16
 * [K, N], q2_t int8 [K, N]) into k-contiguous planes code01_nk int16 [N, K], q2_nk int8
 * [N, K] for triposplat_b200_gemm_nf24_split_nk (once, at load). */
int triposplat_b200_nf24_codes_to_nk(const int16_t* code01_t, const int8_t* q2_t, int K, int N,
                                     int16_t* code01_nk, int8_t* q2_nk);

/* No reference counterpart: triposplat_b200_gemm_nf24_split_range on k-contiguous planes.
 * Row n holds output column n's K codes, rows ldk elements apart (ldk >= K; an offset
 * pointer with ldk > K selects a window of input features).  16-byte aligned planes,
 * ldk % 16 == 0.  Same modes and status codes as the split entry, plus mode 4: GELU(tanh)
 * written into `out` read as the split buffer of an [M, count] activation (256-byte
 * aligned, stride_out == count), under the row scales triposplat_b200_ln_modulate_split_bound
 * stored there. */
int triposplat_b200_gemm_nf24_split_nk(const void* split, int M, int K, const int16_t* code01_nk,
                                       const int8_t* q2_nk, int ldk, const float* scale,
                                       const float* bias, float* out, int N, int start, int count,
                                       int stride_out, int mode, const float* gate, int gate_ld,
                                       int rows_per_batch);

/* replaces scripts/gemm_nf24_i16_avx512.c:222-224 (rows per CTA tile here) */
int triposplat_gemm_rnf8_avx512_row_tile(void);
/* replaces scripts/gemm_nf24_i16_avx512.c:226-228; returns 4 (= nf24_i16) */
int triposplat_gemm_rnf8_avx512_residual_mode(void);

/* ------------------------------------------------ fused NF24 MLP and QKV projection -----
 * The reference's fused CPU entry points, on device pointers.  Each stage runs as one
 * tensor-core launch over all rows; the intermediate (hidden [M, 4096] or qkv [B*L, N])
 * lives in the library workspace between launches (the chunked MLP uses the caller's
 * hidden buffer instead). */

/* replaces scripts/native_nf24_mlp_avx512.c:143-205: out = GELU_tanh(x W1 + b1) W2 + b2;
 * K = 1024, H = 4096, N = 1024 as the reference requires (-1 null, -2 sizes / strides) */
int triposplat_mlp_nf24_gelu_f32_avx512(const float* x, const uint8_t* w1_code01_t,
                                        const uint8_t* w1_code2_t, const float* w1_scales,
                                        const float* w1_bias, const uint8_t* w2_code01_t,
                                        const uint8_t* w2_code2_t, const float* w2_scales,
                                        const float* w2_bias, float* out, int M, int K, int H,
                                        int N, int stride_x, int stride_out, int threads);
/* replaces scripts/native_nf24_mlp_chunked_avx512.c:3-60: the same over chunks of
 * chunk_rows rows, hidden [hidden_capacity_rows, H] supplied by the caller (device) */
int triposplat_mlp_nf24_gelu_chunked_f32_avx512(
    const float* x, const uint8_t* w1_code01_t, const uint8_t* w1_code2_t,
    const float* w1_scales, const float* w1_bias, const uint8_t* w2_code01_t,
    const uint8_t* w2_code2_t, const float* w2_scales, const float* w2_bias, float* hidden,
    float* out, int M, int K, int H, int N, int stride_x, int stride_out,
    int hidden_capacity_rows, int chunk_rows, int threads);
/* replace scripts/native_nf24_mlp_avx512.c:207-213 (row tile of the GEMM; hidden bytes of
 * one row tile) */
int triposplat_mlp_nf24_row_tile(void);
int triposplat_mlp_nf24_hidden_workspace_bytes_per_thread(void);
/* replaces scripts/gemm_nf24_qkv_direct_avx512.c:87-199: x [B*L, K] . W [K, 3*H*64] + b,
 * then the RoPE / per-head RMSNorm / pack of
 * triposplat_qkv_rope_rmsnorm_pack_f32_avx512_v2 (q_bhld [B,H,L,64], packed_k / packed_v
 * [B,H,64,L_padded], zero tail) */
int triposplat_gemm_nf24_qkv_rope_rmsnorm_pack_f32_avx512(
    const float* x, const uint8_t* codes0_t, const uint8_t* codes1_t, const uint8_t* codes2_t,
    const float* scales0, const float* scales1, const float* scales2, const float* codebook,
    const float* bias, const float* frequencies, const float* q_gamma, const float* k_gamma,
    float* q_bhld, float* packed_k, float* packed_v, int B, int L, int K, int N, int H, int D,
    int L_padded, int frequency_batches, int threads, int stages);
/* replace scripts/gemm_nf24_qkv_direct_avx512.c:201-207 (row tile; residual mode 4 =
 * nf24_i16) and scripts/gemm_nf24_qkv_direct_tile_avx512.c:149-151 (qkv bytes of one row
 * tile) */
int triposplat_gemm_nf24_qkv_direct_row_tile(void);
int triposplat_gemm_nf24_qkv_direct_residual_mode(void);
int triposplat_gemm_nf24_qkv_direct_tile_bytes(void);

/* ---------------------------------------------------------------- exact SDPA ---------
 * O = softmax(0.125 * Q K^T + key_bias) V, head_dim 64, q/k/v/out [B, H, L, 64] fp32. */

/* replaces scripts/native_sdpa_avx512_exact_q8t512.c:137-332; key bias [Lk] shared by all (b,h) */
int triposplat_sdpa_f32_avx512_exact_q8t512(const float* q, const float* k, const float* v,
                                            const float* key_bias_or_null, float* out, int B,
                                            int H, int Lq, int Lk, int D, int has_key_bias,
                                            int key_bias_len, int threads);
/* replaces scripts/native_sdpa_avx512_exact_q8t512.c:334-351 (alias) */
int triposplat_sdpa_f32(const float* q, const float* k, const float* v, const float* bias,
                        float* out, int B, int H, int Lq, int Lk, int D, int has_key_bias,
                        int key_bias_len, int threads);
/* replaces scripts/native_sdpa_avx512_exact_q8.c:52 (same mathematics) */
int triposplat_sdpa_f32_avx512_exact_q8(const float* q, const float* k, const float* v,
                                        const float* bias, float* out, int B, int H, int Lq,
                                        int Lk, int D, int has_key_bias, int key_bias_len,
                                        int threads);
/* replaces scripts/native_sdpa_avx512_exact_q8t512_packed.c:3-158:
 * packed K/V [B, H, 64, Lkp] (Lkp >= Lk, Lkp % 16 == 0), output [B, Lq, H, 64] */
int triposplat_sdpa_f32_avx512_exact_q8t512_packed_blhd(
    const float* q, const float* packed_k, const float* packed_v, const float* key_bias_or_null,
    float* out_blhd, int B, int H, int Lq, int Lk, int D, int Lkp, int has_key_bias,
    int key_bias_len, int threads);
/* replaces scripts/native_sdpa_avx512_exact_q8t512_packed.c:160-162; returns 1 */
int triposplat_sdpa_packed_output_is_blhd(void);
/* No reference counterpart: per-(b,h) key bias rows bias_bh_stride elements apart
 * (0 = one shared [Lk] row, NULL = no bias) and BHLD (0) / BLHD (1) output. */
int triposplat_sdpa_f32_cuda_bias_bh(const float* q, const float* k, const float* v,
                                     const float* bias, long long bias_bh_stride, float* out,
                                     int B, int H, int Lq, int Lk, int out_blhd);
/* replace scripts/native_sdpa_avx512_exact_q8t512.c:64-70 (tile sizes used here) */
/* No reference counterpart: query-row sharding of one attention over a group of ranks
 * (one per GPU).  Rank r owns tokens [token_starts[r], token_starts[r+1]) of the L-token
 * sequence (interior starts multiples of 128).  Per attention each rank splits its own
 * tokens (RoPE + per-head RMSNorm, as triposplat_b200_qkv_rope_rmsnorm_sdpa_f32) into Q
 * planes of its rows and its key tiles of a K / V plane set, passes a peer barrier
 * (triposplat_b200_peer_barrier), pulls the other ranks' key tiles from their plane sets
 * over NVLink (CUDA IPC mappings, plain loads) and attends its rows to all L keys.  The
 * outputs are bit-identical to the unsharded fused call.  Plane buffers are caller-owned,
 * 256-byte aligned, sized by the two queries below. */
uint64_t triposplat_b200_attn_q_planes_bytes(int BH, int Lq);
uint64_t triposplat_b200_attn_kv_planes_bytes(int BH, int Lk);
/* qkv_rows [B, t1 - t0, 3, H, 64] (tokens [t0, t1)); frequencies [fb, L, H, 64]; t0 % 128 == 0,
 * t1 % 128 == 0 or t1 == L; -3 otherwise */
int triposplat_b200_qkv_split_rows_f32(const float* qkv_rows, const float* frequencies,
                                       const float* q_gamma, const float* k_gamma, int B, int L,
                                       int H, int t0, int t1, int frequency_batches, void* q_planes,
                                       void* kv_planes);
/* kv_planes_by_rank[r]: rank r's plane set as mapped here; token_starts: world + 1 entries */
int triposplat_b200_kv_planes_gather(const uint64_t* kv_planes_by_rank, const int* token_starts,
                                     int world, int rank, int BH, int L);
/* No reference counterpart: cached condition keys.  The condition tokens do not change
 * across sampler steps: their keys / values are split once per image into a K / V plane
 * set (per-head RMSNorm of the keys; kv [B, Lk, 2, H, 64]), and each step splits only its
 * queries (per-head RMSNorm, no rotation; q [B, Lq, H, 64]) before
 * triposplat_b200_attend_rows_f32.  Bit-identical to triposplat_b200_q_kv_rmsnorm_sdpa_f32. */
int triposplat_b200_kv_split_f32(const float* kv, const float* k_gamma, int B, int Lk, int H,
                                 void* kv_planes);
int triposplat_b200_q_split_f32(const float* q, const float* q_gamma, int B, int Lq, int H,
                                void* q_planes);

/* Lq query rows (q_planes) against L keys (a complete kv_planes); out [B, Lq, H, 64] */
int triposplat_b200_attend_rows_f32(const void* q_planes, const void* kv_planes, float* out_blhd,
                                    int B, int H, int Lq, int L);
/* The same, output written into a split buffer of [B * Lq, H * 64] (see
 * triposplat_b200_qkv_rope_rmsnorm_sdpa_split). */
int triposplat_b200_attend_rows_split(const void* q_planes, const void* kv_planes, int B, int H,
                                      int Lq, int L, void* out_split);

int triposplat_sdpa_key_tile(void);
int triposplat_sdpa_query_block(void);
/* replace scripts/native_sdpa_avx512_exact_q8t512.c:77-100; GPU timings are host enqueue
 * times (pack_ns = split kernels, compute_ns = attention kernel), allocate/free are 0 */
void triposplat_sdpa_q8t512_profile_reset(void);
int triposplat_sdpa_q8t512_profile_get(uint64_t* calls, uint64_t* allocate_ns, uint64_t* pack_ns,
                                       uint64_t* compute_ns, uint64_t* free_ns);
/* replace scripts/native_sdpa_avx512_exact_q8t512.c:51-62 (library-wide workspace) */
int triposplat_sdpa_q8t512_workspace_stats(uint64_t* allocations, uint64_t* capacity_bytes);
void triposplat_sdpa_q8t512_workspace_release(void);

/* ---------------------------------------------------------------- prologue / epilogue - */

/* replaces scripts/native_norm_rope_avx512.c:13-49 */
int triposplat_layernorm_f32_avx512(const float* input, const float* weight, const float* bias,
                                    float* output, int64_t rows, int cols, float eps,
                                    int has_affine, int threads);
/* replaces scripts/native_norm_rope_avx512.c:51-83 */
int triposplat_multihead_rmsnorm_f32_avx512(const float* input, const float* gamma, float* output,
                                            int64_t outer, int heads, int dim, float eps,
                                            int threads);
/* replaces scripts/native_norm_rope_avx512.c:85-110 */
int triposplat_rope_complex_f32_avx512(const float* input, const float* freqs_interleaved,
                                       float* output, int64_t vectors, int dim, int threads);
/* replaces scripts/native_gelu_avx512.c:44-68 */
int triposplat_gelu_tanh_f32_avx512(const float* input, float* output, int64_t count, int threads);
/* replaces scripts/native_silu_avx512_extra.c:28-45 */
int triposplat_silu_f32_avx512(const float* input, float* output, int64_t count, int threads);
/* replaces scripts/native_block_elementwise_avx512.c:9-22 */
int triposplat_modulate_inplace_f32_avx512(float* h, const float* scale, const float* shift,
                                           int batch, int rows, int cols, int threads);
/* replaces scripts/native_block_elementwise_avx512.c:24-35 */
int triposplat_gated_residual_inplace_f32_avx512(float* base, float* delta, const float* gate,
                                                 int batch, int rows, int cols, int threads);
/* replaces scripts/native_block_elementwise_avx512.c:37-46 */
int triposplat_add_inplace_f32_avx512(float* base, const float* delta, int64_t count, int threads);
/* replaces scripts/native_sampler_avx512.c:19-54 */
int triposplat_cfg_combine_inplace_f32_avx512(float* positive, const float* negative,
                                              const float* guidance, int batch,
                                              int64_t elements_per_batch, int threads);
/* replaces scripts/native_sampler_avx512.c:56-89 */
int triposplat_euler_update_inplace_f32_avx512(float* sample, const float* prediction,
                                               const float* dt, int batch,
                                               int64_t elements_per_batch, int threads);
/* scripts/native_sampler_avx512.c:91-130: Adams-Bashforth-2 step
 * x -= dt*((1+r)*v - r*v_prev), r = 0.5*dt/max(dt_prev, 1e-12), per batch entry. */
int triposplat_ab2_update_inplace_f32_avx512(float* sample, const float* prediction,
                                             const float* previous_prediction, const float* dt,
                                             const float* previous_dt, int batch,
                                             int64_t elements_per_batch, int threads);
/* No reference counterpart: CFG combine + Euler step in one kernel, bit-identical to the
 * two reference calls in sequence (positive is not overwritten). */
int triposplat_b200_cfg_euler_update_f32(float* sample, const float* positive,
                                         const float* negative, const float* guidance,
                                         const float* dt, int batch, int64_t elements_per_batch);
/* replaces scripts/native_qkv_postprocess_v2_avx512.c:45-105 */
int triposplat_qkv_rope_rmsnorm_pack_f32_avx512_v2(const float* qkv, const float* frequencies,
                                                   const float* q_gamma, const float* k_gamma,
                                                   float* q_bhld, float* packed_k,
                                                   float* packed_v, int B, int L, int H, int D,
                                                   int L_padded, int frequency_batches,
                                                   int threads);
/* replaces scripts/native_qkv_postprocess_avx512.c:23-116 (the first version: same
 * arguments and results as _v2) */
int triposplat_qkv_rope_rmsnorm_pack_f32_avx512(const float* qkv, const float* frequencies,
                                                const float* q_gamma, const float* k_gamma,
                                                float* q_bhld, float* packed_k, float* packed_v,
                                                int B, int L, int H, int D, int L_padded,
                                                int frequency_batches, int threads);
/* replace scripts/native_qkv_postprocess_avx512.c:118-120 (tokens per work tile) and
 * scripts/native_qkv_postprocess_v2_avx512.c:193-195 (returns 1: only the packed tail is
 * cleared).  The token tile is this build's: 64 tokens per CTA of the GPU kernel (the
 * reference's CPU kernel returns its 16-token tile), as the row-tile queries report the
 * GPU tiles; no caller derives a layout from it. */
int triposplat_qkv_postprocess_token_tile(void);
int triposplat_qkv_postprocess_v2_tail_only_clear(void);
/* replaces scripts/native_qkv_postprocess_v2_avx512.c:107-191 (selected_indices is a
 * device pointer; it is copied back once to validate it as the reference does) */
int triposplat_q_kv_selected_rope_rmsnorm_pack_f32_avx512_v2(
    const float* q, const float* kv, const float* frequencies, const int64_t* selected_indices,
    const float* q_gamma, const float* k_gamma, float* q_bhld, float* packed_k, float* packed_v,
    int B, int Lq, int Lk, int H, int D, int Lk_padded, int frequency_batches, int threads);
/* replaces scripts/native_embeddings_avx512.c:97-125: out[b] = [cos(t_b f) | sin(t_b f) | 0] */
int triposplat_timestep_embedding_f32_avx512(const float* timesteps, const float* frequencies,
                                             float* output, int batch, int half_dim,
                                             int output_dim, int threads);
/* scripts/native_embeddings_avx512.c:58-95: per row and axis [sin | cos] of x*f(*2)*pi over
 * frequency_dim frequencies, zero padding to channels; -1 null, -2 bad sizes. */
int triposplat_pcd_position_embedding_f32_avx512(const float* positions, const float* frequencies,
                                                 float* output, int64_t rows, int input_dims,
                                                 int frequency_dim, int channels, int double_pi,
                                                 int threads);
/* scripts/native_repo_avx512.c:69-83: lhs *= rhs; -1 null, -2 elements <= 0. */
int triposplat_mul_inplace_f32_avx512(float* lhs, const float* rhs, int64_t elements, int threads);
/* scripts/native_repo_avx512.c:85-129: RePo phasors, interleaved complex (cos, sin) of
 * (x*tanh_f + x*residual_f)*pi per vector and axis; -1 delta/output null, -2 a frequency
 * array null, -3 bad sizes. */
int triposplat_repo_phasor_f32_avx512(const float* delta, const float* freq_tanh_0,
                                      const float* freq_residual_0, int freq_dim_0,
                                      const float* freq_tanh_1, const float* freq_residual_1,
                                      int freq_dim_1, const float* freq_tanh_2,
                                      const float* freq_residual_2, int freq_dim_2,
                                      float* output_interleaved, int64_t vectors, int threads);
/* No reference counterpart: the selected-query post-process without RoPE or an index list
 * (cross-attention: condition tokens carry no position).  q [B,Lq,H,64], kv [B,Lk,2,H,64]
 * -> q_bhld [B,H,Lq,64], packed k/v [B,H,64,Lk_padded]; k and q get 8/max(||x||,1e-12)*gamma. */
int triposplat_b200_q_kv_rmsnorm_pack_f32(const float* q, const float* kv, const float* q_gamma,
                                          const float* k_gamma, float* q_bhld, float* packed_k,
                                          float* packed_v, int B, int Lq, int Lk, int H,
                                          int Lk_padded);

/* No reference counterpart: triposplat_qkv_rope_rmsnorm_pack_f32_avx512_v2 followed by
 * triposplat_sdpa_f32_avx512_exact_q8t512_packed_blhd in one call.  qkv [B,L,3,H,64],
 * frequencies [frequency_batches, L, H, 64] (interleaved cos/sin) -> out_blhd [B,L,H,64];
 * q / k / v go straight to the attention's split format (same results bit for bit as the
 * two calls).  D must be 64. */
int triposplat_b200_qkv_rope_rmsnorm_sdpa_f32(const float* qkv, const float* frequencies,
                                              const float* q_gamma, const float* k_gamma,
                                              float* out_blhd, int B, int L, int H, int D,
                                              int frequency_batches);
/* No reference counterpart: triposplat_b200_q_kv_rmsnorm_pack_f32 followed by the packed
 * SDPA in one call (cross-attention).  q [B,Lq,H,64], kv [B,Lk,2,H,64] -> out_blhd [B,Lq,H,64]. */
int triposplat_b200_q_kv_rmsnorm_sdpa_f32(const float* q, const float* kv, const float* q_gamma,
                                          const float* k_gamma, float* out_blhd, int B, int Lq,
                                          int Lk, int H);
/* No reference counterpart: the two entries above (D = 64) with the output written into
 * out_split, a split buffer (triposplat_b200_split_bytes(B * Lq, H * 64) bytes, 256-byte
 * aligned) of the [B * Lq, H * 64] output: the out-projection GEMM's input without an
 * fp32 round trip.  Row scale 2^-s fixed per batch from the largest V value (every
 * |O| * 2^s < 2^15); the planes equal the split of the fp32 output under those scales. */
int triposplat_b200_qkv_rope_rmsnorm_sdpa_split(const float* qkv, const float* frequencies,
                                                const float* q_gamma, const float* k_gamma, int B,
                                                int L, int H, int frequency_batches,
                                                void* out_split);
int triposplat_b200_q_kv_rmsnorm_sdpa_split(const float* q, const float* kv, const float* q_gamma,
                                            const float* k_gamma, int B, int Lq, int Lk, int H,
                                            void* out_split);

/* ---- Tensor-parallel reduction over NVLink peer memory (no reference counterpart) ----
 * ipc_alloc: cudaMalloc'd, zeroed buffer plus its 64-byte CUDA IPC handle; ipc_open maps a
 * handle of another process of the node; ipc_close / ipc_free release them.
 * peer_barrier: one-warp barrier of `world` ranks through their flag arrays (flag_ptrs[r] =
 * rank r's array of `world` uint32 as mapped here; counter = this rank's epoch word);
 * waits are bounded (2 s) and report through triposplat_b200_status().
 * peer_reduce_residual_f32: x += gate[row / rows_per_batch] * sum_r part_r (mode 2) or
 * x += sum_r part_r (mode 3), partials read from every rank's memory and summed in rank
 * order; cols % 4 == 0, 16-byte aligned pointers. */
int triposplat_b200_ipc_alloc(uint64_t bytes, void** dev_ptr, uint8_t* handle_out);
int triposplat_b200_ipc_free(void* dev_ptr);
int triposplat_b200_ipc_open(const uint8_t* handle, void** dev_ptr);
int triposplat_b200_ipc_close(void* dev_ptr);
int triposplat_b200_peer_barrier(const uint64_t* flag_ptrs, int rank, int world, uint32_t* counter);
int triposplat_b200_peer_reduce_residual_f32(const uint64_t* part_ptrs, int world, float* x,
                                             int64_t rows, int cols, int mode, const float* gate,
                                             int gate_ld, int64_t rows_per_batch);

#ifdef __cplusplus
}
#endif

#endif /* TRIPOSPLAT_B200_H */
