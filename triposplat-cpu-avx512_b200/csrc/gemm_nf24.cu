// NF24 int16 dequant GEMM for sm_100a:  Y[M, count] = X[M, K] . W[:, start:start+count] + b
//
// Weight semantics (reference scripts/gemm_nf24_i16_avx512.c:26-33):
//   W[k, n] = scale[n] * (256 * q01[k, n] + q2[k, n]),   q01 int16 [K, N], q2 int8 [K, N]
//
// Design.
//  * X (fp32) is split by `nf24_split_rows` (or a producer such as the fused LayerNorm)
//    into two exact-sum fp16 planes X' = hi + lo after an exact per-row power-of-two
//    pre-scale (undone in the epilogue), so fp16's range never clips and hi + lo carries
//    ~22 significant bits.
//  * W/256 = q01 + q2/256 is first written as two exact fp16 values (any |q01| <= 1023;
//    the packer emits |q01| <= 636):
//        A1 = 2*floor(q01/2)          (even integer)
//        A2 = (q01 & 1) + q2/256      (multiple of 1/256 in [-0.5, 1.5))
//    built from the raw codes with integer/bit operations and one HFMA2 each (magic-
//    exponent construction), then renormalised by Fast2Sum (Dekker 1971) in fp16 into
//        S = fp16_rn(W/256),  T = W/256 - S  (exact, |T| <= 2^-11 |S|),
//    in registers, and written straight into tensor memory.
//  * The tcgen05 MMA computes the TRANSPOSED product D[n, m] = sum_k A[n, k] * X'[m, k]
//    with A (weights) read from TMEM and X' (hi or lo plane, TMA-loaded with 128-B
//    swizzle) from shared memory:  3 MMAs per k-step (S.hi, S.lo, T.hi).  The omitted
//    T.lo term is at most 2^-11 * 2^-11 = 2^-22 of |x w| per product: the same order as
//    the hi + lo representation error of X itself (~2^-22), well under the reference's
//    fp32 accumulation error over K.
//  * Accuracy: the tensor core's fp32 accumulation truncates, so an error that grows
//    linearly with the number of accumulation steps builds up in a long-lived accumulator
//    (measured: rmse 1.8e-5 relative at K = 4096, 16x the fp32 reference).  Each k-block
//    (64 k; NK_KPP of them for the k-contiguous layout) is therefore accumulated into a
//    FRESH TMEM partial (double-buffered) and promoted into round-to-nearest fp32 running
//    sums held in the epilogue warps' registers, which keeps the error at the level of a
//    64- (64 * NK_KPP-) long dot product.
//    Epilogue: y = sum * rowscale[m] * 256*scale[n] + bias[n], then one of: store,
//    GELU(tanh) + store, gated residual out += gate[b] * y, residual out += y, or
//    GELU(tanh) written straight into the next GEMM's split format (fp16 hi / lo planes
//    under a per-row power-of-two pre-scale fixed beforehand from a bound on the row).
//
// Warp roles (448 threads, one CTA per SM):
//   warp 0       TMA producer (codes and X planes)
//   warp 1       TMEM allocator + single-thread MMA issuer
//   warps 2..5   weight decoders (raw codes smem -> registers -> TMEM), k pairs 0..19 of
//                every 64-k block
//   warps 6..13  promotion + epilogue; two warps per TMEM lane quarter, 96 tokens each.
//                They also decode k pairs 20..25 / 26..31 of block kb+2 as soon as the
//                MMAs of block kb retire (their promotion work leaves them idle most of a
//                k-block; the dedicated decoders alone could not keep up with the MMAs)
//
// Columns whose layout TMA cannot address (N % 16 != 0, unaligned pointers) go to
// `nf24_gemm_simt`, which reproduces the reference's scalar tail kernel
// (scripts/gemm_nf24_i16_avx512_tail.c:32-47) operation for operation.
#include <cuda_fp16.h>

#include <atomic>
#include <mutex>

#include "common.cuh"
#include "runtime.h"

namespace tsb {
namespace gemm {

constexpr int BN = 128;  // weight columns per CTA = TMEM lanes = MMA M
constexpr int BM = 192;  // tokens per CTA = MMA N
constexpr int BK = 64;   // k per stage: one 128-B swizzle row of fp16
constexpr int XS = 3;    // X stages (hi + lo planes)
constexpr int CS = 2;    // raw-code stages
constexpr int AS = 2;    // decoded-weight stages in TMEM
constexpr int X_PLANE = BM * BK * 2;       // 24 KB
constexpr int X_STAGE = 2 * X_PLANE;       // 48 KB
constexpr int C16_BYTES = BK * BN * 2;     // 16 KB
constexpr int C8_BYTES = BK * BN;          //  8 KB
constexpr int C_STAGE = C16_BYTES + C8_BYTES;
constexpr int NUM_EPI_WARPS = 8;
constexpr int EPI_COLS = BM / 2;  // tokens per epilogue warp
constexpr int NUM_THREADS = 32 * (6 + NUM_EPI_WARPS);
constexpr int DEC_ARRIVALS = 4 + NUM_EPI_WARPS;  // warps decoding a share of every stage
// k pairs (of 32 per 64-k block) decoded by each of warps 2..5 and by each epilogue warp,
// balanced so the epilogue warps' promotion plus decode share fits in one k-block
constexpr int DEC_PAIRS = 20;
constexpr int EPI_PAIRS = 6;
static_assert(DEC_PAIRS + 2 * EPI_PAIRS == BK / 2, "decode shares cover the block");
// the same split for the k-contiguous code layout, whose decode is cheaper
// (measured: the decoder warps alone keep up, so the epilogue warps only promote)
constexpr int NK_DEC_PAIRS = 32;
constexpr int NK_EPI_PAIRS = (BK / 2 - NK_DEC_PAIRS) / 2;
static_assert(NK_DEC_PAIRS % 2 == 0 && NK_EPI_PAIRS % 2 == 0 &&
              NK_DEC_PAIRS + 2 * NK_EPI_PAIRS == BK / 2, "k-contiguous decode shares");
constexpr int NK_DEC_ARRIVALS = 4 + (NK_EPI_PAIRS ? NUM_EPI_WARPS : 0);
// k-blocks accumulated in one TMEM partial before it is promoted, for the k-contiguous
// layout of the model path.  Two halve the promotions and their barrier round trips per k;
// the partial's truncation error grows with its length (about sqrt(2) over one block's,
// still inside fp32 semantics).  The reference layout behind the drop-in entry points keeps
// one block per partial (its accuracy against the reference kernel is unchanged).  The
// epilogue warps' decode shares are paced by each block's MMA completion (a_empty), not by
// the promotions.
#ifndef TSB_GEMM_KPP
#define TSB_GEMM_KPP 2
#endif
constexpr int NK_KPP = TSB_GEMM_KPP;
static_assert(NK_KPP == 1 || NK_KPP == 2 || NK_KPP == 4, "k-blocks per partial");
constexpr int TMEM_COLS = 512;
constexpr int ACC_COL = 0;        // 2 partial buffers x BM fp32 columns
constexpr int A_COL = 2 * BM;     // AS stages x (32 cols A1 + 32 cols A2)
static_assert(A_COL + AS * 64 <= TMEM_COLS, "TMEM budget");
// Outputs leave asynchronously: each epilogue warp writes 12-row x 32-column chunks into a
// double-buffered shared-memory slot and one lane hands them to the TMA (store, or
// reduce-add for the residual modes), so the tile-end store overlaps the next tile's
// k-blocks.  Two code stages leave room for the slots.
constexpr int OUT_ROWS = 12;
constexpr int OUT_CHUNK = OUT_ROWS * 32;                            // floats
constexpr int OUT_STAGE_BYTES = NUM_EPI_WARPS * 2 * OUT_CHUNK * 4;  // 24 KB
static_assert(EPI_COLS % OUT_ROWS == 0, "whole chunks per epilogue warp");
constexpr int NUM_BARS = 2 * XS + 2 * CS + 2 * AS + 5;
constexpr int SMEM_BYTES = 1024 /*align slack*/ + XS * X_STAGE + CS * C_STAGE + OUT_STAGE_BYTES +
                           2 * NUM_EPI_WARPS * EPI_COLS * 4 + NUM_BARS * 8 + 16;
static_assert(SMEM_BYTES <= 232448, "shared memory per block");


enum Epilogue : int { kStore = 0, kGelu = 1, kGatedResidual = 2, kResidual = 3, kGeluSplit = 4 };

struct Params {
  const float* rscale;  // [Mp] inverse row pre-scale of the split X
  const float* scale;   // [N]
  const float* bias;    // [N]
  float* out;           // [M, stride_out]; read-modify-write for the residual modes
  int M, K, N, start, count, stride_out;
  int mode;             // Epilogue
  const float* gate;    // kGatedResidual: gate[(m / rows_per_batch) * gate_ld + n]
  int gate_ld, rows_per_batch;
  int* status;
  const float* next_rs;  // kGeluSplit: [Mp] inverse pre-scales 2^-s of the split being written
};

// GELU(tanh) = 0.5 x (1 + tanh(u)), u = sqrt(2/pi) (x + 0.044715 x^3), evaluated through the
// identity 0.5 (1 + tanh(u)) = 1 / (1 + e^(-2u)) as x / (1 + 2^t), t = -2 u log2(e): one ex2
// and one fast division instead of a full tanhf, with no cancellation for either sign of x
// (relative error a few ulp; 2^t overflowing for x below about -9.7 gives -0 where the
// exact value is below 1e-36 in magnitude).  The epilogue warps evaluate it for every
// output of a GELU GEMM while they also promote the next tile's partial sums.
constexpr float kGeluT = -2.0f * 0.7978845608028654f * 1.4426950408889634f;
__device__ __forceinline__ float ex2_approx(float t) {
  float e;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(t));
  return e;
}
__device__ __forceinline__ float rcp_approx(float d) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(d));
  return r;
}
__device__ __forceinline__ float gelu_tanh(float x) {
  const float t = kGeluT * fmaf(0.044715f * x, x * x, x);
  return x * rcp_approx(1.0f + ex2_approx(t));
}
// The same for two values at once (packed fp32x2 multiplies / adds, each lane rounded
// exactly as gelu_tanh rounds it, so both give the same bits).
__device__ __forceinline__ float2 gelu_tanh2(float2 x) {
  uint64_t xv, c, xx, in, t;
  asm("mov.b64 %0, {%1, %2};" : "=l"(xv) : "f"(x.x), "f"(x.y));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(c) : "l"(xv), "l"(0x3d3727133d372713ull));   // 0.044715 x
  asm("mul.rn.f32x2 %0, %1, %1;" : "=l"(xx) : "l"(xv));                              // x * x
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(in) : "l"(c), "l"(xx), "l"(xv));
  const uint64_t kt = (uint64_t)__float_as_uint(kGeluT) | ((uint64_t)__float_as_uint(kGeluT) << 32);
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(t) : "l"(in), "l"(kt));
  float t0, t1;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(t0), "=f"(t1) : "l"(t));
  return make_float2(x.x * rcp_approx(1.0f + ex2_approx(t0)), x.y * rcp_approx(1.0f + ex2_approx(t1)));
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// Round-to-nearest fp16x2 add / subtract (explicit .rn: never contracted with a multiply)
__device__ __forceinline__ uint32_t hadd2_rn(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t hsub2_rn(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Decode NP k pairs (k = 2*pair0 .. 2*(pair0+NP)-1) of weight column nl from a raw-code
// stage into the fp16 operands S / T (S + T = W/256 exactly) and store them to this
// warp's TMEM lanes (S at column pair0, T at column 32 + pair0 of the stage).
template <int NP>
__device__ __forceinline__ void decode_pairs(const uint8_t* cstage, int nl, int pair0, uint32_t ta) {
  // explicit shared-memory loads, all issued before the arithmetic (the stage pointer is
  // generic after the kernel's alignment arithmetic, and generic loads are slower)
  const uint32_t a16 = smem_u32(cstage) + (2 * pair0 * BN + nl) * 2;
  const uint32_t a8 = smem_u32(cstage) + C16_BYTES + 2 * pair0 * BN + nl;
  uint32_t v[2 * NP], bb[2 * NP];
#pragma unroll
  for (int i = 0; i < 2 * NP; ++i) {
    asm volatile("ld.shared.u16 %0, [%1];" : "=r"(v[i]) : "r"(a16 + i * BN * 2));
    asm volatile("ld.shared.u8 %0, [%1];" : "=r"(bb[i]) : "r"(a8 + i * BN));
  }
  const __half2 two = __floats2half2_rn(2.0f, 2.0f);
  const __half2 m3072 = __floats2half2_rn(-3072.0f, -3072.0f);
  const __half2 inv256 = __floats2half2_rn(1.0f / 256.0f, 1.0f / 256.0f);
  const __half2 m4p5 = __floats2half2_rn(-4.5f, -4.5f);
  uint32_t r1[NP], r2[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const uint32_t pq = __byte_perm(v[2 * i], v[2 * i + 1], 0x5410);
    const uint32_t pc = __byte_perm(bb[2 * i], bb[2 * i + 1], 0x5410);
    const uint32_t f1 = ((pq >> 1) & 0x03FF03FFu) ^ 0x66006600u;
    const uint32_t f2 = (((pq << 8) & 0x01000100u) | pc) ^ 0x64806480u;
    const uint32_t a1 = h2_bits(__hfma2(bits_h2(f1), two, m3072));
    const uint32_t a2 = h2_bits(__hfma2(bits_h2(f2), inv256, m4p5));
    // Fast2Sum in fp16 (valid: a1 == 0 or |a1| >= 2 > |a2|): S = fp16_rn(W/256) and the
    // exact remainder T = W/256 - S, |T| <= 2^-11 |S|
    r1[i] = hadd2_rn(a1, a2);
    r2[i] = hsub2_rn(a2, hsub2_rn(r1[i], a1));
  }
  // NP columns of A1 and of A2 (NP = 20 or 6: x16 + x4 or x4 + x2 stores)
  static_assert(NP == 20 || NP == 6, "decode share");
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const uint32_t* r = half ? r2 : r1;
    const uint32_t t = ta + half * 32 + pair0;
    if constexpr (NP == 20) {
      tmem_st16(t, *reinterpret_cast<const uint32_t(*)[16]>(r));
      tmem_st4(t + 16, r[16], r[17], r[18], r[19]);
    } else {
      tmem_st4(t, r[0], r[1], r[2], r[3]);
      tmem_st2(t + 4, r[4], r[5]);
    }
  }
}

// Shared-memory loads of 1, 2 or 4 consecutive 32-bit words.
template <int W>
__device__ __forceinline__ void lds_words(uint32_t addr, uint32_t* d) {
  if constexpr (W == 4)
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3]) : "r"(addr));
  else if constexpr (W == 2)
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(d[0]), "=r"(d[1]) : "r"(addr));
  else
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(d[0]) : "r"(addr));
}

// Words [W0, W0 + NW) of a swizzled row (row_addr: the row's first byte; 16-byte chunk c
// of the row lives at chunk c ^ sw), loaded with the widest aligned accesses (unrolled at
// compile time, so d stays in registers).
template <int W0, int NW, int I = 0>
__device__ __forceinline__ void lds_row_words(uint32_t row_addr, uint32_t sw, uint32_t* d) {
  if constexpr (I < NW) {
    constexpr int byte = 4 * (W0 + I);
    constexpr int left = NW - I;
    constexpr int in_chunk = (16 - (byte & 15)) / 4;
    constexpr int W = ((byte & 15) == 0 && left >= 4) ? 4
                      : (((byte & 7) == 0 && left >= 2 && in_chunk >= 2) ? 2 : 1);
    const uint32_t addr = row_addr + (((uint32_t)(byte >> 4) ^ sw) << 4) + (byte & 15);
    lds_words<W>(addr, d + I);
    lds_row_words<W0, NW, I + W>(row_addr, sw, d);
  }
}

// Words r[0, NW) to consecutive TMEM columns from t (this warp's lanes), in 16/8/4/2-wide
// stores.
template <int NW, int I = 0>
__device__ __forceinline__ void tmem_st_run(uint32_t t, const uint32_t* r) {
  if constexpr (NW - I >= 16) {
    tmem_st16(t + I, *reinterpret_cast<const uint32_t(*)[16]>(r + I));
    tmem_st_run<NW, I + 16>(t, r);
  } else if constexpr (NW - I >= 8) {
    tmem_st8(t + I, *reinterpret_cast<const uint32_t(*)[8]>(r + I));
    tmem_st_run<NW, I + 8>(t, r);
  } else if constexpr (NW - I >= 4) {
    tmem_st4(t + I, r[I], r[I + 1], r[I + 2], r[I + 3]);
    tmem_st_run<NW, I + 4>(t, r);
  } else if constexpr (NW - I >= 2) {
    tmem_st2(t + I, r[I], r[I + 1]);
    tmem_st_run<NW, I + 2>(t, r);
  }
}

// decode_pairs for the k-contiguous code layout ([N][K] planes, see nf24_codes_to_nk):
// the stage holds row nl of the q01 tile as 128 B (64 k, TMA 128-B swizzle: chunk c at
// c ^ (nl & 7)) and of the q2 tile as 64 B (64-B swizzle: chunk c at c ^ ((nl >> 1) & 3)),
// so a thread reads its own column with 16-byte loads and a warp's load instruction covers
// whole 128-byte bank rows.  Pairs [P0, P0 + NP) of the 64-k block.
template <int P0, int NP>
__device__ __forceinline__ void decode_pairs_nk_regs(const uint8_t* cstage, int nl, uint32_t (&r1)[NP],
                                                     uint32_t (&r2)[NP]) {
  static_assert(P0 % 2 == 0 && NP % 2 == 0, "q2 words hold two k pairs");
  const uint32_t row16 = smem_u32(cstage) + nl * 128;
  const uint32_t row8 = smem_u32(cstage) + C16_BYTES + nl * 64;
  uint32_t pq[NP], pb[NP / 2];
  lds_row_words<P0, NP>(row16, nl & 7, pq);            // q01: one word per k pair
  lds_row_words<P0 / 2, NP / 2>(row8, (nl >> 1) & 3, pb);  // q2: one word per 4 k
  const __half2 two = __floats2half2_rn(2.0f, 2.0f);
  const __half2 m3072 = __floats2half2_rn(-3072.0f, -3072.0f);
  const __half2 inv256 = __floats2half2_rn(1.0f / 256.0f, 1.0f / 256.0f);
  const __half2 m4p5 = __floats2half2_rn(-4.5f, -4.5f);
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const uint32_t pc = __byte_perm(pb[i >> 1], 0u, (i & 1) ? 0x4342 : 0x4140);
    const uint32_t f1 = ((pq[i] >> 1) & 0x03FF03FFu) ^ 0x66006600u;
    const uint32_t f2 = (((pq[i] << 8) & 0x01000100u) | pc) ^ 0x64806480u;
    const uint32_t a1 = h2_bits(__hfma2(bits_h2(f1), two, m3072));
    const uint32_t a2 = h2_bits(__hfma2(bits_h2(f2), inv256, m4p5));
    r1[i] = hadd2_rn(a1, a2);
    r2[i] = hsub2_rn(a2, hsub2_rn(r1[i], a1));
  }
}

template <int P0, int NP>
__device__ __forceinline__ void decode_pairs_nk(const uint8_t* cstage, int nl, uint32_t ta) {
  uint32_t r1[NP], r2[NP];
  decode_pairs_nk_regs<P0, NP>(cstage, nl, r1, r2);
  tmem_st_run<NP>(ta + P0, r1);
  tmem_st_run<NP>(ta + 32 + P0, r2);
}

// 14 warps put four warps on some SM sub-partitions (16K registers each): 128 registers
// per thread is the most that can launch.
template <int MODE, bool NK, int KPP>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    nf24_gemm_tc(const __grid_constant__ CUtensorMap tm_xhi,
                 const __grid_constant__ CUtensorMap tm_xlo,
                 const __grid_constant__ CUtensorMap tm_c16,
                 const __grid_constant__ CUtensorMap tm_c8,
                 const __grid_constant__ CUtensorMap tm_out, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* xs = smem;
  constexpr int kCS = CS;  // code stages
  uint8_t* cs = xs + XS * X_STAGE;
  float* ostage = reinterpret_cast<float*>(cs + kCS * C_STAGE);  // output staging slots
  // [8 epilogue warps][96] row scales, then (kGeluSplit) [8][96] output pre-scales
  float* rs_s = reinterpret_cast<float*>(cs + kCS * C_STAGE + OUT_STAGE_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(rs_s + 2 * NUM_EPI_WARPS * EPI_COLS);
  uint64_t* x_full = bars;
  uint64_t* x_empty = x_full + XS;
  uint64_t* c_full = x_empty + XS;
  uint64_t* c_empty = c_full + CS;
  uint64_t* a_full = c_empty + CS;
  uint64_t* a_empty = a_full + AS;
  uint64_t* acc_full = a_empty + AS;  // [2]
  uint64_t* acc_free = acc_full + 2;  // [2]
  uint64_t* mma_done = acc_free + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  // persistent CTAs: tile t = blockIdx.x + i * gridDim.x, weight tiles fastest (CTAs
  // running together share the token tile); every role walks the same tile sequence, and
  // pipeline stages / barrier phases run on one k-block counter g across tiles
  const int kblocks = (p.K + BK - 1) / BK;
  const int n_tiles = (p.count + BN - 1) / BN;
  const int num_tiles = n_tiles * ((p.M + BM - 1) / BM);
  const int my_tiles = blockIdx.x < num_tiles ? (num_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int total_g = my_tiles * kblocks;
  // partials: groups of KPP k-blocks per tile, numbered G across tiles (buffer G & 1)
  static_assert(KPP == 1 || NK, "the [K][N] layout keeps one k-block per partial");
  const int groups = (kblocks + KPP - 1) / KPP;

  if (threadIdx.x == 0) {
    for (int i = 0; i < XS; ++i) { mbar_init(&x_full[i], 1); mbar_init(&x_empty[i], 1); }
    constexpr int arrivals = NK ? NK_DEC_ARRIVALS : DEC_ARRIVALS;
    for (int i = 0; i < kCS; ++i) { mbar_init(&c_full[i], 1); mbar_init(&c_empty[i], arrivals); }
    for (int i = 0; i < AS; ++i) { mbar_init(&a_full[i], arrivals); mbar_init(&a_empty[i], 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(&acc_full[i], 1); mbar_init(&acc_free[i], NUM_EPI_WARPS); }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_xhi);
    tma_prefetch_desc(&tm_xlo);
    tma_prefetch_desc(&tm_c16);
    tma_prefetch_desc(&tm_c8);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (elect_one()) {
      int last_c[kCS], last_x[XS];
      for (int i = 0; i < kCS; ++i) last_c[i] = -1;
      for (int i = 0; i < XS; ++i) last_x[i] = -1;
      bool ok = true;
      for (int g = 0; g < total_g && ok; ++g) {
        const int kb = g % kblocks, t = blockIdx.x + (g / kblocks) * gridDim.x;
        const int n0 = (t % n_tiles) * BN, m0 = (t / n_tiles) * BM;
        const int c = g % kCS, x = g % XS;
        if (g >= kCS &&
            !mbar_wait(&c_empty[c], ((g / kCS) & 1) ^ 1, p.status, kDevTimeoutProducer, abort_flag)) {
          ok = false;
          break;
        }
        uint8_t* cdst = cs + c * C_STAGE;
        mbar_arrive_expect_tx(&c_full[c], C_STAGE);
        if constexpr (NK) {  // [N][K] planes: x = k
          tma_load_2d(cdst, &tm_c16, &c_full[c], kb * BK, p.start + n0);
          tma_load_2d(cdst + C16_BYTES, &tm_c8, &c_full[c], kb * BK, p.start + n0);
        } else {             // [K][N] planes: x = n
          tma_load_2d(cdst, &tm_c16, &c_full[c], p.start + n0, kb * BK);
          tma_load_2d(cdst + C16_BYTES, &tm_c8, &c_full[c], p.start + n0, kb * BK);
        }
        last_c[c] = g;
        if (g >= XS &&
            !mbar_wait(&x_empty[x], ((g / XS) & 1) ^ 1, p.status, kDevTimeoutProducer, abort_flag)) {
          ok = false;
          break;
        }
        uint8_t* xdst = xs + x * X_STAGE;
        mbar_arrive_expect_tx(&x_full[x], X_STAGE);
        tma_load_2d(xdst, &tm_xhi, &x_full[x], kb * BK, m0);
        tma_load_2d(xdst + X_PLANE, &tm_xlo, &x_full[x], kb * BK, m0);
        last_x[x] = g;
      }
      if (*abort_flag) {
        // never leave the CTA while a bulk copy may still write its shared memory
        for (int i = 0; i < kCS; ++i)
          if (last_c[i] >= 0) mbar_wait(&c_full[i], (last_c[i] / kCS) & 1, p.status, kDevTimeoutProducer, nullptr);
        for (int i = 0; i < XS; ++i)
          if (last_x[i] >= 0) mbar_wait(&x_full[i], (last_x[i] / XS) & 1, p.status, kDevTimeoutProducer, nullptr);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (elect_one()) {
      constexpr uint32_t idesc = idesc_f16_f32(BN, BM);
      bool ok = true;
      for (int g = 0; g < total_g && ok; ++g) {
        const int kb = g % kblocks;
        const int G = (g / kblocks) * groups + kb / KPP;
        const bool first = kb % KPP == 0, last = kb % KPP == KPP - 1 || kb == kblocks - 1;
        const int x = g % XS, a = g % AS, b = G & 1;
        ok = mbar_wait(&x_full[x], (g / XS) & 1, p.status, kDevTimeoutMma, abort_flag) &&
             mbar_wait(&a_full[a], (g / AS) & 1, p.status, kDevTimeoutMma, abort_flag) &&
             (!first || G < 2 ||
              mbar_wait(&acc_free[b], ((G >> 1) & 1) ^ 1, p.status, kDevTimeoutMma, abort_flag));
        if (!ok) break;
        tc_fence_after();
        const uint32_t hi = smem_u32(xs + x * X_STAGE);
        const uint32_t lo = hi + X_PLANE;
        const uint32_t a_col = tmem + A_COL + a * 64;
        const uint32_t d = tmem + ACC_COL + b * BM;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint64_t dhi = sw128_kmajor_desc(hi + kk * 32);
          const uint64_t dlo = sw128_kmajor_desc(lo + kk * 32);
          const uint32_t a1 = a_col + kk * 8;
          const uint32_t a2 = a_col + 32 + kk * 8;
          // S.hi + S.lo + T.hi; the dropped T.lo is below 2^-22 of |x w| per product
          mma_f16_ts(d, a1, dhi, idesc, !first || kk != 0);  // fresh partial per group
          mma_f16_ts(d, a1, dlo, idesc, 1);
          mma_f16_ts(d, a2, dhi, idesc, 1);
        }
        mma_commit(&x_empty[x]);
        mma_commit(&a_empty[a]);
        if (last) mma_commit(&acc_full[b]);
      }
      // Retire every issued MMA before teardown frees TMEM (also on the error path).
      mma_commit(mma_done);
      mbar_wait(mma_done, 0, p.status, kDevTimeoutMma, nullptr);
    }
  } else if (warp < 6) {
    // ---------------- weight decoders ----------------
    const uint32_t sub = warp & 3;  // TMEM lane quarter this warp may touch
    const int nl = sub * 32 + lane;
    const uint32_t lane_base = (sub * 32) << 16;
    for (int g = 0; g < total_g; ++g) {
      const int c = g % kCS, a = g % AS;
      bool ok = mbar_wait(&c_full[c], (g / kCS) & 1, p.status, kDevTimeoutConsumer, abort_flag);
      if constexpr (NK) {
        // decode into registers as soon as the codes land; only the TMEM store waits for
        // the stage's previous MMAs, so the decode stays off the MMA's critical path
        if (!__all_sync(0xffffffffu, ok)) break;
        uint32_t r1[NK_DEC_PAIRS], r2[NK_DEC_PAIRS];
        decode_pairs_nk_regs<0, NK_DEC_PAIRS>(cs + c * C_STAGE, nl, r1, r2);
        __syncwarp();
        if (lane == 0) mbar_arrive(&c_empty[c]);
        if (g >= AS)
          ok = mbar_wait(&a_empty[a], ((g / AS) & 1) ^ 1, p.status, kDevTimeoutConsumer, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) break;
        tc_fence_after();
        const uint32_t ta = tmem + lane_base + A_COL + a * 64;
        tmem_st_run<NK_DEC_PAIRS>(ta, r1);
        tmem_st_run<NK_DEC_PAIRS>(ta + 32, r2);
      } else {
        if (ok && g >= AS)
          ok = mbar_wait(&a_empty[a], ((g / AS) & 1) ^ 1, p.status, kDevTimeoutConsumer, abort_flag);
        // the tcgen05 st below is warp-collective: leave the loop as a whole warp
        if (!__all_sync(0xffffffffu, ok)) break;
        tc_fence_after();
        decode_pairs<DEC_PAIRS>(cs + c * C_STAGE, nl, 0, tmem + lane_base + A_COL + a * 64);
        __syncwarp();
        if (lane == 0) mbar_arrive(&c_empty[c]);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[a]);
    }
  } else {
    // ---------------- promotion + epilogue ----------------
    const uint32_t sub = warp & 3;
    const int half = (warp - 6) >> 2;  // which 96-token half of the tile
    const int nl = sub * 32 + lane;
    const uint32_t lane_base = (sub * 32) << 16;
    const int pair0 = DEC_PAIRS + half * EPI_PAIRS;
    // this warp's decode share of k-block kbd into A stage kbd % AS (free: either never
    // used, or the MMAs of block kbd - AS retired, which acc_full of that block tells)
    auto decode_share = [&](int kbd) -> bool {
      if constexpr (NK && NK_EPI_PAIRS == 0) return true;  // the decoder warps do it all
      const int c = kbd % kCS;
      const bool got = mbar_wait(&c_full[c], (kbd / kCS) & 1, p.status, kDevTimeoutEpilogue, abort_flag);
      if (!__all_sync(0xffffffffu, got)) return false;
      const uint32_t ta = tmem + lane_base + A_COL + (kbd % AS) * 64;
      if constexpr (NK) {
        if constexpr (NK_EPI_PAIRS > 0) {
          if (half == 0)
            decode_pairs_nk<NK_DEC_PAIRS, NK_EPI_PAIRS>(cs + c * C_STAGE, nl, ta);
          else
            decode_pairs_nk<NK_DEC_PAIRS + NK_EPI_PAIRS, NK_EPI_PAIRS>(cs + c * C_STAGE, nl, ta);
        }
      } else {
        decode_pairs<EPI_PAIRS>(cs + c * C_STAGE, nl, pair0, ta);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&c_empty[c]);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[kbd % AS]);
      return true;
    };
    bool ok = true;
    for (int gd = 0; gd < AS && gd < total_g && ok; ++gd) ok = decode_share(gd);
    for (int i = 0; i < my_tiles && ok; ++i) {
    const int t = blockIdx.x + i * gridDim.x;
    const int n0 = (t % n_tiles) * BN, m0 = (t / n_tiles) * BM;
    // this tile's row pre-scales into the warp's private slice of shared memory (read
    // back at the store; the loads complete while the k-blocks run)
    float* rsw = rs_s + (warp - 6) * EPI_COLS;
    float* osw = rsw + NUM_EPI_WARPS * EPI_COLS;  // kGeluSplit
    __syncwarp();
    for (int j = lane; j < EPI_COLS; j += 32) {
      const int m = m0 + half * EPI_COLS + j;
      rsw[j] = m < p.M ? p.rscale[m] : 0.0f;
      // 2^s from the stored 2^-s: exponent field 127 + s = 254 - (127 - s), exact
      if constexpr (MODE == kGeluSplit)
        osw[j] = m < p.M ? __int_as_float((254 << 23) - __float_as_int(p.next_rs[m])) : 0.0f;
    }
    __syncwarp();
    float sum[EPI_COLS];
#pragma unroll
    for (int j = 0; j < EPI_COLS; ++j) sum[j] = 0.0f;
    for (int kg = 0; kg < groups && ok; ++kg) {
      const int G = i * groups + kg, b = G & 1;
      if constexpr (!(NK && NK_EPI_PAIRS == 0)) {
        // this warp's decode share of the blocks two ahead of the group's blocks, each as
        // soon as the MMAs of the block whose A stage it reuses retire (a_empty phase)
        const int g0 = i * kblocks + kg * KPP, g1 = min(g0 + KPP, (i + 1) * kblocks);
        for (int gg = g0; gg < g1 && ok; ++gg) {
          if (gg + AS >= total_g) break;
          ok = mbar_wait(&a_empty[gg % AS], (gg / AS) & 1, p.status, kDevTimeoutEpilogue, abort_flag);
          ok = __all_sync(0xffffffffu, ok);
          if (ok) {
            tc_fence_after();
            ok = decode_share(gg + AS);
          }
        }
        if (!ok) break;
      }
      ok = mbar_wait(&acc_full[b], (G >> 1) & 1, p.status, kDevTimeoutEpilogue, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      const uint32_t col = tmem + lane_base + ACC_COL + b * BM + half * EPI_COLS;
#pragma unroll
      for (int q = 0; q < EPI_COLS / 16; ++q) {
        uint32_t v[16];
        tmem_ld16(col + q * 16, v);
        tmem_wait_ld();
        reg_fence(v);
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
          float2 a = make_float2(sum[q * 16 + j], sum[q * 16 + j + 1]);
          asm("add.rn.f32x2 %0, %0, %1;" : "+l"(*reinterpret_cast<uint64_t*>(&a))
              : "l"((uint64_t)v[j] | ((uint64_t)v[j + 1] << 32)));
          sum[q * 16 + j] = a.x;
          sum[q * 16 + j + 1] = a.y;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_free[b]);
    }
    if (ok) {
        // asynchronous store: 12-row chunks through this warp's two shared-memory slots
        const int nw0 = n0 + sub * 32;  // this warp's first column (relative to start)
        const int nloc = n0 + nl;
        const bool col_ok = nloc < p.count;
        const int n = p.start + (col_ok ? nloc : 0);
        const float sc = col_ok ? p.scale[n] * 256.0f : 0.0f;
        const float bi = col_ok ? p.bias[n] : 0.0f;
        const int mbase = m0 + half * EPI_COLS;
#pragma unroll
        for (int j = 0; j < EPI_COLS; ++j) sum[j] *= rsw[j];
        float g0 = 1.0f, g1 = 1.0f;
        int jb = EPI_COLS;
        if constexpr (MODE == kGatedResidual) {
          const int b0 = mbase / p.rows_per_batch;
          jb = (b0 + 1) * p.rows_per_batch - mbase;
          g0 = col_ok ? p.gate[(int64_t)b0 * p.gate_ld + n] : 0.0f;
          g1 = (col_ok && jb < EPI_COLS && mbase + jb < p.M) ? p.gate[(int64_t)(b0 + 1) * p.gate_ld + n] : 0.0f;
        }
        float* wst = ostage + (warp - 6) * 2 * OUT_CHUNK;
        if (nw0 < p.count) {
#pragma unroll
          for (int c = 0; c < EPI_COLS / OUT_ROWS; ++c) {
            if (mbase + c * OUT_ROWS >= p.M) break;  // rows past M (warp-uniform)
            float* buf = wst + (c & 1) * OUT_CHUNK;
            // the slot's previous store (two chunks back, possibly of the previous tile)
            // has finished reading it
            if (lane == 0) bulk_wait_group_read<1>();
            __syncwarp();
            if constexpr (MODE == kGeluSplit) {
              // the slot as fp16 [2 planes][OUT_ROWS][32]: a = GELU(y) * 2^s, hi = rn(a),
              // lo = rn(a - hi) (the split kernels' arithmetic, with s fixed beforehand)
              __half* hb = reinterpret_cast<__half*>(buf);
#pragma unroll
              for (int j = 0; j < OUT_ROWS; j += 2) {  // two rows at a time (packed GELU)
                const int r = c * OUT_ROWS + j;
                const float2 g = gelu_tanh2(make_float2(fmaf(sum[r], sc, bi), fmaf(sum[r + 1], sc, bi)));
                const float2 s2 = *reinterpret_cast<const float2*>(&osw[r]);
                const float a0 = g.x * s2.x, a1 = g.y * s2.y;
                const __half2 h = __floats2half2_rn(a0, a1);
                const float2 hf = __half22float2(h);
                const __half2 l = __floats2half2_rn(a0 - hf.x, a1 - hf.y);
                hb[j * 32 + lane] = __low2half(h);
                hb[(j + 1) * 32 + lane] = __high2half(h);
                hb[OUT_ROWS * 32 + j * 32 + lane] = __low2half(l);
                hb[OUT_ROWS * 32 + (j + 1) * 32 + lane] = __high2half(l);
              }
            } else {
#pragma unroll
              for (int j = 0; j < OUT_ROWS; ++j) {
                const int r = c * OUT_ROWS + j;
                float v = fmaf(sum[r], sc, bi);
                if constexpr (MODE == kGelu) v = gelu_tanh(v);
                if constexpr (MODE == kGatedResidual) v *= (r < jb ? g0 : g1);
                buf[j * 32 + lane] = v;
              }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              if constexpr (MODE == kGeluSplit)
                tma_store_3d(&tm_out, buf, nw0, mbase + c * OUT_ROWS, 0);
              else if constexpr (MODE == kStore || MODE == kGelu)
                tma_store_2d(&tm_out, buf, nw0, mbase + c * OUT_ROWS);
              else
                tma_reduce_add_2d(&tm_out, buf, nw0, mbase + c * OUT_ROWS);
              bulk_commit_group();
            }
          }
        }
      }
    }  // tile loop
    // every asynchronous store complete before the CTA's shared memory goes away
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// X fp32 [M, K] (row stride stride_x) -> hi, lo fp16 [M, Kp] and inverse row scales rs [Mp].
// One warp per row; the row is pre-scaled by 2^s so its max lands in [2^14, 2^15) (s clamped
// to [-60, 60]).  Rows M..Mp-1 only get rs = 0 so every scale the GEMM reads is defined.
// 2^s (|s| <= 126) built in the exponent field; x * pow2f(s) is the correctly rounded x * 2^s
__device__ __forceinline__ float pow2f(int s) { return __int_as_float((127 + s) << 23); }

__device__ __forceinline__ int split_shift(float mx) {
  if (!(mx > 0.0f) || !(mx <= 3.402823466e38f)) return 0;
  const int s = 14 - ilogbf(mx);
  return s < -60 ? -60 : (s > 60 ? 60 : s);
}

// Inverse pre-scale 2^-s for the split of GELU(X . W + b), chosen before that product exists
// from the row's euclidean norm: |y_n| <= |x|_2 * max_n |W[:, n]|_2 + max_n |b_n| (Cauchy-
// Schwarz) and |GELU(y)| <= max(|y|, 0.1701), so with 2^-6 of relative slack for the rounding
// of the norm and of the product the row's largest GELU output times 2^s stays below 2^15
// (fp16's range never clips).  A bound above the true maximum only lowers s: the split values
// carry the same bits times a power of two, except values that become fp16-subnormal, whose
// absolute error stays below 2^-25 of 2^-s.
__device__ __forceinline__ float gelu_split_rscale(float sumsq, float wnorm, float bmax) {
  const float bound = fmaxf(fmaf(sqrtf(sumsq), wnorm, bmax) * (1.0f + 0x1p-6f), 0.25f);
  return pow2f(-split_shift(bound));
}

__global__ void nf24_split_rows(const float* __restrict__ x, int M, int Mp, int K, int Kp,
                                int stride_x, __half* __restrict__ hi, __half* __restrict__ lo,
                                float* __restrict__ rs) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= Mp) return;
  if (row >= M) {
    if (lane == 0) rs[row] = 0.0f;
    return;
  }
  const float* xr = x + (int64_t)row * stride_x;
  float mx = 0.0f;
  for (int k = lane; k < K; k += 32) mx = fmaxf(mx, fabsf(xr[k]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const int shift = split_shift(mx);
  __half* hr = hi + (int64_t)row * Kp;
  __half* lr = lo + (int64_t)row * Kp;
  for (int k = lane * 2; k < Kp; k += 64) {
    const float a = k < K ? xr[k] * pow2f(shift) : 0.0f;
    const float b = k + 1 < K ? xr[k + 1] * pow2f(shift) : 0.0f;
    const __half2 h = __floats2half2_rn(a, b);
    const float2 hf = __half22float2(h);
    *reinterpret_cast<__half2*>(hr + k) = h;
    *reinterpret_cast<__half2*>(lr + k) = __floats2half2_rn(a - hf.x, b - hf.y);
  }
  if (lane == 0) rs[row] = pow2f(-shift);
}

// Register-resident variants for rows of NV * 128 floats (16-byte aligned rows): the row is
// read from HBM once (the generic kernels read it two to four times), and the pre-scale is a
// multiplication by the exact power of two (identical to ldexpf in the normal range the
// shift keeps the values in).  One warp per row; lane i owns float4 groups i, i+32, ...

template <int NV>
__device__ __forceinline__ void store_split_row(const float4 (&v)[NV], float mx, int lane, __half* hr,
                                                __half* lr, float* rs_row) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const int shf = split_shift(mx);
  const float p2 = pow2f(shf);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const float a0 = v[i].x * p2, a1 = v[i].y * p2, a2 = v[i].z * p2, a3 = v[i].w * p2;
    const __half2 h01 = __floats2half2_rn(a0, a1), h23 = __floats2half2_rn(a2, a3);
    const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
    const __half2 l01 = __floats2half2_rn(a0 - f01.x, a1 - f01.y), l23 = __floats2half2_rn(a2 - f23.x, a3 - f23.y);
    const int c = (i * 32 + lane) * 4;
    *reinterpret_cast<uint2*>(hr + c) = make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h23));
    *reinterpret_cast<uint2*>(lr + c) = make_uint2(*reinterpret_cast<const uint32_t*>(&l01), *reinterpret_cast<const uint32_t*>(&l23));
  }
  if (lane == 0) *rs_row = pow2f(-shf);
}

template <int NV>
__global__ void __launch_bounds__(256) nf24_split_rows_reg(const float* __restrict__ x, int M, int Mp,
                                                           int stride_x, __half* __restrict__ hi,
                                                           __half* __restrict__ lo, float* __restrict__ rs) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= Mp) return;
  if (row >= M) {
    if (lane == 0) rs[row] = 0.0f;
    return;
  }
  const float4* xr = reinterpret_cast<const float4*>(x + (int64_t)row * stride_x);
  float4 v[NV];
  float mx = 0.0f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    v[i] = xr[i * 32 + lane];
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
  }
  constexpr int K = NV * 128;
  store_split_row<NV>(v, mx, lane, hi + (int64_t)row * K, lo + (int64_t)row * K, rs + row);
}

// four CTAs (32 rows in flight) per SM: the row loads are the kernel's latency
template <int NV>
__global__ void __launch_bounds__(256, 4) ln_modulate_split_reg(
    const float* __restrict__ x, int M, int Mp, float eps, const float* __restrict__ shift,
    const float* __restrict__ scale, int mod_ld, int rows_per_batch, __half* __restrict__ hi,
    __half* __restrict__ lo, float* __restrict__ rs, float* __restrict__ next_rs, float wnorm,
    float bmax) {
  constexpr int C = NV * 128;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= Mp) return;
  if (row >= M) {
    if (lane == 0) {
      rs[row] = 0.0f;
      if (next_rs) next_rs[row] = 0.0f;
    }
    return;
  }
  const float4* xr = reinterpret_cast<const float4*>(x + (int64_t)row * C);
  float4 v[NV];
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    v[i] = xr[i * 32 + lane];
    s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / (float)C;
  float var = 0.0f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const float d0 = v[i].x - mean, d1 = v[i].y - mean, d2 = v[i].z - mean, d3 = v[i].w - mean;
    var = fmaf(d0, d0, fmaf(d1, d1, fmaf(d2, d2, fmaf(d3, d3, var))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
  const float inv = 1.0f / sqrtf(var / (float)C + eps);
  const int b = row / rows_per_batch;
  const float4* sh = shift ? reinterpret_cast<const float4*>(shift + (int64_t)b * mod_ld) : nullptr;
  const float4* sc = scale ? reinterpret_cast<const float4*>(scale + (int64_t)b * mod_ld) : nullptr;
  float mx = 0.0f, ss = 0.0f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    float4 y = make_float4((v[i].x - mean) * inv, (v[i].y - mean) * inv, (v[i].z - mean) * inv, (v[i].w - mean) * inv);
    if (sc) {
      const float4 a = sc[i * 32 + lane], c = sh[i * 32 + lane];
      y = make_float4(y.x * (1.0f + a.x) + c.x, y.y * (1.0f + a.y) + c.y, y.z * (1.0f + a.z) + c.z,
                      y.w * (1.0f + a.w) + c.w);
    }
    v[i] = y;
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(y.x), fabsf(y.y)), fmaxf(fabsf(y.z), fabsf(y.w))));
    ss = fmaf(y.x, y.x, fmaf(y.y, y.y, fmaf(y.z, y.z, fmaf(y.w, y.w, ss))));
  }
  if (next_rs) {  // warp-uniform
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) next_rs[row] = gelu_split_rscale(ss, wnorm, bmax);
  }
  store_split_row<NV>(v, mx, lane, hi + (int64_t)row * C, lo + (int64_t)row * C, rs + row);
}

// LayerNorm (no affine; the reference's two-pass mean / biased variance / 1/sqrtf(var+eps),
// scripts/native_norm_rope_avx512.c:26-41), optional adaLN modulation h*(1+scale[b])+shift[b]
// (scripts/native_block_elementwise_avx512.c:9-22), written straight to the GEMM's split
// format (per-row scale as nf24_split_rows).  One warp per row.
__device__ __forceinline__ float ln_mod_value(const float* xr, int c, float mean, float inv,
                                              const float* sh, const float* sc) {
  float a = (xr[c] - mean) * inv;
  if (sc) a = a * (1.0f + sc[c]) + sh[c];
  return a;
}

__global__ void ln_modulate_split(const float* __restrict__ x, int M, int Mp, int C, int Kp,
                                  float eps, const float* __restrict__ shift,
                                  const float* __restrict__ scale, int mod_ld, int rows_per_batch,
                                  __half* __restrict__ hi, __half* __restrict__ lo,
                                  float* __restrict__ rs, float* __restrict__ next_rs, float wnorm,
                                  float bmax) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= Mp) return;
  if (row >= M) {
    if (lane == 0) {
      rs[row] = 0.0f;
      if (next_rs) next_rs[row] = 0.0f;
    }
    return;
  }
  const float* xr = x + (int64_t)row * C;
  float s = 0.0f;
  for (int c = lane; c < C; c += 32) s += xr[c];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / (float)C;
  float v = 0.0f;
  for (int c = lane; c < C; c += 32) {
    const float d = xr[c] - mean;
    v = fmaf(d, d, v);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const float inv = 1.0f / sqrtf(v / (float)C + eps);
  const int b = row / rows_per_batch;
  const float* sh = shift ? shift + (int64_t)b * mod_ld : nullptr;
  const float* sc = scale ? scale + (int64_t)b * mod_ld : nullptr;
  float mx = 0.0f, ss = 0.0f;
  for (int c = lane; c < C; c += 32) {
    const float a = ln_mod_value(xr, c, mean, inv, sh, sc);
    mx = fmaxf(mx, fabsf(a));
    ss = fmaf(a, a, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (next_rs) {  // warp-uniform
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) next_rs[row] = gelu_split_rscale(ss, wnorm, bmax);
  }
  const int shf = split_shift(mx);
  __half* hr = hi + (int64_t)row * Kp;
  __half* lr = lo + (int64_t)row * Kp;
  for (int k = lane * 2; k < Kp; k += 64) {
    const float a = k < C ? ln_mod_value(xr, k, mean, inv, sh, sc) * pow2f(shf) : 0.0f;
    const float bb = k + 1 < C ? ln_mod_value(xr, k + 1, mean, inv, sh, sc) * pow2f(shf) : 0.0f;
    const __half2 h = __floats2half2_rn(a, bb);
    const float2 hf = __half22float2(h);
    *reinterpret_cast<__half2*>(hr + k) = h;
    *reinterpret_cast<__half2*>(lr + k) = __floats2half2_rn(a - hf.x, bb - hf.y);
  }
  if (lane == 0) rs[row] = pow2f(-shf);
}

// Reference-order scalar kernel: one thread per output, acc = bias, then an in-order
// fmaf chain over k with w = (float)(256*q01 + q2) * scale[n] (the reference tail kernel's
// arithmetic, scripts/gemm_nf24_i16_avx512_tail.c:32-47: bit-identical outputs).
// The CTA (128 columns of one row) stages SIMT_KC k values of the row and of its columns'
// combined codes in shared memory, all loads issued together, then each thread runs its
// in-order chain over the chunk from shared memory (a chain over global memory waits one
// memory latency per k).
constexpr int SIMT_KC = 64;
__global__ void __launch_bounds__(128) nf24_gemm_simt(
    const float* __restrict__ x, const int16_t* __restrict__ c01, const int8_t* __restrict__ q2,
    const float* __restrict__ scale, const float* __restrict__ bias, float* __restrict__ out, int M,
    int K, int N, int start, int count, int stride_x, int stride_out) {
  __shared__ float xs[SIMT_KC];
  __shared__ int32_t qs[SIMT_KC][128];
  const int j0 = blockIdx.x * blockDim.x;
  const int j = j0 + threadIdx.x;
  const int m = blockIdx.y;
  if (m >= M) return;  // CTA-uniform
  const int cols = min(128, count - j0);
  const float* xr = x + (int64_t)m * stride_x;
  const bool active = j < count;
  const int n = start + (active ? j : 0);
  const float sc = active ? scale[n] : 0.0f;
  float acc = active ? bias[n] : 0.0f;
  for (int k0 = 0; k0 < K; k0 += SIMT_KC) {
    const int kc = min(SIMT_KC, K - k0);
    __syncthreads();  // the previous chunk is consumed
    for (int e = threadIdx.x; e < kc * cols; e += blockDim.x) {
      const int kk = e / cols, c = e - kk * cols;
      const int64_t idx = (int64_t)(k0 + kk) * N + start + j0 + c;
      qs[kk][c] = (int32_t)c01[idx] * 256 + (int32_t)q2[idx];
    }
    if (threadIdx.x < kc) xs[threadIdx.x] = xr[k0 + threadIdx.x];
    __syncthreads();
    if (active) {
#pragma unroll 8
      for (int kk = 0; kk < kc; ++kk) acc = fmaf(xs[kk], __fmul_rn((float)qs[kk][threadIdx.x], sc), acc);
    }
  }
  if (active) out[(int64_t)m * stride_out + j] = acc;
}

}  // namespace gemm

// Split activations: planes [M, Kp] (Kp = K rounded to 8) and row scales [Mp] (Mp = M
// rounded to 4), laid out back to back in one buffer of split_bytes(M, K).
struct SplitPlanes {
  const __half* hi;
  const __half* lo;
  const float* rs;
  int M, K, Kp, Mp;
};

static inline size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

static size_t split_bytes(int M, int K) { return split_buffer_layout(M, K).bytes; }

static SplitPlanes split_layout(uint8_t* base, int M, int K) {
  const SplitLayout l = split_buffer_layout(M, K);
  SplitPlanes sp;
  sp.M = M;
  sp.K = K;
  sp.Kp = l.Kp;
  sp.Mp = l.Mp;
  sp.hi = reinterpret_cast<const __half*>(base);
  sp.lo = reinterpret_cast<const __half*>(base + l.lo_offset);
  sp.rs = reinterpret_cast<const float*>(base + l.rs_offset);
  return sp;
}

static int launch_split(const float* x, int stride_x, const SplitPlanes& sp, cudaStream_t stream) {
  using namespace gemm;
  LaunchScope scope(kKGemmSplit, stream);
  __half* hi = const_cast<__half*>(sp.hi);
  __half* lo = const_cast<__half*>(sp.lo);
  float* rs = const_cast<float*>(sp.rs);
  const unsigned grid = (unsigned)((sp.Mp + 7) / 8);
  const bool vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (stride_x & 3) == 0 && sp.Kp == sp.K;
  if (vec && sp.K == 1024)
    nf24_split_rows_reg<8><<<grid, 256, 0, stream>>>(x, sp.M, sp.Mp, stride_x, hi, lo, rs);
  else if (vec && sp.K == 2048)
    nf24_split_rows_reg<16><<<grid, 256, 0, stream>>>(x, sp.M, sp.Mp, stride_x, hi, lo, rs);
  else if (vec && sp.K == 4096)
    nf24_split_rows_reg<32><<<grid, 256, 0, stream>>>(x, sp.M, sp.Mp, stride_x, hi, lo, rs);
  else
    nf24_split_rows<<<grid, 256, 0, stream>>>(x, sp.M, sp.Mp, sp.K, sp.Kp, stride_x, hi, lo, rs);
  return launch_status();
}

static int ln_modulate_split_launch(const float* x, int M, int C, float eps, const float* shift,
                                    const float* scale, int mod_ld, int rows_per_batch,
                                    void* split, void* next_split, int next_K, float wnorm,
                                    float bmax) {
  if (!x || !split || (!shift) != (!scale)) return kNullPointer;
  if (M <= 0 || C <= 0 || eps < 0.0f || rows_per_batch <= 0 || (scale && mod_ld < C))
    return kBadDims;
  if (reinterpret_cast<uintptr_t>(split) & 255) return kBadAlignment;
  int st = entry_check();
  if (st != kOk) return st;
  const SplitPlanes sp = split_layout(static_cast<uint8_t*>(split), M, C);
  float* next_rs = next_split ? const_cast<float*>(split_layout(static_cast<uint8_t*>(next_split), M, next_K).rs)
                              : nullptr;
  cudaStream_t stream = current_stream();
  {
    LaunchScope scope(kKElementwise, stream);
    const bool vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && C == 1024 && (mod_ld & 3) == 0 &&
                     ((reinterpret_cast<uintptr_t>(shift) | reinterpret_cast<uintptr_t>(scale)) & 15) == 0;
    if (vec)
      gemm::ln_modulate_split_reg<8><<<(sp.Mp + 7) / 8, 256, 0, stream>>>(
          x, M, sp.Mp, eps, shift, scale, mod_ld, rows_per_batch, const_cast<__half*>(sp.hi),
          const_cast<__half*>(sp.lo), const_cast<float*>(sp.rs), next_rs, wnorm, bmax);
    else
      gemm::ln_modulate_split<<<(sp.Mp + 7) / 8, 256, 0, stream>>>(
          x, M, sp.Mp, C, sp.Kp, eps, shift, scale, mod_ld, rows_per_batch,
          const_cast<__half*>(sp.hi), const_cast<__half*>(sp.lo), const_cast<float*>(sp.rs),
          next_rs, wnorm, bmax);
  }
  return launch_status();
}

struct EpilogueArgs {
  int mode = gemm::kStore;
  const float* gate = nullptr;
  int gate_ld = 0, rows_per_batch = 1;
};

// [K][N] -> [N][K] for both code planes (one-time prepack of a weight into the
// k-contiguous layout the NK decoder reads); 32 x 32 tiles through shared memory.
__global__ void nf24_codes_to_nk_kernel(const int16_t* __restrict__ c01, const int8_t* __restrict__ q2,
                                        int K, int N, int16_t* __restrict__ c01_nk,
                                        int8_t* __restrict__ q2_nk) {
  __shared__ int16_t t16[32][33];
  __shared__ int8_t t8[32][36];
  const int n0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;
  for (int j = ty; j < 32; j += 8) {
    const int k = k0 + j, n = n0 + tx;
    if (k < K && n < N) {
      t16[j][tx] = c01[(size_t)k * N + n];
      t8[j][tx] = q2[(size_t)k * N + n];
    }
  }
  __syncthreads();
  for (int j = ty; j < 32; j += 8) {
    const int n = n0 + j, k = k0 + tx;
    if (n < N && k < K) {
      c01_nk[(size_t)n * K + k] = t16[tx][j];
      q2_nk[(size_t)n * K + k] = t8[tx][j];
    }
  }
}

// Columns [start, start + count) of the [K][N] code planes -> k-contiguous [count][ldk]
// planes for the drop-in entry points (ldk = K rounded up to 16; codes past K are written
// as 0 and never read: the GEMM's tensor map ends at K).  One CTA per 64 k x 64 columns.
// Loads: 16-byte vectors along a k row (128 contiguous bytes of q01, 64 of q2 per 8
// threads).  Each thread packs two consecutive k of q01 (four of q2) per column into a
// 32-bit word with byte permutes and stores the words into shared memory as column rows
// (q01: 32 words, q2: 16 words per column), the 16-byte chunks of a row XOR-swizzled by
// bits 3-5 of the column so the eight column groups of a warp's stores hit different
// banks.  Stores: each column's 64 k as 128 (q01) / 64 (q2) contiguous bytes.
// Needs N % 16 == 0, start % 16 == 0, count % 16 == 0 and 16-byte aligned planes.
__global__ void __launch_bounds__(256) nf24_codes_window_to_nk(
    const int16_t* __restrict__ c01, const int8_t* __restrict__ q2, int K, int N, int start,
    int count, int ldk, int16_t* __restrict__ c01_nk, int8_t* __restrict__ q2_nk) {
  __shared__ __align__(16) uint32_t w16[64 * 32];  // [column][k pair], chunks swizzled
  __shared__ __align__(16) uint32_t w8[64 * 16];   // [column][k quad], chunks swizzled
  const int t = threadIdx.x;
  const int k0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  {
    // q01: thread (k pair p, column group g of 8 columns)
    const int g = t & 7, p = t >> 3;
    const int k = k0 + 2 * p, n = n0 + 8 * g;
    int4 a = make_int4(0, 0, 0, 0), b = a;
    if (n < count) {
      const int16_t* src = c01 + (size_t)k * N + start + n;
      if (k < K) a = __ldg(reinterpret_cast<const int4*>(src));
      if (k + 1 < K) b = __ldg(reinterpret_cast<const int4*>(src + N));
    }
    const uint32_t av[4] = {(uint32_t)a.x, (uint32_t)a.y, (uint32_t)a.z, (uint32_t)a.w};
    const uint32_t bv[4] = {(uint32_t)b.x, (uint32_t)b.y, (uint32_t)b.z, (uint32_t)b.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      // column 8g + j: its q01 at k (low half) and k + 1 (high half)
      const uint32_t sel = (j & 1) ? 0x7632u : 0x5410u;
      const uint32_t wv = __byte_perm(av[j >> 1], bv[j >> 1], sel);
      const int c = 8 * g + j;
      const int chunk = (p >> 2) ^ ((c >> 3) & 7);
      w16[c * 32 + chunk * 4 + (p & 3)] = wv;
    }
  }
  if (t < 128) {
    // q2: thread (k quad q, column group g of 8 columns)
    const int g = t & 7, q = t >> 3;
    const int k = k0 + 4 * q, n = n0 + 8 * g;
    uint2 r[4] = {make_uint2(0, 0), make_uint2(0, 0), make_uint2(0, 0), make_uint2(0, 0)};
    if (n < count) {
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (k + e < K) r[e] = __ldg(reinterpret_cast<const uint2*>(q2 + (size_t)(k + e) * N + start + n));
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      // column 8g + j: bytes j of rows k .. k + 3
      const int h = j >> 2, sh = (j & 3) * 8;
      const uint32_t b0 = ((h ? r[0].y : r[0].x) >> sh) & 0xFFu;
      const uint32_t b1 = ((h ? r[1].y : r[1].x) >> sh) & 0xFFu;
      const uint32_t b2 = ((h ? r[2].y : r[2].x) >> sh) & 0xFFu;
      const uint32_t b3 = ((h ? r[3].y : r[3].x) >> sh) & 0xFFu;
      const int c = 8 * g + j;
      const int chunk = (q >> 2) ^ ((c >> 3) & 3);
      w8[c * 16 + chunk * 4 + (q & 3)] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
    }
  }
  __syncthreads();
#pragma unroll
  for (int pass = 0; pass < 2; ++pass) {  // q01: 8 threads per column, 16 bytes each
    const int c = pass * 32 + (t >> 3), ch = t & 7;
    const int n = n0 + c, k = k0 + ch * 8;
    if (n < count && k < ldk) {
      const int4 v = *reinterpret_cast<const int4*>(&w16[c * 32 + ((ch ^ ((c >> 3) & 7)) * 4)]);
      *reinterpret_cast<int4*>(c01_nk + (size_t)n * ldk + k) = v;
    }
  }
  {  // q2: 4 threads per column, 16 bytes each
    const int c = t >> 2, ch = t & 3;
    const int n = n0 + c, k = k0 + ch * 16;
    if (n < count && k < ldk) {
      const int4 v = *reinterpret_cast<const int4*>(&w8[c * 16 + ((ch ^ ((c >> 3) & 3)) * 4)]);
      *reinterpret_cast<int4*>(q2_nk + (size_t)n * ldk + k) = v;
    }
  }
}

// Tensor-core GEMM on already split activations.  ldk == 0: the reference's [K][N] code
// planes; ldk > 0: k-contiguous [N][K] planes (nf24_codes_to_nk) with rows ldk elements
// apart (ldk > K for a window of input features).
// kpp_one (k-contiguous planes only): one k-block per tensor-memory partial, the drop-in
// entry points' accuracy, instead of NK_KPP.
static int launch_tc(const SplitPlanes& sp, const int16_t* c01, const int8_t* q2,
                     const float* scale, const float* bias, float* out, int N, int start,
                     int count, int stride_out, const EpilogueArgs& ep, int* status,
                     cudaStream_t stream, int ldk = 0, bool kpp_one = false) {
  using namespace gemm;
  const int M = sp.M, K = sp.K;
  CUtensorMap m_hi, m_lo, m_c16, m_c8;
  {
    const uint64_t dims[2] = {(uint64_t)sp.Kp, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)sp.Kp * 2};
    const uint32_t box[2] = {BK, BM};
    if (!encode_tmap(&m_hi, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(sp.hi), dims,
                     strides, box, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_tmap(&m_lo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(sp.lo), dims,
                     strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return kLaunchFailed;
  }
  const bool nk = ldk > 0;
  if (!nk) {
    const uint64_t dims[2] = {(uint64_t)N, (uint64_t)K};
    const uint64_t s16[1] = {(uint64_t)N * 2};
    const uint64_t s8[1] = {(uint64_t)N};
    const uint32_t box[2] = {BN, BK};
    if (!encode_tmap(&m_c16, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<int16_t*>(c01), dims,
                     s16, box, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode_tmap(&m_c8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(q2), dims, s8,
                     box, CU_TENSOR_MAP_SWIZZLE_NONE))
      return kLaunchFailed;
  } else {
    // rows of 64 k: 128 B of q01 (128-B swizzle), 64 B of q2 (64-B swizzle)
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)N};
    const uint64_t s16[1] = {(uint64_t)ldk * 2};
    const uint64_t s8[1] = {(uint64_t)ldk};
    const uint32_t box[2] = {BK, BN};
    if (!encode_tmap(&m_c16, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<int16_t*>(c01), dims,
                     s16, box, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_tmap(&m_c8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(q2), dims, s8,
                     box, CU_TENSOR_MAP_SWIZZLE_64B))
      return kLaunchFailed;
  }
  CUtensorMap m_out;  // the [M, count] output, for the epilogue's TMA stores
  const float* next_rs = nullptr;
  if (ep.mode == kGeluSplit) {
    // out is the split buffer of an [M, count] activation: its two fp16 planes as one
    // [2][M][Kp] tensor (the planes are 256-byte aligned, so the plane stride is too)
    const SplitPlanes nx = split_layout(reinterpret_cast<uint8_t*>(out), M, count);
    const uint64_t dims[3] = {(uint64_t)count, (uint64_t)M, 2};
    const uint64_t strides[2] = {(uint64_t)nx.Kp * 2,
                                 (uint64_t)(reinterpret_cast<const uint8_t*>(nx.lo) -
                                            reinterpret_cast<const uint8_t*>(nx.hi))};
    const uint32_t box[3] = {32, OUT_ROWS, 2};
    if (!encode_tmap(&m_out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(nx.hi), dims,
                     strides, box, CU_TENSOR_MAP_SWIZZLE_NONE))
      return kLaunchFailed;
    next_rs = nx.rs;
  } else {
    const uint64_t dims[2] = {(uint64_t)count, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)stride_out * 4};
    const uint32_t box[2] = {32, OUT_ROWS};
    if (!encode_tmap(&m_out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, out, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_NONE))
      return kLaunchFailed;
  }
  Params prm{sp.rs, scale, bias, out, M, K, N, start, count, stride_out,
             ep.mode, ep.gate, ep.gate_ld, ep.rows_per_batch, status, next_rs};
  // per kernel: one bit per device ordinal once its shared-memory attribute is set; SM
  // count per device.  Atomic: host threads on their own streams launch concurrently (a
  // thread that sees a bit unset sets the attribute itself before launching).
  static std::atomic<uint64_t> attr_done[11];
  static std::atomic<int> sm_count[64];
  int dev = 0;
  cudaGetDevice(&dev);
  int sms = sm_count[dev & 63].load(std::memory_order_acquire);
  if (sms == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    sms = n > 0 ? n : 148;
    sm_count[dev & 63].store(sms, std::memory_order_release);
  }
  // one persistent CTA per SM (or one per tile when there are fewer tiles)
  const long long tiles = (long long)((count + BN - 1) / BN) * ((M + BM - 1) / BM);
  const dim3 grid((unsigned)(tiles < sms ? tiles : sms));
  const int smem = SMEM_BYTES;
  auto run = [&](auto kernel, int mode) {
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_done[mode].load(std::memory_order_acquire) & bit)) {
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      attr_done[mode].fetch_or(bit, std::memory_order_acq_rel);
    }
    LaunchScope scope(kKGemmTc, stream);
    kernel<<<grid, NUM_THREADS, smem, stream>>>(m_hi, m_lo, m_c16, m_c8, m_out, prm);
  };
  if (nk && kpp_one) {
    switch (ep.mode) {
      case kStore: run(nf24_gemm_tc<kStore, true, 1>, 9); break;
      case kGelu: run(nf24_gemm_tc<kGelu, true, 1>, 10); break;
      default: return kLaunchFailed;
    }
  } else if (nk) {
    switch (ep.mode) {
      case kGelu: run(nf24_gemm_tc<kGelu, true, NK_KPP>, 4 + kGelu); break;
      case kGatedResidual: run(nf24_gemm_tc<kGatedResidual, true, NK_KPP>, 4 + kGatedResidual); break;
      case kResidual: run(nf24_gemm_tc<kResidual, true, NK_KPP>, 4 + kResidual); break;
      case kGeluSplit: run(nf24_gemm_tc<kGeluSplit, true, NK_KPP>, 8); break;
      default: run(nf24_gemm_tc<kStore, true, NK_KPP>, 4 + kStore); break;
    }
  } else {
    switch (ep.mode) {
      case kGelu: run(nf24_gemm_tc<kGelu, false, 1>, kGelu); break;
      case kGatedResidual: run(nf24_gemm_tc<kGatedResidual, false, 1>, kGatedResidual); break;
      case kResidual: run(nf24_gemm_tc<kResidual, false, 1>, kResidual); break;
      default: run(nf24_gemm_tc<kStore, false, 1>, kStore); break;
    }
  }
  return launch_status();
}

// Rows from which the drop-in entry points copy the codes into k-contiguous planes.
constexpr int kNkMinRows = 2048;

// k-contiguous copy of columns [start, start + count) of a weight's code planes, placed in
// the workspace by the caller (nk_codes_bytes).
struct NkCodes {
  const int16_t* c01 = nullptr;
  const int8_t* q2 = nullptr;
  int ldk = 0;
};
static int nk_ldk(int K) { return (K + 15) & ~15; }
static size_t nk_codes_bytes(int K, int count) {
  const size_t n = (size_t)count * nk_ldk(K);
  return ((n * 2 + 255) & ~static_cast<size_t>(255)) + ((n + 255) & ~static_cast<size_t>(255));
}
static int copy_codes_nk(const int16_t* c01, const int8_t* q2, int K, int N, int start, int count,
                         uint8_t* dst, cudaStream_t stream, NkCodes& nk) {
  const int ldk = nk_ldk(K);
  int16_t* d16 = reinterpret_cast<int16_t*>(dst);
  int8_t* d8 = reinterpret_cast<int8_t*>(dst + (((size_t)count * ldk * 2 + 255) & ~static_cast<size_t>(255)));
  LaunchScope scope(kKGemmSplit, stream);
  nf24_codes_window_to_nk<<<dim3((count + 63) / 64, (K + 63) / 64), 256, 0, stream>>>(
      c01, q2, K, N, start, count, ldk, d16, d8);
  nk.c01 = d16;
  nk.q2 = d8;
  nk.ldk = ldk;
  return launch_status();
}

// Host launcher shared by the full / range / tail entry points.
static int gemm_launch(const float* x, const int16_t* c01, const int8_t* q2, const float* scale,
                       const float* bias, float* out, int M, int K, int N, int start, int count,
                       int stride_x, int stride_out, bool allow_tc) {
  using namespace gemm;
  int st = entry_check();
  if (st != kOk) return st;
  if (!is_device_pointer(x) || !is_device_pointer(c01) || !is_device_pointer(q2) ||
      !is_device_pointer(scale) || !is_device_pointer(bias) || !is_device_pointer(out))
    return kNotDevicePointer;
  cudaStream_t stream = current_stream();
  // the tensor-core kernel reads the code planes and writes `out` through TMA: 16-byte
  // aligned bases and row strides
  const bool aligned = ((reinterpret_cast<uintptr_t>(c01) | reinterpret_cast<uintptr_t>(q2) |
                         reinterpret_cast<uintptr_t>(out)) & 15) == 0 && (stride_out % 4) == 0;
  const bool tc = allow_tc && (N % 16 == 0) && (start % 16 == 0) && aligned;
  if (!tc) {
    dim3 grid((count + 127) / 128, M);
    LaunchScope scope(kKGemmSimt, stream);
    nf24_gemm_simt<<<grid, 128, 0, stream>>>(x, c01, q2, scale, bias, out, M, K, N, start, count,
                                             stride_x, stride_out);
    return launch_status();
  }
  // From kNkMinRows rows on, the codes of the requested columns are first copied into
  // k-contiguous planes in the workspace (3 bytes per weight read and written once per
  // call): the k-contiguous kernel decodes a column's 64 codes with two 16-byte
  // shared-memory loads per thread instead of byte gathers, ~13% less GEMM time, which
  // pays for the copy once a weight serves ~1800 rows (measured at 4096 x 1024 x 3072).
  // Fewer rows keep the [K][N] kernel, which reads each code once.  One k-block per
  // partial keeps the two paths bit-identical row for row.
  if (M < kNkMinRows) {
    uint8_t* ws = static_cast<uint8_t*>(workspace(split_bytes(M, K), stream));
    if (!ws) return kWorkspace;
    const SplitPlanes sp = split_layout(ws, M, K);
    if ((st = launch_split(x, stride_x, sp, stream)) != kOk) return st;
    return launch_tc(sp, c01, q2, scale, bias, out, N, start, count, stride_out, EpilogueArgs(),
                     device_status(), stream);
  }
  const size_t sx = (split_bytes(M, K) + 255) & ~static_cast<size_t>(255);
  uint8_t* ws = static_cast<uint8_t*>(workspace(sx + nk_codes_bytes(K, count), stream));
  if (!ws) return kWorkspace;
  const SplitPlanes sp = split_layout(ws, M, K);
  NkCodes nk;
  if ((st = launch_split(x, stride_x, sp, stream)) != kOk) return st;
  if ((st = copy_codes_nk(c01, q2, K, N, start, count, ws + sx, stream, nk)) != kOk) return st;
  return launch_tc(sp, nk.c01, nk.q2, scale + start, bias + start, out, count, 0, count,
                   stride_out, EpilogueArgs(), device_status(), stream, nk.ldk, true);
}

}  // namespace tsb

// ---------------------------------------------------------------------------
// C-ABI (same names, argument lists and status codes as the reference library
// libtriposplat_gemm_nf24_i16_avx512.so).  Pointers are CUDA device pointers;
// the work is queued on the stream set by triposplat_b200_set_stream (default
// stream otherwise).  `threads` is accepted and ignored.  For NF24, codes0_t is
// the int16 q01 [K, N] plane, codes1_t (== codes2_t) the int8 q2 [K, N] plane and
// scales0 (== scales1 == scales2) the per-column scale; codebook is not read.
// ---------------------------------------------------------------------------
extern "C" {

// scripts/gemm_nf24_i16_avx512.c:151-197
int triposplat_gemm_rnf8_avx512_range(const float* x, const uint8_t* codes0_t,
                                      const uint8_t* codes1_t, const uint8_t* codes2_t,
                                      const float* scales0, const float* scales1,
                                      const float* scales2, const float* codebook,
                                      const float* bias, float* out, int M, int K, int N,
                                      int output_start, int output_count, int stride_x,
                                      int stride_out, int threads, int stages) {
  (void)threads;
  if (!x || !codes0_t || !codes1_t || !codes2_t || !scales0 || !scales1 || !scales2 ||
      !codebook || !bias || !out)
    return tsb::kNullPointer;
  if (M <= 0 || K <= 0 || N <= 0 || output_start < 0 || output_count <= 0 || stages != 3)
    return tsb::kBadDims;
  if (output_start + output_count > N || stride_x < K || stride_out < output_count)
    return tsb::kBadRange;
  if ((output_start & 15) != 0 || (output_count & 15) != 0) return tsb::kBadAlignment;
  return tsb::gemm_launch(x, reinterpret_cast<const int16_t*>(codes0_t),
                          reinterpret_cast<const int8_t*>(codes1_t), scales0, bias, out, M, K, N,
                          output_start, output_count, stride_x, stride_out, true);
}

// scripts/gemm_nf24_i16_avx512.c:199-220
int triposplat_gemm_rnf8_avx512(const float* x, const uint8_t* codes0_t, const uint8_t* codes1_t,
                                const uint8_t* codes2_t, const float* scales0,
                                const float* scales1, const float* scales2,
                                const float* codebook, const float* bias, float* out, int M,
                                int K, int N, int stride_x, int stride_out, int threads,
                                int stages) {
  return triposplat_gemm_rnf8_avx512_range(x, codes0_t, codes1_t, codes2_t, scales0, scales1,
                                           scales2, codebook, bias, out, M, K, N, 0, N, stride_x,
                                           stride_out, threads, stages);
}

// scripts/gemm_nf24_i16_avx512_tail.c:8-49 (any N; the reference-order scalar kernel)
int triposplat_gemm_rnf8_avx512_tail(const float* x, const uint8_t* codes0_t,
                                     const uint8_t* codes1_t, const uint8_t* codes2_t,
                                     const float* scales0, const float* scales1,
                                     const float* scales2, const float* codebook,
                                     const float* bias, float* out, int M, int K, int N,
                                     int stride_x, int stride_out, int threads, int stages) {
  (void)threads;
  if (!x || !codes0_t || !codes1_t || !codes2_t || !scales0 || !scales1 || !scales2 ||
      !codebook || !bias || !out)
    return tsb::kNullPointer;
  if (M <= 0 || K <= 0 || N <= 0 || stride_x < K || stride_out < N || stages != 3)
    return tsb::kBadDims;
  return tsb::gemm_launch(x, reinterpret_cast<const int16_t*>(codes0_t),
                          reinterpret_cast<const int8_t*>(codes1_t), scales0, bias, out, M, K, N,
                          0, N, stride_x, stride_out, false);
}

// scripts/gemm_nf24_i16_avx512.c:222-224: rows per CTA tile here (the CPU returns ROW_TILE)
int triposplat_gemm_rnf8_avx512_row_tile(void) { return tsb::gemm::BM; }

// scripts/gemm_nf24_i16_avx512.c:226-228: 4 = nf24_i16
int triposplat_gemm_rnf8_avx512_residual_mode(void) { return 4; }

}  // extern "C"

// ---------------------------------------------------------------------------
// Fused entry points for B200 (no reference counterpart).  They pass activations
// between kernels in the GEMM's split format — fp16 hi/lo planes plus one power-of-two
// scale per row — so the LayerNorm, modulation, GELU and residual
// passes of the block are folded into the kernels that produce or consume them.
// A split buffer holds triposplat_b200_split_bytes(M, K) bytes.
// ---------------------------------------------------------------------------
extern "C" {

uint64_t triposplat_b200_split_bytes(int M, int K) {
  if (M <= 0 || K <= 0) return 0;
  return tsb::split_bytes(M, K);
}

// X fp32 [M, K] (row stride stride_x) -> split buffer.
int triposplat_b200_split_f32(const float* x, int M, int K, int stride_x, void* split) {
  using namespace tsb;
  if (!x || !split) return kNullPointer;
  if (M <= 0 || K <= 0 || stride_x < K) return kBadDims;
  if (reinterpret_cast<uintptr_t>(split) & 255) return kBadAlignment;
  int st = entry_check();
  if (st != kOk) return st;
  return launch_split(x, stride_x, split_layout(static_cast<uint8_t*>(split), M, K),
                      current_stream());
}

// LayerNorm without affine (eps) over rows of x [M, C], then, if shift and scale are
// given ([B, mod_ld], batch b = row / rows_per_batch), h*(1+scale[b]) + shift[b]; the
// result goes straight to a split buffer.
int triposplat_b200_ln_modulate_split(const float* x, int M, int C, float eps, const float* shift,
                                      const float* scale, int mod_ld, int rows_per_batch,
                                      void* split) {
  return tsb::ln_modulate_split_launch(x, M, C, eps, shift, scale, mod_ld, rows_per_batch, split,
                                       nullptr, 0, 0.0f, 0.0f);
}

// triposplat_b200_ln_modulate_split, and in the same pass the row scales of the split buffer
// next_split (an [M, next_K] activation) for a following
// triposplat_b200_gemm_nf24_split_nk mode 4 (GELU into next_split): per row
// 2^-s with GELU(h . W + b) * 2^s below 2^15 for any W whose columns have euclidean norm at
// most wnorm and any bias with |b| <= bmax (h = this row as split).  The planes of
// next_split are left to that GEMM.
int triposplat_b200_ln_modulate_split_bound(const float* x, int M, int C, float eps,
                                            const float* shift, const float* scale, int mod_ld,
                                            int rows_per_batch, void* split, void* next_split,
                                            int next_K, float wnorm, float bmax) {
  using namespace tsb;
  if (!next_split) return kNullPointer;
  if (next_K <= 0 || !(wnorm >= 0.0f) || !(bmax >= 0.0f) || !(wnorm < 3.0e38f) || !(bmax < 3.0e38f))
    return kBadDims;
  if (reinterpret_cast<uintptr_t>(next_split) & 255) return kBadAlignment;
  return ln_modulate_split_launch(x, M, C, eps, shift, scale, mod_ld, rows_per_batch, split,
                                  next_split, next_K, wnorm, bmax);
}

// NF24 GEMM on a split buffer (M x K) with one of the epilogues
//   mode 0: out = y;  1: out = GELU_tanh(y);  2: out += gate[row / rows_per_batch] * y
//   (gate row stride gate_ld, column n);  3: out += y,
// y = X . W + bias over all N columns (N % 16 == 0), out row stride stride_out.
int triposplat_b200_gemm_nf24_split(const void* split, int M, int K, const int16_t* code01_t,
                                    const int8_t* q2_t, const float* scale, const float* bias,
                                    float* out, int N, int stride_out, int mode,
                                    const float* gate, int gate_ld, int rows_per_batch) {
  using namespace tsb;
  if (!split || !code01_t || !q2_t || !scale || !bias || !out) return kNullPointer;
  if (M <= 0 || K <= 0 || N <= 0 || stride_out < N || mode < 0 || mode > 3) return kBadDims;
  if (mode == gemm::kGatedResidual && (!gate || gate_ld < N || rows_per_batch <= 0))
    return kBadRange;
  if ((N % 16) != 0 || (stride_out % 4) != 0 ||
      ((reinterpret_cast<uintptr_t>(code01_t) | reinterpret_cast<uintptr_t>(q2_t) |
        reinterpret_cast<uintptr_t>(split) | reinterpret_cast<uintptr_t>(out)) & 15) != 0)
    return kBadAlignment;
  int st = entry_check();
  if (st != kOk) return st;
  EpilogueArgs ep;
  ep.mode = mode;
  ep.gate = gate;
  ep.gate_ld = gate_ld;
  ep.rows_per_batch = rows_per_batch > 0 ? rows_per_batch : 1;
  return launch_tc(split_layout(static_cast<uint8_t*>(const_cast<void*>(split)), M, K), code01_t,
                   q2_t, scale, bias, out, N, 0, N, stride_out, ep, device_status(),
                   current_stream());
}

// No reference counterpart: triposplat_b200_gemm_nf24_split restricted to the output
// columns [start, start + count) of an N-column weight (out is [M, count], stride_out
// elements per row) -- the column windows a tensor-parallel rank computes.  start and count
// are multiples of 16 (the weights' TMA addressing).
int triposplat_b200_gemm_nf24_split_range(const void* split, int M, int K, const int16_t* code01_t,
                                          const int8_t* q2_t, const float* scale, const float* bias,
                                          float* out, int N, int start, int count, int stride_out,
                                          int mode, const float* gate, int gate_ld,
                                          int rows_per_batch) {
  using namespace tsb;
  if (!split || !code01_t || !q2_t || !scale || !bias || !out) return kNullPointer;
  if (M <= 0 || K <= 0 || N <= 0 || count <= 0 || start < 0 || stride_out < count || mode < 0 || mode > 3)
    return kBadDims;
  if (start + count > N) return kBadRange;
  // the gate is indexed by the weight's column: each batch row holds N entries
  if (mode == gemm::kGatedResidual && (!gate || gate_ld < N || rows_per_batch <= 0))
    return kBadRange;
  if ((N % 16) != 0 || (start % 16) != 0 || (count % 16) != 0 || (stride_out % 4) != 0 ||
      ((reinterpret_cast<uintptr_t>(code01_t) | reinterpret_cast<uintptr_t>(q2_t) |
        reinterpret_cast<uintptr_t>(split) | reinterpret_cast<uintptr_t>(out)) & 15) != 0)
    return kBadAlignment;
  int st = entry_check();
  if (st != kOk) return st;
  EpilogueArgs ep;
  ep.mode = mode;
  ep.gate = gate;
  ep.gate_ld = gate_ld;
  ep.rows_per_batch = rows_per_batch > 0 ? rows_per_batch : 1;
  return launch_tc(split_layout(static_cast<uint8_t*>(const_cast<void*>(split)), M, K), code01_t,
                   q2_t, scale, bias, out, N, start, count, stride_out, ep, device_status(),
                   current_stream());
}

// No reference counterpart: copies a weight's reference-layout code planes (code01_t int16
// [K, N], q2_t int8 [K, N]) into the k-contiguous planes code01_nk int16 [N, K] and
// q2_nk int8 [N, K] read by triposplat_b200_gemm_nf24_split_nk (done once, at load).
int triposplat_b200_nf24_codes_to_nk(const int16_t* code01_t, const int8_t* q2_t, int K, int N,
                                     int16_t* code01_nk, int8_t* q2_nk) {
  using namespace tsb;
  if (!code01_t || !q2_t || !code01_nk || !q2_nk) return kNullPointer;
  if (K <= 0 || N <= 0 || K / 32 >= 65535) return kBadDims;
  int st = entry_check();
  if (st != kOk) return st;
  cudaStream_t stream = current_stream();
  LaunchScope scope(kKElementwise, stream);
  nf24_codes_to_nk_kernel<<<dim3((N + 31) / 32, (K + 31) / 32), dim3(32, 8), 0, stream>>>(
      code01_t, q2_t, K, N, code01_nk, q2_nk);
  return launch_status();
}

// No reference counterpart: triposplat_b200_gemm_nf24_split_range on k-contiguous code planes
// (triposplat_b200_nf24_codes_to_nk).  Row n of the planes holds the K codes of output column
// n, rows ldk elements apart (ldk >= K; ldk > K with the planes offset by k0 selects the input
// features [k0, k0 + K) of a wider weight).  Plane pointers 16-byte aligned, ldk % 16 == 0.
// mode 4: GELU_tanh(y) written into the split buffer `out` of an [M, count] activation
// (256-byte aligned, stride_out == count) whose row scales were filled beforehand by
// triposplat_b200_ln_modulate_split_bound; out[m, :] gets the fp16 planes of
// GELU(y[m, :]) * 2^s_m for the stored inverse scale 2^-s_m.
int triposplat_b200_gemm_nf24_split_nk(const void* split, int M, int K, const int16_t* code01_nk,
                                       const int8_t* q2_nk, int ldk, const float* scale,
                                       const float* bias, float* out, int N, int start, int count,
                                       int stride_out, int mode, const float* gate, int gate_ld,
                                       int rows_per_batch) {
  using namespace tsb;
  if (!split || !code01_nk || !q2_nk || !scale || !bias || !out) return kNullPointer;
  if (M <= 0 || K <= 0 || N <= 0 || count <= 0 || start < 0 || stride_out < count || mode < 0 ||
      mode > gemm::kGeluSplit)
    return kBadDims;
  if (start + count > N || ldk < K) return kBadRange;
  if (mode == gemm::kGeluSplit && (stride_out != count || (reinterpret_cast<uintptr_t>(out) & 255)))
    return kBadAlignment;
  if (mode == gemm::kGatedResidual && (!gate || gate_ld < N || rows_per_batch <= 0))
    return kBadRange;
  // outputs leave through TMA stores: 16-byte aligned base and row stride
  if ((ldk % 16) != 0 || (stride_out % 4) != 0 ||
      ((reinterpret_cast<uintptr_t>(code01_nk) | reinterpret_cast<uintptr_t>(q2_nk) |
        reinterpret_cast<uintptr_t>(split) | reinterpret_cast<uintptr_t>(out)) & 15) != 0)
    return kBadAlignment;
  int st = entry_check();
  if (st != kOk) return st;
  EpilogueArgs ep;
  ep.mode = mode;
  ep.gate = gate;
  ep.gate_ld = gate_ld;
  ep.rows_per_batch = rows_per_batch > 0 ? rows_per_batch : 1;
  return launch_tc(split_layout(static_cast<uint8_t*>(const_cast<void*>(split)), M, K), code01_nk,
                   q2_nk, scale, bias, out, N, start, count, stride_out, ep, device_status(),
                   current_stream(), ldk);
}

}  // extern "C"

// ===========================================================================
// Allocation-free NF24 GEMM.
//
// Some callers cannot let a library call cudaMalloc: code recorded into a CUDA graph
// (allocation is not a capturable stream operation), hosts whose device memory is owned
// by their own allocator or a fixed memory plan (an inference server, a framework's
// caching allocator), and latency-critical loops that cannot absorb cudaMalloc's
// implicit device-wide synchronisation.  For them this entry point computes exactly
// what triposplat_gemm_rnf8_avx512 computes, but takes its scratch (the fp16 hi/lo
// activation planes and their row scales) from the fixed array below instead of the
// library workspace, and never allocates.
//
// Limits and sharing: the scratch is 32 MiB per device and holds 2*M*Kp fp16 values plus
// Mp floats (Kp = K rounded up to 8, Mp = M rounded up to 4, each part padded to 256
// bytes); larger problems are rejected with -6.  Every call on
// a device uses the same array, so two calls whose kernels overlap on the GPU (different
// streams, no ordering between them) race on it: order them on one stream or with
// events.  The split kernel writes every byte the GEMM later reads, so nothing has to
// start at zero and nothing carries over from the previous call.
// ===========================================================================
namespace tsb {
namespace gemm {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch for each device, resolved once with that device
// current (the host-side name of a __device__ array is not a device address).
static void* g_noalloc_addr[64] = {};
static std::mutex g_noalloc_mutex;

static int noalloc_scratch(uint8_t** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return kNoDevice;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return kLaunchFailed;
    }
    g_noalloc_addr[dev] = p;
  }
  *out = static_cast<uint8_t*>(g_noalloc_addr[dev]);
  return kOk;
}

}  // namespace gemm
}  // namespace tsb

extern "C" {

// No counterpart in the reference.  Same arguments and results as
// triposplat_gemm_rnf8_avx512; allocates no memory (see the block comment above).
// Additional status: -6 when the split activations (see above) exceed the 32 MiB scratch;
// -4 when N % 16 != 0 or a code pointer is not 16-byte aligned (this entry has only the
// tensor-core path).  The first call on each device resolves the scratch address; make
// that first call before capturing any stream.
int triposplat_gemm_nf24_noalloc(const float* x, const uint8_t* codes0_t, const uint8_t* codes1_t,
                                 const uint8_t* codes2_t, const float* scales0,
                                 const float* scales1, const float* scales2,
                                 const float* codebook, const float* bias, float* out, int M,
                                 int K, int N, int stride_x, int stride_out, int threads,
                                 int stages) {
  using namespace tsb;
  using namespace tsb::gemm;
  (void)threads;
  if (!x || !codes0_t || !codes1_t || !codes2_t || !scales0 || !scales1 || !scales2 ||
      !codebook || !bias || !out)
    return kNullPointer;
  if (M <= 0 || K <= 0 || N <= 0 || stages != 3) return kBadDims;
  if (stride_x < K || stride_out < N) return kBadRange;
  const int16_t* c01 = reinterpret_cast<const int16_t*>(codes0_t);
  const int8_t* q2 = reinterpret_cast<const int8_t*>(codes1_t);
  if ((N % 16) != 0 || (stride_out % 4) != 0 ||
      ((reinterpret_cast<uintptr_t>(c01) | reinterpret_cast<uintptr_t>(q2) |
        reinterpret_cast<uintptr_t>(out)) & 15) != 0)
    return kBadAlignment;
  if (split_bytes(M, K) > kNoAllocScratchBytes) return -6;
  int st = entry_check_no_alloc();
  if (st != kOk) return st;
  if (!is_device_pointer(x) || !is_device_pointer(c01) || !is_device_pointer(q2) ||
      !is_device_pointer(scales0) || !is_device_pointer(bias) || !is_device_pointer(out))
    return kNotDevicePointer;
  uint8_t* ws = nullptr;
  if ((st = noalloc_scratch(&ws)) != kOk) return st;
  int* status = device_status_no_alloc();  // first call on a device: maps the status word
  if (status == nullptr) return kLaunchFailed;
  cudaStream_t stream = current_stream();
  const SplitPlanes sp = split_layout(ws, M, K);
  if ((st = launch_split(x, stride_x, sp, stream)) != kOk) return st;
  return launch_tc(sp, c01, q2, scales0, bias, out, N, 0, N, stride_out, EpilogueArgs(), status,
                   stream);
}

}  // extern "C"

// ===========================================================================
// The reference's fused NF24 entry points: the MLP (fc1 -> GELU(tanh) -> fc2,
// scripts/native_nf24_mlp_avx512.c:143-205 and the chunked variant
// scripts/native_nf24_mlp_chunked_avx512.c:3-60) and the QKV projection with its
// RoPE / RMSNorm / pack epilogue (scripts/gemm_nf24_qkv_direct_avx512.c:87-199).
// Same names, argument lists and status codes.  On the GPU the CPU's per-row-tile
// fusion (a hidden tile kept in cache) is not the win: each stage is one persistent
// tensor-core launch over all rows, and the intermediate (hidden [M, H] or qkv [M, N])
// lives in the library workspace -- or, for the chunked MLP, in the caller's hidden
// buffer -- between launches.
// ===========================================================================
extern "C" int triposplat_qkv_rope_rmsnorm_pack_f32_avx512_v2(
    const float* qkv, const float* frequencies, const float* q_gamma, const float* k_gamma,
    float* q_bhld, float* packed_k, float* packed_v, int B, int L, int H, int D, int L_padded,
    int frequency_batches, int threads);
extern "C" int triposplat_gelu_tanh_f32_avx512(const float* input, float* output, int64_t count,
                                               int threads);

namespace tsb {

constexpr int kMlpIn = 1024, kMlpHidden = 4096, kMlpOut = 1024;  // native_nf24_mlp_avx512.c:9-15

// One NF24 Linear of fp32 rows x [M, K] (row stride stride_x) into out [M, N] (row stride
// stride_out), optionally GELU(tanh) applied to the result.  Tensor-core path through the
// split planes at split_ws (split_bytes(M, K) bytes) when the code planes and the output
// allow TMA; otherwise the SIMT kernel (then GELU as a separate pass, which needs a
// contiguous output).
static bool linear_rows_tc(const int16_t* c01, const int8_t* q2, const float* out, int N,
                           int stride_out) {
  return (N % 16) == 0 && (stride_out % 4) == 0 &&
         ((reinterpret_cast<uintptr_t>(c01) | reinterpret_cast<uintptr_t>(q2) |
           reinterpret_cast<uintptr_t>(out)) & 15) == 0;
}
static int linear_rows(const float* x, int stride_x, int M, int K, const int16_t* c01,
                       const int8_t* q2, const float* scale, const float* bias, float* out, int N,
                       int stride_out, bool gelu, uint8_t* split_ws, cudaStream_t stream,
                       const NkCodes* nk = nullptr) {
  using namespace gemm;
  int st;
  if (linear_rows_tc(c01, q2, out, N, stride_out)) {
    const SplitPlanes sp = split_layout(split_ws, M, K);
    if ((st = launch_split(x, stride_x, sp, stream)) != kOk) return st;
    EpilogueArgs ep;
    ep.mode = gelu ? kGelu : kStore;
    if (nk)  // the weight's k-contiguous copy (one k-block per partial: the same bits)
      return launch_tc(sp, nk->c01, nk->q2, scale, bias, out, N, 0, N, stride_out, ep,
                       device_status(), stream, nk->ldk, true);
    return launch_tc(sp, c01, q2, scale, bias, out, N, 0, N, stride_out, ep, device_status(),
                     stream);
  }
  if (gelu && stride_out != N) return kBadAlignment;
  {
    dim3 grid((N + 127) / 128, M);
    LaunchScope scope(kKGemmSimt, stream);
    nf24_gemm_simt<<<grid, 128, 0, stream>>>(x, c01, q2, scale, bias, out, M, K, N, 0, N,
                                             stride_x, stride_out);
  }
  if ((st = launch_status()) != kOk || !gelu) return st;
  return triposplat_gelu_tanh_f32_avx512(out, out, (int64_t)M * N, 0);
}

// fc1 -> GELU -> fc2 over `rows` rows; hidden [rows, H] contiguous; workspace split planes
// for the fc1 input and the fc2 input.
static int mlp_rows(const float* x, int stride_x, int rows, const int16_t* w1c, const int8_t* w1q,
                    const float* w1s, const float* w1b, const int16_t* w2c, const int8_t* w2q,
                    const float* w2s, const float* w2b, float* hidden, float* out, int stride_out,
                    uint8_t* split_x, uint8_t* split_h, cudaStream_t stream,
                    const NkCodes* nk1 = nullptr, const NkCodes* nk2 = nullptr) {
  int st = linear_rows(x, stride_x, rows, kMlpIn, w1c, w1q, w1s, w1b, hidden, kMlpHidden,
                       kMlpHidden, true, split_x, stream, nk1);
  if (st != kOk) return st;
  return linear_rows(hidden, kMlpHidden, rows, kMlpHidden, w2c, w2q, w2s, w2b, out, kMlpOut,
                     stride_out, false, split_h, stream, nk2);
}

// From kNkMinRows rows on, the MLP's two weights are copied into k-contiguous planes once
// per call (after `off` bytes of the workspace); nk1 / nk2 stay empty otherwise or where a
// stage takes the scalar kernel.
static int mlp_nk_codes(int M, const int16_t* w1c, const int8_t* w1q, const int16_t* w2c,
                        const int8_t* w2q, const float* hidden, const float* out, int stride_out,
                        uint8_t* ws, size_t off, cudaStream_t stream, NkCodes& nk1, NkCodes& nk2,
                        bool& use1, bool& use2) {
  use1 = use2 = false;
  if (M < kNkMinRows) return kOk;
  int st;
  if (linear_rows_tc(w1c, w1q, hidden, kMlpHidden, kMlpHidden)) {
    if ((st = copy_codes_nk(w1c, w1q, kMlpIn, kMlpHidden, 0, kMlpHidden, ws + off, stream, nk1)) != kOk)
      return st;
    use1 = true;
  }
  if (linear_rows_tc(w2c, w2q, out, kMlpOut, stride_out)) {
    if ((st = copy_codes_nk(w2c, w2q, kMlpHidden, kMlpOut, 0, kMlpOut,
                            ws + off + nk_codes_bytes(kMlpIn, kMlpHidden), stream, nk2)) != kOk)
      return st;
    use2 = true;
  }
  return kOk;
}
static size_t mlp_nk_bytes(int M) {
  return M < kNkMinRows ? 0 : nk_codes_bytes(kMlpIn, kMlpHidden) + nk_codes_bytes(kMlpHidden, kMlpOut);
}

static bool all_device_pointers(const void* const* p, int n) {
  for (int i = 0; i < n; ++i)
    if (!is_device_pointer(p[i])) return false;
  return true;
}

}  // namespace tsb

extern "C" {

// scripts/native_nf24_mlp_avx512.c:143-205: out = GELU_tanh(x W1 + b1) W2 + b2 for
// K = 1024, H = 4096, N = 1024 (the reference's fixed sizes and checks: -1 null, -2 sizes
// or strides).  The hidden activations live in the library workspace (M x 4096 floats).
int triposplat_mlp_nf24_gelu_f32_avx512(const float* x, const uint8_t* w1_code01_t,
                                        const uint8_t* w1_code2_t, const float* w1_scales,
                                        const float* w1_bias, const uint8_t* w2_code01_t,
                                        const uint8_t* w2_code2_t, const float* w2_scales,
                                        const float* w2_bias, float* out, int M, int K, int H,
                                        int N, int stride_x, int stride_out, int threads) {
  using namespace tsb;
  (void)threads;
  if (!x || !w1_code01_t || !w1_code2_t || !w1_scales || !w1_bias || !w2_code01_t ||
      !w2_code2_t || !w2_scales || !w2_bias || !out)
    return kNullPointer;
  if (M <= 0 || K != kMlpIn || H != kMlpHidden || N != kMlpOut || stride_x < K ||
      stride_out < N)
    return kBadDims;
  int st = entry_check();
  if (st != kOk) return st;
  const void* ptrs[] = {x, w1_code01_t, w1_code2_t, w1_scales, w1_bias, w2_code01_t,
                        w2_code2_t, w2_scales, w2_bias, out};
  if (!all_device_pointers(ptrs, 10)) return kNotDevicePointer;
  cudaStream_t stream = current_stream();
  const size_t sx = align256(split_bytes(M, K)), hb = align256((size_t)M * H * 4);
  const size_t sh = align256(split_bytes(M, H));
  uint8_t* ws = static_cast<uint8_t*>(workspace(sx + hb + sh + mlp_nk_bytes(M), stream));
  if (!ws) return kWorkspace;
  const auto* w1c = reinterpret_cast<const int16_t*>(w1_code01_t);
  const auto* w1q = reinterpret_cast<const int8_t*>(w1_code2_t);
  const auto* w2c = reinterpret_cast<const int16_t*>(w2_code01_t);
  const auto* w2q = reinterpret_cast<const int8_t*>(w2_code2_t);
  float* hidden = reinterpret_cast<float*>(ws + sx);
  NkCodes nk1, nk2;
  bool u1, u2;
  if ((st = mlp_nk_codes(M, w1c, w1q, w2c, w2q, hidden, out, stride_out, ws, sx + hb + sh, stream,
                         nk1, nk2, u1, u2)) != kOk)
    return st;
  return mlp_rows(x, stride_x, M, w1c, w1q, w1_scales, w1_bias, w2c, w2q, w2_scales, w2_bias,
                  hidden, out, stride_out, ws, ws + sx + hb, stream, u1 ? &nk1 : nullptr,
                  u2 ? &nk2 : nullptr);
}

// scripts/native_nf24_mlp_chunked_avx512.c:3-60: the same MLP over chunks of chunk_rows
// rows, the hidden activations of a chunk in the caller's buffer hidden
// [hidden_capacity_rows, H] (device memory); -2 also for chunk_rows <= 0 or
// hidden_capacity_rows < chunk_rows.
int triposplat_mlp_nf24_gelu_chunked_f32_avx512(
    const float* x, const uint8_t* w1_code01_t, const uint8_t* w1_code2_t,
    const float* w1_scales, const float* w1_bias, const uint8_t* w2_code01_t,
    const uint8_t* w2_code2_t, const float* w2_scales, const float* w2_bias, float* hidden,
    float* out, int M, int K, int H, int N, int stride_x, int stride_out,
    int hidden_capacity_rows, int chunk_rows, int threads) {
  using namespace tsb;
  (void)threads;
  if (!x || !w1_code01_t || !w1_code2_t || !w1_scales || !w1_bias || !w2_code01_t ||
      !w2_code2_t || !w2_scales || !w2_bias || !hidden || !out)
    return kNullPointer;
  if (M <= 0 || K != kMlpIn || H != kMlpHidden || N != kMlpOut || stride_x < K ||
      stride_out < N || chunk_rows <= 0 || hidden_capacity_rows < chunk_rows)
    return kBadDims;
  int st = entry_check();
  if (st != kOk) return st;
  const void* ptrs[] = {x, w1_code01_t, w1_code2_t, w1_scales, w1_bias, w2_code01_t,
                        w2_code2_t, w2_scales, w2_bias, hidden, out};
  if (!all_device_pointers(ptrs, 11)) return kNotDevicePointer;
  cudaStream_t stream = current_stream();
  const int cr = chunk_rows < M ? chunk_rows : M;
  const size_t sx = align256(split_bytes(cr, K)), sh = align256(split_bytes(cr, H));
  // the k-contiguous copies (from kNkMinRows rows in total) serve every chunk
  uint8_t* ws = static_cast<uint8_t*>(workspace(sx + sh + mlp_nk_bytes(M), stream));
  if (!ws) return kWorkspace;
  const auto* w1c = reinterpret_cast<const int16_t*>(w1_code01_t);
  const auto* w1q = reinterpret_cast<const int8_t*>(w1_code2_t);
  const auto* w2c = reinterpret_cast<const int16_t*>(w2_code01_t);
  const auto* w2q = reinterpret_cast<const int8_t*>(w2_code2_t);
  NkCodes nk1, nk2;
  bool u1, u2;
  if ((st = mlp_nk_codes(M, w1c, w1q, w2c, w2q, hidden, out, stride_out, ws, sx + sh, stream, nk1,
                         nk2, u1, u2)) != kOk)
    return st;
  for (int start = 0; start < M; start += cr) {
    const int rows = start + cr <= M ? cr : M - start;
    st = mlp_rows(x + (int64_t)start * stride_x, stride_x, rows, w1c, w1q, w1_scales, w1_bias,
                  w2c, w2q, w2_scales, w2_bias, hidden, out + (int64_t)start * stride_out,
                  stride_out, ws, ws + sx, stream, u1 ? &nk1 : nullptr, u2 ? &nk2 : nullptr);
    if (st != kOk) return st;
  }
  return kOk;
}

// scripts/native_nf24_mlp_avx512.c:207-213
int triposplat_mlp_nf24_row_tile(void) { return tsb::gemm::BM; }
int triposplat_mlp_nf24_hidden_workspace_bytes_per_thread(void) {
  return tsb::gemm::BM * tsb::kMlpHidden * (int)sizeof(float);  // one row tile's hidden rows
}

// scripts/gemm_nf24_qkv_direct_avx512.c:87-199: qkv = x W + b (x [B*L, K] contiguous,
// W [K, N = 3*H*64]) followed by the RoPE / per-head RMSNorm / pack of
// triposplat_qkv_rope_rmsnorm_pack_f32_avx512_v2: q_bhld [B, H, L, 64], packed_k / packed_v
// [B, H, 64, L_padded] with a zero tail.  Status codes as the reference (-1 null; -2 sizes,
// N != 3*H*D, D != 64, L_padded < L or % 16, frequency_batches not 1 or B, stages != 3).
// qkv [B*L, N] lives in the library workspace between the two launches.
int triposplat_gemm_nf24_qkv_rope_rmsnorm_pack_f32_avx512(
    const float* x, const uint8_t* codes0_t, const uint8_t* codes1_t, const uint8_t* codes2_t,
    const float* scales0, const float* scales1, const float* scales2, const float* codebook,
    const float* bias, const float* frequencies, const float* q_gamma, const float* k_gamma,
    float* q_bhld, float* packed_k, float* packed_v, int B, int L, int K, int N, int H, int D,
    int L_padded, int frequency_batches, int threads, int stages) {
  using namespace tsb;
  (void)threads;
  if (!x || !codes0_t || !codes1_t || !codes2_t || !scales0 || !scales1 || !scales2 ||
      !codebook || !bias || !frequencies || !q_gamma || !k_gamma || !q_bhld || !packed_k ||
      !packed_v)
    return kNullPointer;
  if (B <= 0 || L <= 0 || K <= 0 || H <= 0 || D != 64 || (int64_t)N != 3LL * H * D ||
      L_padded < L || (L_padded & 15) != 0 || (frequency_batches != 1 && frequency_batches != B) ||
      stages != 3 || (int64_t)B * L > 0x7fffffffLL)
    return kBadDims;
  int st = entry_check();
  if (st != kOk) return st;
  const void* ptrs[] = {x, codes0_t, codes1_t, scales0, bias, frequencies, q_gamma, k_gamma,
                        q_bhld, packed_k, packed_v};
  if (!all_device_pointers(ptrs, 11)) return kNotDevicePointer;
  cudaStream_t stream = current_stream();
  const int M = B * L;
  const size_t qb = align256((size_t)M * N * 4), sx = align256(split_bytes(M, K));
  const auto* c01 = reinterpret_cast<const int16_t*>(codes0_t);
  const auto* q2 = reinterpret_cast<const int8_t*>(codes1_t);
  float* qkv = nullptr;
  // from kNkMinRows rows on, the projection reads a k-contiguous copy of its codes
  // (qkv itself is 256-byte aligned in the workspace, its rows N = 3 * H * 64 floats)
  const bool use_nk = M >= kNkMinRows &&
                      ((reinterpret_cast<uintptr_t>(c01) | reinterpret_cast<uintptr_t>(q2)) & 15) == 0;
  uint8_t* ws = static_cast<uint8_t*>(
      workspace(qb + sx + (use_nk ? nk_codes_bytes(K, N) : 0), stream));
  if (!ws) return kWorkspace;
  qkv = reinterpret_cast<float*>(ws);
  NkCodes nk;
  if (use_nk && (st = copy_codes_nk(c01, q2, K, N, 0, N, ws + qb + sx, stream, nk)) != kOk) return st;
  st = linear_rows(x, K, M, K, c01, q2, scales0, bias, qkv, N, N, false, ws + qb, stream,
                   use_nk ? &nk : nullptr);
  if (st != kOk) return st;
  return triposplat_qkv_rope_rmsnorm_pack_f32_avx512_v2(qkv, frequencies, q_gamma, k_gamma, q_bhld,
                                                        packed_k, packed_v, B, L, H, D, L_padded,
                                                        frequency_batches, 0);
}

// scripts/gemm_nf24_qkv_direct_avx512.c:201-207 and gemm_nf24_qkv_direct_tile_avx512.c:149-151
int triposplat_gemm_nf24_qkv_direct_row_tile(void) { return tsb::gemm::BM; }
int triposplat_gemm_nf24_qkv_direct_residual_mode(void) { return 4; }
int triposplat_gemm_nf24_qkv_direct_tile_bytes(void) {
  return tsb::gemm::BM * 3072 * (int)sizeof(float);  // one row tile of the 3072-wide qkv
}

}  // extern "C"
