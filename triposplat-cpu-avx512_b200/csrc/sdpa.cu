// Exact scaled-dot-product attention for sm_100a, head_dim 64, scale 1/8:
//   O = softmax(0.125 * Q K^T + bias_key) V
// (reference scripts/native_sdpa_avx512_exact_q8t512.c:137-332; packed-K/V, BLHD-output
// variant scripts/native_sdpa_avx512_exact_q8t512_packed.c:3-158).
//
// Split precision.  fp32 inputs are split into two fp16 planes (hi + lo, ~22 significant
// bits) after an exact power-of-two pre-scale (per query row for Q; per 128-key tile for
// K and V), and each product is formed with three tensor-core passes
// (hi.hi + hi.lo + lo.hi; the lo.lo term is ~2^-22 relative and dropped):
//   S = Qh Kh^T + Qh Kl^T + Ql Kh^T                (tcgen05, Q and K from shared memory)
//   O_t = Ph Vh + Ph Vl + Pl Vh                     (tcgen05, P from tensor memory)
// The pre-scales fold into constants the softmax already multiplies by, so they are free.
//
// Exact online softmax.  Keys are processed in tiles of 128, each read once from tensor
// memory in four 32-key chunks.  Every chunk's max is checked against a running reference
// max m before its p = 2^(s*log2e - m) are formed; m is raised (to an integer, so the
// factor applied to what was accumulated is an exact power of two) only when a chunk
// exceeds it by more than 8, which after the first chunk of a row is rare: the result is
// the same exact softmax (the common factor cancels in O/l) and p stays <= 2^8.  P is
// formed as p * 2^7 (<= 2^15, inside fp16 range, and small terms stay out of fp16's
// subnormal range), split into fp16 hi/lo in registers and written over S in tensor
// memory.  Each tile's P.V goes into a FRESH TMEM
// accumulator O_t that the softmax warps add into fp32 registers before the next P.V: the
// tensor core's fp32 accumulation truncates, and one accumulator carried over all tiles
// drifts linearly with the key count (measured: 3e-5 relative rmse at 8192 keys, 60x the
// fp32 reference), while 24 accumulation steps per tile stay at the reference's level.
// The V tiles' power-of-two pre-scales are made relative to the largest one of the head
// and folded into the exponent of p; the row sum l is kept in fp32.  No Lq x Lk matrix is
// ever materialised and no score is skipped.
//
// Two softmax teams split the key tiles of a row (split-K): team 0 takes the even tiles,
// team 1 the odd ones, each with its own reference max, row sum and fp32 O accumulators;
// at the end the two partial softmaxes are merged with exact power-of-two factors (both
// references are integers).  The teams' phases interleave on the SM's pipes, and the
// scores of a team's next tile are computed while it works on the current one.
//
// CTA: one (b, h) and 128 query rows, 384 threads, one CTA per SM.
//   warp 0 / 2  TMA producers of the K / V^T tiles (two stages each)
//   warp 1      TMEM allocator + QK^T issuer;  warp 3  P.V issuer (separate threads, so a
//               team's next QK never waits behind the other team's P)
//   warps 4..7  softmax team 0, warps 8..11 team 1; thread = query row = TMEM lane.  The
//               teams also write the Q tile (hi / lo plane) into shared memory.
// TMEM (512 columns): three S / P buffers (tile t uses buffer t % 3; P overwrites S in
// place: for every 16-key chunk, P_hi goes to its first 8 columns and P_lo to the next 8),
// then O of team 0 and O of team 1 (64 columns each).
// Ordering: QK(t) waits only for P.V(t-3), the last reader of its buffer; P.V(t) writes
// team (t & 1)'s O only after that team folded its previous O into registers (p_full).
//
// Output: fp32 (BHLD or BLHD), or straight into the NF24 GEMM's split format for the
// out-projection ([B*Lq, H*64] fp16 hi / lo planes + one power-of-two scale per row).  A
// row's scale must be known before any of its heads is written, and O is a convex
// combination of V rows, so |O| <= max |V| over the batch's keys and heads
// < 2^15 * (largest inverse V-tile pre-scale of the batch): that bound fixes the scale
// (value * 2^s < 2^15), and the planes equal the split of the fp32 output under it.  Either
// way the teams merge their halves through shared memory and the item's 128 x 64 output is
// staged there and written in row order (16 threads per row), not as a 128-byte piece per
// thread.
#include <cuda_fp16.h>

#include <atomic>

#include "common.cuh"
#include "runtime.h"

namespace tsb {
namespace sdpa {

constexpr int D = 64;
constexpr int BQ = 128;
constexpr int BKV = 128;
constexpr int NUM_THREADS = 384;
// Register budget: 384 threads x 168 registers at launch (one CTA per SM; the host checks
// the compiled count).  Warpgroup 0 (TMA producers, MMA issuers) drops to 56 and each
// softmax team rises to 224: 56 + 2 x 224 = 504 = 3 x 168.
constexpr uint32_t REGS_LAUNCH = 168;
constexpr uint32_t REGS_CONTROL = 56;
constexpr uint32_t REGS_SOFTMAX = 224;
static_assert(REGS_LAUNCH * NUM_THREADS <= 65536, "launch allocation");
static_assert((REGS_CONTROL + 2 * REGS_SOFTMAX) * 128 <= REGS_LAUNCH * NUM_THREADS, "register split");
constexpr int TMEM_COLS = 512;
constexpr int NSB = 3;                  // score / P buffers: tile t uses S_COL + (t % 3) * BKV
constexpr int S_COL = 0;
constexpr int O_COL = NSB * BKV;        // 384: O of team 0, then O of team 1 (64 columns each)
static_assert(O_COL + 2 * D <= TMEM_COLS, "TMEM budget");
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units
constexpr float P_LIFT = 7.0f;  // p' = p * 2^7 <= 2^15 < fp16 max
constexpr int PLANE = 128 * D * 2;      // 16 KB: one 128 x 64 fp16 tile
constexpr int STAGE = 2 * PLANE;        // hi + lo planes of one Q, K or V^T tile
// Q, 2 K stages, 2 V stages, per-warp bias [8][BKV], team 0's maxima / sums [BQ] each (two
// arrays of 2 * BQ), the exchange / output tile [BQ][OUT_PITCH], V-scale shares [8], barriers.
// Rows of the tile are padded to 68 floats: the eight threads of a quarter warp (eight rows)
// then reach eight different 4-bank groups with their float4 accesses (a 64-float pitch would
// put them all on the same banks).  Team 0 writes its partial rows there, team 1 merges each
// row in place and then the whole tile goes out in row order, 16 threads per 256-byte row.
constexpr int OUT_PITCH = 68;
constexpr int SMEM_BYTES = 1024 + 5 * STAGE + 8 * BKV * 4 + 4 * BQ * 4 + BQ * OUT_PITCH * 4 + 8 * 4 +
                           32 * 8 + 16;
constexpr float LOG2E = 1.4426950408889634f;

struct Params {
  const float* qinv;  // [BH * Lq]   inverse pre-scale of each query row
  const float* kinv;  // [BH * T]    inverse pre-scale of each key tile
  const float* vinv;  // [BH * T]
  const float* bias;  // nullable; bias for (bh, key j) = bias[bh * bias_bh_stride + j]
  long long bias_bh_stride;
  float* out;
  int H, Lq, Lk, T;
  int out_blhd;
  int* status;
  int Qt, BH;  // query tiles per head, heads x batch: work item j = (bh = j / Qt, tile j % Qt)
  // nullable: O written as the split planes [B*Lq, H*64] with row scales ors (BLHD rows)
  __half* ohi;
  __half* olo;
  float* ors;
};

// 2^s for |s| <= 126 built in the exponent field: x * pow2i(s) is the correctly rounded
// x * 2^s (what ldexpf computes) for a fraction of its instructions
__device__ __forceinline__ float pow2i(int s) { return __int_as_float((127 + s) << 23); }

// s with mx * 2^s in [2^14, 2^15) (clamped to [-60, 60]; 0 for 0 / non-finite)
__device__ __forceinline__ int pow2_shift(float mx) {
  if (!(mx > 0.0f) || !(mx <= 3.402823466e38f)) return 0;
  int s = 14 - ilogbf(mx);
  return s < -60 ? -60 : (s > 60 ? 60 : s);
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// max over 32 values (16 three-input max instructions)
__device__ __forceinline__ float max32(const float (&v)[32]) {
  float a[11];
#pragma unroll
  for (int i = 0; i < 10; ++i) a[i] = max3(v[3 * i], v[3 * i + 1], v[3 * i + 2]);
  a[10] = fmaxf(v[30], v[31]);
  const float b0 = max3(a[0], a[1], a[2]), b1 = max3(a[3], a[4], a[5]), b2 = max3(a[6], a[7], a[8]);
  return max3(max3(b0, b1, b2), a[9], a[10]);
}

// Max over one 32-key chunk, in log2 units (x = s*c2 (+ bias)).
template <bool PLAIN>
__device__ __forceinline__ float chunk_max(const uint32_t (&s)[32], const float* bt, float c2) {
  float x[32];
#pragma unroll
  for (int j = 0; j < 32; ++j)
    x[j] = PLAIN ? __uint_as_float(s[j]) : fmaf(__uint_as_float(s[j]), c2, bt[j]);
  const float m = max32(x);
  return PLAIN ? m * c2 : m;  // c2 >= 0
}

// Packed fp32x2 arithmetic (one instruction for two lanes of fp32 work).
__device__ __forceinline__ uint64_t f2pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// 2^x on the FMA pipe for a pair of values (the MUFU pipe that ex2 uses is shared by both
// softmax teams of an SM).  Range reduction x = j + f, j = round-to-nearest(x) by the
// 1.5 * 2^23 addition, f in [-1/2, 1/2]; 2^f by a degree-5 polynomial whose coefficients
// minimise the maximum relative error on [-1/2, 1/2] (Remez exchange, computed by
// csrc/gen_exp2_poly.py: 2.1e-7 in float32 Horner, the order of ex2.approx); 2^j added to
// the exponent field.  x is clamped at -125 so the result stays a normal float (ex2 gives
// 0 below -126; both are far below what the fp16 P planes keep).
// Measured on config 2(a) (B2 H16 L8192, same build): no pairs on the FMA pipe 1.363 ms,
// a quarter (0x88) 1.445 ms, half (0xAA) 1.572 ms -- the softmax is bound by its dependency
// chain, not by MUFU throughput, and the polynomial's extra instructions lengthen it; so by
// default every exponential stays on ex2.
#ifndef TSB_POLY_PAIRS
#define TSB_POLY_PAIRS 0x00u  // of each 16-key chunk's 8 pairs, these go to the FMA pipe
#endif
constexpr uint32_t kPolyPairs = TSB_POLY_PAIRS;
__device__ __forceinline__ void exp2_poly2(float x0, float x1, float& p0, float& p1) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  x0 = fmaxf(x0, -125.0f);
  x1 = fmaxf(x1, -125.0f);
  const uint64_t xm = f2pack(x0, x1);
  const uint64_t t = f2add(xm, f2pack(kMagic, kMagic));            // 1.5 * 2^23 + j
  const uint64_t f = f2sub(xm, f2sub(t, f2pack(kMagic, kMagic)));  // x - j
  uint64_t r = f2pack(0x1.5c08e6p-10f, 0x1.5c08e6p-10f);
  r = f2fma(r, f, f2pack(0x1.3d0c52p-7f, 0x1.3d0c52p-7f));
  r = f2fma(r, f, f2pack(0x1.c6b6e4p-5f, 0x1.c6b6e4p-5f));
  r = f2fma(r, f, f2pack(0x1.ebf918p-3f, 0x1.ebf918p-3f));
  r = f2fma(r, f, f2pack(0x1.62e428p-1f, 0x1.62e428p-1f));
  r = f2fma(r, f, f2pack(0x1.000002p+0f, 0x1.000002p+0f));
  float r0, r1, t0, t1;
  f2unpack(r, r0, r1);
  f2unpack(t, t0, t1);
  // the low bits of t hold j (two's complement); j << 23 lands on the exponent field
  p0 = __uint_as_float(__float_as_uint(r0) + (__float_as_uint(t0) << 23));
  p1 = __uint_as_float(__float_as_uint(r1) + (__float_as_uint(t1) << 23));
}

// p = 2^(s*c2 (+ bias) + nm) for one 16-key chunk (s[0..15]): two packed partial row sums,
// fp16 hi/lo split, written over the chunk's scores in tensor memory (8 columns P_hi,
// 8 columns P_lo).  The pairs of kPolyPairs take 2^x from exp2_poly2, the others from ex2.
template <bool PLAIN>
__device__ __forceinline__ void chunk_exp_store(const uint32_t* s, const float* bt, uint64_t c2x2,
                                                uint64_t nmx2, uint64_t (&ps)[2], uint32_t taddr) {
  uint32_t pk[16];
#pragma unroll
  for (int j = 0; j < 16; j += 2) {
    const uint64_t sx = f2pack(__uint_as_float(s[j]), __uint_as_float(s[j + 1]));
    const uint64_t off = PLAIN ? nmx2 : f2add(f2pack(bt[j], bt[j + 1]), nmx2);
    float x0, x1;
    f2unpack(f2fma(sx, c2x2, off), x0, x1);
    float p0, p1;
    if ((kPolyPairs >> (j >> 1)) & 1u) {
      exp2_poly2(x0, x1, p0, p1);
    } else {
      p0 = ex2(x0);
      p1 = ex2(x1);
    }
    const uint64_t px = f2pack(p0, p1);
    ps[(j >> 1) & 1] = f2add(ps[(j >> 1) & 1], px);
    // hi: p with the 13 low mantissa bits cleared (exact in fp16 for p >= 2^-14),
    // lo: the exact fp32 remainder
    const float h0 = __uint_as_float(__float_as_uint(p0) & 0xFFFFE000u);
    const float h1 = __uint_as_float(__float_as_uint(p1) & 0xFFFFE000u);
    float l0, l1;
    f2unpack(f2sub(px, f2pack(h0, h1)), l0, l1);
    const __half2 hh = __floats2half2_rn(h0, h1);
    const __half2 ll = __floats2half2_rn(l0, l1);
    pk[j >> 1] = *reinterpret_cast<const uint32_t*>(&hh);
    pk[8 + (j >> 1)] = *reinterpret_cast<const uint32_t*>(&ll);
  }
  tmem_st16(taddr, pk);
}

// Raise this row's reference max where the 32-key chunk C exceeds it by more than the
// threshold (warp-uniform: the caller votes).  The new reference is an integer, so the
// factor alpha = 2^(m_old - m_new) is an exact power of two and the accumulators, the
// partial row sums and the P chunks already written for this tile (fp16 hi/lo, rescaled
// in tensor memory) all keep exactly the values they would have had with m_new from the
// start, up to fp16 rounding of terms that fall below 2^-14 (subnormal).
template <int C>
__device__ __forceinline__ void raise_reference(uint32_t srow, float cm, float& m_run, float& l_run,
                                                uint64_t (&ps)[2], float (&o_acc)[D]) {
  const float m_new = cm > m_run + RESCALE_THRESHOLD ? ceilf(cm) : m_run;
  const float alpha = m_new == m_run ? 1.0f : ex2(m_run - m_new);  // 0 when m_run = -inf
#pragma unroll
  for (int d = 0; d < D; ++d) o_acc[d] *= alpha;
  l_run *= alpha;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    float a, b;
    f2unpack(ps[i], a, b);
    ps[i] = f2pack(a * alpha, b * alpha);
  }
  if (C > 0) {
    const __half2 a2 = __float2half2_rn(alpha);
    tmem_wait_st();  // the chunks below were stored asynchronously
#pragma unroll 1
    for (int c = 0; c < 2 * C; ++c) {
      uint32_t pv[16];
      tmem_ld16(srow + c * 16, pv);
      tmem_wait_ld();
      reg_fence(pv);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const __half2 h = __hmul2(*reinterpret_cast<const __half2*>(&pv[j]), a2);
        pv[j] = *reinterpret_cast<const uint32_t*>(&h);
      }
      tmem_st16(srow + c * 16, pv);
    }
  }
  m_run = m_new;
}

// One 32-key chunk: issue the next chunk's load, check the chunk max against the
// reference, form p and P.  `cur` holds this chunk's scores; `nxt` receives chunk C+1.
template <bool PLAIN, int C>
__device__ __forceinline__ void softmax_chunk(uint32_t srow, const uint32_t (&cur)[32],
                                              uint32_t (&nxt)[32], const float* bt, float c2,
                                              float vshift, float& m_run, float& l_run,
                                              uint64_t (&ps)[2], float (&o_acc)[D]) {
  if (C < 3) tmem_ld32(srow + (C + 1) * 32, nxt);
  const float cm = chunk_max<PLAIN>(cur, bt + C * 32, c2);
  if (__any_sync(0xffffffffu, cm > m_run + RESCALE_THRESHOLD))
    raise_reference<C>(srow, cm, m_run, l_run, ps, o_acc);
  // p' = 2^(x - m + 7 + vshift): p' <= 2^15 keeps P in fp16's range while lifting small
  // terms out of fp16's subnormal range (the 2^7 cancels in O / l)
  const float nm = vshift + P_LIFT - (m_run == -INFINITY ? 0.0f : m_run);
  const uint64_t c2x2 = f2pack(c2, c2), nmx2 = f2pack(nm, nm);
  chunk_exp_store<PLAIN>(cur, bt + C * 32, c2x2, nmx2, ps, srow + C * 32);
  chunk_exp_store<PLAIN>(cur + 16, bt + C * 32 + 16, c2x2, nmx2, ps, srow + C * 32 + 16);
  if (C < 3) {
    tmem_wait_ld();
    reg_fence(nxt);
  }
}

// One key tile of the softmax warps, after S(t) is in tensor memory and O_{t-1} complete.
// Single pass over the scores: each 32-key chunk is checked against the running
// reference max before its p are formed (the reference is raised, rarely, by
// raise_reference), and each chunk's tensor-memory load is issued before the previous
// chunk is processed, so one load latency is exposed per tile.
template <bool PLAIN>
__device__ __forceinline__ void softmax_tile(uint32_t srow, uint32_t orow, bool merge_o, const float* bt, float c2,
                                             float vshift, float& m_run, float& l_run,
                                             float (&o_acc)[D]) {
  uint32_t sa[32], sb[32];
  if (merge_o) {
    // O_{t-1} (relative to the current reference max) into the fp32 accumulators, loaded
    // together with the first score chunk
    uint32_t o0[32], o1[32];
    tmem_ld32(orow, o0);
    tmem_ld32(orow + 32, o1);
    tmem_ld32(srow, sa);
    tmem_wait_ld();
    reg_fence(o0);
    reg_fence(o1);
#pragma unroll
    for (int d = 0; d < 32; d += 2) {
      f2unpack(f2add(f2pack(o_acc[d], o_acc[d + 1]), f2pack(__uint_as_float(o0[d]), __uint_as_float(o0[d + 1]))),
               o_acc[d], o_acc[d + 1]);
      f2unpack(f2add(f2pack(o_acc[32 + d], o_acc[33 + d]), f2pack(__uint_as_float(o1[d]), __uint_as_float(o1[d + 1]))),
               o_acc[32 + d], o_acc[33 + d]);
    }
  } else {
    tmem_ld32(srow, sa);
    tmem_wait_ld();
  }
  reg_fence(sa);
  uint64_t ps[2] = {0ull, 0ull};  // packed (+0.0f, +0.0f)
  softmax_chunk<PLAIN, 0>(srow, sa, sb, bt, c2, vshift, m_run, l_run, ps, o_acc);
  softmax_chunk<PLAIN, 1>(srow, sb, sa, bt, c2, vshift, m_run, l_run, ps, o_acc);
  softmax_chunk<PLAIN, 2>(srow, sa, sb, bt, c2, vshift, m_run, l_run, ps, o_acc);
  softmax_chunk<PLAIN, 3>(srow, sb, sa, bt, c2, vshift, m_run, l_run, ps, o_acc);
  float s0, s1, s2, s3;
  f2unpack(ps[0], s0, s1);
  f2unpack(ps[1], s2, s3);
  l_run = fmaf((s0 + s1) + (s2 + s3), ex2(-vshift), l_run);  // sum of unshifted p
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    sdpa_fwd_tc(const __grid_constant__ CUtensorMap tm_qhi, const __grid_constant__ CUtensorMap tm_qlo,
                const __grid_constant__ CUtensorMap tm_khi, const __grid_constant__ CUtensorMap tm_klo,
                const __grid_constant__ CUtensorMap tm_vhi, const __grid_constant__ CUtensorMap tm_vlo,
                const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* q_s = smem;                 // [hi, lo] Q tile (128 rows x 64, 128-byte swizzle)
  uint8_t* k_st = q_s + STAGE;         // [2][hi, lo] K tiles
  uint8_t* v_st = k_st + 2 * STAGE;    // [2][hi, lo] V^T tiles, each two [64 x 64] blocks
  float* bias_s = reinterpret_cast<float*>(v_st + 2 * STAGE);  // [8 warps][BKV], log2 units
  float* xm = bias_s + 8 * BKV;        // [2 teams][BQ] final reference maxima
  float* xl = xm + 2 * BQ;             // [2 teams][BQ] final row sums
  float* xo = xl + 2 * BQ;             // [BQ][OUT_PITCH] team 0's partial rows, then the output tile
  float* xvb = xo + BQ * OUT_PITCH;    // [8 softmax warps] partial max of the batch's V scales
  uint64_t* bars = reinterpret_cast<uint64_t*>(xvb + 8);
  uint64_t* q_full = bars + 0;   // Q tile of the item loaded (TMA bytes)
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [3] QK(t) retired into S buffer t % 3
  uint64_t* pv_done = bars + 12; // [3] P.V(t) retired (read buffer t % 3; wrote team t&1's O)
  uint64_t* p_full = bars + 15;  // [2] per team: P(t) written, its previous O merged
  uint64_t* qk_done = bars + 17; // QK issuer's MMAs retired (teardown)
  uint64_t* pv_all = bars + 18;  // P.V issuer's MMAs retired (teardown)
  uint64_t* xbar = bars + 19;    // team 0's partial of the item is published (4 arrivals)
  uint64_t* q_empty = bars + 20; // the item's QK MMAs retired: Q shared memory reusable
  uint64_t* xfree = bars + 21;   // team 1 has written the item's tile out (4 arrivals)
  uint64_t* xstage = bars + 22;  // team 1 has staged the merged tile (4 arrivals)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 23);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const int T = p.T;
  // persistent CTAs: work item j = blockIdx.x + i * gridDim.x (query tiles of one head
  // consecutive, so CTAs running together share the head's K / V in L2); every role walks
  // the same items, and stages / barrier phases run on the global tile counter G = i*T + t
  const int items = p.Qt * p.BH;
  const int my_items = (int)blockIdx.x < items ? (items - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  auto item_of = [&](int i, int& bh, int& q0) {
    const int j = blockIdx.x + i * gridDim.x;
    bh = j / p.Qt;
    q0 = (j - bh * p.Qt) * BQ;
  };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    mbar_init(xfree, 4);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1); mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1); mbar_init(&v_empty[i], 1);
      mbar_init(&p_full[i], 4);
    }
    for (int i = 0; i < NSB; ++i) { mbar_init(&s_full[i], 1); mbar_init(&pv_done[i], 1); }
    mbar_init(qk_done, 1);
    mbar_init(pv_all, 1);
    mbar_init(xbar, 4);
    mbar_init(xstage, 4);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_qhi); tma_prefetch_desc(&tm_qlo);
    tma_prefetch_desc(&tm_khi); tma_prefetch_desc(&tm_klo);
    tma_prefetch_desc(&tm_vhi); tma_prefetch_desc(&tm_vlo);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    setmaxnreg_dec<REGS_CONTROL>();
  if (warp == 0 || warp == 2) {
    // ---------------- TMA producers: warp 0 the K tiles, warp 2 the V^T tiles --------
    if (elect_one()) {
      const bool is_k = warp == 0;
      uint64_t* full = is_k ? k_full : v_full;
      uint64_t* empty = is_k ? k_empty : v_empty;
      uint8_t* base = is_k ? k_st : v_st;
      int issued[2] = {-1, -1};
      int q_issued = -1;
      bool ok = true;
      for (int i = 0; i < my_items && ok; ++i) {
        int bh, q0;
        item_of(i, bh, q0);
        if (is_k) {
          // the item's Q tile, once the previous item's QK MMAs have read the old one
          // (rows past Lq read as zeros)
          if (i >= 1 && !mbar_wait(q_empty, (i - 1) & 1, p.status, kDevTimeoutProducer, abort_flag)) break;
          mbar_arrive_expect_tx(q_full, STAGE);
          tma_load_3d(q_s, &tm_qhi, q_full, 0, q0, bh);
          tma_load_3d(q_s + PLANE, &tm_qlo, q_full, 0, q0, bh);
          q_issued = i;
        }
        for (int t = 0; t < T; ++t) {
          const int G = i * T + t, st = G & 1;
          if (G >= 2 && !mbar_wait(&empty[st], ((G >> 1) & 1) ^ 1, p.status, kDevTimeoutProducer, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* d = base + st * STAGE;
          mbar_arrive_expect_tx(&full[st], STAGE);
          if (is_k) {
            tma_load_3d(d, &tm_khi, &full[st], 0, t * BKV, bh);
            tma_load_3d(d + PLANE, &tm_klo, &full[st], 0, t * BKV, bh);
          } else {
            tma_load_3d(d, &tm_vhi, &full[st], t * BKV, 0, bh);
            tma_load_3d(d + PLANE / 2, &tm_vhi, &full[st], t * BKV + 64, 0, bh);
            tma_load_3d(d + PLANE, &tm_vlo, &full[st], t * BKV, 0, bh);
            tma_load_3d(d + PLANE + PLANE / 2, &tm_vlo, &full[st], t * BKV + 64, 0, bh);
          }
          issued[st] = G;
        }
      }
      if (*abort_flag) {
        // never leave the CTA while a bulk copy may still write its shared memory
        for (int i = 0; i < 2; ++i)
          if (issued[i] >= 0) mbar_wait(&full[i], (issued[i] >> 1) & 1, p.status, kDevTimeoutProducer, nullptr);
        if (q_issued >= 0) mbar_wait(q_full, q_issued & 1, p.status, kDevTimeoutProducer, nullptr);
      }
    }
  } else if (warp == 1) {
    // ---------------- QK^T issuer ----------------
    // QK(t) goes into S buffer t % 3 as soon as its K tile is in and P.V(t-3), the last
    // reader of that buffer, has retired; P.V is issued by warp 3, so the scores of a
    // team's next tile never wait behind the other team's P.
    if (elect_one()) {
      constexpr uint32_t idesc_s = idesc_f16_f32(BQ, BKV);
      bool ok = true;
      const uint32_t qh = smem_u32(q_s), ql = qh + PLANE;
      for (int i = 0; i < my_items && ok; ++i) {
      ok = mbar_wait(q_full, i & 1, p.status, kDevTimeoutMma, abort_flag);
      for (int t = 0; t < T && ok; ++t) {
        const int G = i * T + t, st = G & 1, sb = G % NSB;
        ok = mbar_wait(&k_full[st], (G >> 1) & 1, p.status, kDevTimeoutMma, abort_flag) &&
             (G < NSB || mbar_wait(&pv_done[sb], ((G - NSB) / NSB) & 1, p.status, kDevTimeoutMma, abort_flag));
        if (!ok) break;
        tc_fence_after();
        const uint32_t kh = smem_u32(k_st + st * STAGE), kl = kh + PLANE;
        const uint32_t sd = tmem + S_COL + sb * BKV;
        // rolled loop: fully unrolled, the loop-invariant descriptors would be hoisted out
        // of the tile loop and overflow this warpgroup's register budget
#pragma unroll 1
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t a_h = sw128_kmajor_desc(qh + kk * 32);
          const uint64_t a_l = sw128_kmajor_desc(ql + kk * 32);
          const uint64_t b_h = sw128_kmajor_desc(kh + kk * 32);
          const uint64_t b_l = sw128_kmajor_desc(kl + kk * 32);
          mma_f16_ss(sd, a_h, b_h, idesc_s, kk != 0);
          mma_f16_ss(sd, a_h, b_l, idesc_s, 1);
          mma_f16_ss(sd, a_l, b_h, idesc_s, 1);
        }
        mma_commit(&k_empty[st]);
        mma_commit(&s_full[sb]);
      }
      if (ok) mma_commit(q_empty);  // this item's QK MMAs retire -> the next Q may land
      }
      mma_commit(qk_done);
      mbar_wait(qk_done, 0, p.status, kDevTimeoutMma, nullptr);
    }
  } else {
    // ---------------- P.V issuer (warp 3) ----------------
    if (elect_one()) {
      constexpr uint32_t idesc_o = idesc_f16_f32(BQ, D);
      bool ok = true;
      const int nt0 = (T + 1) / 2, nt1 = T / 2;  // tiles of team 0 / team 1 per item
      for (int i = 0; i < my_items && ok; ++i)
      for (int t = 0; t < T && ok; ++t) {
        const int G = i * T + t, st = G & 1, team = t & 1;
        const int c = i * (team ? nt1 : nt0) + (t >> 1);  // the team's global tile count
        ok = mbar_wait(&p_full[team], c & 1, p.status, kDevTimeoutMma, abort_flag) &&
             mbar_wait(&v_full[st], (G >> 1) & 1, p.status, kDevTimeoutMma, abort_flag);
        if (!ok) break;
        tc_fence_after();
        const uint32_t vh = smem_u32(v_st + st * STAGE), vl = vh + PLANE;
        const uint32_t ps = tmem + S_COL + (G % NSB) * BKV;
        const uint32_t od = tmem + O_COL + team * D;
#pragma unroll 1
        for (int kk = 0; kk < BKV / 16; ++kk) {
          const uint32_t ph = ps + kk * 16;  // P_hi for keys 16kk..16kk+15
          const uint32_t pl = ph + 8;        // P_lo
          const uint32_t voff = (kk >> 2) * (PLANE / 2) + (kk & 3) * 32;
          const uint64_t b_h = sw128_kmajor_desc(vh + voff);
          const uint64_t b_l = sw128_kmajor_desc(vl + voff);
          mma_f16_ts(od, ph, b_h, idesc_o, kk != 0);  // fresh O_t per key tile
          mma_f16_ts(od, ph, b_l, idesc_o, 1);
          mma_f16_ts(od, pl, b_h, idesc_o, 1);
        }
        mma_commit(&v_empty[st]);
        mma_commit(&pv_done[G % NSB]);
      }
      mma_commit(pv_all);
      mbar_wait(pv_all, 0, p.status, kDevTimeoutMma, nullptr);
    }
  }
  } else {
    setmaxnreg_inc<REGS_SOFTMAX>();
    // ---------------- softmax: team 0 takes even tiles, team 1 odd tiles ---------------
    const int team = (warp - 4) >> 2;
    const uint32_t sub = warp & 3;
    const int r = sub * 32 + lane;  // query row within the tile == TMEM lane
    const uint32_t trow = tmem + ((sub * 32) << 16);
    float* bt = bias_s + (warp - 4) * BKV;
    const uint32_t orow = trow + O_COL + team * D;
    bool ok = true;
    // An item's scales — the row's Q pre-scale, this lane's share of the head's V-tile
    // scales and the K scale of the team's first tile — are loaded one item ahead into
    // registers, so their latency hides behind the previous item's tiles instead of delaying
    // its first.
    constexpr int PF_V = 3;
    float pf_cq = 0.0f, pf_k0 = 0.0f, pf_v[PF_V];
    auto prefetch = [&](int i) {
      int bh_, q0_;
      item_of(i, bh_, q0_);
      const int qr = q0_ + r;
      pf_cq = qr < p.Lq ? p.qinv[(int64_t)bh_ * p.Lq + qr] : 0.0f;
      pf_k0 = team < T ? p.kinv[(int64_t)bh_ * T + team] : 0.0f;
#pragma unroll
      for (int k = 0; k < PF_V; ++k) {
        const int t = lane + 32 * k;
        pf_v[k] = t < T ? p.vinv[(int64_t)bh_ * T + t] : 0.0f;
      }
    };
    if (my_items > 0) prefetch(0);
    for (int i = 0; i < my_items && ok; ++i) {
    int bh, q0;
    item_of(i, bh, q0);
    const int qrow = q0 + r;
    const bool row_valid = qrow < p.Lq;
    const float cq = 0.125f * LOG2E * pf_cq;
    const float* bias_row = p.bias ? p.bias + (int64_t)bh * p.bias_bh_stride : nullptr;
    // reference V scale of the head: the largest per-tile inverse pre-scale (the lanes'
    // prefetched shares, the rest of a long sequence's tiles, then a warp max)
    float vref = pf_v[0];
#pragma unroll
    for (int k = 1; k < PF_V; ++k) vref = fmaxf(vref, pf_v[k]);
    for (int t = lane + 32 * PF_V; t < T; t += 32) vref = fmaxf(vref, p.vinv[(int64_t)bh * T + t]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) vref = fmaxf(vref, __shfl_xor_sync(0xffffffffu, vref, o));
    // the team's first tile's K and V scales (tile `team`: lane `team`'s first share)
    const float k0_cur = pf_k0, v0_cur = __shfl_sync(0xffffffffu, pf_v[0], team);
    // the next item's scales are requested after this item's first tile: right here the
    // previous item's output stores still fill the load / store queue
    bool pf_next = i + 1 < my_items;
    const int vref_exp = __float_as_int(vref) >> 23;
    float m_run = -INFINITY, l_run = 0.0f;
    float o_acc[D];
#pragma unroll
    for (int d = 0; d < D; ++d) o_acc[d] = 0.0f;
    int n = 0;  // tiles this team has processed in this item
    for (int t = team; t < T; t += 2, ++n) {
      const int G = i * T + t, sb = G % NSB;
      const bool plain = bias_row == nullptr && (t + 1) * BKV <= p.Lk;  // no bias, no masking
      if (!plain) {
        // key bias (+ -inf past Lk) for this tile, staged in a warp-private buffer
        __syncwarp();
#pragma unroll
        for (int ii = 0; ii < BKV / 32; ++ii) {
          const int jl = ii * 32 + lane;
          const int j = t * BKV + jl;
          bt[jl] = j < p.Lk ? (bias_row ? bias_row[j] * LOG2E : 0.0f) : -INFINITY;
        }
        __syncwarp();
      }
      const float c2 = cq * (n == 0 ? k0_cur : p.kinv[(int64_t)bh * T + t]);
      // exponent offset folding this V tile's pre-scale relative to the head reference
      const float vshift =
          (float)((__float_as_int(n == 0 ? v0_cur : p.vinv[(int64_t)bh * T + t]) >> 23) - vref_exp);
      ok = mbar_wait(&s_full[sb], (G / NSB) & 1, p.status, kDevTimeoutConsumer, abort_flag);
      // this team's previous O, P.V(G-2), retired long ago; it is folded in with the scores
      if (ok && n > 0) {
        const int Gp = G - 2;
        ok = mbar_wait(&pv_done[Gp % NSB], (Gp / NSB) & 1, p.status, kDevTimeoutConsumer, abort_flag);
      }
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      const uint32_t srow = trow + S_COL + sb * BKV;
      if (plain)
        softmax_tile<true>(srow, orow, n > 0, bt, c2, vshift, m_run, l_run, o_acc);
      else
        softmax_tile<false>(srow, orow, n > 0, bt, c2, vshift, m_run, l_run, o_acc);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[team]);
      if (pf_next) {
        prefetch(i + 1);
        pf_next = false;
      }
    }
    if (pf_next) prefetch(i + 1);  // a team without tiles in this item
    // output split: this warp's share of the batch's V-tile scales (the loads issue before
    // the wait for the last P.V; the 8 shares meet in the exchange)
    float vb_part = 0.0f;
    if (p.ohi) {
      const float* vb = p.vinv + (int64_t)(bh / p.H) * p.H * T;
      const int cnt = p.H * T;
#pragma unroll 4
      for (int e = (warp - 4) * 32 + lane; e < cnt; e += 256) vb_part = fmaxf(vb_part, vb[e]);
    }
    if (ok && n > 0) {
      // the team's last O of the item
      const int Gl = i * T + team + 2 * (n - 1);
      ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[Gl % NSB], (Gl / NSB) & 1, p.status,
                                             kDevTimeoutEpilogue, abort_flag));
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t o[32];
          tmem_ld32(orow + hh * 32, o);
          tmem_wait_ld();
          reg_fence(o);
#pragma unroll
          for (int d = 0; d < 32; ++d) o_acc[hh * 32 + d] += __uint_as_float(o[d]);
        }
      }
    }
    // End of the item.  Team 0 (the even tiles; its last tile's scores come first) publishes
    // its partial softmax of every row — reference max, sum, all 64 O values — and goes on
    // to the next item; team 1 merges it with its own (common reference, factors
    // 2^(m_team - m), exact since both references are integers, or -inf for a team without
    // tiles), stages the merged 128 x 64 tile in place and writes it out in row order.
    if (p.ohi) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) vb_part = fmaxf(vb_part, __shfl_xor_sync(0xffffffffu, vb_part, o));
    }
    float* xrow = xo + r * OUT_PITCH;  // team 0's partial of row r, then the merged row
    if (team == 0) {
      // team 1 has written out the previous item's tile before the buffer is reused
      if (ok && i >= 1)
        ok = __all_sync(0xffffffffu, mbar_wait(xfree, (i - 1) & 1, p.status, kDevTimeoutEpilogue, abort_flag));
      if (ok) {
        xm[r] = m_run;
        xl[r] = l_run;
#pragma unroll
        for (int d = 0; d < D; d += 4)
          *reinterpret_cast<float4*>(xrow + d) = make_float4(o_acc[d], o_acc[d + 1], o_acc[d + 2], o_acc[d + 3]);
        if (p.ohi && lane == 0) xvb[warp - 4] = vb_part;
        __syncwarp();
        if (lane == 0) mbar_arrive(xbar);
      }
    } else {
      if (p.ohi && lane == 0) xvb[warp - 4] = vb_part;
      if (ok)
        ok = __all_sync(0xffffffffu, mbar_wait(xbar, i & 1, p.status, kDevTimeoutEpilogue, abort_flag));
      if (ok && row_valid) {
        const float m0 = xm[r], l0 = xl[r];
        const float m = fmaxf(m_run, m0);
        const float f1 = m_run == m ? 1.0f : ex2(m_run - m);  // 0 for a team with no tiles
        const float f0 = m0 == m ? 1.0f : ex2(m0 - m);
        const float f = vref / (l0 * f0 + l_run * f1);
        // dimensions 0..31 as team 0's own (o0 f0 + o1 f1), 32..63 as team 1's own
#pragma unroll
        for (int d = 0; d < D; d += 4) {
          const float4 o0 = *reinterpret_cast<const float4*>(xrow + d);
          const float a[4] = {o0.x, o0.y, o0.z, o0.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            if (d < 32) o_acc[d + e] = (a[e] * f0 + o_acc[d + e] * f1) * f;
            else o_acc[d + e] = (o_acc[d + e] * f1 + a[e] * f0) * f;
          }
          *reinterpret_cast<float4*>(xrow + d) = make_float4(o_acc[d], o_acc[d + 1], o_acc[d + 2], o_acc[d + 3]);
        }
      }
      // team 1's four warps have staged their rows
      __syncwarp();
      if (lane == 0) mbar_arrive(xstage);
      ok = ok && __all_sync(0xffffffffu, mbar_wait(xstage, i & 1, p.status, kDevTimeoutEpilogue, abort_flag));
      if (ok) {
        // the item's output, row by row: 16 threads per row, 4 consecutive values each
        const int b = bh / p.H, hh = bh % p.H;
        const int tid = (warp - 8) * 32 + lane;
        int s = 0;
        float sc = 1.0f;
        if (p.ohi) {
          float vbat = xvb[0];
#pragma unroll
          for (int w = 1; w < 8; ++w) vbat = fmaxf(vbat, xvb[w]);
          // |O| <= max |V| < 2^15 * vbat; 2^-6 of slack for the rounding of P.V and of 1/l
          s = pow2_shift(32768.0f * vbat * (1.0f + 0x1p-6f));
          sc = pow2i(s);
        }
#pragma unroll 1
        for (int f4 = tid; f4 < BQ * (D / 4); f4 += BQ) {
          const int row = f4 / (D / 4), c = (f4 % (D / 4)) * 4;
          const int qr = q0 + row;
          if (qr >= p.Lq) continue;
          const float4 v = *reinterpret_cast<const float4*>(xo + row * OUT_PITCH + c);
          if (p.ohi) {
            const int64_t off = ((int64_t)b * p.Lq + qr) * ((int64_t)p.H * D) + hh * D + c;
            const float a0 = v.x * sc, a1 = v.y * sc, a2 = v.z * sc, a3 = v.w * sc;
            const __half2 h01 = __floats2half2_rn(a0, a1), h23 = __floats2half2_rn(a2, a3);
            const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
            const __half2 l01 = __floats2half2_rn(a0 - f01.x, a1 - f01.y);
            const __half2 l23 = __floats2half2_rn(a2 - f23.x, a3 - f23.y);
            *reinterpret_cast<uint2*>(p.ohi + off) =
                make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h23));
            *reinterpret_cast<uint2*>(p.olo + off) =
                make_uint2(*reinterpret_cast<const uint32_t*>(&l01), *reinterpret_cast<const uint32_t*>(&l23));
          } else {
            float* dst = p.out_blhd ? p.out + (((int64_t)b * p.Lq + qr) * p.H + hh) * D + c
                                    : p.out + ((int64_t)bh * p.Lq + qr) * D + c;
            *reinterpret_cast<float4*>(dst) = v;
          }
        }
        if (p.ohi && hh == 0 && tid < BQ && q0 + tid < p.Lq) p.ors[(int64_t)b * p.Lq + q0 + tid] = pow2i(-s);
      }
      // the buffer (and the V-scale shares) may be reused for the next item
      __syncwarp();
      if (lane == 0) mbar_arrive(xfree);
    }
    }  // item loop
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Pre-split kernels
// ---------------------------------------------------------------------------
// Q [BH, Lq, 64] fp32 -> hi/lo fp16 [BH, Lq, 64], qinv [BH*Lq].  One warp per row.
__global__ void sdpa_split_q(const float* __restrict__ q, int64_t rows, __half* __restrict__ hi,
                             __half* __restrict__ lo, float* __restrict__ qinv) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float2 v = *reinterpret_cast<const float2*>(q + row * D + lane * 2);
  float mx = fmaxf(fabsf(v.x), fabsf(v.y));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const int s = pow2_shift(mx);
  const float a = v.x * pow2i(s), b = v.y * pow2i(s);
  const __half2 h = __floats2half2_rn(a, b);
  const float2 hf = __half22float2(h);
  *reinterpret_cast<__half2*>(hi + row * D + lane * 2) = h;
  *reinterpret_cast<__half2*>(lo + row * D + lane * 2) = __floats2half2_rn(a - hf.x, b - hf.y);
  if (lane == 0) qinv[row] = pow2i(-s);
}

// One CTA per (bh, 128-key tile): K -> hi/lo [BH, Lkt, 64]; V -> transposed hi/lo
// [BH, 64, Lkt]; one power-of-two pre-scale per tile for each.  Keys >= Lk are zero.
// Element (j, d) of K (or V) is read at base + bh*bh_stride + j*j_stride + d*d_stride,
// which covers both the [B,H,Lk,64] layout and the packed [B,H,64,Lkp] one.
__global__ void __launch_bounds__(256) sdpa_split_kv(
    const float* __restrict__ k, const float* __restrict__ v, int64_t bh_stride, int64_t j_stride,
    int64_t d_stride, int Lk, int Lkt, __half* __restrict__ khi, __half* __restrict__ klo,
    __half* __restrict__ vhi, __half* __restrict__ vlo, float* __restrict__ kinv,
    float* __restrict__ vinv) {
  __shared__ float vt[BKV][D + 1];
  __shared__ float red[2][8];
  const int t = blockIdx.x, bh = blockIdx.y, T = gridDim.x;
  const int j0 = t * BKV;
  const float* kb = k + (int64_t)bh * bh_stride;
  const float* vb = v + (int64_t)bh * bh_stride;
  float kmx = 0.0f, vmx = 0.0f;
  for (int e = threadIdx.x; e < BKV * D; e += 256) {
    int j, d;
    if (d_stride == 1) { j = e / D; d = e % D; } else { d = e / BKV; j = e % BKV; }
    const int jj = j0 + j;
    float kv = 0.0f, vv = 0.0f;
    if (jj < Lk) {
      kv = kb[(int64_t)jj * j_stride + (int64_t)d * d_stride];
      vv = vb[(int64_t)jj * j_stride + (int64_t)d * d_stride];
    }
    vt[j][d] = vv;
    kmx = fmaxf(kmx, fabsf(kv));
    vmx = fmaxf(vmx, fabsf(vv));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    kmx = fmaxf(kmx, __shfl_xor_sync(0xffffffffu, kmx, o));
    vmx = fmaxf(vmx, __shfl_xor_sync(0xffffffffu, vmx, o));
  }
  if ((threadIdx.x & 31) == 0) { red[0][threadIdx.x >> 5] = kmx; red[1][threadIdx.x >> 5] = vmx; }
  __syncthreads();
  kmx = red[0][0]; vmx = red[1][0];
#pragma unroll
  for (int w = 1; w < 8; ++w) { kmx = fmaxf(kmx, red[0][w]); vmx = fmaxf(vmx, red[1][w]); }
  const int sk = pow2_shift(kmx), sv = pow2_shift(vmx);
  // K rows: thread handles (row j, 8 dims); reads are L1/L2 hits from the first pass
  for (int e = threadIdx.x; e < BKV * (D / 8); e += 256) {
    const int j = e / (D / 8), d0 = (e % (D / 8)) * 8;
    const int jj = j0 + j;
    __align__(16) __half h8[8];
    __align__(16) __half l8[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float x = jj < Lk ? kb[(int64_t)jj * j_stride + (int64_t)(d0 + i) * d_stride] * pow2i(sk) : 0.0f;
      const __half hh = __float2half_rn(x);
      h8[i] = hh;
      l8[i] = __float2half_rn(x - __half2float(hh));
    }
    const int64_t off = ((int64_t)bh * Lkt + jj) * D + d0;
    *reinterpret_cast<uint4*>(khi + off) = *reinterpret_cast<uint4*>(h8);
    *reinterpret_cast<uint4*>(klo + off) = *reinterpret_cast<uint4*>(l8);
  }
  // V transposed: thread handles (dim d, 8 keys)
  for (int e = threadIdx.x; e < D * (BKV / 8); e += 256) {
    const int d = e / (BKV / 8), jb = (e % (BKV / 8)) * 8;
    __align__(16) __half h8[8];
    __align__(16) __half l8[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float x = vt[jb + i][d] * pow2i(sv);
      const __half hh = __float2half_rn(x);
      h8[i] = hh;
      l8[i] = __float2half_rn(x - __half2float(hh));
    }
    const int64_t off = ((int64_t)bh * D + d) * Lkt + j0 + jb;
    *reinterpret_cast<uint4*>(vhi + off) = *reinterpret_cast<uint4*>(h8);
    *reinterpret_cast<uint4*>(vlo + off) = *reinterpret_cast<uint4*>(l8);
  }
  if (threadIdx.x == 0) {
    kinv[(int64_t)bh * T + t] = pow2i(-sk);
    vinv[(int64_t)bh * T + t] = pow2i(-sv);
  }
}


// Fused QKV post-process -> attention split format (no reference counterpart; the
// composition of scripts/native_qkv_postprocess_v2_avx512.c:45-191 with the split above).
// One CTA per (bh, 128-token tile), eight lanes per token: RoPE + 8/max(||.||,1e-12)*gamma
// on q and k (rope_rms64's arithmetic and sum order), then q rows straight to the Q planes
// (per-row pre-scale, as
// sdpa_split_q) and the tile's k / v through shared memory to the K and V^T planes (per-tile
// pre-scales, as sdpa_split_kv): the same bits as the two-kernel path, with q / k / v never
// written to HBM in fp32.  Source layouts: kSelected = false: qkv [B, L, 3, H, 64]
// (q, k and v of token t); kSelected = true: q [B, Lq, H, 64] and kv [B, Lk, 2, H, 64], RoPE
// frequency row of query i = sel[i] (no frequencies: no rotation).

// Key tiles tile0 + blockIdx.y of the sequence (Lk tokens).  kvsrc holds src_L token rows
// per batch starting at token src_t0 (the whole sequence: 0, Lk; a query-row shard: its own
// token range); self-attention Q rows of token t go to row t - q_t0 of the Q planes.
template <bool kSelected>
__global__ void __launch_bounds__(256, 3) qkv_split_k(
    const float* __restrict__ qsrc, const float* __restrict__ kvsrc, const float* __restrict__ freqs,
    const int64_t* __restrict__ sel, const float* __restrict__ qg, const float* __restrict__ kg,
    int H, int Lq, int Lk, int Lkt, int fb, int tile0, int src_t0, int src_L, int q_t0,
    __half* __restrict__ qhi, __half* __restrict__ qlo,
    float* __restrict__ qinv, __half* __restrict__ khi, __half* __restrict__ klo,
    __half* __restrict__ vhi, __half* __restrict__ vlo, float* __restrict__ kinv,
    float* __restrict__ vinv) {
  extern __shared__ float sm_kv[];
  float(*vt)[D + 1] = reinterpret_cast<float(*)[D + 1]>(sm_kv);  // [BKV][65]: V for the transpose
  __shared__ float red[2][8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // heads fastest (blockIdx.x): CTAs running together read the same token rows' heads, so
  // each token's q / k / v row of all heads streams from DRAM once, in order
  const int bh = blockIdx.x, b = bh / H, h = bh % H;
  const int fbb = fb == 1 ? 0 : b;
  const int tile = blockIdx.y + tile0, T = Lkt / BKV;
  const int t_end = min(Lk, src_t0 + src_L);  // tokens past it read as zeros
  // eight lanes per token, four tokens per warp at a time: lane j of a token holds the
  // complex pairs j, j + 8, j + 16, j + 24 (the butterfly order of rope_rms64 kept: levels
  // 16 and 8 are the lane's own adds, 4 / 2 / 1 shuffles inside the token's lanes)
  const int grp = lane >> 3, jl = lane & 7;
  const float2* gq2 = reinterpret_cast<const float2*>(qg + (int64_t)h * 64);
  const float2* gk2 = reinterpret_cast<const float2*>(kg + (int64_t)h * 64);
  // RoPE + 8/max(||.||, 1e-12) * gamma of one token's row (4 pairs per lane), and its max
  auto rope_rms8 = [&](const float2 (&x)[4], const float2 (&f)[4], const float2* g,
                       float2 (&y)[4]) -> float {
    float sq[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      y[k] = make_float2(fmaf(x[k].x, f[k].x, -(x[k].y * f[k].y)), fmaf(x[k].x, f[k].y, x[k].y * f[k].x));
      sq[k] = fmaf(y[k].x, y[k].x, y[k].y * y[k].y);
    }
    float ss = (sq[0] + sq[2]) + (sq[1] + sq[3]);
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float fac = 8.0f / fmaxf(sqrtf(ss), 1.0e-12f);
    float mx = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 gg = g[jl + 8 * k];
      y[k] = make_float2(y[k].x * fac * gg.x, y[k].y * fac * gg.y);
      mx = fmaxf(mx, fmaxf(fabsf(y[k].x), fabsf(y[k].y)));
    }
    return mx;
  };
  if (tile < T) {
    const int t0 = tile * BKV;
    float kmx = 0.0f, vmx = 0.0f;
    float2 kreg[4][4];  // this lane's pairs of its 4 k rows until the tile's scale is known;
                        // V goes through shared memory (transpose)
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = warp * 16 + u * 4 + grp;  // token within the tile
      const int t = t0 + i;
      float2 qx[4], kx[4], vx[4], fr[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        qx[k] = kx[k] = vx[k] = make_float2(0.0f, 0.0f);
        fr[k] = make_float2(1.0f, 0.0f);
      }
      const bool valid = t < t_end;
      if (valid) {
        const int64_t r = (int64_t)b * src_L + (t - src_t0);
        const float* ks = kSelected ? kvsrc + (r * 2 * H + h) * 64 : kvsrc + (r * 3 * H + H + h) * 64;
        const float2* f2 = freqs ? reinterpret_cast<const float2*>(freqs + (((int64_t)fbb * Lk + t) * H + h) * 64)
                                 : nullptr;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (f2) fr[k] = f2[jl + 8 * k];
          if (!kSelected) qx[k] = reinterpret_cast<const float2*>(ks - (int64_t)H * 64)[jl + 8 * k];
          kx[k] = reinterpret_cast<const float2*>(ks)[jl + 8 * k];
          vx[k] = reinterpret_cast<const float2*>(ks + (int64_t)H * 64)[jl + 8 * k];
        }
      }
      if (!kSelected) {
        float2 qy[4];
        const float qmx = rope_rms8(qx, fr, gq2, qy);
        float m = qmx;
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (valid) {
          const int sq2 = pow2_shift(m);
          const int64_t row = (int64_t)bh * Lq + (t - q_t0);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float a = qy[k].x * pow2i(sq2), c = qy[k].y * pow2i(sq2);
            const __half2 hh = __floats2half2_rn(a, c);
            const float2 hf = __half22float2(hh);
            *reinterpret_cast<__half2*>(qhi + row * D + 2 * (jl + 8 * k)) = hh;
            *reinterpret_cast<__half2*>(qlo + row * D + 2 * (jl + 8 * k)) = __floats2half2_rn(a - hf.x, c - hf.y);
          }
          if (jl == 0) qinv[row] = pow2i(-sq2);
        }
      }
      float2 ky[4];
      const float km = rope_rms8(kx, fr, gk2, ky);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        kreg[u][k] = valid ? ky[k] : make_float2(0.0f, 0.0f);
        vt[i][2 * (jl + 8 * k)] = vx[k].x;
        vt[i][2 * (jl + 8 * k) + 1] = vx[k].y;
        vmx = fmaxf(vmx, fmaxf(fabsf(vx[k].x), fabsf(vx[k].y)));
      }
      if (valid) kmx = fmaxf(kmx, km);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      kmx = fmaxf(kmx, __shfl_xor_sync(0xffffffffu, kmx, o));
      vmx = fmaxf(vmx, __shfl_xor_sync(0xffffffffu, vmx, o));
    }
    if (lane == 0) { red[0][warp] = kmx; red[1][warp] = vmx; }
    __syncthreads();
    kmx = red[0][0]; vmx = red[1][0];
#pragma unroll
    for (int w = 1; w < 8; ++w) { kmx = fmaxf(kmx, red[0][w]); vmx = fmaxf(vmx, red[1][w]); }
    const int sk = pow2_shift(kmx), sv = pow2_shift(vmx);
    // K rows straight from registers
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t row = (int64_t)bh * Lkt + t0 + warp * 16 + u * 4 + grp;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float a = kreg[u][k].x * pow2i(sk), c = kreg[u][k].y * pow2i(sk);
        const __half2 hh = __floats2half2_rn(a, c);
        const float2 hf = __half22float2(hh);
        *reinterpret_cast<__half2*>(khi + row * D + 2 * (jl + 8 * k)) = hh;
        *reinterpret_cast<__half2*>(klo + row * D + 2 * (jl + 8 * k)) = __floats2half2_rn(a - hf.x, c - hf.y);
      }
    }
    for (int e = threadIdx.x; e < D * (BKV / 8); e += 256) {
      const int d = e / (BKV / 8), jb = (e % (BKV / 8)) * 8;
      __align__(16) __half h8[8];
      __align__(16) __half l8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float x = vt[jb + i][d] * pow2i(sv);
        const __half hh = __float2half_rn(x);
        h8[i] = hh;
        l8[i] = __float2half_rn(x - __half2float(hh));
      }
      const int64_t off = ((int64_t)bh * D + d) * Lkt + t0 + jb;
      *reinterpret_cast<uint4*>(vhi + off) = *reinterpret_cast<uint4*>(h8);
      *reinterpret_cast<uint4*>(vlo + off) = *reinterpret_cast<uint4*>(l8);
    }
    if (threadIdx.x == 0) {
      kinv[(int64_t)bh * T + tile] = pow2i(-sk);
      vinv[(int64_t)bh * T + tile] = pow2i(-sv);
    }
  }
}

// Selected-query rows of the fused post-process (the q half of qkv_split_k<true>): RMSNorm
// (and RoPE with the frequency row sel[i]) into the Q planes; one CTA per (bh, 128 queries),
// no shared memory, so it runs at full occupancy.
// Four rows per warp at a time, eight lanes per row: lane j of a row holds the complex
// pairs j, j + 8, j + 16, j + 24.  rope_rms64's butterfly adds pair l to pair l + 16, then
// l + 8, 4, 2, 1: here the first two levels are the lane's own adds and the last three are
// shuffles inside the row's eight lanes, so the sum (and every result bit) is the same,
// with three dependent shuffles per reduction instead of five and four rows in flight.
__global__ void __launch_bounds__(256) selected_q_split_k(
    const float* __restrict__ qsrc, const float* __restrict__ freqs, const int64_t* __restrict__ sel,
    const float* __restrict__ qg, int H, int Lq, int Lk, int fb, __half* __restrict__ qhi,
    __half* __restrict__ qlo, float* __restrict__ qinv) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = lane >> 3, j = lane & 7;
  const int bh = blockIdx.x, b = bh / H, h = bh % H;  // heads fastest, as qkv_split_k
  const int fbb = fb == 1 ? 0 : b;
  const int tile = blockIdx.y;
  const float2* g2 = reinterpret_cast<const float2*>(qg + (int64_t)h * 64);
  float2 gq[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) gq[k] = g2[j + 8 * k];
  // 16 rows per warp: four passes of four rows, all loads issued first
  float2 qx[4][4], fr[4][4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int qi = tile * BKV + warp * 16 + u * 4 + grp;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      qx[u][k] = make_float2(0.0f, 0.0f);
      fr[u][k] = make_float2(1.0f, 0.0f);  // no frequencies: identity rotation
    }
    if (qi < Lq) {
      const float2* src = reinterpret_cast<const float2*>(qsrc + (((int64_t)b * Lq + qi) * H + h) * 64);
      const float2* f2 = freqs ? reinterpret_cast<const float2*>(freqs + (((int64_t)fbb * Lk + sel[qi]) * H + h) * 64)
                               : nullptr;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        qx[u][k] = src[j + 8 * k];
        if (f2) fr[u][k] = f2[j + 8 * k];
      }
    }
  }
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int qi = tile * BKV + warp * 16 + u * 4 + grp;
    float2 y[4];
    float sq[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 x = qx[u][k], f = fr[u][k];
      y[k] = make_float2(fmaf(x.x, f.x, -(x.y * f.y)), fmaf(x.x, f.y, x.y * f.x));
      sq[k] = fmaf(y[k].x, y[k].x, y[k].y * y[k].y);
    }
    float ss = (sq[0] + sq[2]) + (sq[1] + sq[3]);  // butterfly levels 16 and 8
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float fac = 8.0f / fmaxf(sqrtf(ss), 1.0e-12f);
    float mx = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      y[k] = make_float2(y[k].x * fac * gq[k].x, y[k].y * fac * gq[k].y);
      mx = fmaxf(mx, fmaxf(fabsf(y[k].x), fabsf(y[k].y)));
    }
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (qi < Lq) {
      const int sq2 = pow2_shift(mx);
      const int64_t row = (int64_t)bh * Lq + qi;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float a = y[k].x * pow2i(sq2), c = y[k].y * pow2i(sq2);
        const __half2 hh = __floats2half2_rn(a, c);
        const float2 hf = __half22float2(hh);
        *reinterpret_cast<__half2*>(qhi + row * D + 2 * (j + 8 * k)) = hh;
        *reinterpret_cast<__half2*>(qlo + row * D + 2 * (j + 8 * k)) = __floats2half2_rn(a - hf.x, c - hf.y);
      }
      if (j == 0) qinv[row] = pow2i(-sq2);
    }
  }
}

constexpr int QKV_SPLIT_SMEM = BKV * (D + 1) * 4;  // the V staging tile

// Query-row sharding: each rank of a group splits the key tiles of its own tokens into its
// K / V plane set; after a peer barrier, kv_gather_k copies every other rank's tiles (the
// key rows, the transposed value rows and the per-tile scales) from that rank's plane set,
// mapped here over NVLink (CUDA IPC), into this rank's set.  Grid: (x, bh, source rank).
constexpr int kMaxGatherRanks = 8;
struct KvGather {
  const uint8_t* src[kMaxGatherRanks];  // each rank's plane set as mapped in this process
  int tlo[kMaxGatherRanks], thi[kMaxGatherRanks];  // each rank's key tiles [tlo, thi)
  unsigned long long off[6];  // byte offsets of khi, klo, vhi, vlo, kinv, vinv in a set
};

__global__ void __launch_bounds__(256) kv_gather_k(KvGather g, uint8_t* __restrict__ dst, int rank,
                                                   int Lkt, int T) {
  const int p = blockIdx.z, bh = blockIdx.y;
  if (p == rank) return;
  const int tiles = g.thi[p] - g.tlo[p];
  if (tiles <= 0) return;
  const int tok0 = g.tlo[p] * BKV;
  const uint8_t* src = g.src[p];
  const int64_t k_units = (int64_t)tiles * BKV * D * 2 / 16;  // 16-byte units per key plane
  const int64_t v_units = (int64_t)tiles * BKV * 2 / 16;      // per transposed value row
  const int64_t total = 2 * k_units + 2 * D * v_units;
  auto offset_of = [&](int64_t u) -> size_t {
    if (u < 2 * k_units) {
      const int plane = (int)(u / k_units);
      return g.off[plane] + ((size_t)bh * Lkt + tok0) * D * 2 + (size_t)(u - plane * k_units) * 16;
    }
    const int64_t v = u - 2 * k_units;
    const int plane = (int)(v / (D * v_units));
    const int64_t w = v - plane * D * v_units;
    const int d = (int)(w / v_units);
    return g.off[2 + plane] + (((size_t)bh * D + d) * Lkt + tok0) * 2 + (size_t)(w - d * v_units) * 16;
  };
  // GATHER_ILP 16-byte loads in flight per thread before their stores: a peer's memory is
  // a few microseconds away, and one outstanding load per thread would leave NVLink idle
  constexpr int GATHER_ILP = 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t u0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u0 < total; u0 += GATHER_ILP * stride) {
    uint4 val[GATHER_ILP];
    size_t off[GATHER_ILP];
#pragma unroll
    for (int e = 0; e < GATHER_ILP; ++e) {
      const int64_t u = u0 + e * stride;
      off[e] = u < total ? offset_of(u) : 0;
      if (u < total)
        asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(val[e].x), "=r"(val[e].y), "=r"(val[e].z), "=r"(val[e].w)
                     : "l"(src + off[e]));
    }
#pragma unroll
    for (int e = 0; e < GATHER_ILP; ++e)
      if (u0 + e * stride < total) *reinterpret_cast<uint4*>(dst + off[e]) = val[e];
  }
  if (blockIdx.x == 0) {
    for (int i = threadIdx.x; i < 2 * tiles; i += blockDim.x) {
      const int plane = i / tiles, j = i - plane * tiles;
      const size_t off = g.off[4 + plane] + ((size_t)bh * T + g.tlo[p] + j) * 4;
      float v;
      asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(src + off));
      *reinterpret_cast<float*>(dst + off) = v;
    }
  }
}

}  // namespace sdpa

struct SdpaCounters {
  uint64_t calls = 0, enqueue_ns = 0, split_ns = 0, attn_ns = 0;
};
static SdpaCounters g_sdpa;

static uint64_t now_ns() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (uint64_t)ts.tv_sec * 1000000000ull + ts.tv_nsec;
}

// Attention inputs in the split format, in the library workspace of the current stream.
struct SplitPlanesSdpa {
  __half *qhi, *qlo, *khi, *klo, *vhi, *vlo;
  float *qinv, *kinv, *vinv;
  int T, Lkt;
};

static size_t al256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// Q planes of Lq rows per head: [qhi | qlo | qinv]
static size_t q_planes_layout(int64_t BH, int Lq, size_t off[2]) {
  const size_t qplane = (size_t)BH * Lq * sdpa::D * 2;
  off[0] = al256(qplane);                 // qlo
  off[1] = off[0] + al256(qplane);        // qinv
  return off[1] + al256((size_t)BH * Lq * 4);
}

// K / V planes of a sequence of Lk keys (T tiles of BKV): [khi | klo | vhi | vlo | kinv | vinv]
static size_t kv_planes_layout(int64_t BH, int Lk, size_t off[6], int& T, int& Lkt) {
  T = (Lk + sdpa::BKV - 1) / sdpa::BKV;
  Lkt = T * sdpa::BKV;
  const size_t kplane = (size_t)BH * Lkt * sdpa::D * 2;
  off[0] = 0;
  off[1] = al256(kplane);
  off[2] = off[1] + al256(kplane);
  off[3] = off[2] + al256(kplane);
  off[4] = off[3] + al256(kplane);
  off[5] = off[4] + al256((size_t)BH * T * 4);
  return off[5] + al256((size_t)BH * T * 4);
}

static void planes_from(uint8_t* q, uint8_t* kv, int64_t BH, int Lq, int Lk, SplitPlanesSdpa& sp) {
  size_t qo[2], ko[6];
  q_planes_layout(BH, Lq, qo);
  kv_planes_layout(BH, Lk, ko, sp.T, sp.Lkt);
  sp.qhi = reinterpret_cast<__half*>(q);
  sp.qlo = reinterpret_cast<__half*>(q + qo[0]);
  sp.qinv = reinterpret_cast<float*>(q + qo[1]);
  sp.khi = reinterpret_cast<__half*>(kv + ko[0]);
  sp.klo = reinterpret_cast<__half*>(kv + ko[1]);
  sp.vhi = reinterpret_cast<__half*>(kv + ko[2]);
  sp.vlo = reinterpret_cast<__half*>(kv + ko[3]);
  sp.kinv = reinterpret_cast<float*>(kv + ko[4]);
  sp.vinv = reinterpret_cast<float*>(kv + ko[5]);
}

static int sdpa_planes(int64_t BH, int Lq, int Lk, cudaStream_t stream, SplitPlanesSdpa& sp) {
  size_t qo[2], ko[6];
  int T, Lkt;
  const size_t qbytes = q_planes_layout(BH, Lq, qo);
  const size_t kvbytes = kv_planes_layout(BH, Lk, ko, T, Lkt);
  uint8_t* ws = static_cast<uint8_t*>(workspace(qbytes + kvbytes, stream));
  if (!ws) return kWorkspace;
  planes_from(ws, ws + qbytes, BH, Lq, Lk, sp);
  return kOk;
}

// Shared-memory opt-in of the fused split kernels, once per device.
static void ensure_qkv_split_attr() {
  using namespace sdpa;
  static std::atomic<uint64_t> attr_done{0};  // one bit per device ordinal
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_done.load(std::memory_order_acquire) >> (dev & 63) & 1)) {
    cudaFuncSetAttribute(qkv_split_k<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, QKV_SPLIT_SMEM);
    cudaFuncSetAttribute(qkv_split_k<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, QKV_SPLIT_SMEM);
    attr_done.fetch_or(1ull << (dev & 63), std::memory_order_acq_rel);
  }
}

// Output in the NF24 GEMM's split format (hi == nullptr: fp32 output).
struct OutSplit {
  __half* hi = nullptr;
  __half* lo = nullptr;
  float* rs = nullptr;
};

// out_split: a split buffer of the [B * Lq, H * 64] output (256-byte aligned)
static OutSplit out_split_of(void* out_split, int64_t B, int Lq, int H) {
  const SplitLayout l = split_buffer_layout((int)(B * Lq), H * sdpa::D);
  uint8_t* base = static_cast<uint8_t*>(out_split);
  OutSplit o;
  o.hi = reinterpret_cast<__half*>(base);
  o.lo = reinterpret_cast<__half*>(base + l.lo_offset);
  o.rs = reinterpret_cast<float*>(base + l.rs_offset);
  return o;
}

// The attention kernel on split planes.
static int sdpa_attend(const SplitPlanesSdpa& sp, const float* bias, int64_t bias_bh_stride,
                       float* out, int64_t BH, int H, int Lq, int Lk, int out_blhd,
                       cudaStream_t stream, const OutSplit& osplit = OutSplit()) {
  using namespace sdpa;
  CUtensorMap m_qhi, m_qlo, m_khi, m_klo, m_vhi, m_vlo;
  const uint32_t box_rows[3] = {64, 128, 1};
  const uint32_t box_vt[3] = {64, 64, 1};
  {
    // Q planes [BH][Lq][64]: 128-row tiles, rows past Lq of a head read as zeros
    const uint64_t dims[3] = {D, (uint64_t)Lq, (uint64_t)BH};
    const uint64_t strides[2] = {D * 2, (uint64_t)Lq * D * 2};
    if (!encode_tmap(&m_qhi, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, sp.qhi, dims, strides, box_rows, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_tmap(&m_qlo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, sp.qlo, dims, strides, box_rows, CU_TENSOR_MAP_SWIZZLE_128B))
      return kLaunchFailed;
  }
  {
    const uint64_t dims[3] = {D, (uint64_t)sp.Lkt, (uint64_t)BH};
    const uint64_t strides[2] = {D * 2, (uint64_t)sp.Lkt * D * 2};
    if (!encode_tmap(&m_khi, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, sp.khi, dims, strides, box_rows, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_tmap(&m_klo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, sp.klo, dims, strides, box_rows, CU_TENSOR_MAP_SWIZZLE_128B))
      return kLaunchFailed;
  }
  {
    const uint64_t dims[3] = {(uint64_t)sp.Lkt, D, (uint64_t)BH};
    const uint64_t strides[2] = {(uint64_t)sp.Lkt * 2, (uint64_t)sp.Lkt * D * 2};
    if (!encode_tmap(&m_vhi, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, sp.vhi, dims, strides, box_vt, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_tmap(&m_vlo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, sp.vlo, dims, strides, box_vt, CU_TENSOR_MAP_SWIZZLE_128B))
      return kLaunchFailed;
  }
  {
    static std::atomic<uint64_t> attr_done{0};  // one bit per device ordinal
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(attr_done.load(std::memory_order_acquire) >> (dev & 63) & 1)) {
      // the warpgroups' setmaxnreg budgets add up to the launch allocation of a kernel
      // compiled with REGS_LAUNCH registers per thread; with fewer, an increase would wait
      // for ever, so refuse to launch instead
      cudaFuncAttributes fa{};
      if (cudaFuncGetAttributes(&fa, sdpa_fwd_tc) != cudaSuccess || fa.numRegs < (int)REGS_LAUNCH) {
        set_last_error("sdpa_fwd_tc was compiled with fewer registers than its warpgroup budget needs");
        return kLaunchFailed;
      }
      cudaFuncSetAttribute(sdpa_fwd_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
      cudaFuncSetAttribute(qkv_split_k<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, QKV_SPLIT_SMEM);
      cudaFuncSetAttribute(qkv_split_k<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, QKV_SPLIT_SMEM);
      attr_done.fetch_or(1ull << (dev & 63), std::memory_order_acq_rel);
    }
  }
  const int Qt = (Lq + BQ - 1) / BQ;
  Params prm{sp.qinv, sp.kinv, sp.vinv, bias, (long long)bias_bh_stride, out, H, Lq, Lk, sp.T, out_blhd,
             device_status(), Qt, (int)BH, osplit.hi, osplit.lo, osplit.rs};
  // persistent: one CTA per SM walking the (head, query tile) items
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
  const long long items = (long long)Qt * BH;
  const dim3 grid((unsigned)(items < sms ? items : sms));
  {
    LaunchScope scope(kKSdpaAttn, stream);
    sdpa_fwd_tc<<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(m_qhi, m_qlo, m_khi, m_klo, m_vhi, m_vlo, prm);
  }
  return launch_status();
}

// k/v element (bh, j, d) at base + bh*bh_stride + j*j_stride + d*d_stride
static int sdpa_launch(const float* q, const float* k, const float* v, int64_t bh_stride,
                       int64_t j_stride, int64_t d_stride, const float* bias,
                       int64_t bias_bh_stride, float* out, int B, int H, int Lq, int Lk,
                       int out_blhd) {
  using namespace sdpa;
  const uint64_t t0 = now_ns();
  int st = entry_check();
  if (st != kOk) return st;
  if (!is_device_pointer(q) || !is_device_pointer(k) || !is_device_pointer(v) ||
      !is_device_pointer(out) || (bias && !is_device_pointer(bias)))
    return kNotDevicePointer;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 15) return kBadAlignment;
  cudaStream_t stream = current_stream();
  const int64_t BH = (int64_t)B * H;
  SplitPlanesSdpa sp;
  if ((st = sdpa_planes(BH, Lq, Lk, stream, sp)) != kOk) return st;
  const int64_t qrows = BH * Lq;
  {
    LaunchScope scope(kKSdpaSplit, stream);
    sdpa_split_q<<<(unsigned)((qrows + 7) / 8), 256, 0, stream>>>(q, qrows, sp.qhi, sp.qlo, sp.qinv);
  }
  {
    LaunchScope scope(kKSdpaSplit, stream);
    sdpa_split_kv<<<dim3(sp.T, (unsigned)BH), 256, 0, stream>>>(k, v, bh_stride, j_stride, d_stride, Lk,
                                                                sp.Lkt, sp.khi, sp.klo, sp.vhi, sp.vlo,
                                                                sp.kinv, sp.vinv);
  }
  if ((st = launch_status()) != kOk) return st;
  const uint64_t t1 = now_ns();
  st = sdpa_attend(sp, bias, bias_bh_stride, out, BH, H, Lq, Lk, out_blhd, stream);
  const uint64_t t2 = now_ns();
  g_sdpa.calls += 1;
  g_sdpa.split_ns += t1 - t0;
  g_sdpa.attn_ns += t2 - t1;
  return st;
}

// Fused post-process + split, then the attention (BLHD output).  qsrc / kvsrc / freqs /
// sel as qkv_split_k; frequency rows: fb batches of [Lk, H, 64].
template <bool kSelected>
static int qkv_sdpa_launch(const float* qsrc, const float* kvsrc, const float* freqs,
                           const int64_t* sel, const float* qg, const float* kg, float* out_blhd,
                           int B, int H, int Lq, int Lk, int fb, void* out_split = nullptr) {
  using namespace sdpa;
  int st = entry_check();
  if (st != kOk) return st;
  void* out = out_split ? out_split : static_cast<void*>(out_blhd);
  if (!is_device_pointer(kvsrc) || !is_device_pointer(qg) || !is_device_pointer(kg) ||
      !is_device_pointer(out) || (qsrc && !is_device_pointer(qsrc)) ||
      (freqs && !is_device_pointer(freqs)))
    return kNotDevicePointer;
  if ((reinterpret_cast<uintptr_t>(kvsrc) | reinterpret_cast<uintptr_t>(out) |
       reinterpret_cast<uintptr_t>(qsrc) | reinterpret_cast<uintptr_t>(freqs) |
       reinterpret_cast<uintptr_t>(qg) | reinterpret_cast<uintptr_t>(kg)) & 15)
    return kBadAlignment;
  if (out_split && (reinterpret_cast<uintptr_t>(out_split) & 255)) return kBadAlignment;
  cudaStream_t stream = current_stream();
  const int64_t BH = (int64_t)B * H;
  SplitPlanesSdpa sp;
  if ((st = sdpa_planes(BH, Lq, Lk, stream, sp)) != kOk) return st;
  // the fused kernel's shared-memory opt-in before its first launch on this device
  ensure_qkv_split_attr();
  const int q_tiles = (Lq + BKV - 1) / BKV;
  // key tiles (with, for self-attention, the query rows of the same tokens) through the
  // shared-memory V staging; selected queries in their own kernel without shared memory
  {
    LaunchScope scope(kKSdpaSplit, stream);
    qkv_split_k<kSelected><<<dim3((unsigned)BH, sp.T), 256, QKV_SPLIT_SMEM, stream>>>(
        qsrc, kvsrc, freqs, sel, qg, kg, H, Lq, Lk, sp.Lkt, fb, 0, 0, Lk, 0, sp.qhi, sp.qlo, sp.qinv,
        sp.khi, sp.klo, sp.vhi, sp.vlo, sp.kinv, sp.vinv);
  }
  if (kSelected) {
    LaunchScope scope(kKSdpaSplit, stream);
    selected_q_split_k<<<dim3((unsigned)BH, q_tiles), 256, 0, stream>>>(
        qsrc, freqs, sel, qg, H, Lq, Lk, fb, sp.qhi, sp.qlo, sp.qinv);
  }
  if ((st = launch_status()) != kOk) return st;
  return sdpa_attend(sp, nullptr, 0, out_blhd, BH, H, Lq, Lk, 1, stream,
                     out_split ? out_split_of(out_split, B, Lq, H) : OutSplit());
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace tsb

// ---------------------------------------------------------------------------
// C-ABI.  Same names, argument lists and status codes as the reference SDPA
// libraries; pointers are CUDA device pointers, `threads` is ignored, work is
// queued on the stream set by triposplat_b200_set_stream.
// ---------------------------------------------------------------------------
extern "C" {

// scripts/native_sdpa_avx512_exact_q8t512.c:137-166 (q/k/v/out [B,H,L,64]; bias [Lk] shared)
int triposplat_sdpa_f32_avx512_exact_q8t512(const float* q, const float* k, const float* v,
                                            const float* key_bias_or_null, float* out, int B,
                                            int H, int Lq, int Lk, int D, int has_key_bias,
                                            int key_bias_len, int threads) {
  (void)threads;
  if (!q || !k || !v || !out) return tsb::kNullPointer;
  if (B <= 0 || H <= 0 || Lq <= 0 || Lk <= 0 || D != 64) return tsb::kBadDims;
  if (has_key_bias && (!key_bias_or_null || key_bias_len != Lk)) return tsb::kBadRange;
  return tsb::sdpa_launch(q, k, v, (int64_t)Lk * 64, 64, 1,
                          has_key_bias ? key_bias_or_null : nullptr, 0, out, B, H, Lq, Lk, 0);
}

// scripts/native_sdpa_avx512_exact_q8t512.c:334-351 (alias)
int triposplat_sdpa_f32(const float* q, const float* k, const float* v, const float* bias,
                        float* out, int B, int H, int Lq, int Lk, int D, int has_key_bias,
                        int key_bias_len, int threads) {
  return triposplat_sdpa_f32_avx512_exact_q8t512(q, k, v, bias, out, B, H, Lq, Lk, D,
                                                 has_key_bias, key_bias_len, threads);
}

// scripts/native_sdpa_avx512_exact_q8.c:52 (the strict-baseline kernel's symbol, same math)
int triposplat_sdpa_f32_avx512_exact_q8(const float* q, const float* k, const float* v,
                                        const float* bias, float* out, int B, int H, int Lq,
                                        int Lk, int D, int has_key_bias, int key_bias_len,
                                        int threads) {
  return triposplat_sdpa_f32_avx512_exact_q8t512(q, k, v, bias, out, B, H, Lq, Lk, D,
                                                 has_key_bias, key_bias_len, threads);
}

// scripts/native_sdpa_avx512_exact_q8t512_packed.c:3-21 (packed K/V [B,H,64,Lkp], out [B,Lq,H,64])
int triposplat_sdpa_f32_avx512_exact_q8t512_packed_blhd(
    const float* q, const float* packed_k, const float* packed_v, const float* key_bias_or_null,
    float* out_blhd, int B, int H, int Lq, int Lk, int D, int Lkp, int has_key_bias,
    int key_bias_len, int threads) {
  (void)threads;
  if (!q || !packed_k || !packed_v || !out_blhd) return tsb::kNullPointer;
  if (B <= 0 || H <= 0 || Lq <= 0 || Lk <= 0 || D != 64 || Lkp < Lk || (Lkp & 15) != 0)
    return tsb::kBadDims;
  if (has_key_bias && (!key_bias_or_null || key_bias_len != Lk)) return tsb::kBadRange;
  return tsb::sdpa_launch(q, packed_k, packed_v, (int64_t)64 * Lkp, 1, Lkp,
                          has_key_bias ? key_bias_or_null : nullptr, 0, out_blhd, B, H, Lq, Lk, 1);
}

// scripts/native_sdpa_avx512_exact_q8t512_packed.c:160-162
int triposplat_sdpa_packed_output_is_blhd(void) { return 1; }

// No reference counterpart: per-(b,h) key bias [B*H, Lk] (bias_bh_stride elements apart,
// 0 = one shared [Lk] row) and a choice of BHLD (0) or BLHD (1) output.
int triposplat_sdpa_f32_cuda_bias_bh(const float* q, const float* k, const float* v,
                                     const float* bias, long long bias_bh_stride, float* out,
                                     int B, int H, int Lq, int Lk, int out_blhd) {
  if (!q || !k || !v || !out) return tsb::kNullPointer;
  if (B <= 0 || H <= 0 || Lq <= 0 || Lk <= 0 || bias_bh_stride < 0) return tsb::kBadDims;
  if (bias && bias_bh_stride != 0 && bias_bh_stride < Lk) return tsb::kBadRange;
  return tsb::sdpa_launch(q, k, v, (int64_t)Lk * 64, 64, 1, bias, bias_bh_stride, out, B, H, Lq,
                          Lk, out_blhd ? 1 : 0);
}

// No reference counterpart: the reference's QKV post-process followed by its packed SDPA
// (scripts/native_qkv_postprocess_v2_avx512.c:45-105, then
// scripts/native_sdpa_avx512_exact_q8t512_packed.c:3-158) in one call: qkv [B, L, 3, H, 64]
// -> attention output [B, L, H, 64], with q / k / v going straight to the attention's split
// format (same results bit for bit as the two calls, without their fp32 intermediates).
int triposplat_b200_qkv_rope_rmsnorm_sdpa_f32(const float* qkv, const float* frequencies,
                                              const float* q_gamma, const float* k_gamma,
                                              float* out_blhd, int B, int L, int H, int D,
                                              int frequency_batches) {
  if (!qkv || !frequencies || !q_gamma || !k_gamma || !out_blhd) return tsb::kNullPointer;
  if (B <= 0 || L <= 0 || H <= 0 || D != 64 || (frequency_batches != 1 && frequency_batches != B))
    return tsb::kBadDims;
  return tsb::qkv_sdpa_launch<false>(nullptr, qkv, frequencies, nullptr, q_gamma, k_gamma, out_blhd,
                                     B, H, L, L, frequency_batches);
}

// No reference counterpart: triposplat_b200_q_kv_rmsnorm_pack_f32 (per-head RMSNorm of q
// [B, Lq, H, 64] and of the keys of kv [B, Lk, 2, H, 64], no RoPE) followed by the packed
// SDPA, in one call with the split format written directly (cross-attention).
int triposplat_b200_q_kv_rmsnorm_sdpa_f32(const float* q, const float* kv, const float* q_gamma,
                                          const float* k_gamma, float* out_blhd, int B, int Lq,
                                          int Lk, int H) {
  if (!q || !kv || !q_gamma || !k_gamma || !out_blhd) return tsb::kNullPointer;
  if (B <= 0 || Lq <= 0 || Lk <= 0 || H <= 0) return tsb::kBadDims;
  return tsb::qkv_sdpa_launch<true>(q, kv, nullptr, nullptr, q_gamma, k_gamma, out_blhd, B, H, Lq, Lk, 1);
}

// No reference counterpart: triposplat_b200_qkv_rope_rmsnorm_sdpa_f32 (D = 64) with the
// output written into out_split, a split buffer (triposplat_b200_split_bytes(B * L, H * 64)
// bytes, 256-byte aligned) of the [B * L, H * 64] attention output: the out-projection's
// GEMM input without an fp32 round trip.  Row scales: 2^-s with s fixed per batch from the
// largest V value (so every |O| * 2^s < 2^15); the planes equal the split of the fp32
// output under those scales.
int triposplat_b200_qkv_rope_rmsnorm_sdpa_split(const float* qkv, const float* frequencies,
                                                const float* q_gamma, const float* k_gamma, int B,
                                                int L, int H, int frequency_batches,
                                                void* out_split) {
  if (!qkv || !frequencies || !q_gamma || !k_gamma || !out_split) return tsb::kNullPointer;
  if (B <= 0 || L <= 0 || H <= 0 || (frequency_batches != 1 && frequency_batches != B))
    return tsb::kBadDims;
  return tsb::qkv_sdpa_launch<false>(nullptr, qkv, frequencies, nullptr, q_gamma, k_gamma, nullptr,
                                     B, H, L, L, frequency_batches, out_split);
}

// No reference counterpart: triposplat_b200_q_kv_rmsnorm_sdpa_f32 with the output written
// into a split buffer of [B * Lq, H * 64] (as triposplat_b200_qkv_rope_rmsnorm_sdpa_split).
int triposplat_b200_q_kv_rmsnorm_sdpa_split(const float* q, const float* kv, const float* q_gamma,
                                            const float* k_gamma, int B, int Lq, int Lk, int H,
                                            void* out_split) {
  if (!q || !kv || !q_gamma || !k_gamma || !out_split) return tsb::kNullPointer;
  if (B <= 0 || Lq <= 0 || Lk <= 0 || H <= 0) return tsb::kBadDims;
  return tsb::qkv_sdpa_launch<true>(q, kv, nullptr, nullptr, q_gamma, k_gamma, nullptr, B, H, Lq, Lk,
                                    1, out_split);
}

// ---- query-row sharding (no reference counterpart) -------------------------------------
// A group of ranks splits one sequence of L tokens by query rows: rank r owns the tokens
// [starts[r], starts[r+1]) (interior starts multiples of the 128-token key tile).  Per
// attention: each rank splits its own tokens (triposplat_b200_qkv_split_rows_f32: Q planes
// of its rows, its key tiles of the shared K / V plane layout), the ranks pass a peer
// barrier, each pulls the other ranks' key tiles (triposplat_b200_kv_planes_gather), and
// attends its query rows to all L keys (triposplat_b200_attend_rows_f32).  Every query row
// sees the same split planes, tiles and warps as in the unsharded call: the outputs are
// bit-identical to triposplat_b200_qkv_rope_rmsnorm_sdpa_f32 on the whole sequence.

// Bytes of the Q planes of Lq rows x BH heads / of the K / V planes of Lk keys x BH heads.
uint64_t triposplat_b200_attn_q_planes_bytes(int BH, int Lq) {
  if (BH <= 0 || Lq <= 0) return 0;
  size_t off[2];
  return tsb::q_planes_layout(BH, Lq, off);
}

uint64_t triposplat_b200_attn_kv_planes_bytes(int BH, int Lk) {
  if (BH <= 0 || Lk <= 0) return 0;
  size_t off[6];
  int T, Lkt;
  return tsb::kv_planes_layout(BH, Lk, off, T, Lkt);
}

// RoPE + per-head RMSNorm + split of tokens [t0, t1) of an L-token sequence: qkv_rows
// [B, t1 - t0, 3, H, 64] (this rank's rows), frequencies [fb, L, H, 64] (the whole
// sequence's table).  Writes the Q planes of the t1 - t0 rows into q_planes and key tiles
// [t0 / 128, ceil(t1 / 128)) into the K / V plane set kv_planes (layout of
// triposplat_b200_attn_kv_planes_bytes(B * H, L)).  t0 % 128 == 0; t1 % 128 == 0 or t1 == L.
int triposplat_b200_qkv_split_rows_f32(const float* qkv_rows, const float* frequencies,
                                       const float* q_gamma, const float* k_gamma, int B, int L,
                                       int H, int t0, int t1, int frequency_batches, void* q_planes,
                                       void* kv_planes) {
  using namespace tsb;
  using namespace tsb::sdpa;
  if (!qkv_rows || !frequencies || !q_gamma || !k_gamma || !q_planes || !kv_planes) return kNullPointer;
  if (B <= 0 || L <= 0 || H <= 0 || (frequency_batches != 1 && frequency_batches != B)) return kBadDims;
  if (t0 < 0 || t1 <= t0 || t1 > L || (t0 % BKV) != 0 || ((t1 % BKV) != 0 && t1 != L)) return kBadRange;
  if (!aligned16(qkv_rows) || !aligned16(frequencies) || !aligned16(q_gamma) || !aligned16(k_gamma) ||
      (reinterpret_cast<uintptr_t>(q_planes) & 255) || (reinterpret_cast<uintptr_t>(kv_planes) & 255))
    return kBadAlignment;
  int st = entry_check();
  if (st != kOk) return st;
  if (!is_device_pointer(qkv_rows) || !is_device_pointer(frequencies) || !is_device_pointer(q_gamma) ||
      !is_device_pointer(k_gamma) || !is_device_pointer(q_planes) || !is_device_pointer(kv_planes))
    return kNotDevicePointer;
  const int64_t BH = (int64_t)B * H;
  const int Lq = t1 - t0;
  SplitPlanesSdpa sp;
  planes_from(static_cast<uint8_t*>(q_planes), static_cast<uint8_t*>(kv_planes), BH, Lq, L, sp);
  ensure_qkv_split_attr();
  cudaStream_t stream = current_stream();
  const int tile0 = t0 / BKV, tiles = (t1 + BKV - 1) / BKV - tile0;
  {
    LaunchScope scope(kKSdpaSplit, stream);
    qkv_split_k<false><<<dim3((unsigned)BH, tiles), 256, QKV_SPLIT_SMEM, stream>>>(
        nullptr, qkv_rows, frequencies, nullptr, q_gamma, k_gamma, H, Lq, L, sp.Lkt,
        frequency_batches, tile0, t0, Lq, t0, sp.qhi, sp.qlo, sp.qinv, sp.khi, sp.klo, sp.vhi,
        sp.vlo, sp.kinv, sp.vinv);
  }
  return launch_status();
}

// Copy the other ranks' key tiles into this rank's K / V plane set.  kv_planes_by_rank[r]:
// rank r's set as mapped in this process (this rank's own set at [rank]); token_starts:
// world + 1 entries, 0 = token_starts[0] < ... < token_starts[world] = L, interior entries
// multiples of 128.  The caller orders it after a barrier that follows every rank's split.
int triposplat_b200_kv_planes_gather(const uint64_t* kv_planes_by_rank, const int* token_starts,
                                     int world, int rank, int BH, int L) {
  using namespace tsb;
  using namespace tsb::sdpa;
  if (!kv_planes_by_rank || !token_starts) return kNullPointer;
  if (world < 1 || world > kMaxGatherRanks || BH <= 0 || L <= 0) return kBadDims;
  if (rank < 0 || rank >= world) return kBadRange;
  if (token_starts[0] != 0 || token_starts[world] != L) return kBadRange;
  KvGather g{};
  int T, Lkt;
  size_t off[6];
  tsb::kv_planes_layout(BH, L, off, T, Lkt);
  for (int i = 0; i < 6; ++i) g.off[i] = off[i];
  for (int r = 0; r < world; ++r) {
    const int a = token_starts[r], b = token_starts[r + 1];
    if (b <= a || (a % BKV) != 0) return kBadRange;
    if (!kv_planes_by_rank[r]) return kNullPointer;
    if (kv_planes_by_rank[r] & 255) return kBadAlignment;
    g.src[r] = reinterpret_cast<const uint8_t*>(kv_planes_by_rank[r]);
    g.tlo[r] = a / BKV;
    g.thi[r] = (b + BKV - 1) / BKV;
  }
  int st = entry_check();
  if (st != kOk) return st;
  cudaStream_t stream = current_stream();
  if (world > 1) {
    LaunchScope scope(kKPeerCopy, stream);
    kv_gather_k<<<dim3(16, (unsigned)BH, (unsigned)world), 256, 0, stream>>>(
        g, reinterpret_cast<uint8_t*>(kv_planes_by_rank[rank]), rank, Lkt, T);
  }
  return launch_status();
}

// Exact attention of Lq query rows (q_planes, from triposplat_b200_qkv_split_rows_f32) to the
// L keys of a complete K / V plane set; output [B, Lq, H, 64] (BLHD).
int triposplat_b200_attend_rows_f32(const void* q_planes, const void* kv_planes, float* out_blhd,
                                    int B, int H, int Lq, int L) {
  using namespace tsb;
  if (!q_planes || !kv_planes || !out_blhd) return kNullPointer;
  if (B <= 0 || H <= 0 || Lq <= 0 || L <= 0) return kBadDims;
  if ((reinterpret_cast<uintptr_t>(q_planes) & 255) || (reinterpret_cast<uintptr_t>(kv_planes) & 255) ||
      !aligned16(out_blhd))
    return kBadAlignment;
  int st = entry_check();
  if (st != kOk) return st;
  if (!is_device_pointer(q_planes) || !is_device_pointer(kv_planes) || !is_device_pointer(out_blhd))
    return kNotDevicePointer;
  const int64_t BH = (int64_t)B * H;
  SplitPlanesSdpa sp;
  planes_from(static_cast<uint8_t*>(const_cast<void*>(q_planes)),
              static_cast<uint8_t*>(const_cast<void*>(kv_planes)), BH, Lq, L, sp);
  return sdpa_attend(sp, nullptr, 0, out_blhd, BH, H, Lq, L, 1, current_stream());
}

// triposplat_b200_attend_rows_f32 with the output written into a split buffer of
// [B * Lq, H * 64] (as triposplat_b200_qkv_rope_rmsnorm_sdpa_split).
int triposplat_b200_attend_rows_split(const void* q_planes, const void* kv_planes, int B, int H,
                                      int Lq, int L, void* out_split) {
  using namespace tsb;
  if (!q_planes || !kv_planes || !out_split) return kNullPointer;
  if (B <= 0 || H <= 0 || Lq <= 0 || L <= 0) return kBadDims;
  if ((reinterpret_cast<uintptr_t>(q_planes) & 255) || (reinterpret_cast<uintptr_t>(kv_planes) & 255) ||
      (reinterpret_cast<uintptr_t>(out_split) & 255))
    return kBadAlignment;
  int st = entry_check();
  if (st != kOk) return st;
  if (!is_device_pointer(q_planes) || !is_device_pointer(kv_planes) || !is_device_pointer(out_split))
    return kNotDevicePointer;
  const int64_t BH = (int64_t)B * H;
  SplitPlanesSdpa sp;
  planes_from(static_cast<uint8_t*>(const_cast<void*>(q_planes)),
              static_cast<uint8_t*>(const_cast<void*>(kv_planes)), BH, Lq, L, sp);
  return sdpa_attend(sp, nullptr, 0, nullptr, BH, H, Lq, L, 1, current_stream(),
                     out_split_of(out_split, B, Lq, H));
}

// ---- cached condition keys (no reference counterpart) ----------------------------------
// The condition tokens do not change across sampler steps, so their keys / values are split
// once per image (triposplat_b200_kv_split_f32: per-head RMSNorm of the keys, values as
// they are) into a K / V plane set that every step's cross-attention reads; per step only
// the queries are split (triposplat_b200_q_split_f32) before triposplat_b200_attend_rows_f32.
// The three calls run the kernels of triposplat_b200_q_kv_rmsnorm_sdpa_f32 with the same
// arguments: bit-identical outputs.

// kv [B, Lk, 2, H, 64] -> kv_planes (layout of triposplat_b200_attn_kv_planes_bytes(B * H, Lk))
int triposplat_b200_kv_split_f32(const float* kv, const float* k_gamma, int B, int Lk, int H,
                                 void* kv_planes) {
  using namespace tsb;
  using namespace tsb::sdpa;
  if (!kv || !k_gamma || !kv_planes) return kNullPointer;
  if (B <= 0 || Lk <= 0 || H <= 0) return kBadDims;
  if (!aligned16(kv) || !aligned16(k_gamma) || (reinterpret_cast<uintptr_t>(kv_planes) & 255))
    return kBadAlignment;
  int st = entry_check();
  if (st != kOk) return st;
  if (!is_device_pointer(kv) || !is_device_pointer(k_gamma) || !is_device_pointer(kv_planes))
    return kNotDevicePointer;
  const int64_t BH = (int64_t)B * H;
  size_t off[6];
  int T, Lkt;
  kv_planes_layout(BH, Lk, off, T, Lkt);
  uint8_t* base = static_cast<uint8_t*>(kv_planes);
  ensure_qkv_split_attr();
  cudaStream_t stream = current_stream();
  {
    LaunchScope scope(kKSdpaSplit, stream);
    qkv_split_k<true><<<dim3((unsigned)BH, T), 256, QKV_SPLIT_SMEM, stream>>>(
        nullptr, kv, nullptr, nullptr, k_gamma, k_gamma, H, 0, Lk, Lkt, 1, 0, 0, Lk, 0, nullptr,
        nullptr, nullptr, reinterpret_cast<__half*>(base + off[0]), reinterpret_cast<__half*>(base + off[1]),
        reinterpret_cast<__half*>(base + off[2]), reinterpret_cast<__half*>(base + off[3]),
        reinterpret_cast<float*>(base + off[4]), reinterpret_cast<float*>(base + off[5]));
  }
  return launch_status();
}

// q [B, Lq, H, 64] -> per-head RMSNorm (no rotation) into q_planes
// (layout of triposplat_b200_attn_q_planes_bytes(B * H, Lq))
int triposplat_b200_q_split_f32(const float* q, const float* q_gamma, int B, int Lq, int H,
                                void* q_planes) {
  using namespace tsb;
  using namespace tsb::sdpa;
  if (!q || !q_gamma || !q_planes) return kNullPointer;
  if (B <= 0 || Lq <= 0 || H <= 0) return kBadDims;
  if (!aligned16(q) || !aligned16(q_gamma) || (reinterpret_cast<uintptr_t>(q_planes) & 255))
    return kBadAlignment;
  int st = entry_check();
  if (st != kOk) return st;
  if (!is_device_pointer(q) || !is_device_pointer(q_gamma) || !is_device_pointer(q_planes))
    return kNotDevicePointer;
  const int64_t BH = (int64_t)B * H;
  size_t off[2];
  q_planes_layout(BH, Lq, off);
  uint8_t* base = static_cast<uint8_t*>(q_planes);
  cudaStream_t stream = current_stream();
  {
    LaunchScope scope(kKSdpaSplit, stream);
    selected_q_split_k<<<dim3((unsigned)BH, (Lq + BKV - 1) / BKV), 256, 0, stream>>>(
        q, nullptr, nullptr, q_gamma, H, Lq, Lq, 1, reinterpret_cast<__half*>(base),
        reinterpret_cast<__half*>(base + off[0]), reinterpret_cast<float*>(base + off[1]));
  }
  return launch_status();
}

// scripts/native_sdpa_avx512_exact_q8t512.c:64-70: tile sizes of this implementation
int triposplat_sdpa_key_tile(void) { return tsb::sdpa::BKV; }
int triposplat_sdpa_query_block(void) { return tsb::sdpa::BQ; }

// scripts/native_sdpa_avx512_exact_q8t512.c:77-100.  On the GPU the call is asynchronous:
// allocate_ns is 0, pack_ns is the host time to validate and enqueue the split kernels,
// compute_ns the host time to encode and enqueue the attention kernel, free_ns is 0.
void triposplat_sdpa_q8t512_profile_reset(void) { tsb::g_sdpa = tsb::SdpaCounters(); }

int triposplat_sdpa_q8t512_profile_get(uint64_t* calls, uint64_t* allocate_ns, uint64_t* pack_ns,
                                       uint64_t* compute_ns, uint64_t* free_ns) {
  if (!calls || !allocate_ns || !pack_ns || !compute_ns || !free_ns) return tsb::kNullPointer;
  *calls = tsb::g_sdpa.calls;
  *allocate_ns = 0;
  *pack_ns = tsb::g_sdpa.split_ns;
  *compute_ns = tsb::g_sdpa.attn_ns;
  *free_ns = 0;
  return 0;
}

// scripts/native_sdpa_avx512_exact_q8t512.c:51-62 -> the library-wide workspace
int triposplat_b200_workspace_stats(uint64_t* allocations, uint64_t* capacity_bytes);
void triposplat_b200_workspace_release(void);

int triposplat_sdpa_q8t512_workspace_stats(uint64_t* allocations, uint64_t* capacity_bytes) {
  return triposplat_b200_workspace_stats(allocations, capacity_bytes);
}

void triposplat_sdpa_q8t512_workspace_release(void) { triposplat_b200_workspace_release(); }

}  // extern "C"
