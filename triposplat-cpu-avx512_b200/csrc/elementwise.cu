// Prologue / epilogue kernels of the flow-model block, exported under the reference's
// symbol names and argument lists so the reference's strict patches bind unchanged:
//   LayerNorm, multi-head RMSNorm, complex RoPE   (scripts/native_norm_rope_avx512.c)
//   GELU(tanh), SiLU                              (scripts/native_gelu_avx512.c,
//                                                  scripts/native_silu_avx512_extra.c)
//   modulate / gated residual / add               (scripts/native_block_elementwise_avx512.c)
//   CFG combine / Euler update                    (scripts/native_sampler_avx512.c)
//   QKV RoPE -> RMSNorm -> K/V pack (v2, selected) (scripts/native_qkv_postprocess_v2_avx512.c)
// All are HBM-bound; they use coalesced 4- or 8-byte accesses, one warp per normalised
// vector, and grids sized in multiples of the SM count.  Pointers are device pointers.
#include <cuda_fp16.h>

#include <climits>

#include "common.cuh"
#include "runtime.h"

namespace tsb {
namespace ew {


inline unsigned grid_for(int64_t work, int per_block) {
  const int64_t blocks = (work + per_block - 1) / per_block;
  const int64_t cap = (int64_t)sm_count() * 16;
  return (unsigned)(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

// one warp per row; two-pass mean / biased variance like the reference (:26-37)
__global__ void layernorm_k(const float* __restrict__ in, const float* __restrict__ w,
                            const float* __restrict__ b, float* __restrict__ out, int64_t rows,
                            int cols, float eps, int affine) {
  const int lane = threadIdx.x & 31;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
       r += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const float* x = in + r * cols;
    float* y = out + r * cols;
    float s = 0.0f;
    for (int c = lane; c < cols; c += 32) s += x[c];
    const float mean = warp_sum(s) / (float)cols;
    float v = 0.0f;
    for (int c = lane; c < cols; c += 32) {
      const float d = x[c] - mean;
      v = fmaf(d, d, v);
    }
    const float inv = 1.0f / sqrtf(warp_sum(v) / (float)cols + eps);
    for (int c = lane; c < cols; c += 32) {
      float t = (x[c] - mean) * inv;
      if (affine) t = fmaf(t, w[c], b[c]);
      y[c] = t;
    }
  }
}

// one warp per vector: y = x * sqrt(dim)/max(||x||, eps) * gamma[head]  (:51-83)
__global__ void rmsnorm_k(const float* __restrict__ in, const float* __restrict__ gamma,
                          float* __restrict__ out, int64_t vectors, int heads, int dim,
                          float eps) {
  const int lane = threadIdx.x & 31;
  const float sd = sqrtf((float)dim);
  for (int64_t v = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); v < vectors;
       v += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const float* x = in + v * dim;
    const float* g = gamma + (int64_t)(v % heads) * dim;
    float ss = 0.0f;
    for (int d = lane; d < dim; d += 32) ss = fmaf(x[d], x[d], ss);
    const float f = sd / fmaxf(sqrtf(warp_sum(ss)), eps);
    for (int d = lane; d < dim; d += 32) out[v * dim + d] = x[d] * f * g[d];
  }
}

// interleaved complex multiply  (:85-110)
__global__ void rope_k(const float2* __restrict__ in, const float2* __restrict__ f,
                       float2* __restrict__ out, int64_t pairs) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < pairs;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float2 x = in[i], w = f[i];
    out[i] = make_float2(x.x * w.x - x.y * w.y, x.x * w.y + x.y * w.x);
  }
}

__device__ __forceinline__ float gelu_tanh(float x) {
  const float inner = 0.7978845608028654f * (x + 0.044715f * (x * x * x));
  return 0.5f * x * (1.0f + tanhf(inner));
}

__global__ void gelu_k(const float* __restrict__ in, float* __restrict__ out, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = gelu_tanh(in[i]);
}

__global__ void silu_k(const float* __restrict__ in, float* __restrict__ out, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = in[i] / (1.0f + expf(-in[i]));
}

// h = h*(1+scale[b]) + shift[b]
__global__ void modulate_k(float* __restrict__ h, const float* __restrict__ scale,
                           const float* __restrict__ shift, int64_t rows_per_batch, int cols,
                           int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols;
    const int c = (int)(i % cols);
    const int64_t bc = (r / rows_per_batch) * cols + c;
    h[i] = h[i] * (1.0f + scale[bc]) + shift[bc];
  }
}

// delta *= gate[b]; base += delta
__global__ void gated_residual_k(float* __restrict__ base, float* __restrict__ delta,
                                 const float* __restrict__ gate, int64_t rows_per_batch,
                                 int cols, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols;
    const int c = (int)(i % cols);
    const float d = delta[i] * gate[(r / rows_per_batch) * cols + c];
    delta[i] = d;
    base[i] = base[i] + d;
  }
}

__global__ void add_k(float* __restrict__ base, const float* __restrict__ delta, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    base[i] += delta[i];
}

// pos = g*pos - (g-1)*neg ; x = x - dt*v   (per batch scalars)
__global__ void cfg_k(float* __restrict__ pos, const float* __restrict__ neg,
                      const float* __restrict__ g, int64_t per_batch, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float gb = g[i / per_batch];
    // g*pos - (g-1)*neg with the reference's three roundings (no contraction)
    pos[i] = __fsub_rn(__fmul_rn(gb, pos[i]), __fmul_rn(__fsub_rn(gb, 1.0f), neg[i]));
  }
}

__global__ void euler_k(float* __restrict__ x, const float* __restrict__ v,
                        const float* __restrict__ dt, int64_t per_batch, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    x[i] = __fsub_rn(x[i], __fmul_rn(dt[i / per_batch], v[i]));
}

// x -= dt * ((1 + r) * v - r * v_prev), r = 0.5 * dt / max(dt_prev, 1e-12), each product and
// difference rounded separately (scripts/native_sampler_avx512.c:91-130)
__global__ void ab2_k(float* __restrict__ x, const float* __restrict__ v,
                      const float* __restrict__ v_prev, const float* __restrict__ dt,
                      const float* __restrict__ dt_prev, int64_t per_batch, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / per_batch;
    const float half_ratio = __fmul_rn(0.5f, __fdiv_rn(dt[b], fmaxf(dt_prev[b], 1.0e-12f)));
    const float cur_scale = __fadd_rn(1.0f, half_ratio);
    const float eff = __fsub_rn(__fmul_rn(cur_scale, v[i]), __fmul_rn(half_ratio, v_prev[i]));
    x[i] = __fsub_rn(x[i], __fmul_rn(dt[b], eff));
  }
}

// CFG combine then Euler step in one pass: x -= dt * (g*pos - (g-1)*neg), rounded exactly as
// the two reference kernels in sequence; `positive` is left unchanged.
__global__ void cfg_euler_k(float* __restrict__ x, const float* __restrict__ pos,
                            const float* __restrict__ neg, const float* __restrict__ g,
                            const float* __restrict__ dt, int64_t per_batch, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / per_batch;
    const float gb = g[b];
    const float v = __fsub_rn(__fmul_rn(gb, pos[i]), __fmul_rn(__fsub_rn(gb, 1.0f), neg[i]));
    x[i] = __fsub_rn(x[i], __fmul_rn(dt[b], v));
  }
}

// One CTA per (bh, 64-token tile).  Q rows go straight to [B,H,L,64]; K and V are
// staged in shared memory and written transposed to the packed [B,H,64,Lp] layout with
// coalesced stores (tail tokens L..Lp-1 are zero).
// Source element (b, token, s, h, d) for s in {q,k,v}: see the two layouts below.
template <bool kSelected>
__global__ void __launch_bounds__(256) qkv_post_k(
    const float* __restrict__ qsrc, const float* __restrict__ kvsrc, const float* __restrict__ freqs,
    const int64_t* __restrict__ sel, const float* __restrict__ qg, const float* __restrict__ kg,
    float* __restrict__ q_bhld, float* __restrict__ pk, float* __restrict__ pv, int H, int Lq,
    int Lk, int Lp, int fb, int kv_tiles) {
  __shared__ float kt[64][65];
  __shared__ float vt[64][65];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y, b = bh / H, h = bh % H;
  const int fbb = fb == 1 ? 0 : b;
  const int tile = blockIdx.x;
  const float2 gq = reinterpret_cast<const float2*>(qg + (int64_t)h * 64)[lane];
  const float2 gk = reinterpret_cast<const float2*>(kg + (int64_t)h * 64)[lane];
  if (tile < kv_tiles) {
    const int t0 = tile * 64;
    for (int i = warp; i < 64; i += 8) {
      const int t = t0 + i;
      float2 ky = make_float2(0.0f, 0.0f), vy = make_float2(0.0f, 0.0f);
      if (t < Lk) {
        const float* f = freqs ? freqs + (((int64_t)fbb * Lk + t) * H + h) * 64 : nullptr;
        const float* ks;
        const float* vs;
        if (kSelected) {  // kv [B, Lk, 2, H, 64]
          ks = kvsrc + (((int64_t)b * Lk + t) * 2 * H + h) * 64;
          vs = ks + (int64_t)H * 64;
        } else {  // qkv [B, L, 3, H, 64]
          ks = kvsrc + (((int64_t)b * Lk + t) * 3 * H + H + h) * 64;
          vs = ks + (int64_t)H * 64;
          const float2 qx = reinterpret_cast<const float2*>(ks - (int64_t)H * 64)[lane];
          const float2 qy = rope_rms64(qx, reinterpret_cast<const float2*>(f)[lane], gq);
          reinterpret_cast<float2*>(q_bhld + ((int64_t)bh * Lq + t) * 64)[lane] = qy;
        }
        ky = rope_rms64(reinterpret_cast<const float2*>(ks)[lane],
                        f ? reinterpret_cast<const float2*>(f)[lane] : make_float2(1.0f, 0.0f), gk);
        vy = reinterpret_cast<const float2*>(vs)[lane];
      }
      kt[2 * lane][i] = ky.x;
      kt[2 * lane + 1][i] = ky.y;
      vt[2 * lane][i] = vy.x;
      vt[2 * lane + 1][i] = vy.y;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < 64 * 64; e += 256) {
      const int d = e >> 6, i = e & 63;
      const int t = t0 + i;
      if (t < Lp) {
        pk[((int64_t)bh * 64 + d) * Lp + t] = kt[d][i];
        pv[((int64_t)bh * 64 + d) * Lp + t] = vt[d][i];
      }
    }
  }
  if (kSelected) {  // selected queries: q [B, Lq, H, 64], frequency row = sel[query]
    for (int i = warp; i < 64; i += 8) {
      const int qi = tile * 64 + i;
      if (qi >= Lq) break;
      float2 fr = make_float2(1.0f, 0.0f);  // no frequencies: identity rotation
      if (freqs) {
        const int64_t key = sel[qi];
        fr = reinterpret_cast<const float2*>(freqs + (((int64_t)fbb * Lk + key) * H + h) * 64)[lane];
      }
      const float2 qx = reinterpret_cast<const float2*>(qsrc + (((int64_t)b * Lq + qi) * H + h) * 64)[lane];
      reinterpret_cast<float2*>(q_bhld + ((int64_t)bh * Lq + qi) * 64)[lane] = rope_rms64(qx, fr, gq);
    }
  }
}

// sin and cos of x by the reference's own method (scripts/native_embeddings_avx512.c:12-56,
// the same in scripts/native_repo_avx512.c:12-56), operation for operation so results are
// bit-identical: q = x * 2/pi rounded to the nearest integer (ties to even; out of int32
// range or NaN -> INT_MIN, the AVX-512 conversion's indefinite value), r = x - q * pi/2 in
// two fused steps with pi/2 split into high and low parts, Taylor polynomials in z = r^2
// for sin (to r^13) and cos (to r^14) by Horner with fused multiply-adds, and the quadrant
// q & 3 selecting / negating the pair.  Explicit _rn intrinsics keep the compiler from
// contracting the separate multiplies and adds.
__device__ __forceinline__ void ref_sincos(float x, float& s_out, float& c_out) {
  const float t = __fmul_rn(x, 0.63661977236758134308f);
  const int q = fabsf(t) < 2147483648.0f ? __float2int_rn(t) : INT_MIN;
  const float qf = __int2float_rn(q);
  float r = __fmaf_rn(-qf, 1.57079625129699707031f, x);
  r = __fmaf_rn(-qf, 7.54978941586159635335e-8f, r);
  const float z = __fmul_rn(r, r);
  float sp = -1.0f / 6227020800.0f;
  sp = __fmaf_rn(sp, z, 1.0f / 39916800.0f);
  sp = __fmaf_rn(sp, z, -1.0f / 362880.0f);
  sp = __fmaf_rn(sp, z, 1.0f / 5040.0f);
  sp = __fmaf_rn(sp, z, -1.0f / 120.0f);
  sp = __fmaf_rn(sp, z, 1.0f / 6.0f);
  const float sin_r = __fsub_rn(r, __fmul_rn(__fmul_rn(r, z), sp));
  float cp = -1.0f / 87178291200.0f;
  cp = __fmaf_rn(cp, z, 1.0f / 479001600.0f);
  cp = __fmaf_rn(cp, z, -1.0f / 3628800.0f);
  cp = __fmaf_rn(cp, z, 1.0f / 40320.0f);
  cp = __fmaf_rn(cp, z, -1.0f / 720.0f);
  cp = __fmaf_rn(cp, z, 1.0f / 24.0f);
  cp = __fmaf_rn(cp, z, -0.5f);
  const float cos_r = __fmaf_rn(cp, z, 1.0f);
  const int quadrant = q & 3;
  s_out = quadrant == 0 ? sin_r : quadrant == 1 ? cos_r : quadrant == 2 ? -sin_r : -cos_r;
  c_out = quadrant == 0 ? cos_r : quadrant == 1 ? -sin_r : quadrant == 2 ? -cos_r : sin_r;
}

constexpr float kRefPi = 3.14159274101257324219f;

// [cos(t*f) | sin(t*f) | 0...] per sample  (scripts/native_embeddings_avx512.c:97-125)
__global__ void timestep_embed_k(const float* __restrict__ t, const float* __restrict__ f,
                                 float* __restrict__ out, int batch, int half, int out_dim) {
  const int b = blockIdx.x;
  if (b >= batch) return;
  for (int i = threadIdx.x; i < out_dim; i += blockDim.x) {
    float v = 0.0f;
    if (i < 2 * half) {
      float sn, cs;
      ref_sincos(__fmul_rn(t[b], f[i < half ? i : i - half]), sn, cs);
      v = i < half ? cs : sn;
    }
    out[(int64_t)b * out_dim + i] = v;
  }
}

// per row and axis [sin(a_0..a_{F-1}) | cos(a_0..)], a = x*f (doubled if double_pi) * pi,
// zero padding to `channels`  (scripts/native_embeddings_avx512.c:58-95)
__global__ void pcd_position_k(const float* __restrict__ pos, const float* __restrict__ f,
                               float* __restrict__ out, int64_t rows, int dims, int F,
                               int channels, int double_pi) {
  const int64_t n = rows * (int64_t)channels;
  const int used = dims * F * 2;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = e / channels;
    const int c = (int)(e - row * channels);
    float v = 0.0f;
    if (c < used) {
      const int axis = c / (2 * F), j = c - axis * 2 * F;
      const int i = j < F ? j : j - F;
      float angle = __fmul_rn(pos[row * dims + axis], f[i]);
      if (double_pi) angle = __fadd_rn(angle, angle);
      float sn, cs;
      ref_sincos(__fmul_rn(angle, kRefPi), sn, cs);
      v = j < F ? sn : cs;
    }
    out[e] = v;
  }
}

// RePo phasors: complex k of vector v on axis a: (cos, sin) of (x*ft + x*fr)*pi,
// x = delta[v, a]  (scripts/native_repo_avx512.c:85-129)
struct RepoFreqs {
  const float* ft[3];
  const float* fr[3];
  int dims[3];
};

__global__ void repo_phasor_k(const float* __restrict__ delta, RepoFreqs fq,
                              float2* __restrict__ out, int64_t vectors) {
  const int total = fq.dims[0] + fq.dims[1] + fq.dims[2];
  const int64_t n = vectors * (int64_t)total;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t v = e / total;
    int k = (int)(e - v * total), a = 0;
    if (k >= fq.dims[0]) { k -= fq.dims[0]; a = 1; if (k >= fq.dims[1]) { k -= fq.dims[1]; a = 2; } }
    const float x = delta[v * 3 + a];
    const float angle = __fmul_rn(__fadd_rn(__fmul_rn(x, fq.ft[a][k]), __fmul_rn(x, fq.fr[a][k])), kRefPi);
    float sn, cs;
    ref_sincos(angle, sn, cs);
    out[e] = make_float2(cs, sn);
  }
}

// lhs *= rhs  (scripts/native_repo_avx512.c:69-83)
__global__ void mul_k(float* __restrict__ lhs, const float* __restrict__ rhs, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    lhs[i] = __fmul_rn(lhs[i], rhs[i]);
}

}  // namespace ew

#define TSB_PREAMBLE()                      \
  do {                                      \
    const int _st = entry_check();          \
    if (_st != kOk) return _st;             \
  } while (0)

}  // namespace tsb

using namespace tsb;
using namespace tsb::ew;

extern "C" {

// scripts/native_norm_rope_avx512.c:13-49
int triposplat_layernorm_f32_avx512(const float* input, const float* weight, const float* bias,
                                    float* output, int64_t rows, int cols, float eps,
                                    int has_affine, int threads) {
  (void)threads;
  if (!input || !output) return kNullPointer;
  if (rows <= 0 || cols <= 0 || eps < 0.0f) return kBadDims;
  if (has_affine && (!weight || !bias)) return kBadRange;
  TSB_PREAMBLE();
  { LaunchScope _scope(kKElementwise, current_stream());
    layernorm_k<<<grid_for(rows, 8), 256, 0, current_stream()>>>(input, weight, bias, output, rows,
                                                               cols, eps, has_affine); }
  return launch_status();
}

// scripts/native_norm_rope_avx512.c:51-83
int triposplat_multihead_rmsnorm_f32_avx512(const float* input, const float* gamma, float* output,
                                            int64_t outer, int heads, int dim, float eps,
                                            int threads) {
  (void)threads;
  if (!input || !gamma || !output) return kNullPointer;
  if (outer <= 0 || heads <= 0 || dim <= 0 || eps < 0.0f) return kBadDims;
  TSB_PREAMBLE();
  const int64_t vectors = outer * heads;
  { LaunchScope _scope(kKElementwise, current_stream());
    rmsnorm_k<<<grid_for(vectors, 8), 256, 0, current_stream()>>>(input, gamma, output, vectors,
                                                                heads, dim, eps); }
  return launch_status();
}

// scripts/native_norm_rope_avx512.c:85-110
int triposplat_rope_complex_f32_avx512(const float* input, const float* freqs_interleaved,
                                       float* output, int64_t vectors, int dim, int threads) {
  (void)threads;
  if (!input || !freqs_interleaved || !output) return kNullPointer;
  if (vectors <= 0 || dim <= 0 || (dim & 1) != 0) return kBadDims;
  TSB_PREAMBLE();
  const int64_t pairs = vectors * dim / 2;
  { LaunchScope _scope(kKElementwise, current_stream());
    rope_k<<<grid_for(pairs, 256), 256, 0, current_stream()>>>(
      reinterpret_cast<const float2*>(input), reinterpret_cast<const float2*>(freqs_interleaved),
      reinterpret_cast<float2*>(output), pairs); }
  return launch_status();
}

// scripts/native_gelu_avx512.c:44-68
int triposplat_gelu_tanh_f32_avx512(const float* input, float* output, int64_t count, int threads) {
  (void)threads;
  if (!input || !output) return kNullPointer;
  if (count <= 0) return kBadDims;
  TSB_PREAMBLE();
  { LaunchScope _scope(kKElementwise, current_stream());
    gelu_k<<<grid_for(count, 256), 256, 0, current_stream()>>>(input, output, count); }
  return launch_status();
}

// scripts/native_silu_avx512_extra.c:28-45
int triposplat_silu_f32_avx512(const float* input, float* output, int64_t count, int threads) {
  (void)threads;
  if (!input || !output) return kNullPointer;
  if (count <= 0) return kBadDims;
  TSB_PREAMBLE();
  { LaunchScope _scope(kKElementwise, current_stream());
    silu_k<<<grid_for(count, 256), 256, 0, current_stream()>>>(input, output, count); }
  return launch_status();
}

// scripts/native_block_elementwise_avx512.c:9-22
int triposplat_modulate_inplace_f32_avx512(float* h, const float* scale, const float* shift,
                                           int batch, int rows, int cols, int threads) {
  (void)threads;
  if (!h || !scale || !shift) return kNullPointer;
  if (batch <= 0 || rows <= 0 || cols <= 0) return kBadDims;
  TSB_PREAMBLE();
  const int64_t n = (int64_t)batch * rows * cols;
  { LaunchScope _scope(kKElementwise, current_stream());
    modulate_k<<<grid_for(n, 256), 256, 0, current_stream()>>>(h, scale, shift, rows, cols, n); }
  return launch_status();
}

// scripts/native_block_elementwise_avx512.c:24-35
int triposplat_gated_residual_inplace_f32_avx512(float* base, float* delta, const float* gate,
                                                 int batch, int rows, int cols, int threads) {
  (void)threads;
  if (!base || !delta || !gate) return kNullPointer;
  if (batch <= 0 || rows <= 0 || cols <= 0) return kBadDims;
  TSB_PREAMBLE();
  const int64_t n = (int64_t)batch * rows * cols;
  { LaunchScope _scope(kKElementwise, current_stream());
    gated_residual_k<<<grid_for(n, 256), 256, 0, current_stream()>>>(base, delta, gate, rows, cols, n); }
  return launch_status();
}

// scripts/native_block_elementwise_avx512.c:37-46
int triposplat_add_inplace_f32_avx512(float* base, const float* delta, int64_t count, int threads) {
  (void)threads;
  if (!base || !delta) return kNullPointer;
  if (count <= 0) return kBadDims;
  TSB_PREAMBLE();
  { LaunchScope _scope(kKElementwise, current_stream());
    add_k<<<grid_for(count, 256), 256, 0, current_stream()>>>(base, delta, count); }
  return launch_status();
}

// scripts/native_sampler_avx512.c:19-54
int triposplat_cfg_combine_inplace_f32_avx512(float* positive, const float* negative,
                                              const float* guidance, int batch,
                                              int64_t elements_per_batch, int threads) {
  (void)threads;
  if (!positive || !negative || !guidance) return kNullPointer;
  if (batch <= 0 || elements_per_batch <= 0) return kBadDims;
  TSB_PREAMBLE();
  const int64_t n = (int64_t)batch * elements_per_batch;
  { LaunchScope _scope(kKElementwise, current_stream());
    cfg_k<<<grid_for(n, 256), 256, 0, current_stream()>>>(positive, negative, guidance,
                                                        elements_per_batch, n); }
  return launch_status();
}

// scripts/native_sampler_avx512.c:56-89
int triposplat_euler_update_inplace_f32_avx512(float* sample, const float* prediction,
                                               const float* dt, int batch,
                                               int64_t elements_per_batch, int threads) {
  (void)threads;
  if (!sample || !prediction || !dt) return kNullPointer;
  if (batch <= 0 || elements_per_batch <= 0) return kBadDims;
  TSB_PREAMBLE();
  const int64_t n = (int64_t)batch * elements_per_batch;
  { LaunchScope _scope(kKElementwise, current_stream());
    euler_k<<<grid_for(n, 256), 256, 0, current_stream()>>>(sample, prediction, dt,
                                                          elements_per_batch, n); }
  return launch_status();
}

// scripts/native_sampler_avx512.c:91-130
int triposplat_ab2_update_inplace_f32_avx512(float* sample, const float* prediction,
                                             const float* previous_prediction, const float* dt,
                                             const float* previous_dt, int batch,
                                             int64_t elements_per_batch, int threads) {
  (void)threads;
  if (!sample || !prediction || !previous_prediction || !dt || !previous_dt) return kNullPointer;
  if (batch <= 0 || elements_per_batch <= 0) return kBadDims;
  TSB_PREAMBLE();
  const int64_t n = (int64_t)batch * elements_per_batch;
  { LaunchScope _scope(kKElementwise, current_stream());
    ab2_k<<<grid_for(n, 256), 256, 0, current_stream()>>>(sample, prediction, previous_prediction,
                                                        dt, previous_dt, elements_per_batch, n); }
  return launch_status();
}

// No reference counterpart: triposplat_cfg_combine_inplace_f32_avx512 followed by
// triposplat_euler_update_inplace_f32_avx512 in one kernel (same results bit for bit;
// `positive` is not overwritten).  guidance and dt hold one value per batch entry.
int triposplat_b200_cfg_euler_update_f32(float* sample, const float* positive,
                                         const float* negative, const float* guidance,
                                         const float* dt, int batch, int64_t elements_per_batch) {
  if (!sample || !positive || !negative || !guidance || !dt) return kNullPointer;
  if (batch <= 0 || elements_per_batch <= 0) return kBadDims;
  TSB_PREAMBLE();
  const int64_t n = (int64_t)batch * elements_per_batch;
  { LaunchScope _scope(kKElementwise, current_stream());
    cfg_euler_k<<<grid_for(n, 256), 256, 0, current_stream()>>>(sample, positive, negative,
                                                              guidance, dt, elements_per_batch, n); }
  return launch_status();
}

// scripts/native_qkv_postprocess_v2_avx512.c:45-105
int triposplat_qkv_rope_rmsnorm_pack_f32_avx512_v2(const float* qkv, const float* frequencies,
                                                   const float* q_gamma, const float* k_gamma,
                                                   float* q_bhld, float* packed_k,
                                                   float* packed_v, int B, int L, int H, int D,
                                                   int L_padded, int frequency_batches,
                                                   int threads) {
  (void)threads;
  if (!qkv || !frequencies || !q_gamma || !k_gamma || !q_bhld || !packed_k || !packed_v)
    return kNullPointer;
  if (B <= 0 || L <= 0 || H <= 0 || D != 64 || L_padded < L || (L_padded & 15) != 0 ||
      (frequency_batches != 1 && frequency_batches != B))
    return kBadDims;
  TSB_PREAMBLE();
  const int tiles = (L_padded + 63) / 64;
  { LaunchScope _scope(kKElementwise, current_stream());
    qkv_post_k<false><<<dim3(tiles, B * H), 256, 0, current_stream()>>>(
      nullptr, qkv, frequencies, nullptr, q_gamma, k_gamma, q_bhld, packed_k, packed_v, H, L, L,
      L_padded, frequency_batches, tiles); }
  return launch_status();
}

// scripts/native_qkv_postprocess_avx512.c:23-116: the first version of the post-process,
// same arguments, checks and results as _v2 (it zeroes all of packed_k / packed_v before
// filling them, _v2 only their tails; every element ends with the same value)
int triposplat_qkv_rope_rmsnorm_pack_f32_avx512(const float* qkv, const float* frequencies,
                                                const float* q_gamma, const float* k_gamma,
                                                float* q_bhld, float* packed_k, float* packed_v,
                                                int B, int L, int H, int D, int L_padded,
                                                int frequency_batches, int threads) {
  return triposplat_qkv_rope_rmsnorm_pack_f32_avx512_v2(qkv, frequencies, q_gamma, k_gamma, q_bhld,
                                                        packed_k, packed_v, B, L, H, D, L_padded,
                                                        frequency_batches, threads);
}

// scripts/native_qkv_postprocess_avx512.c:118-120: tokens per work tile (64 here)
int triposplat_qkv_postprocess_token_tile(void) { return 64; }

// scripts/native_qkv_postprocess_v2_avx512.c:193-195: 1 = only the padded tail of the packed
// K / V rows is cleared (the rest is written)
int triposplat_qkv_postprocess_v2_tail_only_clear(void) { return 1; }

// scripts/native_qkv_postprocess_v2_avx512.c:107-191
int triposplat_q_kv_selected_rope_rmsnorm_pack_f32_avx512_v2(
    const float* q, const float* kv, const float* frequencies, const int64_t* selected_indices,
    const float* q_gamma, const float* k_gamma, float* q_bhld, float* packed_k, float* packed_v,
    int B, int Lq, int Lk, int H, int D, int Lk_padded, int frequency_batches, int threads) {
  (void)threads;
  if (!q || !kv || !frequencies || !selected_indices || !q_gamma || !k_gamma || !q_bhld ||
      !packed_k || !packed_v)
    return kNullPointer;
  if (B <= 0 || Lq <= 0 || Lk <= 0 || H <= 0 || D != 64 || Lk_padded < Lk ||
      (Lk_padded & 15) != 0 || (frequency_batches != 1 && frequency_batches != B))
    return kBadDims;
  TSB_PREAMBLE();
  // The reference validates every index on the host before computing (:128-130); the
  // indices live in device memory here, so they are copied back once for the same check.
  int64_t* host = static_cast<int64_t*>(malloc(sizeof(int64_t) * (size_t)Lq));
  if (!host) return kWorkspace;
  cudaStream_t s = current_stream();
  if (cudaMemcpyAsync(host, selected_indices, sizeof(int64_t) * (size_t)Lq, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess) {
    free(host);
    return kLaunchFailed;
  }
  for (int i = 0; i < Lq; ++i)
    if (host[i] < 0 || host[i] >= Lk) {
      free(host);
      return kBadRange;
    }
  free(host);
  const int kv_tiles = (Lk_padded + 63) / 64;
  const int q_tiles = (Lq + 63) / 64;
  const int tiles = kv_tiles > q_tiles ? kv_tiles : q_tiles;
  { LaunchScope _scope(kKElementwise, current_stream());
    qkv_post_k<true><<<dim3(tiles, B * H), 256, 0, s>>>(q, kv, frequencies, selected_indices,
                                                     q_gamma, k_gamma, q_bhld, packed_k, packed_v,
                                                     H, Lq, Lk, Lk_padded, frequency_batches,
                                                     kv_tiles); }
  return launch_status();
}

// scripts/native_embeddings_avx512.c:97-125
int triposplat_timestep_embedding_f32_avx512(const float* timesteps, const float* frequencies,
                                             float* output, int batch, int half_dim,
                                             int output_dim, int threads) {
  (void)threads;
  if (!timesteps || !frequencies || !output) return kNullPointer;
  if (batch <= 0 || half_dim <= 0 || output_dim < half_dim * 2) return kBadDims;
  TSB_PREAMBLE();
  { LaunchScope _scope(kKElementwise, current_stream());
    timestep_embed_k<<<batch, 256, 0, current_stream()>>>(timesteps, frequencies, output, batch,
                                                        half_dim, output_dim); }
  return launch_status();
}

// scripts/native_embeddings_avx512.c:58-95
int triposplat_pcd_position_embedding_f32_avx512(const float* positions, const float* frequencies,
                                                 float* output, int64_t rows, int input_dims,
                                                 int frequency_dim, int channels, int double_pi,
                                                 int threads) {
  (void)threads;
  if (!positions || !frequencies || !output) return kNullPointer;
  if (rows <= 0 || input_dims <= 0 || frequency_dim <= 0 ||
      channels < input_dims * frequency_dim * 2)
    return kBadDims;
  TSB_PREAMBLE();
  { LaunchScope _scope(kKElementwise, current_stream());
    pcd_position_k<<<grid_for(rows * (int64_t)channels, 256), 256, 0, current_stream()>>>(
        positions, frequencies, output, rows, input_dims, frequency_dim, channels, double_pi); }
  return launch_status();
}

// scripts/native_repo_avx512.c:69-83
int triposplat_mul_inplace_f32_avx512(float* lhs, const float* rhs, int64_t elements, int threads) {
  (void)threads;
  if (!lhs || !rhs) return kNullPointer;
  if (elements <= 0) return kBadDims;
  TSB_PREAMBLE();
  { LaunchScope _scope(kKElementwise, current_stream());
    mul_k<<<grid_for(elements, 256), 256, 0, current_stream()>>>(lhs, rhs, elements); }
  return launch_status();
}

// scripts/native_repo_avx512.c:85-129 (status -1 delta / output null, -2 a frequency null,
// -3 bad sizes, as the reference)
int triposplat_repo_phasor_f32_avx512(const float* delta, const float* freq_tanh_0,
                                      const float* freq_residual_0, int freq_dim_0,
                                      const float* freq_tanh_1, const float* freq_residual_1,
                                      int freq_dim_1, const float* freq_tanh_2,
                                      const float* freq_residual_2, int freq_dim_2,
                                      float* output_interleaved, int64_t vectors, int threads) {
  (void)threads;
  if (!delta || !output_interleaved) return -1;
  if (!freq_tanh_0 || !freq_residual_0 || !freq_tanh_1 || !freq_residual_1 || !freq_tanh_2 ||
      !freq_residual_2)
    return -2;
  if (vectors <= 0 || freq_dim_0 <= 0 || freq_dim_1 <= 0 || freq_dim_2 <= 0) return -3;
  TSB_PREAMBLE();
  RepoFreqs fq{{freq_tanh_0, freq_tanh_1, freq_tanh_2},
               {freq_residual_0, freq_residual_1, freq_residual_2},
               {freq_dim_0, freq_dim_1, freq_dim_2}};
  const int64_t n = vectors * (int64_t)(freq_dim_0 + freq_dim_1 + freq_dim_2);
  { LaunchScope _scope(kKElementwise, current_stream());
    repo_phasor_k<<<grid_for(n, 256), 256, 0, current_stream()>>>(
        delta, fq, reinterpret_cast<float2*>(output_interleaved), vectors); }
  return launch_status();
}

// No reference counterpart: the selected-query post-process without RoPE and without
// an index list (every query row kept): per-head 8/max(||x||,1e-12)*gamma on q and k,
// q -> [B,H,Lq,64], k/v -> packed [B,H,64,Lk_padded].  Used for cross-attention, whose
// condition tokens carry no position.
int triposplat_b200_q_kv_rmsnorm_pack_f32(const float* q, const float* kv, const float* q_gamma,
                                          const float* k_gamma, float* q_bhld, float* packed_k,
                                          float* packed_v, int B, int Lq, int Lk, int H,
                                          int Lk_padded) {
  if (!q || !kv || !q_gamma || !k_gamma || !q_bhld || !packed_k || !packed_v) return kNullPointer;
  if (B <= 0 || Lq <= 0 || Lk <= 0 || H <= 0 || Lk_padded < Lk || (Lk_padded & 15) != 0)
    return kBadDims;
  TSB_PREAMBLE();
  const int kv_tiles = (Lk_padded + 63) / 64;
  const int q_tiles = (Lq + 63) / 64;
  const int tiles = kv_tiles > q_tiles ? kv_tiles : q_tiles;
  { LaunchScope _scope(kKElementwise, current_stream());
    qkv_post_k<true><<<dim3(tiles, B * H), 256, 0, current_stream()>>>(
      q, kv, nullptr, nullptr, q_gamma, k_gamma, q_bhld, packed_k, packed_v, H, Lq, Lk,
      Lk_padded, 1, kv_tiles); }
  return launch_status();
}

}  // extern "C"
