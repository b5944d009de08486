/*
 * CPU oracle for the TripoSplat flow-model hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is a plain-C restatement of the
 * reference's AVX-512 kernels, written from their documented arithmetic, and it
 * is used exclusively as the checker by tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py.  The product library never links, loads or
 * calls it, and there is no code path in the product that falls back to it.
 *
 * Parity pinning: tests/test_oracle_golden.py checks every function here
 * against golden vectors produced by the reference's own compiled kernels
 * (tests/golden/make_golden.py) and, when oracle/_ref exists, against those
 * kernels directly on fresh seeded inputs.
 *
 * Citations are paths inside the reference project.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static void set_threads(int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
}

/*
 * NF24 int16 dequant GEMM, output columns [start, start+count).
 * scripts/gemm_nf24_i16_avx512.c:26-33 (decode: (float)(256*q01 + q2) * scale),
 * :63-94 (fmaf chain over k in ascending order, seeded with bias),
 * :151-197 (range semantics, out is [M, count] with stride_out),
 * scripts/gemm_nf24_i16_avx512_tail.c:32-47 (same arithmetic, scalar).
 * With -ffp-contract=off the weight product and the fmaf chain round exactly as
 * the reference's vector code does, so this is bit-identical to it.
 */
int oracle_gemm_nf24(const float* x, const int16_t* code01, const int8_t* q2,
                     const float* scale, const float* bias, float* out,
                     int M, int K, int N, int start, int count,
                     int stride_x, int stride_out, int threads) {
  if (!x || !code01 || !q2 || !scale || !bias || !out) return -1;
  if (M <= 0 || K <= 0 || N <= 0 || start < 0 || count <= 0) return -2;
  if (start + count > N || stride_x < K || stride_out < count) return -3;
  set_threads(threads);
#pragma omp parallel
  {
    float* w = (float*)malloc(sizeof(float) * (size_t)count);
#pragma omp for schedule(static)
    for (int m = 0; m < M; ++m) {
      const float* xr = x + (int64_t)m * stride_x;
      float* yr = out + (int64_t)m * stride_out;
      for (int j = 0; j < count; ++j) yr[j] = bias[start + j];
      for (int k = 0; k < K; ++k) {
        const int16_t* c01 = code01 + (int64_t)k * N + start;
        const int8_t* c2 = q2 + (int64_t)k * N + start;
        for (int j = 0; j < count; ++j) {
          const int32_t q = (int32_t)c01[j] * 256 + (int32_t)c2[j];
          w[j] = (float)q * scale[start + j];
        }
        const float xv = xr[k];
        for (int j = 0; j < count; ++j) yr[j] = fmaf(xv, w[j], yr[j]);
      }
    }
    free(w);
  }
  return 0;
}

/*
 * Exact SDPA, head_dim 64, fixed scale 0.125, optional additive key bias.
 * scripts/native_sdpa_avx512_exact_q8t512.c:232-311: keys are processed in
 * tiles of 512; per tile the scores are s = 0.125*dot(q,k) + bias, the tile
 * max is taken, w = exp(s - tile_max), the tile sum and tile output are formed
 * and merged into the running (max, sum, acc) by rescaling both sides;
 * :313-319 the output is acc / sum.
 * bias_bh_stride = 0 means one [Lk] bias shared by every (b, h) as in the
 * reference ABI (:153, :258); a non-zero stride selects a per-(b,h) row.
 * out_blhd selects the [B, Lq, H, 64] output of
 * scripts/native_sdpa_avx512_exact_q8t512_packed.c:147-154.
 * k/v are the standard [B,H,Lk,64] layout.
 */
enum { ORACLE_D = 64, ORACLE_KEY_TILE = 512 };

int oracle_sdpa(const float* q, const float* k, const float* v,
                const float* bias, int64_t bias_bh_stride, float* out,
                int B, int H, int Lq, int Lk, int out_blhd, int threads) {
  if (!q || !k || !v || !out) return -1;
  if (B <= 0 || H <= 0 || Lq <= 0 || Lk <= 0) return -2;
  set_threads(threads);
  const int64_t rows = (int64_t)B * H * Lq;
#pragma omp parallel
  {
    float* s = (float*)malloc(sizeof(float) * ORACLE_KEY_TILE);
#pragma omp for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
      const int64_t bh = r / Lq;
      const int i = (int)(r % Lq);
      const int b = (int)(bh / H), h = (int)(bh % H);
      const float* qr = q + r * ORACLE_D;
      const float* kb = k + bh * (int64_t)Lk * ORACLE_D;
      const float* vb = v + bh * (int64_t)Lk * ORACLE_D;
      const float* bb = bias ? bias + bh * bias_bh_stride : NULL;
      float gmax = -INFINITY, gsum = 0.0f;
      float acc[ORACLE_D], loc[ORACLE_D];
      for (int d = 0; d < ORACLE_D; ++d) acc[d] = 0.0f;
      for (int j0 = 0; j0 < Lk; j0 += ORACLE_KEY_TILE) {
        const int cnt = (j0 + ORACLE_KEY_TILE <= Lk) ? ORACLE_KEY_TILE : (Lk - j0);
        float lmax = -INFINITY;
        for (int j = 0; j < cnt; ++j) {
          const float* kr = kb + (int64_t)(j0 + j) * ORACLE_D;
          float dot = 0.0f;
          for (int d = 0; d < ORACLE_D; ++d) dot = fmaf(qr[d], kr[d], dot);
          float sc = dot * 0.125f;
          if (bb) sc += bb[j0 + j];
          s[j] = sc;
          if (sc > lmax) lmax = sc;
        }
        float lsum = 0.0f;
        for (int d = 0; d < ORACLE_D; ++d) loc[d] = 0.0f;
        for (int j = 0; j < cnt; ++j) {
          const float w = expf(s[j] - lmax);
          lsum += w;
          const float* vr = vb + (int64_t)(j0 + j) * ORACLE_D;
          for (int d = 0; d < ORACLE_D; ++d) loc[d] = fmaf(w, vr[d], loc[d]);
        }
        const float nmax = lmax > gmax ? lmax : gmax;
        const float os = isinf(gmax) ? 0.0f : expf(gmax - nmax);
        const float ls = expf(lmax - nmax);
        for (int d = 0; d < ORACLE_D; ++d) acc[d] = fmaf(loc[d], ls, acc[d] * os);
        gsum = gsum * os + lsum * ls;
        gmax = nmax;
      }
      float* dst = out_blhd ? out + (((int64_t)b * Lq + i) * H + h) * ORACLE_D
                            : out + r * ORACLE_D;
      const float inv = 1.0f / gsum;
      for (int d = 0; d < ORACLE_D; ++d) dst[d] = acc[d] * inv;
    }
    free(s);
  }
  return 0;
}

/* scripts/native_norm_rope_avx512.c:13-49: mean, biased variance,
 * 1/sqrtf(var + eps), optional affine. */
int oracle_layernorm(const float* in, const float* w, const float* b, float* out,
                     int64_t rows, int cols, float eps, int has_affine) {
  if (!in || !out) return -1;
  if (rows <= 0 || cols <= 0 || eps < 0.0f) return -2;
  if (has_affine && (!w || !b)) return -3;
  for (int64_t r = 0; r < rows; ++r) {
    const float* x = in + r * cols;
    float* y = out + r * cols;
    double sum = 0.0;
    for (int c = 0; c < cols; ++c) sum += x[c];
    const float mean = (float)(sum / cols);
    double var = 0.0;
    for (int c = 0; c < cols; ++c) { const double d = (double)x[c] - mean; var += d * d; }
    const float inv = 1.0f / sqrtf((float)(var / cols) + eps);
    for (int c = 0; c < cols; ++c) {
      float t = (x[c] - mean) * inv;
      if (has_affine) t = fmaf(t, w[c], b[c]);
      y[c] = t;
    }
  }
  return 0;
}

/* scripts/native_norm_rope_avx512.c:51-83: y = x * sqrt(dim)/max(||x||, eps) * gamma[head]. */
int oracle_multihead_rmsnorm(const float* in, const float* gamma, float* out,
                             int64_t outer, int heads, int dim, float eps) {
  if (!in || !gamma || !out) return -1;
  if (outer <= 0 || heads <= 0 || dim <= 0 || eps < 0.0f) return -2;
  for (int64_t vct = 0; vct < outer * heads; ++vct) {
    const int h = (int)(vct % heads);
    const float* x = in + vct * dim;
    float* y = out + vct * dim;
    double ss = 0.0;
    for (int d = 0; d < dim; ++d) ss += (double)x[d] * x[d];
    const float norm = sqrtf((float)ss);
    const float f = sqrtf((float)dim) / fmaxf(norm, eps);
    for (int d = 0; d < dim; ++d) y[d] = x[d] * f * gamma[(int64_t)h * dim + d];
  }
  return 0;
}

/* scripts/native_norm_rope_avx512.c:85-110: interleaved complex multiply
 * (x_re + i x_im)(f_re + i f_im). */
int oracle_rope_complex(const float* in, const float* freqs, float* out,
                        int64_t vectors, int dim) {
  if (!in || !freqs || !out) return -1;
  if (vectors <= 0 || dim <= 0 || (dim & 1)) return -2;
  for (int64_t i = 0; i < vectors * dim; i += 2) {
    const float xr = in[i], xi = in[i + 1], fr = freqs[i], fi = freqs[i + 1];
    out[i] = xr * fr - xi * fi;
    out[i + 1] = xr * fi + xi * fr;
  }
  return 0;
}

/* scripts/native_gelu_avx512.c:44-67: 0.5 x (1 + tanh(0.7978845608 (x + 0.044715 x^3))). */
int oracle_gelu_tanh(const float* in, float* out, int64_t n) {
  if (!in || !out) return -1;
  if (n <= 0) return -2;
  for (int64_t i = 0; i < n; ++i) {
    const float x = in[i];
    const float inner = 0.7978845608028654f * (x + 0.044715f * (x * x * x));
    out[i] = 0.5f * x * (1.0f + tanhf(inner));
  }
  return 0;
}

/* scripts/native_silu_avx512_extra.c:28-45: x / (1 + exp(-x)). */
int oracle_silu(const float* in, float* out, int64_t n) {
  if (!in || !out) return -1;
  if (n <= 0) return -2;
  for (int64_t i = 0; i < n; ++i) out[i] = in[i] / (1.0f + expf(-in[i]));
  return 0;
}

/* scripts/native_block_elementwise_avx512.c:9-22: h = h*(1+scale[b]) + shift[b]. */
int oracle_modulate_inplace(float* h, const float* scale, const float* shift,
                            int batch, int rows, int cols) {
  if (!h || !scale || !shift) return -1;
  if (batch <= 0 || rows <= 0 || cols <= 0) return -2;
  for (int64_t r = 0; r < (int64_t)batch * rows; ++r) {
    const int b = (int)(r / rows);
    for (int c = 0; c < cols; ++c) {
      float* p = h + r * cols + c;
      *p = *p * (1.0f + scale[(int64_t)b * cols + c]) + shift[(int64_t)b * cols + c];
    }
  }
  return 0;
}

/* scripts/native_block_elementwise_avx512.c:24-35: delta *= gate[b]; base += delta. */
int oracle_gated_residual_inplace(float* base, float* delta, const float* gate,
                                  int batch, int rows, int cols) {
  if (!base || !delta || !gate) return -1;
  if (batch <= 0 || rows <= 0 || cols <= 0) return -2;
  for (int64_t r = 0; r < (int64_t)batch * rows; ++r) {
    const int b = (int)(r / rows);
    for (int c = 0; c < cols; ++c) {
      const int64_t i = r * cols + c;
      delta[i] = delta[i] * gate[(int64_t)b * cols + c];
      base[i] = base[i] + delta[i];
    }
  }
  return 0;
}

/* scripts/native_block_elementwise_avx512.c:37-46. */
int oracle_add_inplace(float* base, const float* delta, int64_t n) {
  if (!base || !delta) return -1;
  if (n <= 0) return -2;
  for (int64_t i = 0; i < n; ++i) base[i] += delta[i];
  return 0;
}

/* scripts/native_sampler_avx512.c:19-54: pos = g*pos - (g-1)*neg per batch. */
int oracle_cfg_combine_inplace(float* pos, const float* neg, const float* guidance,
                               int batch, int64_t n) {
  if (!pos || !neg || !guidance) return -1;
  if (batch <= 0 || n <= 0) return -2;
  for (int b = 0; b < batch; ++b) {
    const float g = guidance[b], gm1 = g - 1.0f;
    for (int64_t i = 0; i < n; ++i) {
      float* p = pos + (int64_t)b * n + i;
      *p = g * *p - gm1 * neg[(int64_t)b * n + i];
    }
  }
  return 0;
}

/* scripts/native_sampler_avx512.c:56-89: x = x - dt[b]*v. */
int oracle_euler_update_inplace(float* sample, const float* pred, const float* dt,
                                int batch, int64_t n) {
  if (!sample || !pred || !dt) return -1;
  if (batch <= 0 || n <= 0) return -2;
  for (int b = 0; b < batch; ++b)
    for (int64_t i = 0; i < n; ++i) {
      float* p = sample + (int64_t)b * n + i;
      *p = *p - dt[b] * pred[(int64_t)b * n + i];
    }
  return 0;
}

/*
 * QKV post-process: RoPE, then per-head L2 normalisation 8/max(||x||,1e-12)*gamma,
 * Q to [B,H,L,64], K and V packed to [B,H,64,Lp] with a zero tail.
 * scripts/native_qkv_postprocess_v2_avx512.c:3-24 (transform), :26-43 (pack),
 * :45-105 (entry, qkv is [B,L,3,H,64], freqs [Fb,L,H,64] interleaved re/im).
 */
static void transform64(const float* src, const float* f, const float* g, float* dst) {
  float rot[ORACLE_D];
  double ss = 0.0;
  for (int d = 0; d < ORACLE_D; d += 2) {
    rot[d] = src[d] * f[d] - src[d + 1] * f[d + 1];
    rot[d + 1] = src[d] * f[d + 1] + src[d + 1] * f[d];
    ss += (double)rot[d] * rot[d] + (double)rot[d + 1] * rot[d + 1];
  }
  const float fac = 8.0f / fmaxf(sqrtf((float)ss), 1.0e-12f);
  for (int d = 0; d < ORACLE_D; ++d) dst[d] = rot[d] * fac * g[d];
}

int oracle_qkv_rope_rmsnorm_pack(const float* qkv, const float* freqs,
                                 const float* q_gamma, const float* k_gamma,
                                 float* q_bhld, float* packed_k, float* packed_v,
                                 int B, int L, int H, int Lp, int freq_batches) {
  if (!qkv || !freqs || !q_gamma || !k_gamma || !q_bhld || !packed_k || !packed_v) return -1;
  if (B <= 0 || L <= 0 || H <= 0 || Lp < L || (Lp & 15) ||
      (freq_batches != 1 && freq_batches != B)) return -2;
  const int D = ORACLE_D;
  float kt[ORACLE_D];
  for (int b = 0; b < B; ++b)
    for (int h = 0; h < H; ++h) {
      const int64_t bh = (int64_t)b * H + h;
      float* pk = packed_k + bh * D * (int64_t)Lp;
      float* pv = packed_v + bh * D * (int64_t)Lp;
      for (int t = 0; t < L; ++t) {
        const float* qs = qkv + (((int64_t)b * L + t) * 3 * H + h) * D;
        const float* ks = qs + (int64_t)H * D;
        const float* vs = ks + (int64_t)H * D;
        const int fb = freq_batches == 1 ? 0 : b;
        const float* f = freqs + (((int64_t)fb * L + t) * H + h) * D;
        transform64(qs, f, q_gamma + (int64_t)h * D, q_bhld + (bh * L + t) * D);
        transform64(ks, f, k_gamma + (int64_t)h * D, kt);
        for (int d = 0; d < D; ++d) {
          pk[(int64_t)d * Lp + t] = kt[d];
          pv[(int64_t)d * Lp + t] = vs[d];
        }
      }
      for (int d = 0; d < D; ++d)
        for (int t = L; t < Lp; ++t) {
          pk[(int64_t)d * Lp + t] = 0.0f;
          pv[(int64_t)d * Lp + t] = 0.0f;
        }
    }
  return 0;
}

/* ---------------------------------------------------------------------------
 * Position / timestep embeddings and the RePo phasor
 * (scripts/native_embeddings_avx512.c:12-125, scripts/native_repo_avx512.c:12-129)
 * ------------------------------------------------------------------------- */

/* sin and cos of x by the reference's own method (native_embeddings_avx512.c:12-56,
   identical in native_repo_avx512.c:12-56): q = x * 2/pi rounded to the nearest integer
   (ties to even; out of int32 range -> INT32_MIN, the AVX-512 conversion's indefinite
   value), r = x - q*pi/2 in two fused steps with pi/2 split into a high and a low part,
   Taylor polynomials in z = r^2 for sin (to r^13) and cos (to r^14) by Horner with fused
   multiply-adds, then the quadrant q & 3 selects and negates the pair. */
static void ref_sincos(float x, float* s_out, float* c_out) {
  const float inv_pio2 = 0.63661977236758134308f;
  const float pio2_hi = 1.57079625129699707031f;
  const float pio2_lo = 7.54978941586159635335e-8f;
  const float t = x * inv_pio2;
  const int32_t q = (fabsf(t) < 2147483648.0f) ? (int32_t)lrintf(t) : INT32_MIN;
  const float qf = (float)q;
  float r = fmaf(-qf, pio2_hi, x);
  r = fmaf(-qf, pio2_lo, r);
  const float z = r * r;
  float sp = -1.0f / 6227020800.0f;
  sp = fmaf(sp, z, 1.0f / 39916800.0f);
  sp = fmaf(sp, z, -1.0f / 362880.0f);
  sp = fmaf(sp, z, 1.0f / 5040.0f);
  sp = fmaf(sp, z, -1.0f / 120.0f);
  sp = fmaf(sp, z, 1.0f / 6.0f);
  const float sin_r = r - (r * z) * sp;
  float cp = -1.0f / 87178291200.0f;
  cp = fmaf(cp, z, 1.0f / 479001600.0f);
  cp = fmaf(cp, z, -1.0f / 3628800.0f);
  cp = fmaf(cp, z, 1.0f / 40320.0f);
  cp = fmaf(cp, z, -1.0f / 720.0f);
  cp = fmaf(cp, z, 1.0f / 24.0f);
  cp = fmaf(cp, z, -0.5f);
  const float cos_r = fmaf(cp, z, 1.0f);
  float s = sin_r, c = cos_r;
  switch (q & 3) {
    case 1: s = cos_r; c = -sin_r; break;
    case 2: s = -sin_r; c = -cos_r; break;
    case 3: s = -cos_r; c = sin_r; break;
    default: break;
  }
  *s_out = s;
  *c_out = c;
}

/* output[sample] = [cos(t f_0..f_{H-1}) | sin(t f_0..) | 0 ...]
   (native_embeddings_avx512.c:97-125) */
int oracle_timestep_embedding(const float* timesteps, const float* frequencies, float* output,
                              int batch, int half_dim, int output_dim) {
  if (!timesteps || !frequencies || !output) return -1;
  if (batch <= 0 || half_dim <= 0 || output_dim < half_dim * 2) return -2;
  for (int b = 0; b < batch; ++b) {
    float* cos_dst = output + (int64_t)b * output_dim;
    float* sin_dst = cos_dst + half_dim;
    for (int i = 0; i < half_dim; ++i) ref_sincos(timesteps[b] * frequencies[i], sin_dst + i, cos_dst + i);
    for (int i = 2 * half_dim; i < output_dim; ++i) cos_dst[i] = 0.0f;
  }
  return 0;
}

/* per row and axis: [sin(a_0..a_{F-1}) | cos(a_0..)] with a = x f (x 2 if double_pi) x pi,
   zero padding to `channels` (native_embeddings_avx512.c:58-95) */
int oracle_pcd_position_embedding(const float* positions, const float* frequencies, float* output,
                                  int64_t rows, int input_dims, int frequency_dim, int channels,
                                  int double_pi) {
  if (!positions || !frequencies || !output) return -1;
  if (rows <= 0 || input_dims <= 0 || frequency_dim <= 0 || channels < input_dims * frequency_dim * 2)
    return -2;
  const float pi = 3.14159274101257324219f;
  for (int64_t r = 0; r < rows; ++r) {
    float* dst = output + r * (int64_t)channels;
    for (int a = 0; a < input_dims; ++a) {
      const float x = positions[r * input_dims + a];
      float* sin_dst = dst + a * (2 * frequency_dim);
      float* cos_dst = sin_dst + frequency_dim;
      for (int i = 0; i < frequency_dim; ++i) {
        float angle = x * frequencies[i];
        if (double_pi) angle = angle + angle;
        angle = angle * pi;
        ref_sincos(angle, sin_dst + i, cos_dst + i);
      }
    }
    for (int i = input_dims * frequency_dim * 2; i < channels; ++i) dst[i] = 0.0f;
  }
  return 0;
}

/* lhs *= rhs elementwise (native_repo_avx512.c:69-83) */
int oracle_mul_inplace(float* lhs, const float* rhs, int64_t n) {
  if (!lhs || !rhs) return -1;
  if (n <= 0) return -2;
  for (int64_t i = 0; i < n; ++i) lhs[i] = lhs[i] * rhs[i];
  return 0;
}

/* RePo rotary phasors: per vector v and axis a (3 axes, dims d_a), for each frequency
   angle = (x ft + x fr) pi with x = delta[v, a], written as interleaved complex
   (cos, sin) along the concatenated axes (native_repo_avx512.c:85-129) */
int oracle_repo_phasor(const float* delta, const float* ft0, const float* fr0, int d0,
                       const float* ft1, const float* fr1, int d1, const float* ft2,
                       const float* fr2, int d2, float* out, int64_t vectors) {
  if (!delta || !out) return -1;
  if (!ft0 || !fr0 || !ft1 || !fr1 || !ft2 || !fr2) return -2;
  if (vectors <= 0 || d0 <= 0 || d1 <= 0 || d2 <= 0) return -3;
  const float* ft[3] = {ft0, ft1, ft2};
  const float* fr[3] = {fr0, fr1, fr2};
  const int dims[3] = {d0, d1, d2};
  const int total = d0 + d1 + d2;
  const float pi = 3.14159274101257324219f;
  for (int64_t v = 0; v < vectors; ++v) {
    float* dst = out + v * (int64_t)(2 * total);
    int k = 0;
    for (int a = 0; a < 3; ++a) {
      const float x = delta[v * 3 + a];
      for (int i = 0; i < dims[a]; ++i, ++k) {
        const float angle = (x * ft[a][i] + x * fr[a][i]) * pi;
        ref_sincos(angle, dst + 2 * k + 1, dst + 2 * k);
      }
    }
  }
  return 0;
}

/* Adams-Bashforth-2 sampler step (scripts/native_sampler_avx512.c:91-130):
   x -= dt * ((1 + r) * v - r * v_prev), r = 0.5 * (dt / max(dt_prev, 1e-12)) */
int oracle_ab2_update_inplace(float* sample, const float* pred, const float* prev, const float* dt,
                              const float* prev_dt, int batch, int64_t per_batch) {
  if (!sample || !pred || !prev || !dt || !prev_dt) return -1;
  if (batch <= 0 || per_batch <= 0) return -2;
  for (int b = 0; b < batch; ++b) {
    const float r = 0.5f * (dt[b] / fmaxf(prev_dt[b], 1.0e-12f));
    const float cur_scale = 1.0f + r;
    for (int64_t i = (int64_t)b * per_batch; i < (int64_t)(b + 1) * per_batch; ++i) {
      const float eff = cur_scale * pred[i] - r * prev[i];
      sample[i] = sample[i] - dt[b] * eff;
    }
  }
  return 0;
}
