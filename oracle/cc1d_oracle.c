/*
 * TEST INFRASTRUCTURE ONLY -- CPU oracle for the causal depthwise conv1d hot
 * path.  It is the checker the tests compare the CUDA kernels against, and
 * the timed CPU baseline of bench.py; it is never called by the product.
 *
 * A plain-C restatement of the reference's CPU kernels (Mojo, not buildable
 * here: no mojo toolchain), parallelised the same way (one task per (b, c)
 * row, as `sync_parallelize` over batch*dim):
 *   fwd    : src/causal_conv1d_mojo/fwd_cpu/kernel.mojo:64-117
 *   bwd    : src/causal_conv1d_mojo/bwd_full_cpu/kernel.mojo:26-105 (dpre),
 *            :174-227 (dinitial_states + boundary dweight), :229-312 (dx,
 *            dweight, dbias)
 *   update : src/causal_conv1d_mojo/update_cpu/kernel.mojo:52-139
 *   varlen : src/causal_conv1d_mojo/causal_conv1d_varlen.py:29-61
 * final_states / dfinal_states follow the pure-PyTorch reference
 * (src/causal_conv1d_mojo/reference.py:50-56: the last W-1 columns of
 * cat([initial_states, x])), and its autograd for the gradient.
 *
 * The parameter structs are the product's C ABI (include/cc1d.h), read here
 * with HOST pointers.  `acc64` selects double accumulation (the checker) or
 * float accumulation (what the reference's CPU kernels do; the port that
 * bench.py times).  dweight/dbias are summed over rows in row order, so the
 * oracle is deterministic.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#include "cc1d.h"

typedef int64_t i64;

/* ---- element access ------------------------------------------------------ */

static inline float bf16_to_f(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline uint16_t f_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
  u += 0x7fffu + ((u >> 16) & 1u); /* round to nearest even */
  return (uint16_t)(u >> 16);
}

static inline double ld(int dt, const void* p, i64 i) {
  switch (dt) {
    case CC1D_F16: return (double)((const _Float16*)p)[i];
    case CC1D_BF16: return (double)bf16_to_f(((const uint16_t*)p)[i]);
    default: return (double)((const float*)p)[i];
  }
}

static inline void st(int dt, void* p, i64 i, double v) {
  switch (dt) {
    case CC1D_F16: ((_Float16*)p)[i] = (_Float16)(float)v; break;
    case CC1D_BF16: ((uint16_t*)p)[i] = f_to_bf16((float)v); break;
    default: ((float*)p)[i] = (float)v; break;
  }
}

/* Exact element copy (final_states, conv_state): no rounding involved. */
static inline void cp(int dt, void* dst, i64 di, const void* src, i64 si) {
  if (dt == CC1D_F32)
    ((float*)dst)[di] = ((const float*)src)[si];
  else
    ((uint16_t*)dst)[di] = ((const uint16_t*)src)[si];
}

static inline void zero(int dt, void* dst, i64 di) {
  if (dt == CC1D_F32)
    ((float*)dst)[di] = 0.f;
  else
    ((uint16_t*)dst)[di] = 0;
}

/* Rounds an accumulator the way the selected precision would hold it. */
static inline double acc_round(int acc64, double v) { return acc64 ? v : (double)(float)v; }

static inline double silu(int acc64, double v) {
  if (acc64) return v / (1.0 + exp(-v));
  float f = (float)v;
  return (double)(f / (1.0f + expf(-f)));
}

static inline double silu_grad(int acc64, double v) {
  if (acc64) {
    double s = 1.0 / (1.0 + exp(-v));
    return s * (1.0 + v * (1.0 - s));
  }
  float f = (float)v;
  float s = 1.0f / (1.0f + expf(-f));
  return (double)(s * (1.0f + f * (1.0f - s)));
}

static void set_threads(int nthreads) {
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#else
  (void)nthreads;
#endif
}

/* ---- forward ------------------------------------------------------------- */

/* Value of cat([initial_states or 0, x]) at position p of row (b, c),
 * p in [-(W-1), L). */
static inline double xcat(const cc1d_fwd_params* p, i64 b, i64 c, i64 pos) {
  if (pos >= 0) return ld(p->dtype, p->x, b * p->x_batch_stride + c * p->x_dim_stride + pos * p->x_seq_stride);
  if (!p->initial_states) return 0.0;
  return ld(p->dtype, p->initial_states,
            b * p->init_batch_stride + c * p->init_dim_stride + (pos + p->width - 1) * p->init_seq_stride);
}

int oracle_fwd(const cc1d_fwd_params* p, int acc64, int nthreads) {
  const i64 B = p->batch, D = p->dim, L = p->seqlen;
  const int W = p->width;
  set_threads(nthreads);
#pragma omp parallel for schedule(static)
  for (i64 bc = 0; bc < B * D; ++bc) {
    const i64 b = bc / D, c = bc % D;
    double w[16];
    for (int k = 0; k < W; ++k) w[k] = ld(p->dtype, p->weight, c * p->weight_dim_stride + k * p->weight_width_stride);
    const double bias = p->bias ? ld(p->dtype, p->bias, c * p->bias_stride) : 0.0;
    for (i64 t = 0; t < L; ++t) {
      const int cur = p->seq_idx ? p->seq_idx[b * p->seq_idx_batch_stride + t * p->seq_idx_seq_stride] : 0;
      double pre = bias;
      for (int k = 0; k < W; ++k) {
        const i64 src = t + k - (W - 1);
        if (src >= 0 && p->seq_idx &&
            p->seq_idx[b * p->seq_idx_batch_stride + src * p->seq_idx_seq_stride] != cur)
          continue;
        pre = acc_round(acc64, pre + w[k] * xcat(p, b, c, src));
      }
      double o = p->silu ? silu(acc64, pre) : pre;
      if (p->seq_idx && cur < 0) o = 0.0;
      st(p->dtype, p->out, b * p->out_batch_stride + c * p->out_dim_stride + t * p->out_seq_stride, o);
    }
    if (p->final_states) {
      for (int j = 0; j < W - 1; ++j) {
        const i64 pos = L - (W - 1) + j;
        const i64 di = b * p->final_batch_stride + c * p->final_dim_stride + j * p->final_seq_stride;
        if (pos >= 0)
          cp(p->dtype, p->final_states, di, p->x, b * p->x_batch_stride + c * p->x_dim_stride + pos * p->x_seq_stride);
        else if (p->initial_states)
          cp(p->dtype, p->final_states, di, p->initial_states,
             b * p->init_batch_stride + c * p->init_dim_stride + (pos + W - 1) * p->init_seq_stride);
        else
          zero(p->dtype, p->final_states, di);
      }
    }
  }
  return 0;
}

/* ---- backward ------------------------------------------------------------ */

typedef struct {
  const cc1d_bwd_params* p;
  i64 b, c;
  double w[16];
  double bias;
  int acc64;
} bwd_row;

static inline int seq_at(const cc1d_bwd_params* p, i64 b, i64 t) {
  return p->seq_idx[b * p->seq_idx_batch_stride + t * p->seq_idx_seq_stride];
}

static inline double bxcat(const bwd_row* r, i64 pos) {
  const cc1d_bwd_params* p = r->p;
  if (pos >= 0) return ld(p->dtype, p->x, r->b * p->x_batch_stride + r->c * p->x_dim_stride + pos * p->x_seq_stride);
  if (!p->initial_states) return 0.0;
  return ld(p->dtype, p->initial_states,
            r->b * p->init_batch_stride + r->c * p->init_dim_stride + (pos + p->width - 1) * p->init_seq_stride);
}

/* dpre[t] (0 outside [0, L) and at padding tokens); bwd_full_cpu/kernel.mojo:26-105. */
static double dpre_at(const bwd_row* r, i64 t) {
  const cc1d_bwd_params* p = r->p;
  const int W = p->width;
  if (t < 0 || t >= p->seqlen) return 0.0;
  int cur = 0;
  if (p->seq_idx) {
    cur = seq_at(p, r->b, t);
    if (cur < 0) return 0.0;
  }
  const double g = ld(p->dtype, p->dout, r->b * p->dout_batch_stride + r->c * p->dout_dim_stride + t * p->dout_seq_stride);
  if (!p->silu) return g;
  double pre = r->bias;
  for (int k = 0; k < W; ++k) {
    const i64 src = t + k - (W - 1);
    if (src >= 0 && p->seq_idx && seq_at(p, r->b, src) != cur) continue;
    pre = acc_round(r->acc64, pre + r->w[k] * bxcat(r, src));
  }
  return acc_round(r->acc64, g * silu_grad(r->acc64, pre));
}

int oracle_bwd(const cc1d_bwd_params* p, int acc64, int nthreads) {
  const i64 B = p->batch, D = p->dim, L = p->seqlen;
  const int W = p->width;
  double* part = (double*)calloc((size_t)(B * D > 0 ? B * D : 1) * (size_t)(W + 1), sizeof(double));
  if (!part) return 1;
  set_threads(nthreads);
#pragma omp parallel for schedule(static)
  for (i64 bc = 0; bc < B * D; ++bc) {
    bwd_row r;
    r.p = p;
    r.b = bc / D;
    r.c = bc % D;
    r.acc64 = acc64;
    for (int k = 0; k < W; ++k)
      r.w[k] = ld(p->dtype, p->weight, r.c * p->weight_dim_stride + k * p->weight_width_stride);
    r.bias = p->bias ? ld(p->dtype, p->bias, r.c * p->bias_stride) : 0.0;
    const i64 b = r.b, c = r.c;
    double* dw = part + bc * (W + 1);
    const void* dfin = p->dfinal_states;
#define DFIN(q) ld(p->dtype, dfin, b * p->dfinal_batch_stride + c * p->dfinal_dim_stride + (q) * p->dfinal_seq_stride)
    /* Sliding window win[k] = dpre[t + k]. */
    double win[16];
    for (int k = 0; k < W; ++k) win[k] = dpre_at(&r, k);
    if (p->initial_states) {
      /* dinit[i] = sum_{k<=i} w[k] dpre[i-k] (+ dfinal where final_states
       * read initial_states); kernel.mojo:210-219. */
      for (int i = 0; i < W - 1; ++i) {
        double acc = 0.0;
        for (int k = 0; k <= i; ++k) acc = acc_round(acc64, acc + r.w[k] * win[i - k]);
        if (dfin && i - L >= 0) acc = acc_round(acc64, acc + DFIN(i - L));
        st(p->dtype, p->dinitial_states,
           b * p->dinit_batch_stride + c * p->dinit_dim_stride + i * p->dinit_seq_stride, acc);
      }
      /* dweight terms that read initial_states; kernel.mojo:221-227. */
      for (int k = 0; k < W; ++k)
        for (int t = 0; t < W - 1 - k; ++t) {
          const double iv = ld(p->dtype, p->initial_states,
                               b * p->init_batch_stride + c * p->init_dim_stride + (t + k) * p->init_seq_stride);
          dw[k] = acc_round(acc64, dw[k] + win[t] * iv);
        }
    }
    for (i64 t = 0; t < L; ++t) {
      const int cur = p->seq_idx ? seq_at(p, b, t) : 0;
      double dxv = 0.0;
      for (int k = 0; k < W; ++k) {
        if (p->seq_idx && (t + k >= L || seq_at(p, b, t + k) != cur)) continue;
        dxv = acc_round(acc64, dxv + r.w[W - 1 - k] * win[k]);
      }
      if (dfin && t + (W - 1) - L >= 0) dxv = acc_round(acc64, dxv + DFIN(t + (W - 1) - L));
      st(p->dtype, p->dx, b * p->dx_batch_stride + c * p->dx_dim_stride + t * p->dx_seq_stride, dxv);
      const double d = win[0];
      dw[W] = acc_round(acc64, dw[W] + d);
      for (int k = 0; k < W; ++k) {
        const i64 src = t + k - (W - 1);
        if (src < 0) continue; /* initial_states terms were added above */
        if (p->seq_idx && seq_at(p, b, src) != cur) continue;
        dw[k] = acc_round(acc64, dw[k] + d * bxcat(&r, src));
      }
      for (int k = 0; k < W - 1; ++k) win[k] = win[k + 1];
      win[W - 1] = dpre_at(&r, t + W);
    }
#undef DFIN
  }
  /* Reduce over rows in row order (deterministic). */
  for (i64 c = 0; c < D; ++c) {
    for (int k = 0; k <= W; ++k) {
      double s = 0.0;
      for (i64 b = 0; b < B; ++b) s = acc_round(acc64, s + part[(b * D + c) * (W + 1) + k]);
      if (k == W && !p->bias) s = 0.0;
      if (k < W) {
        p->dwdb_acc[c * W + k] = (float)s;
        if (p->dweight_out) st(p->dtype, p->dweight_out, c * p->dweight_dim_stride + k * p->dweight_width_stride, s);
      } else {
        p->dwdb_acc[D * W + c] = (float)s;
        if (p->dbias_out && p->bias) st(p->dtype, p->dbias_out, c * p->dbias_stride, s);
      }
    }
  }
  free(part);
  return 0;
}

/* ---- decode update ------------------------------------------------------- */

int oracle_update(const cc1d_update_params* p, int acc64, int nthreads) {
  const i64 B = p->batch, D = p->dim, L = p->seqlen, S = p->state_len;
  const int W = p->width, H = W - 1;
  set_threads(nthreads);
#pragma omp parallel for schedule(static)
  for (i64 bc = 0; bc < B * D; ++bc) {
    const i64 b = bc / D, c = bc % D;
    const i64 ob = b * p->out_batch_stride + c * p->out_dim_stride;
    i64 row = b;
    if (p->conv_state_indices) {
      const int r = p->conv_state_indices[b];
      if (r < 0 || r >= p->state_rows) { /* padding (or an index past the pool) */
        for (i64 i = 0; i < L; ++i) st(p->dtype, p->out, ob + i * p->out_seq_stride, 0.0);
        continue;
      }
      row = r;
    }
    const i64 sb = row * p->state_batch_stride + c * p->state_dim_stride;
    const i64 xb = b * p->x_batch_stride + c * p->x_dim_stride;
    double w[16], win[16];
    for (int k = 0; k < W; ++k) w[k] = ld(p->dtype, p->weight, c * p->weight_dim_stride + k * p->weight_width_stride);
    const double bias = p->bias ? ld(p->dtype, p->bias, c * p->bias_stride) : 0.0;
    i64 head = 0;
    if (p->cache_seqlens) {
      i64 cs = (i64)p->cache_seqlens[b] % S;
      if (cs < 0) cs += S;
      i64 ui = (cs - H) % S;
      if (ui < 0) ui += S;
      for (int j = 0; j < H; ++j) {
        win[j] = ld(p->dtype, p->conv_state, sb + ui * p->state_seq_stride);
        ui = (ui + 1) % S;
      }
      head = ui;
    } else {
      for (int j = 0; j < H; ++j) win[j] = ld(p->dtype, p->conv_state, sb + (S - H + j) * p->state_seq_stride);
      /* Shift: new state = last S values of cat([state, x]). */
      for (i64 j = 0; j < S; ++j) {
        const i64 src = L + j;
        if (src < S)
          cp(p->dtype, p->conv_state, sb + j * p->state_seq_stride, p->conv_state, sb + src * p->state_seq_stride);
        else
          cp(p->dtype, p->conv_state, sb + j * p->state_seq_stride, p->x, xb + (src - S) * p->x_seq_stride);
      }
    }
    for (i64 i = 0; i < L; ++i) {
      if (p->cache_seqlens) {
        cp(p->dtype, p->conv_state, sb + head * p->state_seq_stride, p->x, xb + i * p->x_seq_stride);
        head = (head + 1) % S;
      }
      win[H] = ld(p->dtype, p->x, xb + i * p->x_seq_stride);
      double acc = bias;
      for (int k = 0; k < W; ++k) acc = acc_round(acc64, acc + w[k] * win[k]);
      if (p->silu) acc = silu(acc64, acc);
      st(p->dtype, p->out, ob + i * p->out_seq_stride, acc);
      for (int k = 0; k < H; ++k) win[k] = win[k + 1];
    }
  }
  return 0;
}

/* ---- varlen states ------------------------------------------------------- */

int oracle_varlen_states(const cc1d_varlen_states_params* p) {
  const i64 S = p->state_len;
  for (i64 i = 0; i < p->batch; ++i) {
    const i64 end = p->cu_seqlens[i + 1];
    i64 start = p->cu_seqlens[i];
    if (start < end - S) start = end - S;
    const i64 n = end - start;
    for (i64 c = 0; c < p->dim; ++c)
      for (i64 j = 0; j < S; ++j) {
        const i64 di = i * p->states_batch_stride + c * p->states_dim_stride + j * p->states_seq_stride;
        if (n > 0 && j >= S - n)
          cp(p->dtype, p->states, di, p->x, (end - S + j) * p->x_token_stride + c * p->x_dim_stride);
        else
          zero(p->dtype, p->states, di);
      }
  }
  return 0;
}

int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
