/*
 * msda_oracle.c -- CPU restatement of multi-scale deformable attention (MSDA),
 * used ONLY as test infrastructure: the checker in tests/, in
 * __graft_entry__.smoke() and in bench.py's cpu_baseline / reference arm.
 * Nothing in the product (msda_triton_b200/) links or calls it.
 *
 * What it restates.  The reference's oracle is msda{2,3}d_pytorch
 * (src/msda_triton/pytorch/msda_2d.py:23-114, src/msda_triton/pytorch/msda_3d.py:23-118):
 *   grid = 2*loc - 1                         (msda_2d.py:66)
 *   grid = clamp(grid, -1+eps, 1-eps)        (msda_2d.py:67-68, only if clamp_grid)
 *   per level: F.grid_sample(value_l, grid, bilinear, zeros, align_corners=False)
 *                                            (msda_2d.py:92-98, msda_3d.py:96-102)
 *   out += sum_p attn[l,p] * sample[l,p]     (msda_2d.py:102-110)
 * and the backward is autograd through those ops.  grid_sample is a torch
 * dependency (uv.lock pins torch 2.9.0); its published align_corners=False,
 * zero-padding semantics are restated here:
 *   ix = ((g + 1) * size - 1) / 2            (source index of normalised g)
 *   corners floor(ix), floor(ix)+1; a corner outside [0, size) reads 0 and
 *   receives no gradient; linear weights (1-f, f) per axis.
 * clamp's backward passes the gradient only where lo <= g <= hi (inclusive).
 *
 * Arithmetic.  Coordinates are computed in float32 exactly as written above
 * (this file is compiled with -ffp-contract=off so no FMA contraction changes
 * the cell a coordinate falls in); the forward output and the per-sample
 * gradient scalars are accumulated in double and rounded to float once at the
 * end; grad_value is accumulated in float (see msda_oracle_bwd).
 *
 * Layouts (all row-major, contiguous, float32):
 *   value      (B, K, H, C)        K = sum over levels of prod(shape_l)
 *   shapes     (L, d) int64        rows (H, W) for d=2, (D, H, W) for d=3
 *   loc        (B, Q, H, L, P, d)  last axis (x, y[, z]) = (W, H[, D]) axes
 *   attn       (B, Q, H, L, P)
 *   out        (B, Q, H*C)
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef struct {
  int64_t size[3];  /* per axis in (x, y, z) order: W, H, D */
  int64_t start;    /* first flattened key of the level */
} level_t;

/* Fill per-level sizes in (x, y, z) order and the exclusive prefix sum of
 * level sizes (the "level start" table). Returns the total key count. */
static int64_t build_levels(int ndim, const int64_t* shapes, int64_t L, level_t* lv) {
  int64_t start = 0;
  for (int64_t l = 0; l < L; ++l) {
    const int64_t* s = shapes + l * ndim;
    int64_t n = 1;
    for (int a = 0; a < ndim; ++a) {
      lv[l].size[a] = s[ndim - 1 - a]; /* shapes row is (.., H, W): reverse to (W, H, ..) */
      n *= s[a];
    }
    if (ndim == 2) lv[l].size[2] = 1;
    lv[l].start = start;
    start += n;
  }
  return start;
}

/* One sampling point, resolved to up to 8 corners. */
typedef struct {
  int ncorner;
  int64_t key[8];      /* flattened key index of each corner (valid ones only) */
  float w[8];          /* interpolation weight of each valid corner */
  float dw[3][8];      /* d weight / d source-index, per axis */
  int pass[3];         /* clamp backward mask per axis (1 = gradient flows) */
} point_t;

static void resolve_point(int ndim, const level_t* lv, const float* loc, int clamp,
                          float lo, float hi, point_t* pt) {
  int64_t i0[3] = {0, 0, 0};
  float f[3] = {0.f, 0.f, 0.f};
  for (int a = 0; a < ndim; ++a) {
    float g = 2.0f * loc[a];
    g = g - 1.0f;
    pt->pass[a] = 1;
    if (clamp) {
      pt->pass[a] = (g >= lo) && (g <= hi);
      if (g < lo) g = lo;
      if (g > hi) g = hi;
    }
    float size = (float)lv->size[a];
    float t = g + 1.0f;
    t = t * size;
    t = t - 1.0f;
    float ix = t / 2.0f;
    float fl = floorf(ix);
    i0[a] = (int64_t)fl;
    f[a] = ix - fl;
  }
  pt->ncorner = 0;
  int ncomb = 1 << ndim;
  for (int c = 0; c < ncomb; ++c) {
    int64_t idx[3] = {0, 0, 0};
    float w = 1.0f;
    float dwa[3] = {1.0f, 1.0f, 1.0f};
    int valid = 1;
    for (int a = 0; a < ndim; ++a) {
      int hi_side = (c >> a) & 1;
      idx[a] = i0[a] + hi_side;
      if (idx[a] < 0 || idx[a] >= lv->size[a]) valid = 0;
      float wa = hi_side ? f[a] : 1.0f - f[a];
      float da = hi_side ? 1.0f : -1.0f;
      for (int b = 0; b < ndim; ++b) dwa[b] *= (b == a) ? da : wa;
      w *= wa;
    }
    if (!valid) continue;
    int64_t key = lv->start + idx[0];
    if (ndim >= 2) key += idx[1] * lv->size[0];
    if (ndim == 3) key += idx[2] * lv->size[0] * lv->size[1];
    int n = pt->ncorner++;
    pt->key[n] = key;
    pt->w[n] = w;
    for (int a = 0; a < 3; ++a) pt->dw[a][n] = (a < ndim) ? dwa[a] : 0.0f;
  }
}

static void clamp_bounds(double eps, float* lo, float* hi) {
  *lo = (float)(-1.0 + eps);
  *hi = (float)(1.0 - eps);
}

/* Forward: out[b,q,h,:] = sum_{l,p} attn * interp(value[b,:,h,:], loc). */
int msda_oracle_fwd(int ndim, const float* value, const int64_t* shapes, int64_t B,
                    int64_t K, int64_t H, int64_t C, int64_t Q, int64_t L, int64_t P,
                    const float* loc, const float* attn, int clamp, double eps, float* out,
                    int nthreads) {
  if (ndim != 2 && ndim != 3) return 1;
  level_t* lv = (level_t*)malloc(sizeof(level_t) * (size_t)(L > 0 ? L : 1));
  if (!lv) return 2;
  if (build_levels(ndim, shapes, L, lv) != K) { free(lv); return 3; }
  float lo, hi;
  clamp_bounds(eps, &lo, &hi);
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#else
  (void)nthreads;
#endif
  const int64_t nrow = B * Q * H;
#pragma omp parallel
  {
    double* acc = (double*)malloc(sizeof(double) * (size_t)(C > 0 ? C : 1));
#pragma omp for schedule(static)
    for (int64_t r = 0; r < nrow; ++r) {
      const int64_t h = r % H;
      const int64_t b = r / (Q * H);
      for (int64_t c = 0; c < C; ++c) acc[c] = 0.0;
      for (int64_t l = 0; l < L; ++l) {
        for (int64_t p = 0; p < P; ++p) {
          const int64_t s = (r * L + l) * P + p;
          point_t pt;
          resolve_point(ndim, &lv[l], loc + s * ndim, clamp, lo, hi, &pt);
          const double a = attn[s];
          for (int n = 0; n < pt.ncorner; ++n) {
            const float* v = value + ((b * K + pt.key[n]) * H + h) * C;
            const double aw = a * (double)pt.w[n];
            for (int64_t c = 0; c < C; ++c) acc[c] += aw * (double)v[c];
          }
        }
      }
      float* o = out + r * C;
      for (int64_t c = 0; c < C; ++c) o[c] = (float)acc[c];
    }
    free(acc);
  }
  free(lv);
  return 0;
}

/* Backward: given grad_out (B, Q, H*C) produce grad_value (B,K,H,C),
 * grad_loc (B,Q,H,L,P,d) and grad_attn (B,Q,H,L,P).  Work is split over
 * (b, h, level) triples: a sample of level l only touches keys of level l, so
 * every thread owns a disjoint slice of grad_value -- no atomics, and the
 * result does not depend on the thread count.  grad_value is accumulated in
 * float in sample order (per-element relative error near 1e-6 even for the
 * coarsest levels, far inside the 1e-4 gradient tolerance); per-sample
 * scalars are accumulated in double. */
int msda_oracle_bwd(int ndim, const float* value, const int64_t* shapes, int64_t B,
                    int64_t K, int64_t H, int64_t C, int64_t Q, int64_t L, int64_t P,
                    const float* loc, const float* attn, int clamp, double eps,
                    const float* grad_out, float* grad_value, float* grad_loc,
                    float* grad_attn, int nthreads) {
  if (ndim != 2 && ndim != 3) return 1;
  level_t* lv = (level_t*)malloc(sizeof(level_t) * (size_t)(L > 0 ? L : 1));
  if (!lv) return 2;
  if (build_levels(ndim, shapes, L, lv) != K) { free(lv); return 3; }
  float lo, hi;
  clamp_bounds(eps, &lo, &hi);
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#else
  (void)nthreads;
#endif
  /* Keys not covered by any level (none when K matches) stay zero. */
  memset(grad_value, 0, sizeof(float) * (size_t)(B * K * H * C));
  const int64_t ntask = B * H * L;
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t task = 0; task < ntask; ++task) {
    const int64_t l = task % L;
    const int64_t bh = task / L;
    const int64_t b = bh / H, h = bh % H;
    for (int64_t q = 0; q < Q; ++q) {
      const int64_t r = (b * Q + q) * H + h;
      const float* go = grad_out + r * C;
      for (int64_t p = 0; p < P; ++p) {
        const int64_t s = (r * L + l) * P + p;
        point_t pt;
        resolve_point(ndim, &lv[l], loc + s * ndim, clamp, lo, hi, &pt);
        const double a = attn[s];
        double g_attn = 0.0;
        double g_ix[3] = {0.0, 0.0, 0.0};
        for (int n = 0; n < pt.ncorner; ++n) {
          const float* v = value + ((b * K + pt.key[n]) * H + h) * C;
          double dot = 0.0;
          for (int64_t c = 0; c < C; ++c) dot += (double)go[c] * (double)v[c];
          g_attn += (double)pt.w[n] * dot;
          for (int ax = 0; ax < ndim; ++ax) g_ix[ax] += (double)pt.dw[ax][n] * dot;
          const double aw = a * (double)pt.w[n];
          float* gvr = grad_value + ((b * K + pt.key[n]) * H + h) * C;
          for (int64_t c = 0; c < C; ++c) gvr[c] += (float)(aw * (double)go[c]);
        }
        grad_attn[s] = (float)g_attn;
        for (int ax = 0; ax < ndim; ++ax) {
          /* d ix / d loc = size: 2 from grid = 2*loc - 1, size/2 from ix */
          const double gl = a * g_ix[ax] * (double)lv[l].size[ax];
          grad_loc[s * ndim + ax] = pt.pass[ax] ? (float)gl : 0.0f;
        }
      }
    }
  }
  free(lv);
  return 0;
}

/* Cell index a coordinate resolves to (test helper for boundary cases). */
int64_t msda_oracle_cell(float loc, int64_t size, int clamp, double eps) {
  float lo, hi;
  clamp_bounds(eps, &lo, &hi);
  float g = 2.0f * loc;
  g = g - 1.0f;
  if (clamp) {
    if (g < lo) g = lo;
    if (g > hi) g = hi;
  }
  float t = g + 1.0f;
  t = t * (float)size;
  t = t - 1.0f;
  return (int64_t)floorf(t / 2.0f);
}
