/*
 * dcnv2_oracle.c — CPU restatement of the reference DCNv2 forward, used ONLY as the test
 * checker and as the timed CPU baseline (it is test infrastructure, never part of libdcnv2).
 *
 * It restates, per precision, what flairziv/tensorrt-dcnv2-plugin computes on its fast path:
 *   bilinear sample        src/dcn_kernel.cu:19-30   (per-corner zero padding, torchvision rules)
 *   deformable im2col      src/dcn_kernel.cu:138-156 (fp32), :184-201 (fp16: cols rounded to
 *                          half), :218-235 (int8: fp32 cols in the integer-amplitude domain)
 *   GEMM + bias epilogues  src/dcn_plugin.cpp:135-174, src/dcn_kernel.cu:168-178, :208-216,
 *                          :241-257
 * and extends it the way torchvision.ops.deform_conv2d (the reference's oracle,
 * python/01_oracle_and_export.py:59-61) does, because the reference fast path ignores both:
 *   batch N > 1            image n reads x[n], offset[n], mask[n] and writes y[n]
 *   deformable groups dg   group g uses offset channels [2*g*T, 2*(g+1)*T), mask channels
 *                          [g*T, (g+1)*T) and input channels [g*C/dg, (g+1)*C/dg)
 *
 * oracle_forward_i8_exact() is the exact int32-domain INT8 definition that the tensor-core
 * kernels implement. Each column value is the bilinear sample of int8 x requantised in fixed
 * point: the mask is clamped to [0, 1] (NaN -> 0), the corner weights a_k = m * fy * fx are
 * formed in single precision as written below, w_k = min(rint(a_k * 65536), 65535) (0 for
 * NaN or a_k <= 0), and c = floor((sum_k w_k * x_k + 32768) / 65536), always in [-128, 127]
 * (|c - m * bilinear(x)| <= 0.5 + 2^-7). The products w_q * c are summed exactly in integers.
 *
 * Compile with -ffp-contract=off so that every float operation rounds as written.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
  int32_t n, c, h, w, out_c, kernel, stride, padding, dilation, groups;
} oracle_shape;

static inline int out_dim(int in, int k, int s, int p, int d) {
  return (in + 2 * p - d * (k - 1) - 1) / s + 1;
}

/* ---- half-precision helpers (IEEE binary16, round to nearest even) ---- */
static inline float round_half(float v) { return (float)(_Float16)v; }

/* ---- src/dcn_kernel.cu:19-30: bilinear<T> on one channel plane, fp32 arithmetic ---- */
static float ref_bilinear(const float* in, int H, int W, float h, float w) {
  if (h <= -1.f || h >= (float)H || w <= -1.f || w >= (float)W) return 0.f;
  int h_low = (int)floorf(h), w_low = (int)floorf(w);
  int h_high = h_low + 1, w_high = w_low + 1;
  float lh = h - (float)h_low, lw = w - (float)w_low, hh = 1.f - lh, hw = 1.f - lw;
  float v1 = (h_low >= 0 && w_low >= 0) ? in[h_low * W + w_low] : 0.f;
  float v2 = (h_low >= 0 && w_high <= W - 1) ? in[h_low * W + w_high] : 0.f;
  float v3 = (h_high <= H - 1 && w_low >= 0) ? in[h_high * W + w_low] : 0.f;
  float v4 = (h_high <= H - 1 && w_high <= W - 1) ? in[h_high * W + w_high] : 0.f;
  return hh * hw * v1 + hh * lw * v2 + lh * hw * v3 + lh * lw * v4;
}

/* Sampling geometry of one (pixel, tap) in the tensor-core kernels' operation order:
 * the mask is folded into the four corner weights, invalid corners get weight 0. */
typedef struct {
  float a[4];
  int idx[4]; /* plane offsets of the corners, -1 when invalid */
} tap_geom;

static tap_geom kernel_geom(int H, int W, int base_h, int base_w, float dh, float dw, float m) {
  tap_geom g;
  float hf = (float)base_h + dh;
  float wf = (float)base_w + dw;
  for (int i = 0; i < 4; ++i) { g.a[i] = 0.f; g.idx[i] = -1; }
  if (hf <= -1.f || hf >= (float)H || wf <= -1.f || wf >= (float)W || isnan(hf) || isnan(wf))
    return g;
  float h0f = floorf(hf), w0f = floorf(wf);
  int h0 = (int)h0f, w0 = (int)w0f;
  float lh = hf - h0f, lw = wf - w0f;
  float hh = 1.f - lh, hw = 1.f - lw;
  float a1 = m * (hh * hw), a2 = m * (hh * lw), a3 = m * (lh * hw), a4 = m * (lh * lw);
  if (h0 >= 0 && w0 >= 0) { g.a[0] = a1; g.idx[0] = h0 * W + w0; }
  if (h0 >= 0 && w0 + 1 <= W - 1) { g.a[1] = a2; g.idx[1] = h0 * W + w0 + 1; }
  if (h0 + 1 <= H - 1 && w0 >= 0) { g.a[2] = a3; g.idx[2] = (h0 + 1) * W + w0; }
  if (h0 + 1 <= H - 1 && w0 + 1 <= W - 1) { g.a[3] = a4; g.idx[3] = (h0 + 1) * W + w0 + 1; }
  return g;
}

/* ---- work splitting over a pthread pool ---- */
typedef void (*range_fn)(void* ctx, int64_t begin, int64_t end);
typedef struct { range_fn fn; void* ctx; int64_t b, e; } range_job;
static void* range_thunk(void* p) {
  range_job* j = (range_job*)p;
  j->fn(j->ctx, j->b, j->e);
  return NULL;
}
static void parallel_for(int64_t total, int threads, range_fn fn, void* ctx) {
  if (threads <= 1 || total < 2) { fn(ctx, 0, total); return; }
  if (threads > 256) threads = 256;
  if (threads > total) threads = (int)total;
  pthread_t tid[256];
  range_job jobs[256];
  int64_t chunk = (total + threads - 1) / threads;
  int started = 0;
  for (int t = 0; t < threads; ++t) {
    int64_t b = t * chunk, e = b + chunk < total ? b + chunk : total;
    if (b >= e) break;
    jobs[t].fn = fn; jobs[t].ctx = ctx; jobs[t].b = b; jobs[t].e = e;
    if (pthread_create(&tid[t], NULL, range_thunk, &jobs[t]) != 0) { fn(ctx, b, e); continue; }
    ++started;
    (void)started;
  }
  for (int t = 0; t < threads; ++t) {
    int64_t b = t * chunk;
    if (b >= total) break;
    pthread_join(tid[t], NULL);
  }
}

/* ---- column matrix (per image) ----
 * cols[(c*T + t) * P + p], the reference's row order r = ic*K*K + i*K + j (dcn_kernel.cu:145-146). */
enum { COLS_F32 = 0, COLS_F16 = 1, COLS_I8REF = 2 };

typedef struct {
  const oracle_shape* s;
  int mode, Ho, Wo, T;
  const float* x;      /* image base [C][H][W] (f32 values; for int8 the integer amplitudes) */
  const float* off;    /* image base [dg*2T][Ho][Wo] */
  const float* mask;   /* image base [dg*T][Ho][Wo] */
  float* cols;         /* [C*T][np] for output pixels [p0, p0 + np) */
  int p0, np;
} cols_ctx;

static void cols_range(void* vctx, int64_t b, int64_t e) {
  cols_ctx* q = (cols_ctx*)vctx;
  const oracle_shape* s = q->s;
  const int H = s->h, W = s->w, K = s->kernel, T = q->T, P = q->Ho * q->Wo;
  const int Cg = s->c / s->groups;
  for (int64_t ct = b; ct < e; ++ct) { /* ct = c*T + t */
    int c = (int)(ct / T), t = (int)(ct % T);
    int g = c / Cg, i = t / K, j = t % K;
    const float* plane = q->x + (size_t)c * H * W;
    const float* dhp = q->off + ((size_t)(g * 2 * T + 2 * t)) * P;
    const float* dwp = q->off + ((size_t)(g * 2 * T + 2 * t + 1)) * P;
    const float* mp = q->mask + ((size_t)(g * T + t)) * P;
    float* out = q->cols + (size_t)ct * q->np;
    for (int pi = 0; pi < q->np; ++pi) {
      int p = q->p0 + pi, oh = p / q->Wo, ow = p % q->Wo;
      /* dcn_kernel.cu:152-153: h_im = oh*stride - pad + i*dil + dh */
      float h_im = (float)(oh * s->stride - s->padding + i * s->dilation) + dhp[p];
      float w_im = (float)(ow * s->stride - s->padding + j * s->dilation) + dwp[p];
      float v = mp[p] * ref_bilinear(plane, H, W, h_im, w_im);
      out[pi] = (q->mode == COLS_F16) ? round_half(v) : v;
    }
  }
}

/* ---- GEMM y[o][p] = sum_k W[o][k] * cols[k][p] in double ---- */
typedef struct {
  const float* w;     /* [O][CKK] */
  const float* cols;  /* [CKK][P] */
  double* acc;        /* [O][P] */
  int CKK, P;
} gemm_ctx;

static void gemm_range(void* vctx, int64_t b, int64_t e) {
  gemm_ctx* q = (gemm_ctx*)vctx;
  for (int64_t o = b; o < e; ++o) {
    double* a = q->acc + (size_t)o * q->P;
    for (int p = 0; p < q->P; ++p) a[p] = 0.0;
    const float* wr = q->w + (size_t)o * q->CKK;
    for (int k = 0; k < q->CKK; ++k) {
      double wk = (double)wr[k];
      if (wk == 0.0) continue;
      const float* cr = q->cols + (size_t)k * q->P;
      for (int p = 0; p < q->P; ++p) a[p] += wk * (double)cr[p];
    }
  }
}

/*
 * Reference fast path, fp32 or fp16 (prec 0 / 1). All arrays are float32; for prec 1 they must
 * hold fp16-representable values (the fp16 tensors widened), and y receives fp16 values.
 *   prec 0: cols = m*bilinear (f32), y = W@cols + b            (dcn_plugin.cpp:162-174)
 *   prec 1: cols = half(m*bilinear), yh = half(W@cols),
 *           y = half(float(yh) + b)                            (dcn_plugin.cpp:148-161, :208-216)
 * Returns 0, or -1 on a bad shape / allocation failure.
 */
int oracle_forward_ref_band(const oracle_shape* s, int prec, const float* x, const float* off,
                            const float* mask, const float* w, const float* b, float* y,
                            int threads, int p_begin, int p_end) {
  if (!s || s->n <= 0 || s->c <= 0 || s->groups <= 0 || s->c % s->groups) return -1;
  const int Ho = out_dim(s->h, s->kernel, s->stride, s->padding, s->dilation);
  const int Wo = out_dim(s->w, s->kernel, s->stride, s->padding, s->dilation);
  if (Ho <= 0 || Wo <= 0) return -1;
  const int T = s->kernel * s->kernel, P = Ho * Wo, CKK = s->c * T, O = s->out_c;
  if (p_begin < 0 || p_end > P || p_begin >= p_end) return -1;
  const int NP = p_end - p_begin;
  float* cols = (float*)malloc(sizeof(float) * (size_t)CKK * NP);
  double* acc = (double*)malloc(sizeof(double) * (size_t)O * NP);
  if (!cols || !acc) { free(cols); free(acc); return -1; }
  for (int n = 0; n < s->n; ++n) {
    cols_ctx cc = {s, prec == 1 ? COLS_F16 : COLS_F32, Ho, Wo, T,
                   x + (size_t)n * s->c * s->h * s->w, off + (size_t)n * s->groups * 2 * T * P,
                   mask + (size_t)n * s->groups * T * P, cols, p_begin, NP};
    parallel_for(CKK, threads, cols_range, &cc);
    gemm_ctx gc = {w, cols, acc, CKK, NP};
    parallel_for(O, threads, gemm_range, &gc);
    float* yn = y + (size_t)n * O * NP;
    for (int o = 0; o < O; ++o) {
      float bo = b ? b[o] : 0.f;
      for (int p = 0; p < NP; ++p) {
        double a = acc[(size_t)o * NP + p];
        yn[(size_t)o * NP + p] = (prec == 1) ? round_half(round_half((float)a) + bo)
                                             : (float)(a + (double)bo);
      }
    }
  }
  free(cols);
  free(acc);
  return 0;
}

/* Whole-image form of oracle_forward_ref_band. */
int oracle_forward_ref(const oracle_shape* s, int prec, const float* x, const float* off,
                       const float* mask, const float* w, const float* b, float* y, int threads) {
  if (!s) return -1;
  const int Ho = out_dim(s->h, s->kernel, s->stride, s->padding, s->dilation);
  const int Wo = out_dim(s->w, s->kernel, s->stride, s->padding, s->dilation);
  if (Ho <= 0 || Wo <= 0) return -1;
  return oracle_forward_ref_band(s, prec, x, off, mask, w, b, y, threads, 0, Ho * Wo);
}

/*
 * Reference INT8 fast path (dcn_plugin.cpp:135-147): cols = m*bilinear(x_q) in fp32 on the integer
 * amplitudes (dcn_kernel.cu:218-235), W widened to float without its scale (:241-244), GEMM, then
 * y = y*(x_scale*w_scale) + bias (:249-253).
 */
int oracle_forward_i8_ref(const oracle_shape* s, const int8_t* xq, const float* off,
                          const float* mask, const int8_t* wq, const float* b, float x_scale,
                          float w_scale, float* y, int threads) {
  if (!s || s->n <= 0 || s->c <= 0 || s->groups <= 0 || s->c % s->groups) return -1;
  const int Ho = out_dim(s->h, s->kernel, s->stride, s->padding, s->dilation);
  const int Wo = out_dim(s->w, s->kernel, s->stride, s->padding, s->dilation);
  if (Ho <= 0 || Wo <= 0) return -1;
  const int T = s->kernel * s->kernel, P = Ho * Wo, CKK = s->c * T, O = s->out_c;
  const size_t xi = (size_t)s->c * s->h * s->w;
  float* xf = (float*)malloc(sizeof(float) * xi);
  float* wf = (float*)malloc(sizeof(float) * (size_t)O * CKK);
  float* cols = (float*)malloc(sizeof(float) * (size_t)CKK * P);
  double* acc = (double*)malloc(sizeof(double) * (size_t)O * P);
  if (!xf || !wf || !cols || !acc) { free(xf); free(wf); free(cols); free(acc); return -1; }
  for (size_t k = 0; k < (size_t)O * CKK; ++k) wf[k] = (float)wq[k];
  const float scale = x_scale * w_scale;
  for (int n = 0; n < s->n; ++n) {
    for (size_t k = 0; k < xi; ++k) xf[k] = (float)xq[(size_t)n * xi + k];
    cols_ctx cc = {s, COLS_I8REF, Ho, Wo, T, xf, off + (size_t)n * s->groups * 2 * T * P,
                   mask + (size_t)n * s->groups * T * P, cols, 0, P};
    parallel_for(CKK, threads, cols_range, &cc);
    gemm_ctx gc = {wf, cols, acc, CKK, P};
    parallel_for(O, threads, gemm_range, &gc);
    float* yn = y + (size_t)n * O * P;
    for (int o = 0; o < O; ++o)
      for (int p = 0; p < P; ++p)
        yn[(size_t)o * P + p] = (float)acc[(size_t)o * P + p] * scale + (b ? b[o] : 0.f);
  }
  free(xf); free(wf); free(cols); free(acc);
  return 0;
}

/* ---- exact int32-domain INT8 ---- */
typedef struct {
  const oracle_shape* s;
  int Ho, Wo, T;
  const int8_t* x; const float* off; const float* mask;
  int8_t* cq; /* [C*T][np] for output pixels [p0, p0 + np) */
  int p0, np;
  int rule;   /* 0: fixed-point rule of the kernels; 1: clamp(rint(m * bilinear(x_q))) */
} qcols_ctx;

/* src/dcn_kernel.cu:19-30 on an int8 plane: ref_bilinear with each corner value widened to
 * float as the reference's int8 im2col reads it (:218-235). */
static float ref_bilinear_i8(const int8_t* in, int H, int W, float h, float w) {
  if (h <= -1.f || h >= (float)H || w <= -1.f || w >= (float)W) return 0.f;
  int h_low = (int)floorf(h), w_low = (int)floorf(w);
  int h_high = h_low + 1, w_high = w_low + 1;
  float lh = h - (float)h_low, lw = w - (float)w_low, hh = 1.f - lh, hw = 1.f - lw;
  float v1 = (h_low >= 0 && w_low >= 0) ? (float)in[h_low * W + w_low] : 0.f;
  float v2 = (h_low >= 0 && w_high <= W - 1) ? (float)in[h_low * W + w_high] : 0.f;
  float v3 = (h_high <= H - 1 && w_low >= 0) ? (float)in[h_high * W + w_low] : 0.f;
  float v4 = (h_high <= H - 1 && w_high <= W - 1) ? (float)in[h_high * W + w_high] : 0.f;
  return hh * hw * v1 + hh * lw * v2 + lh * hw * v3 + lh * lw * v4;
}

static float i8_mask(float m) { return isnan(m) ? 0.f : fminf(fmaxf(m, 0.f), 1.f); }
/* 16-bit fixed-point corner weight: rint(a * 2^16) (nearest even), 0 for NaN or a <= 0,
 * at most 65535. */
static int32_t i8_weight(float a) {
  const float v = a * 65536.f; /* exact: power-of-two scaling */
  if (!(v > 0.f)) return 0;
  const float r = rintf(v);
  return r >= 65535.f ? 65535 : (int32_t)r;
}
static int8_t requant(tap_geom* g, const int8_t* plane) {
  int32_t sum = 32768;
  for (int k = 0; k < 4; ++k)
    if (g->idx[k] >= 0) sum += i8_weight(g->a[k]) * (int32_t)plane[g->idx[k]];
  /* floor division by 2^16 (gcc's >> on a negative int is an arithmetic shift) */
  return (int8_t)(sum >> 16);
}

static void qcols_range(void* vctx, int64_t b, int64_t e) {
  qcols_ctx* q = (qcols_ctx*)vctx;
  const oracle_shape* s = q->s;
  const int H = s->h, W = s->w, K = s->kernel, T = q->T, P = q->Ho * q->Wo;
  const int Cg = s->c / s->groups;
  for (int64_t ct = b; ct < e; ++ct) {
    int c = (int)(ct / T), t = (int)(ct % T);
    int g = c / Cg, i = t / K, j = t % K;
    const int8_t* plane = q->x + (size_t)c * H * W;
    const float* dhp = q->off + ((size_t)(g * 2 * T + 2 * t)) * P;
    const float* dwp = q->off + ((size_t)(g * 2 * T + 2 * t + 1)) * P;
    const float* mp = q->mask + ((size_t)(g * T + t)) * P;
    int8_t* out = q->cq + (size_t)ct * q->np;
    for (int pi = 0; pi < q->np; ++pi) {
      const int p = q->p0 + pi, oh = p / q->Wo, ow = p % q->Wo;
      const int bh = oh * s->stride - s->padding + i * s->dilation;
      const int bw = ow * s->stride - s->padding + j * s->dilation;
      if (q->rule == 0) {
        tap_geom gm = kernel_geom(H, W, bh, bw, dhp[p], dwp[p], i8_mask(mp[p]));
        out[pi] = requant(&gm, plane);
      } else {
        /* the reference's fp32 column (dcn_kernel.cu:218-235) rounded to nearest (even) */
        const float v = mp[p] * ref_bilinear_i8(plane, H, W, (float)bh + dhp[p],
                                                (float)bw + dwp[p]);
        float r = rintf(v);
        r = r < -127.f ? -127.f : (r > 127.f ? 127.f : r);
        out[pi] = (int8_t)(isnan(v) ? 0.f : r);
      }
    }
  }
}

typedef struct {
  const int8_t* w; const int8_t* cq; int64_t* acc; int CKK, P;
} igemm_ctx;

static void igemm_range(void* vctx, int64_t b, int64_t e) {
  igemm_ctx* q = (igemm_ctx*)vctx;
  for (int64_t o = b; o < e; ++o) {
    int64_t* a = q->acc + (size_t)o * q->P;
    for (int p = 0; p < q->P; ++p) a[p] = 0;
    const int8_t* wr = q->w + (size_t)o * q->CKK;
    for (int k = 0; k < q->CKK; ++k) {
      int64_t wk = wr[k];
      if (!wk) continue;
      const int8_t* cr = q->cq + (size_t)k * q->P;
      for (int p = 0; p < q->P; ++p) a[p] += wk * (int64_t)cr[p];
    }
  }
}

/*
 * Exact INT8 on output pixels [p_begin, p_end) of every image: cq per column value by
 * `rule` (0: the fixed-point rule of requant() above, which the kernels implement; 1: the
 * reference's fp32 column m * bilinear(x_q) rounded to nearest and clamped to [-127, 127]),
 * acc = sum w_q*cq in int64, y = acc*s + b in double with s = fl32(x_scale*w_scale).
 * y, acc_out (optional, int64) and cols_out (optional, int8 [N][C*T][np]) are laid out
 * [N][O][np] / [N][C*T][np] with np = p_end - p_begin.
 */
int oracle_forward_i8_exact_band(const oracle_shape* s, const int8_t* xq, const float* off,
                                 const float* mask, const int8_t* wq, const float* b,
                                 float x_scale, float w_scale, double* y, int64_t* acc_out,
                                 int8_t* cols_out, int threads, int p_begin, int p_end, int rule) {
  if (!s || s->n <= 0 || s->c <= 0 || s->groups <= 0 || s->c % s->groups) return -1;
  if (rule != 0 && rule != 1) return -1;
  const int Ho = out_dim(s->h, s->kernel, s->stride, s->padding, s->dilation);
  const int Wo = out_dim(s->w, s->kernel, s->stride, s->padding, s->dilation);
  if (Ho <= 0 || Wo <= 0) return -1;
  const int T = s->kernel * s->kernel, P = Ho * Wo, CKK = s->c * T, O = s->out_c;
  if (p_begin < 0 || p_end > P || p_begin >= p_end) return -1;
  const int NP = p_end - p_begin;
  const size_t xi = (size_t)s->c * s->h * s->w;
  int8_t* cq = (int8_t*)malloc((size_t)CKK * NP);
  int64_t* acc = (int64_t*)malloc(sizeof(int64_t) * (size_t)O * NP);
  if (!cq || !acc) { free(cq); free(acc); return -1; }
  const double scale = (double)(x_scale * w_scale);
  for (int n = 0; n < s->n; ++n) {
    qcols_ctx qc = {s, Ho, Wo, T, xq + (size_t)n * xi, off + (size_t)n * s->groups * 2 * T * P,
                    mask + (size_t)n * s->groups * T * P, cq, p_begin, NP, rule};
    parallel_for(CKK, threads, qcols_range, &qc);
    if (cols_out) memcpy(cols_out + (size_t)n * CKK * NP, cq, (size_t)CKK * NP);
    igemm_ctx gc = {wq, cq, acc, CKK, NP};
    parallel_for(O, threads, igemm_range, &gc);
    for (int o = 0; o < O; ++o)
      for (int p = 0; p < NP; ++p) {
        int64_t a = acc[(size_t)o * NP + p];
        if (acc_out) acc_out[((size_t)n * O + o) * NP + p] = a;
        if (y) y[((size_t)n * O + o) * NP + p] = (double)a * scale + (b ? (double)b[o] : 0.0);
      }
  }
  free(cq);
  free(acc);
  return 0;
}

/* Whole-image form of oracle_forward_i8_exact_band with the kernels' fixed-point rule. */
int oracle_forward_i8_exact(const oracle_shape* s, const int8_t* xq, const float* off,
                            const float* mask, const int8_t* wq, const float* b, float x_scale,
                            float w_scale, double* y, int64_t* acc_out, int8_t* cols_out,
                            int threads) {
  if (!s) return -1;
  const int Ho = out_dim(s->h, s->kernel, s->stride, s->padding, s->dilation);
  const int Wo = out_dim(s->w, s->kernel, s->stride, s->padding, s->dilation);
  if (Ho <= 0 || Wo <= 0) return -1;
  return oracle_forward_i8_exact_band(s, xq, off, mask, wq, b, x_scale, w_scale, y, acc_out,
                                      cols_out, threads, 0, Ho * Wo, 0);
}

/*
 * Per-tensor symmetric quantiser of the reference INT8 tests (src/test_dcn_int8.cu:31-42):
 * scale = max|v|/127 (1 when all zero), q = clamp(lroundf(v/scale), -127, 127).
 */
float oracle_quantize_sym(const float* src, int64_t n, int8_t* dst) {
  float mx = 0.f;
  for (int64_t i = 0; i < n; ++i) mx = fmaxf(mx, fabsf(src[i]));
  float scale = (mx > 0.f) ? mx / 127.f : 1.f;
  for (int64_t i = 0; i < n; ++i) {
    long q = lroundf(src[i] / scale);
    q = q < -127 ? -127 : (q > 127 ? 127 : q);
    dst[i] = (int8_t)q;
  }
  return scale;
}

/* Reference naive kernel semantics (src/dcn_kernel.cu:33-65), fp32, with N and groups: an
 * independent restatement (no column matrix) used to cross-check the im2col restatement. */
int oracle_forward_direct(const oracle_shape* s, const float* x, const float* off,
                          const float* mask, const float* w, const float* b, float* y) {
  if (!s || s->n <= 0 || s->c <= 0 || s->groups <= 0 || s->c % s->groups) return -1;
  const int H = s->h, W = s->w, K = s->kernel, T = K * K, O = s->out_c, C = s->c;
  const int Ho = out_dim(H, K, s->stride, s->padding, s->dilation);
  const int Wo = out_dim(W, K, s->stride, s->padding, s->dilation);
  if (Ho <= 0 || Wo <= 0) return -1;
  const int P = Ho * Wo, Cg = C / s->groups;
  for (int n = 0; n < s->n; ++n)
    for (int oc = 0; oc < O; ++oc)
      for (int p = 0; p < P; ++p) {
        int oh = p / Wo, ow = p % Wo;
        double acc = b ? b[oc] : 0.0;
        for (int ic = 0; ic < C; ++ic) {
          int g = ic / Cg;
          const float* plane = x + ((size_t)n * C + ic) * H * W;
          for (int t = 0; t < T; ++t) {
            int i = t / K, j = t % K;
            const float* ob = off + ((size_t)n * s->groups * 2 * T) * P;
            float dh = ob[(size_t)(g * 2 * T + 2 * t) * P + p];
            float dw = ob[(size_t)(g * 2 * T + 2 * t + 1) * P + p];
            float m = mask[((size_t)n * s->groups * T + g * T + t) * P + p];
            float h_im = (float)(oh * s->stride - s->padding + i * s->dilation) + dh;
            float w_im = (float)(ow * s->stride - s->padding + j * s->dilation) + dw;
            acc += (double)w[((size_t)oc * C + ic) * T + t] *
                   (double)(m * ref_bilinear(plane, H, W, h_im, w_im));
          }
        }
        y[((size_t)n * O + oc) * P + p] = (float)acc;
      }
  return 0;
}
