/*
 * CPU oracle for the rustnn dense-contraction path (TEST INFRASTRUCTURE).
 *
 * Plain-C restatement of the reference's CPU arithmetic, used only to check
 * the CUDA library and as the timed CPU baseline.  See rnn_oracle.h for the
 * pinning story.  Each function cites the reference file:line it follows;
 * summation order inside the GEMM differs from the reference's rayon split
 * (which itself varies with the thread count, main.rs:61-63), so parity with
 * this oracle is tolerance based, exactly as it is between two runs of the
 * reference with different thread counts.
 */
#include "rnn_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ======================================================================= */
/* rng.rs                                                                   */
/* ======================================================================= */

static uint64_t splitmix_next(uint64_t *z) {
    /* rng.rs:10-16 */
    *z += 0x9E3779B97F4A7C15ULL;
    uint64_t x = *z;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ULL;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBULL;
    return x ^ (x >> 31);
}

void orc_rng_new(orc_rng *r, uint64_t seed) {
    /* rng.rs:8-20: z starts at seed + golden, and each draw adds it again */
    uint64_t z = seed + 0x9E3779B97F4A7C15ULL;
    for (int i = 0; i < 4; i++) r->s[i] = splitmix_next(&z);
}

static inline uint64_t rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

uint64_t orc_rng_next_u64(orc_rng *r) {
    /* xoshiro256++, rng.rs:23-36 */
    uint64_t *s = r->s;
    uint64_t res = rotl(s[0] + s[3], 23) + s[0];
    uint64_t t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl(s[3], 45);
    return res;
}

float orc_rng_uniform(orc_rng *r) {
    /* rng.rs:50-52: 24 random bits times 2^-24, in f32 */
    return (float)(orc_rng_next_u64(r) >> 40) * (1.0f / (float)(1ULL << 24));
}

float orc_rng_normal(orc_rng *r) {
    /* Box-Muller, rng.rs:55-59, all in f32 */
    float u1 = orc_rng_uniform(r);
    if (u1 < 1e-7f) u1 = 1e-7f;
    float u2 = orc_rng_uniform(r);
    const float tau = 6.28318530717958647692f;
    return sqrtf(-2.0f * logf(u1)) * cosf(tau * u2);
}

uint64_t orc_rng_below(orc_rng *r, uint64_t n) { return orc_rng_next_u64(r) % n; }

void orc_rand_vec(float *out, size_t n, orc_rng *r) {
    for (size_t i = 0; i < n; i++) out[i] = orc_rng_normal(r);
}

/* ======================================================================= */
/* threads                                                                  */
/* ======================================================================= */

static int g_threads = 0;
void orc_set_threads(int n) {
    g_threads = n;
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#endif
}
int orc_get_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ======================================================================= */
/* gemm.rs: packed 6x16 register-blocked kernel (MR/NR/KC of gemm.rs:11-13) */
/* ======================================================================= */

#define MR 6
#define NR 16
#define KC 256

typedef float v8f __attribute__((vector_size(32)));

static inline v8f ld8(const float *p) { v8f v; memcpy(&v, p, 32); return v; }
static inline void st8(float *p, v8f v) { memcpy(p, &v, 32); }

/* C[mr x nr] (+)= Apanel[MR x kc] Bpanel[kc x NR]; gemm.rs:124-214 */
static void micro(int kc, const float *ap, const float *bp, float *c, int ldc,
                  int mr, int nr, int accumulate) {
    v8f c0[MR], c1[MR];
    for (int i = 0; i < MR; i++) { c0[i] = (v8f){0}; c1[i] = (v8f){0}; }
    for (int p = 0; p < kc; p++) {
        v8f b0 = ld8(bp + p * NR), b1 = ld8(bp + p * NR + 8);
        for (int i = 0; i < MR; i++) {
            float a = ap[p * MR + i];
            v8f av = {a, a, a, a, a, a, a, a};
            c0[i] += av * b0;
            c1[i] += av * b1;
        }
    }
    if (mr == MR && nr == NR) {
        for (int i = 0; i < MR; i++) {
            float *d = c + (size_t)i * ldc;
            if (accumulate) {
                st8(d, ld8(d) + c0[i]);
                st8(d + 8, ld8(d + 8) + c1[i]);
            } else {
                st8(d, c0[i]);
                st8(d + 8, c1[i]);
            }
        }
    } else {
        float tmp[MR * NR];
        for (int i = 0; i < MR; i++) { st8(tmp + i * NR, c0[i]); st8(tmp + i * NR + 8, c1[i]); }
        for (int i = 0; i < mr; i++) {
            float *row = c + (size_t)i * ldc;
            for (int j = 0; j < nr; j++) row[j] = accumulate ? row[j] + tmp[i * NR + j] : tmp[i * NR + j];
        }
    }
}

/* PackedA::pack / pack_t, gemm.rs:54-113.  Layout: block q of KC rows of K,
 * then panel i of MR rows, element (p, r) at p*MR + r. */
static void pack_a(float *dst, const float *a, int m, int k, int at, int mpad) {
    int mpan = mpad / MR;
    int nb = (k + KC - 1) / KC;
    for (int q = 0; q < nb; q++) {
        int pc = q * KC, kc = k - pc < KC ? k - pc : KC;
        float *blk = dst + (size_t)q * KC * mpad;
        for (int i = 0; i < mpan; i++) {
            float *panel = blk + (size_t)i * kc * MR;
            for (int p = 0; p < kc; p++)
                for (int r = 0; r < MR; r++) {
                    int row = i * MR + r;
                    float v = 0.0f;
                    if (row < m) v = at ? a[(size_t)(pc + p) * m + row] : a[(size_t)row * k + pc + p];
                    panel[p * MR + r] = v;
                }
        }
    }
}

/* PackedB::pack / pack_t, gemm.rs:340-400 */
static void pack_b(float *dst, const float *b, int n, int k, int bt, int npad) {
    int npan = npad / NR;
    int nb = (k + KC - 1) / KC;
    for (int q = 0; q < nb; q++) {
        int pc = q * KC, kc = k - pc < KC ? k - pc : KC;
        float *blk = dst + (size_t)q * KC * npad;
        for (int j = 0; j < npan; j++) {
            float *panel = blk + (size_t)j * kc * NR;
            for (int p = 0; p < kc; p++)
                for (int t = 0; t < NR; t++) {
                    int col = j * NR + t;
                    float v = 0.0f;
                    if (col < n) v = bt ? b[(size_t)col * k + pc + p] : b[(size_t)(pc + p) * n + col];
                    panel[p * NR + t] = v;
                }
        }
    }
}

/* Shared body of matmul (parallel over MR panels, gemm.rs:471-491) and
 * gemm_small (sequential, gemm.rs:500-545). */
static void gemm_impl(int m, int n, int k, const float *a, int at, const float *b,
                      int bt, float *c, int acc, int parallel) {
    if (m == 0 || n == 0) return;
    if (k == 0) {
        if (!acc) memset(c, 0, sizeof(float) * (size_t)m * n);
        return;
    }
    int mpan = (m + MR - 1) / MR, npan = (n + NR - 1) / NR, nb = (k + KC - 1) / KC;
    int mpad = mpan * MR, npad = npan * NR;
    float *ap = (float *)malloc(sizeof(float) * (size_t)nb * KC * mpad);
    float *bp = (float *)malloc(sizeof(float) * (size_t)nb * KC * npad);
    pack_a(ap, a, m, k, at, mpad);
    pack_b(bp, b, n, k, bt, npad);
#pragma omp parallel for schedule(dynamic, 4) if (parallel && (long)m * n * k > (1L << 18))
    for (int i = 0; i < mpan; i++) {
        int mr = m - i * MR < MR ? m - i * MR : MR;
        for (int j = 0; j < npan; j++) {
            int nr = n - j * NR < NR ? n - j * NR : NR;
            for (int q = 0; q < nb; q++) {
                int kc = k - q * KC < KC ? k - q * KC : KC;
                const float *apan = ap + (size_t)q * KC * mpad + (size_t)i * kc * MR;
                const float *bpan = bp + (size_t)q * KC * npad + (size_t)j * kc * NR;
                micro(kc, apan, bpan, c + (size_t)i * MR * n + j * NR, n, mr, nr, q > 0 || acc);
            }
        }
    }
    free(ap);
    free(bp);
}

void orc_matmul(int m, int n, int k, const float *a, int at, const float *b,
                int bt, float *c, int acc) {
    gemm_impl(m, n, k, a, at, b, bt, c, acc, 1);
}

static void gemm_small(int m, int n, int k, const float *a, int at, const float *b,
                       int bt, float *c, int acc) {
    gemm_impl(m, n, k, a, at, b, bt, c, acc, 0);
}

/* gemm.rs:555-598.  K is split into chunks of KC rows; each chunk adds
 * into a private accumulator and the partials are summed in chunk order. */
void orc_matmul_dw(int m, int n, int k, const float *a, const float *b, float *c) {
    if (m == 0 || n == 0 || k == 0) return;
    int rows = KC < k ? KC : k;
    int nchunk = (k + rows - 1) / rows;
    int nt = orc_get_threads();
    if (nt > nchunk) nt = nchunk;
    float *acc = (float *)calloc((size_t)nt * m * n, sizeof(float));
#pragma omp parallel num_threads(nt)
    {
        int t = 0, T = 1;
#ifdef _OPENMP
        t = omp_get_thread_num();
        T = omp_get_num_threads();
#endif
        float *mine = acc + (size_t)t * m * n;
        /* static contiguous partition of chunks: deterministic for fixed nt */
        int lo = (int)((long)nchunk * t / T), hi = (int)((long)nchunk * (t + 1) / T);
        for (int ch = lo; ch < hi; ch++) {
            int k0 = ch * rows, kk = k - k0 < rows ? k - k0 : rows;
            gemm_small(m, n, kk, a + (size_t)k0 * m, 1, b + (size_t)k0 * n, 0, mine, 1);
        }
    }
    for (int t = 0; t < nt; t++) {
        const float *src = acc + (size_t)t * m * n;
        for (size_t i = 0; i < (size_t)m * n; i++) c[i] += src[i];
    }
    free(acc);
}

void orc_naive_matmul(int m, int n, int k, const float *a, int at, const float *b,
                      int bt, float *c) {
    /* check.rs:105-122 */
    for (int i = 0; i < m; i++)
        for (int j = 0; j < n; j++) {
            float s = 0.0f;
            for (int p = 0; p < k; p++) {
                float av = at ? a[(size_t)p * m + i] : a[(size_t)i * k + p];
                float bv = bt ? b[(size_t)j * k + p] : b[(size_t)p * n + j];
                s += av * bv;
            }
            c[(size_t)i * n + j] = s;
        }
}

/* ======================================================================= */
/* conv.rs + nn.rs Conv2d                                                   */
/* ======================================================================= */

typedef struct {
    int cin, cout, k, stride, pad, h, w, oh, ow;
} conv_spec; /* conv.rs:10-37 */

static conv_spec mkspec(int cin, int cout, int k, int stride, int pad, int h, int w) {
    conv_spec s = {cin, cout, k, stride, pad, h, w, 0, 0};
    s.oh = (h + 2 * pad - k) / stride + 1; /* nn.rs:148-150 */
    s.ow = (w + 2 * pad - k) / stride + 1;
    return s;
}

/* im2col of one image: col[ckk x hw], row r = (ci, kh, kw) in RowMap order
 * (conv.rs:49-58), zero outside the border (gather_span, conv.rs:75-120). */
static void im2col(const conv_spec *s, const float *x, float *col) {
    int hw = s->oh * s->ow;
    for (int ci = 0; ci < s->cin; ci++)
        for (int kh = 0; kh < s->k; kh++)
            for (int kw = 0; kw < s->k; kw++) {
                float *dst = col + (size_t)((ci * s->k + kh) * s->k + kw) * hw;
                for (int oy = 0; oy < s->oh; oy++) {
                    int iy = oy * s->stride + kh - s->pad;
                    for (int ox = 0; ox < s->ow; ox++) {
                        int ix = ox * s->stride + kw - s->pad;
                        float v = 0.0f;
                        if (iy >= 0 && iy < s->h && ix >= 0 && ix < s->w)
                            v = x[((size_t)ci * s->h + iy) * s->w + ix];
                        dst[oy * s->ow + ox] = v;
                    }
                }
            }
}

/* col2im accumulate (scatter_span, conv.rs:124-165) */
static void col2im_add(const conv_spec *s, const float *col, float *dx) {
    int hw = s->oh * s->ow;
    for (int ci = 0; ci < s->cin; ci++)
        for (int kh = 0; kh < s->k; kh++)
            for (int kw = 0; kw < s->k; kw++) {
                const float *src = col + (size_t)((ci * s->k + kh) * s->k + kw) * hw;
                for (int oy = 0; oy < s->oh; oy++) {
                    int iy = oy * s->stride + kh - s->pad;
                    if (iy < 0 || iy >= s->h) continue;
                    for (int ox = 0; ox < s->ow; ox++) {
                        int ix = ox * s->stride + kw - s->pad;
                        if (ix < 0 || ix >= s->w) continue;
                        dx[((size_t)ci * s->h + iy) * s->w + ix] += src[oy * s->ow + ox];
                    }
                }
            }
}

void orc_conv2d_fwd(const float *x, int n, int cin, int h, int w, const float *wt,
                    int cout, int k, int stride, int pad, float *y) {
    conv_spec s = mkspec(cin, cout, k, stride, pad, h, w);
    int ckk = cin * k * k, hw = s.oh * s.ow;
#pragma omp parallel
    {
        float *col = (float *)malloc(sizeof(float) * (size_t)ckk * hw);
#pragma omp for schedule(dynamic)
        for (int i = 0; i < n; i++) {
            /* forward_image, conv.rs:169-203: Y[cout x hw] = W im2col(X) */
            im2col(&s, x + (size_t)i * cin * h * w, col);
            gemm_small(cout, hw, ckk, wt, 0, col, 0, y + (size_t)i * cout * hw, 0);
        }
        free(col);
    }
}

void orc_conv2d_dgrad(const float *dy, int n, int cin, int h, int w, const float *wt,
                      int cout, int k, int stride, int pad, float *dx) {
    conv_spec s = mkspec(cin, cout, k, stride, pad, h, w);
    int ckk = cin * k * k, hw = s.oh * s.ow;
#pragma omp parallel
    {
        float *dcol = (float *)malloc(sizeof(float) * (size_t)ckk * hw);
#pragma omp for schedule(dynamic)
        for (int i = 0; i < n; i++) {
            /* dx_image, conv.rs:207-246: dX = col2im(W^T dY) */
            float *dxi = dx + (size_t)i * cin * h * w;
            memset(dxi, 0, sizeof(float) * (size_t)cin * h * w);
            gemm_small(ckk, hw, cout, wt, 1, dy + (size_t)i * cout * hw, 0, dcol, 0);
            col2im_add(&s, dcol, dxi);
        }
        free(dcol);
    }
}

void orc_conv2d_wgrad(const float *x, const float *dy, int n, int cin, int h, int w,
                      int cout, int k, int stride, int pad, float *dw) {
    conv_spec s = mkspec(cin, cout, k, stride, pad, h, w);
    int ckk = cin * k * k, hw = s.oh * s.ow;
    int nt = orc_get_threads();
    if (nt > n) nt = n;
    float *acc = (float *)calloc((size_t)nt * cout * ckk, sizeof(float));
#pragma omp parallel num_threads(nt)
    {
        int t = 0, T = 1;
#ifdef _OPENMP
        t = omp_get_thread_num();
        T = omp_get_num_threads();
#endif
        float *col = (float *)malloc(sizeof(float) * (size_t)ckk * hw);
        float *mine = acc + (size_t)t * cout * ckk;
        int lo = (int)((long)n * t / T), hi = (int)((long)n * (t + 1) / T);
        for (int i = lo; i < hi; i++) {
            /* dw_image, conv.rs:283-322: dW += dY im2col(X)^T */
            im2col(&s, x + (size_t)i * cin * h * w, col);
            gemm_small(cout, ckk, hw, dy + (size_t)i * cout * hw, 0, col, 1, mine, 1);
        }
        free(col);
    }
    /* nn.rs:218-226: reduce the private accumulators, then w.g += dw */
    for (int t = 0; t < nt; t++) {
        const float *src = acc + (size_t)t * cout * ckk;
        for (size_t i = 0; i < (size_t)cout * ckk; i++) dw[i] += src[i];
    }
    free(acc);
}

/* ======================================================================= */
/* nn.rs BatchNorm2d                                                        */
/* ======================================================================= */

void orc_bn_fwd_train(float *y, int n, int c, int hw, const float *gamma,
                      const float *beta, float *rmean, float *rvar, float mom,
                      float eps, int relu, float *xhat, float *invstd) {
    float m = (float)((size_t)n * hw);
    float *mean = (float *)malloc(sizeof(float) * c);
    float *var = (float *)malloc(sizeof(float) * c);
    /* batch_stats, nn.rs:301-322: f64 sums */
#pragma omp parallel for
    for (int ci = 0; ci < c; ci++) {
        double s = 0.0, s2 = 0.0;
        for (int i = 0; i < n; i++) {
            const float *p = y + ((size_t)i * c + ci) * hw;
            for (int q = 0; q < hw; q++) {
                double v = (double)p[q];
                s += v;
                s2 += v * v;
            }
        }
        double mu = s / (double)m;
        mean[ci] = (float)mu;
        double va = s2 / (double)m - mu * mu;
        var[ci] = (float)(va > 0.0 ? va : 0.0);
    }
    /* run_train, nn.rs:330-336 */
    for (int ci = 0; ci < c; ci++) {
        invstd[ci] = 1.0f / sqrtf(var[ci] + eps);
        rmean[ci] = (1.0f - mom) * rmean[ci] + mom * mean[ci];
        float den = m - 1.0f > 1.0f ? m - 1.0f : 1.0f;
        float unb = var[ci] * m / den;
        rvar[ci] = (1.0f - mom) * rvar[ci] + mom * unb;
    }
    /* nn.rs:338-353 */
#pragma omp parallel for
    for (long idx = 0; idx < (long)n * c; idx++) {
        int ci = (int)(idx % c);
        float mu = mean[ci], is = invstd[ci], g = gamma[ci], b = beta[ci];
        float *yc = y + (size_t)idx * hw;
        float *xh = xhat + (size_t)idx * hw;
        for (int q = 0; q < hw; q++) {
            float h = (yc[q] - mu) * is;
            xh[q] = h;
            float v = g * h + b;
            yc[q] = relu ? (v > 0.0f ? v : 0.0f) : v;
        }
    }
    free(mean);
    free(var);
}

void orc_bn_fwd_eval(float *y, int n, int c, int hw, const float *gamma,
                     const float *beta, const float *rmean, const float *rvar,
                     float eps, int relu) {
    /* nn.rs:358-369 */
    for (long idx = 0; idx < (long)n * c; idx++) {
        int ci = (int)(idx % c);
        float is = 1.0f / sqrtf(rvar[ci] + eps);
        float sc = gamma[ci] * is, sh = beta[ci] - gamma[ci] * is * rmean[ci];
        float *yc = y + (size_t)idx * hw;
        for (int q = 0; q < hw; q++) {
            float v = sc * yc[q] + sh;
            yc[q] = relu ? (v > 0.0f ? v : 0.0f) : v;
        }
    }
}

void orc_bn_bwd(const float *dy, const float *xhat, int n, int c, int hw,
                const float *gamma, const float *invstd, float *dx, float *dgamma,
                float *dbeta) {
    float m = (float)((size_t)n * hw);
    float *dg = (float *)malloc(sizeof(float) * c);
    float *db = (float *)malloc(sizeof(float) * c);
    /* nn.rs:391-406: f32 sums over images then pixels */
#pragma omp parallel for
    for (int ci = 0; ci < c; ci++) {
        float a = 0.0f, b = 0.0f;
        for (int i = 0; i < n; i++) {
            size_t base = ((size_t)i * c + ci) * hw;
            for (int q = 0; q < hw; q++) {
                a += dy[base + q] * xhat[base + q];
                b += dy[base + q];
            }
        }
        dg[ci] = a;
        db[ci] = b;
    }
    /* nn.rs:408-422 */
#pragma omp parallel for
    for (long idx = 0; idx < (long)n * c; idx++) {
        int ci = (int)(idx % c);
        float s = gamma[ci] * invstd[ci] / m;
        const float *dyc = dy + (size_t)idx * hw, *xh = xhat + (size_t)idx * hw;
        float *dxc = dx + (size_t)idx * hw;
        for (int q = 0; q < hw; q++) dxc[q] = s * (m * dyc[q] - db[ci] - xh[q] * dg[ci]);
    }
    for (int ci = 0; ci < c; ci++) {
        dgamma[ci] += dg[ci];
        dbeta[ci] += db[ci];
    }
    free(dg);
    free(db);
}

/* ======================================================================= */
/* nn.rs elementwise / pooling / classifier / loss / SGD                    */
/* ======================================================================= */

void orc_relu_back(float *d, const float *y, size_t len) {
    for (size_t i = 0; i < len; i++)
        if (y[i] <= 0.0f) d[i] = 0.0f;
}
void orc_add(float *a, const float *b, size_t len) {
    for (size_t i = 0; i < len; i++) a[i] += b[i];
}
void orc_add_relu(float *a, const float *b, size_t len) {
    for (size_t i = 0; i < len; i++) {
        float v = a[i] + b[i];
        a[i] = v > 0.0f ? v : 0.0f;
    }
}
void orc_gap_fwd(const float *x, int nc, int hw, float *y) {
    for (int i = 0; i < nc; i++) {
        float s = 0.0f;
        for (int q = 0; q < hw; q++) s += x[(size_t)i * hw + q];
        y[i] = s / (float)hw;
    }
}
void orc_gap_bwd(const float *dy, int nc, int hw, float *dx) {
    for (int i = 0; i < nc; i++) {
        float v = dy[i] / (float)hw;
        for (int q = 0; q < hw; q++) dx[(size_t)i * hw + q] = v;
    }
}

void orc_fc_fwd(const float *x, int n, int fin, int fout, const float *w,
                const float *b, float *y) {
    /* nn.rs:501-520: s starts at the bias */
    for (int i = 0; i < n; i++)
        for (int o = 0; o < fout; o++) {
            float s = b[o];
            for (int j = 0; j < fin; j++) s += w[(size_t)o * fin + j] * x[(size_t)i * fin + j];
            y[(size_t)i * fout + o] = s;
        }
}

void orc_fc_bwd(const float *x, const float *dy, int n, int fin, int fout,
                const float *w, float *dw, float *db, float *dx) {
    /* backward_w, nn.rs:524-539 (skips exact zeros like the reference) */
    for (int i = 0; i < n; i++)
        for (int o = 0; o < fout; o++) {
            float g = dy[(size_t)i * fout + o];
            if (g == 0.0f) continue;
            db[o] += g;
            for (int j = 0; j < fin; j++) dw[(size_t)o * fin + j] += g * x[(size_t)i * fin + j];
        }
    /* backward_x, nn.rs:541-557 */
    memset(dx, 0, sizeof(float) * (size_t)n * fin);
    for (int i = 0; i < n; i++)
        for (int o = 0; o < fout; o++) {
            float g = dy[(size_t)i * fout + o];
            if (g == 0.0f) continue;
            for (int j = 0; j < fin; j++) dx[(size_t)i * fin + j] += g * w[(size_t)o * fin + j];
        }
}

float orc_softmax_ce(const float *logits, const uint32_t *labels, int n, int nclass,
                     float smooth, float *dlogits, int *correct) {
    /* nn.rs:573-637 */
    float inv = 1.0f / (float)n, loss = 0.0f;
    int corr = 0;
    for (int i = 0; i < n; i++) {
        const float *z = logits + (size_t)i * nclass;
        float *d = dlogits + (size_t)i * nclass;
        int y = (int)labels[i];
        float mx = -INFINITY;
        int arg = 0;
        for (int j = 0; j < nclass; j++)
            if (z[j] > mx) { mx = z[j]; arg = j; }
        if (arg == y) corr++;
        float sum = 0.0f;
        for (int j = 0; j < nclass; j++) {
            float e = expf(z[j] - mx);
            d[j] = e;
            sum += e;
        }
        float lse = mx + logf(sum);
        float on = 1.0f - smooth, off = smooth / (float)nclass;
        float l = on * (lse - z[y]);
        if (smooth > 0.0f) {
            float s = 0.0f;
            for (int j = 0; j < nclass; j++) s += lse - z[j];
            l += off * s;
        }
        for (int j = 0; j < nclass; j++) {
            float t = j == y ? on + off : off;
            d[j] = (d[j] / sum - t) * inv;
        }
        loss += l;
    }
    if (correct) *correct = corr;
    return loss * inv;
}

void orc_sgd_step(float *v, float *g, float *m, size_t len, float lr, float mom,
                  float wd, int decay) {
    /* Param::step, nn.rs:102-110 */
    float w = decay ? wd : 0.0f;
    for (size_t i = 0; i < len; i++) {
        float gg = g[i] + w * v[i];
        m[i] = mom * m[i] + gg;
        v[i] -= lr * (gg + mom * m[i]);
        g[i] = 0.0f;
    }
}

/* ======================================================================= */
/* model.rs ResNet                                                          */
/* ======================================================================= */

typedef struct {
    float *v, *g, *m;
    size_t n;
    int decay;
} oparam;

static void param_init(oparam *p, size_t n, int decay) {
    p->v = (float *)calloc(n ? n : 1, sizeof(float));
    p->g = (float *)calloc(n ? n : 1, sizeof(float));
    p->m = (float *)calloc(n ? n : 1, sizeof(float));
    p->n = n;
    p->decay = decay;
}
static void param_free(oparam *p) { free(p->v); free(p->g); free(p->m); }

/* Param::kaiming, nn.rs:95-100 */
static void param_kaiming(oparam *p, size_t fan_in, size_t n, orc_rng *r) {
    param_init(p, n, 1);
    float s = sqrtf(2.0f / (float)fan_in);
    for (size_t i = 0; i < n; i++) p->v[i] = orc_rng_normal(r) * s;
}

typedef struct {
    oparam w;
    int cin, cout, k, stride, pad;
    const float *x; /* cached forward input (not owned), nn.rs:126 */
    int xn, xh, xw;
} oconv;

static void conv_new(oconv *c, int cin, int cout, int k, int stride, int pad, orc_rng *r) {
    /* Conv2d::new, nn.rs:132-145 */
    memset(c, 0, sizeof(*c));
    c->cin = cin; c->cout = cout; c->k = k; c->stride = stride; c->pad = pad;
    param_kaiming(&c->w, (size_t)cin * k * k, (size_t)cout * cin * k * k, r);
}
static int conv_out(const oconv *c, int h) { return (h + 2 * c->pad - c->k) / c->stride + 1; }
static void conv_fwd(oconv *c, const float *x, int n, int h, int w, float *y, int train) {
    orc_conv2d_fwd(x, n, c->cin, h, w, c->w.v, c->cout, c->k, c->stride, c->pad, y);
    if (train) { c->x = x; c->xn = n; c->xh = h; c->xw = w; }
}
static void conv_bwd_w(oconv *c, const float *dy) {
    orc_conv2d_wgrad(c->x, dy, c->xn, c->cin, c->xh, c->xw, c->cout, c->k, c->stride, c->pad, c->w.g);
}
static void conv_bwd(oconv *c, const float *dy, float *dx) {
    conv_bwd_w(c, dy); /* nn.rs:230-250 */
    orc_conv2d_dgrad(dy, c->xn, c->cin, c->xh, c->xw, c->w.v, c->cout, c->k, c->stride, c->pad, dx);
}

typedef struct {
    oparam g, b;
    float *rm, *rv, *xhat, *invstd;
    size_t xcap;
    int c, n, hw;
} obn;

static void bn_new(obn *b, int c) {
    /* BatchNorm2d::new, nn.rs:267-278 */
    memset(b, 0, sizeof(*b));
    param_init(&b->g, c, 0);
    for (int i = 0; i < c; i++) b->g.v[i] = 1.0f;
    param_init(&b->b, c, 0);
    b->rm = (float *)calloc(c, sizeof(float));
    b->rv = (float *)malloc(sizeof(float) * c);
    for (int i = 0; i < c; i++) b->rv[i] = 1.0f;
    b->invstd = (float *)calloc(c, sizeof(float));
    b->c = c;
}
static void bn_free(obn *b) {
    param_free(&b->g); param_free(&b->b);
    free(b->rm); free(b->rv); free(b->xhat); free(b->invstd);
}
static void bn_fwd(obn *b, float *y, int n, int hw, int train, int relu) {
    if (train) {
        size_t need = (size_t)n * b->c * hw;
        if (need > b->xcap) { free(b->xhat); b->xhat = (float *)malloc(sizeof(float) * need); b->xcap = need; }
        b->n = n; b->hw = hw;
        orc_bn_fwd_train(y, n, b->c, hw, b->g.v, b->b.v, b->rm, b->rv, 0.1f, 1e-5f, relu, b->xhat, b->invstd);
    } else {
        orc_bn_fwd_eval(y, n, b->c, hw, b->g.v, b->b.v, b->rm, b->rv, 1e-5f, relu);
    }
}
static void bn_bwd(obn *b, const float *dy, float *dx) {
    orc_bn_bwd(dy, b->xhat, b->n, b->c, b->hw, b->g.v, b->invstd, dx, b->g.g, b->b.g);
}

typedef struct {
    oconv c1, c2, dc;
    obn b1, b2, db;
    int has_down;
    int cin, cout, stride;
    /* activations of the last training forward */
    float *h1, *out, *s;
    size_t cap_h, cap_in;
    int n, h, w, oh, ow;
} oblock;

static void block_new(oblock *b, int cin, int cout, int stride, orc_rng *r) {
    /* BasicBlock::new, model.rs:21-37: c1, c2, then the shortcut conv */
    memset(b, 0, sizeof(*b));
    b->cin = cin; b->cout = cout; b->stride = stride;
    bn_new(&b->b2, cout);
    for (int i = 0; i < cout; i++) b->b2.g.v[i] = 0.0f; /* zero_gamma */
    conv_new(&b->c1, cin, cout, 3, stride, 1, r);
    bn_new(&b->b1, cout);
    conv_new(&b->c2, cout, cout, 3, 1, 1, r);
    b->has_down = stride != 1 || cin != cout;
    if (b->has_down) {
        conv_new(&b->dc, cin, cout, 1, stride, 0, r);
        bn_new(&b->db, cout);
    }
}
static void block_free(oblock *b) {
    param_free(&b->c1.w); param_free(&b->c2.w);
    bn_free(&b->b1); bn_free(&b->b2);
    if (b->has_down) { param_free(&b->dc.w); bn_free(&b->db); }
    free(b->h1); free(b->out); free(b->s);
}

static void block_fwd(oblock *b, const float *x, int n, int h, int w, int train) {
    /* model.rs:39-55 */
    int oh = conv_out(&b->c1, h), ow = conv_out(&b->c1, w);
    size_t no = (size_t)n * b->cout * oh * ow;
    if (no > b->cap_h) {
        free(b->h1); free(b->out); free(b->s);
        b->h1 = (float *)malloc(sizeof(float) * no);
        b->out = (float *)malloc(sizeof(float) * no);
        b->s = (float *)malloc(sizeof(float) * no);
        b->cap_h = no;
    }
    b->n = n; b->h = h; b->w = w; b->oh = oh; b->ow = ow;
    conv_fwd(&b->c1, x, n, h, w, b->h1, train);
    bn_fwd(&b->b1, b->h1, n, oh * ow, train, 1);
    conv_fwd(&b->c2, b->h1, n, oh, ow, b->out, train);
    bn_fwd(&b->b2, b->out, n, oh * ow, train, 0);
    if (b->has_down) {
        conv_fwd(&b->dc, x, n, h, w, b->s, train);
        bn_fwd(&b->db, b->s, n, oh * ow, train, 0);
        orc_add_relu(b->out, b->s, no);
    } else {
        orc_add_relu(b->out, x, no);
    }
}

/* d [n,cout,oh,ow] is consumed; dx [n,cin,h,w] written.  model.rs:57-72 */
static void block_bwd(oblock *b, float *d, float *dx) {
    size_t no = (size_t)b->n * b->cout * b->oh * b->ow;
    size_t ni = (size_t)b->n * b->cin * b->h * b->w;
    orc_relu_back(d, b->out, no);
    float *t = (float *)malloc(sizeof(float) * no);
    float *dmain = (float *)malloc(sizeof(float) * no);
    bn_bwd(&b->b2, d, t);
    conv_bwd(&b->c2, t, dmain);
    orc_relu_back(dmain, b->h1, no);
    bn_bwd(&b->b1, dmain, t);
    conv_bwd(&b->c1, t, dx);
    if (b->has_down) {
        float *ds = (float *)malloc(sizeof(float) * ni);
        bn_bwd(&b->db, d, t);
        conv_bwd(&b->dc, t, ds);
        orc_add(dx, ds, ni);
        free(ds);
    } else {
        orc_add(dx, d, ni);
    }
    free(t);
    free(dmain);
}

struct orc_resnet {
    oconv stem;
    obn stem_bn;
    oblock *blocks;
    int nblocks;
    oparam fcw, fcb;
    int fin, fout;
    float *stem_out;
    size_t cap_stem;
    float *pooled;
    size_t cap_pool;
    int n, fh, fw;
};

orc_resnet *orc_resnet_new(int depth_n, int width, int nclass, uint64_t seed) {
    /* ResNet::new, model.rs:112-133: blocks consume the rng first, then the
     * stem conv, then the classifier (nn.rs:487-498, weights halved). */
    orc_resnet *net = (orc_resnet *)calloc(1, sizeof(orc_resnet));
    orc_rng r;
    orc_rng_new(&r, seed);
    int widths[3] = {width, width * 2, width * 4};
    net->nblocks = 3 * depth_n;
    net->blocks = (oblock *)calloc(net->nblocks, sizeof(oblock));
    int cin = width, bi = 0;
    for (int s = 0; s < 3; s++)
        for (int b = 0; b < depth_n; b++) {
            int stride = (s > 0 && b == 0) ? 2 : 1;
            block_new(&net->blocks[bi++], cin, widths[s], stride, &r);
            cin = widths[s];
        }
    conv_new(&net->stem, 3, width, 3, 1, 1, &r);
    bn_new(&net->stem_bn, width);
    net->fin = width * 4;
    net->fout = nclass;
    param_kaiming(&net->fcw, net->fin, (size_t)net->fin * nclass, &r);
    for (size_t i = 0; i < net->fcw.n; i++) net->fcw.v[i] *= 0.5f;
    param_init(&net->fcb, nclass, 0);
    return net;
}

void orc_resnet_free(orc_resnet *net) {
    if (!net) return;
    param_free(&net->stem.w);
    bn_free(&net->stem_bn);
    for (int i = 0; i < net->nblocks; i++) block_free(&net->blocks[i]);
    free(net->blocks);
    param_free(&net->fcw);
    param_free(&net->fcb);
    free(net->stem_out);
    free(net->pooled);
    free(net);
}

/* for_each_param order, model.rs:159-168 and model.rs:74-86 */
static int collect_params(const orc_resnet *net, oparam **out) {
    int k = 0;
    out[k++] = (oparam *)&net->stem.w;
    out[k++] = (oparam *)&net->stem_bn.g;
    out[k++] = (oparam *)&net->stem_bn.b;
    for (int i = 0; i < net->nblocks; i++) {
        oblock *b = &net->blocks[i];
        out[k++] = &b->c1.w; out[k++] = &b->b1.g; out[k++] = &b->b1.b;
        out[k++] = &b->c2.w; out[k++] = &b->b2.g; out[k++] = &b->b2.b;
        if (b->has_down) { out[k++] = &b->dc.w; out[k++] = &b->db.g; out[k++] = &b->db.b; }
    }
    out[k++] = (oparam *)&net->fcw;
    out[k++] = (oparam *)&net->fcb;
    return k;
}

int orc_resnet_num_tensors(const orc_resnet *net) {
    oparam *ps[4096];
    return collect_params(net, ps);
}

size_t orc_resnet_num_params(const orc_resnet *net) {
    oparam *ps[4096];
    int k = collect_params(net, ps);
    size_t n = 0;
    for (int i = 0; i < k; i++) n += ps[i]->n;
    return n;
}

void orc_resnet_param_info(const orc_resnet *net, int64_t *sizes, int *decay) {
    oparam *ps[4096];
    int k = collect_params(net, ps);
    for (int i = 0; i < k; i++) { sizes[i] = (int64_t)ps[i]->n; decay[i] = ps[i]->decay; }
}

static void copy_flat(const orc_resnet *net, float *out, int which) {
    oparam *ps[4096];
    int k = collect_params(net, ps);
    size_t off = 0;
    for (int i = 0; i < k; i++) {
        const float *src = which == 0 ? ps[i]->v : which == 1 ? ps[i]->g : ps[i]->m;
        memcpy(out + off, src, sizeof(float) * ps[i]->n);
        off += ps[i]->n;
    }
}
void orc_resnet_get_params(const orc_resnet *net, float *out) { copy_flat(net, out, 0); }
void orc_resnet_get_grads(const orc_resnet *net, float *out) { copy_flat(net, out, 1); }
void orc_resnet_get_moments(const orc_resnet *net, float *out) { copy_flat(net, out, 2); }

void orc_resnet_set_params(orc_resnet *net, const float *in) {
    oparam *ps[4096];
    int k = collect_params(net, ps);
    size_t off = 0;
    for (int i = 0; i < k; i++) { memcpy(ps[i]->v, in + off, sizeof(float) * ps[i]->n); off += ps[i]->n; }
}
void orc_resnet_zero_grads(orc_resnet *net) {
    oparam *ps[4096];
    int k = collect_params(net, ps);
    for (int i = 0; i < k; i++) memset(ps[i]->g, 0, sizeof(float) * ps[i]->n);
}

/* for_each_buffer order, model.rs:170-176 and model.rs:88-97 */
static int collect_bns(const orc_resnet *net, obn **out) {
    int k = 0;
    out[k++] = (obn *)&net->stem_bn;
    for (int i = 0; i < net->nblocks; i++) {
        oblock *b = &net->blocks[i];
        out[k++] = &b->b1; out[k++] = &b->b2;
        if (b->has_down) out[k++] = &b->db;
    }
    return k;
}
size_t orc_resnet_num_buffers(const orc_resnet *net) {
    obn *bs[2048];
    int k = collect_bns(net, bs);
    size_t n = 0;
    for (int i = 0; i < k; i++) n += 2 * (size_t)bs[i]->c;
    return n;
}
void orc_resnet_get_buffers(const orc_resnet *net, float *out) {
    obn *bs[2048];
    int k = collect_bns(net, bs);
    size_t off = 0;
    for (int i = 0; i < k; i++) {
        memcpy(out + off, bs[i]->rm, sizeof(float) * bs[i]->c); off += bs[i]->c;
        memcpy(out + off, bs[i]->rv, sizeof(float) * bs[i]->c); off += bs[i]->c;
    }
}

static void resnet_forward_hw(orc_resnet *net, const float *x, int n, int h, int w,
                              int train, float *logits) {
    int c = net->stem.cout;
    size_t ns = (size_t)n * c * h * w;
    if (ns > net->cap_stem) { free(net->stem_out); net->stem_out = (float *)malloc(sizeof(float) * ns); net->cap_stem = ns; }
    conv_fwd(&net->stem, x, n, h, w, net->stem_out, train);
    bn_fwd(&net->stem_bn, net->stem_out, n, h * w, train, 1);
    const float *cur = net->stem_out;
    int ch = h, cw = w;
    for (int i = 0; i < net->nblocks; i++) {
        oblock *b = &net->blocks[i];
        block_fwd(b, cur, n, ch, cw, train);
        cur = b->out;
        ch = b->oh; cw = b->ow;
    }
    net->n = n; net->fh = ch; net->fw = cw;
    size_t np = (size_t)n * net->fin;
    if (np > net->cap_pool) { free(net->pooled); net->pooled = (float *)malloc(sizeof(float) * np); net->cap_pool = np; }
    orc_gap_fwd(cur, n * net->fin, ch * cw, net->pooled);
    orc_fc_fwd(net->pooled, n, net->fin, net->fout, net->fcw.v, net->fcb.v, logits);
}

void orc_resnet_backward(orc_resnet *net, const float *dlogits) {
    /* model.rs:148-157 */
    int n = net->n;
    float *dpool = (float *)malloc(sizeof(float) * (size_t)n * net->fin);
    orc_fc_bwd(net->pooled, dlogits, n, net->fin, net->fout, net->fcw.v, net->fcw.g, net->fcb.g, dpool);
    size_t nd = (size_t)n * net->fin * net->fh * net->fw;
    float *d = (float *)malloc(sizeof(float) * nd);
    orc_gap_bwd(dpool, n * net->fin, net->fh * net->fw, d);
    free(dpool);
    for (int i = net->nblocks - 1; i >= 0; i--) {
        oblock *b = &net->blocks[i];
        float *dx = (float *)malloc(sizeof(float) * (size_t)b->n * b->cin * b->h * b->w);
        block_bwd(b, d, dx);
        free(d);
        d = dx;
    }
    size_t ns = (size_t)n * net->stem.cout * net->stem.xh * net->stem.xw;
    orc_relu_back(d, net->stem_out, ns);
    float *t = (float *)malloc(sizeof(float) * ns);
    bn_bwd(&net->stem_bn, d, t);
    conv_bwd_w(&net->stem, t); /* stem dX is discarded, model.rs:156 */
    free(t);
    free(d);
}

void orc_resnet_step(orc_resnet *net, float lr, float mom, float wd) {
    /* model.rs:206-208 */
    oparam *ps[4096];
    int k = collect_params(net, ps);
    for (int i = 0; i < k; i++) orc_sgd_step(ps[i]->v, ps[i]->g, ps[i]->m, ps[i]->n, lr, mom, wd, ps[i]->decay);
}

void orc_resnet_forward(orc_resnet *net, const float *x, int n, int h, int w,
                        int train, float *logits) {
    /* model.rs:135-146 */
    resnet_forward_hw(net, x, n, h, w, train, logits);
}

float orc_resnet_train_step(orc_resnet *net, const float *x, const uint32_t *labels,
                            int n, float smooth, float lr, float mom, float wd,
                            int *correct) {
    /* train.rs:684-699 with a 3 x 32 x 32 batch */
    float *logits = (float *)malloc(sizeof(float) * (size_t)n * net->fout);
    float *dl = (float *)malloc(sizeof(float) * (size_t)n * net->fout);
    resnet_forward_hw(net, x, n, 32, 32, 1, logits);
    float loss = orc_softmax_ce(logits, labels, n, net->fout, smooth, dl, correct);
    orc_resnet_backward(net, dl);
    orc_resnet_step(net, lr, mom, wd);
    free(logits);
    free(dl);
    return loss;
}

void orc_resnet_eval(orc_resnet *net, const uint8_t *images,
                     const uint8_t *labels, int len, int batch, float *out2) {
    /* eval.rs:15-43 */
    const int pix = 3 * 32 * 32;
    float *x = (float *)malloc(sizeof(float) * (size_t)batch * pix);
    uint32_t *lab = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)batch);
    float *lg = (float *)malloc(sizeof(float) * (size_t)batch * net->fout);
    float *dl = (float *)malloc(sizeof(float) * (size_t)batch * net->fout);
    float sum = 0.0f;
    size_t correct = 0, seen = 0;
    for (int s = 0; s < len;) {
        int bs = batch < len - s ? batch : len - s;
        orc_make_batch_eval(images, labels, (size_t)s, bs, 0, x, lab);
        resnet_forward_hw(net, x, bs, 32, 32, 0, lg);
        int c = 0;
        float l = orc_softmax_ce(lg, lab, bs, net->fout, 0.0f, dl, &c);
        /* sum += l * bs as f32: a rounded product, then the add (the Rust
         * expression is not fused) */
        volatile float prod = l * (float)bs;
        sum += prod;
        correct += (size_t)c;
        seen += (size_t)bs;
        s += bs;
    }
    out2[0] = sum / (float)seen;
    out2[1] = (float)correct / (float)seen;
    free(x);
    free(lab);
    free(lg);
    free(dl);
}

uint64_t orc_resnet_flops(const orc_resnet *net, int h, int w) {
    /* model.rs:179-198 */
    uint64_t f = 0;
    int hh = h, ww = w, c = net->stem.cout;
    f += 2ULL * 3 * 9 * c * hh * ww;
    for (int i = 0; i < net->nblocks; i++) {
        const oblock *b = &net->blocks[i];
        int s = b->c1.stride, oh = hh / s, ow = ww / s;
        f += 2ULL * b->c1.cin * 9 * b->c1.cout * oh * ow;
        f += 2ULL * b->c2.cin * 9 * b->c2.cout * oh * ow;
        if (b->has_down) f += 2ULL * b->dc.cin * b->dc.cout * oh * ow;
        hh = oh; ww = ow;
        c = b->c2.cout;
    }
    f += 2ULL * c * net->fout;
    return f;
}

/* ======================================================================= */
/* attn.rs                                                                  */
/* ======================================================================= */

int orc_rel_index(int th, int tw, int mh, int mw, uint32_t *idx) {
    /* RelGeom::new, attn.rs:29-45 */
    int sy, sx, scale, oy, ox;
    if (mh == th) {
        sy = 2 * th - 1; sx = 2 * tw - 1; scale = 1; oy = th - 1; ox = tw - 1;
    } else {
        sy = 2 * (th - 1) + mh; sx = 2 * (tw - 1) + mw; scale = 2; oy = mh - 1; ox = mw - 1;
    }
    if (idx) {
        size_t k = 0;
        for (int qy = 0; qy < th; qy++)
            for (int qx = 0; qx < tw; qx++)
                for (int my = 0; my < mh; my++)
                    for (int mx = 0; mx < mw; mx++) {
                        int dy = scale * qy - my + oy, dx = scale * qx - mx + ox;
                        idx[k++] = (uint32_t)(dy * sx + dx);
                    }
    }
    return sy * sx;
}

void orc_attn_fwd(int n, int h, int dh, int tq, int tk, int mask_diag,
                  const uint32_t *relidx, int nrel, const float *q, int qstride,
                  int qoff, const float *kv, int kvstride, int koff, int voff,
                  const float *tau, const float *rel, float *p, float *o) {
    const int c = h * dh;
#pragma omp parallel
    {
        float *Q = (float *)malloc(sizeof(float) * (size_t)tq * dh);
        float *K = (float *)malloc(sizeof(float) * (size_t)tk * dh);
        float *V = (float *)malloc(sizeof(float) * (size_t)tk * dh);
        float *S = (float *)malloc(sizeof(float) * (size_t)tq * tk);
        float *O = (float *)malloc(sizeof(float) * (size_t)tq * dh);
#pragma omp for schedule(dynamic)
        for (int i = 0; i < n; i++) {
            for (int hd = 0; hd < h; hd++) {
                /* gather, attn.rs:176-178 */
                for (int r = 0; r < tq; r++)
                    memcpy(Q + (size_t)r * dh, q + ((size_t)i * tq + r) * qstride + qoff + hd * dh, sizeof(float) * dh);
                for (int r = 0; r < tk; r++) {
                    memcpy(K + (size_t)r * dh, kv + ((size_t)i * tk + r) * kvstride + koff + hd * dh, sizeof(float) * dh);
                    memcpy(V + (size_t)r * dh, kv + ((size_t)i * tk + r) * kvstride + voff + hd * dh, sizeof(float) * dh);
                }
                gemm_small(tq, tk, dh, Q, 0, K, 1, S, 0); /* S = Q K^T */
                const float t = tau[hd];
                const float *rb = rel + (size_t)hd * nrel;
                float *pr = p + (((size_t)i * h + hd) * tq) * tk;
                for (int qi = 0; qi < tq; qi++) {
                    const float *sr = S + (size_t)qi * tk;
                    float *dr = pr + (size_t)qi * tk;
                    const uint32_t *ridx = relidx + (size_t)qi * tk;
                    float mx = -INFINITY;
                    for (int kj = 0; kj < tk; kj++) {
                        float val = t * sr[kj] + rb[ridx[kj]];
                        dr[kj] = (mask_diag && kj == qi) ? -INFINITY : val;
                        if (dr[kj] > mx) mx = dr[kj];
                    }
                    float sum = 0.0f;
                    for (int kj = 0; kj < tk; kj++) {
                        float e = dr[kj] == -INFINITY ? 0.0f : expf(dr[kj] - mx);
                        dr[kj] = e;
                        sum += e;
                    }
                    float inv = 1.0f / sum;
                    for (int kj = 0; kj < tk; kj++) dr[kj] *= inv;
                }
                gemm_small(tq, dh, tk, pr, 0, V, 0, O, 0); /* O = P V */
                for (int qi = 0; qi < tq; qi++)
                    memcpy(o + ((size_t)i * tq + qi) * c + hd * dh, O + (size_t)qi * dh, sizeof(float) * dh);
            }
        }
        free(Q); free(K); free(V); free(S); free(O);
    }
}

void orc_attn_bwd(int n, int h, int dh, int tq, int tk, const uint32_t *relidx,
                  int nrel, const float *q, int qstride, int qoff,
                  const float *kv, int kvstride, int koff, int voff,
                  const float *tau, const float *p, const float *dout,
                  float *dq, float *dkv, float *dtau, float *drel) {
    const int c = h * dh;
    /* per-image partials of dtau / drel, summed in image order afterwards
     * (attn.rs:247-342 folds per worker and reduces) */
    float *at = (float *)calloc((size_t)n * h, sizeof(float));
    float *ar = (float *)calloc((size_t)n * h * nrel, sizeof(float));
#pragma omp parallel
    {
        float *Q = (float *)malloc(sizeof(float) * (size_t)tq * dh);
        float *K = (float *)malloc(sizeof(float) * (size_t)tk * dh);
        float *V = (float *)malloc(sizeof(float) * (size_t)tk * dh);
        float *DO = (float *)malloc(sizeof(float) * (size_t)tq * dh);
        float *S = (float *)malloc(sizeof(float) * (size_t)tq * tk);
        float *SD = (float *)malloc(sizeof(float) * (size_t)tq * tk);
        float *DQ = (float *)malloc(sizeof(float) * (size_t)tq * dh);
        float *DK = (float *)malloc(sizeof(float) * (size_t)tk * dh);
        float *DV = (float *)malloc(sizeof(float) * (size_t)tk * dh);
#pragma omp for schedule(dynamic)
        for (int i = 0; i < n; i++) {
            for (int hd = 0; hd < h; hd++) {
                for (int r = 0; r < tq; r++) {
                    memcpy(Q + (size_t)r * dh, q + ((size_t)i * tq + r) * qstride + qoff + hd * dh, sizeof(float) * dh);
                    memcpy(DO + (size_t)r * dh, dout + ((size_t)i * tq + r) * c + hd * dh, sizeof(float) * dh);
                }
                for (int r = 0; r < tk; r++) {
                    memcpy(K + (size_t)r * dh, kv + ((size_t)i * tk + r) * kvstride + koff + hd * dh, sizeof(float) * dh);
                    memcpy(V + (size_t)r * dh, kv + ((size_t)i * tk + r) * kvstride + voff + hd * dh, sizeof(float) * dh);
                }
                const float *pr = p + (((size_t)i * h + hd) * tq) * tk;
                /* dV = P^T dO, attn.rs:270-274 */
                gemm_small(tk, dh, tq, pr, 1, DO, 0, DV, 0);
                for (int r = 0; r < tk; r++) {
                    float *d = dkv + ((size_t)i * tk + r) * kvstride + voff + hd * dh;
                    for (int z = 0; z < dh; z++) d[z] += DV[(size_t)r * dh + z];
                }
                /* dP = dO V^T, then dS = P (dP - rowdot), attn.rs:276-290 */
                gemm_small(tq, tk, dh, DO, 0, V, 1, S, 0);
                for (int qi = 0; qi < tq; qi++) {
                    float *sr = S + (size_t)qi * tk;
                    const float *prr = pr + (size_t)qi * tk;
                    float dot = 0.0f;
                    for (int kj = 0; kj < tk; kj++) dot += sr[kj] * prr[kj];
                    for (int kj = 0; kj < tk; kj++) sr[kj] = prr[kj] * (sr[kj] - dot);
                }
                /* dtau from the recomputed raw scores, attn.rs:292-308 */
                gemm_small(tq, tk, dh, Q, 0, K, 1, SD, 0);
                float acc = 0.0f;
                for (size_t z = 0; z < (size_t)tq * tk; z++) acc += S[z] * SD[z];
                at[(size_t)i * h + hd] += acc;
                /* drel, attn.rs:309-315 */
                float *arh = ar + ((size_t)i * h + hd) * nrel;
                for (int qi = 0; qi < tq; qi++)
                    for (int kj = 0; kj < tk; kj++)
                        arh[relidx[(size_t)qi * tk + kj]] += S[(size_t)qi * tk + kj];
                const float t = tau[hd];
                for (size_t z = 0; z < (size_t)tq * tk; z++) S[z] *= t;
                /* dQ = dS K, dK = dS^T Q, attn.rs:318-327 */
                gemm_small(tq, dh, tk, S, 0, K, 0, DQ, 0);
                for (int r = 0; r < tq; r++) {
                    float *d = dq + ((size_t)i * tq + r) * qstride + qoff + hd * dh;
                    for (int z = 0; z < dh; z++) d[z] += DQ[(size_t)r * dh + z];
                }
                gemm_small(tk, dh, tq, S, 1, Q, 0, DK, 0);
                for (int r = 0; r < tk; r++) {
                    float *d = dkv + ((size_t)i * tk + r) * kvstride + koff + hd * dh;
                    for (int z = 0; z < dh; z++) d[z] += DK[(size_t)r * dh + z];
                }
            }
        }
        free(Q); free(K); free(V); free(DO); free(S); free(SD); free(DQ); free(DK); free(DV);
    }
    for (int i = 0; i < n; i++) {
        for (int hd = 0; hd < h; hd++) dtau[hd] += at[(size_t)i * h + hd];
        for (size_t z = 0; z < (size_t)h * nrel; z++) drel[z] += ar[(size_t)i * h * nrel + z];
    }
    free(at);
    free(ar);
}

/* ======================================================================= */
/* norm.rs LayerNorm                                                        */
/* ======================================================================= */

void orc_layernorm_fwd(const float *x, int rows, int c, const float *g, const float *b,
                       float eps, float *y, float *xhat, float *invstd) {
#pragma omp parallel for
    for (int r = 0; r < rows; r++) {
        const float *xr = x + (size_t)r * c;
        double s = 0.0, s2 = 0.0;
        for (int j = 0; j < c; j++) {
            s += (double)xr[j];
            s2 += (double)xr[j] * (double)xr[j];
        }
        double m = (double)c, mu = s / m;
        double va = s2 / m - mu * mu;
        float var = (float)(va > 0.0 ? va : 0.0);
        float is = 1.0f / sqrtf(var + eps);
        if (invstd) invstd[r] = is;
        for (int j = 0; j < c; j++) {
            float hh = (xr[j] - (float)mu) * is;
            if (xhat) xhat[(size_t)r * c + j] = hh;
            y[(size_t)r * c + j] = g[j] * hh + b[j];
        }
    }
}

void orc_layernorm_bwd(const float *dy, const float *xhat, const float *invstd, int rows,
                       int c, const float *g, float *dx, float *dg, float *db) {
    for (int r = 0; r < rows; r++)
        for (int j = 0; j < c; j++) {
            dg[j] += dy[(size_t)r * c + j] * xhat[(size_t)r * c + j];
            db[j] += dy[(size_t)r * c + j];
        }
    float inv = 1.0f / (float)c;
#pragma omp parallel for
    for (int r = 0; r < rows; r++) {
        const float *dyr = dy + (size_t)r * c, *xh = xhat + (size_t)r * c;
        float m1 = 0.0f, m2 = 0.0f;
        for (int j = 0; j < c; j++) {
            float d = dyr[j] * g[j];
            m1 += d;
            m2 += d * xh[j];
        }
        for (int j = 0; j < c; j++) {
            float d = dyr[j] * g[j];
            dx[(size_t)r * c + j] = invstd[r] * (d - m1 * inv - xh[j] * m2 * inv);
        }
    }
}

/* ======================================================================= */
/* linear.rs                                                                */
/* ======================================================================= */

void orc_linear_fwd(const float *x, int rows, int fin, int fout, const float *w, const float *b,
                    float *y) {
    orc_matmul(rows, fout, fin, x, 0, w, 1, y, 0);
    if (b)
        for (int r = 0; r < rows; r++)
            for (int o = 0; o < fout; o++) y[(size_t)r * fout + o] += b[o];
}

void orc_linear_bwd(const float *x, const float *dy, int rows, int fin, int fout, const float *w,
                    float *dw, float *db, float *dx) {
    orc_matmul_dw(fout, fin, rows, dy, x, dw);
    if (db)
        for (int r = 0; r < rows; r++)
            for (int o = 0; o < fout; o++) db[o] += dy[(size_t)r * fout + o];
    orc_matmul(rows, fin, fout, dy, 0, w, 0, dx, 0);
}

/* ======================================================================= */
/* optim.rs                                                                 */
/* ======================================================================= */

void orc_newton_schulz(float *g, int rows, int cols, int steps) {
    /* optim.rs:124-145: work on the wide orientation (m <= n) */
    int m, n, tr;
    if (rows <= cols) { m = rows; n = cols; tr = 0; } else { m = cols; n = rows; tr = 1; }
    float *x = (float *)malloc(sizeof(float) * (size_t)m * n);
    float *a = (float *)malloc(sizeof(float) * (size_t)m * m);
    float *aa = (float *)malloc(sizeof(float) * (size_t)m * m);
    float *t = (float *)malloc(sizeof(float) * (size_t)m * n);
    if (!tr) memcpy(x, g, sizeof(float) * (size_t)m * n);
    else
        for (int i = 0; i < rows; i++)
            for (int j = 0; j < cols; j++) x[(size_t)j * rows + i] = g[(size_t)i * cols + j];
    float ss = 0.0f;
    for (size_t i = 0; i < (size_t)m * n; i++) ss += x[i] * x[i];
    float norm = sqrtf(ss) + 1e-7f;
    float inv = 1.0f / norm;
    for (size_t i = 0; i < (size_t)m * n; i++) x[i] *= inv;
    const float A = 3.4445f, B = -4.7750f, Cc = 2.0315f; /* optim.rs:24-26 */
    for (int s = 0; s < steps; s++) {
        gemm_small(m, m, n, x, 0, x, 1, a, 0);   /* A = X X^T */
        gemm_small(m, m, m, a, 0, a, 0, aa, 0);  /* AA = A A */
        for (size_t i = 0; i < (size_t)m * m; i++) a[i] = B * a[i] + Cc * aa[i];
        gemm_small(m, n, m, a, 0, x, 0, t, 0);   /* T = B X */
        for (size_t i = 0; i < (size_t)m * n; i++) x[i] = A * x[i] + t[i];
    }
    if (!tr) memcpy(g, x, sizeof(float) * (size_t)m * n);
    else
        for (int i = 0; i < rows; i++)
            for (int j = 0; j < cols; j++) g[(size_t)i * cols + j] = x[(size_t)j * rows + i];
    free(x); free(a); free(aa); free(t);
}

void orc_muon_step(float *v, float *g, float *m, int rows, int cols, int steps, float lr,
                   float mom, float wd, int decay) {
    /* optim.rs:184-197 */
    size_t n = (size_t)rows * cols;
    float wdp = decay ? wd : 0.0f;
    for (size_t i = 0; i < n; i++) {
        m[i] = mom * m[i] + g[i];
        g[i] += mom * m[i];
    }
    orc_newton_schulz(g, rows, cols, steps);
    float scale = 0.2f * sqrtf((float)(rows > cols ? rows : cols));
    for (size_t i = 0; i < n; i++) {
        v[i] -= lr * (scale * g[i] + wdp * v[i]);
        g[i] = 0.0f;
    }
}

void orc_adamw_step(float *v, float *g, float *m, float *v2, size_t n, float lr, float wd,
                    int decay, float b1, float b2, float eps, int t) {
    /* step_adam, optim.rs:205-233 */
    float w = decay ? wd : 0.0f;
    float c1 = 1.0f - powf(b1, (float)(t + 1));
    float c2 = 1.0f - powf(b2, (float)(t + 1));
    for (size_t i = 0; i < n; i++) {
        m[i] = b1 * m[i] + (1.0f - b1) * g[i];
        v2[i] = b2 * v2[i] + (1.0f - b2) * g[i] * g[i];
        v[i] -= lr * ((m[i] / c1) / (sqrtf(v2[i] / c2) + eps) + w * v[i]);
        g[i] = 0.0f;
    }
}

float orc_clip(float *g, size_t n, float max) {
    /* clip_, optim.rs:237-250: f64 sum of squares */
    double sq = 0.0;
    for (size_t i = 0; i < n; i++) sq += (double)g[i] * (double)g[i];
    float norm = (float)sqrt(sq);
    if (norm > max && norm > 0.0f) {
        float s = max / norm;
        for (size_t i = 0; i < n; i++) g[i] *= s;
    }
    return norm;
}

void orc_ema_update(float *e, const float *v, size_t n, float decay, int t) {
    /* Ema::update, optim.rs:281-286 (t already incremented) */
    float cap = (1.0f + (float)t) / (10.0f + (float)t);
    float d = decay < cap ? decay : cap;
    for (size_t i = 0; i < n; i++) e[i] = d * e[i] + (1.0f - d) * v[i];
}

/* ======================================================================= */
/* rustvit glue                                                             */
/* ======================================================================= */

void orc_layerscale_fwd(const float *x, int rows, int c, const float *l, float *y) {
    for (size_t i = 0; i < (size_t)rows * c; i++) y[i] = x[i] * l[i % c];
}

void orc_layerscale_bwd(const float *dy, const float *x, int rows, int c, const float *l, float *dl,
                        float *dx) {
    for (int r = 0; r < rows; r++)
        for (int j = 0; j < c; j++) dl[j] += dy[(size_t)r * c + j] * x[(size_t)r * c + j];
    for (size_t i = 0; i < (size_t)rows * c; i++) dx[i] = dy[i] * l[i % c];
}

static float sigmoidf_(float z) { return 1.0f / (1.0f + expf(-z)); }

void orc_swiglu_act_fwd(const float *ab, int rows, int h, float *u) {
    for (int r = 0; r < rows; r++)
        for (int j = 0; j < h; j++) {
            float a = ab[(size_t)r * 2 * h + j];
            u[(size_t)r * h + j] = a * sigmoidf_(a) * ab[(size_t)r * 2 * h + h + j];
        }
}

void orc_swiglu_act_bwd(const float *du, const float *ab, int rows, int h, float *dab) {
    for (int r = 0; r < rows; r++)
        for (int j = 0; j < h; j++) {
            float a = ab[(size_t)r * 2 * h + j], b = ab[(size_t)r * 2 * h + h + j];
            float s = sigmoidf_(a), d = du[(size_t)r * h + j];
            dab[(size_t)r * 2 * h + j] = d * b * s * (1.0f + a * (1.0f - s));
            dab[(size_t)r * 2 * h + h + j] = d * a * s;
        }
}

void orc_dwconv3_fwd(const float *x, int n, int th, int tw, int c, const float *w, const float *b,
                     float *y) {
    size_t img = (size_t)th * tw * c;
    for (int i = 0; i < n; i++) {
        const float *xi = x + i * img;
        float *yi = y + i * img;
        for (int oy = 0; oy < th; oy++)
            for (int ox = 0; ox < tw; ox++) {
                float *dst = yi + ((size_t)oy * tw + ox) * c;
                for (int j = 0; j < c; j++) dst[j] = b[j];
                for (int ky = 0; ky < 3; ky++) {
                    int sy = oy + ky - 1;
                    if (sy < 0 || sy >= th) continue;
                    for (int kx = 0; kx < 3; kx++) {
                        int sx = ox + kx - 1;
                        if (sx < 0 || sx >= tw) continue;
                        const float *wr = w + (size_t)(ky * 3 + kx) * c;
                        const float *src = xi + ((size_t)sy * tw + sx) * c;
                        for (int j = 0; j < c; j++) dst[j] += wr[j] * src[j];
                    }
                }
            }
    }
}

void orc_dwconv3_bwd(const float *dy, const float *x, int n, int th, int tw, int c, const float *w,
                     float *dw, float *db, float *dx) {
    size_t img = (size_t)th * tw * c;
    memset(dx, 0, sizeof(float) * img * n);
    for (int i = 0; i < n; i++) {
        const float *dyi = dy + i * img, *xi = x + i * img;
        float *dxi = dx + i * img;
        for (int oy = 0; oy < th; oy++)
            for (int ox = 0; ox < tw; ox++) {
                const float *d = dyi + ((size_t)oy * tw + ox) * c;
                for (int j = 0; j < c; j++) db[j] += d[j];
                for (int ky = 0; ky < 3; ky++) {
                    int sy = oy + ky - 1;
                    if (sy < 0 || sy >= th) continue;
                    for (int kx = 0; kx < 3; kx++) {
                        int sx = ox + kx - 1;
                        if (sx < 0 || sx >= tw) continue;
                        size_t s = ((size_t)sy * tw + sx) * c;
                        float *acc = dw + (size_t)(ky * 3 + kx) * c;
                        const float *wr = w + (size_t)(ky * 3 + kx) * c;
                        for (int j = 0; j < c; j++) {
                            acc[j] += d[j] * xi[s + j];
                            dxi[s + j] += wr[j] * d[j];
                        }
                    }
                }
            }
    }
}

void orc_seqpool_fwd(const float *x, int n, int t, int c, const float *p, float *z, float *w) {
    for (int i = 0; i < n; i++) {
        const float *xi = x + (size_t)i * t * c;
        float *wi = w + (size_t)i * t, *zi = z + (size_t)i * c;
        float mx = -INFINITY;
        for (int j = 0; j < t; j++) {
            float s = 0.0f;
            for (int k = 0; k < c; k++) s += xi[(size_t)j * c + k] * p[k];
            wi[j] = s;
            if (s > mx) mx = s;
        }
        float sum = 0.0f;
        for (int j = 0; j < t; j++) { wi[j] = expf(wi[j] - mx); sum += wi[j]; }
        float inv = 1.0f / sum;
        for (int k = 0; k < c; k++) zi[k] = 0.0f;
        for (int j = 0; j < t; j++) {
            wi[j] *= inv;
            for (int k = 0; k < c; k++) zi[k] += wi[j] * xi[(size_t)j * c + k];
        }
    }
}

void orc_seqpool_bwd(const float *dz, const float *x, const float *w, int n, int t, int c,
                     const float *p, float *dp, float *dx) {
    float *dwv = (float *)malloc(sizeof(float) * t);
    memset(dx, 0, sizeof(float) * (size_t)n * t * c);
    for (int i = 0; i < n; i++) {
        const float *xi = x + (size_t)i * t * c, *wi = w + (size_t)i * t, *dzi = dz + (size_t)i * c;
        float *dxi = dx + (size_t)i * t * c;
        float dot = 0.0f;
        for (int j = 0; j < t; j++) {
            float s = 0.0f;
            for (int k = 0; k < c; k++) {
                s += dzi[k] * xi[(size_t)j * c + k];
                dxi[(size_t)j * c + k] += wi[j] * dzi[k];
            }
            dwv[j] = s;
            dot += s * wi[j];
        }
        for (int j = 0; j < t; j++) {
            float ds = wi[j] * (dwv[j] - dot);
            for (int k = 0; k < c; k++) {
                dp[k] += ds * xi[(size_t)j * c + k];
                dxi[(size_t)j * c + k] += ds * p[k];
            }
        }
    }
    free(dwv);
}

void orc_droppath_mask(int n, float p, uint64_t seed, float *mask) {
    float keep = 1.0f - p;
    orc_rng r;
    orc_rng_new(&r, seed);
    for (int i = 0; i < n; i++) mask[i] = orc_rng_uniform(&r) < keep ? 1.0f / keep : 0.0f;
}

void orc_token_merge_fwd(const float *z, int n, int th, int c, float *y) {
    int t2 = th / 2;
    const int dys[4] = {0, 0, 1, 1}, dxs[4] = {0, 1, 0, 1};
    for (int i = 0; i < n; i++)
        for (int oy = 0; oy < t2; oy++)
            for (int ox = 0; ox < t2; ox++)
                for (int q = 0; q < 4; q++) {
                    const float *src = z + (((size_t)i * th + 2 * oy + dys[q]) * th + 2 * ox + dxs[q]) * c;
                    float *dst = y + (((size_t)i * t2 + oy) * t2 + ox) * 4 * c + (size_t)q * c;
                    memcpy(dst, src, sizeof(float) * c);
                }
}

void orc_token_merge_bwd(const float *dy, int n, int th, int c, float *dz) {
    int t2 = th / 2;
    const int dys[4] = {0, 0, 1, 1}, dxs[4] = {0, 1, 0, 1};
    for (int i = 0; i < n; i++)
        for (int oy = 0; oy < t2; oy++)
            for (int ox = 0; ox < t2; ox++)
                for (int q = 0; q < 4; q++) {
                    float *dst = dz + (((size_t)i * th + 2 * oy + dys[q]) * th + 2 * ox + dxs[q]) * c;
                    const float *src = dy + (((size_t)i * t2 + oy) * t2 + ox) * 4 * c + (size_t)q * c;
                    memcpy(dst, src, sizeof(float) * c);
                }
}

void orc_tok_from_nchw(const float *x, int n, int c, int hw, float *y) {
    for (int i = 0; i < n; i++)
        for (int ci = 0; ci < c; ci++)
            for (int q = 0; q < hw; q++)
                y[((size_t)i * hw + q) * c + ci] = x[((size_t)i * c + ci) * hw + q];
}

void orc_tok_to_nchw(const float *x, int n, int c, int hw, float *y) {
    for (int i = 0; i < n; i++)
        for (int ci = 0; ci < c; ci++)
            for (int q = 0; q < hw; q++)
                y[((size_t)i * c + ci) * hw + q] = x[((size_t)i * hw + q) * c + ci];
}

void orc_taxo_fwd(float *zf, const float *zc, int n, int nf, int nc, const uint32_t *parent) {
    for (int i = 0; i < n; i++)
        for (int k = 0; k < nf; k++) zf[(size_t)i * nf + k] += zc[(size_t)i * nc + parent[k]];
}

void orc_taxo_bwd(const float *dzf, const float *dzc, int n, int nf, int nc, const uint32_t *parent,
                  float *dc) {
    for (int i = 0; i < n; i++) {
        memcpy(dc + (size_t)i * nc, dzc + (size_t)i * nc, sizeof(float) * nc);
        for (int k = 0; k < nf; k++) dc[(size_t)i * nc + parent[k]] += dzf[(size_t)i * nf + k];
    }
}

float orc_ce_soft(const float *logits, const float *target, const uint32_t *hard, int n, int nclass,
                  float scale, float *dz, int *correct) {
    float inv = 1.0f / (float)n, loss = 0.0f;
    int corr = 0;
    for (int i = 0; i < n; i++) {
        const float *z = logits + (size_t)i * nclass, *t = target + (size_t)i * nclass;
        float *d = dz + (size_t)i * nclass;
        float mx = -INFINITY;
        int arg = 0;
        for (int j = 0; j < nclass; j++)
            if (z[j] > mx) { mx = z[j]; arg = j; }
        float sum = 0.0f;
        for (int j = 0; j < nclass; j++) { d[j] = expf(z[j] - mx); sum += d[j]; }
        float lse = mx + logf(sum), l = 0.0f;
        for (int j = 0; j < nclass; j++) {
            l += t[j] * (lse - z[j]);
            d[j] = (d[j] / sum - t[j]) * inv * scale;
        }
        loss += l;
        corr += arg == (int)hard[i];
    }
    if (correct) *correct = corr;
    return loss * inv;
}

float orc_kl_distill(const float *s, const float *t, int n, int nclass, float temp, float scale,
                     float *dz) {
    float inv = 1.0f / (float)n, it = 1.0f / temp, total = 0.0f;
    float *ps = (float *)malloc(sizeof(float) * nclass), *pt = (float *)malloc(sizeof(float) * nclass);
    for (int i = 0; i < n; i++) {
        const float *zs = s + (size_t)i * nclass, *zt = t + (size_t)i * nclass;
        float *d = dz + (size_t)i * nclass;
        for (int pass = 0; pass < 2; pass++) {
            const float *z = pass ? zt : zs;
            float *o = pass ? pt : ps;
            float mx = -INFINITY;
            for (int j = 0; j < nclass; j++) mx = z[j] > mx ? z[j] : mx;
            float sm = 0.0f;
            for (int j = 0; j < nclass; j++) { o[j] = expf((z[j] - mx) * it); sm += o[j]; }
            float is = 1.0f / sm;
            for (int j = 0; j < nclass; j++) o[j] *= is;
        }
        float l = 0.0f;
        for (int j = 0; j < nclass; j++) {
            if (pt[j] > 1e-9f) {
                float a = pt[j] > 1e-9f ? pt[j] : 1e-9f, b = ps[j] > 1e-9f ? ps[j] : 1e-9f;
                l += pt[j] * (logf(a) - logf(b));
            }
            d[j] += temp * (ps[j] - pt[j]) * inv * scale;
        }
        total += l * temp * temp;
    }
    free(ps); free(pt);
    return total * inv;
}

float orc_hint_mse(const float *pred, const float *target, int n, int c, float scale, float *dz) {
    float inv = 1.0f / (float)((size_t)n * c), l = 0.0f;
    for (int i = 0; i < n; i++) {
        float s = 0.0f;
        for (int j = 0; j < c; j++) {
            float e = pred[(size_t)i * c + j] - target[(size_t)i * c + j];
            s += e * e;
            dz[(size_t)i * c + j] += 2.0f * e * inv * scale;
        }
        l += s;
    }
    return l * inv * scale;
}

/* ---------------------------------------------------------------- rustvit initialisers */

/* Param::trunc_normal, nn.rs:77-89: resample |z| > 2 up to 8 times, clamp. */
void orc_trunc_normal(orc_rng *r, float *out, size_t n, float std) {
    for (size_t i = 0; i < n; i++) {
        float z = orc_rng_normal(r);
        int tries = 0;
        while (fabsf(z) > 2.0f && tries < 8) {
            z = orc_rng_normal(r);
            tries++;
        }
        if (z < -2.0f) z = -2.0f;
        if (z > 2.0f) z = 2.0f;
        out[i] = z * std;
    }
}

/* Param::kaiming, nn.rs:95-100. */
void orc_kaiming(orc_rng *r, float *out, size_t n, int fan_in) {
    const float s = sqrtf(2.0f / (float)fan_in);
    for (size_t i = 0; i < n; i++) out[i] = orc_rng_normal(r) * s;
}
