/* CPU oracle, data pipeline (TEST INFRASTRUCTURE ONLY): a plain-C
 * restatement of the reference's batch builders in data.rs — RandAugment on
 * the bytes, crop / flip / normalise, random erasing, the eval batch and the
 * mixup / cutmix of a batch.
 *
 * This file is compiled with -ffp-contract=off: the reference's f32
 * expressions are evaluated operation by operation (Rust does not fuse a
 * multiply and an add), and a fused multiply-add would round differently and
 * change bytes after the `as u8` truncations. */
#include "rnn_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define IMG 32
#define CH 3
#define PLANE (IMG * IMG)
#define PIX (CH * PLANE)

/* The reference calls f32 logf / cosf / sinf (glibc here, as for the Rust
 * build on this host).  glibc's single-precision results are not correctly
 * rounded for a few percent of arguments; with cr_math set they are replaced
 * by the correctly rounded value ((float) of the double function), which is
 * the convention of the device implementation.  Off by default. */
static int g_cr_math = 0;
void orc_data_set_cr_math(int on) { g_cr_math = on; }
static float o_logf(float x) { return g_cr_math ? (float)log((double)x) : logf(x); }
static float o_cosf(float x) { return g_cr_math ? (float)cos((double)x) : cosf(x); }
static float o_sinf(float x) { return g_cr_math ? (float)sin((double)x) : sinf(x); }

/* Rng::normal (rng.rs:55-59) with the functions above */
static float data_normal(orc_rng *r) {
    float u1 = orc_rng_uniform(r);
    if (u1 < 1e-7f) u1 = 1e-7f;
    float u2 = orc_rng_uniform(r);
    const float tau = 6.28318530717958647692f;
    return sqrtf(-2.0f * o_logf(u1)) * o_cosf(tau * u2);
}

/* data.rs:13-14 */
static const float MEAN[3] = {0.5071f, 0.4865f, 0.4409f};
static const float STDV[3] = {0.2673f, 0.2564f, 0.2762f};

/* data.rs:95-98 */
static float norm(uint8_t v, int c) { return ((float)v / 255.0f - MEAN[c]) / STDV[c]; }

/* f32 -> u8 of `v.clamp(0.0, 255.0) as u8`: saturate, truncate toward zero */
static uint8_t clamp_u8(float v) {
    if (v < 0.0f) v = 0.0f;
    if (v > 255.0f) v = 255.0f;
    return (uint8_t)v;
}

/* data.rs:105-111: outside the image reads mid-grey */
static uint8_t px(const uint8_t *im, int c, int y, int x) {
    if (y < 0 || x < 0 || y >= IMG || x >= IMG) return 128;
    return im[c * PLANE + y * IMG + x];
}

/* data.rs:114-135: inverse affine resampling, bilinear */
static void affine(uint8_t *im, float a, float b, float tx, float c_, float d, float ty) {
    uint8_t src[PIX];
    memcpy(src, im, PIX);
    const float cy = (float)IMG / 2.0f - 0.5f, cx = cy;
    for (int ch = 0; ch < CH; ch++)
        for (int y = 0; y < IMG; y++)
            for (int x = 0; x < IMG; x++) {
                float fy = (float)y - cy, fx = (float)x - cx;
                float sx = a * fx + b * fy + tx + cx;
                float sy = c_ * fx + d * fy + ty + cy;
                float x0f = floorf(sx), y0f = floorf(sy);
                float wx = sx - x0f, wy = sy - y0f;
                int x0 = (int)x0f, y0 = (int)y0f;
                float p00 = px(src, ch, y0, x0), p01 = px(src, ch, y0, x0 + 1);
                float p10 = px(src, ch, y0 + 1, x0), p11 = px(src, ch, y0 + 1, x0 + 1);
                float v = p00 * (1.0f - wx) * (1.0f - wy) + p01 * wx * (1.0f - wy) + p10 * (1.0f - wx) * wy +
                          p11 * wx * wy;
                im[ch * PLANE + y * IMG + x] = clamp_u8(v);
            }
}

/* data.rs:137-142 */
static void blend(uint8_t *im, const uint8_t *other, float f) {
    for (int i = 0; i < PIX; i++) {
        float v = (float)other[i] + f * ((float)im[i] - (float)other[i]);
        im[i] = clamp_u8(v);
    }
}

/* data.rs:144-156 */
static void grayscale(const uint8_t *im, uint8_t *g) {
    for (int p = 0; p < PLANE; p++) {
        float v = 0.299f * (float)im[p] + 0.587f * (float)im[PLANE + p] + 0.114f * (float)im[2 * PLANE + p];
        uint8_t u = clamp_u8(v);
        for (int c = 0; c < CH; c++) g[c * PLANE + p] = u;
    }
}

/* data.rs:160-164 */
static void posterize(uint8_t *im, float v) {
    uint32_t bits = 8 - (uint32_t)(4.0f * v);
    uint8_t mask = (uint8_t)~((1u << (8 - bits)) - 1);
    for (int i = 0; i < PIX; i++) im[i] &= mask;
}

/* data.rs:166-173 */
static void solarize(uint8_t *im, float v) {
    uint8_t th = clamp_u8(255.0f * (1.0f - v));
    for (int i = 0; i < PIX; i++)
        if (im[i] >= th) im[i] = (uint8_t)(255 - im[i]);
}

/* data.rs:176-187 */
static void autocontrast(uint8_t *im) {
    for (int c = 0; c < CH; c++) {
        uint8_t *s = im + c * PLANE;
        uint8_t lo = 255, hi = 0;
        for (int i = 0; i < PLANE; i++) {
            if (s[i] < lo) lo = s[i];
            if (s[i] > hi) hi = s[i];
        }
        if (hi > lo) {
            float k = 255.0f / (float)(hi - lo);
            for (int i = 0; i < PLANE; i++) s[i] = clamp_u8((float)(uint8_t)(s[i] - lo) * k);
        }
    }
}

/* data.rs:190-207 */
static void equalize(uint8_t *im) {
    for (int c = 0; c < CH; c++) {
        uint8_t *s = im + c * PLANE;
        uint32_t hist[256] = {0}, cdf[256];
        for (int i = 0; i < PLANE; i++) hist[s[i]]++;
        uint32_t acc = 0, lo = 0;
        int found = 0;
        for (int i = 0; i < 256; i++) {
            acc += hist[i];
            cdf[i] = acc;
            if (!found && acc > 0) {
                lo = acc;
                found = 1;
            }
        }
        uint32_t den = (uint32_t)PLANE > lo ? (uint32_t)PLANE - lo : 0;
        if (den < 1) den = 1;
        for (int i = 0; i < PLANE; i++) s[i] = (uint8_t)(((cdf[s[i]] - lo) * 255u) / den);
    }
}

/* data.rs:227-237: 3x3 blur tap, centre 5, neighbours 3/8, over 8 */
static uint8_t blur_tap(const uint8_t *src, int c, int y, int x) {
    float s = 0.0f;
    for (int dy = 0; dy < 3; dy++)
        for (int dx = 0; dx < 3; dx++) {
            float w = (dy == 1 && dx == 1) ? 5.0f : 1.0f / 8.0f * 3.0f;
            s += w * (float)px(src, c, y + dy - 1, x + dx - 1);
        }
    return clamp_u8(s / 8.0f);
}

/* data.rs:209-253 */
static void apply_op(uint8_t *im, int op, float v, orc_rng *rng) {
    /* data.rs:262-263: the sign is drawn for every op */
    float sign = (orc_rng_next_u64(rng) >> 32) & 1u ? 1.0f : -1.0f;
    float f = 1.0f + sign * 0.9f * v;
    uint8_t tmp[PIX];
    switch (op) {
        case 0: affine(im, 1.0f, sign * 0.3f * v, 0.0f, 0.0f, 1.0f, 0.0f); break;
        case 1: affine(im, 1.0f, 0.0f, 0.0f, sign * 0.3f * v, 1.0f, 0.0f); break;
        case 2: affine(im, 1.0f, 0.0f, sign * 10.0f * v, 0.0f, 1.0f, 0.0f); break;
        case 3: affine(im, 1.0f, 0.0f, 0.0f, 0.0f, 1.0f, sign * 10.0f * v); break;
        case 4: {
            float t = sign * 30.0f * v * 3.14159265358979323846f / 180.0f;
            affine(im, o_cosf(t), -o_sinf(t), 0.0f, o_sinf(t), o_cosf(t), 0.0f);
            break;
        }
        case 5: posterize(im, v); break;
        case 6: solarize(im, v); break;
        case 7: autocontrast(im); break;
        case 8: equalize(im); break;
        case 9: memset(tmp, 0, PIX); blend(im, tmp, f); break;
        case 10: grayscale(im, tmp); blend(im, tmp, f); break;
        case 11: {
            grayscale(im, tmp);
            uint32_t sum = 0;
            for (int p = 0; p < PLANE; p++) sum += tmp[p];
            memset(tmp, (int)(uint8_t)(sum / PLANE), PIX);
            blend(im, tmp, f);
            break;
        }
        default: {
            uint8_t src[PIX];
            memcpy(src, im, PIX);
            memcpy(tmp, im, PIX);
            for (int c = 0; c < CH; c++)
                for (int y = 1; y < IMG - 1; y++)
                    for (int x = 1; x < IMG - 1; x++) tmp[c * PLANE + y * IMG + x] = blur_tap(src, c, y, x);
            blend(im, tmp, f);
        }
    }
}

/* data.rs:297-306 */
static void randaugment(uint8_t *work, float ra_mag, int ra_n, orc_rng *rng) {
    if (ra_mag <= 0.0f) return;
    for (int i = 0; i < ra_n; i++) {
        int op = (int)orc_rng_below(rng, 13);
        float v = ra_mag * (1.0f + 0.5f * data_normal(rng));
        if (v < 0.0f) v = 0.0f;
        if (v > 1.0f) v = 1.0f;
        apply_op(work, op, v, rng);
    }
}

/* data.rs:331-360 */
static void crop_flip_normalize(const uint8_t *src, float *dst, int dy, int dx, int flip) {
    for (int c = 0; c < CH; c++) {
        float border = -MEAN[c] / STDV[c];
        for (int y = 0; y < IMG; y++) {
            int sy = y + dy;
            float *row = dst + c * PLANE + y * IMG;
            for (int x = 0; x < IMG; x++) {
                int sx = (flip ? IMG - 1 - x : x) + dx;
                row[x] = (sy >= 0 && sy < IMG && sx >= 0 && sx < IMG) ? norm(src[c * PLANE + sy * IMG + sx], c)
                                                                       : border;
            }
        }
    }
}

/* data.rs:364-377 */
static void random_erase(float *dst, float erase, int erase_side, orc_rng *rng) {
    if (erase <= 0.0f || orc_rng_uniform(rng) >= erase) return;
    int cy = (int)orc_rng_below(rng, IMG), cx = (int)orc_rng_below(rng, IMG);
    int h = erase_side / 2;
    int y0 = cy - h > 0 ? cy - h : 0, y1 = cy + h < IMG ? cy + h : IMG;
    int x0 = cx - h > 0 ? cx - h : 0, x1 = cx + h < IMG ? cx + h : IMG;
    for (int c = 0; c < CH; c++)
        for (int y = y0; y < y1; y++)
            for (int x = x0; x < x1; x++) dst[c * PLANE + y * IMG + x] = data_normal(rng);
}

void orc_make_batch_train(const uint8_t *images, const uint8_t *labels, const uint8_t *coarse,
                          const uint32_t *idx, int bs, int pad, float ra_mag, int ra_n, float erase,
                          int erase_side, uint64_t seed, float *out, uint32_t *labels_out,
                          uint32_t *coarse_out) {
    /* data.rs:384-412: each image has its own generator, seeded from the
     * batch seed and its slot in the batch */
    for (int b = 0; b < bs; b++) {
        labels_out[b] = labels[idx[b]];
        if (coarse && coarse_out) coarse_out[b] = coarse[idx[b]];
    }
    for (int b = 0; b < bs; b++) {
        orc_rng rng;
        orc_rng_new(&rng, seed ^ ((uint64_t)b * 0x9E3779B97F4A7C15ULL));
        uint8_t work[PIX];
        memcpy(work, images + (size_t)idx[b] * PIX, PIX);
        randaugment(work, ra_mag, ra_n, &rng);
        int dy = 0, dx = 0;
        if (pad > 0) { /* crop_offset, data.rs:309-318 */
            dy = (int)orc_rng_below(&rng, (uint64_t)(2 * pad + 1)) - pad;
            dx = (int)orc_rng_below(&rng, (uint64_t)(2 * pad + 1)) - pad;
        }
        int flip = (int)((orc_rng_next_u64(&rng) >> 32) & 1u);
        float *dst = out + (size_t)b * PIX;
        crop_flip_normalize(work, dst, dy, dx, flip);
        random_erase(dst, erase, erase_side, &rng);
    }
}

void orc_make_batch_eval(const uint8_t *images, const uint8_t *labels, size_t start, int bs, int flip,
                         float *out, uint32_t *labels_out) {
    /* data.rs:494-512: no shift, so every source pixel is inside the image */
    for (int b = 0; b < bs; b++) labels_out[b] = labels[start + (size_t)b];
    for (int b = 0; b < bs; b++)
        crop_flip_normalize(images + (start + (size_t)b) * PIX, out + (size_t)b * PIX, 0, 0, flip);
}

/* data.rs:417-431 */
static float beta_like(float a, orc_rng *rng) {
    float u = orc_rng_uniform(rng);
    if (a >= 1.0f) return u;
    if (u < 0.5f) return powf(2.0f * u, 1.0f / a) * 0.5f;
    return 1.0f - powf(2.0f * (1.0f - u), 1.0f / a) * 0.5f;
}

int orc_mix_batch(float *x, int bs, float alpha_mix, float alpha_cut, float sw, uint64_t *state,
                  uint32_t *perm, float *lam, int *rect) {
    /* data.rs:467-491 with cutmix (:436-456) and mixup (:459-469) */
    orc_rng rng;
    memcpy(rng.s, state, sizeof(rng.s));
    for (int i = 0; i < bs; i++) perm[i] = (uint32_t)i;
    for (int i = bs - 1; i >= 1; i--) { /* Rng::shuffle, rng.rs:61-65 */
        uint32_t j = (uint32_t)orc_rng_below(&rng, (uint64_t)i + 1);
        uint32_t t = perm[i];
        perm[i] = perm[j];
        perm[j] = t;
    }
    for (int i = 0; i < bs; i++) lam[i] = 1.0f;
    int kind = 0; /* 0 none, 1 mixup, 2 cutmix */
    if (!(alpha_mix <= 0.0f && alpha_cut <= 0.0f)) {
        int cut = alpha_cut > 0.0f && (alpha_mix <= 0.0f || orc_rng_uniform(&rng) < sw);
        float l = beta_like(cut ? alpha_cut : alpha_mix, &rng);
        float *src = (float *)malloc(sizeof(float) * (size_t)bs * PIX);
        memcpy(src, x, sizeof(float) * (size_t)bs * PIX);
        if (cut) {
            kind = 2;
            float r = sqrtf(1.0f - l);
            int side = (int)((float)IMG * r);
            if (side > IMG) side = IMG;
            int cy = (int)orc_rng_below(&rng, IMG), cx = (int)orc_rng_below(&rng, IMG);
            int y0 = cy - side / 2 > 0 ? cy - side / 2 : 0, y1 = cy + side / 2 < IMG ? cy + side / 2 : IMG;
            int x0 = cx - side / 2 > 0 ? cx - side / 2 : 0, x1 = cx + side / 2 < IMG ? cx + side / 2 : IMG;
            float area = (float)((y1 - y0) * (x1 - x0)) / (float)(IMG * IMG);
            for (int b = 0; b < bs; b++) {
                for (int c = 0; c < CH; c++)
                    for (int y = y0; y < y1; y++)
                        for (int xx = x0; xx < x1; xx++) {
                            int o = c * PLANE + y * IMG + xx;
                            x[(size_t)b * PIX + o] = src[(size_t)perm[b] * PIX + o];
                        }
                lam[b] = 1.0f - area;
            }
            if (rect) {
                rect[0] = y0;
                rect[1] = y1;
                rect[2] = x0;
                rect[3] = x1;
            }
        } else {
            kind = 1;
            for (int b = 0; b < bs; b++) {
                size_t p = (size_t)perm[b] * PIX, o = (size_t)b * PIX;
                for (int i = 0; i < PIX; i++) x[o + i] = l * src[o + i] + (1.0f - l) * src[p + i];
                lam[b] = l;
            }
        }
        free(src);
    }
    memcpy(state, rng.s, sizeof(rng.s));
    return kind;
}
