/*
 * fixture.c -- seeded synthetic inputs (CPU). TEST INFRASTRUCTURE ONLY.
 * The algorithm is stated in fixture.h; the device copy lives in the
 * product library and must stay operation-for-operation identical.
 */
#include "fixture.h"
#include "ds4f_oracle.h"

#include <math.h>
#include <string.h>

#define FX_G UINT64_C(0x9E3779B97F4A7C15)

uint64_t fx_mix64(uint64_t x) {
    x += FX_G;
    x = (x ^ (x >> 30)) * UINT64_C(0xBF58476D1CE4E5B9);
    x = (x ^ (x >> 27)) * UINT64_C(0x94D049BB133111EB);
    return x ^ (x >> 31);
}

uint64_t fx_tid(uint32_t layer, uint32_t kind, uint32_t x, uint32_t t) {
    return ((uint64_t)layer << 40) | ((uint64_t)(kind & 0xFF) << 32) |
           ((uint64_t)(x & 0xFFFFFF) << 8) | (uint64_t)(t & 0xFF);
}

uint64_t fx_key(uint64_t seed, uint64_t tid) {
    return fx_mix64(fx_mix64(seed) ^ tid);
}

static double dbits(uint64_t b) { double d; memcpy(&d, &b, 8); return d; }
static uint64_t ubits(double d) { uint64_t b; memcpy(&b, &d, 8); return b; }

/* Natural log for s > 0 from + - * / only. */
double fx_ln(double s) {
    uint64_t b = ubits(s);
    int ex = (int)((b >> 52) & 0x7FF);
    int adj = 0;
    if (ex == 0) {                       /* subnormal: scale by 2^54 */
        s = s * 18014398509481984.0;
        b = ubits(s);
        ex = (int)((b >> 52) & 0x7FF);
        adj = 54;
    }
    int e = ex - 1023 - adj;
    double m = dbits((b & UINT64_C(0x000FFFFFFFFFFFFF)) |
                     UINT64_C(0x3FF0000000000000));
    if (m > 1.4142135623730951) { m = m * 0.5; e += 1; }
    double t = (m - 1.0) / (m + 1.0);
    double t2 = t * t;
    double p = 1.0 / 23.0;
    p = p * t2 + 1.0 / 21.0;
    p = p * t2 + 1.0 / 19.0;
    p = p * t2 + 1.0 / 17.0;
    p = p * t2 + 1.0 / 15.0;
    p = p * t2 + 1.0 / 13.0;
    p = p * t2 + 1.0 / 11.0;
    p = p * t2 + 1.0 / 9.0;
    p = p * t2 + 1.0 / 7.0;
    p = p * t2 + 1.0 / 5.0;
    p = p * t2 + 1.0 / 3.0;
    p = p * t2 + 1.0;
    double lt = (2.0 * t) * p;
    return (double)e * 0.6931471805599453 + lt;
}

double fx_gauss(uint64_t key, uint64_t i) {
    uint64_t base = fx_mix64(key + i);
    for (uint64_t k = 0; k < 64; k++) {
        uint64_t z1 = fx_mix64(base + (2 * k) * FX_G);
        uint64_t z2 = fx_mix64(base + (2 * k + 1) * FX_G);
        double v1 = (double)(z1 >> 11) * 2.220446049250313e-16 - 1.0;
        double v2 = (double)(z2 >> 11) * 2.220446049250313e-16 - 1.0;
        double s = v1 * v1 + v2 * v2;
        if (s > 0.0 && s < 1.0) {
            double f = sqrt((-2.0 * fx_ln(s)) / s);
            return v1 * f;
        }
    }
    return 0.0;
}

float fx_value(uint64_t key, uint64_t i, double sigma) {
    return (float)(fx_gauss(key, i) * sigma);
}

uint16_t fx_bf16_rne(float f) {
    uint32_t b;
    memcpy(&b, &f, 4);
    if ((b & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((b >> 16) | 0x40);
    b += 0x7FFFu + ((b >> 16) & 1u);
    return (uint16_t)(b >> 16);
}

/* Magnitude of canonical positive byte b (0..0x77 or 0x7E). */
static float f8_mag(int b) { return orc_f8_value((uint8_t)b); }

uint8_t fx_f8_encode(float v) {
    int neg = v < 0.0f;
    float a = fabsf(v);
    int byte;
    if (!(a < 448.0f)) {
        byte = 0x7E;
    } else {
        int lo = 0, hi = 0x77;           /* largest b with mag(b) <= a */
        while (lo < hi) {
            int mid = (lo + hi + 1) >> 1;
            if (f8_mag(mid) <= a) lo = mid; else hi = mid - 1;
        }
        int b0 = lo, b1 = (lo == 0x77) ? 0x7E : lo + 1;
        double d0 = (double)a - (double)f8_mag(b0);
        double d1 = (double)f8_mag(b1) - (double)a;
        if (d0 < d1) byte = b0;
        else if (d1 < d0) byte = b1;
        else byte = (b0 & 1) ? b1 : b0;
    }
    return (uint8_t)(byte | (neg ? 0x80 : 0));
}

int fx_ceil_log2(float y) {
    uint32_t b;
    memcpy(&b, &y, 4);
    int ex = (int)((b >> 23) & 0xFF), adj = 0;
    if (ex == 0) {
        y = y * 4294967296.0f;           /* 2^32, exact */
        memcpy(&b, &y, 4);
        ex = (int)((b >> 23) & 0xFF);
        adj = 32;
    }
    int e = ex - 127 - adj;
    return (b & 0x7FFFFFu) ? e + 1 : e;
}

static const float k_mags[8] = {0.0f, 0.5f, 1.0f, 1.5f,
                                2.0f, 3.0f, 4.0f, 6.0f};

int fx_e2m1_encode(float q) {
    float a = fabsf(q);
    int best = 0;
    float bd = a;
    for (int i = 1; i < 8; i++) {
        float d = fabsf(a - k_mags[i]);
        if (d < bd) { bd = d; best = i; }
    }
    return (q < 0.0f ? 8 : 0) | best;
}

void fx_fill_f32(float *dst, int64_t n, uint64_t key, double sigma) {
    for (int64_t i = 0; i < n; i++) dst[i] = fx_value(key, (uint64_t)i, sigma);
}

void fx_fill_bf16(uint16_t *dst, int64_t n, uint64_t key, double sigma) {
    for (int64_t i = 0; i < n; i++)
        dst[i] = fx_bf16_rne(fx_value(key, (uint64_t)i, sigma));
}

int fx_quant_fp8(int R, int C, uint64_t key, double sigma, uint8_t *vals,
                 float *scales) {
    if (R % 128 || C % 128) return -1;
    int SR = R / 128, SC = C / 128;
    static float blk[128 * 128];         /* not re-entrant: test helper */
    for (int br = 0; br < SR; br++)
        for (int bc = 0; bc < SC; bc++) {
            float amax = 0.0f;
            for (int r = 0; r < 128; r++)
                for (int c = 0; c < 128; c++) {
                    float w = fx_value(key, (uint64_t)(br * 128 + r) * C +
                                                (uint64_t)(bc * 128 + c),
                                       sigma);
                    blk[r * 128 + c] = w;
                    float a = fabsf(w);
                    if (a > amax) amax = a;
                }
            float s = amax > 0.0f ? amax / 448.0f : 1.0f;
            scales[br * SC + bc] = s;
            for (int r = 0; r < 128; r++)
                for (int c = 0; c < 128; c++)
                    vals[(int64_t)(br * 128 + r) * C + bc * 128 + c] =
                        fx_f8_encode(blk[r * 128 + c] / s);
        }
    return 0;
}

int fx_quant_mxfp4(int R, int C, uint64_t key, double sigma, uint8_t *vals,
                   uint8_t *scales) {
    if (C % 32) return -1;
    int64_t n = (int64_t)R * C;
    for (int64_t bi = 0; bi < n / 32; bi++) {
        float xs[32];
        float m = 0.0f;
        for (int j = 0; j < 32; j++) {
            xs[j] = fx_value(key, (uint64_t)(bi * 32 + j), sigma);
            float a = fabsf(xs[j]);
            if (a > m) m = a;
        }
        int k = m > 0.0f ? fx_ceil_log2(m / 6.0f) : -127;
        if (k < -127) k = -127;
        if (k > 127) k = 127;
        uint8_t sb = (uint8_t)((k + 127) & 0xFF);
        scales[bi] = sb;
        float s = orc_e8m0_value(sb);
        for (int j = 0; j < 32; j += 2) {
            int n0 = fx_e2m1_encode(s != 0.0f ? xs[j] / s : 0.0f);
            int n1 = fx_e2m1_encode(s != 0.0f ? xs[j + 1] / s : 0.0f);
            vals[(bi * 32 + j) / 2] = (uint8_t)(n0 | (n1 << 4));
        }
    }
    return 0;
}

int fx_expert(int fmt, int H, int M, uint64_t seed, uint32_t layer,
              uint32_t expert, double sigma, uint8_t *slot) {
    OrcExpertLayout lay;
    if (orc_expert_layout(fmt, H, M, &lay) != 0) return -1;
    for (int t = 0; t < 3; t++) {
        int R = t < 2 ? M : H, C = t < 2 ? H : M;
        uint64_t key = fx_key(seed, fx_tid(layer, FX_KIND_EXPERT, expert,
                                           (uint32_t)t));
        int rc = fmt == ORC_FMT_FP8
            ? fx_quant_fp8(R, C, key, sigma, slot + lay.rel_v[t],
                           (float *)(void *)(slot + lay.rel_s[t]))
            : fx_quant_mxfp4(R, C, key, sigma, slot + lay.rel_v[t],
                             slot + lay.rel_s[t]);
        if (rc != 0) return -1;
    }
    return 0;
}

void fx_trunk(int H, int M, int E, uint64_t seed, uint32_t layer,
              double sigma, uint16_t *norm, uint16_t *router,
              uint16_t *sh_gate, uint16_t *sh_up, uint16_t *sh_down,
              uint16_t *sh_gw) {
    for (int i = 0; i < H; i++) norm[i] = 0x3F80;      /* bf16 1.0 */
    fx_fill_bf16(router, (int64_t)E * H,
                 fx_key(seed, fx_tid(layer, FX_KIND_ROUTER, 0, 0)), sigma);
    fx_fill_bf16(sh_gate, (int64_t)M * H,
                 fx_key(seed, fx_tid(layer, FX_KIND_SHARED, 0, 0)), sigma);
    fx_fill_bf16(sh_up, (int64_t)M * H,
                 fx_key(seed, fx_tid(layer, FX_KIND_SHARED, 0, 1)), sigma);
    fx_fill_bf16(sh_down, (int64_t)H * M,
                 fx_key(seed, fx_tid(layer, FX_KIND_SHARED, 0, 2)), sigma);
    fx_fill_bf16(sh_gw, (int64_t)H,
                 fx_key(seed, fx_tid(layer, FX_KIND_SHARED, 0, 3)), sigma);
}
