/* RoPE table of the MTP attention, built exactly as the reference builds
   it (src/forward_rope.c:178-187, no scaling): freq_i = pow(theta,
   -2 i / rot), angle = l * freq_i, then {cos, sin} of the angle, each of
   the three with the reference's own all-float routines (src/lz_mathf.c:
   musl's powf and glibc's sinf/cosf with every intermediate in float).
   Those routines are not correctly rounded, so a table built from
   correctly rounded values differs from the reference's by an ulp at some
   positions, which changes draft logits and, at temperature, sampled
   drafts.  This header restates the published algorithms with the same
   constants and the same float operation order.

   Host code, C99 and C++: compile without floating-point contraction
   (-ffp-contract=off) so that every float multiply and add rounds
   separately, as in the reference's own build. */
#ifndef LZ98_ROPE_TABLE_H
#define LZ98_ROPE_TABLE_H

#include <stdint.h>
#include <string.h>

static inline uint32_t lzr_bits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}
static inline float lzr_float(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}
/* a float rounded through memory (the reference's evaluation barrier) */
static inline float lzr_round(float x) {
    volatile float y = x;
    return y;
}

/* ---- pow: log2 by a 16-interval table and a degree-5 polynomial, then
   2^(y log2 x) by a 32-entry table and a cubic (musl powf, float form). */

/* log2 table: per interval, 1/c and log2(c) (c near the interval's
   centre); polynomial for log1p(r)/ln2 */
static const float lzr_log2_invc[16] = {
    1.39890718460083f, 1.3403141498565674f, 1.2864322662353516f, 1.2367150783538818f,
    1.1906976699829102f, 1.147982120513916f, 1.1082251071929932f, 1.0711297988891602f,
    1.0364372730255127f, 1.0f, 0.9492859840393066f, 0.8951049447059631f,
    0.8476821780204773f, 0.8050314784049988f, 0.7664670944213867f, 0.7314286231994629f};
static const float lzr_log2_logc[16] = {
    -0.4843002259731293f, -0.42257124185562134f, -0.3633754253387451f, -0.30651310086250305f,
    -0.25180721282958984f, -0.19910015165805817f, -0.148251011967659f, -0.09913323819637299f,
    -0.05163281410932541f, 0.0f, 0.07508531957864761f, 0.15987126529216766f,
    0.23840466141700745f, 0.3128829002380371f, 0.38370421528816223f, 0.45121103525161743f};
static const float lzr_log2_poly[5] = {0.28845757246017456f, -0.3609260618686676f, 0.4808984696865082f,
                                       -0.721347451210022f, 1.4426950216293335f};
/* 2^(i/32) as float bit patterns; cubic for 2^r */
static const uint32_t lzr_exp2_tab[32] = {
    0x3f800000u, 0x3f82cd87u, 0x3f85aac3u, 0x3f88980fu, 0x3f8b95c2u, 0x3f8ea43au, 0x3f91c3d3u, 0x3f94f4f0u,
    0x3f9837f0u, 0x3f9b8d3au, 0x3f9ef532u, 0x3fa27043u, 0x3fa5fed7u, 0x3fa9a15bu, 0x3fad583fu, 0x3fb123f6u,
    0x3fb504f3u, 0x3fb8fbafu, 0x3fbd08a4u, 0x3fc12c4du, 0x3fc5672au, 0x3fc9b9beu, 0x3fce248cu, 0x3fd2a81eu,
    0x3fd744fdu, 0x3fdbfbb8u, 0x3fe0ccdfu, 0x3fe5b907u, 0x3feac0c7u, 0x3fefe4bau, 0x3ff5257du, 0x3ffa83b3u};
static const float lzr_exp2_poly[3] = {0.055503614246845245f, 0.24022845923900604f, 0.6931471824645996f};

/* log2 of the positive normal float with bits ix */
static inline float lzr_log2(uint32_t ix) {
    const uint32_t off = 0x3f330000u;
    const uint32_t tmp = ix - off;
    const int i = (int)((tmp >> 19) % 16u);
    const uint32_t top = tmp & 0xff800000u;
    const int k = (int32_t)top >> 23;
    const float z = lzr_float(ix - top);
    const float r = z * lzr_log2_invc[i] - 1.0f;
    const float yl0 = lzr_log2_logc[i] + (float)k;
    const float r2 = r * r;
    float y = lzr_log2_poly[0] * r + lzr_log2_poly[1];
    const float p = lzr_log2_poly[2] * r + lzr_log2_poly[3];
    const float r4 = r2 * r2;
    float q = lzr_log2_poly[4] * r + yl0;
    q = p * r2 + q;
    y = y * r4 + q;
    return y;
}

/* 2^xd, xd in (-150, 128] */
static inline float lzr_exp2(float xd) {
    const float x32 = xd * 32.0f;
    int k = (int)x32;
    const float frac = x32 - (float)k;
    if (frac > 0.5f || (frac == 0.5f && (k & 1)))
        k += 1;
    else if (frac < -0.5f || (frac == -0.5f && (k & 1)))
        k -= 1;
    const float r = xd - (float)k * 0.03125f;
    const uint32_t t = lzr_exp2_tab[k & 31];
    int kexp = k >> 5, twice = 0;
    float s;
    if (kexp > 127) {
        kexp = 127;
        twice = 1;
    }
    if (kexp >= -126) {
        s = lzr_float((t & 0x007fffffu) | ((uint32_t)(kexp + 127) << 23));
    } else {
        const int shift = kexp + 149;
        s = lzr_float(t) * lzr_float(shift > 0 ? 1u << shift : 1u);
    }
    const float r2 = r * r;
    float y = lzr_exp2_poly[0] * r + lzr_exp2_poly[1];
    float z = lzr_exp2_poly[2] * r + 1.0f;
    z = y * r2 + z;
    y = z * s;
    if (twice) y *= 2.0f;
    return y;
}

/* pow(x, y) for a positive finite base and a finite exponent (the only
   inputs the table takes: theta > 0, -2 i / rot); y = 0 or x = 1 give 1 */
static inline float lzr_powf(float x, float y) {
    uint32_t ix = lzr_bits(x);
    const uint32_t iy = lzr_bits(y);
    if ((iy << 1) == 0u || ix == 0x3f800000u) return 1.0f;
    if (ix < 0x00800000u) {          /* subnormal base: normalised, negative biased exponent */
        ix = lzr_bits(x * 8388608.0f) & 0x7fffffffu;
        ix -= 23u << 23;
    }
    const float ylogx = y * lzr_log2(ix);
    if (ylogx > 128.0f) return lzr_float(0x7f800000u);
    if (ylogx <= -150.0f) return 0.0f;
    return lzr_exp2(ylogx);
}

/* ---- sin / cos: reduction by pi/2 (one multiply-subtract below 120, a
   192-bit 4/pi table above), then the odd or even polynomial by quadrant
   (glibc sincosf, float form). */

typedef struct {
    float sign[4];                  /* sign of sine by quadrant */
    float hpi_inv, hpi;             /* 2/pi * 2^24, pi/2 */
    float c0, c1, c2, c3, c4;       /* cosine polynomial */
    float s1, s2, s3;               /* sine polynomial */
} LzrSinCos;

static const LzrSinCos lzr_sincos[2] = {
    {{1.0f, -1.0f, -1.0f, 1.0f}, 10680707.0f, 1.5707963705062866f, 1.0f, -0.5f, 0.04166662320494652f,
     -0.0013886763481423259f, 2.4390450562350452e-05f, -0.16666655242443085f, 0.008332177996635437f,
     -0.0001951729936990887f},
    {{1.0f, -1.0f, -1.0f, 1.0f}, 10680707.0f, 1.5707963705062866f, -1.0f, 0.5f, -0.04166662320494652f,
     0.0013886763481423259f, -2.4390450562350452e-05f, -0.16666655242443085f, 0.008332177996635437f,
     -0.0001951729936990887f}};

/* 4/pi to 192 bits, as overlapping 32-bit windows */
static const uint32_t lzr_inv_pio4[24] = {
    0xa2u,       0xa2f9u,     0xa2f983u,   0xa2f9836eu, 0xf9836e4eu, 0x836e4e44u, 0x6e4e4415u, 0x4e441529u,
    0x441529fcu, 0x1529fc27u, 0x29fc2757u, 0xfc2757d1u, 0x2757d1f5u, 0x57d1f534u, 0xd1f534ddu, 0xf534ddc0u,
    0x34ddc0dbu, 0xddc0db62u, 0xc0db6295u, 0xdb629599u, 0x6295993cu, 0x95993c43u, 0x993c4390u, 0x3c439041u};

static inline uint32_t lzr_top12(float x) { return (lzr_bits(x) >> 20) & 0x7ffu; }

static inline float lzr_reduce_fast(float x, const LzrSinCos* p, int* np) {
    const float r = x * p->hpi_inv;
    const int n = ((int32_t)r + 0x800000) >> 24;
    *np = n;
    return x - (float)n * p->hpi;
}

static inline float lzr_reduce_large(uint32_t xi, int* np) {
    const uint32_t* arr = &lzr_inv_pio4[(xi >> 26) & 15u];
    const int shift = (int)((xi >> 23) & 7u);
    xi = (xi & 0xffffffu) | 0x800000u;
    xi <<= shift;
    uint64_t r0 = (uint64_t)(uint32_t)(xi * arr[0]);   /* a 32-bit product */
    const uint64_t r1 = (uint64_t)xi * arr[4];
    const uint64_t r2 = (uint64_t)xi * arr[8];
    r0 = (r2 >> 32) | (r0 << 32);
    r0 += r1;
    const uint64_t n = (r0 + ((uint64_t)1 << 61)) >> 62;
    r0 -= n << 62;
    const float x = lzr_round((float)(int64_t)r0);      /* the integer rounds to float first */
    *np = (int)n;
    return x * 3.4061216748705226e-19f;                 /* pi / 2^63 */
}

static inline float lzr_sincos_poly(float x, float x2, const LzrSinCos* p, int n) {
    if ((n & 1) == 0) {
        const float x3 = x * x2;
        const float s1 = p->s2 + x2 * p->s3;
        const float x7 = x3 * x2;
        const float s = x + x3 * p->s1;
        return s + x7 * s1;
    }
    const float x4 = x2 * x2;
    const float c2 = p->c3 + x2 * p->c4;
    const float c1 = p->c0 + x2 * p->c1;
    const float x6 = x4 * x2;
    const float c = c1 + x4 * p->c2;
    return c + x6 * c2;
}

/* cosine (cos = 1) or sine (cos = 0) of y */
static inline float lzr_sincosf(float y, int cos) {
    const LzrSinCos* p = &lzr_sincos[0];
    const float pio4 = 0.7853981852531433f;
    int n;
    if (lzr_top12(y) < lzr_top12(pio4)) {
        const float x2 = y * y;
        if (lzr_top12(y) < lzr_top12(0.000244140625f)) return cos ? 1.0f : y;
        return lzr_sincos_poly(y, x2, p, cos);
    }
    if (lzr_top12(y) < lzr_top12(120.0f)) {
        const float x = lzr_reduce_fast(y, p, &n);
        const float s = p->sign[n & 3];
        if (n & 2) p = &lzr_sincos[1];
        return lzr_sincos_poly(x * s, x * x, p, cos ? n ^ 1 : n);
    }
    if (lzr_top12(y) < lzr_top12(lzr_float(0x7f800000u))) {
        const uint32_t xi = lzr_bits(y);
        const int sign = (int)(xi >> 31);
        const float x = lzr_reduce_large(xi, &n);
        const float s = p->sign[(n + sign) & 3];
        if ((n + sign) & 2) p = &lzr_sincos[1];
        return lzr_sincos_poly(x * s, x * x, p, cos ? n ^ 1 : n);
    }
    return y - y;   /* inf or nan */
}

/* The table: for l in [0, seq_len), i in [0, rot/2): out[(l half + i) 2]
   = cos(l freq_i), out[... + 1] = sin(l freq_i). */
static inline void lz98_rope_table(float theta, int rot, int seq_len, float* out) {
    const int half = rot / 2;
    for (int i = 0; i < half; i++) {
        const float freq = lzr_powf(theta, -2.0f * (float)i / (float)rot);
        for (int l = 0; l < seq_len; l++) {
            const float ang = (float)l * freq;
            out[((size_t)l * half + i) * 2] = lzr_sincosf(ang, 1);
            out[((size_t)l * half + i) * 2 + 1] = lzr_sincosf(ang, 0);
        }
    }
}

#endif
