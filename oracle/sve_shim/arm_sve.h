/* arm_sve.h (shim) -- TEST INFRASTRUCTURE ONLY.
 *
 * A portable scalar implementation of exactly the Arm SVE ACLE intrinsics that the
 * reference's flash.c uses, so that flash.c compiles unmodified on x86 (gcc) for the oracle
 * build in oracle/Makefile. Written from the ACLE / Arm ARM instruction descriptions:
 *   - vectors are fixed-length structs of SVE_SHIM_VL bits (default 512, the vector length
 *     of the reference's own recorded QEMU runs, flash_long.log:10);
 *   - predicates keep one flag per byte, as SVE does, so a b32 predicate governs 32-bit
 *     lanes and a b16 predicate 16-bit lanes;
 *   - BFDOT (svbfdot_f32) adds the two exact bf16 products of each lane pair in fp32 and then
 *     the accumulator (the architectural BFDOT uses a round-to-odd intermediate; the
 *     difference is at fp32 rounding level);
 *   - FEXPA (svexpa_f32) follows the Arm ARM: bits [5:0] index a table holding the fraction
 *     of 2^(i/64), bits [13:6] become the exponent field;
 *   - FADDV is a pairwise tree reduction, BFCVT rounds to nearest even.
 * Nothing in the product includes this header.
 */
#ifndef TS_SVE_SHIM_ARM_SVE_H
#define TS_SVE_SHIM_ARM_SVE_H

#include <math.h>
#include <stdint.h>
#include <string.h>

#ifndef SVE_SHIM_VL
#define SVE_SHIM_VL 512
#endif
#define SVE_NB (SVE_SHIM_VL / 8)
#define SVE_NW (SVE_SHIM_VL / 32)
#define SVE_NH (SVE_SHIM_VL / 16)

typedef uint16_t bfloat16_t;
typedef struct { uint8_t b[SVE_NB]; } svbool_t;
typedef struct { float v[SVE_NW]; } svfloat32_t;
typedef struct { uint32_t v[SVE_NW]; } svuint32_t;
typedef struct { int32_t v[SVE_NW]; } svint32_t;
typedef struct { uint16_t v[SVE_NH]; } svbfloat16_t;
typedef struct { uint16_t v[SVE_NH]; } svuint16_t;

#define SVE_INL static inline __attribute__((always_inline, unused))
#define PW(pg, i) ((pg).b[4 * (i)] != 0) /* 32-bit lane i active */
#define PH(pg, i) ((pg).b[2 * (i)] != 0) /* 16-bit lane i active */

SVE_INL uint64_t svcntw(void) { return SVE_NW; }
SVE_INL uint64_t svcnth(void) { return SVE_NH; }

SVE_INL svbool_t svptrue_b32(void) {
    svbool_t p;
    memset(&p, 0, sizeof p);
    for (int i = 0; i < SVE_NW; i++) p.b[4 * i] = 1;
    return p;
}
SVE_INL svbool_t svpfalse_b(void) {
    svbool_t p;
    memset(&p, 0, sizeof p);
    return p;
}
SVE_INL svbool_t svwhilelt_b32_s32(int32_t a, int32_t n) {
    svbool_t p;
    memset(&p, 0, sizeof p);
    for (int i = 0; i < SVE_NW; i++) p.b[4 * i] = ((int64_t)a + i < (int64_t)n);
    return p;
}
SVE_INL svbool_t svwhilelt_b16_s32(int32_t a, int32_t n) {
    svbool_t p;
    memset(&p, 0, sizeof p);
    for (int i = 0; i < SVE_NH; i++) p.b[2 * i] = ((int64_t)a + i < (int64_t)n);
    return p;
}
SVE_INL int svptest_any(svbool_t pg, svbool_t p) {
    for (int i = 0; i < SVE_NB; i++)
        if (pg.b[i] && p.b[i]) return 1;
    return 0;
}

SVE_INL svfloat32_t svdup_n_f32(float x) {
    svfloat32_t r;
    for (int i = 0; i < SVE_NW; i++) r.v[i] = x;
    return r;
}
SVE_INL svuint32_t svdup_n_u32(uint32_t x) {
    svuint32_t r;
    for (int i = 0; i < SVE_NW; i++) r.v[i] = x;
    return r;
}
SVE_INL svuint16_t svdup_n_u16(uint16_t x) {
    svuint16_t r;
    for (int i = 0; i < SVE_NH; i++) r.v[i] = x;
    return r;
}
SVE_INL svint32_t svindex_s32(int32_t base, int32_t step) {
    svint32_t r;
    for (int i = 0; i < SVE_NW; i++) r.v[i] = base + i * step;
    return r;
}

SVE_INL svfloat32_t svreinterpret_f32_u32(svuint32_t a) {
    svfloat32_t r;
    memcpy(&r, &a, sizeof r);
    return r;
}
SVE_INL svuint32_t svreinterpret_u32_f32(svfloat32_t a) {
    svuint32_t r;
    memcpy(&r, &a, sizeof r);
    return r;
}
SVE_INL svuint16_t svreinterpret_u16_bf16(svbfloat16_t a) {
    svuint16_t r;
    memcpy(&r, &a, sizeof r);
    return r;
}

/* _x forms: inactive lanes are "don't care"; computing every lane is a valid choice. */
SVE_INL svfloat32_t svadd_f32_x(svbool_t pg, svfloat32_t a, svfloat32_t b) {
    (void)pg;
    for (int i = 0; i < SVE_NW; i++) a.v[i] = a.v[i] + b.v[i];
    return a;
}
SVE_INL svfloat32_t svsub_f32_x(svbool_t pg, svfloat32_t a, svfloat32_t b) {
    (void)pg;
    for (int i = 0; i < SVE_NW; i++) a.v[i] = a.v[i] - b.v[i];
    return a;
}
SVE_INL svfloat32_t svmul_f32_x(svbool_t pg, svfloat32_t a, svfloat32_t b) {
    (void)pg;
    for (int i = 0; i < SVE_NW; i++) a.v[i] = a.v[i] * b.v[i];
    return a;
}
SVE_INL svfloat32_t svneg_f32_x(svbool_t pg, svfloat32_t a) {
    (void)pg;
    for (int i = 0; i < SVE_NW; i++) a.v[i] = -a.v[i];
    return a;
}
/* FMLA: a + b*c, fused. */
SVE_INL svfloat32_t svmla_f32_x(svbool_t pg, svfloat32_t a, svfloat32_t b, svfloat32_t c) {
    (void)pg;
    for (int i = 0; i < SVE_NW; i++) a.v[i] = fmaf(b.v[i], c.v[i], a.v[i]);
    return a;
}
/* FMAD: a*b + c, fused. */
SVE_INL svfloat32_t svmad_f32_x(svbool_t pg, svfloat32_t a, svfloat32_t b, svfloat32_t c) {
    (void)pg;
    for (int i = 0; i < SVE_NW; i++) a.v[i] = fmaf(a.v[i], b.v[i], c.v[i]);
    return a;
}
SVE_INL svfloat32_t svmax_f32_m(svbool_t pg, svfloat32_t a, svfloat32_t b) {
    for (int i = 0; i < SVE_NW; i++)
        if (PW(pg, i)) a.v[i] = (b.v[i] > a.v[i]) ? b.v[i] : a.v[i];
    return a;
}
SVE_INL svfloat32_t svsel_f32(svbool_t p, svfloat32_t a, svfloat32_t b) {
    for (int i = 0; i < SVE_NW; i++)
        if (!PW(p, i)) a.v[i] = b.v[i];
    return a;
}
SVE_INL svbool_t svacge_f32(svbool_t pg, svfloat32_t a, svfloat32_t b) {
    svbool_t p = svpfalse_b();
    for (int i = 0; i < SVE_NW; i++) p.b[4 * i] = PW(pg, i) && (fabsf(a.v[i]) >= fabsf(b.v[i]));
    return p;
}
SVE_INL svbool_t svcmpgt_f32(svbool_t pg, svfloat32_t a, svfloat32_t b) {
    svbool_t p = svpfalse_b();
    for (int i = 0; i < SVE_NW; i++) p.b[4 * i] = PW(pg, i) && (a.v[i] > b.v[i]);
    return p;
}
SVE_INL svbool_t svcmplt_f32(svbool_t pg, svfloat32_t a, svfloat32_t b) {
    svbool_t p = svpfalse_b();
    for (int i = 0; i < SVE_NW; i++) p.b[4 * i] = PW(pg, i) && (a.v[i] < b.v[i]);
    return p;
}

/* Pairwise tree over the active lanes (inactive lanes contribute +0). */
SVE_INL float svaddv_f32(svbool_t pg, svfloat32_t a) {
    float t[SVE_NW];
    for (int i = 0; i < SVE_NW; i++) t[i] = PW(pg, i) ? a.v[i] : 0.0f;
    for (int w = SVE_NW / 2; w > 0; w /= 2)
        for (int i = 0; i < w; i++) t[i] = t[i] + t[i + w];
    return t[0];
}
SVE_INL float svmaxv_f32(svbool_t pg, svfloat32_t a) {
    float m = -INFINITY;
    for (int i = 0; i < SVE_NW; i++)
        if (PW(pg, i) && a.v[i] > m) m = a.v[i];
    return m;
}
/* LASTA: the element after the last active one; element 0 when none is active. */
SVE_INL float svlasta_f32(svbool_t pg, svfloat32_t a) {
    int last = -1;
    for (int i = 0; i < SVE_NW; i++)
        if (PW(pg, i)) last = i;
    return a.v[(last + 1) % SVE_NW];
}

/* FEXPA: result = (bits[13:6] << 23) | frac(2^(bits[5:0]/64)). */
SVE_INL svfloat32_t svexpa_f32(svuint32_t a) {
    static uint32_t table[64];
    static int init = 0;
    if (!init) {
        for (int i = 0; i < 64; i++) table[i] = (uint32_t)llround((exp2((double)i / 64.0) - 1.0) * 8388608.0);
        init = 1;
    }
    svfloat32_t r;
    for (int i = 0; i < SVE_NW; i++) {
        const uint32_t x = a.v[i];
        const uint32_t bits = (((x >> 6) & 0xffu) << 23) | table[x & 63u];
        memcpy(&r.v[i], &bits, 4);
    }
    return r;
}

SVE_INL svbfloat16_t svld1_bf16(svbool_t pg, const bfloat16_t *p) {
    svbfloat16_t r;
    for (int i = 0; i < SVE_NH; i++) r.v[i] = PH(pg, i) ? p[i] : 0;
    return r;
}
SVE_INL svfloat32_t svld1_f32(svbool_t pg, const float *p) {
    svfloat32_t r;
    for (int i = 0; i < SVE_NW; i++) r.v[i] = PW(pg, i) ? p[i] : 0.0f;
    return r;
}
SVE_INL void svst1_f32(svbool_t pg, float *p, svfloat32_t a) {
    for (int i = 0; i < SVE_NW; i++)
        if (PW(pg, i)) p[i] = a.v[i];
}
SVE_INL void svst1_u16(svbool_t pg, uint16_t *p, svuint16_t a) {
    for (int i = 0; i < SVE_NH; i++)
        if (PH(pg, i)) p[i] = a.v[i];
}
SVE_INL svuint32_t svld1uh_gather_s32index_u32(svbool_t pg, const uint16_t *base, svint32_t idx) {
    svuint32_t r;
    for (int i = 0; i < SVE_NW; i++) r.v[i] = PW(pg, i) ? (uint32_t)base[idx.v[i]] : 0u;
    return r;
}
SVE_INL void svst1h_u32(svbool_t pg, uint16_t *p, svuint32_t a) {
    for (int i = 0; i < SVE_NW; i++)
        if (PW(pg, i)) p[i] = (uint16_t)a.v[i];
}

SVE_INL float sve_shim_bf16_to_f32(uint16_t h) {
    uint32_t x = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &x, 4);
    return f;
}
SVE_INL uint16_t sve_shim_f32_to_bf16_rne(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    if (((x >> 23) & 0xffu) == 0xffu) return (uint16_t)((x >> 16) | ((x & 0x7fffffu) ? 0x40u : 0u));
    x += 0x7fffu + ((x >> 16) & 1u);
    return (uint16_t)(x >> 16);
}

/* BFDOT: acc[i] += a[2i]*b[2i] + a[2i+1]*b[2i+1] (products exact in fp32). */
SVE_INL svfloat32_t svbfdot_f32(svfloat32_t acc, svbfloat16_t a, svbfloat16_t b) {
    for (int i = 0; i < SVE_NW; i++) {
        const float p0 = sve_shim_bf16_to_f32(a.v[2 * i]) * sve_shim_bf16_to_f32(b.v[2 * i]);
        const float p1 = sve_shim_bf16_to_f32(a.v[2 * i + 1]) * sve_shim_bf16_to_f32(b.v[2 * i + 1]);
        acc.v[i] = acc.v[i] + (p0 + p1);
    }
    return acc;
}
/* BFCVT: each 32-bit lane -> bf16 in the even (low) half of its container, odd half 0. */
SVE_INL svbfloat16_t svcvt_bf16_f32_x(svbool_t pg, svfloat32_t a) {
    (void)pg;
    svbfloat16_t r;
    for (int i = 0; i < SVE_NW; i++) {
        r.v[2 * i] = sve_shim_f32_to_bf16_rne(a.v[i]);
        r.v[2 * i + 1] = 0;
    }
    return r;
}
/* UZP1: even-numbered elements of a, then of b. */
SVE_INL svbfloat16_t svuzp1_bf16(svbfloat16_t a, svbfloat16_t b) {
    svbfloat16_t r;
    for (int i = 0; i < SVE_NH / 2; i++) {
        r.v[i] = a.v[2 * i];
        r.v[SVE_NH / 2 + i] = b.v[2 * i];
    }
    return r;
}

#endif /* TS_SVE_SHIM_ARM_SVE_H */
