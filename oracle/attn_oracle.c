/* attn_oracle.c -- TEST INFRASTRUCTURE ONLY: the CPU oracle for the B200 attention path.
 *
 * A plain-C restatement of the reference algorithm in flash.c (liujiang833/transfer_station)
 * that the parity tests, __graft_entry__.smoke() and bench.py's CPU-baseline leg use as the
 * checker. Nothing in the product (transfer_station_b200/) links or calls this file.
 *
 * Parity status: PINNED. tests/golden/ holds vectors produced by the reference's own
 * flash.c (compiled natively through oracle/sve_shim, see oracle/Makefile and
 * tests/golden/make_golden.py); tests/test_oracle.py checks this restatement against them
 * (attn_ref bit-exact, the blocked kernel within the reference's own tolerance).
 *
 * Contents, each citing the reference lines it restates:
 *   orc_f32_to_bf16 / orc_bf16_to_f32   flash.c:78-92   (RNE, NaN/Inf passthrough)
 *   orc_fill_lcg                        flash.c:867-871, 1030, 1055-1060 (LCG, order Q,K,V)
 *   orc_fill_normal / orc_fill_uniform  seeded splitmix64 + Box-Muller / uniform generators for
 *                                       the benchmark configs (not in the reference)
 *   orc_attn_ref                        flash.c:262-314 (scalar fp32 exact-softmax oracle)
 *   orc_attn_blocked                    flash.c:727-864 with 344-580 (the blocked online-softmax
 *                                       kernel: BQ x bk tiles, causal block break, masked-block
 *                                       rule, alpha = 0 on a row's first block, P rounded to bf16
 *                                       while l sums the unrounded exponentials, zero row when
 *                                       l == 0). exp is libm expf where flash.c uses its SVE
 *                                       fast_exp (flash.c:216-246, rel. err ~2e-6): the two differ
 *                                       far below the bf16 rounding of P.
 *   orc_pack_v_full                     flash.c:714-718 (V -> V^T [Hkv][D][Sk])
 *   orc_ref_rowset                      flash.c:900-913 (spread rows incl. Sq-1)
 *   orc_cmp_rows                        flash.c:958-980 (mad <= TOL*maxref, NaN counted
 *                                       out of band) + the abs / rel-L2 bounds of the task
 *   orc_attn_pairs                      flash.c:874-887
 *   orc_ref_scratch_bytes               flash.c:658-682 (the reference's scratch size)
 *   orc_pick_bk_model                   README.md:359-436 (analytical bk model, any BQ)
 *   orc_combine                         merge of (m, l, acc) partials in base-2 units
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

uint16_t orc_f32_to_bf16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    if (((x >> 23) & 0xffu) == 0xffu) return (uint16_t)(x >> 16);
    x += 0x7fffu + ((x >> 16) & 1u);
    return (uint16_t)(x >> 16);
}

float orc_bf16_to_f32(uint16_t h) {
    uint32_t x = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &x, 4);
    return f;
}

void orc_f32_to_bf16_array(const float *in, uint16_t *out, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = orc_f32_to_bf16(in[i]);
}

void orc_bf16_to_f32_array(const uint16_t *in, float *out, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = orc_bf16_to_f32(in[i]);
}

/* flash.c:867-871: rng = rng*1664525 + 1013904223; frand = ((rng>>8)&0xffff)/32768 - 1.
 * The state runs straight through Q, then K, then V (flash.c:1055-1060). */
static float lcg_frand(uint32_t *rng) {
    *rng = *rng * 1664525u + 1013904223u;
    return ((*rng >> 8) & 0xffffu) / 32768.0f - 1.0f;
}

void orc_fill_lcg(uint16_t *Q, size_t nq, uint16_t *K, size_t nk, uint16_t *V, size_t nv, uint32_t seed) {
    uint32_t rng = seed;
    for (size_t i = 0; i < nq; i++) Q[i] = orc_f32_to_bf16(lcg_frand(&rng));
    for (size_t i = 0; i < nk; i++) K[i] = orc_f32_to_bf16(lcg_frand(&rng));
    for (size_t i = 0; i < nv; i++) V[i] = orc_f32_to_bf16(lcg_frand(&rng));
}

/* splitmix64 (Steele, Lea, Flood 2014) -> uniform doubles in (0, 1). */
static uint64_t splitmix64(uint64_t *s) {
    uint64_t z = (*s += 0x9e3779b97f4a7c15ull); /* ORC_SM64_GAMMA */
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

static double u01(uint64_t *s) { return ((double)(splitmix64(s) >> 11) + 0.5) * (1.0 / 9007199254740992.0); }

/* N(mean, sigma) by Box-Muller, two values per pair of uniforms, RNE to bf16. splitmix64's
 * state advances by a constant per draw, so pair p (draws 2p, 2p+1) starts from
 * state + 2p * gamma: the pairs are filled in parallel with the same values as one
 * sequential pass, and the state ends where that pass would leave it. */
#define ORC_SM64_GAMMA 0x9e3779b97f4a7c15ull
void orc_fill_normal(uint16_t *out, size_t n, uint64_t *state, float mean, float sigma) {
    const double two_pi = 6.283185307179586476925286766559;
    const uint64_t s0 = *state;
    const long long npairs = (long long)((n + 1) / 2);
#pragma omp parallel for schedule(static)
    for (long long pi = 0; pi < npairs; pi++) {
        uint64_t st = s0 + (uint64_t)(2 * pi) * ORC_SM64_GAMMA;
        const double u1 = u01(&st), u2 = u01(&st);
        const double r = sqrt(-2.0 * log(u1));
        const size_t i = 2 * (size_t)pi;
        out[i] = orc_f32_to_bf16((float)(mean + sigma * r * cos(two_pi * u2)));
        if (i + 1 < n) out[i + 1] = orc_f32_to_bf16((float)(mean + sigma * r * sin(two_pi * u2)));
    }
    *state = s0 + (uint64_t)(2 * npairs) * ORC_SM64_GAMMA;
}

/* One draw per element; parallel by the same state arithmetic. */
void orc_fill_uniform(uint16_t *out, size_t n, uint64_t *state, float lo, float hi) {
    const uint64_t s0 = *state;
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; i++) {
        uint64_t st = s0 + (uint64_t)i * ORC_SM64_GAMMA;
        out[i] = orc_f32_to_bf16((float)(lo + (hi - lo) * u01(&st)));
    }
    *state = s0 + (uint64_t)n * ORC_SM64_GAMMA;
}

/* flash.c:262-314. Row order and float arithmetic order follow the reference exactly, so
 * results match it bit for bit; rows are independent, so OpenMP over (h, row) keeps that. */
void orc_attn_ref(const uint16_t *Q, const uint16_t *K, const uint16_t *V, float *O, int Hq, int Hkv, int Sq,
                  int Sk, int D, int causal, const int *rows, int nrows) {
    const int group = Hq / Hkv;
    const float scale = 1.0f / sqrtf((float)D);
#pragma omp parallel
    {
        float *s = (float *)malloc(sizeof(float) * (size_t)Sk);
#pragma omp for collapse(2) schedule(dynamic, 1)
        for (int h = 0; h < Hq; h++)
            for (int t = 0; t < nrows; t++) {
                const int kv = h / group;
                const uint16_t *Qh = Q + (size_t)h * Sq * D, *Kh = K + (size_t)kv * Sk * D,
                               *Vh = V + (size_t)kv * Sk * D;
                const int i = rows[t];
                const int lim = causal ? (Sk - Sq + i) : (Sk - 1);
                float mx = -INFINITY;
                for (int j = 0; j < Sk; j++) {
                    if (j > lim) {
                        s[j] = -INFINITY;
                        continue;
                    }
                    float a = 0;
                    for (int d = 0; d < D; d++)
                        a += orc_bf16_to_f32(Qh[(size_t)i * D + d]) * orc_bf16_to_f32(Kh[(size_t)j * D + d]);
                    a *= scale;
                    s[j] = a;
                    if (a > mx) mx = a;
                }
                float sum = 0;
                for (int j = 0; j < Sk; j++) {
                    if (s[j] == -INFINITY)
                        s[j] = 0;
                    else {
                        s[j] = expf(s[j] - mx);
                        sum += s[j];
                    }
                }
                const float inv = (sum > 0) ? 1.0f / sum : 0.0f;
                for (int j = 0; j < Sk; j++) s[j] *= inv;
                for (int d = 0; d < D; d++) {
                    float a = 0;
                    for (int j = 0; j < Sk; j++) a += s[j] * orc_bf16_to_f32(Vh[(size_t)j * D + d]);
                    O[((size_t)h * Sq + i) * D + d] = a;
                }
            }
        free(s);
    }
}

/* flash.c:714-718 / 327-342: Vp[kv][d][k] = V[kv][k][d]. */
void orc_pack_v_full(const uint16_t *V, uint16_t *Vp, int Hkv, int Sk, int D) {
    for (int kv = 0; kv < Hkv; kv++)
        for (int k = 0; k < Sk; k++)
            for (int d = 0; d < D; d++)
                Vp[((size_t)kv * D + d) * Sk + k] = V[((size_t)kv * Sk + k) * D + d];
}

/* The blocked online-softmax kernel of flash.c:727-864. One (head, query block) per task.
 * Q/K/V are bf16 bit patterns; V is V^T [Hkv][D][Sk] when v_prepacked. bq is the query
 * block (flash.c's compile-time BQ), bk the key block. Only rows [row_lo, row_hi) of each
 * head are computed (others untouched), so a caller can time a bounded sample. */
void orc_attn_blocked_rows(const uint16_t *Q, const uint16_t *K, const uint16_t *V, float *O, int Hq, int Hkv,
                           int Sq, int Sk, int D, int causal, int bk, int bq, int v_prepacked, int row_lo,
                           int row_hi, int nthreads) {
    const int group = Hq / Hkv;
    const float scale = 1.0f / sqrtf((float)D);
    const int off = Sk - Sq;
    if (row_lo < 0) row_lo = 0;
    if (row_hi > Sq) row_hi = Sq;
    const int qb_lo = row_lo / bq, qb_hi = (row_hi + bq - 1) / bq;
    const int nqb = qb_hi - qb_lo;
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#else
    (void)nthreads;
#endif
#pragma omp parallel
    {
        float *S = (float *)malloc(sizeof(float) * (size_t)bq * bk);
        uint16_t *Pb = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)bq * bk);
        float *acc = (float *)malloc(sizeof(float) * (size_t)bq * D);
        float *pv = (float *)malloc(sizeof(float) * (size_t)D);
        float *qf = (float *)malloc(sizeof(float) * (size_t)bq * D);
        float *kf = (float *)malloc(sizeof(float) * (size_t)bk * D);
        float *vt = (float *)malloc(sizeof(float) * (size_t)D * bk); /* V^T block as fp32 */
        float m[4096], l[4096], al[4096];
#pragma omp for collapse(2) schedule(dynamic, 1)
        for (int h = 0; h < Hq; h++)
            for (int qq = 0; qq < nqb; qq++) {
                const int qi = (qb_lo + qq) * bq;
                const int kv = h / group;
                const uint16_t *Qh = Q + (size_t)h * Sq * D, *Kh = K + (size_t)kv * Sk * D,
                               *Vh = V + (size_t)kv * Sk * D;
                int rq = Sq - qi;
                if (rq > bq) rq = bq;
                for (int i = 0; i < rq; i++) {
                    m[i] = -INFINITY;
                    l[i] = 0;
                    for (int d = 0; d < D; d++) qf[(size_t)i * D + d] = orc_bf16_to_f32(Qh[(size_t)(qi + i) * D + d]);
                }
                memset(acc, 0, sizeof(float) * (size_t)rq * D);
                for (int kj = 0; kj < Sk; kj += bk) {
                    if (causal && kj > off + qi + rq - 1) break; /* flash.c:799-800 */
                    int rk = Sk - kj;
                    if (rk > bk) rk = bk;
                    for (int j = 0; j < rk; j++)
                        for (int d = 0; d < D; d++)
                            kf[(size_t)j * D + d] = orc_bf16_to_f32(Kh[(size_t)(kj + j) * D + d]);
                    for (int d = 0; d < D; d++)
                        for (int j = 0; j < rk; j++)
                            vt[(size_t)d * bk + j] = v_prepacked ? orc_bf16_to_f32(Vh[(size_t)d * Sk + kj + j])
                                                                 : orc_bf16_to_f32(Vh[(size_t)(kj + j) * D + d]);
                    /* qk_tile, flash.c:352-423 */
                    for (int i = 0; i < rq; i++)
                        for (int j = 0; j < rk; j++) {
                            float a = 0;
                            const float *qr = qf + (size_t)i * D, *kr = kf + (size_t)j * D;
                            for (int d = 0; d < D; d++) a += qr[d] * kr[d];
                            S[(size_t)i * bk + j] = a * scale;
                        }
                    /* softmax_block, flash.c:518-580 */
                    for (int i = 0; i < rq; i++) {
                        int jmax = rk;
                        if (causal) {
                            const int lim = off + qi + i - kj;
                            jmax = (lim + 1 < rk) ? lim + 1 : rk;
                            if (jmax < 0) jmax = 0;
                        }
                        float mij = -INFINITY;
                        for (int j = 0; j < jmax; j++)
                            if (S[(size_t)i * bk + j] > mij) mij = S[(size_t)i * bk + j];
                        if (mij == -INFINITY) {
                            for (int j = 0; j < rk; j++) Pb[(size_t)i * bk + j] = 0;
                            al[i] = 1.f;
                            continue;
                        }
                        const float mnew = (m[i] > mij) ? m[i] : mij;
                        const float alpha = (m[i] == -INFINITY) ? 0.f : expf(m[i] - mnew);
                        float sum = 0;
                        for (int j = 0; j < rk; j++) {
                            const float e = (j < jmax) ? expf(S[(size_t)i * bk + j] - mnew) : 0.f;
                            sum += e;
                            Pb[(size_t)i * bk + j] = orc_f32_to_bf16(e);
                        }
                        l[i] = alpha * l[i] + sum;
                        m[i] = mnew;
                        al[i] = alpha;
                    }
                    /* pv_acc, flash.c:433-510: acc = al*acc + sum_k P*V (one FMA) */
                    for (int i = 0; i < rq; i++) {
                        for (int d = 0; d < D; d++) {
                            float a = 0;
                            const float *vr = vt + (size_t)d * bk;
                            for (int k = 0; k < rk; k++) a += orc_bf16_to_f32(Pb[(size_t)i * bk + k]) * vr[k];
                            pv[d] = a;
                        }
                        float *ar = acc + (size_t)i * D;
                        for (int d = 0; d < D; d++) ar[d] = fmaf(ar[d], al[i], pv[d]);
                    }
                }
                for (int i = 0; i < rq; i++) { /* flash.c:851-860 */
                    if (qi + i < row_lo || qi + i >= row_hi) continue;
                    const float inv = (l[i] > 0) ? 1.f / l[i] : 0.f;
                    for (int d = 0; d < D; d++) O[((size_t)h * Sq + qi + i) * D + d] = acc[(size_t)i * D + d] * inv;
                }
            }
        free(S);
        free(Pb);
        free(acc);
        free(pv);
        free(qf);
        free(kf);
        free(vt);
    }
}

void orc_attn_blocked(const uint16_t *Q, const uint16_t *K, const uint16_t *V, float *O, int Hq, int Hkv, int Sq,
                      int Sk, int D, int causal, int bk, int bq, int v_prepacked, int nthreads) {
    orc_attn_blocked_rows(Q, K, V, O, Hq, Hkv, Sq, Sk, D, causal, bk, bq, v_prepacked, 0, Sq, nthreads);
}

/* flash.c:900-913 */
int orc_ref_rowset(int Sq, int ref_cap, int *rows) {
    if (ref_cap <= 0 || ref_cap >= Sq) {
        for (int i = 0; i < Sq; i++) rows[i] = i;
        return Sq;
    }
    if (ref_cap == 1) {
        rows[0] = Sq - 1;
        return 1;
    }
    for (int t = 0; t < ref_cap; t++) rows[t] = (int)(((int64_t)t * (Sq - 1)) / (ref_cap - 1));
    return ref_cap;
}

/* flash.c:958-980 plus the task's two extra bounds. res[0]=mad, res[1]=maxref,
 * res[2]=rel_l2 = ||k-r||_2 / ||r||_2 over the finite checked elements. Returns nbad
 * (non-finite elements on either side, counted out of band like the reference). */
long orc_cmp_rows(const float *Oref, const float *Odut, int Hq, int Sq, int D, const int *rows, int nrows,
                  double *res) {
    float mad = 0, maxref = 0;
    double num = 0, den = 0;
    long nbad = 0;
    for (int h = 0; h < Hq; h++)
        for (int t = 0; t < nrows; t++)
            for (int d = 0; d < D; d++) {
                const size_t idx = ((size_t)h * Sq + rows[t]) * D + d;
                const float r = Oref[idx], k = Odut[idx], ad = fabsf(k - r);
                if (!isfinite(k) || !isfinite(r)) {
                    nbad++;
                    continue;
                }
                if (ad > mad) mad = ad;
                if (fabsf(r) > maxref) maxref = fabsf(r);
                num += (double)(k - r) * (double)(k - r);
                den += (double)r * (double)r;
            }
    res[0] = mad;
    res[1] = maxref;
    res[2] = den > 0 ? sqrt(num / den) : sqrt(num);
    return nbad;
}

/* flash.c:874-887 */
double orc_attn_pairs(int Sq, int Sk, int causal) {
    if (!causal) return (double)Sq * Sk;
    double n = 0;
    for (int i = 0; i < Sq; i++) {
        int cnt = Sk - Sq + i + 1;
        if (cnt > Sk) cnt = Sk;
        if (cnt < 0) cnt = 0;
        n += cnt;
    }
    return n;
}

/* flash.c:658-672: Vt[D*bk]bf16, Pb[BQ*bk]bf16, S[BQ*bk]f32, pv[D], acc[BQ*D], m, l, al[BQ],
 * each 64-B aligned, total rounded to 64. */
size_t orc_ref_scratch_bytes(int D, int bk, int bq) {
    const size_t a = 64;
    size_t off = 0;
    const size_t sizes[8] = {(size_t)D * bk * 2, (size_t)bq * bk * 2, 4u * (size_t)bq * bk, 4u * (size_t)D,
                             4u * (size_t)bq * D, 4u * (size_t)bq, 4u * (size_t)bq, 4u * (size_t)bq};
    for (int i = 0; i < 8; i++) {
        off = (off + a - 1) & ~(a - 1);
        off += sizes[i];
    }
    return (off + a - 1) & ~(a - 1);
}

/* README.md:359-436: largest power-of-two bk in [16, 4096] with
 * 2*(6*bk*(D+BQ) + 6*BQ*D + 4*D + 12*BQ) <= l2; floor 16; D < 1 clamped; exact arithmetic
 * in unsigned __int128 so the model has no overflow anywhere. */
int orc_pick_bk_model(int D, size_t l2, int bq) {
    const unsigned __int128 d = D < 1 ? 1u : (unsigned)D, B = (unsigned)bq;
    int best = 16;
    for (int bk = 16; bk <= 4096; bk *= 2) {
        const unsigned __int128 ws = 6u * (unsigned __int128)bk * (d + B) + 6u * B * d + 4u * d + 12u * B;
        if (2u * ws > (unsigned __int128)l2) break;
        best = bk;
    }
    return best;
}

/* Merge nparts partials (m in base-2 units, l, unnormalised acc) into O. */
void orc_combine(const float *m, const float *l, const float *acc, int nparts, int rows, int D, float *O) {
    for (int r = 0; r < rows; r++) {
        float mx = -INFINITY;
        for (int s = 0; s < nparts; s++)
            if (m[(size_t)s * rows + r] > mx) mx = m[(size_t)s * rows + r];
        double L = 0;
        for (int s = 0; s < nparts; s++) {
            const float ms = m[(size_t)s * rows + r];
            if (ms != -INFINITY) L += exp2((double)ms - mx) * l[(size_t)s * rows + r];
        }
        for (int d = 0; d < D; d++) {
            double a = 0;
            for (int s = 0; s < nparts; s++) {
                const float ms = m[(size_t)s * rows + r];
                if (ms != -INFINITY) a += exp2((double)ms - mx) * acc[((size_t)s * rows + r) * D + d];
            }
            O[(size_t)r * D + d] = L > 0 ? (float)(a / L) : 0.f;
        }
    }
}
