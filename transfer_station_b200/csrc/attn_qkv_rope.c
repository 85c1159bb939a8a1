/* attn_qkv_rope.c -- host layer of the QKV producer (attn_qkv_rope.h): validates a call and
 * hands it to the launcher in qkv_rope.cu. Allocates nothing; the only device memory it
 * touches besides the caller's tensors is the status word of the caller's scratch block. */
#include <limits.h>
#include <math.h>
#include <stdint.h>
#include <stddef.h>

#include "attn_qkv_rope.h"
#include "fa_launch.h"

static int ts_al16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

int attn_rope_table_stream(float *cos_sin, int max_pos, int rot, double theta, void *stream) {
    if (!cos_sin || max_pos < 1 || rot < 16 || rot > ATTN_D_MAX || rot % 16 != 0 || !(theta > 1.0) || !isfinite(theta))
        return ATTN_ERR_ARGS;
    if ((size_t)max_pos * (size_t)rot > (size_t)LLONG_MAX / 4) return ATTN_ERR_ARGS;
    if (ts_cc_major() != 10) return ATTN_ERR_NOT_SM100;
    return ts_launch_rope_table(cos_sin, max_pos, rot, theta, stream);
}

/* Shared checks of both producers; fills everything but the cache fields. */
static int ts_rope_fill(ts_rope_problem *P, const uint16_t *qkv, const int *positions, const float *cos_sin,
                        int max_pos, const uint16_t *q_norm_w, const uint16_t *k_norm_w, float eps, int B, int S,
                        int Hq, int Hkv, int D, int rot, int style, uint16_t *Q, uint16_t *K, uint16_t *V,
                        void *scratch) {
    if (!qkv || !positions || !Q || !K || !V || !scratch) return ATTN_ERR_ARGS;
    if (B < 0 || S < 0 || Hq < 1 || Hkv < 1 || (D != 64 && D != 128 && D != 256)) return ATTN_ERR_ARGS;
    if (rot < 0 || rot > D || rot % 16 != 0 || (style != ATTN_ROPE_NEOX && style != ATTN_ROPE_GPTJ)) return ATTN_ERR_ARGS;
    if (rot > 0 && (!cos_sin || max_pos < 1)) return ATTN_ERR_ARGS;
    if ((q_norm_w || k_norm_w) && !(eps >= 0.0f && isfinite(eps))) return ATTN_ERR_ARGS;
    if ((long long)B * S > INT_MAX) return ATTN_ERR_ARGS;
    const long long htot = (long long)Hq + 2LL * Hkv;
    const long long n_vec = (long long)B * S * htot;
    if (n_vec > LLONG_MAX / (8LL * D)) return ATTN_ERR_ARGS;
    if (!ts_al16(qkv) || !ts_al16(Q) || !ts_al16(K) || !ts_al16(V) || !ts_al16(cos_sin) || !ts_al16(q_norm_w) ||
        !ts_al16(k_norm_w) || ((uintptr_t)scratch % ATTN_SCRATCH_ALIGN) != 0)
        return ATTN_ERR_ALIGN;
    P->qkv = qkv;
    P->positions = positions;
    P->cos_sin = rot > 0 ? cos_sin : NULL;
    P->q_norm_w = q_norm_w;
    P->k_norm_w = k_norm_w;
    P->Q = Q;
    P->K = K;
    P->V = V;
    P->block_table = NULL;
    P->status = (int *)scratch; /* the status word heads every scratch block */
    P->n_vec = n_vec;
    P->eps = eps;
    P->B = B;
    P->S = S;
    P->Hq = Hq;
    P->Hkv = Hkv;
    P->D = D;
    P->rot = rot;
    P->style = style;
    P->max_pos = rot > 0 ? max_pos : INT_MAX;
    P->cache_len = 0;
    P->page_size = P->num_pages = P->max_pages = 0;
    return ATTN_OK;
}

/* Every argument is checked before the device is consulted. */
static int ts_rope_run(const ts_rope_problem *P, void *stream) {
    if (ts_cc_major() != 10) return ATTN_ERR_NOT_SM100;
    int rc = ts_clear_status(P->status, stream);
    if (rc != ATTN_OK) return rc;
    return ts_launch_qkv_rope(P, stream);
}

int attn_qkv_rope_stream(const uint16_t *qkv, const int *positions, const float *cos_sin, int max_pos,
                         const uint16_t *q_norm_w, const uint16_t *k_norm_w, float eps, int B, int S, int Hq, int Hkv,
                         int D, int rot, int style, uint16_t *Q, uint16_t *K_cache, uint16_t *V_cache, int cache_len,
                         void *scratch, void *stream) {
    ts_rope_problem P;
    int rc = ts_rope_fill(&P, qkv, positions, cos_sin, max_pos, q_norm_w, k_norm_w, eps, B, S, Hq, Hkv, D, rot, style,
                          Q, K_cache, V_cache, scratch);
    if (rc != ATTN_OK) return rc;
    if (cache_len < 1) return ATTN_ERR_ARGS;
    P.cache_len = cache_len;
    return ts_rope_run(&P, stream);
}

int attn_qkv_rope_paged_stream(const uint16_t *qkv, const int *positions, const float *cos_sin, int max_pos,
                               const uint16_t *q_norm_w, const uint16_t *k_norm_w, float eps, int B, int S, int Hq,
                               int Hkv, int D, int rot, int style, uint16_t *Q, uint16_t *K_pages, uint16_t *V_pages,
                               const int *block_table, int page_size, int num_pages, int max_pages, void *scratch,
                               void *stream) {
    ts_rope_problem P;
    int rc = ts_rope_fill(&P, qkv, positions, cos_sin, max_pos, q_norm_w, k_norm_w, eps, B, S, Hq, Hkv, D, rot, style,
                          Q, K_pages, V_pages, scratch);
    if (rc != ATTN_OK) return rc;
    if (!block_table || page_size < 1 || num_pages < 1 || max_pages < 1) return ATTN_ERR_ARGS;
    if ((long long)page_size * max_pages > INT_MAX) return ATTN_ERR_ARGS;
    P.block_table = block_table;
    P.page_size = page_size;
    P.num_pages = num_pages;
    P.max_pages = max_pages;
    return ts_rope_run(&P, stream);
}
