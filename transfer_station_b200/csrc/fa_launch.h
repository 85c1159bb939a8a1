/* fa_launch.h -- the plain-C contract between the host layer (attn_flash.c) and the CUDA
 * launchers (*.cu). The host layer validates arguments, plans the split-KV decomposition and
 * carves the scratch block; the launchers build TMA descriptors and launch kernels. */
#ifndef TS_FA_LAUNCH_H
#define TS_FA_LAUNCH_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Scratch block layout (device memory, caller-owned, ATTN_SCRATCH_ALIGN-aligned):
 *   [0, 256)                       int status word (+ padding)
 *   [256, 256 + cap*4)             partial m   [nsplit][rows]
 *   then                           partial l   [nsplit][rows]
 *   then                           partial acc [nsplit][rows][D]
 * where cap = ATTN_PARTIAL_ROWS, and the three regions are sized for D at the full cap. */
#define TS_SCRATCH_CTRL_BYTES 256

typedef struct fa_problem {
    const uint16_t *Q, *K, *V; /* device pointers */
    float *O;                  /* normalised output [Hq][Sq][D]; NULL in partial mode */
    float *part_m, *part_l, *part_acc; /* where the kernel writes partials, [nsplit][Hq*Sq](,[D]) */
    float *out_m, *out_l, *out_acc;    /* caller's single partial (write_partials mode) */
    int *status;               /* device status word */
    int Hq, Hkv, Sq, Sk;       /* Sk = keys present in K/V (local shard length) */
    int Sk_total, k_begin;     /* global key axis length and this shard's first key */
    int D, causal, v_prepacked;
    int o_bf16;                /* 1: O holds bf16 bits [Hq][Sq][D] (RNE as flash.c:78-92), else fp32 */
    int nsplit;                /* >1: split the key range, write partials, then combine */
    int keys_per_split;        /* multiple of the key tile */
    int write_partials;        /* 1: leave the result as (m, l, acc) partials, no combine */
    /* Tensor-core path work plan. Units (query-row tiles of one kv head, kv-major) below
     * n_direct run over the whole key range; units from n_direct on run as `nsplit` key pieces
     * of keys_per_split keys each, writing partials [piece][row - row_base] (row = global row
     * of [Hq*Sq]; the split units' rows are exactly [row_base, Hq*Sq)), merged by the combine.
     * Decode splits every unit (n_direct = 0); a prefill whose last wave would run less than
     * half full splits only that wave's units. */
    int n_direct;
    int row_base;
    /* Paged K/V (paged != 0, tensor-core path only): K and V are pools
     * [num_pages][hkv_local][page_size][D]; kv head index = b * hkv_local + kv_local for
     * sequence b, whose keys live in pages block_table[b * max_pages + k / page_size] and whose
     * length is seq_lens[b] (device arrays); Sk is the bound max_pages * page_size. */
    const int *block_table, *seq_lens;
    int paged, page_size, max_pages, num_pages, hkv_local;
    float scale_log2;          /* (1/sqrt(D)) * log2(e) */
    /* 0: the caller cleared the status word before the launch. Otherwise the tensor-core
     * kernel clears it itself (CTA 0 zeroes status[0], then stores this value in status[1];
     * error reports wait for that store), so no memset has to sit between two launches. */
    unsigned status_gen;
} fa_problem;

/* Number of SMs of the current device (cached). */
int ts_num_sms(void);
/* Compute capability major of the current device (cached). */
int ts_cc_major(void);
/* The tcgen05 path applies to this problem (D multiple of 8, <= 128, aligned pointers,
 * Sk multiple of 8 when V is pre-transposed). Otherwise the SIMT path runs. */
int ts_tc_supported(const fa_problem *p);
/* Units (CTAs per split) of the tcgen05 path for this problem, and query rows per unit. */
int ts_tc_ctas_per_split(const fa_problem *p);
int ts_tc_unit_rows(const fa_problem *p);

/* Launch the main kernel (tcgen05 or SIMT path chosen inside) plus, when nsplit > 1 and
 * !write_partials, the combine kernel. Returns 0 or a negative ATTN_ERR_* code. */
int ts_launch_attention(const fa_problem *p, void *stream);

/* Launch the combine kernel alone on partial arrays. */
int ts_launch_combine(const float *m, const float *l, const float *acc, int nparts, int rows, int D,
                      float *O, float *out_m, float *out_l, int out_bf16, void *stream);

/* The same with each part's m/l and acc `ps_ml` / `ps_acc` floats apart (m[s*ps_ml + r],
 * acc[s*ps_acc + r*D + c]): packed per-rank partials gathered by one collective. */
int ts_launch_combine_strided(const float *m, const float *l, const float *acc, int nparts, int rows, int D,
                              size_t ps_ml, size_t ps_acc, float *O, float *out_m, float *out_l, int out_bf16,
                              void *stream);

/* The main attention kernel alone (tensor-core or general path), without the merge of split
 * key pieces that ts_launch_attention adds: the pieces stay in the partial arrays. */
int ts_launch_attention_pieces(const fa_problem *p, void *stream);

/* The key-split decode's merge over NVLink (fa_peer.cu): nparts local key pieces [nparts][rows]
 * (0: an empty shard) -> every rank's exchange block -> O [rows][D] fp32. */
int ts_launch_peer_merge(const float *m, const float *l, const float *acc, int nparts, int rows, int D,
                         float *O, void *const *blocks, int world, int rank, unsigned epoch, int *status,
                         void *stream);

/* The QKV producer (qkv_rope.cu): one validated call of attn_qkv_rope_stream or
 * attn_qkv_rope_paged_stream. n_vec = B*S*(Hq + 2*Hkv) head vectors of D elements. */
typedef struct ts_rope_problem {
    const uint16_t *qkv;
    const int *positions;
    const float *cos_sin;
    const uint16_t *q_norm_w, *k_norm_w;
    uint16_t *Q, *K, *V;
    const int *block_table; /* NULL: contiguous cache [B*Hkv][cache_len][D] */
    int *status;
    long long n_vec;
    float eps;
    int B, S, Hq, Hkv, D, rot, style, max_pos;
    int cache_len;                         /* contiguous cache rows per (sequence, kv head) */
    int page_size, num_pages, max_pages;   /* paged cache */
} ts_rope_problem;

int ts_launch_qkv_rope(const ts_rope_problem *p, void *stream);
int ts_launch_rope_table(float *cos_sin, int max_pos, int rot, double theta, void *stream);

/* A fresh nonzero status generation (fa_problem.status_gen), unique within the process. */
unsigned ts_next_status_gen(void);

/* Zero the device status word (async). */
int ts_clear_status(int *status, void *stream);
/* Synchronise the stream, read and clear the status word. */
int ts_read_status(int *status, void *stream, int *value);

#ifdef __cplusplus
}
#endif

#endif /* TS_FA_LAUNCH_H */
