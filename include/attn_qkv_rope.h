/* attn_qkv_rope.h -- C ABI of the producer upstream of attn_flash on B200 (sm_100a).
 *
 * A transformer layer's fused QKV projection writes, per token, the q heads, then the k heads,
 * then the v heads of that token. Before attention, the q and k heads take a per-head RMSNorm
 * (Qwen3's q_norm / k_norm; optional) and a rotary position embedding, Q moves to attn_flash's
 * [B*Hq][S][D] layout and K/V land in the key cache at each token's position. These entry
 * points do all of that in one HBM pass. The reference has no counterpart: its projections
 * "never reach this kernel" (flash.c:1301-1304), so this is the caller-side step of the path,
 * built to the published formulas:
 *   RMSNorm (Zhang & Sennrich, 2019):  y_i = x_i * rsqrt(mean_j(x_j^2) + eps) * w_i
 *   RoPE (Su et al., RoFormer, 2021), frequency f_i = theta^(-2i/rot), angle a = pos * f_i:
 *     ATTN_ROPE_NEOX  pairs (i, i + rot/2):  x_i' = x_i cos a - x_{i+rot/2} sin a,
 *                                            x_{i+rot/2}' = x_{i+rot/2} cos a + x_i sin a
 *     ATTN_ROPE_GPTJ  pairs (2i, 2i + 1):    x_2i' = x_2i cos a - x_2i+1 sin a,
 *                                            x_2i+1' = x_2i+1 cos a + x_2i sin a
 *   elements at or beyond rot pass through.
 * Arithmetic is fp32 (x * cos and y * sin each rounded to fp32, then one fp32 add or
 * subtract, no fused multiply-add) with ONE rounding to bf16 at the end (round to nearest
 * even, as flash.c:78-92 rounds; a NaN becomes the canonical bf16 NaN); v heads are copied bit
 * for bit.
 *
 * Layouts (device pointers, contiguous, bf16 bit patterns unless noted):
 *   qkv        [B*S][(Hq + 2*Hkv) * D]    token t = b*S + s
 *   positions  int32 [B*S]                token t's position: its row of cos_sin and its slot
 *                                         in the key cache
 *   cos_sin    fp32 [max_pos][rot]        cos(p f_i) in column i, sin(p f_i) in column rot/2 + i
 *                                         (attn_rope_table_stream fills it)
 *   q_norm_w, k_norm_w  [D]               RMSNorm weights of q / k heads; NULL skips that norm
 *   Q          [B*Hq][S][D]               attn_flash's Q (batch folded into heads)
 *   contiguous cache:  K_cache, V_cache   [B*Hkv][cache_len][D]; token t of sequence b goes to
 *                                         row positions[t]. cache_len = S with positions 0..S-1
 *                                         gives attn_flash's K and V for that prompt.
 *   paged cache:       K_pages, V_pages   [num_pages][Hkv][page_size][D] with block_table
 *                                         int32 [B][max_pages], attn_flash_paged_stream's
 *                                         layout: position p of sequence b lives in page
 *                                         block_table[b*max_pages + p/page_size], row
 *                                         p % page_size.
 * Requirements: D in {64, 128, 256}; rot a multiple of 16 in [0, D] (0: no rotation); every
 * tensor pointer 16-byte aligned. A token whose position lies outside [0, max_pos) (when
 * rot > 0), outside the cache, or whose page id lies outside [0, num_pages) is skipped whole
 * (none of its heads is written) and the call's scratch status reports it: attn_flash_status
 * on the same scratch block returns ATTN_ERR_DEVICE. Scratch: any block sized by
 * attn_flash_scratch_bytes (only its status word is used); a call clears the word first.
 * Returns ATTN_OK or an ATTN_ERR_* code (attn_flash.h). Asynchronous on `stream`.
 */
#ifndef ATTN_QKV_ROPE_B200_H
#define ATTN_QKV_ROPE_B200_H

#include <stddef.h>
#include <stdint.h>

#include "attn_flash.h"

#ifdef __cplusplus
extern "C" {
#endif

#define ATTN_ROPE_GPTJ 0 /* interleaved pairs (2i, 2i + 1) */
#define ATTN_ROPE_NEOX 1 /* rotate-half pairs (i, i + rot/2): Llama, Qwen */

/* Fill cos_sin [max_pos][rot] for frequencies theta^(-2i/rot): angle, cosine and sine in
 * double precision, rounded once to fp32. rot a positive multiple of 16 (at most 256). */
int attn_rope_table_stream(float *cos_sin, int max_pos, int rot, double theta, void *stream);

/* Producer into a contiguous key cache. */
int attn_qkv_rope_stream(const uint16_t *qkv, const int *positions, const float *cos_sin,
                         int max_pos, const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                         float eps, int B, int S, int Hq, int Hkv, int D, int rot, int style,
                         uint16_t *Q, uint16_t *K_cache, uint16_t *V_cache, int cache_len,
                         void *scratch, void *stream);

/* Producer into a paged key cache. */
int attn_qkv_rope_paged_stream(const uint16_t *qkv, const int *positions, const float *cos_sin,
                               int max_pos, const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                               float eps, int B, int S, int Hq, int Hkv, int D, int rot, int style,
                               uint16_t *Q, uint16_t *K_pages, uint16_t *V_pages,
                               const int *block_table, int page_size, int num_pages,
                               int max_pages, void *scratch, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* ATTN_QKV_ROPE_B200_H */
