/* attn_flash_diag.h -- diagnostic entry points of the B200 attention library.
 *
 * None of these is part of the attention path and none has a counterpart in the reference
 * (flash.c runs on one CPU core). They exist so that tests can check, through the same C ABI,
 * what the attention entry points alone cannot show: that a kernel's result does not depend
 * on what an earlier kernel left in tensor memory, the accuracy of the kernel's exponential,
 * and that a bounded wait that runs out is reported without a hang. Device pointers; every
 * call is asynchronous on `stream` and allocates nothing.
 */
#ifndef ATTN_FLASH_DIAG_H
#define ATTN_FLASH_DIAG_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Device status codes the kernels OR into the scratch status word (the `device_code` of
 * attn_flash_status). */
#define ATTN_DEV_TIMEOUT_Q 1      /* a Q tile never arrived */
#define ATTN_DEV_TIMEOUT_KV 2     /* a K/V stage never arrived or was never released */
#define ATTN_DEV_TIMEOUT_S 4      /* the softmax waited too long for a score tile */
#define ATTN_DEV_TIMEOUT_P 8      /* the MMA issuer waited too long for a P tile */
#define ATTN_DEV_TIMEOUT_DRAIN 16 /* teardown waited too long for in-flight copies / MMAs */
#define ATTN_DEV_BAD_PAGE 32      /* a block table held a page id outside the pool */
#define ATTN_DEV_BAD_POS 64       /* a token position outside the rotary table or the cache */
#define ATTN_DEV_TIMEOUT_PEER 128 /* a peer GPU's partials never arrived (multi-GPU merge) */

/* The work plan attn_flash_stream would use for this problem on the tensor-core path of a GPU
 * with `sms` SMs: pure host arithmetic, no device is touched. out[0..4] = nsplit (key pieces
 * per unit), keys_per_split, n_direct (units run whole before a split last wave, 0 when every
 * unit is split or none is), row_base (first query row of the split units), units (query-row
 * tiles x kv heads). Returns ATTN_OK or ATTN_ERR_ARGS. */
int attn_diag_plan(int Hq, int Hkv, int Sq, int Sk, int D, int causal, int sms, int out[5]);

/* Writes the 32-bit pattern `bits` into every lane and column of the tensor memory (TMEM) of
 * every SM, by CTAs that allocate all 512 columns, store, and free them again. */
int attn_diag_fill_tmem(uint32_t bits, void *stream);

/* y[i] = 2^x[i] by one of the attention kernel's two exponentials: */
#define ATTN_DIAG_EXP2_POLY 0 /* the FMA-pipe polynomial (inputs clamped at -125) */
#define ATTN_DIAG_EXP2_MUFU 1 /* the hardware ex2.approx.ftz.f32 */
int attn_diag_exp2(const float *x, float *y, int n, int method, void *stream);

/* Runs the tensor-core attention kernel (head_dim 128, at most 128 query rows per kv head:
 * (Hq / Hkv) * Sq <= 128) in a build whose producer never loads Q, so the MMA issuer's bounded
 * wait for Q runs out after its limit (about 2 s) and every role of every CTA unwinds: the
 * kernel returns, O is left unwritten, and attn_flash_status(scratch, ...) reports
 * ATTN_ERR_DEVICE with ATTN_DEV_TIMEOUT_Q in the device code -- or ATTN_DEV_TIMEOUT_KV: the
 * producer's wait for a K/V slot the MMA never frees starts at the same moment, and whichever
 * wait expires first is reported. The context stays usable.
 * scratch: at least attn_flash_scratch_bytes(128, bk) bytes. */
int attn_diag_wait_timeout(const uint16_t *Q, const uint16_t *K, const uint16_t *V, float *O, int Hq,
                           int Hkv, int Sq, int Sk, void *scratch, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* ATTN_FLASH_DIAG_H */
