/* attn_flash.h -- C ABI of the B200 (sm_100a) bf16 flash-attention forward.
 *
 * Drop-in for the attention entry points of flash.c (liujiang833/transfer_station):
 * the same names, the same argument meaning, the same bk contract. What changes is where
 * the tensors live: every tensor pointer here is a DEVICE pointer (cudaMalloc'd, or
 * managed memory), and the caller-owned scratch block is device memory too.
 *
 * Tensor layouts (all contiguous, row-major, no strides -- as in flash.c):
 *   Q  bf16 bit patterns (uint16_t)  [Hq ][Sq][D]
 *   K  bf16 bit patterns             [Hkv][Sk][D]
 *   V  bf16 bit patterns             [Hkv][Sk][D], or V^T [Hkv][D][Sk] when v_prepacked=1
 *   O  fp32                          [Hq ][Sq][D]
 * Query head h reads kv head h / (Hq/Hkv): MHA (Hkv==Hq), GQA, MQA (Hkv==1).
 * Batch is folded into the head axis: Q [B*Hq][Sq][D], K/V [B*Hkv][Sk][D] maps batch b's
 * head hq to kv head b*Hkv + hq/group, which is exactly (b*Hq+hq)/group.
 * Scale is 1/sqrt(D). causal uses the bottom-right convention: query row i attends keys
 * j <= Sk - Sq + i; a row that attends no key at all gets a zero output row.
 *
 * Nothing here allocates device memory. Every call is asynchronous on its stream except
 * attn_flash(), which keeps the reference's blocking, void-returning contract.
 *
 * Threads: like flash.c (re-entrant given one scratch block per calling thread,
 * flash.c:588-592), any number of host threads may call these entry points at once as long as
 * each uses its own scratch block; give each thread its own stream for the calls to overlap.
 * The library's only shared state is a per-device cache of device attributes and the launch
 * counter, both safe to use concurrently.
 */
#ifndef ATTN_FLASH_B200_H
#define ATTN_FLASH_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* bk contract, unchanged from flash.c:132-134: a power of two in [16, 4096]; anything
 * else prints the contract to stderr and abort()s, at both doors (attn_flash and
 * attn_flash_scratch_bytes), exactly as flash.c:641-647 does. */
#define ATTN_BK_MIN 16
#define ATTN_BK_MAX 4096
#define ATTN_BK_DEFAULT 128

/* Scratch alignment. flash.c:607 used a 64-B cache line; device scratch wants 256 B
 * (cudaMalloc returns 256-B aligned blocks, so any cudaMalloc'd block qualifies). */
#define ATTN_SCRATCH_ALIGN 256

/* The largest key tile the B200 kernel runs (keys per TMEM score tile). bk values above it
 * are legal and run with this tile; bk values below 128 run with this tile too (the GPU
 * result does not depend on bk beyond bf16 rounding noise, as on the CPU). */
#define ATTN_GPU_KEY_TILE 128

/* Largest head_dim the kernels accept. */
#define ATTN_D_MAX 256

/* Decode partial rows the scratch block holds (split-KV partials (m, l, acc[D])).
 * Scratch size stays independent of Sq and Sk, as in flash.c; a call whose split-KV plan
 * would need more partial rows uses fewer splits. */
#define ATTN_PARTIAL_ROWS 65536

/* Status codes of the *_stream entry points. */
#define ATTN_OK 0
#define ATTN_ERR_ARGS -1        /* bad shape / null pointer / Hq % Hkv != 0 / D out of range */
#define ATTN_ERR_ALIGN -2       /* a device pointer is not 16-byte aligned */
#define ATTN_ERR_CUDA -3        /* a CUDA runtime/driver call failed */
#define ATTN_ERR_DEVICE -4      /* the kernel reported a bounded wait that ran out (see scratch status) */
#define ATTN_ERR_NOT_SM100 -5   /* the current device is not compute capability 10.x */

/* Per-phase timers of flash.c:704-706. The reference adds each phase's seconds into *tm on
 * every call (flash.c:822-849), so a caller zeroes it once and accumulates. On the GPU the four
 * phases run fused in one kernel (and V is never transposed: packv has no counterpart), so
 * attn_flash() adds nothing: *tm keeps whatever the caller had accumulated. Time the kernel
 * with CUDA events. */
struct attn_times {
    double packv, qxk, softmax, sxv;
};

/* Bytes of device scratch one attn_flash call needs for this head_dim and key-block size.
 * Replaces flash.c:679-682 (attn_flash_scratch_bytes). Validates bk (abort on violation,
 * as flash.c). Independent of Sq and Sk: a status word plus ATTN_PARTIAL_ROWS split-KV
 * partial rows of (D + 2) floats. */
size_t attn_flash_scratch_bytes(int D, int bk);

/* Tile-config picker. Replaces attn_flash_pick_bk(int D, size_t l2_bytes), specified at
 * README.md:137-140,359-436 of the reference (absent from its shipped flash.c). First the
 * reference's analytical model at the GPU's query block BQ=128: the largest power of two
 * bk in [16, 4096] with 2*(6*bk*(D+BQ) + 6*BQ*D + 4*D + 12*BQ) <= l2_bytes (floor 16, cap
 * 4096, D < 1 clamped to 1, size_t arithmetic throughout); then clamped to
 * ATTN_GPU_KEY_TILE, the largest key tile the B200 kernel has. Always a legal bk. */
int attn_flash_pick_bk(int D, size_t l2_bytes);

/* The attention forward. Replaces flash.c:727-864 (static attn_flash). Device pointers.
 * Blocking: returns after the result is in O, like the CPU reference. Aborts with a
 * message on a bad bk (the reference contract) and on any other error (the void signature
 * cannot report one; use attn_flash_stream for a status code). */
void attn_flash(const uint16_t *Q, const uint16_t *K, const uint16_t *V, float *O, int Hq,
                int Hkv, int Sq, int Sk, int D, int causal, int bk, void *scratch,
                int v_prepacked, struct attn_times *tm);

/* Asynchronous variant of attn_flash on an explicit stream (a cudaStream_t passed as
 * void*; NULL = legacy default stream). Same arguments and semantics as attn_flash;
 * returns ATTN_OK or a negative status (bk is still validated by abort). A device-side
 * failure (a bounded wait that ran out) is recorded in the scratch status word: read it
 * with attn_flash_status. Concurrent calls must use distinct scratch blocks. */
int attn_flash_stream(const uint16_t *Q, const uint16_t *K, const uint16_t *V, float *O,
                      int Hq, int Hkv, int Sq, int Sk, int D, int causal, int bk,
                      void *scratch, int v_prepacked, void *stream);

/* Output element types of attn_flash_stream_out. */
#define ATTN_OUT_F32 0  /* fp32, the reference's O (flash.c:727-729) */
#define ATTN_OUT_BF16 1 /* bf16 bit patterns, rounded as flash.c:78-92 rounds P */

/* attn_flash_stream with a choice of output element type: out_dtype ATTN_OUT_F32 is exactly
 * attn_flash_stream; ATTN_OUT_BF16 writes O as uint16_t bf16 bits [Hq][Sq][D] (round to
 * nearest even, NaN/Inf passed through), halving the output bytes: each element equals the
 * rounding of what the fp32 call returns. An extension of the reference's interface, which
 * writes fp32 O only (flash.c:727-729); any other out_dtype returns ATTN_ERR_ARGS. */
int attn_flash_stream_out(const uint16_t *Q, const uint16_t *K, const uint16_t *V, void *O,
                          int out_dtype, int Hq, int Hkv, int Sq, int Sk, int D, int causal, int bk,
                          void *scratch, int v_prepacked, void *stream);

/* Attention over a paged K/V cache (decode, or a few new query positions per sequence). No
 * counterpart in the reference, whose K and V are contiguous (flash.c:727-729): this is the
 * serving-side layout. B sequences; Q [B*Hq][Sq][D] and O [B*Hq][Sq][D] (fp32) as in
 * attn_flash with batch folded into heads; K_pages and V_pages are pools
 * [num_pages][Hkv][page_size][D] of bf16 bits; sequence b's keys are, in order, the rows of
 * pages block_table[b * max_pages + 0 ..] and it has seq_lens[b] of them (clamped to
 * [0, max_pages * page_size]; a sequence with none gets zero rows). block_table and seq_lens
 * are device int arrays. causal: query i of sequence b sees keys 0 .. seq_lens[b] - Sq + i.
 * page_size is 8, 16, 32, 64 or a multiple of 128; D a multiple of 8 up to 128; all pointers
 * 16-byte aligned. A page id outside [0, num_pages) is caught by the kernel: it stops and
 * attn_flash_status returns ATTN_ERR_DEVICE. Scratch as for attn_flash_stream. */
int attn_flash_paged_stream(const uint16_t *Q, const uint16_t *K_pages, const uint16_t *V_pages,
                            const int *block_table, const int *seq_lens, float *O, int B, int Hq,
                            int Hkv, int Sq, int D, int causal, int page_size, int num_pages,
                            int max_pages, void *scratch, void *stream);

/* Synchronises `stream`, reads and clears the device status word in `scratch`.
 * Returns ATTN_OK, or ATTN_ERR_DEVICE when a kernel on that scratch reported a failure
 * (the raw device code goes to *device_code when non-NULL), or ATTN_ERR_CUDA. */
int attn_flash_status(void *scratch, void *stream, int *device_code);

/* Human-readable name of a status code. */
const char *attn_flash_strerror(int status);

/* Diagnostic: number of CUDA kernels this library has launched in this process (all
 * devices, all entry points). No counterpart in flash.c; benchmarks use it to report how
 * many of the library's kernels ran inside a timed region. */
unsigned long long attn_flash_kernel_launches(void);

/* Key-sharded partial attention for multi-GPU long-context decode (no counterpart in
 * flash.c, whose single call covers all keys; this is the per-GPU half of the key split
 * of flash.c:798's key loop). K and V hold keys [k_begin, k_begin + Sk_local) of a key
 * axis of length Sk_total; masking uses global key positions. Writes, per query row r of
 * [Hq*Sq], the reference max m[r] in base-2 units of the scaled score (the partial's
 * exponents are exp2(s*scale*log2(e) - m[r]); -inf if the row saw no key), the
 * denominator l[r] and the UNnormalised accumulator acc[r][D]. */
int attn_flash_partial_stream(const uint16_t *Q, const uint16_t *K, const uint16_t *V,
                              float *m, float *l, float *acc, int Hq, int Hkv, int Sq,
                              int Sk_local, int Sk_total, int k_begin, int D, int causal,
                              int bk, void *scratch, int v_prepacked, void *stream);

/* Merges nparts partials laid out [nparts][rows] (m, l) and [nparts][rows][D] (acc), as
 * produced by attn_flash_partial_stream on disjoint key ranges, into O [rows][D] fp32:
 * O = sum_s 2^(m_s - m*) acc_s / sum_s 2^(m_s - m*) l_s (a zero row where every l_s is 0),
 * m* = max_s m_s. */
int attn_flash_combine_stream(const float *m, const float *l, const float *acc, int nparts,
                              int rows, int D, float *O, void *stream);

/* Floats of one packed partial: m [rows], l [rows], padding to a multiple of 4 floats, then
 * acc [rows][D]. A rank of a key-split decode lets attn_flash_partial_stream write its m, l and
 * acc into one such block, so one all-gather moves every rank's partials together. No
 * counterpart in the reference (one call on one core). */
size_t attn_flash_packed_floats(int rows, int D);

/* attn_flash_combine_stream over nparts packed partials laid out back to back:
 * parts[s * attn_flash_packed_floats(rows, D) + ...] (what one all-gather of the per-rank
 * blocks produces). */
int attn_flash_combine_packed_stream(const float *parts, int nparts, int rows, int D, float *O,
                                     void *stream);

/* ---- The key-split decode merged over NVLink with peer stores: one kernel per rank, no
 * collective library. No counterpart in the reference (one call on one core); it distributes
 * the online-softmax merge of flash.c:535-576 over the GPUs of one node. ----
 *
 * Each rank owns one exchange block of attn_flash_peer_block_bytes(world, Hq*Sq, D) bytes of its
 * device memory, zeroed once before the first call, and maps every peer's block into its address
 * space (attn_peer_export on the owner, attn_peer_import on the others: CUDA IPC, peer access
 * enabled). */
#define ATTN_PEERS_MAX 8           /* ranks of one merge (the GPUs of one node) */
#define ATTN_PEER_HANDLE_BYTES 128 /* bytes of an exported block handle */

/* Bytes of one rank's exchange block. Layout, the same on every rank: uint32 flags
 * [ATTN_PEERS_MAX][128] (the epoch each rank's merge CTA c reached), then two buffers (epoch
 * parity) of `world` slots, slot s holding rank s's packed partial (attn_flash_packed_floats(rows,
 * D) floats: m [rows], l [rows], padding, acc [rows][D]) rounded up to 256 bytes. */
size_t attn_flash_peer_block_bytes(int world, int rows, int D);

/* Writes an ATTN_PEER_HANDLE_BYTES handle of the device block at dev_ptr (any block inside a
 * cudaMalloc allocation) that other processes on the node can import. */
int attn_peer_export(void *dev_ptr, void *handle);
/* Maps a peer's exported block into this process (on the current device); *dev_ptr receives its
 * address here. attn_peer_close(dev_ptr, handle) unmaps it. */
int attn_peer_import(const void *handle, void **dev_ptr);
int attn_peer_close(void *dev_ptr, const void *handle);

/* attn_flash_partial_stream on this rank's key shard, then ONE merge kernel: it merges the
 * shard's key pieces per row, stores the rank's (m, l, acc) into slot `rank` of every rank's
 * exchange block over NVLink, raises its flags there, waits (bounded) until every rank's partials
 * reached its own block, and writes the full attention O [Hq][Sq][D] fp32 -- on every rank.
 * blocks[r] is rank r's exchange block as mapped in this process (blocks[rank] its own). epoch
 * numbers the calls made with these blocks: 1 for the first call, +1 per call, the same on every
 * rank, and every rank makes every call (a rank with an empty shard passes Sk_local = 0).
 * A peer that never arrives ends the wait after ~2 s with ATTN_DEV_TIMEOUT_PEER in the status
 * word (attn_flash_status). Requires Hq*Sq <= ATTN_PARTIAL_ROWS. */
int attn_flash_decode_peers_stream(const uint16_t *Q, const uint16_t *K, const uint16_t *V, float *O,
                                   int Hq, int Hkv, int Sq, int Sk_local, int Sk_total, int k_begin,
                                   int D, int causal, int bk, void *scratch, void *const *blocks,
                                   int world, int rank, unsigned int epoch, void *stream);

/* attn_flash without a scratch argument, for callers that cannot allocate device memory (a
 * host whose device memory belongs to its own pool allocator, or a foreign-function binding
 * with nowhere to keep a device buffer between calls). No counterpart in the reference: its
 * scratch is host memory the caller passes in. Uses a fixed 4 MiB block of device memory
 * declared by the library (held on every GPU that loads it until exit) and calls no
 * allocator. Accepts at most 4096 query rows (Hq*Sq) -- decode-shaped calls -- and returns
 * ATTN_ERR_ARGS beyond that. All calls on a device share the block: calls whose GPU work
 * overlaps race. The first call on a device looks the block up; the address is kept until
 * exit, so do not call it on a device again after cudaDeviceReset. Blocks until the work on
 * `stream` is done (it synchronises the stream), so it is never captured into a CUDA graph: on
 * a capturing stream it returns ATTN_ERR_ARGS and does nothing. Returns ATTN_OK or a status
 * code. */
int attn_flash_noalloc(const uint16_t *Q, const uint16_t *K, const uint16_t *V, float *O, int Hq,
                       int Hkv, int Sq, int Sk, int D, int causal, int bk, int v_prepacked,
                       void *stream);

#ifdef __cplusplus
}
#endif

#endif /* ATTN_FLASH_B200_H */
