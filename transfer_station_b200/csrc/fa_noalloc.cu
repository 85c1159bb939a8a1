// fa_noalloc.cu -- attn_flash_noalloc: the attention call for callers that cannot allocate.
//
// attn_flash / attn_flash_stream need a caller-owned device scratch block (a status word
// plus the split-KV partials). Some callers have no way to provide one: a host application
// whose device memory is owned entirely by its own pool and which forbids libraries from
// calling cudaMalloc, or a thin foreign-function binding (Go, Java, a scripting language)
// that has nowhere to keep a device buffer alive between calls. This entry point serves
// them. Its scratch is a fixed block of device memory that the library itself declares (a
// file-scope __device__ array), so the call allocates nothing.
//
// Limits and sharing rules, stated for the user:
//   * The block is kNoallocBytes = 4 MiB. It exists on every GPU that loads the library and
//     stays allocated until the process exits.
//   * A call may have at most kNoallocMaxRows = 4096 query rows (Hq * Sq): decode-shaped work.
//     Larger calls are rejected with ATTN_ERR_ARGS and a message on stderr. Within that
//     limit the key axis is split only as far as the partials fit in the block.
//   * Every call on a device shares the one block, which keeps the last call's contents.
//     The status word is cleared at the start of each call; every partial the kernels read
//     is written earlier in the same call. Two calls whose GPU work overlaps (different
//     streams, or different host threads) race on the block: serialise them.
//   * The first call on a device looks up the block's device address with
//     cudaGetSymbolAddress (under a mutex), with that device current. No call may be made
//     while its stream is being captured (every call synchronises the stream): such a call
//     returns ATTN_ERR_ARGS and touches nothing. The address is kept for the life of the
//     process: after cudaDeviceReset on a device the library's module is loaded anew and the
//     block may move, so a process that resets a device must not call this entry point on
//     that device again.
//   * The call returns when its work has finished (it synchronises `stream`), so that a
//     device-side failure can be reported in its return value.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "attn_flash.h"
#include "fa_launch.h"

namespace {

constexpr size_t kNoallocBytes = 4u << 20;  // 4 MiB
constexpr long long kNoallocMaxRows = 4096;  // query rows (Hq * Sq) per call
constexpr size_t kAlign = 256;
constexpr int kMaxDevices = 64;

}  // namespace

// The block itself. Host code must not pass this name to a kernel: in host code it is a
// host-side stand-in, not a device address. Kernels receive the address looked up below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocBytes];

static std::mutex g_noalloc_mu;
static void *g_noalloc_ptr[kMaxDevices];

// Device address of g_noalloc_scratch on the current device, looked up once per device.
static int noalloc_block(void **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return ATTN_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return ATTN_ERR_CUDA;
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return ATTN_OK;
}

static size_t round_up(size_t x) { return (x + kAlign - 1) & ~(kAlign - 1); }

// Bytes of the block a plan with `prow` partial rows of width D uses (status word first).
static size_t noalloc_bytes(long long prow, int D) {
    return round_up(TS_SCRATCH_CTRL_BYTES) + round_up((size_t)prow * 4) * 2 + round_up((size_t)prow * D * 4);
}

extern "C" int attn_flash_noalloc(const uint16_t *Q, const uint16_t *K, const uint16_t *V, float *O, int Hq, int Hkv,
                                  int Sq, int Sk, int D, int causal, int bk, int v_prepacked, void *stream) {
    if (bk < ATTN_BK_MIN || bk > ATTN_BK_MAX || (bk & (bk - 1)) != 0) {
        fprintf(stderr, "attn_flash_noalloc: bk=%d is invalid -- bk must be a POWER OF TWO in [%d, %d]\n", bk,
                ATTN_BK_MIN, ATTN_BK_MAX);
        abort();
    }
    if (!Q || !K || !V || !O || Hq < 1 || Hkv < 1 || Hq % Hkv != 0 || Sq < 1 || Sk < 1 || D < 1 || D > ATTN_D_MAX)
        return ATTN_ERR_ARGS;
    if ((long long)Hkv * Sk > 0x7fffffffLL) return ATTN_ERR_ARGS;  // K/V rows are indexed with int
    const long long rows = (long long)Hq * Sq;
    if (rows > kNoallocMaxRows) {
        fprintf(stderr,
                "attn_flash_noalloc: Hq*Sq = %lld query rows exceeds this entry point's limit of %lld "
                "(its fixed %zu-byte device scratch); use attn_flash_stream with a caller-owned scratch block\n",
                rows, kNoallocMaxRows, kNoallocBytes);
        return ATTN_ERR_ARGS;
    }
    if (ts_cc_major() != 10) return ATTN_ERR_NOT_SM100;
    // it synchronises the stream (the status readback), which no stream capture allows
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(static_cast<cudaStream_t>(stream), &cap) != cudaSuccess ||
        cap != cudaStreamCaptureStatusNone)
        return ATTN_ERR_ARGS;
    void *block = nullptr;
    int rc = noalloc_block(&block);
    if (rc != ATTN_OK) return rc;

    fa_problem p;
    memset(&p, 0, sizeof p);
    p.Q = Q;
    p.K = K;
    p.V = V;
    p.O = O;
    p.Hq = Hq;
    p.Hkv = Hkv;
    p.Sq = Sq;
    p.Sk = Sk;
    p.Sk_total = Sk;
    p.D = D;
    p.causal = causal ? 1 : 0;
    p.v_prepacked = v_prepacked ? 1 : 0;
    p.scale_log2 = (1.0f / sqrtf((float)D)) * 1.4426950408889634f;

    // Split plan: the makespan model of the scratch-block path, T(s) = ceil(ctas*s/SMs) *
    // (blocks/s + 1), limited to the splits whose partials fit in the fixed block.
    const int nblk = (Sk + ATTN_GPU_KEY_TILE - 1) / ATTN_GPU_KEY_TILE;
    const int ctas = ts_tc_supported(&p) ? ts_tc_ctas_per_split(&p) : (int)((rows + 7) / 8);
    const int sms = ts_num_sms() > 0 ? ts_num_sms() : 1;
    int best = 1;
    double best_t = 1e300;
    for (int s = 1; s <= nblk / 2 && s <= 256; ++s) {
        const int bps = (nblk + s - 1) / s;
        if ((nblk + bps - 1) / bps != s) continue;
        if (s > 1 && noalloc_bytes(rows * s, D) > kNoallocBytes) break;
        const double t = (double)((ctas * (long long)s + sms - 1) / sms) * ((double)bps + 1.0);
        if (t < best_t * 0.999) {
            best_t = t;
            best = s;
        }
    }
    const int bps = (nblk + best - 1) / best;
    p.nsplit = best;
    p.keys_per_split = bps * ATTN_GPU_KEY_TILE;

    // Carve: status word, then m, l, acc for rows * nsplit partial rows.
    char *b = static_cast<char *>(block);
    const long long prow = rows * p.nsplit;
    size_t off = round_up(TS_SCRATCH_CTRL_BYTES);
    p.status = reinterpret_cast<int *>(b);
    p.part_m = reinterpret_cast<float *>(b + off);
    off += round_up((size_t)prow * 4);
    p.part_l = reinterpret_cast<float *>(b + off);
    off += round_up((size_t)prow * 4);
    p.part_acc = reinterpret_cast<float *>(b + off);

    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaMemsetAsync(p.status, 0, sizeof(int), st) != cudaSuccess) return ATTN_ERR_CUDA;
    rc = ts_launch_attention(&p, stream);
    if (rc != ATTN_OK) return rc;
    int status = 0;
    if (cudaMemcpyAsync(&status, p.status, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess)
        return ATTN_ERR_CUDA;
    if (cudaStreamSynchronize(st) != cudaSuccess) return ATTN_ERR_CUDA;
    return status ? ATTN_ERR_DEVICE : ATTN_OK;
}
