// fa_diag.cu -- diagnostic entry points (include/attn_flash_diag.h) that let the tests reach
// what the attention entry points alone cannot: the state a previous kernel leaves in tensor
// memory, the kernel's exponential approximation, and the path a bounded wait takes when it
// runs out. None of them is on the attention path; none allocates device memory.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "attn_flash.h"
#include "attn_flash_diag.h"
#include "fa_launch.h"
#include "sm100_ptx.cuh"

extern "C" void ts_count_launch(void);

namespace ts {

static_assert(kDevErrTimeoutQ == ATTN_DEV_TIMEOUT_Q && kDevErrTimeoutKV == ATTN_DEV_TIMEOUT_KV &&
                  kDevErrTimeoutS == ATTN_DEV_TIMEOUT_S && kDevErrTimeoutP == ATTN_DEV_TIMEOUT_P &&
                  kDevErrTimeoutDrain == ATTN_DEV_TIMEOUT_DRAIN && kDevErrBadPage == ATTN_DEV_BAD_PAGE &&
                  kDevErrBadPos == ATTN_DEV_BAD_POS && kDevErrTimeoutPeer == ATTN_DEV_TIMEOUT_PEER,
              "the header's device codes mirror the kernels'");

// Dynamic shared memory per fill CTA: more than half an SM's 228 KB, so no two fill CTAs
// share an SM and each one allocates all 512 TMEM columns of the SM it runs on.
constexpr int kFillSmem = 120 * 1024;

// Writes `bits` into every lane and column of this SM's tensor memory, then frees it.
__global__ void __launch_bounds__(128, 1) tmem_fill_kernel(uint32_t bits) {
    __shared__ uint32_t slot;  // the launch's dynamic shared memory is only reserved, never used
    const int warp = threadIdx.x >> 5;
    if (warp == 0) {
        tmem_alloc(smem_u32(&slot), 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t base = slot + ((uint32_t)(warp * 32) << 16);  // this warp's 32 lanes
    uint32_t v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = bits;
    for (int c = 0; c < 512; c += 32) tmem_st32(base + c, v);
    tmem_wait_st();
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(slot, 512);
    }
}

// y = 2^x by the attention kernel's own exponentials: method 0 the FMA-pipe polynomial
// (exp2_fma2, two values per call), method 1 the MUFU ex2.approx.ftz.
__global__ void exp2_diag_kernel(const float *x, float *y, int n, int method) {
    const int i = 2 * (int)(blockIdx.x * blockDim.x + threadIdx.x);
    if (i >= n) return;
    const float2 v = make_float2(x[i], i + 1 < n ? x[i + 1] : 0.f);
    float2 r;
    if (method == 0) {
        r = exp2_fma2(v);
    } else {
        r.x = ex2(v.x);
        r.y = ex2(v.y);
    }
    y[i] = r.x;
    if (i + 1 < n) y[i + 1] = r.y;
}

}  // namespace ts

extern "C" int ts_launch_tc_noq(const fa_problem *P, void *stream);

extern "C" int attn_diag_fill_tmem(uint32_t bits, void *stream) {
    if (ts_cc_major() != 10) return ATTN_ERR_NOT_SM100;
    const int sms = ts_num_sms() > 0 ? ts_num_sms() : 1;
    if (cudaFuncSetAttribute(ts::tmem_fill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, ts::kFillSmem) !=
        cudaSuccess)
        return ATTN_ERR_CUDA;
    // several CTAs per SM in turn, so every SM's tensor memory is written at least once
    ts::tmem_fill_kernel<<<4 * sms, 128, ts::kFillSmem, static_cast<cudaStream_t>(stream)>>>(bits);
    if (cudaGetLastError() != cudaSuccess) return ATTN_ERR_CUDA;
    ts_count_launch();
    return ATTN_OK;
}

extern "C" int attn_diag_exp2(const float *x, float *y, int n, int method, void *stream) {
    if (!x || !y || n < 0 || (method != ATTN_DIAG_EXP2_POLY && method != ATTN_DIAG_EXP2_MUFU)) return ATTN_ERR_ARGS;
    if (ts_cc_major() != 10) return ATTN_ERR_NOT_SM100;
    if (n == 0) return ATTN_OK;
    const int pairs = (n + 1) / 2;
    ts::exp2_diag_kernel<<<(pairs + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, n, method);
    if (cudaGetLastError() != cudaSuccess) return ATTN_ERR_CUDA;
    ts_count_launch();
    return ATTN_OK;
}

extern "C" int attn_diag_wait_timeout(const uint16_t *Q, const uint16_t *K, const uint16_t *V, float *O, int Hq,
                                      int Hkv, int Sq, int Sk, void *scratch, void *stream) {
    if (!Q || !K || !V || !O || !scratch || Hq < 1 || Hkv < 1 || Hq % Hkv != 0 || Sq < 1 || Sk < 1)
        return ATTN_ERR_ARGS;
    if ((long long)(Hq / Hkv) * Sq > 128 || (long long)Hkv * Sk > 0x7fffffffLL) return ATTN_ERR_ARGS;
    if (((uintptr_t)Q | (uintptr_t)K | (uintptr_t)V | (uintptr_t)O | (uintptr_t)scratch) & 15u) return ATTN_ERR_ALIGN;
    if (ts_cc_major() != 10) return ATTN_ERR_NOT_SM100;
    fa_problem p;
    memset(&p, 0, sizeof p);
    p.Q = Q;
    p.K = K;
    p.V = V;
    p.O = O;
    p.Hq = Hq;
    p.Hkv = Hkv;
    p.Sq = Sq;
    p.Sk = p.Sk_total = Sk;
    p.D = 128;
    p.scale_log2 = 0.08838834764831845f * 1.4426950408889634f;
    p.nsplit = 1;
    p.keys_per_split = ((Sk + ATTN_GPU_KEY_TILE - 1) / ATTN_GPU_KEY_TILE) * ATTN_GPU_KEY_TILE;
    p.status = static_cast<int *>(scratch);  // the status word leads the scratch block
    int rc = ts_clear_status(p.status, stream);
    if (rc != ATTN_OK) return rc;
    return ts_launch_tc_noq(&p, stream);
}
