// fa_aux.cu -- the CUDA-core side of the attention path:
//   * fa_simt_kernel: the general-shape kernel (any head_dim 1..256, unaligned pointers,
//     V^T with Sk not a multiple of 8). One warp per query row; same online-softmax state
//     as flash.c:518-580 (bf16-rounded P, l summing the unrounded exponentials, zero row
//     when no key is live), one key at a time.
//   * fa_combine_kernel: merges split-KV partials (m, l, acc) into O, or into one partial.
//   * status-word helpers and the top-level launcher called by the C host layer.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <atomic>

#include "attn_flash.h"
#include "fa_launch.h"
#include "sm100_ptx.cuh"

extern "C" int ts_launch_tc(const fa_problem *P, void *stream);

static std::atomic<unsigned long long> g_kernel_launches{0};

extern "C" void ts_count_launch(void) { g_kernel_launches.fetch_add(1, std::memory_order_relaxed); }

extern "C" unsigned long long attn_flash_kernel_launches(void) {
    return g_kernel_launches.load(std::memory_order_relaxed);
}

static std::atomic<unsigned> g_status_gen{0};

extern "C" unsigned ts_next_status_gen(void) {
    unsigned g;
    do {
        g = g_status_gen.fetch_add(1, std::memory_order_relaxed) + 1;
    } while (g == 0);
    return g;
}

namespace ts {

__device__ __forceinline__ float ex2f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) { return __uint_as_float(((uint32_t)b) << 16); }

struct SimtParams {
    const uint16_t *Q, *K, *V;
    float *O, *part_m, *part_l, *part_acc;
    int Hq, Hkv, Sq, Sk, Sk_total, k_begin, D, causal, v_prepacked;
    int keys_per_split, partial, o_bf16;
    float scale_log2;
};

constexpr int kSimtMaxU = ATTN_D_MAX / 32;  // columns per lane

__global__ void __launch_bounds__(256) fa_simt_kernel(const SimtParams p) {
    const int lane = threadIdx.x & 31;
    const long long total_rows = (long long)p.Hq * p.Sq;
    const long long grow = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (grow >= total_rows) return;
    const int split = blockIdx.y;
    const int h = (int)(grow / p.Sq), i = (int)(grow % p.Sq);
    const int kv = h / (p.Hq / p.Hkv);
    const int kb0 = split * p.keys_per_split;
    const int kb1 = min(p.Sk, kb0 + p.keys_per_split);
    long long lim = p.causal ? ((long long)p.Sk_total - p.Sq + i - p.k_begin) : (long long)(p.Sk - 1);
    const int kend = (int)max((long long)kb0, min((long long)kb1, lim + 1));

    float q[kSimtMaxU], acc[kSimtMaxU];
#pragma unroll
    for (int u = 0; u < kSimtMaxU; ++u) {
        const int c = lane + 32 * u;
        q[u] = (c < p.D) ? bf16_bits_to_f32(p.Q[grow * p.D + c]) : 0.f;
        acc[u] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    const uint16_t *Kh = p.K + (size_t)kv * p.Sk * p.D;
    const uint16_t *Vh = p.V + (size_t)kv * p.Sk * p.D;
    for (int k = kb0; k < kend; ++k) {
        float part = 0.f;
#pragma unroll
        for (int u = 0; u < kSimtMaxU; ++u) {
            const int c = lane + 32 * u;
            if (c < p.D) part = fmaf(q[u], bf16_bits_to_f32(Kh[(size_t)k * p.D + c]), part);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        const float s = part * p.scale_log2;
        if (s > m) {
            const float alpha = (m == -INFINITY) ? 0.f : ex2f(m - s);
            l *= alpha;
#pragma unroll
            for (int u = 0; u < kSimtMaxU; ++u) acc[u] *= alpha;
            m = s;
        }
        const float e = ex2f(s - m);
        l += e;
        const float pb = __bfloat162float(__float2bfloat16_rn(e));
#pragma unroll
        for (int u = 0; u < kSimtMaxU; ++u) {
            const int c = lane + 32 * u;
            if (c < p.D) {
                const float v = p.v_prepacked ? bf16_bits_to_f32(Vh[(size_t)c * p.Sk + k])
                                              : bf16_bits_to_f32(Vh[(size_t)k * p.D + c]);
                acc[u] = fmaf(pb, v, acc[u]);
            }
        }
    }
    if (p.partial) {
        const size_t pr = (size_t)split * total_rows + grow;
        if (lane == 0) {
            p.part_m[pr] = m;
            p.part_l[pr] = l;
        }
#pragma unroll
        for (int u = 0; u < kSimtMaxU; ++u) {
            const int c = lane + 32 * u;
            if (c < p.D) p.part_acc[pr * p.D + c] = acc[u];
        }
    } else {
        const float inv = (l > 0.f) ? 1.f / l : 0.f;
#pragma unroll
        for (int u = 0; u < kSimtMaxU; ++u) {
            const int c = lane + 32 * u;
            if (c < p.D) {
                if (p.o_bf16)
                    reinterpret_cast<uint16_t *>(p.O)[grow * p.D + c] = (uint16_t)f32_to_bf16_bits(acc[u] * inv);
                else
                    p.O[grow * p.D + c] = acc[u] * inv;
            }
        }
    }
}

// One warp per row: O[r] = sum_s 2^(m_s - m*) acc_s[r] / sum_s 2^(m_s - m*) l_s[r] (zero row
// when every l_s is 0). With out_m != nullptr the merged partial (m*, L, unnormalised acc) is
// written instead. The lanes read the parts' m and l in parallel and reduce them with shuffles;
// then lane i owns columns 4i..4i+3 (VEC, D % 4 == 0) or column i of every 32 (scalar), and the
// loads of all parts are independent, so a row's reads are in flight together.
template <bool VEC>
__global__ void __launch_bounds__(256) fa_combine_kernel(const float *__restrict__ m, const float *__restrict__ l,
                                                         const float *__restrict__ acc, int nparts, int rows, int D,
                                                         size_t ps_ml, size_t ps_acc, float *__restrict__ out,
                                                         float *__restrict__ out_m, float *__restrict__ out_l,
                                                         int out_bf16) {
    pdl_wait();  // the partials come from the previous grid of the stream
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= rows) return;
    float mx = -INFINITY;
    for (int s = lane; s < nparts; s += 32) mx = fmaxf(mx, m[(size_t)s * ps_ml + r]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float L = 0.f;
    for (int s = lane; s < nparts; s += 32) {
        const float ms = m[(size_t)s * ps_ml + r];
        if (ms != -INFINITY) L = fmaf(ex2f(ms - mx), l[(size_t)s * ps_ml + r], L);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    const float inv = out_m ? 1.f : ((L > 0.f) ? 1.f / L : 0.f);
    if (VEC) {
        for (int c = 4 * lane; c < D; c += 128) {
            float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
            for (int s = 0; s < nparts; ++s) {
                const float ms = m[(size_t)s * ps_ml + r];
                const float w = (ms != -INFINITY) ? ex2f(ms - mx) : 0.f;
                const float4 x = *reinterpret_cast<const float4 *>(acc + (size_t)s * ps_acc + (size_t)r * D + c);
                a.x = fmaf(w, x.x, a.x);
                a.y = fmaf(w, x.y, a.y);
                a.z = fmaf(w, x.z, a.z);
                a.w = fmaf(w, x.w, a.w);
            }
            if (out_bf16)  // out holds bf16 bits; D % 4 == 0 keeps the 8-byte store aligned
                *reinterpret_cast<uint2 *>(reinterpret_cast<uint16_t *>(out) + (size_t)r * D + c) =
                    make_uint2(f32_to_bf16_bits(a.x * inv) | (f32_to_bf16_bits(a.y * inv) << 16),
                               f32_to_bf16_bits(a.z * inv) | (f32_to_bf16_bits(a.w * inv) << 16));
            else
                *reinterpret_cast<float4 *>(out + (size_t)r * D + c) =
                    make_float4(a.x * inv, a.y * inv, a.z * inv, a.w * inv);
        }
    } else {
        for (int c = lane; c < D; c += 32) {
            float a = 0.f;
#pragma unroll 4
            for (int s = 0; s < nparts; ++s) {
                const float ms = m[(size_t)s * ps_ml + r];
                const float w = (ms != -INFINITY) ? ex2f(ms - mx) : 0.f;
                a = fmaf(w, acc[(size_t)s * ps_acc + (size_t)r * D + c], a);
            }
            if (out_bf16)
                reinterpret_cast<uint16_t *>(out)[(size_t)r * D + c] = (uint16_t)f32_to_bf16_bits(a * inv);
            else
                out[(size_t)r * D + c] = a * inv;
        }
    }
    if (out_m && lane == 0) {
        out_m[r] = mx;
        out_l[r] = L;
    }
}

// Few parts (2..4: a prefill's last-wave split, most decode splits), normalised output: one
// thread per (row, 4 columns). A thread's loads -- every part's m, l and its 4 columns of acc --
// do not depend on one another, so they are all in flight at once (one memory round trip
// instead of reduce-then-load); the m and l loads of a warp's 32 lanes hit one address each.
template <int NP>
__global__ void __launch_bounds__(256) fa_combine_few(const float *__restrict__ m, const float *__restrict__ l,
                                                      const float *__restrict__ acc, int rows, int D, size_t ps_ml,
                                                      size_t ps_acc, float *__restrict__ out, int out_bf16) {
    pdl_wait();  // the partials come from the previous grid of the stream
    pdl_trigger();
    const int cpr = D >> 2;  // float4 chunks per row (D % 4 == 0)
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long r = idx / cpr;
    if (r >= rows) return;
    const int c = (int)(idx - r * cpr) * 4;
    float ms[NP], ls[NP];
    float4 a[NP];
#pragma unroll
    for (int s = 0; s < NP; ++s) {
        ms[s] = m[(size_t)s * ps_ml + r];
        ls[s] = l[(size_t)s * ps_ml + r];
        a[s] = *reinterpret_cast<const float4 *>(acc + (size_t)s * ps_acc + (size_t)r * D + c);
    }
    float mx = ms[0];
#pragma unroll
    for (int s = 1; s < NP; ++s) mx = fmaxf(mx, ms[s]);
    float L = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int s = 0; s < NP; ++s) {
        const float w = (ms[s] != -INFINITY) ? ex2f(ms[s] - mx) : 0.f;
        L = fmaf(w, ls[s], L);
        o.x = fmaf(w, a[s].x, o.x);
        o.y = fmaf(w, a[s].y, o.y);
        o.z = fmaf(w, a[s].z, o.z);
        o.w = fmaf(w, a[s].w, o.w);
    }
    const float inv = (L > 0.f) ? 1.f / L : 0.f;
    o = make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
    if (out_bf16)
        *reinterpret_cast<uint2 *>(reinterpret_cast<uint16_t *>(out) + (size_t)r * D + c) =
            make_uint2(f32_to_bf16_bits(o.x) | (f32_to_bf16_bits(o.y) << 16),
                       f32_to_bf16_bits(o.z) | (f32_to_bf16_bits(o.w) << 16));
    else
        *reinterpret_cast<float4 *>(out + (size_t)r * D + c) = o;
}

}  // namespace ts

// Per-device attribute caches. Host threads may call the library concurrently (one scratch
// block each), so the cache slots are atomics; two threads filling a slot store the same value.
static int cached_device_attr(std::atomic<int> (&cache)[64], cudaDeviceAttr attr, int on_error) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return on_error;
    if (dev >= 0 && dev < 64) {
        const int v = cache[dev].load(std::memory_order_relaxed);
        if (v) return v;
    }
    int v = 0;
    if (cudaDeviceGetAttribute(&v, attr, dev) != cudaSuccess) return on_error;
    if (dev >= 0 && dev < 64) cache[dev].store(v, std::memory_order_relaxed);
    return v;
}

extern "C" int ts_num_sms(void) {
    static std::atomic<int> cached[64];
    return cached_device_attr(cached, cudaDevAttrMultiProcessorCount, 0);
}

extern "C" int ts_cc_major(void) {
    static std::atomic<int> cached[64];
    return cached_device_attr(cached, cudaDevAttrComputeCapabilityMajor, -1);
}

// Launches with programmatic dependent launch allowed: the grid may start while the previous
// grid of the stream finishes; the kernel's pdl_wait() orders its memory accesses after it.
template <typename... KArgs, typename... Args>
static int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...) != cudaSuccess) return ATTN_ERR_CUDA;
    ts_count_launch();
    return ATTN_OK;
}

extern "C" int ts_launch_combine_strided(const float *m, const float *l, const float *acc, int nparts, int rows,
                                         int D, size_t ps_ml, size_t ps_acc, float *O, float *out_m, float *out_l,
                                         int out_bf16, void *stream) {
    if (rows <= 0) return ATTN_OK;
    const int warps = 8;
    dim3 grid((rows + warps - 1) / warps);
    const bool vec = (D % 4 == 0) && (ps_acc % 4 == 0) && ((((uintptr_t)acc) | ((uintptr_t)O)) & 15u) == 0;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (vec && !out_m && nparts >= 2 && nparts <= 4) {
        const long long threads = (long long)rows * (D / 4);
        const dim3 g((unsigned)((threads + 255) / 256));
        if (nparts == 2) return launch_pdl(ts::fa_combine_few<2>, g, dim3(256), st, m, l, acc, rows, D, ps_ml, ps_acc,
                                           O, out_bf16);
        if (nparts == 3) return launch_pdl(ts::fa_combine_few<3>, g, dim3(256), st, m, l, acc, rows, D, ps_ml, ps_acc,
                                           O, out_bf16);
        return launch_pdl(ts::fa_combine_few<4>, g, dim3(256), st, m, l, acc, rows, D, ps_ml, ps_acc, O, out_bf16);
    }
    if (vec)
        return launch_pdl(ts::fa_combine_kernel<true>, grid, dim3(32 * warps), st, m, l, acc, nparts, rows, D, ps_ml,
                          ps_acc, O, out_m, out_l, out_bf16);
    return launch_pdl(ts::fa_combine_kernel<false>, grid, dim3(32 * warps), st, m, l, acc, nparts, rows, D, ps_ml,
                      ps_acc, O, out_m, out_l, out_bf16);
}

extern "C" int ts_launch_combine(const float *m, const float *l, const float *acc, int nparts, int rows, int D,
                                 float *O, float *out_m, float *out_l, int out_bf16, void *stream) {
    return ts_launch_combine_strided(m, l, acc, nparts, rows, D, (size_t)rows, (size_t)rows * D, O, out_m, out_l,
                                     out_bf16, stream);
}

static int launch_simt(const fa_problem *P, void *stream, int partial) {
    ts::SimtParams s;
    s.Q = P->Q;
    s.K = P->K;
    s.V = P->V;
    s.O = P->O;
    s.part_m = P->part_m;
    s.part_l = P->part_l;
    s.part_acc = P->part_acc;
    s.Hq = P->Hq;
    s.Hkv = P->Hkv;
    s.Sq = P->Sq;
    s.Sk = P->Sk;
    s.Sk_total = P->Sk_total;
    s.k_begin = P->k_begin;
    s.D = P->D;
    s.causal = P->causal;
    s.v_prepacked = P->v_prepacked;
    s.keys_per_split = P->keys_per_split;
    s.partial = partial;
    s.o_bf16 = P->o_bf16;
    s.scale_log2 = P->scale_log2;
    const long long rows = (long long)P->Hq * P->Sq;
    const int warps = 8;
    dim3 grid((unsigned)((rows + warps - 1) / warps), P->nsplit);
    ts::fa_simt_kernel<<<grid, 32 * warps, 0, static_cast<cudaStream_t>(stream)>>>(s);
    if (cudaGetLastError() != cudaSuccess) return ATTN_ERR_CUDA;
    ts_count_launch();
    return ATTN_OK;
}

extern "C" int ts_launch_attention_pieces(const fa_problem *P, void *stream) {
    return ts_tc_supported(P) ? ts_launch_tc(P, stream) : launch_simt(P, stream, 1);
}

extern "C" int ts_launch_attention(const fa_problem *P, void *stream) {
    const bool tc = ts_tc_supported(P) != 0;
    int rc = tc ? ts_launch_tc(P, stream) : launch_simt(P, stream, (P->nsplit > 1 || P->write_partials) ? 1 : 0);
    if (rc != ATTN_OK || P->nsplit <= 1) return rc;
    // merge the key pieces of the split rows [base, Hq*Sq) (all rows on the general path)
    const int rows = P->Hq * P->Sq;
    const int base = tc ? P->row_base : 0;
    const int obf = P->write_partials ? 0 : P->o_bf16;
    float *out = P->write_partials ? P->out_acc + (size_t)base * P->D
                                   : (obf ? reinterpret_cast<float *>(reinterpret_cast<uint16_t *>(P->O) +
                                                                      (size_t)base * P->D)
                                          : P->O + (size_t)base * P->D);
    return ts_launch_combine(P->part_m, P->part_l, P->part_acc, P->nsplit, rows - base, P->D, out,
                             P->write_partials ? P->out_m + base : nullptr,
                             P->write_partials ? P->out_l + base : nullptr, obf, stream);
}

extern "C" int ts_clear_status(int *status, void *stream) {
    return cudaMemsetAsync(status, 0, sizeof(int), static_cast<cudaStream_t>(stream)) == cudaSuccess ? ATTN_OK
                                                                                                    : ATTN_ERR_CUDA;
}

extern "C" int ts_read_status(int *status, void *stream, int *value) {
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaStreamSynchronize(st) != cudaSuccess) return ATTN_ERR_CUDA;
    int v = 0;
    if (cudaMemcpy(&v, status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return ATTN_ERR_CUDA;
    if (v != 0 && cudaMemset(status, 0, sizeof(int)) != cudaSuccess) return ATTN_ERR_CUDA;
    if (value) *value = v;
    return ATTN_OK;
}
