// qkv_rope.cu -- the producer upstream of the attention kernels: split a fused QKV projection,
// apply the per-head RMSNorm and the rotary embedding to q and k heads, and write Q in the
// attention's [B*Hq][S][D] layout and K/V into a contiguous or paged key cache -- one pass over
// HBM. Byte work, so no tensor cores; the design goal is to keep HBM busy in both directions.
//
// Pipeline (three persistent CTAs per SM: 72 registers, a 64 KB ring each -- occupancy is
// what hides the per-token load latency). The input is one flat array of head vectors
// (D bf16 each), so it is cut into 16 KB chunks of whole vectors. One producer thread streams
// the CTA's chunks into a ring of shared-memory stages with untiled bulk copies
// (cp.async.bulk, completion counted on an mbarrier per stage): the reads stay in flight no
// matter how long the consumers take. Eight consumer warps take each stage (the norm weights
// sit in shared memory as fp32, loaded once per CTA): a head vector is
// handled by G = D/16 lanes, 16 elements (two 16-byte shared loads) each; results go straight
// to global memory with 16-byte stores. Each warp releases the stage as soon as its bytes are
// in registers. A CTA streams one contiguous run of chunks, so a lane meets each token once in
// a row: the per-token work (position, destination rows, validity, the lane's cos/sin slice)
// runs only when the token changes, and the per-vector work is the arithmetic itself. The
// kernel is specialised on D, the pairing and the cache kind. Every wait is bounded.
//
// A lane owns both members of each pair it rotates -- for the rotate-half form elements
// [8li, 8li+8) and [rot/2 + 8li, +8), for the interleaved form 16 consecutive elements -- so the
// rotation needs no shuffle; only the norm's sum of squares crosses lanes (log2(D/16) shuffles).
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "attn_qkv_rope.h"
#include "fa_launch.h"
#include "sm100_ptx.cuh"

extern "C" void ts_count_launch(void);

namespace ts {

namespace {

constexpr int kRopeConsumerWarps = 8;
constexpr int kRopeThreads = 32 * (kRopeConsumerWarps + 1);  // + the producer warp
constexpr int kRopeChunk = 16384;                            // bytes per stage
constexpr int kRopeStages = 4;  // 64 KB ring: three CTAs per SM
// ring, then full/empty barriers, then the two norm weights as fp32 [2][ATTN_D_MAX]
constexpr int kRopeSmem = kRopeStages * kRopeChunk + 2 * kRopeStages * 8 + 2 * ATTN_D_MAX * 4;

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ void unpack8(uint4 w, float *f) {
    f[0] = bf16_lo(w.x), f[1] = bf16_hi(w.x), f[2] = bf16_lo(w.y), f[3] = bf16_hi(w.y);
    f[4] = bf16_lo(w.z), f[5] = bf16_hi(w.z), f[6] = bf16_lo(w.w), f[7] = bf16_hi(w.w);
}

__device__ __forceinline__ uint4 pack8(const float *x) {
    return make_uint4(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]), pack_bf16x2(x[4], x[5]),
                      pack_bf16x2(x[6], x[7]));
}

// Everything about the token a lane is working on that does not depend on the head: where its
// q rows and cache rows go, whether it is valid, and the lane's cos/sin slice of its position.
// Recomputed only when the lane moves to another token.
struct TokenState {
    long long t;         // token index (-1: none yet)
    uint16_t *q_base;    // Q row of head 0
    long long kv_off;    // K/V cache row of kv head 0, elements from the cache base
    long long q_stride;  // elements between consecutive q heads (S*D)
    long long kv_stride; // elements between consecutive kv heads
    bool ok;
    float c[8], sn[8];
};

template <int D, bool PAGED>
__device__ __forceinline__ void load_token(const ts_rope_problem &a, TokenState &T, long long t, int li,
                                           bool rot_lane) {
    T.t = t;
    const int p = __ldg(a.positions + t);
    const int b = (int)((uint32_t)t / (uint32_t)a.S);
    const int s = (int)((uint32_t)t - (uint32_t)b * (uint32_t)a.S);
    bool ok = p >= 0 && (a.rot == 0 || p < a.max_pos);
    int code = kDevErrBadPos;
    T.q_stride = (long long)a.S * D;
    T.q_base = a.Q + ((long long)b * a.Hq * a.S + s) * D;
    if (PAGED) {
        const int lp = ok ? p / a.page_size : 0;
        ok = ok && lp < a.max_pages;
        int page = ok ? __ldg(a.block_table + (long long)b * a.max_pages + lp) : 0;
        if (ok && (page < 0 || page >= a.num_pages)) {
            ok = false;
            code = kDevErrBadPage;
        }
        T.kv_stride = (long long)a.page_size * D;
        T.kv_off = ((long long)page * a.Hkv * a.page_size + (p - lp * a.page_size)) * D;
    } else {
        ok = ok && p < a.cache_len;
        T.kv_stride = (long long)a.cache_len * D;
        T.kv_off = ((long long)b * a.Hkv * a.cache_len + p) * D;
    }
    T.ok = ok;
    if (!ok && li == 0) atomicOr(a.status, code);
    if (ok && rot_lane) {
        const float *row = a.cos_sin + (long long)p * a.rot + 8 * li;
        const float *srow = row + (a.rot >> 1);
        const float4 c0 = __ldg(reinterpret_cast<const float4 *>(row));
        const float4 c1 = __ldg(reinterpret_cast<const float4 *>(row + 4));
        const float4 s0 = __ldg(reinterpret_cast<const float4 *>(srow));
        const float4 s1 = __ldg(reinterpret_cast<const float4 *>(srow + 4));
        T.c[0] = c0.x, T.c[1] = c0.y, T.c[2] = c0.z, T.c[3] = c0.w;
        T.c[4] = c1.x, T.c[5] = c1.y, T.c[6] = c1.z, T.c[7] = c1.w;
        T.sn[0] = s0.x, T.sn[1] = s0.y, T.sn[2] = s0.z, T.sn[3] = s0.w;
        T.sn[4] = s1.x, T.sn[5] = s1.y, T.sn[6] = s1.z, T.sn[7] = s1.w;
    }
}

// The two 8-element chunks a lane owns, as element offsets into the head vector. Rotate-half
// lanes below rot/16 own elements [8li, 8li+8) and their partners [rot/2 + 8li, +8), so a
// rotation never leaves the lane; the remaining lanes own 16 pass-through elements after rot.
// The interleaved pairing keeps 16 consecutive elements per lane. Either way the lane's
// frequencies are 8li .. 8li+7 when it rotates.
template <bool NEOX>
__device__ __forceinline__ void lane_chunks(const ts_rope_problem &a, int li, int &oa, int &ob, bool &rot_lane) {
    if (NEOX) {
        rot_lane = li < (a.rot >> 4);
        oa = rot_lane ? 8 * li : a.rot + 16 * (li - (a.rot >> 4));
        ob = rot_lane ? (a.rot >> 1) + 8 * li : oa + 8;
    } else {
        rot_lane = 16 * li < a.rot;
        oa = 16 * li;
        ob = oa + 8;
    }
}

template <int D, bool NEOX, bool PAGED>
__global__ void __maxnreg__(72) qkv_rope_kernel(ts_rope_problem a) {
    constexpr int G = D / 16;                        // lanes per head vector, 16 elements each
    constexpr int CV = kRopeChunk / (D * 2);         // head vectors per stage
    constexpr int NG = kRopeConsumerWarps * 32 / G;  // lane groups of the consumers
    constexpr int PER = CV / NG;                     // vectors per group and stage
    constexpr unsigned FULL = 0xffffffffu;
    static_assert(PER * NG == CV, "stage must split evenly over the lane groups");
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int abort_flag;
    const uint32_t ring = smem_u32(smem);
    const uint32_t full0 = ring + kRopeStages * kRopeChunk;
    const uint32_t empty0 = full0 + 8 * kRopeStages;
    float *wq = reinterpret_cast<float *>(smem + kRopeStages * kRopeChunk + 16 * kRopeStages);
    float *wk = wq + ATTN_D_MAX;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Each CTA streams one contiguous run of chunks, so consecutive stages continue a token.
    const long long n_chunks = (a.n_vec + CV - 1) / CV;
    const long long per_cta = n_chunks / gridDim.x, extra = n_chunks % gridDim.x;
    const long long c_begin = blockIdx.x * per_cta + (blockIdx.x < extra ? blockIdx.x : extra);
    const long long c_end = c_begin + per_cta + (blockIdx.x < extra ? 1 : 0);

    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int st = 0; st < kRopeStages; ++st) {
            mbar_init(full0 + 8 * st, 1);
            mbar_init(empty0 + 8 * st, kRopeConsumerWarps);
        }
        fence_mbar_init();
    }
    for (int e = threadIdx.x; e < D; e += blockDim.x) {
        wq[e] = a.q_norm_w ? bf16_lo(__ldg(a.q_norm_w + e)) : 1.f;
        wk[e] = a.k_norm_w ? bf16_lo(__ldg(a.k_norm_w + e)) : 1.f;
    }
    __syncthreads();

    if (warp == kRopeConsumerWarps) {  // producer
        if (lane == 0) {
            long long k = 0;
            for (long long c = c_begin; c < c_end; ++c, ++k) {
                const int st = (int)(k % kRopeStages);
                const uint32_t round = (uint32_t)(k / kRopeStages);
                if (round > 0 && !mbar_wait(empty0 + 8 * st, (round - 1) & 1u, &abort_flag, a.status,
                                            kDevErrTimeoutKV))
                    break;
                const long long v0 = c * CV;
                const long long nv = a.n_vec - v0 < CV ? a.n_vec - v0 : CV;
                const uint32_t bytes = (uint32_t)(nv * D * 2);
                mbar_expect_tx(full0 + 8 * st, bytes);
                bulk_load(ring + st * kRopeChunk, a.qkv + v0 * D, bytes, full0 + 8 * st);
            }
            // Copies still in flight must land before the CTA exits (the consumers waited for
            // all of them unless the CTA is aborting): the last issue of each stage.
            for (long long j = (k > kRopeStages ? k - kRopeStages : 0); j < k; ++j) {
                const int st = (int)(j % kRopeStages);
                volatile int never = 0;
                if (!mbar_wait(full0 + 8 * st, (uint32_t)(j / kRopeStages) & 1u, &never, a.status,
                               kDevErrTimeoutDrain))
                    break;
            }
        }
        return;
    }

    // consumers: group grp takes vectors grp, grp + NG, ... of each stage
    const int li = lane % G;
    const int grp = threadIdx.x / G;  // 0 .. NG-1
    const int Htot = a.Hq + 2 * a.Hkv;
    int oa, ob;
    bool rot_lane;
    lane_chunks<NEOX>(a, li, oa, ob, rot_lane);
    const bool has_qn = a.q_norm_w != nullptr, has_kn = a.k_norm_w != nullptr;
    TokenState T;
    T.t = -1;
    // (token, head) of this group's next vector; starts at vector c_begin*CV + grp
    long long t = 0;
    int h = 0;
    {
        const long long v = c_begin * CV + grp;
        t = v / Htot;
        h = (int)(v - t * Htot);
    }

    long long k = 0;
    for (long long c = c_begin; c < c_end; ++c, ++k) {
        const int st = (int)(k % kRopeStages);
        if (!mbar_wait(full0 + 8 * st, (uint32_t)(k / kRopeStages) & 1u, &abort_flag, a.status, kDevErrTimeoutKV))
            break;
        const uint8_t *stage = smem + st * kRopeChunk + (size_t)grp * (D * 2);
        const long long vbase = c * CV + grp;
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            const uint4 raj = *reinterpret_cast<const uint4 *>(stage + (size_t)j * NG * (D * 2) + oa * 2);
            const uint4 rbj = *reinterpret_cast<const uint4 *>(stage + (size_t)j * NG * (D * 2) + ob * 2);
            if (j == PER - 1) {  // the stage's last bytes are in registers: release it
                __syncwarp();
                if (lane == 0) mbar_arrive(empty0 + 8 * st);
            }
            const bool act = vbase + (long long)j * NG < a.n_vec;
            if (act && t != T.t) load_token<D, PAGED>(a, T, t, li, rot_lane);
            const int kind = h < a.Hq ? 0 : (h < a.Hq + a.Hkv ? 1 : 2);  // q, k, v head
            float x[16];
            unpack8(raj, x);
            unpack8(rbj, x + 8);
            // RMSNorm: every group reduces (the shuffles need the full warp); only q/k heads
            // with a weight apply it. 1/D is exact (D is a power of two).
            float ss = 0.f;
#pragma unroll
            for (int e = 0; e < 16; ++e) ss = fmaf(x[e], x[e], ss);
#pragma unroll
            for (int o = G / 2; o >= 1; o >>= 1) ss += __shfl_xor_sync(FULL, ss, o, G);
            if (kind == 0 ? has_qn : (kind == 1 && has_kn)) {
                const float r = rsqrtf(__fmaf_rn(ss, 1.0f / (float)D, a.eps));
                const float *w = kind == 0 ? wq : wk;
                float wv[16];
                *reinterpret_cast<float4 *>(wv) = *reinterpret_cast<const float4 *>(w + oa);
                *reinterpret_cast<float4 *>(wv + 4) = *reinterpret_cast<const float4 *>(w + oa + 4);
                *reinterpret_cast<float4 *>(wv + 8) = *reinterpret_cast<const float4 *>(w + ob);
                *reinterpret_cast<float4 *>(wv + 12) = *reinterpret_cast<const float4 *>(w + ob + 4);
#pragma unroll
                for (int e = 0; e < 16; ++e) x[e] = __fmul_rn(__fmul_rn(x[e], r), wv[e]);
            }
            if (kind < 2 && rot_lane) {
                if (NEOX) {  // pairs (x[e], x[8 + e]) at frequency 8li + e
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const float u = x[e], w = x[8 + e];
                        x[e] = __fsub_rn(__fmul_rn(u, T.c[e]), __fmul_rn(w, T.sn[e]));
                        x[8 + e] = __fadd_rn(__fmul_rn(w, T.c[e]), __fmul_rn(u, T.sn[e]));
                    }
                } else {  // pairs (x[2e], x[2e + 1]) at frequency 8li + e
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const float u = x[2 * e], w = x[2 * e + 1];
                        x[2 * e] = __fsub_rn(__fmul_rn(u, T.c[e]), __fmul_rn(w, T.sn[e]));
                        x[2 * e + 1] = __fadd_rn(__fmul_rn(w, T.c[e]), __fmul_rn(u, T.sn[e]));
                    }
                }
            }
            if (act && T.ok) {
                uint16_t *dst = kind == 0   ? T.q_base + h * T.q_stride
                                : kind == 1 ? a.K + T.kv_off + (h - a.Hq) * T.kv_stride
                                            : a.V + T.kv_off + (h - a.Hq - a.Hkv) * T.kv_stride;
                *reinterpret_cast<uint4 *>(dst + oa) = kind < 2 ? pack8(x) : raj;  // v heads keep their bits
                *reinterpret_cast<uint4 *>(dst + ob) = kind < 2 ? pack8(x + 8) : rbj;
            }
            h += NG;
            while (h >= Htot) {
                h -= Htot;
                ++t;
            }
        }
    }
}

// cos_sin[p][i] = cos(p * theta^(-2i/rot)), cos_sin[p][rot/2 + i] = the sine; double precision,
// one rounding to fp32.
__global__ void rope_table_kernel(float *cs, int max_pos, int rot, double theta) {
    const int half = rot >> 1;
    const long long n = (long long)max_pos * half;
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
        const long long p = e / half;
        const int i = (int)(e - p * half);
        const double f = pow(theta, -2.0 * i / rot);
        double sv, cv;
        sincos((double)p * f, &sv, &cv);
        cs[p * rot + i] = (float)cv;
        cs[p * rot + half + i] = (float)sv;
    }
}

}  // namespace

}  // namespace ts

// Once per device and kernel instance: opt in to the ring's shared memory and read how many CTAs
// fit on an SM (0: not set up yet). Concurrent first calls both do the same work.
template <int D, bool NEOX, bool PAGED>
static int rope_resident() {
    static std::atomic<int> resident[64];
    auto kern = ts::qkv_rope_kernel<D, NEOX, PAGED>;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return -1;
    const bool cached = dev >= 0 && dev < 64;
    if (cached) {
        const int r = resident[dev].load(std::memory_order_acquire);
        if (r > 0) return r;
    }
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, ts::kRopeSmem) != cudaSuccess)
        return -1;
    int r = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&r, kern, ts::kRopeThreads, ts::kRopeSmem) != cudaSuccess ||
        r < 1)
        r = 1;
    if (cached) resident[dev].store(r, std::memory_order_release);
    return r;
}

template <int D>
static int pick_rope_resident(const ts_rope_problem *p) {
    const bool neox = p->style == ATTN_ROPE_NEOX, paged = p->block_table != nullptr;
    if (neox) return paged ? rope_resident<D, true, true>() : rope_resident<D, true, false>();
    return paged ? rope_resident<D, false, true>() : rope_resident<D, false, false>();
}

template <int D>
static void (*pick_rope_kernel(const ts_rope_problem *p))(ts_rope_problem) {
    const bool neox = p->style == ATTN_ROPE_NEOX, paged = p->block_table != nullptr;
    if (neox) return paged ? ts::qkv_rope_kernel<D, true, true> : ts::qkv_rope_kernel<D, true, false>;
    return paged ? ts::qkv_rope_kernel<D, false, true> : ts::qkv_rope_kernel<D, false, false>;
}

extern "C" int ts_launch_qkv_rope(const ts_rope_problem *p, void *stream) {
    if (p->n_vec <= 0) return ATTN_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    void (*kern)(ts_rope_problem) = nullptr;
    int resident = 0;  // CTAs per SM: one persistent wave of them
    switch (p->D) {
    case 64: kern = pick_rope_kernel<64>(p), resident = pick_rope_resident<64>(p); break;
    case 128: kern = pick_rope_kernel<128>(p), resident = pick_rope_resident<128>(p); break;
    case 256: kern = pick_rope_kernel<256>(p), resident = pick_rope_resident<256>(p); break;
    default: return ATTN_ERR_ARGS;
    }
    if (resident < 0) return ATTN_ERR_CUDA;
    const long long chunks = (p->n_vec * p->D * 2 + ts::kRopeChunk - 1) / ts::kRopeChunk;
    const long long wave = (long long)ts_num_sms() * resident;
    kern<<<(unsigned)(chunks < wave ? chunks : wave), ts::kRopeThreads, ts::kRopeSmem, st>>>(*p);
    if (cudaGetLastError() != cudaSuccess) return ATTN_ERR_CUDA;
    ts_count_launch();
    return ATTN_OK;
}

extern "C" int ts_launch_rope_table(float *cos_sin, int max_pos, int rot, double theta, void *stream) {
    const long long n = (long long)max_pos * (rot / 2);
    if (n <= 0) return ATTN_OK;
    const long long need = (n + 255) / 256;
    const long long cap = (long long)ts_num_sms() * 8;
    ts::rope_table_kernel<<<(unsigned)(need < cap ? need : cap), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        cos_sin, max_pos, rot, theta);
    if (cudaGetLastError() != cudaSuccess) return ATTN_ERR_CUDA;
    ts_count_launch();
    return ATTN_OK;
}
