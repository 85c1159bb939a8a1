// fa_peer.cu -- the key-split decode's merge over NVLink, in one kernel per rank.
//
// A long-context decode splits the key axis over the GPUs of a node: rank r attends keys
// [k_begin, k_begin + Sk_local) of every kv head and ends with per-row partials (m, l, acc) of
// its key pieces -- the key loop of flash.c:798 split across GPUs, whose online-softmax merge
// (flash.c:535-576) must then run across the ranks. fa_peer_merge_kernel does that merge with
// plain peer stores, no collective library:
//   1. each CTA owns a fixed range of rows; its warps merge this rank's key pieces for those
//      rows and store the merged (m, l, acc) into slot `rank` of EVERY rank's exchange block
//      (its own included) through the peers' mapped pointers -- NVLink stores;
//   2. the CTA fences at system scope and raises its flag in every rank's block (the flag holds
//      the call's epoch);
//   3. it waits, bounded, until every rank's flag for this CTA reached the epoch in its OWN
//      block, then merges the world slots of its rows into O from local memory.
// The exchange block is double-buffered by epoch parity: a rank writes epoch e+1 only after its
// epoch-e merge saw every rank's epoch-e flag, and no rank reaches that point before every other
// rank finished reading epoch e-1, the buffer e+1 reuses.
//
// Exchange block layout (bytes), identical on every rank:
//   [0, kPeerFlagBytes)           uint32 flags [ATTN_PEERS_MAX][kPeerMaxCtas] (epoch reached)
//   then 2 buffers x world slots  packed partial (attn_flash_packed_floats(rows, D) floats,
//                                 rounded up to 256 bytes): m [rows], l [rows], pad, acc [rows][D]
// Every wait is bounded (kWaitLimitNs); a wait that runs out sets ATTN_DEV_TIMEOUT_PEER in the
// status word and leaves that CTA's rows of O unwritten.
#include <cuda.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "attn_flash.h"
#include "fa_launch.h"
#include "sm100_ptx.cuh"

extern "C" void ts_count_launch(void);

namespace ts {

constexpr int kPeerMaxCtas = 128;
constexpr size_t kPeerFlagBytes = (size_t)ATTN_PEERS_MAX * kPeerMaxCtas * 4;

__host__ __device__ inline size_t peer_slot_bytes(int rows, int D) {
    const size_t f = ((2 * (size_t)rows + 3) & ~(size_t)3) + (size_t)rows * D;
    return (f * 4 + 255) & ~(size_t)255;
}

struct PeerParams {
    const float *m, *l, *acc;  // this rank's key pieces [nparts][rows] (, [D])
    int nparts, rows, D, rows_per_cta;
    float *O;
    unsigned char *blocks[ATTN_PEERS_MAX];  // every rank's exchange block, mapped here
    int world, rank;
    unsigned epoch;
    int *status;
};

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_relaxed_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// Merges `n` partials of one row for the VW consecutive columns [col, col + VW) a lane owns:
// m_at(s) and l_at(s) give part s's m and l, acc_at(s, col, out) loads its VW acc values. The
// lanes load the parts' m and l in parallel (one round trip for up to 32 parts), and the acc loads
// of all parts are independent, so they are in flight together. Returns the merged m and L; `a`
// receives the lane's unnormalised acc values.
template <int VW, typename M, typename L, typename A>
__device__ __forceinline__ float2 merge_parts(int n, int lane, bool live, M m_at, L l_at, A acc_at, float (&a)[VW]) {
    float mx = -INFINITY;
    for (int s = lane; s < n; s += 32) mx = fmaxf(mx, m_at(s));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float Lsum = 0.f;
#pragma unroll
    for (int e = 0; e < VW; ++e) a[e] = 0.f;
    for (int s0 = 0; s0 < n; s0 += 32) {
        const int s = s0 + lane;
        float w = 0.f;
        if (s < n) {
            const float ms = m_at(s);
            w = (ms != -INFINITY) ? ex2_approx(ms - mx) : 0.f;
            Lsum = fmaf(w, l_at(s), Lsum);
        }
        const int cnt = min(32, n - s0);
#pragma unroll 4
        for (int k = 0; k < cnt; ++k) {
            const float wk = __shfl_sync(0xffffffffu, w, k);
            if (live) {
                float x[VW];
                acc_at(s0 + k, x);
#pragma unroll
                for (int e = 0; e < VW; ++e) a[e] = fmaf(wk, x[e], a[e]);
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) Lsum += __shfl_xor_sync(0xffffffffu, Lsum, o);
    return make_float2(mx, Lsum);
}

template <int VW>
__device__ __forceinline__ void load_vec(const float *src, float (&x)[VW], bool coherent) {
    if constexpr (VW == 4) {
        const float4 v = coherent ? __ldcg(reinterpret_cast<const float4 *>(src)) : *reinterpret_cast<const float4 *>(src);
        x[0] = v.x;
        x[1] = v.y;
        x[2] = v.z;
        x[3] = v.w;
    } else {
        x[0] = coherent ? __ldcg(src) : *src;
    }
}

template <int VW>
__device__ __forceinline__ void store_vec(float *dst, const float (&x)[VW]) {
    if constexpr (VW == 4)
        *reinterpret_cast<float4 *>(dst) = make_float4(x[0], x[1], x[2], x[3]);
    else
        *dst = x[0];
}

// The CTA's (row, 32*VW-column chunk) tasks are spread over its warps; lane i owns the VW
// columns chunk * 32 * VW + VW * i (VW = 4 when D % 4 == 0: 16-byte loads and NVLink stores).
template <int VW>
__global__ void __launch_bounds__(256) fa_peer_merge_kernel(const PeerParams p) {
    __shared__ int s_fail;
    pdl_wait();  // the key pieces come from the previous grid of the stream
    pdl_trigger();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int c = blockIdx.x;
    const int r0 = c * p.rows_per_cta, r1 = min(p.rows, r0 + p.rows_per_cta);
    constexpr int CW = 32 * VW;  // columns per task
    const int nchunk = (p.D + CW - 1) / CW;
    const int ntask = max(0, r1 - r0) * nchunk;
    const int buf = (int)(p.epoch & 1u);
    const size_t slot_bytes = peer_slot_bytes(p.rows, p.D);
    const size_t ml = (2 * (size_t)p.rows + 3) & ~(size_t)3;
    auto slot = [&](unsigned char *blk, int src) {
        return reinterpret_cast<float *>(blk + kPeerFlagBytes + ((size_t)buf * p.world + src) * slot_bytes);
    };
    if (threadIdx.x == 0) s_fail = 0;

    // 1. merge this rank's key pieces; one rank: that is the output. Otherwise store the merged
    //    (m, l, acc) into slot `rank` of every rank's block.
    for (int t = warp; t < ntask; t += nwarps) {
        const int r = r0 + t / nchunk, col = (t % nchunk) * CW + VW * lane;
        const bool live = col < p.D;
        float a[VW];
        const float2 v = merge_parts<VW>(
            p.nparts, lane, live, [&](int s) { return p.m[(size_t)s * p.rows + r]; },
            [&](int s) { return p.l[(size_t)s * p.rows + r]; },
            [&](int s, float(&x)[VW]) { load_vec<VW>(p.acc + ((size_t)s * p.rows + r) * p.D + col, x, false); }, a);
        if (p.world == 1) {
            if (live) {
                const float inv = v.y > 0.f ? 1.f / v.y : 0.f;
#pragma unroll
                for (int e = 0; e < VW; ++e) a[e] *= inv;
                store_vec<VW>(p.O + (size_t)r * p.D + col, a);
            }
            continue;
        }
        for (int q = 0; q < p.world; ++q) {
            float *dst = slot(p.blocks[q], p.rank);
            if (lane == 0 && col == 0) {
                dst[r] = v.x;
                dst[p.rows + r] = v.y;
            }
            if (live) store_vec<VW>(dst + ml + (size_t)r * p.D + col, a);
        }
    }
    if (p.world == 1) return;

    // 2. this CTA's rows are in every block: raise its flag everywhere. The CTA barrier orders
    //    every thread's stores before the flag threads' system-scope releases (fences are
    //    cumulative over what the fencing thread has synchronised with), which order them before
    //    the flags; thread q releases to rank q, so the releases run side by side.
    __syncthreads();
    if (threadIdx.x < p.world) {
        unsigned *flags = reinterpret_cast<unsigned *>(p.blocks[threadIdx.x]);
        st_release_sys(flags + (size_t)p.rank * kPeerMaxCtas + c, p.epoch);
    }

    // 3. wait (bounded) for every rank's flag of this CTA in the own block: relaxed polls, then
    //    one acquire fence once the flag is seen; the CTA barrier passes it on to every thread
    if (threadIdx.x < p.world) {
        const unsigned *flag =
            reinterpret_cast<const unsigned *>(p.blocks[p.rank]) + (size_t)threadIdx.x * kPeerMaxCtas + c;
        const uint64_t t0 = globaltimer_ns();
        while ((int)(ld_relaxed_sys(flag) - p.epoch) < 0) {
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
                atomicOr(p.status, kDevErrTimeoutPeer);
                s_fail = 1;
                break;
            }
        }
        fence_acq_rel_sys();
    }
    __syncthreads();
    if (s_fail) return;

    // 4. merge the world slots of this CTA's rows into O (L2-coherent reads of peer-written data)
    unsigned char *own = p.blocks[p.rank];
    for (int t = warp; t < ntask; t += nwarps) {
        const int r = r0 + t / nchunk, col = (t % nchunk) * CW + VW * lane;
        const bool live = col < p.D;
        float a[VW];
        const float2 v = merge_parts<VW>(
            p.world, lane, live, [&](int s) { return __ldcg(slot(own, s) + r); },
            [&](int s) { return __ldcg(slot(own, s) + p.rows + r); },
            [&](int s, float(&x)[VW]) { load_vec<VW>(slot(own, s) + ml + (size_t)r * p.D + col, x, true); }, a);
        if (live) {
            const float inv = v.y > 0.f ? 1.f / v.y : 0.f;
#pragma unroll
            for (int e = 0; e < VW; ++e) a[e] *= inv;
            store_vec<VW>(p.O + (size_t)r * p.D + col, a);
        }
    }
}

}  // namespace ts

extern "C" size_t attn_flash_peer_block_bytes(int world, int rows, int D) {
    if (world < 1 || world > ATTN_PEERS_MAX || rows < 0 || D < 1 || D > ATTN_D_MAX) return 0;
    return ts::kPeerFlagBytes + 2 * (size_t)world * ts::peer_slot_bytes(rows, D);
}

extern "C" int ts_launch_peer_merge(const float *m, const float *l, const float *acc, int nparts, int rows, int D,
                                    float *O, void *const *blocks, int world, int rank, unsigned epoch, int *status,
                                    void *stream) {
    ts::PeerParams p;
    memset(&p, 0, sizeof p);
    p.m = m;
    p.l = l;
    p.acc = acc;
    p.nparts = nparts;
    p.rows = rows;
    p.D = D;
    p.O = O;
    for (int q = 0; q < world; ++q) p.blocks[q] = static_cast<unsigned char *>(blocks[q]);
    p.world = world;
    p.rank = rank;
    p.epoch = epoch;
    p.status = status;
    // the same row split on every rank (it depends on rows only): CTA c of every rank owns the
    // same rows, so each CTA waits for the same CTA index of its peers
    const int ctas = rows < ts::kPeerMaxCtas ? (rows > 0 ? rows : 1) : ts::kPeerMaxCtas;
    p.rows_per_cta = (rows + ctas - 1) / ctas;
    // programmatic dependent launch: may start while the partial kernel finishes (pdl_wait)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas);
    cfg.blockDim = dim3(256);
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const bool vec = D % 4 == 0 && ((((uintptr_t)acc) | ((uintptr_t)O)) & 15u) == 0;
    const cudaError_t e = vec ? cudaLaunchKernelEx(&cfg, ts::fa_peer_merge_kernel<4>, p)
                              : cudaLaunchKernelEx(&cfg, ts::fa_peer_merge_kernel<1>, p);
    if (e != cudaSuccess) return ATTN_ERR_CUDA;
    ts_count_launch();
    return ATTN_OK;
}

// ---------------------------------------------------------------- CUDA IPC of exchange blocks
// A handle is the allocation's cudaIpcMemHandle_t followed by the block's byte offset inside
// that allocation (a caching allocator hands out blocks inside larger allocations).
typedef CUresult (*GetAddressRangeFn)(CUdeviceptr *, size_t *, CUdeviceptr);

static GetAddressRangeFn address_range_fn() {
    static const GetAddressRangeFn fn = []() -> GetAddressRangeFn {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return reinterpret_cast<GetAddressRangeFn>(ptr);
        return nullptr;
    }();
    return fn;
}

static_assert(sizeof(cudaIpcMemHandle_t) + 8 <= ATTN_PEER_HANDLE_BYTES, "handle size");

extern "C" int attn_peer_export(void *dev_ptr, void *handle) {
    if (!dev_ptr || !handle) return ATTN_ERR_ARGS;
    GetAddressRangeFn range = address_range_fn();
    if (!range) return ATTN_ERR_CUDA;
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS) return ATTN_ERR_CUDA;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base)) != cudaSuccess) return ATTN_ERR_CUDA;
    const uint64_t off = reinterpret_cast<uint64_t>(dev_ptr) - static_cast<uint64_t>(base);
    memset(handle, 0, ATTN_PEER_HANDLE_BYTES);
    memcpy(handle, &h, sizeof h);
    memcpy(static_cast<char *>(handle) + sizeof h, &off, 8);
    return ATTN_OK;
}

extern "C" int attn_peer_import(const void *handle, void **dev_ptr) {
    if (!handle || !dev_ptr) return ATTN_ERR_ARGS;
    cudaIpcMemHandle_t h;
    uint64_t off = 0;
    memcpy(&h, handle, sizeof h);
    memcpy(&off, static_cast<const char *>(handle) + sizeof h, 8);
    void *base = nullptr;
    if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return ATTN_ERR_CUDA;
    *dev_ptr = static_cast<char *>(base) + off;
    return ATTN_OK;
}

extern "C" int attn_peer_close(void *dev_ptr, const void *handle) {
    if (!dev_ptr || !handle) return ATTN_ERR_ARGS;
    uint64_t off = 0;
    memcpy(&off, static_cast<const char *>(handle) + sizeof(cudaIpcMemHandle_t), 8);
    return cudaIpcCloseMemHandle(static_cast<char *>(dev_ptr) - off) == cudaSuccess ? ATTN_OK : ATTN_ERR_CUDA;
}
