// fa_fwd_sm100.cu -- bf16 flash-attention forward on the Blackwell tensor core (sm_100a).
//
// Replaces the hot loop of flash.c's attn_flash (flash.c:779-861): qk_tile (flash.c:352-423)
// becomes a tcgen05 MMA S = Q K^T with S in TMEM; softmax_block (flash.c:518-580) runs on
// the TMEM score tile in softmax warpgroups (one thread per query row); pv_acc
// (flash.c:433-510) becomes a second tcgen05 MMA O += P V whose A operand P is written back
// into TMEM as bf16 and whose B operand V is read from shared memory in place -- MN-major
// for V [keys][D], K-major for a pre-transposed V^T [D][Sk] -- so pack_vt (flash.c:327-342)
// disappears. The final normalise (flash.c:851-860) is the epilogue.
//
// Work decomposition. The `group` query heads that share kv head `kv` are contiguous in Q
// ([Hq][Sq][D] == [Hkv][group*Sq][D]), so each kv head owns one packed [group*Sq][D]
// matrix of query rows that all read the same K/V. A CTA takes NQT tiles of 128 packed
// rows (256 rows for NQT=2) and streams the kv head's K/V tiles once for all of them. Such a
// unit, or one key piece of it, is a work item; the grid has at most one CTA per SM, each
// walking its share of the items (below).
//
// Roles (one CTA per SM): warp 0 issues TMA loads (Q once, then K_j, V_j alternating
// through an NS-slot ring); warp 1 owns TMEM and issues the MMAs from one thread;
// warps 4.. are softmax warpgroups, one per query tile, thread r of a warpgroup owning
// TMEM lane r = query row r. Per key block j and tile t:
//   MMA:      S_t = Q_t K_j^T                      -> commit s_full[t]
//   softmax:  mask, row max, P = 2^(S*c - m) bf16 -> TMEM (aliasing S_t), l update,
//             rescale O_t when its max moved       -> arrive p_full[t]
//   MMA:      O_t += P_t V_j ; S_t = Q_t K_{j+1}^T  -> commit s_full[t]
// tcgen05.commit fires only when every earlier MMA of the issuing thread finished, so the
// s_full completion that delivers S_t(j) also proves PV_t(j-1) wrote O_t: the softmax can
// rescale O_t right after reading S_t(j). With two tiles the tensor core computes one
// tile's PV+QK while the other tile's softmax runs.
//
// Online-softmax state per row follows flash.c:535-576: running max m, alpha =
// exp(m_old - m_new) (0 on a row's first live block), P rounded to bf16 while l sums the
// UNrounded fp32 exponentials, a block with no live key leaves the state unchanged, and a
// row that never sees a key ends with l == 0 and a zero output row. One refinement: the
// running max is only moved when the block max exceeds it by more than 2^kRescaleLog2
// (in exp2 units); otherwise the old max stays the reference and P may exceed 1 by at most
// that factor. The quotient acc/l is the same mathematical value; this skips most O
// rescales (TMEM round trips).
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <atomic>
#include <type_traits>

#include "attn_flash.h"
#include "fa_launch.h"
#include "sm100_ptx.cuh"

extern "C" void ts_count_launch(void);

namespace ts {

constexpr int kBM = 128;              // query rows per tile (TMEM lanes)
constexpr int kBN = ATTN_GPU_KEY_TILE;  // keys per tile
constexpr float kRescaleLog2 = 8.0f;  // lazy max update threshold, in log2 units
constexpr float kRedoSum = 256.0f;    // 2^kRescaleLog2: a speculative row sum above it means a redo
constexpr int kSmemBudget = 200 * 1024;

struct TcParams {
    float *O;                          // normalised output (global rows)
    float *out_m, *out_l, *out_acc;    // caller partials (global rows) when write_partials
    float *part_m, *part_l, *part_acc; // key-piece partials [piece][row - row_base]
    int *status;
    int rows_per_kv;  // group * Sq
    int total_rows;   // Hq * Sq
    int Sq, Sk, Sk_total, k_begin;
    int D, causal, Hkv, tiles_per_kv;
    int n_direct;        // units [0, n_direct) run whole; the rest as `pieces` key pieces
    int pieces, keys_per_piece;
    int row_base, part_rows;  // split units cover global rows [row_base, row_base + part_rows)
    int write_partials;
    int o_bf16;   // 1: O is bf16 bits (round to nearest even), else fp32
    int o_tma;    // 1: fp32 O is written through the staging boxes by TMA (tmO maps O)
    int n_items;  // work items (units, or units and key pieces); the grid has min(n_items, SMs) CTAs
    int snake;    // 1: alternate the direction of the per-CTA item walk every round (causal)
    int group;    // query heads per kv head
    int head_units;  // causal: units per query head when every unit lies within one head, else 0
    // Paged K/V (paged != 0): K and V are pools [num_pages][hkv_local][page_size][D]; the unit
    // kv index is b * hkv_local + kv_local for sequence b, whose keys are the pages
    // block_table[b * max_pages + k / page_size] and whose length is seq_lens[b].
    const int *block_table, *seq_lens;
    int paged, page_size, max_pages, num_pages, hkv_local;
    float scale_log2;
    // 0: the host cleared the status word before the launch; otherwise CTA 0 clears it and then
    // publishes this call's generation in status[1] (error reports wait for that, report_error)
    unsigned gen;
};

template <int DP, int NQT>
struct TcConfig {
    static constexpr int QTILE = kBM * DP * 2;   // bytes of one Q tile
    static constexpr int KVTILE = kBN * DP * 2;  // bytes of one K or V tile
    static constexpr int NS_RAW = (kSmemBudget - NQT * QTILE) / KVTILE;
    static constexpr int NS = NS_RAW > 8 ? 8 : NS_RAW;  // K/V ring slots
    static constexpr int NBAR = 3 + 2 * NS + 3 * NQT;   // q_full/empty, done, kv_full/empty, s/p/o_full
    static constexpr int PID_WIN = 256;  // paged K/V: page ids staged in shared memory at a time
    // Output staging (two-tile instances): one [32 rows][32 fp32] box (128-byte rows, 128-byte
    // swizzle) per softmax warp, written from registers and stored to O by TMA.
    static constexpr int OSTAGE = 32 * 32 * 4;
    static constexpr int NOSTAGE = NQT == 2 ? 8 : 0;  // one-tile instances keep per-row stores
    static constexpr int SMEM = 1024 + NQT * QTILE + NS * KVTILE + NOSTAGE * OSTAGE + NBAR * 8 + 16;
    static constexpr int smem_bytes(bool paged) { return SMEM + (paged ? PID_WIN * 4 : 0); }
    static_assert(smem_bytes(true) <= 227 * 1024, "shared memory per CTA");
    static constexpr int THREADS = 128 + 128 * NQT;
    static constexpr uint32_t TMEM_COLS = (NQT * kBN + NQT * DP) <= 256 ? 256u : 512u;
    static_assert(NS >= 2, "K/V ring needs at least two slots");
    static_assert(DP % 64 == 0 && DP <= 128, "padded head_dim must be 64 or 128");
    static_assert(NQT * kBN + NQT * DP <= 512, "TMEM budget");
};

__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }
__device__ __forceinline__ uint32_t f2u(float f) { return __float_as_uint(f); }

// Waits without honouring the abort flag: used only at teardown, to let TMA copies and MMAs
// that are already in flight land before the CTA releases its shared memory and TMEM.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity, int *status, unsigned gen) {
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
            report_error(status, kDevErrTimeoutDrain, gen);
            return;
        }
    }
}

// GENERAL=false: every work item is a whole unit that writes normalised O (plain prefill/decode
// without splits); GENERAL=true adds key pieces and caller-partial output. NOQ=true is the
// diagnostic build of attn_diag_wait_timeout only: its producer never loads Q, so the MMA
// issuer's bounded wait for Q runs out and the whole CTA takes the abort path.
//
// Persistent: the grid has at most one CTA per SM and each CTA walks the work items
// blockIdx.x, blockIdx.x + gridDim.x, ... (for causal masking in alternating directions over
// the longest-first list, so the long and short units even out per CTA). Every barrier keeps
// counting phases across items, so the next item's Q load, first QK and first softmax block
// overlap the previous item's last PV and epilogue.
template <int DP, int NQT, bool VT, bool GENERAL, bool PAGED, bool NOQ = false>
__global__ void __launch_bounds__(TcConfig<DP, NQT>::THREADS, 1)
    fa_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                 const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                 const TcParams p) {
    using C = TcConfig<DP, NQT>;
    constexpr int NS = C::NS;
    constexpr int NBOX_D = DP / 64;     // 64-element (128-byte) boxes across the head dim
    constexpr int BOX_ROWS128 = 128 * 128;  // bytes of one [128 rows][64 cols] bf16 box

    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_u32 = smem_u32(smem_raw);
    const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
    uint8_t *smem = smem_raw + (base_u32 - raw_u32);

    const uint32_t sQ = base_u32;
    const uint32_t sKV = base_u32 + NQT * C::QTILE;
    const uint32_t sO = sKV + NS * C::KVTILE;  // output staging, 1024-byte aligned
    const uint32_t bar0 = sO + C::NOSTAGE * C::OSTAGE;
    const uint32_t q_full = bar0;         // Q tiles of an item landed
    const uint32_t q_empty = bar0 + 8;    // every QK of an item finished: Q may be reloaded
    const uint32_t done_bar = bar0 + 16;
    auto kv_full = [&](int s) { return bar0 + 24 + 8u * s; };
    auto kv_empty = [&](int s) { return bar0 + 24 + 8u * (NS + s); };
    auto s_full = [&](int t) { return bar0 + 24 + 8u * (2 * NS + t); };           // scores S_t ready
    auto p_full = [&](int t) { return bar0 + 24 + 8u * (2 * NS + NQT + t); };     // P_t stored
    auto o_full = [&](int t) { return bar0 + 24 + 8u * (2 * NS + 2 * NQT + t); }; // an item's O_t final
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + (bar0 - base_u32) + C::NBAR * 8);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    int *pid_win = reinterpret_cast<int *>(tmem_slot + 4);  // paged K/V: C::PID_WIN page ids

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    // ---------------- work items
    // Item index q -> unit (row tile of one kv head) and key piece.
    // !GENERAL: non-causal q = kv * tiles + tile. Causal: a unit's key range grows with its query
    //   position within its head (the group's heads are stacked in the packed rows), so q walks
    //   the positions from the last down, every kv head and every query head of the group at
    //   each position: the longest units come first.
    // GENERAL: kv-major units; units below n_direct run whole, each later unit as `pieces` key
    //   pieces.
    struct Item {
        int kv, row0, piece, kb0, kb1, nblk;
        int sk, sk_total;  // keys present (local) and the key axis length the causal rule uses
    };
    auto item_at = [&](int q) {
        Item it;
        int tile;
        it.piece = -1;
        if (!GENERAL) {
            if (p.causal && p.head_units > 0) {
                const int hk = p.Hkv * p.group;
                const int rem = q % hk;
                it.kv = rem % p.Hkv;
                tile = (rem / p.Hkv) * p.head_units + (p.head_units - 1 - q / hk);
            } else if (p.causal) {  // units straddle heads: highest row tile first
                it.kv = q % p.Hkv;
                tile = p.tiles_per_kv - 1 - q / p.Hkv;
            } else {
                it.kv = q / p.tiles_per_kv;
                tile = q % p.tiles_per_kv;
            }
        } else {
            int u = q;
            if (u >= p.n_direct) {
                const int w = u - p.n_direct;
                u = p.n_direct + w / p.pieces;
                it.piece = w % p.pieces;
            }
            it.kv = u / p.tiles_per_kv;
            tile = u % p.tiles_per_kv;
        }
        it.row0 = tile * kBM * NQT;
        it.sk = p.Sk;
        it.sk_total = p.Sk_total;
        if constexpr (PAGED) {  // this sequence's own length, within its block table
            const int len = __ldg(p.seq_lens + it.kv / p.hkv_local);
            it.sk = it.sk_total = max(0, min(len, p.Sk));
        }
        it.kb0 = it.piece < 0 ? 0 : it.piece * p.keys_per_piece;  // local key range [kb0, kb1)
        it.kb1 = it.piece < 0 ? it.sk : min(it.sk, it.kb0 + p.keys_per_piece);
        int kend = it.kb1;
        if (p.causal) {
            const int rlast = min(it.row0 + kBM * NQT, p.rows_per_kv) - 1;
            const int i_hi = (it.row0 / p.Sq == rlast / p.Sq) ? (rlast % p.Sq) : (p.Sq - 1);
            const long long lim = (long long)it.sk_total - p.Sq + i_hi - p.k_begin;  // last live local key
            if (lim + 1 < (long long)kend) kend = (int)max(lim + 1, (long long)it.kb0);
        }
        it.nblk = kend > it.kb0 ? (kend - it.kb0 + kBN - 1) / kBN : 0;
        return it;
    };
    // this CTA's r-th item (or >= n_items when there is none)
    auto item_index = [&](int r) {
        const int G = (int)gridDim.x, b = (int)blockIdx.x;
        return r * G + ((p.snake && (r & 1)) ? (G - 1 - b) : b);
    };

    // ---------------- setup
    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        mbar_init(q_empty, 1);
        mbar_init(done_bar, 1);
        for (int s = 0; s < NS; ++s) {
            mbar_init(kv_full(s), 1);
            mbar_init(kv_empty(s), 1);
        }
        for (int t = 0; t < NQT; ++t) {
            mbar_init(s_full(t), 1);
            mbar_init(p_full(t), 128);
            mbar_init(o_full(t), 1);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
        if (p.o_tma) tma_prefetch_desc(&tmO);
        if constexpr (!PAGED && !NOQ) {
            // The first item's Q tiles and K/V tile 0 into L2 while the previous grid finishes: the
            // CTA's first loads, after the dependency wait below, then come from L2.
            const int q0 = item_index(0);
            if (q0 < p.n_items) {
                const Item it = item_at(q0);
                if (it.nblk > 0) {
#pragma unroll
                    for (int b = 0; b < NBOX_D; ++b) {
#pragma unroll
                        for (int t = 0; t < NQT; ++t) tma_prefetch_l2_3d(&tmQ, b * 64, it.row0 + t * kBM, it.kv);
                        tma_prefetch_l2_3d(&tmK, b * 64, it.kb0, it.kv);
                        if (!VT) tma_prefetch_l2_3d(&tmV, b * 64, it.kb0, it.kv);
                    }
                    if (VT)
#pragma unroll
                        for (int b = 0; b < kBN / 64; ++b) tma_prefetch_l2_3d(&tmV, it.kb0 + b * 64, 0, it.kv);
                }
            }
        }
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // The set-up above reads no global memory (the L2 prefetch returns nothing to the thread), so
    // it may overlap the previous grid of the stream (programmatic dependent launch); everything
    // below comes after that grid.
    pdl_wait();
    pdl_trigger();
    if (p.gen != 0 && blockIdx.x == 0 && threadIdx.x == 0) {
        *reinterpret_cast<volatile int *>(p.status) = 0;
        __threadfence();
        atomicExch(reinterpret_cast<unsigned *>(p.status) + 1, p.gen);
    }

    // Register budgets per warpgroup (NQT=2 launches 384 threads x 168 registers): the
    // producer/MMA warpgroup gives registers up, the two softmax warpgroups take them:
    // 128 x 128 + 256 x 184 = 63488 <= 384 x 168 = 64512 (neither side spills).
    if (warp < 4) {
        if constexpr (NQT == 2) regs_dec<128>();
    if (warp == 0 && PAGED) {
        // ============================ TMA producer, paged K/V (the whole warp)
        // The warp stages C::PID_WIN page ids of the item at a time in shared memory (checking
        // each id of a page that holds live keys against the pool; ids of pages past the
        // sequence's end are never read), then lane 0 issues each tile's loads from there: a
        // 128-key tile is 128 / page_size boxes of page_size rows (page_size <= 128) or a
        // 128-row part of one page; the 128-byte swizzle repeats every 8 rows, so the boxes
        // land where one 128-row box would. A chunk past the end reuses the tile's first page
        // (its keys are masked).
        const int P = p.page_size;
        const int cs = P < kBN ? P : kBN;
        const int nch = kBN / cs;
        uint32_t gl = 0;
        int qi = 0;
        bool ok = true, q_inflight = false;
        for (int r = 0; ok; ++r) {
            const int q = item_index(r);
            if (q >= p.n_items) break;
            const Item it = item_at(q);
            if (it.nblk == 0) continue;
            const int kv = it.kv, kb0 = it.kb0;
            const int b = kv / p.hkv_local, kvl = kv % p.hkv_local;
            const int used = (it.sk + P - 1) / P;  // pages that hold this sequence's keys
            const int *row = p.block_table + (size_t)b * p.max_pages;
            if (lane == 0) {
                if (qi > 0 && !mbar_wait(q_empty, (qi - 1) & 1, abort_flag, p.status, kDevErrTimeoutQ, p.gen)) ok = false;
                if (ok) {
                    mbar_expect_tx(q_full, NQT * C::QTILE);
#pragma unroll
                    for (int t = 0; t < NQT; ++t)
#pragma unroll
                        for (int bx = 0; bx < NBOX_D; ++bx)
                            tma_load_3d(sQ + t * C::QTILE + bx * BOX_ROWS128, &tmQ, q_full, bx * 64,
                                        it.row0 + t * kBM, kv);
                    q_inflight = true;
                }
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            int win_base = -1;
            const int nload = 2 * it.nblk;
            for (int i = 0; i < nload; ++i, ++gl) {
                const int key0 = kb0 + (i >> 1) * kBN;
                const int pg_lo = key0 / P, pg_hi = (key0 + kBN - 1) / P;
                if (win_base < 0 || pg_hi >= win_base + C::PID_WIN) {  // warp-uniform
                    win_base = pg_lo;
                    bool bad = false;
                    for (int e = lane; e < C::PID_WIN; e += 32) {
                        const int pg = win_base + e;
                        int id = -1;
                        if (pg < used && pg < p.max_pages) {
                            id = __ldg(row + pg);
                            if (id < 0 || id >= p.num_pages) bad = true;
                        }
                        pid_win[e] = id;
                    }
                    bad = __any_sync(0xffffffffu, bad);
                    __syncwarp();
                    if (bad) {
                        if (lane == 0) {
                            *abort_flag = 1;
                            report_error(p.status, kDevErrBadPage, p.gen);
                        }
                        ok = false;
                        break;
                    }
                }
                const int slot = gl % NS;
                const int round = gl / NS;
                const uint32_t bar = kv_full(slot);
                if (lane == 0) {
                    if (round > 0 &&
                        !mbar_wait(kv_empty(slot), (round - 1) & 1, abort_flag, p.status, kDevErrTimeoutKV, p.gen))
                        ok = false;
                    else
                        mbar_expect_tx(bar, C::KVTILE);  // armed before any lane's copy can land
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;  // gl counts the loads issued so far
                // lane c issues chunk c's boxes, so a tile of many small pages goes out in parallel
                const uint32_t dst = sKV + slot * C::KVTILE;
                const CUtensorMap *tm = (i & 1) == 0 ? &tmK : &tmV;
                for (int c = lane; c < nch; c += 32) {
                    const int key = key0 + c * cs;
                    int id = pid_win[key / P - win_base];
                    if (id < 0) id = pid_win[pg_lo - win_base];
#pragma unroll
                    for (int bx = 0; bx < NBOX_D; ++bx)
                        tma_load_3d(dst + bx * (kBN * 128) + c * cs * 128, tm, bar, bx * 64, key % P,
                                    id * p.hkv_local + kvl);
                }
                __syncwarp();
            }
            if (ok) {
                q_inflight = false;
                ++qi;
            }
        }
        if (!ok && lane == 0) {  // let the copies already in flight land before the CTA exits
            if (q_inflight) drain_wait(q_full, qi & 1, p.status, p.gen);
            for (uint32_t i = gl > (uint32_t)NS ? gl - NS : 0u; i < gl; ++i)
                drain_wait(kv_full(i % NS), (i / NS) & 1, p.status, p.gen);
        }
        __syncwarp();
    } else if (warp == 0) {
        // ============================ TMA producer
        if (lane == 0) {
            uint32_t gl = 0;   // K/V tile loads issued, over all items
            int qi = 0;        // items with at least one key block, so far
            bool ok = true, q_inflight = false;
            for (int r = 0; ok; ++r) {
                const int q = item_index(r);
                if (q >= p.n_items) break;
                const Item it = item_at(q);
                if (it.nblk == 0) continue;
                const int kv = it.kv, kb0 = it.kb0;
                // the previous item's QKs have all finished reading Q
                if (qi > 0 && !mbar_wait(q_empty, (qi - 1) & 1, abort_flag, p.status, kDevErrTimeoutQ, p.gen)) {
                    ok = false;
                    break;
                }
                if constexpr (!NOQ) {
                    mbar_expect_tx(q_full, NQT * C::QTILE);
#pragma unroll
                    for (int t = 0; t < NQT; ++t)
#pragma unroll
                        for (int b = 0; b < NBOX_D; ++b)
                            tma_load_3d(sQ + t * C::QTILE + b * BOX_ROWS128, &tmQ, q_full, b * 64,
                                        it.row0 + t * kBM, kv);
                    q_inflight = true;
                }
                const int nload = 2 * it.nblk;
                for (int i = 0; i < nload; ++i, ++gl) {
                    const int slot = gl % NS;
                    const int round = gl / NS;
                    if (round > 0 &&
                        !mbar_wait(kv_empty(slot), (round - 1) & 1, abort_flag, p.status, kDevErrTimeoutKV, p.gen)) {
                        ok = false;
                        break;
                    }
                    const int key0 = kb0 + (i >> 1) * kBN;
                    const uint32_t dst = sKV + slot * C::KVTILE;
                    const uint32_t bar = kv_full(slot);
                    mbar_expect_tx(bar, C::KVTILE);
                    if ((i & 1) == 0) {
#pragma unroll
                        for (int b = 0; b < NBOX_D; ++b)
                            tma_load_3d(dst + b * (kBN * 128), &tmK, bar, b * 64, key0, kv);
                    } else if (!VT) {
#pragma unroll
                        for (int b = 0; b < NBOX_D; ++b)
                            tma_load_3d(dst + b * (kBN * 128), &tmV, bar, b * 64, key0, kv);
                    } else {
#pragma unroll
                        for (int b = 0; b < kBN / 64; ++b)
                            tma_load_3d(dst + b * (DP * 128), &tmV, bar, key0 + b * 64, 0, kv);
                    }
                }
                if (ok) {
                    q_inflight = false;
                    ++qi;
                }
            }
            if (!ok) {  // let the copies already in flight land before the CTA exits
                if (q_inflight) drain_wait(q_full, qi & 1, p.status, p.gen);
                for (uint32_t i = gl > (uint32_t)NS ? gl - NS : 0u; i < gl; ++i)
                    drain_wait(kv_full(i % NS), (i / NS) & 1, p.status, p.gen);
            }
        }
    } else if (warp == 1) {
        // ============================ MMA issuer (one thread)
        if (lane == 0) {
            constexpr uint32_t idesc_qk = idesc_bf16_f32(kBM, kBN, 0, 0);
            constexpr uint32_t idesc_pv = idesc_bf16_f32(kBM, DP, 0, VT ? 0 : 1);
            auto issue_qk = [&](int t, int slot) {
                const uint32_t qa = sQ + t * C::QTILE;
                const uint32_t kb = sKV + slot * C::KVTILE;
                const uint32_t d_tmem = tmem_base + t * kBN;
#pragma unroll
                for (int ks = 0; ks < DP / 16; ++ks) {
                    const uint32_t off = (ks >> 2) * BOX_ROWS128 + (ks & 3) * 32;
                    umma_ss(d_tmem, sdesc_sw128(qa + off, 16, 1024), sdesc_sw128(kb + off, 16, 1024), idesc_qk,
                            ks > 0 ? 1u : 0u);
                }
            };
            auto issue_pv = [&](int t, int slot, bool accumulate) {
                const uint32_t vb = sKV + slot * C::KVTILE;
                const uint32_t d_tmem = tmem_base + NQT * kBN + t * DP;
                const uint32_t a_tmem = tmem_base + t * kBN;
#pragma unroll
                for (int ks = 0; ks < kBN / 16; ++ks) {
                    uint64_t bdesc;
                    if (!VT)  // V [keys][D]: MN-major; LBO = next 64-column block of D, SBO = next 8 keys
                        bdesc = sdesc_sw128(vb + ks * 16 * 128, kBN * 128, 1024);
                    else      // V^T [D][keys]: K-major, like K
                        bdesc = sdesc_sw128(vb + (ks >> 2) * (DP * 128) + (ks & 3) * 32, 16, 1024);
                    umma_ts(d_tmem, a_tmem + ks * 8, bdesc, idesc_pv, (accumulate || ks > 0) ? 1u : 0u);
                }
            };
            uint32_t gc = 0;   // K/V tiles consumed, over all items
            uint32_t pp = 0;   // P handoffs consumed per tile, over all items
            int qi = 0;
            bool ok = true;
            for (int r = 0; ok; ++r) {
                const int q = item_index(r);
                if (q >= p.n_items) break;
                const Item it = item_at(q);
                const int nblk = it.nblk;
                if (nblk == 0) continue;
                const uint32_t sK0 = gc % NS;
                ok = mbar_wait_fast(q_full, qi & 1, abort_flag, p.status, kDevErrTimeoutQ, p.gen) &&
                     mbar_wait_fast(kv_full(sK0), (gc / NS) & 1, abort_flag, p.status, kDevErrTimeoutKV, p.gen);
                if (!ok) break;
                tc_fence_after();
#pragma unroll
                for (int t = 0; t < NQT; ++t) {
                    issue_qk(t, sK0);
                    tc_commit(s_full(t));
                }
                tc_commit(kv_empty(sK0));
                if (nblk == 1) tc_commit(q_empty);
                for (int j = 0; ok && j < nblk; ++j) {
                    const uint32_t iV = gc + 2 * j + 1, iK = gc + 2 * j + 2;
                    const int sV = iV % NS, sK = iK % NS;
                    const bool more = j + 1 < nblk;
#pragma unroll
                    for (int t = 0; t < NQT; ++t) {
                        // V_j and K_{j+1} are normally resident long before P_t(j): waiting for
                        // them first keeps the P handoff the only wait between the softmax and
                        // the issue
                        if (t == 0 && !mbar_wait_fast(kv_full(sV), (iV / NS) & 1, abort_flag, p.status, kDevErrTimeoutKV, p.gen)) {
                            ok = false;
                            break;
                        }
                        if (t == 0 && more &&
                            !mbar_wait_fast(kv_full(sK), (iK / NS) & 1, abort_flag, p.status, kDevErrTimeoutKV, p.gen)) {
                            ok = false;
                            break;
                        }
                        if (!mbar_wait_fast(p_full(t), pp & 1, abort_flag, p.status, kDevErrTimeoutP, p.gen)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        issue_pv(t, sV, j > 0);
                        if (more) {
                            issue_qk(t, sK);
                            tc_commit(s_full(t));
                        } else {
                            tc_commit(o_full(t));  // the item's O_t is final
                        }
                    }
                    if (!ok) break;
                    ++pp;
                    tc_commit(kv_empty(sV));
                    if (more) tc_commit(kv_empty(sK));
                    if (j == nblk - 2) tc_commit(q_empty);  // the item's last QKs were just issued
                }
                gc += 2 * nblk;
                ++qi;
            }
            // Every MMA issued above must finish before TMEM is released.
            tc_commit(done_bar);
            drain_wait(done_bar, 0, p.status, p.gen);
        }
        __syncwarp();
    }
        // teardown (producer/MMA warpgroup): every TMEM user has fenced, then warp 1 frees TMEM
        tc_fence_before();
        __syncthreads();
        if (warp == 1) {
            __syncwarp();
            tc_fence_after();
            tmem_dealloc(tmem_base, C::TMEM_COLS);
        }
    } else {
        if constexpr (NQT == 2) regs_inc<184>();
        // ============================ softmax / correction / epilogue
        const int t = (warp - 4) >> 2;
        const int quad = warp & 3;
        const int r = quad * 32 + lane;
        const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
        const uint32_t tS = tmem_base + lane_off + t * kBN;
        const uint32_t tO = tmem_base + lane_off + NQT * kBN + t * DP;
        const float sl2 = p.scale_log2;
        const float2 c2 = make_float2(sl2, sl2);
        uint32_t sp = 0;  // score-tile phases consumed, over all items
        uint32_t op = 0;  // items finished (o_full phases consumed)
        bool ok = true;
        for (int ri = 0; ok; ++ri) {
        const int qidx = item_index(ri);
        if (qidx >= p.n_items) break;
        const Item it = item_at(qidx);
        const int kv = it.kv, row0 = it.row0, piece = it.piece, kb0 = it.kb0, kb1 = it.kb1, nblk = it.nblk;
        const int prow = row0 + t * kBM + r;  // packed row within this kv head
        const bool valid = prow < p.rows_per_kv;
        const int ipos = valid ? prow % p.Sq : 0;
        const int sk_total = PAGED ? it.sk_total : p.Sk_total, sk = PAGED ? it.sk : p.Sk;
        const long long lim = p.causal ? ((long long)sk_total - p.Sq + ipos - p.k_begin)
                                       : (long long)(sk - 1);  // last live local key of this row
        const long long lastkey = min(lim, (long long)kb1 - 1);

        float m = -INFINITY, l = 0.f;
        float ms = 0.f;  // m * scale_log2, rounded once (0 while m is -inf)
        for (int j = 0; j < nblk; ++j) {
            // The path decisions need no scores, so they are made before the wait.
            const long long key0 = kb0 + (long long)j * kBN;
            const long long nv = lastkey - key0 + 1;
            // `full`: every row of this warp sees every key of the block (no tail, no causal
            // cut). The choice must be warp-uniform: every path issues warp-collective tcgen05.st.
            const bool full = __all_sync(0xffffffffu, nv >= kBN);
            // `spec`: a full block of a warp whose rows all have a running max. P is computed
            // against that max, so the exponentials do not wait for a max pass over all 128
            // columns first. A row whose block max exceeds its running max by more than
            // kRescaleLog2 (in log2 units) has a P above 2^kRescaleLog2, so its row sum is above
            // it too; only then (any row of the warp) is the block redone exactly below. Every P is
            // positive, so a row sum within the bound proves each of its P is -- no per-element max
            // is tracked. The redo is rare: the first block sets a max that later blocks seldom
            // exceed by that much (a sum above the bound with no single P above it only costs
            // the exact pass).
            const bool spec = full && __all_sync(0xffffffffu, m != -INFINITY);
            ok = mbar_wait(s_full(t), sp & 1, abort_flag, p.status, kDevErrTimeoutS, p.gen);
            ++sp;
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            tc_fence_after();
            uint32_t sr[128];
            float rs0 = 0.f, rs1 = 0.f;
            bool redo = true;
            if (spec) {
                const float2 nms2 = make_float2(-ms, -ms);
                float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
                // 16 score columns at a time: the next chunk's load is issued before this
                // chunk's exponentials and waited for after its P store, and the chunk boundaries
                // keep the compiler's schedule chunk by chunk (one upfront 128-column load
                // measured 13% slower).
                // Exponentials: all on MUFU with two tiles per CTA (prefill: the MUFU unit has
                // room, and the polynomial's FMA-pipe instructions cost issue slots); with one
                // tile (decode, where MUFU is the bottleneck) 2 of every 8 pairs take the
                // polynomial exp2 on the FMA pipe.
                tmem_ld16p(tS, sr);
#pragma unroll
                for (int cc = 0; cc < 8; ++cc) {
                    uint32_t pk[8];
                    if (cc < 7) tmem_ld16_nowait(tS + 16 * (cc + 1), sr + 16 * (cc + 1));
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        const float s0 = u2f(sr[16 * cc + 2 * u]), s1 = u2f(sr[16 * cc + 2 * u + 1]);
                        const float2 x = __ffma2_rn(make_float2(s0, s1), c2, nms2);
                        float2 pr;
                        if (NQT == 1 && u < 2) {
                            pr = exp2_fma2(x);
                        } else {
                            pr.x = ex2(x.x);
                            pr.y = ex2(x.y);
                        }
                        if (u & 1)
                            acc1 = __fadd2_rn(acc1, pr);
                        else
                            acc0 = __fadd2_rn(acc0, pr);
                        pk[u] = pack_bf16x2(pr.x, pr.y);
                    }
                    tmem_st8(tS + cc * 8, pk);
                    if (cc < 7) tmem_wait_ld16(sr + 16 * (cc + 1));
                }
                rs0 = acc0.x + acc1.x;
                rs1 = acc0.y + acc1.y;
                redo = __any_sync(0xffffffffu, rs0 + rs1 > kRedoSum);
                if (redo) tmem_wait_st();  // the speculative P stores land before the exact ones
            } else if (__all_sync(0xffffffffu, nv <= 0)) {
                // No row of this warp sees any key of the block (a causal tile below the
                // diagonal of its item's last block): P = 0, m, l and O stay as they are.
                uint32_t zero[16];
#pragma unroll
                for (int u = 0; u < 16; ++u) zero[u] = 0u;
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) tmem_st16(tS + cc * 16, zero);
                redo = false;
            } else {
                tmem_ld128(tS, sr);
            }
            if (!redo) {
                l += rs0 + rs1;
            } else {
                float mb;
                if (full) {
                    float mx[8];
#pragma unroll
                    for (int k = 0; k < 8; ++k) mx[k] = fmax3(u2f(sr[k]), u2f(sr[8 + k]), u2f(sr[16 + k]));
#pragma unroll
                    for (int c = 24; c < 128; c += 16)
#pragma unroll
                        for (int k = 0; k < 8; ++k) mx[k] = fmax3(mx[k], u2f(sr[c + k]), u2f(sr[c + 8 + k]));
                    mb = fmaxf(fmax3(mx[0], mx[1], mx[2]), fmax3(fmax3(mx[3], mx[4], mx[5]), mx[6], mx[7]));
                } else {
                    const int nvalid = nv < 0 ? 0 : (int)nv;
#pragma unroll
                    for (int c = 0; c < 128; ++c)
                        if (c >= nvalid) sr[c] = f2u(-INFINITY);
                    float mx0 = u2f(sr[0]), mx1 = u2f(sr[1]), mx2 = u2f(sr[2]), mx3 = u2f(sr[3]);
#pragma unroll
                    for (int c = 4; c < 128; c += 4) {
                        mx0 = fmaxf(mx0, u2f(sr[c]));
                        mx1 = fmaxf(mx1, u2f(sr[c + 1]));
                        mx2 = fmaxf(mx2, u2f(sr[c + 2]));
                        mx3 = fmaxf(mx3, u2f(sr[c + 3]));
                    }
                    mb = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
                }
                float m_new = m;
                if (mb > m && (m == -INFINITY || (mb - m) * sl2 > kRescaleLog2)) m_new = mb;
                const float alpha = (m_new == m) ? 1.f : ((m == -INFINITY) ? 0.f : ex2((m - m_new) * sl2));
                ms = (m_new == -INFINITY) ? 0.f : __fmul_rn(m_new, sl2);
                if (full) {
                    // P = 2^(s*c - m*c) by one packed FMA per pair; 3 of every 8 pairs take the
                    // polynomial exp2 on the FMA pipe, the rest the MUFU unit, so both run at once.
                    const float2 nms2 = make_float2(-ms, -ms);
                    float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll
                    for (int cc = 0; cc < 4; ++cc) {
                        uint32_t pk[16];
#pragma unroll
                        for (int u = 0; u < 16; ++u) {
                            const float2 x = __ffma2_rn(
                                make_float2(u2f(sr[32 * cc + 2 * u]), u2f(sr[32 * cc + 2 * u + 1])), c2, nms2);
                            float2 pr;
                            if ((u & 7) < 3) {
                                pr = exp2_fma2(x);
                            } else {
                                pr.x = ex2(x.x);
                                pr.y = ex2(x.y);
                            }
                            if (u & 1)
                                acc1 = __fadd2_rn(acc1, pr);
                            else
                                acc0 = __fadd2_rn(acc0, pr);
                            pk[u] = pack_bf16x2(pr.x, pr.y);
                        }
                        tmem_st16(tS + cc * 16, pk);
                    }
                    rs0 = acc0.x + acc1.x;
                    rs1 = acc0.y + acc1.y;
                } else {
#pragma unroll
                    for (int cc = 0; cc < 4; ++cc) {
                        uint32_t pk[16];
#pragma unroll
                        for (int u = 0; u < 16; ++u) {
                            // Rounded multiply, then subtract (never fused): the row's max element
                            // gives exactly 2^0 = 1, as exp(S - m) does in flash.c:566.
                            const float p0 = ex2(__fsub_rn(__fmul_rn(u2f(sr[32 * cc + 2 * u]), sl2), ms));
                            const float p1 = ex2(__fsub_rn(__fmul_rn(u2f(sr[32 * cc + 2 * u + 1]), sl2), ms));
                            rs0 += p0;
                            rs1 += p1;
                            pk[u] = pack_bf16x2(p0, p1);
                        }
                        tmem_st16(tS + cc * 16, pk);
                    }
                }
                l = l * alpha + (rs0 + rs1);
                m = m_new;
                // O_t holds P V through block j-1 (complete: S_t(j) was committed after it).
                if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
                    for (int cc = 0; cc < DP / 32; ++cc) {
                        uint32_t o[32];
                        tmem_ld32(tO + cc * 32, o);
#pragma unroll
                        for (int u = 0; u < 32; ++u) o[u] = f2u(u2f(o[u]) * alpha);
                        tmem_st32(tO + cc * 32, o);
                    }
                }
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(p_full(t));
        }
        bool have_o = false;
        if (ok && nblk > 0) {
            have_o = mbar_wait(o_full(t), op & 1, abort_flag, p.status, kDevErrTimeoutS, p.gen);
            ++op;
            have_o = __all_sync(0xffffffffu, have_o);
            ok = have_o;
            if (have_o) tc_fence_after();
        }
        if (ok) {
            // ------------------------ epilogue
            const int D = p.D;
            const size_t grow = (size_t)kv * p.rows_per_kv + prow;  // row of [Hq*Sq]
            float *dst;
            float mult;
            bool out_bf16 = false, to_o = false;
            if (GENERAL && (piece >= 0 || p.write_partials)) {
                // (m, l, unnormalised acc): a key piece's slot, or the caller's partial row
                const size_t slot = piece >= 0 ? (size_t)piece * p.part_rows + (grow - p.row_base) : grow;
                float *pm = piece >= 0 ? p.part_m : p.out_m;
                float *pl = piece >= 0 ? p.part_l : p.out_l;
                if (valid) {
                    pm[slot] = (m == -INFINITY) ? -INFINITY : __fmul_rn(m, sl2);
                    pl[slot] = l;
                }
                dst = (piece >= 0 ? p.part_acc : p.out_acc) + slot * D;
                mult = 1.f;
            } else {
                dst = p.O + grow * D;  // bf16 output: element offsets of a uint16_t array
                mult = (l > 0.f) ? 1.f / l : 0.f;
                out_bf16 = p.o_bf16 != 0;
                to_o = true;
            }
            auto store_rows = [&](auto bf16_tag) {
                constexpr bool kBf16 = decltype(bf16_tag)::value;
#pragma unroll
                for (int cc = 0; cc < DP / 32; ++cc) {
                    uint32_t o[32];
                    if (have_o) {
                        tmem_ld32(tO + cc * 32, o);
                    } else {
#pragma unroll
                        for (int u = 0; u < 32; ++u) o[u] = 0u;
                    }
                    if (valid) {
#pragma unroll
                        for (int v = 0; v < 8; ++v) {
                            const int c = cc * 32 + 4 * v;
                            if (c < D) {
                                float4 w = make_float4(u2f(o[4 * v]) * mult, u2f(o[4 * v + 1]) * mult,
                                                       u2f(o[4 * v + 2]) * mult, u2f(o[4 * v + 3]) * mult);
                                if constexpr (kBf16) {
                                    uint16_t *ob = reinterpret_cast<uint16_t *>(p.O) + grow * D + c;
                                    *reinterpret_cast<uint2 *>(ob) =
                                        make_uint2(f32_to_bf16_bits(w.x) | (f32_to_bf16_bits(w.y) << 16),
                                                   f32_to_bf16_bits(w.z) | (f32_to_bf16_bits(w.w) << 16));
                                } else {
                                    *reinterpret_cast<float4 *>(dst + c) = w;
                                }
                            }
                        }
                    }
                }
            };
            if (NQT == 2 && to_o && !out_bf16 && p.o_tma) {
                // Normalised fp32 O through TMA: per 32-column chunk, each lane writes its row's
                // 128 bytes into the warp's [32 rows][32 floats] box (16-byte piece v of row r
                // at piece v ^ (r & 7), the 128-byte swizzle, so the eight lanes of a shared-
                // memory phase hit distinct banks), then lane 0 stores the box to rows
                // [y0, y0 + 32) of this kv head's output. Rows past rows_per_kv and columns past
                // D lie outside the tensor map and are not written. (A per-row st.global.v4
                // touches 32 cache lines per warp instruction.)
                const uint32_t buf = sO + (uint32_t)(warp - 4) * C::OSTAGE;
                const int y0 = row0 + t * kBM + quad * 32;
#pragma unroll
                for (int cc = 0; cc < DP / 32; ++cc) {
                    if (cc * 32 >= D) break;
                    uint32_t o[32];
                    if (have_o) {
                        tmem_ld32(tO + cc * 32, o);
                    } else {
#pragma unroll
                        for (int u = 0; u < 32; ++u) o[u] = 0u;
                    }
                    if (lane == 0) bulk_wait_read0();  // the previous box has been read out
                    __syncwarp();
#pragma unroll
                    for (int v = 0; v < 8; ++v)
                        st_shared_v4(buf + lane * 128 + ((v ^ (lane & 7)) << 4), u2f(o[4 * v]) * mult,
                                     u2f(o[4 * v + 1]) * mult, u2f(o[4 * v + 2]) * mult, u2f(o[4 * v + 3]) * mult);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0 && y0 < p.rows_per_kv) {  // a box wholly past the rows is not stored
                        tma_store_3d(&tmO, buf, cc * 32, y0, kv);
                        bulk_commit();
                    }
                }
            } else if (out_bf16) {
                store_rows(std::true_type{});
            } else {
                store_rows(std::false_type{});
            }
        }
        }
        // teardown (softmax warpgroups): this warp's output stores complete, TMEM reads done
        // before the dealloc below
        if (lane == 0) bulk_wait0();
        tc_fence_before();
        __syncthreads();
    }
}

// ------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// Looked up once (thread-safe static initialisation); nullptr if the driver lacks the entry.
static EncodeTiledFn encode_fn() {
    static const EncodeTiledFn fn = []() -> EncodeTiledFn {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return reinterpret_cast<EncodeTiledFn>(ptr);
        return nullptr;
    }();
    return fn;
}

// The fp32 output as a 3-D tensor map {D, rows_per_kv, Hkv} (the layout of Q) for the epilogue's
// TMA stores: boxes of [32 rows][32 floats], 128-byte swizzle.
static bool make_map_o(CUtensorMap *m, float *O, uint64_t D, uint64_t rows, uint64_t hkv) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {D, rows, hkv};
    cuuint64_t strides[2] = {D * 4, rows * D * 4};
    cuuint32_t box[3] = {32, 32, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, O, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// 3-D bf16 tensor map with 128-byte swizzle: dims {d0 (contiguous), d1, d2}, byte strides of
// d1 and d2, box {64, box1, 1}. Out-of-range elements read as zero.
static bool make_map_3d(CUtensorMap *m, const void *base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1,
                        uint64_t s2, uint32_t box1) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {d0, d1, d2};
    cuuint64_t strides[2] = {s1, s2};
    cuuint32_t box[3] = {64, box1, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int DP, int NQT, bool VT, bool GENERAL, bool PAGED, bool NOQ = false>
static int launch_tc_inst(cudaStream_t st, const CUtensorMap &tmQ, const CUtensorMap &tmK, const CUtensorMap &tmV,
                          const CUtensorMap &tmO, const TcParams &prm, dim3 grid) {
    using C = TcConfig<DP, NQT>;
    auto kern = fa_tc_kernel<DP, NQT, VT, GENERAL, PAGED, NOQ>;
    static std::atomic<int> attr_done[64];  // the shared-memory opt-in, once per device
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return ATTN_ERR_CUDA;
    const bool cached = dev >= 0 && dev < 64;
    if (!cached || !attr_done[dev].load(std::memory_order_acquire)) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::smem_bytes(PAGED)) !=
            cudaSuccess)
            return ATTN_ERR_CUDA;
        if (cached) attr_done[dev].store(1, std::memory_order_release);
    }
    // programmatic dependent launch: the kernel's set-up may overlap the previous grid's tail
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(C::THREADS);
    cfg.dynamicSmemBytes = C::smem_bytes(PAGED);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, tmQ, tmK, tmV, tmO, prm) != cudaSuccess) return ATTN_ERR_CUDA;
    ts_count_launch();
    return ATTN_OK;
}

template <int DP, int NQT, bool VT, bool NOQ = false>
static int launch_tc(const fa_problem *P, cudaStream_t st, int tiles_per_kv) {
    const int group = P->Hq / P->Hkv;
    const uint64_t rows = (uint64_t)group * P->Sq;
    const uint64_t D = (uint64_t)P->D;
    CUtensorMap tmQ, tmK, tmV;
    if (!make_map_3d(&tmQ, P->Q, D, rows, P->Hkv, D * 2, rows * D * 2, kBM)) return ATTN_ERR_CUDA;
    if (P->paged) {  // page pools: {D, rows of a page, page x kv head}, boxes of up to 128 rows
        const uint64_t ps = (uint64_t)P->page_size;
        const uint32_t box = P->page_size < kBN ? (uint32_t)P->page_size : (uint32_t)kBN;
        const uint64_t planes = (uint64_t)P->num_pages * P->hkv_local;
        if (!make_map_3d(&tmK, P->K, D, ps, planes, D * 2, ps * D * 2, box)) return ATTN_ERR_CUDA;
        if (!make_map_3d(&tmV, P->V, D, ps, planes, D * 2, ps * D * 2, box)) return ATTN_ERR_CUDA;
    } else {
        if (!make_map_3d(&tmK, P->K, D, P->Sk, P->Hkv, D * 2, (uint64_t)P->Sk * D * 2, kBN)) return ATTN_ERR_CUDA;
        if (!VT) {
            if (!make_map_3d(&tmV, P->V, D, P->Sk, P->Hkv, D * 2, (uint64_t)P->Sk * D * 2, kBN))
                return ATTN_ERR_CUDA;
        } else if (!make_map_3d(&tmV, P->V, P->Sk, D, P->Hkv, (uint64_t)P->Sk * 2, (uint64_t)P->Sk * D * 2, DP)) {
            return ATTN_ERR_CUDA;
        }
    }
    CUtensorMap tmO;
    memset(&tmO, 0, sizeof tmO);
    // fp32 normalised output of a two-tile instance: stored by TMA (any other output keeps per-row
    // stores)
    const int o_tma = NQT == 2 && P->O != nullptr && !P->o_bf16 && !P->write_partials;
    if (o_tma && !make_map_o(&tmO, P->O, D, rows, (uint64_t)P->Hkv)) return ATTN_ERR_CUDA;
    TcParams prm;
    prm.O = P->O;
    prm.o_tma = o_tma;
    prm.out_m = P->out_m;
    prm.out_l = P->out_l;
    prm.out_acc = P->out_acc;
    prm.part_m = P->part_m;
    prm.part_l = P->part_l;
    prm.part_acc = P->part_acc;
    prm.status = P->status;
    prm.rows_per_kv = (int)rows;
    prm.total_rows = P->Hq * P->Sq;
    prm.Sq = P->Sq;
    prm.Sk = P->Sk;
    prm.Sk_total = P->Sk_total;
    prm.k_begin = P->k_begin;
    prm.D = P->D;
    prm.causal = P->causal;
    prm.Hkv = P->Hkv;
    prm.tiles_per_kv = tiles_per_kv;
    const int units = tiles_per_kv * P->Hkv;
    prm.n_direct = P->nsplit > 1 ? P->n_direct : units;
    prm.pieces = P->nsplit > 1 ? P->nsplit : 1;
    prm.keys_per_piece = P->keys_per_split;
    prm.row_base = P->row_base;
    prm.part_rows = P->Hq * P->Sq - P->row_base;
    prm.write_partials = P->write_partials;
    prm.o_bf16 = P->o_bf16;
    prm.block_table = P->block_table;
    prm.seq_lens = P->seq_lens;
    prm.paged = P->paged;
    prm.page_size = P->page_size;
    prm.max_pages = P->max_pages;
    prm.num_pages = P->num_pages;
    prm.hkv_local = P->hkv_local > 0 ? P->hkv_local : 1;
    prm.scale_log2 = P->scale_log2;
    prm.gen = P->status_gen;
    prm.group = group;
    prm.head_units = (P->Sq % (kBM * NQT) == 0) ? P->Sq / (kBM * NQT) : 0;
    const int sms = ts_num_sms() > 0 ? ts_num_sms() : 1;
    if constexpr (NOQ) {  // the diagnostic build: plain work plan only
        prm.n_items = units;
        prm.snake = 0;
        return launch_tc_inst<DP, NQT, VT, false, false, true>(st, tmQ, tmK, tmV, tmO, prm, dim3(min(units, sms)));
    }
    if (prm.n_direct == units && !prm.write_partials && !P->paged) {
        prm.n_items = units;
        prm.snake = prm.causal;
        return launch_tc_inst<DP, NQT, VT, false, false>(st, tmQ, tmK, tmV, tmO, prm, dim3(min(units, sms)));
    }
    prm.n_items = prm.n_direct + (units - prm.n_direct) * prm.pieces;
    prm.snake = 0;
    if (P->paged)  // paged K/V: the general work plan, V row-major
        return launch_tc_inst<DP, NQT, false, true, true>(st, tmQ, tmK, tmV, tmO, prm, dim3(min(prm.n_items, sms)));
    return launch_tc_inst<DP, NQT, VT, true, false>(st, tmQ, tmK, tmV, tmO, prm, dim3(min(prm.n_items, sms)));
}

static int nqt_for(const fa_problem *P) {
    const long long rows = (long long)(P->Hq / P->Hkv) * P->Sq;
    return rows > kBM ? 2 : 1;
}

}  // namespace ts

extern "C" int ts_tc_supported(const fa_problem *P) {
    if (P->D % 8 != 0 || P->D > 128 || P->D < 8) return 0;
    if (P->v_prepacked && P->Sk % 8 != 0) return 0;
    if (((uintptr_t)P->Q | (uintptr_t)P->K | (uintptr_t)P->V) & 15u) return 0;
    const float *out = P->O ? P->O : P->part_acc;
    if (((uintptr_t)out) & 15u) return 0;
    if (ts::encode_fn() == nullptr) return 0;
    return 1;
}

extern "C" int ts_tc_unit_rows(const fa_problem *P) { return ts::kBM * ts::nqt_for(P); }

extern "C" int ts_tc_ctas_per_split(const fa_problem *P) {
    const long long rows = (long long)(P->Hq / P->Hkv) * P->Sq;
    const int nqt = ts::nqt_for(P);
    const long long tiles = (rows + ts::kBM * nqt - 1) / (ts::kBM * nqt);
    return (int)(tiles * P->Hkv);
}

// attn_diag_wait_timeout's launch: the NOQ build at head_dim 128, one 128-row tile per unit.
extern "C" int ts_launch_tc_noq(const fa_problem *P, void *stream) {
    using namespace ts;
    if (P->D != 128 || (long long)(P->Hq / P->Hkv) * P->Sq > kBM || P->paged || P->v_prepacked) return ATTN_ERR_ARGS;
    if (encode_fn() == nullptr) return ATTN_ERR_CUDA;
    return launch_tc<128, 1, false, true>(P, static_cast<cudaStream_t>(stream), 1);
}

extern "C" int ts_launch_tc(const fa_problem *P, void *stream) {
    using namespace ts;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const long long rows = (long long)(P->Hq / P->Hkv) * P->Sq;
    const int nqt = nqt_for(P);
    const int tiles = (int)((rows + kBM * nqt - 1) / (kBM * nqt));
    const int dp = P->D <= 64 ? 64 : 128;
    const bool vt = P->v_prepacked != 0;
#define TS_LAUNCH(DPV, NQTV)                                                                      \
    do {                                                                                          \
        return vt ? launch_tc<DPV, NQTV, true>(P, st, tiles) : launch_tc<DPV, NQTV, false>(P, st, tiles); \
    } while (0)
    if (dp == 64) {
        if (nqt == 2) TS_LAUNCH(64, 2);
        TS_LAUNCH(64, 1);
    }
    if (nqt == 2) TS_LAUNCH(128, 2);
    TS_LAUNCH(128, 1);
#undef TS_LAUNCH
}
