// Tree and unified attention on tcgen05 tensor cores (sm_100a).
//
// Bit for bit the CPU oracle's restatement (oracle/numerics.py attend): the
// B200's tcgen05 kind::f16 MMA accumulates per 16-deep step with every
// product and the accumulator aligned to the largest exponent, truncated 25
// bits below it, summed and rounded toward zero (measured:
// tests/golden/tensorcore_probe.npz), and the kernel fixes every other
// rounding:
//   S = Q K^T in eight 16-deep steps from zero; per 64-key tile the masked
//   row max, alpha = exp2((m_old - m_new) sl2), O *= alpha before P V,
//   P = bf16(exp2(s sl2 - m sl2)) with the softmax exp2 (qexp2s); the row
//   sum in eight partials (key j of a tile goes to partial j % 8, in key
//   order) combined as ((l0 + l1) + (l2 + l3)) + ((l4 + l5) + (l6 + l7));
//   then the LSE merge with bf16 roundings and the per-head fp8
//   quantisation.
//
// Block: 64 query rows of one cu_a segment x 4 query heads of one KV head
// (2 when the GQA group is 2) as two M=128 tiles (rows 0-63 one head, rows
// 64-127 the next) that share every K/V tile. 16 warps:
//   warp 0       TMA loader: each item's call list, Q once, then K tiles of
//                64 keys into a 2-stage ring - the segment's own keys as
//                contiguous rows, the resident keys one box per page through
//                the block table (the warp runs the load loops and waits,
//                lane 0 issues, as in every issuing warp here);
//   warp 10      TMA loader of the V tiles, the same way, into a 3-stage ring
//                (its own warp, so a V tile is requested as soon as its slot
//                frees);
//   warp 1       TMEM allocator and S issuer: S = Q K^T into one of two
//                TMEM buffers per M tile, so the next tile's S runs while the
//                softmax works on this one;
//   warp 11      P V issuer: O += P V with P read from TMEM (the A operand)
//                and V read MN-major from shared memory, as soon as an M
//                tile's P is written; it also zeroes the V rows of a paged
//                tile past the last key (pool rows there may hold anything,
//                and 0 * NaN is NaN). Two issuers, each waiting on one
//                barrier at a time: one thread polling both kinds of work
//                took 300-600 cycles a step and sat about 2,000 cycles in
//                each tile's 16 S issues, so each P V went out 2-4k cycles
//                after its P;
//   warps 2-9    softmax, one thread per row of an M tile: S from TMEM (read
//                twice: the row max, then exp2), bf16 P written back over the
//                tile's S (tcgen05.st), then the row's O *= alpha in TMEM
//                once the previous P V is done (the thread's own rescale: a
//                separate correction warp set, handling both M tiles in turn
//                behind a barrier per tile, held each P V about 2.6 us after
//                its P was ready); after a call B its normaliser goes to the
//                store warps, after call A the same thread merges with the
//                call-B output (bf16, over it) and takes the row's absolute
//                max;
//   warps 12-15  store warps, one thread per row of each M tile: a call B's
//                O normalised to bf16 into shared memory once its last P V is
//                done (the next call's first P V waits for that read), and
//                the merged row quantised per head to fp8 and stored, while
//                the softmax warps go on (a call-A epilogue waits for the
//                row's shared memory to be free again).
// TMEM (512 columns): O [2 M tiles][128] | S [2 M tiles][2 buffers][64], the
// first 32 columns of an S buffer holding that tile's P once computed.
// A tcgen05.mma of M=128, K=16 takes about 26 ns at N=64 and 35 ns at
// N=128 on an idle SM (measured), and the issuing thread waits for each, so
// the S of the next tile is issued as soon as its buffer frees rather than
// after the softmax of this one.
// Every wait is bounded (about a second): a wait that gives up sets a status
// bit and the abort flag, the other roles stop at their next wait, the MMA
// issuers drain their MMAs and the loaders their copies before TMEM is freed.
#include "tc_common.cuh"

namespace qb {
namespace attn_tc {

using namespace qb::tc;

constexpr int D = 128;
constexpr int QR = 64;  // query rows per block
constexpr int KT = 64;  // keys per tile
constexpr int KST = 2;  // K stages: a K tile is free once its S MMAs are done
constexpr int VST = 3;  // V stages: a V tile is free once its P V MMAs are done
constexpr int MAX_CALLS = QR + 1;
constexpr int FIRST_SOFT = 2, V_WARP = 10, PV_WARP = 11, FIRST_STORE = 12;
constexpr int NUM_THREADS = 16 * 32;

constexpr int Q_BYTES = 2 * 2 * 128 * 128;  // [mt][half][128 rows][128 B]
constexpr int KV_HALF = 64 * 128;           // [64 keys][64 dims]
constexpr int KV_TILE = 2 * KV_HALF;        // K or V: two 64-dim halves
constexpr int OB_ROW = 256;                 // a row's call-B output: 128 bf16
constexpr int OFF_K = Q_BYTES;
constexpr int OFF_V = OFF_K + KST * KV_TILE;
constexpr int OFF_OB = OFF_V + VST * KV_TILE;
constexpr int OFF_AUX = OFF_OB + 2 * 128 * OB_ROW;  // OB: [mt 2][128 rows]

// TMEM: O [mt][128 columns] at 0; S [mt][buffer][64 columns] at 256 + mt *
// 128 + buffer * 64, its first 32 columns overwritten by the tile's bf16 P
// (two keys a column), which the P V MMA reads as its A operand
constexpr uint32_t TM_O = 0, TM_S = 256;

// S: M=128, N=64; P V: M=128, N=128 with B (V) MN-major; bf16 in, f32 out
constexpr uint32_t IDESC_S = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(KT >> 3) << 17) |
                             ((uint32_t)(128 >> 4) << 24);
constexpr uint32_t IDESC_PV = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) |
                              ((uint32_t)(D >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);

enum : int { CALL_READS = 0, CALL_OWN = 1, CALL_UNIFIED = 2 };

struct Call {
    int kind, group, n_keys, key_end, q_first, n_tiles;
};

// One work item (a 64-row query tile x one head group): filled by the loader
// warp, read by the other roles, released by all of them.
struct Info {
    int seg, row0, h0, hk, seg_start, seg_end;
    int n_calls, total_tiles;
    int s_grp[QR];  // read group per tile row (-1: reads nothing resident)
    Call calls[MAX_CALLS];
};

struct Aux {
    uint64_t q_full, q_empty;
    uint64_t info_full[2], info_empty[2];
    uint64_t k_full[KST], k_empty[KST], v_full[VST], v_empty[VST];
    // per S/P buffer (tile parity) and M tile; phase = tile / 2, so a producer
    // can only complete a buffer's next phase after every waiter observed
    // the previous one (a parity wait needs that)
    uint64_t s_full[2][2], p_full[2][2], pv_done[2][2];
    uint64_t drain[2];  // [S issuer, P V issuer]
    // per M tile: an item's merged rows are in shared memory (softmax ->
    // store warps) / stored, the rows free again (store warps -> softmax)
    uint64_t y_full[2], y_empty[2];
    // per M tile: a call's normaliser is written (softmax -> store warps) /
    // its O read and its bf16 output in shared memory (store warps -> P V
    // issuer and softmax)
    uint64_t b_full[2], o_free[2];
    uint32_t tmem_base;
    int abort;
    float ep_amax[2][128];  // [mt][row] the merged row's absolute max
    float ep_inv[2][128];   // [mt][row] 1 / l of a call-B output
    Info info[2];
};

constexpr size_t SMEM_BYTES = OFF_AUX + sizeof(Aux) + 1024;
static_assert(SMEM_BYTES <= 232448, "shared memory");

__device__ __forceinline__ int read_group(const int32_t* cu_q, int64_t n_reads, int idx) {
    int lo = 0, hi = (int)n_reads;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (cu_q[mid] <= idx) lo = mid; else hi = mid;
    }
    return lo;
}

__device__ __forceinline__ uint32_t bf16x2_bits(float a, float b) {
    bf162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Two merged outputs as a bf16 pair (f32x2 arithmetic): a = bf16(o inv);
// with call B, bf16(a + (b - a) w), b the call-B output (bf16 pair ob).
__device__ __forceinline__ uint32_t merge_pair(uint32_t o0, uint32_t o1, uint32_t ob,
                                               uint64_t inv2, uint64_t w2, bool has_b) {
    float a0, a1;
    f2unpack(f2mul(f2pack(__uint_as_float(o0), __uint_as_float(o1)), inv2), a0, a1);
    const uint32_t y = bf16x2_bits(a0, a1);
    if (!has_b) return y;
    const uint64_t a = f2pack(__uint_as_float(y << 16), __uint_as_float(y & 0xFFFF0000u));
    const uint64_t b = f2pack(__uint_as_float(ob << 16), __uint_as_float(ob & 0xFFFF0000u));
    float s0, s1;
    f2unpack(f2add(a, f2mul(f2sub(b, a), w2)), s0, s1);
    return bf16x2_bits(s0, s1);
}

// Operand descriptors. Q: [mt][half][128 rows][128 B]; K, V: [half][64][128 B].
__device__ __forceinline__ uint64_t q_desc(uint32_t q_base, int mt, int ks) {
    return sw128_desc(q_base + (uint32_t)(mt * 32768 + (ks >> 2) * 16384)) + (uint64_t)(2 * (ks & 3));
}
__device__ __forceinline__ uint64_t k_desc(uint32_t k_base, int ks) {
    return sw128_desc(k_base + (uint32_t)((ks >> 2) * KV_HALF)) + (uint64_t)(2 * (ks & 3));
}
__device__ __forceinline__ uint64_t v_desc(uint32_t v_base, int kk) {
    return sw128_mn_desc(v_base + (uint32_t)(kk * 16 * 128), KV_HALF, 1024);
}

// UE8M0: the output's per-head scales are powers of two (the reference's
// use_ue8m0 mode of merge_attn_quant and the unified path's quant).
template <bool UNIFIED, bool UE8M0>
__global__ void __launch_bounds__(NUM_THREADS, 1)
attention_tc_kernel(const __grid_constant__ CUtensorMap map_q,
                    const __grid_constant__ CUtensorMap map_k,
                    const __grid_constant__ CUtensorMap map_v,
                    const __grid_constant__ CUtensorMap map_kp,
                    const __grid_constant__ CUtensorMap map_vp, int64_t rows, int n_q, int n_kv,
                    int hp, const int32_t* __restrict__ cu_a, const int32_t* __restrict__ tiles,
                    int n_tiles, const int32_t* __restrict__ read_cu_q,
                    const int32_t* __restrict__ read_used, const int32_t* __restrict__ read_table,
                    int64_t n_reads, int64_t table_width, const int32_t* __restrict__ source,
                    int64_t n_pages, int page_tokens, float scale, uint8_t* __restrict__ q_out,
                    float* __restrict__ scale_out, int64_t scale_ld, uint32_t* status) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024 - (raw & 1023)) & 1023);
    Aux* aux = reinterpret_cast<Aux*>(smem + OFF_AUX);
    volatile int* abort_flag = &aux->abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int group_sz = n_q / n_kv;
    const int per_kv = group_sz / hp;
    const int n_hg = n_kv * per_kv;  // head groups
    const int n_items = n_tiles * n_hg;
    const int nmt = hp >> 1;

    if (threadIdx.x == 0) {
        mbar_init(&aux->q_full, 1);
        mbar_init(&aux->q_empty, 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&aux->info_full[b], 1);
            // released by the S issuer, the active softmax warps, the V
            // loader, the P V issuer and the store warps
            mbar_init(&aux->info_empty[b], 1 + 4 * nmt + 1 + 1 + 4);
        }
        for (int st = 0; st < KST; ++st) {
            mbar_init(&aux->k_full[st], 1);
            mbar_init(&aux->k_empty[st], 1);
        }
        for (int st = 0; st < VST; ++st) {
            mbar_init(&aux->v_full[st], 1);
            mbar_init(&aux->v_empty[st], 1);
        }
        for (int m = 0; m < 2; ++m) {
            mbar_init(&aux->s_full[0][m], 1);
            mbar_init(&aux->s_full[1][m], 1);
            mbar_init(&aux->p_full[0][m], 4);
            mbar_init(&aux->p_full[1][m], 4);
            mbar_init(&aux->pv_done[0][m], 1);
            mbar_init(&aux->pv_done[1][m], 1);
        }
        mbar_init(&aux->drain[0], 1);
        for (int m = 0; m < 2; ++m) {
            mbar_init(&aux->y_full[m], 4);
            mbar_init(&aux->y_empty[m], 4);
            mbar_init(&aux->b_full[m], 4);
            mbar_init(&aux->o_free[m], 4);
        }
        mbar_init(&aux->drain[1], 1);
        aux->abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
                         smem_u32(&aux->tmem_base))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = aux->tmem_base;

    if (warp == 0) {
        // ---------------- loader: item info, Q, K and V tiles ----------------
        int g = 0, jq = 0;    // tiles loaded, Q loads issued
        int nk = 0, nv = 0;   // K and V tiles whose loads were issued
        bool ok = true;
        for (int item = blockIdx.x, k = 0; item < n_items && ok; item += gridDim.x, ++k) {
            const int slot = k & 1;
            if (k >= 2 && !mbar_wait(&aux->info_empty[slot], (uint32_t)((k - 2) >> 1) & 1u,
                                     abort_flag, status, STATUS_ATTN_LOAD))
                break;
            Info* inf = &aux->info[slot];
            const int tile = item / n_hg, hg = item % n_hg;
            const int seg = tiles[2 * tile], row0 = tiles[2 * tile + 1];
            const int hk = hg / per_kv;
            const int h0 = hk * group_sz + (hg % per_kv) * hp;
            const int seg_start = cu_a[seg], seg_end = cu_a[seg + 1];
            const bool good = seg_start >= 0 && seg_end <= rows && row0 >= seg_start && row0 < seg_end;
            // read group per tile row, two rows per lane
            for (int r = lane; r < QR; r += 32) {
                int grp = -1;
                if (!UNIFIED && good && row0 + r < seg_end && n_reads > 0) {
                    const int src = source[row0 + r];
                    if (src >= 0) {
                        if (src >= read_cu_q[n_reads]) atomicOr(status, STATUS_BAD_INDEX);
                        else grp = read_group(read_cu_q, n_reads, src);
                    }
                }
                inf->s_grp[r] = grp;
            }
            __threadfence_block();
            __syncwarp();
            if (lane == 0) {
                // the item's attention calls: each distinct read group (resident
                // keys, not causal) ascending, then the segment's own keys
                // (causal); or the one causal paged call of the unified path
                int nc = 0, total = 0;
                auto add = [&](int kind, int grp, int n_keys, int q_first, bool causal) {
                    int key_end = causal ? min(n_keys, q_first + QR) : n_keys;
                    if (key_end < 0) key_end = 0;
                    const int nt = (key_end + KT - 1) / KT;
                    inf->calls[nc++] = Call{kind, grp, n_keys, key_end, q_first, nt};
                    total += nt;
                };
                if (!good) {
                    atomicOr(status, STATUS_BAD_INDEX);
                } else if (UNIFIED) {
                    int used = read_used[seg];
                    const int q_len = seg_end - seg_start;
                    if (used < q_len ||
                        (int64_t)((used + page_tokens - 1) / page_tokens) > table_width) {
                        atomicOr(status, STATUS_BAD_INDEX);
                        used = q_len;
                    }
                    add(CALL_UNIFIED, seg, used, used - q_len + (row0 - seg_start), true);
                } else {
                    int cur = -1;
                    while (true) {
                        int next = INT_MAX;
                        for (int i = 0; i < QR; ++i) {
                            const int x = inf->s_grp[i];
                            if (x > cur && x < next) next = x;
                        }
                        if (next == INT_MAX) break;
                        cur = next;
                        int used = read_used[cur];
                        if (used < 0 ||
                            (int64_t)((used + page_tokens - 1) / page_tokens) > table_width) {
                            atomicOr(status, STATUS_BAD_INDEX);
                            used = 0;
                        }
                        if (used > 0) {
                            add(CALL_READS, cur, used, 0, false);
                        } else {
                            // a read group without keys: its rows attend to their own keys only
                            for (int i = 0; i < QR; ++i)
                                if (inf->s_grp[i] == cur) inf->s_grp[i] = -1;
                        }
                    }
                    add(CALL_OWN, -1, seg_end - seg_start, row0 - seg_start, true);
                }
                inf->seg = seg;
                inf->row0 = row0;
                inf->h0 = h0;
                inf->hk = hk;
                inf->seg_start = seg_start;
                inf->seg_end = seg_end;
                inf->n_calls = nc;
                inf->total_tiles = total;
                mbar_arrive(&aux->info_full[slot]);
            }
            // the Q and K loads: the warp runs the loops and waits, lane 0 issues
            __syncwarp();
            const int nc = inf->n_calls, total = inf->total_tiles;
            {
                if (total > 0) {
                    // Q of the item's heads, once the previous item's S MMAs are done
                    if (jq > 0 && !mbar_wait(&aux->q_empty, (uint32_t)(jq - 1) & 1u, abort_flag,
                                             status, STATUS_ATTN_LOAD)) {
                        ok = false;
                    } else {
                        if (lane == 0) {
                            mbar_arrive_expect_tx(&aux->q_full, (uint32_t)(nmt * 32768));
                            for (int mt = 0; mt < nmt; ++mt)
                                for (int hh = 0; hh < 2; ++hh)
                                    for (int half = 0; half < 2; ++half)
                                        tma_load_2d(smem_u32(smem + mt * 32768 + half * 16384 + hh * 8192),
                                                    &map_q, (h0 + 2 * mt + hh) * D + half * 64, row0,
                                                    &aux->q_full);
                        }
                        __syncwarp();
                        ++jq;
                    }
                }
                for (int c = 0; c < nc && ok; ++c) {
                    const Call cl = inf->calls[c];
                    for (int t = 0; t < cl.n_tiles; ++t, ++g) {
                        // K may run KST tiles ahead of the S MMAs (the V tiles
                        // have their own loader warp)
                        const int j0 = t * KT;
                        const int32_t* trow =
                            cl.kind == CALL_OWN
                                ? nullptr
                                : read_table +
                                      (int64_t)(cl.kind == CALL_UNIFIED ? seg : cl.group) * table_width;
                        for (int kv = 0; kv < 1 && ok; ++kv) {
                            const int n = kv == 0 ? nk : nv;
                            const int nst = kv == 0 ? KST : VST;
                            const int st = n % nst;
                            uint64_t* full = kv == 0 ? &aux->k_full[st] : &aux->v_full[st];
                            uint64_t* empty = kv == 0 ? &aux->k_empty[st] : &aux->v_empty[st];
                            if (!mbar_wait(empty, ((uint32_t)(n / nst) & 1u) ^ 1u, abort_flag,
                                           status, STATUS_ATTN_LOAD)) {
                                ok = false;
                                break;
                            }
                            uint8_t* dst = smem + (kv == 0 ? OFF_K : OFF_V) + st * KV_TILE;
                            const CUtensorMap* own_map = kv == 0 ? &map_k : &map_v;
                            const CUtensorMap* page_map = kv == 0 ? &map_kp : &map_vp;
                            if (lane == 0) {
                            mbar_arrive_expect_tx(full, KV_TILE);
                            if (cl.kind == CALL_OWN) {
                                const int y = seg_start + j0;
                                for (int half = 0; half < 2; ++half)
                                    tma_load_2d(smem_u32(dst + half * KV_HALF), own_map,
                                                hk * D + half * 64, y, full);
                            } else {
                                for (int pg = 0; pg < KT / page_tokens; ++pg) {
                                    const int key = j0 + pg * page_tokens;
                                    int64_t page = 0;  // keys past the last one: any valid page
                                    if (key < cl.n_keys) {
                                        page = trow[key / page_tokens];
                                        if (page < 0 || page >= n_pages) {
                                            atomicOr(status, STATUS_BAD_INDEX);
                                            page = 0;
                                        }
                                    }
                                    const int y = (int)(page * page_tokens);
                                    const int off = pg * page_tokens * 128;
                                    for (int half = 0; half < 2; ++half)
                                        tma_load_2d(smem_u32(dst + half * KV_HALF + off), page_map,
                                                    hk * D + half * 64, y, full);
                                }
                            }
                            }
                            __syncwarp();
                            if (kv == 0) ++nk; else ++nv;
                        }
                        if (!ok) break;
                    }
                }
            }
        }
        // no copy may still be landing when the block exits
        if (lane == 0) {
            if (jq > 0) mbar_drain(&aux->q_full, (uint32_t)(jq - 1) & 1u, status, STATUS_ATTN_LOAD);
            for (int j = (nk > KST ? nk - KST : 0); j < nk; ++j)
                mbar_drain(&aux->k_full[j % KST], (uint32_t)(j / KST) & 1u, status,
                           STATUS_ATTN_LOAD);
            for (int j = (nv > VST ? nv - VST : 0); j < nv; ++j)
                mbar_drain(&aux->v_full[j % VST], (uint32_t)(j / VST) & 1u, status,
                           STATUS_ATTN_LOAD);
        }
    } else if (warp == 1) {
        // ------ S issuer: S = Q K^T of each tile in order, into the tile's
        // S buffer (g & 1) once the P V two tiles back, which read the P
        // written over it, is done. The whole warp runs the loop and waits,
        // lane 0 issues: with lane 0 looping alone while the other lanes
        // sat at a block barrier, the attention ran 5% slower ------
        const uint32_t q_base = smem_u32(smem);
        {
            int gs = 0, jq = 0;
            bool ok = true;
            for (int item = blockIdx.x, k = 0; item < n_items && ok; item += gridDim.x, ++k) {
                const int slot = k & 1;
                if (!mbar_wait(&aux->info_full[slot], (uint32_t)(k >> 1) & 1u, abort_flag, status,
                               STATUS_ATTN_MMA))
                    break;
                const Info* inf = &aux->info[slot];
                const int n_calls = inf->n_calls, total = inf->total_tiles;
                for (int c = 0, j = 0; c < n_calls && ok; ++c) {
                    const int n_t = inf->calls[c].n_tiles;
                    for (int t = 0; t < n_t; ++t, ++gs, ++j) {
                        // the item's Q, the tile's K, and its S buffer
                        if (j == 0)
                            ok = mbar_wait(&aux->q_full, (uint32_t)(jq++) & 1u, abort_flag, status,
                                           STATUS_ATTN_MMA);
                        if (ok)
                            ok = mbar_wait(&aux->k_full[gs % KST], (uint32_t)(gs / KST) & 1u,
                                           abort_flag, status, STATUS_ATTN_MMA);
                        for (int mt = 0; mt < nmt && ok && gs > 1; ++mt)
                            ok = mbar_wait(&aux->pv_done[gs & 1][mt], (uint32_t)((gs - 2) >> 1) & 1u,
                                           abort_flag, status, STATUS_ATTN_MMA);
                        if (!ok) break;
                        tc_fence_after();
                        const uint32_t k_base = smem_u32(smem + OFF_K + (gs % KST) * KV_TILE);
                        if (lane == 0) {
                        for (int mt = 0; mt < nmt; ++mt) {
                            const uint32_t s_tm = tmem + TM_S + (uint32_t)(mt * 128 + (gs & 1) * 64);
#pragma unroll
                            for (int kk = 0; kk < D / 16; ++kk)
                                mma_bf16_ss(s_tm, q_desc(q_base, mt, kk), k_desc(k_base, kk), IDESC_S,
                                            kk > 0 ? 1u : 0u);
                            mma_commit(&aux->s_full[gs & 1][mt]);
                        }
                        mma_commit(&aux->k_empty[gs % KST]);  // the K tile is free once these are done
                        // the item's last S: Q may be reloaded once these are done
                        if (j == total - 1) mma_commit(&aux->q_empty);
                        }
                        __syncwarp();
                    }
                }
                // done with the item's info (its S MMAs are all issued)
                if (lane == 0) mbar_arrive(&aux->info_empty[slot]);
                __syncwarp();
            }
            // every MMA issued must finish before TMEM is freed
            if (lane == 0) mma_commit(&aux->drain[0]);
            __syncwarp();
            mbar_drain(&aux->drain[0], 0, status, STATUS_ATTN_MMA);
        }
    } else if (warp == PV_WARP) {
        // ------ P V issuer (the warp waits, lane 0 issues, the warp zeroes
        // V tails; waits by lane 0 alone with the verdict broadcast were
        // slower): O += P V
        // of each tile and M tile in order, with P read from TMEM (the A
        // operand, bf16 over the tile's S) and V MN-major from shared
        // memory, as soon as that M tile's P is written ------
        auto wait0 = [&](uint64_t* bar, uint32_t parity) -> bool {
            return mbar_wait(bar, parity, abort_flag, status, STATUS_ATTN_MMA);
        };
        int g = 0, eb = 0;  // tiles; call-B outputs the store warps took from O
        bool ok = true;
        for (int item = blockIdx.x, k = 0; item < n_items && ok; item += gridDim.x, ++k) {
            const int slot = k & 1;
            if (!wait0(&aux->info_full[slot], (uint32_t)(k >> 1) & 1u)) break;
            const Info* inf = &aux->info[slot];
            const int n_calls = inf->n_calls;
            for (int c = 0; c < n_calls && ok; ++c) {
                const Call cl = inf->calls[c];
                for (int t = 0; t < cl.n_tiles && ok; ++t, ++g) {
                    const int st = g % VST;
                    uint8_t* vd = smem + OFF_V + st * KV_TILE;
                    const uint32_t v_base = smem_u32(vd);
                    if (!wait0(&aux->v_full[st], (uint32_t)(g / VST) & 1u)) {
                        ok = false;
                        break;
                    }
                    const int valid = cl.n_keys - t * KT;
                    if (cl.kind != CALL_OWN && valid < KT) {
                        // the V rows past the last key: zeros (pool rows there
                        // may hold anything, and 0 * NaN is NaN)
                        const int first = valid < 0 ? 0 : valid;
                        for (int idx = first * 8 + lane; idx < KT * 8; idx += 32) {
                            const int r = idx >> 3, ch = idx & 7;
                            *reinterpret_cast<uint4*>(vd + r * 128 + ch * 16) = make_uint4(0, 0, 0, 0);
                            *reinterpret_cast<uint4*>(vd + KV_HALF + r * 128 + ch * 16) =
                                make_uint4(0, 0, 0, 0);
                        }
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                        __syncwarp();
                    }
                    // a call's first P V overwrites O: after a call B, once the
                    // store warps have read it
                    const bool after_b = t == 0 && c > 0 && inf->calls[c - 1].kind == CALL_READS;
                    for (int mt = 0; mt < nmt; ++mt) {
                        if (!wait0(&aux->p_full[g & 1][mt], (uint32_t)(g >> 1) & 1u) ||
                            (after_b && !wait0(&aux->o_free[mt], (uint32_t)eb & 1u))) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        if (lane == 0) {
                            // A = P (bf16, two keys a column) in TMEM over S
                            const uint32_t p_tm = tmem + TM_S + (uint32_t)(mt * 128 + (g & 1) * 64);
#pragma unroll
                            for (int kk = 0; kk < KT / 16; ++kk)
                                mma_bf16_ts(tmem + TM_O + (uint32_t)(mt * 128), p_tm + (uint32_t)(kk * 8),
                                            v_desc(v_base, kk), IDESC_PV, (t > 0 || kk > 0) ? 1u : 0u);
                            mma_commit(&aux->pv_done[g & 1][mt]);
                        }
                        __syncwarp();
                    }
                    if (!ok) break;
                    if (after_b) ++eb;
                    if (lane == 0) mma_commit(&aux->v_empty[st]);
                    __syncwarp();
                }
            }
            // done with the item's info (its P V are all issued)
            if (lane == 0) mbar_arrive(&aux->info_empty[slot]);
            __syncwarp();
        }
        // every MMA issued must finish before TMEM is freed
        if (lane == 0) mma_commit(&aux->drain[1]);
        __syncwarp();
        mbar_drain(&aux->drain[1], 0, status, STATUS_ATTN_MMA);
    } else if (warp == V_WARP) {
        // ---------------- V loader: the V tiles of every item's calls, up to
        // VST tiles ahead of the P V MMAs (the K loader runs on its own); the
        // warp runs the loop and waits, lane 0 issues ----------------
        {
            int nv = 0;
            bool ok = true;
            for (int item = blockIdx.x, k = 0; item < n_items && ok; item += gridDim.x, ++k) {
                const int slot = k & 1;
                if (!mbar_wait(&aux->info_full[slot], (uint32_t)(k >> 1) & 1u, abort_flag, status,
                               STATUS_ATTN_LOAD))
                    break;
                const Info* inf = &aux->info[slot];
                const int hk = inf->hk, seg = inf->seg, seg_start = inf->seg_start;
                for (int c = 0; c < inf->n_calls && ok; ++c) {
                    const Call cl = inf->calls[c];
                    const int32_t* trow =
                        cl.kind == CALL_OWN
                            ? nullptr
                            : read_table + (int64_t)(cl.kind == CALL_UNIFIED ? seg : cl.group) * table_width;
                    for (int t = 0; t < cl.n_tiles; ++t, ++nv) {
                        const int st = nv % VST;
                        if (!mbar_wait(&aux->v_empty[st], ((uint32_t)(nv / VST) & 1u) ^ 1u, abort_flag,
                                       status, STATUS_ATTN_LOAD)) {
                            ok = false;
                            break;
                        }
                        uint8_t* dst = smem + OFF_V + st * KV_TILE;
                        uint64_t* full = &aux->v_full[st];
                        if (lane == 0) {
                        mbar_arrive_expect_tx(full, KV_TILE);
                        const int j0 = t * KT;
                        if (cl.kind == CALL_OWN) {
                            for (int half = 0; half < 2; ++half)
                                tma_load_2d(smem_u32(dst + half * KV_HALF), &map_v, hk * D + half * 64,
                                            seg_start + j0, full);
                        } else {
                            for (int pg = 0; pg < KT / page_tokens; ++pg) {
                                const int key = j0 + pg * page_tokens;
                                int64_t page = 0;  // keys past the last one: any valid page
                                if (key < cl.n_keys) {
                                    page = trow[key / page_tokens];
                                    if (page < 0 || page >= n_pages) {
                                        atomicOr(status, STATUS_BAD_INDEX);
                                        page = 0;
                                    }
                                }
                                const int y = (int)(page * page_tokens);
                                const int off = pg * page_tokens * 128;
                                for (int half = 0; half < 2; ++half)
                                    tma_load_2d(smem_u32(dst + half * KV_HALF + off), &map_vp,
                                                hk * D + half * 64, y, full);
                            }
                        }
                        }
                        __syncwarp();
                    }
                }
                if (!ok) break;
                if (lane == 0) mbar_arrive(&aux->info_empty[slot]);
                __syncwarp();
            }
            // no copy may still be landing when the block exits
            for (int j = (nv > VST ? nv - VST : 0); j < nv; ++j)
                mbar_drain(&aux->v_full[j % VST], (uint32_t)(j / VST) & 1u, status,
                           STATUS_ATTN_LOAD);
        }
    } else if (warp >= FIRST_STORE) {
        // ------- store warps: pass 2 of an item's call-A epilogue, one thread
        // per row of each M tile: the merged row (bf16, in shared memory)
        // quantised per head to fp8 and stored -------
        const int q4 = warp & 3;
        const int i = q4 * 32 + lane;
        const int qi = i & (QR - 1);
        const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
        int g = 0, ea = 0, eb = 0;  // tiles; call-A and call-B epilogues done
        bool ok = true;
        for (int item = blockIdx.x, k = 0; item < n_items && ok; item += gridDim.x, ++k) {
            const int slot = k & 1;
            if (!mbar_wait(&aux->info_full[slot], (uint32_t)(k >> 1) & 1u, abort_flag, status,
                           STATUS_ATTN_SOFTMAX))
                break;
            const Info* inf = &aux->info[slot];
            const int n_calls = inf->n_calls;
            // each call B's output: once its last P V is done, O normalised
            // (bf16) into the shared-memory rows of the read group's members
            for (int c = 0; c < n_calls && ok; ++c) {
                const Call cl = inf->calls[c];
                g += cl.n_tiles;
                if (cl.kind != CALL_READS) continue;
                const bool member = inf->s_grp[qi] == cl.group;
                for (int mt = 0; mt < nmt && ok; ++mt) {
                    if (!mbar_wait(&aux->b_full[mt], (uint32_t)eb & 1u, abort_flag, status,
                                   STATUS_ATTN_SOFTMAX) ||
                        !mbar_wait(&aux->pv_done[(g - 1) & 1][mt], (uint32_t)((g - 1) >> 1) & 1u,
                                   abort_flag, status, STATUS_ATTN_SOFTMAX)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const float inv = aux->ep_inv[mt][i];
                    const uint32_t o_addr = tmem + lane_off + TM_O + (uint32_t)(mt * 128);
                    uint8_t* obrow = smem + OFF_OB + (mt * 128 + i) * OB_ROW;
                    if (__any_sync(0xffffffffu, member)) {
#pragma unroll 1
                        for (int c0 = 0; c0 < D; c0 += 32) {
                            uint32_t r[32];
                            tmem_ld32_nowait(o_addr + (uint32_t)c0, r);
                            tmem_wait_ld();
                            uint32_t ob[16];
#pragma unroll
                            for (int j = 0; j < 16; ++j)
                                ob[j] = bf16x2_bits(__fmul_rn(__uint_as_float(r[2 * j]), inv),
                                                    __fmul_rn(__uint_as_float(r[2 * j + 1]), inv));
                            if (member) {
#pragma unroll
                                for (int u = 0; u < 4; ++u) {
                                    const int j = (c0 >> 3) + u;
                                    *reinterpret_cast<uint4*>(obrow + ((j ^ (i & 15)) << 4)) =
                                        make_uint4(ob[4 * u], ob[4 * u + 1], ob[4 * u + 2], ob[4 * u + 3]);
                                }
                            }
                        }
                    }
                    // O read before the next call's first P V
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&aux->o_free[mt]);
                }
                ++eb;
            }
            if (ok && n_calls > 0) {  // every item with calls ends in a call-A epilogue
                const int row0 = inf->row0, seg_end = inf->seg_end, h0 = inf->h0;
                for (int mt = 0; mt < nmt && ok; ++mt) {
                    if (!mbar_wait(&aux->y_full[mt], (uint32_t)ea & 1u, abort_flag, status,
                                   STATUS_ATTN_SOFTMAX)) {
                        ok = false;
                        break;
                    }
                    const float amax = aux->ep_amax[mt][i];
                    const uint8_t* yrow = smem + OFF_OB + (mt * 128 + i) * OB_ROW;
                        const int row = row0 + qi;
                        const int h = h0 + 2 * mt + (i >> 6);
                        const float sc = UE8M0 ? ue8m0_scale(amax) : group_scale(amax);
                        const GroupDivider dv(sc);
                        const bool big = !(amax < 0x1p+100f);  // the quotient range bound
                        const float inv = ue8m0_inverse(sc);
                        uint8_t* out = q_out + ((int64_t)(row < seg_end ? row : row0) * n_q + h) * D;
#pragma unroll 1
                        for (int c0 = 0; c0 < D; c0 += 32) {
                            uint32_t yv[16];
#pragma unroll
                            for (int u = 0; u < 4; ++u) {
                                const int j = (c0 >> 3) + u;
                                const uint4 v4 = *reinterpret_cast<const uint4*>(yrow + ((j ^ (i & 15)) << 4));
                                yv[4 * u] = v4.x;
                                yv[4 * u + 1] = v4.y;
                                yv[4 * u + 2] = v4.z;
                                yv[4 * u + 3] = v4.w;
                            }
                            float qv[32];
                            bool rare = UE8M0 ? false : big;
#pragma unroll
                            for (int j = 0; j < 16; ++j) {
                                qv[2 * j] = __uint_as_float(yv[j] << 16);
                                qv[2 * j + 1] = __uint_as_float(yv[j] & 0xFFFF0000u);
                                if (UE8M0) {  // y * 2^-e, exact
                                    f2unpack(f2mul(f2pack(qv[2 * j], qv[2 * j + 1]),
                                                   f2pack(inv, inv)),
                                             qv[2 * j], qv[2 * j + 1]);
                                } else {
                                    dv.quant2_sat(qv[2 * j], qv[2 * j + 1], rare);
                                }
                            }
                            if (rare) {  // a zero, tiny or non-finite value: the exact path
#pragma unroll
                                for (int j = 0; j < 16; ++j) {
                                    float a = __uint_as_float(yv[j] << 16);
                                    float b = __uint_as_float(yv[j] & 0xFFFF0000u);
                                    dv.quant2(a, b);
                                    qv[2 * j] = a;
                                    qv[2 * j + 1] = b;
                                }
                            }
                            uint32_t packed[8];
#pragma unroll
                            for (int j = 0; j < 32; j += 4)
                                packed[j >> 2] = (uint32_t)fp8x2(qv[j], qv[j + 1]) |
                                                 ((uint32_t)fp8x2(qv[j + 2], qv[j + 3]) << 16);
                            if (row < seg_end) {
                                uint4* o4 = reinterpret_cast<uint4*>(out + c0);
                                o4[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
                                o4[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
                            }
                        }
                        if (row < seg_end) scale_out[(int64_t)h * scale_ld + row] = sc;
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&aux->y_empty[mt]);
                }
                ++ea;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&aux->info_empty[slot]);
        }
    } else {
        // ------- softmax, then each call's epilogue: one thread per row of an M tile -------
        const int mt = (warp - FIRST_SOFT) >> 2;
        if (mt < nmt) {
            const int q4 = warp & 3;
            const int i = q4 * 32 + lane;
            const int qi = i & (QR - 1);
            const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
            const uint32_t o_addr = tmem + lane_off + TM_O + (uint32_t)(mt * 128);
            // this row's call-B output (bf16): 16-byte chunk j at (j ^ i % 16) * 16
            uint8_t* obrow = smem + OFF_OB + (mt * 128 + i) * OB_ROW;
            const float sl2 = __fmul_rn(scale, 1.44269504088896341f);
            const uint64_t sl = f2pack(sl2, sl2);
            // tiles; call-A and call-B epilogues handed to the store warps,
            // and the call-B ones seen through
            int g = 0, ea = 0, eb = 0, ebw = 0;
            bool ok = true;
            for (int item = blockIdx.x, k = 0; item < n_items && ok; item += gridDim.x, ++k) {
                const int slot = k & 1;
                if (!mbar_wait(&aux->info_full[slot], (uint32_t)(k >> 1) & 1u, abort_flag, status,
                               STATUS_ATTN_SOFTMAX))
                    break;
                const Info* inf = &aux->info[slot];
                const int n_calls = inf->n_calls;
                float lse_b = 0.0f;  // this row's call-B log-sum-exp
                for (int c = 0; c < n_calls && ok; ++c) {
                    const Call cl = inf->calls[c];
                    const bool causal = cl.kind != CALL_READS;
                    const int qpos = cl.q_first + qi;
                    // keys [0, visible) exist for this row
                    const int visible = causal ? min(cl.key_end, qpos + 1) : cl.key_end;
                    float m = -INFINITY;
                    // eight row-sum partials (key j of a tile goes to partial
                    // j % 8) as four f32x2 pairs: L[q] holds partials 2q, 2q + 1
                    uint64_t L[4] = {0, 0, 0, 0};
                    for (int t = 0; t < cl.n_tiles; ++t, ++g) {
                        // S of this tile in buffer g & 1; its P goes over it
                        const uint32_t s_addr =
                            tmem + lane_off + TM_S + (uint32_t)(mt * 128 + (g & 1) * 64);
                        if (!mbar_wait(&aux->s_full[g & 1][mt], (uint32_t)(g >> 1) & 1u, abort_flag,
                                       status, STATUS_ATTN_SOFTMAX)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const int lim = visible - t * KT;  // keys [0, lim) of the tile exist
                        // warp-uniform: every lane sees the whole tile (no
                        // masking), and how many 16-key chunks any lane sees
                        // (later chunks are masked for the whole warp: skipped)
                        const bool whole = __all_sync(0xffffffffu, lim >= KT);
                        const int seen = __reduce_max_sync(0xffffffffu, (unsigned)max(lim, 0));
                        const int chunks = min(KT / 16, (seen + 15) >> 4);
                        // pass 1: the masked row max
                        float mx = -INFINITY;
#pragma unroll 1
                        for (int c0 = 0; c0 < chunks * 16; c0 += 16) {
                            uint32_t sr[16];
                            tmem_ld16_nowait(s_addr + (uint32_t)c0, sr);
                            tmem_wait_ld();
                            if (whole) {
#pragma unroll
                                for (int k = 0; k < 16; k += 2)
                                    mx = fmax3(mx, __uint_as_float(sr[k]), __uint_as_float(sr[k + 1]));
                            } else {
#pragma unroll
                                for (int k = 0; k < 16; k += 2)
                                    mx = fmax3(mx, c0 + k < lim ? __uint_as_float(sr[k]) : -INFINITY,
                                               c0 + k + 1 < lim ? __uint_as_float(sr[k + 1]) : -INFINITY);
                            }
                        }
                        const float m_new = fmaxf(m, mx);
                        float alpha, msl;
                        if (m_new == -INFINITY) {
                            alpha = 1.0f;
                            msl = 0.0f;
                        } else {
                            alpha = qexp2s(__fmul_rn(__fsub_rn(m, m_new), sl2));
                            msl = __fmul_rn(m_new, sl2);
                        }
                        m = m_new;
                        const uint64_t a2 = f2pack(alpha, alpha);
#pragma unroll
                        for (int q = 0; q < 4; ++q) L[q] = f2mul(L[q], a2);
                        const uint64_t nm = f2pack(-msl, -msl);
                        // pass 2: p = exp2(s sl2 - m sl2), the row-sum partials, bf16 P
#pragma unroll 1
                        for (int c0 = 0; c0 < KT; c0 += 16) {
                            uint32_t pk[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                            if (c0 < chunks * 16) {
                                uint32_t sr[16];
                                tmem_ld16_nowait(s_addr + (uint32_t)c0, sr);
                                tmem_wait_ld();
                                float pv[16];
#pragma unroll
                                for (int k = 0; k < 16; k += 2) {
                                    float s0 = __uint_as_float(sr[k]), s1 = __uint_as_float(sr[k + 1]);
                                    if (!whole) {
                                        s0 = c0 + k < lim ? s0 : -INFINITY;
                                        s1 = c0 + k + 1 < lim ? s1 : -INFINITY;
                                    }
                                    f2unpack(f2fma(f2pack(s0, s1), sl, nm), pv[k], pv[k + 1]);
                                    qexp2s_x2(pv[k], pv[k + 1]);
                                }
#pragma unroll
                                for (int k = 0; k < 16; k += 2) {
                                    // keys c0 + k, + 1 (c0 % 8 == 0): partials k % 8, k % 8 + 1
                                    L[(k >> 1) & 3] = f2add(L[(k >> 1) & 3], f2pack(pv[k], pv[k + 1]));
                                    pk[k >> 1] = bf16x2_bits(pv[k], pv[k + 1]);
                                }
                            }
                            // keys c0 .. c0 + 15 as 8 bf16 pairs over S columns c0 / 2 ..
                            // (already read: this chunk's S is in registers)
                            tmem_st8(s_addr + (uint32_t)(c0 >> 1), pk);
                        }
                        if (t > 0) {
                            // O *= alpha before this tile's P V, once the P V
                            // before it (the last to write O) is done
                            if (!mbar_wait(&aux->pv_done[(g - 1) & 1][mt],
                                           (uint32_t)((g - 1) >> 1) & 1u, abort_flag, status,
                                           STATUS_ATTN_SOFTMAX)) {
                                tmem_wait_st();
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            if (__any_sync(0xffffffffu, alpha != 1.0f)) {
                                const uint64_t a2 = f2pack(alpha, alpha);
#pragma unroll 1
                                for (int c0 = 0; c0 < D; c0 += 32) {
                                    uint32_t r[32];
                                    tmem_ld32_nowait(o_addr + (uint32_t)c0, r);
                                    tmem_wait_ld();
#pragma unroll
                                    for (int j = 0; j < 32; j += 2) {
                                        float x, y;
                                        f2unpack(f2mul(f2pack(__uint_as_float(r[j]),
                                                              __uint_as_float(r[j + 1])),
                                                       a2),
                                                 x, y);
                                        r[j] = __float_as_uint(x);
                                        r[j + 1] = __float_as_uint(y);
                                    }
                                    tmem_st32(o_addr + (uint32_t)c0, r);
                                }
                            }
                        }
                        // P (and O rescaled) stored before the P V reads them
                        tmem_wait_st();
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&aux->p_full[g & 1][mt]);
                    }
                    if (!ok) break;
                    // ---- epilogue of call c for this row ----
                    float lsum[8];
#pragma unroll
                    for (int q = 0; q < 4; ++q) f2unpack(L[q], lsum[2 * q], lsum[2 * q + 1]);
                    const float l = __fadd_rn(__fadd_rn(__fadd_rn(lsum[0], lsum[1]), __fadd_rn(lsum[2], lsum[3])),
                                              __fadd_rn(__fadd_rn(lsum[4], lsum[5]), __fadd_rn(lsum[6], lsum[7])));
                    const float inv = __frcp_rn(l);
                    if (cl.kind == CALL_READS) {
                        // the normalised call-B output (bf16, for the rows of this
                        // read group) is the store warps' work: they wait for the
                        // call's last P V, read O and leave it in shared memory
                        if (inf->s_grp[qi] == cl.group) lse_b = __fmaf_rn(m, scale, qlnf(l));
                        aux->ep_inv[mt][i] = inv;
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&aux->b_full[mt]);
                        ++eb;
                        continue;
                    }
                    // call A: its last P V done, the store warps through with the
                    // last item's rows and with this item's call-B outputs
                    bool got = mbar_wait(&aux->pv_done[(g - 1) & 1][mt], (uint32_t)((g - 1) >> 1) & 1u,
                                         abort_flag, status, STATUS_ATTN_SOFTMAX);
                    if (got && ea > 0)
                        got = mbar_wait(&aux->y_empty[mt], (uint32_t)(ea - 1) & 1u, abort_flag, status,
                                        STATUS_ATTN_SOFTMAX);
                    for (; got && ebw < eb; ++ebw)
                        got = mbar_wait(&aux->o_free[mt], (uint32_t)ebw & 1u, abort_flag, status,
                                        STATUS_ATTN_SOFTMAX);
                    if (!got) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    {
                        // merge with call B, per-head fp8 quantisation, store
                        const float lse_a = __fmaf_rn(m, scale, qlnf(l));
                        const bool has_b = !UNIFIED && inf->s_grp[qi] >= 0;
                        float w = 0.0f;
                        if (has_b) w = bf16_round(sigmoidf_ref(__fsub_rn(lse_b, lse_a)));
                        const uint64_t inv2 = f2pack(inv, inv), w2 = f2pack(w, w);
                        // pass 1: the merged row (bf16) over the row's call-B output
                        // (each chunk read before it is overwritten) and its amax;
                        // pass 2: from there, quantised and stored
                        uint8_t* yrow = obrow;
                        float amax = 0.0f;
#pragma unroll 1
                        for (int c0 = 0; c0 < D; c0 += 32) {
                            uint32_t r[32], ob[16];
                            tmem_ld32_nowait(o_addr + (uint32_t)c0, r);
                            if (has_b) {
#pragma unroll
                                for (int u = 0; u < 4; ++u) {
                                    const int j = (c0 >> 3) + u;
                                    const uint4 b4 = *reinterpret_cast<const uint4*>(obrow + ((j ^ (i & 15)) << 4));
                                    ob[4 * u] = b4.x;
                                    ob[4 * u + 1] = b4.y;
                                    ob[4 * u + 2] = b4.z;
                                    ob[4 * u + 3] = b4.w;
                                }
                            } else {
#pragma unroll
                                for (int j = 0; j < 16; ++j) ob[j] = 0;
                            }
                            tmem_wait_ld();
                            uint32_t yv[16];
#pragma unroll
                            for (int j = 0; j < 16; ++j) {
                                yv[j] = merge_pair(r[2 * j], r[2 * j + 1], ob[j], inv2, w2, has_b);
                                amax = fmaxf(amax, fabsf(__uint_as_float(yv[j] << 16)));
                                amax = fmaxf(amax, fabsf(__uint_as_float(yv[j] & 0xFFFF0000u)));
                            }
#pragma unroll
                            for (int u = 0; u < 4; ++u) {
                                const int j = (c0 >> 3) + u;
                                *reinterpret_cast<uint4*>(yrow + ((j ^ (i & 15)) << 4)) =
                                    make_uint4(yv[4 * u], yv[4 * u + 1], yv[4 * u + 2], yv[4 * u + 3]);
                            }
                        }
                        // pass 2 (quantisation and store) goes to the store warps
                        aux->ep_amax[mt][i] = amax;
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&aux->y_full[mt]);
                        ++ea;
                    }
                    // O (and the call-B output) read before the next call's first P V
                    tc_fence_before();
                }
                // done with the item's info (its calls and epilogues are through)
                __syncwarp();
                if (lane == 0) mbar_arrive(&aux->info_empty[slot]);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem)
                     : "memory");
    }
}

}  // namespace attn_tc

// Launch of the tcgen05 kernel; returns -1 when the shapes are not its
// (odd GQA group, page size not dividing 64), the caller then uses the
// mma.sync kernel.
int launch_attention_tc(bool unified, const char* who, const void* q, const void* k,
                        const void* v, int64_t rows, int n_q, int n_kv, const int32_t* cu,
                        const int32_t* tiles, int64_t n_tiles, const int32_t* read_cu_q,
                        const int32_t* read_used, const int32_t* table, int64_t n_reads,
                        int64_t table_width, const int32_t* source, const void* k_pool,
                        const void* v_pool, int64_t n_pages, int page_tokens,
                        float softmax_scale, void* q_out, float* scale_out, int64_t scale_ld,
                        bool ue8m0, void* stream) {
    using namespace attn_tc;
    const int group = n_q / n_kv;
    if (group % 2 != 0) return -1;
    const int hp = group % 4 == 0 ? 4 : 2;
    const bool paged = unified || n_reads > 0;
    if (paged && (page_tokens <= 0 || KT % page_tokens != 0 || page_tokens < 8)) return -1;
    if (!unified && rows < 1) return QB_OK;
    uint32_t* status = device_status_ptr();
    if (!status) return launch_status(who);
    CUtensorMap mq, mk, mv, mkp, mvp;
    const CUtensorMapDataType bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B;
    int st = encode_2d(&mq, bf, q, (int64_t)n_q * D, rows, (int64_t)n_q * D * 2, 64, QR, sw, who);
    if (st) return st;
    if (!unified) {
        st = encode_2d(&mk, bf, k, (int64_t)n_kv * D, rows, (int64_t)n_kv * D * 2, 64, KT, sw, who);
        if (st) return st;
        st = encode_2d(&mv, bf, v, (int64_t)n_kv * D, rows, (int64_t)n_kv * D * 2, 64, KT, sw, who);
        if (st) return st;
    } else {
        mk = mq;
        mv = mq;
    }
    if (paged) {
        const int64_t pool_rows = n_pages * (int64_t)page_tokens;
        st = encode_2d(&mkp, bf, k_pool, (int64_t)n_kv * D, pool_rows, (int64_t)n_kv * D * 2, 64,
                       page_tokens, sw, who);
        if (st) return st;
        st = encode_2d(&mvp, bf, v_pool, (int64_t)n_kv * D, pool_rows, (int64_t)n_kv * D * 2, 64,
                       page_tokens, sw, who);
        if (st) return st;
    } else {
        mkp = mk;
        mvp = mv;
    }
    auto kernel = unified ? (ue8m0 ? attention_tc_kernel<true, true> : attention_tc_kernel<true, false>)
                          : (ue8m0 ? attention_tc_kernel<false, true> : attention_tc_kernel<false, false>);
    static std::atomic<bool> attr[2][2][MAX_DEVICES];
    if (!set_smem_once(attr[unified][ue8m0], kernel, (int)SMEM_BYTES)) return launch_status(who);
    // persistent: one block per SM walks the items (query tile x head group,
    // head groups of a tile adjacent so they share K/V in L2)
    const int64_t items = n_tiles * (int64_t)(n_kv * (group / hp));
    if (items > 0x7fffffffLL) return invalid("attention: too many work items");
    const int64_t sms = sm_count();
    const unsigned grid = (unsigned)(items < sms ? items : sms);
    kernel<<<grid, NUM_THREADS, SMEM_BYTES, (cudaStream_t)stream>>>(
        mq, mk, mv, mkp, mvp, rows, n_q, n_kv, hp, cu, tiles, (int)n_tiles, read_cu_q, read_used,
        table, n_reads, table_width, source, n_pages, page_tokens, softmax_scale,
        (uint8_t*)q_out, scale_out, scale_ld, status);
    return launch_status(who);
}

}  // namespace qb
