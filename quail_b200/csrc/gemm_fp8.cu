// FP8 e4m3 block-scaled GEMM on tcgen05 tensor cores (sm_100a).
//
//   out[m, n] = bf16( sum_kb P_kb[m, n] * a_scale[kb, m] * w_scale[n / 128, kb] )
//   P_kb[m, n] = sum_{k in block kb} a[m, k] * w[n, k]        (128-wide K blocks)
//
// The scales are arbitrary fp32 values (1x128 for activations, 128x128 for
// weights), so they cannot ride on the MX block-scale hardware path (UE8M0
// only); each 128-deep K block is accumulated by the tensor cores into its
// own TMEM buffer and promoted into fp32 registers by the epilogue warps with
// that block's scales, while the tensor cores fill the next buffer.
//
// Persistent kernel, one block per SM, 19 warps:
//   warp 0      TMA producer: A [128 x 128] and W [BN x 128] tiles into a
//               4-stage shared-memory ring (128-byte swizzle), one mbarrier
//               transaction per stage;
//   warp 1      allocates TMEM (512 columns: 512 / BN accumulator buffers)
//               and issues tcgen05.mma
//               (M=128, N=BN, K=32, kind::f8f6f4) from one thread;
//   warp 2      scale loader: the K block's 128 activation scales and BN/128
//               weight scales into an 8-slot shared-memory ring by cp.async,
//               up to 8 K blocks ahead of the epilogue (the activation scales
//               stream from HBM, and a load issued one K block ahead stalls
//               the promotion on DRAM latency);
//   warps 3-18  epilogue: warp w reads TMEM lanes 32*(w%4).. (its rows) and
//               columns (w-3)/4 * BN/4 .. (its slice), scales and accumulates.
// No cluster launch and no TMA multicast: every block loads its own tiles.
//
// SILU (the MLP's gate_up projection, weights [gate; up] of inter rows
// each): a 256-wide tile is 128 gate columns j*128.. and the same 128 up
// columns inter + j*128.. (two 128-row weight boxes), and the epilogue
// writes q = fp8(silu(bf16 gate) * bf16 up / scale) with one scale per row
// and tile (one 128-column quantisation group) instead of the bf16
// product: the same bits as the bf16 GEMM followed by qb_silu_mul_quant.
// Epilogue warp w holds gate columns 32*(w-3)/4.. and the matching up
// columns of its rows; the row's group max is exchanged between the four
// warps of the same rows through shared memory and an mbarrier.
// Every mbarrier wait is bounded (about one second); a wait that gives up
// sets a status bit, makes the other roles stop, drains the copies and MMAs
// in flight and frees TMEM before the block exits.
#include <cudaTypedefs.h>

#include <type_traits>

#include "tc_common.cuh"

namespace {

using namespace qb;
using namespace qb::tc;

constexpr int BM = 128;
constexpr int BK = 128;
constexpr int MAX_STAGES = 4;
constexpr int EPI_WARPS = 16;
constexpr int FIRST_EPI_WARP = 3;
constexpr int NUM_THREADS = (FIRST_EPI_WARP + EPI_WARPS) * 32;
constexpr int SCALE_SLOTS = 8;

// BN: tile width; NST: shared-memory pipeline stages; TSTORE: the tile is
// written through a 128-byte-swizzled shared-memory staging area by TMA
// stores (one 32 x 64 box per epilogue warp) instead of per-thread row
// stores, so the epilogue returns to the next tile at once.
template <int BN, int NST = MAX_STAGES, bool TSTORE = false, bool SILU = false>
struct Cfg {
    static constexpr int STAGES = NST;
    static_assert(NST >= 2 && NST <= MAX_STAGES, "stages");
    static constexpr int A_BYTES = BM * BK;
    static constexpr int B_BYTES = BN * BK;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int NBUF = 512 / BN;       // accumulator buffers in TMEM
    static constexpr int TMEM_COLS = NBUF * BN;  // all 512 columns
    static constexpr int SLICE = BN / 4;      // columns per epilogue warp
    static_assert(!TSTORE || SLICE == 64, "TMA-store staging rows are 128 bytes");
    static constexpr int OUT_BYTES = TSTORE ? EPI_WARPS * 32 * SLICE * 2 : 0;
    static constexpr int SCALE_OFF = STAGES * STAGE_BYTES + OUT_BYTES;
    static_assert(!SILU || (BN == 256 && !TSTORE), "SILU tiles are 128 gate + 128 up columns");
    // SILU: per-row group max partials, [2 tile parities][4 slices][BM rows]
    static constexpr int RED_OFF = SCALE_OFF + SCALE_SLOTS * 528;
    static constexpr int RED_BYTES = SILU ? 2 * 4 * BM * 4 : 0;
    static constexpr int BAR_OFF = RED_OFF + RED_BYTES;
    static constexpr int BAR_BYTES = 512;
    static constexpr int SMEM = BAR_OFF + BAR_BYTES + 1024;
    // instruction descriptor: D f32, A/B e4m3, both K-major, N, M=128
    static constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(BN >> 3) << 17) |
                                      ((uint32_t)(BM >> 4) << 24);
};

// one K block's scales: a[r] for tile row r (0 past the last row), w[j] for
// the tile's j-th 128-column weight block
struct ScaleSlot {
    float a[BM];
    float w[4];
};
static_assert(sizeof(ScaleSlot) == 528, "scale slot layout");

struct Barriers {
    uint64_t full[MAX_STAGES];
    uint64_t empty[MAX_STAGES];
    uint64_t tmem_full[4];
    uint64_t tmem_empty[4];
    uint64_t scale_full[SCALE_SLOTS];
    uint64_t scale_empty[SCALE_SLOTS];
    uint64_t drain;
    uint64_t red_full[2];  // SILU: a tile's group-max partials are in shared memory
    uint32_t tmem_base;
    int abort;
};

__device__ __forceinline__ void mma_f8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// acc[0..1] = fma(v[0..1], s, acc[0..1]): two IEEE fp32 FMAs in one
// instruction (fma.rn.f32x2), each rounded exactly as fmaf would.
__device__ __forceinline__ void fma2(float* acc, const uint32_t* v, float s) {
    uint64_t a, x, y;
    asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(acc[0]), "f"(acc[1]));
    asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "r"(v[0]), "r"(v[1]));
    asm("mov.b64 %0, {%1, %1};" : "=l"(y) : "f"(s));
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(a) : "l"(x), "l"(y));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(acc[0]), "=f"(acc[1]) : "l"(a));
}

// OutT = bf16 (the library) or float (numerics probes: the fp32 accumulator);
// uint8_t with SILU (fp8 e4m3 rows of N/2 columns, their scales at
// q_scale[j * q_scale_ld + row]).
// map_c (bf16 out, box 64 x 32, 128-byte swizzle) is read only when TSTORE.
template <int BN, typename OutT = bf16, int NST = MAX_STAGES, bool TSTORE = false,
          bool SILU = false>
__global__ void __launch_bounds__(NUM_THREADS, 1)
gemm_fp8_bs_kernel(const __grid_constant__ CUtensorMap map_a,
                   const __grid_constant__ CUtensorMap map_b,
                   const __grid_constant__ CUtensorMap map_c, const float* __restrict__ a_scale,
                   int64_t a_scale_ld, const float* __restrict__ w_scale, OutT* __restrict__ out,
                   float* __restrict__ q_scale, int64_t q_scale_ld, int M, int N, int K,
                   uint32_t* status) {
    using C = Cfg<BN, NST, TSTORE, SILU>;
    constexpr int STAGES = C::STAGES;
    static_assert(!TSTORE || sizeof(OutT) == 2, "TMA stores write bf16");
    static_assert(!SILU || sizeof(OutT) == 1, "SILU writes fp8");
    extern __shared__ uint8_t smem_raw[];
    // SWIZZLE_128B tiles need 1024-byte aligned shared memory
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
    ScaleSlot* scales = reinterpret_cast<ScaleSlot*>(smem + C::SCALE_OFF);
    Barriers* bars = reinterpret_cast<Barriers*>(smem + C::BAR_OFF);
    volatile int* abort_flag = &bars->abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int num_n = N / BN;
    const int num_m = (M + BM - 1) / BM;
    const int total = num_m * num_n;
    const int n_kb = K / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], 1);
        }
        for (int b = 0; b < C::NBUF; ++b) {
            mbar_init(&bars->tmem_full[b], 1);
            mbar_init(&bars->tmem_empty[b], EPI_WARPS);
        }
        for (int s = 0; s < SCALE_SLOTS; ++s) {
            mbar_init(&bars->scale_full[s], 32);
            mbar_init(&bars->scale_empty[s], EPI_WARPS);
        }
        mbar_init(&bars->drain, 1);
        mbar_init(&bars->red_full[0], EPI_WARPS);
        mbar_init(&bars->red_full[1], EPI_WARPS);
        bars->abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&bars->tmem_base)),
                     "r"(C::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = bars->tmem_base;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a))
                         : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_b))
                         : "memory");
            int it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
                const int m0 = (tile / num_n) * BM, n0 = (tile % num_n) * BN;
                for (int kb = 0; kb < n_kb; ++kb, ++it) {
                    const int s = it % STAGES;
                    const uint32_t round = (uint32_t)(it / STAGES);
                    if (!mbar_wait(&bars->empty[s], (round & 1u) ^ 1u, abort_flag, status,
                                   STATUS_GEMM_PRODUCER)) {
                        ok = false;
                        break;
                    }
                    uint8_t* sa = smem + s * C::STAGE_BYTES;
                    mbar_arrive_expect_tx(&bars->full[s], C::STAGE_BYTES);
                    tma_load_2d(smem_u32(sa), &map_a, kb * BK, m0, &bars->full[s]);
                    if constexpr (SILU) {
                        // gate rows j*128.., up rows N/2 + j*128..: one 256-row tile
                        const int j0 = (tile % num_n) * 128;
                        tma_load_2d(smem_u32(sa + C::A_BYTES), &map_b, kb * BK, j0,
                                    &bars->full[s]);
                        tma_load_2d(smem_u32(sa + C::A_BYTES + 128 * BK), &map_b, kb * BK,
                                    N / 2 + j0, &bars->full[s]);
                    } else {
                        tma_load_2d(smem_u32(sa + C::A_BYTES), &map_b, kb * BK, n0,
                                    &bars->full[s]);
                    }
                }
            }
            // no copy may still be landing when the block exits: wait for the
            // last load issued on each stage
            for (int j = (it > STAGES ? it - STAGES : 0); j < it; ++j) {
                const int s = j % STAGES;
                if (!mbar_try_wait(smem_u32(&bars->full[s]), (uint32_t)(j / STAGES) & 1u)) {
                    int flag = 0;
                    mbar_wait(&bars->full[s], (uint32_t)(j / STAGES) & 1u, &flag, status,
                              STATUS_GEMM_DRAIN);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int it = 0, acc_it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
                for (int kb = 0; kb < n_kb; ++kb, ++it, ++acc_it) {
                    const int s = it % STAGES;
                    if (!mbar_wait(&bars->full[s], (uint32_t)(it / STAGES) & 1u, abort_flag,
                                   status, STATUS_GEMM_MMA)) {
                        ok = false;
                        break;
                    }
                    const int buf = acc_it % C::NBUF;
                    const uint32_t use = (uint32_t)(acc_it / C::NBUF);
                    if (!mbar_wait(&bars->tmem_empty[buf], (use & 1u) ^ 1u, abort_flag, status,
                                   STATUS_GEMM_MMA)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + s * C::STAGE_BYTES);
                    const uint64_t adesc = sw128_desc(sa);
                    const uint64_t bdesc = sw128_desc(sa + C::A_BYTES);
                    const uint32_t d = tmem_base + (uint32_t)(buf * BN);
#pragma unroll
                    for (int k = 0; k < BK / 32; ++k)  // 32 bytes of K per MMA
                        mma_f8(d, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), C::IDESC,
                               k > 0 ? 1u : 0u);
                    mma_commit(&bars->empty[s]);
                    mma_commit(&bars->tmem_full[buf]);
                }
            }
            // every MMA issued must finish before TMEM is freed
            mma_commit(&bars->drain);
            int flag = 0;
            mbar_wait(&bars->drain, 0, &flag, status, STATUS_GEMM_DRAIN);
        }
    } else if (warp == 2) {
        // ---------------- scale loader ----------------
        int it = 0;
        constexpr int NB = BN / 128;
        for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
            const int m0 = (tile / num_n) * BM, n0 = (tile % num_n) * BN;
            bool ok = true;
            for (int kb = 0; kb < n_kb; ++kb, ++it) {
                const int slot = it % SCALE_SLOTS;
                const uint32_t round = (uint32_t)(it / SCALE_SLOTS);
                if (!mbar_wait(&bars->scale_empty[slot], (round & 1u) ^ 1u, abort_flag, status,
                               STATUS_GEMM_EPILOGUE)) {
                    ok = false;
                    break;
                }
                ScaleSlot* sl = scales + slot;
                const float* col = a_scale + (int64_t)kb * a_scale_ld;
#pragma unroll
                for (int j = 0; j < BM / 32; ++j) {
                    const int r = j * 32 + lane;
                    const bool valid = m0 + r < M;
                    cp_async4(smem_u32(&sl->a[r]), valid ? col + m0 + r : a_scale,
                              valid ? 4u : 0u);
                }
                if (lane < NB) {
                    // the weight block of the tile's lane-th 128 columns
                    const int wb = SILU ? (tile % num_n) + lane * (N / 256) : n0 / 128 + lane;
                    cp_async4(smem_u32(&sl->w[lane]), w_scale + (int64_t)wb * n_kb + kb, 4u);
                }
                cp_async_arrive(&bars->scale_full[slot]);
            }
            if (!ok) break;
        }
        // copies still in flight complete on their own; none may land after exit
        asm volatile("cp.async.wait_all;" ::: "memory");
    } else {
        // ---------------- epilogue: promote, accumulate, store ----------------
        const int ew = warp - FIRST_EPI_WARP;
        const int quarter = warp & 3;          // TMEM lanes this warp may access
        // its column slice (SILU: gate columns col0.., up columns 128 + col0..)
        const int col0 = (ew >> 2) * (SILU ? 32 : C::SLICE);
        const int row_in_tile = quarter * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
        int acc_it = 0, tcount = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, ++tcount) {
            const int m0 = (tile / num_n) * BM, n0 = (tile % num_n) * BN;
            const int m = m0 + row_in_tile;
            const bool valid = m < M;
            const int wblk = col0 / 128;
            float acc[C::SLICE];
#pragma unroll
            for (int j = 0; j < C::SLICE; ++j) acc[j] = 0.0f;
            for (int kb = 0; kb < n_kb; ++kb, ++acc_it) {
                const int slot = acc_it % SCALE_SLOTS;
                if (!mbar_wait(&bars->scale_full[slot], (uint32_t)(acc_it / SCALE_SLOTS) & 1u,
                               abort_flag, status, STATUS_GEMM_EPILOGUE)) {
                    ok = false;
                    break;
                }
                const float a_sc = scales[slot].a[row_in_tile];
                const float sc = a_sc * scales[slot].w[SILU ? 0 : wblk];
                const float sc_up = SILU ? a_sc * scales[slot].w[1] : sc;
                const int buf = acc_it % C::NBUF;
                if (!mbar_wait(&bars->tmem_full[buf], (uint32_t)(acc_it / C::NBUF) & 1u, abort_flag,
                               status, STATUS_GEMM_EPILOGUE)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t taddr = tmem_base + lane_addr + (uint32_t)(buf * BN + col0);
#pragma unroll
                for (int c = 0; c < C::SLICE; c += 32) {
                    // two loads in flight per wait
                    uint32_t v[32];
                    // SILU: the second 32 columns are the up half's
                    const uint32_t cc = (SILU && c > 0) ? 128u : (uint32_t)c;
                    tmem_ld16_nowait(taddr + cc, v);
                    tmem_ld16_nowait(taddr + cc + 16u, v + 16);
                    tmem_wait_ld();
                    if (c + 32 >= C::SLICE) {
                        // the buffer's last columns are in registers: hand it
                        // back to the MMA before the last FMAs
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) {
                            mbar_arrive(&bars->tmem_empty[buf]);
                            mbar_arrive(&bars->scale_empty[slot]);
                        }
                    }
#pragma unroll
                    for (int j = 0; j < 32; j += 2)
                        fma2(acc + c + j, v + j, (SILU && c > 0) ? sc_up : sc);
                }
            }
            if (!ok) break;
            if constexpr (SILU) {
                // y = (g sigmoid(g)) u on the bf16-rounded accumulators, as
                // qb_silu_mul_quant computes it from the bf16 GEMM output
                float amax = 0.0f;
#pragma unroll
                for (int i = 0; i < 32; i += 2) {
                    const bf162 g2 = __floats2bfloat162_rn(acc[i], acc[i + 1]);
                    const bf162 u2 = __floats2bfloat162_rn(acc[32 + i], acc[33 + i]);
                    const float g0 = __low2float(g2), g1 = __high2float(g2);
                    float sa = g0, sb = g1;
                    bool rare = false;
                    sigmoidf_ref_x2_fast(sa, sb, rare);
                    if (rare) {  // g below about -86 or NaN: the exact path
                        sa = g0;
                        sb = g1;
                        sigmoidf_ref_x2(sa, sb);
                    }
                    const uint64_t gs = f2mul(f2pack(g0, g1), f2pack(sa, sb));
                    f2unpack(f2mul(gs, f2pack(__low2float(u2), __high2float(u2))), acc[i],
                             acc[i + 1]);
                    amax = fmaxf(amax, fabsf(acc[i]));
                    amax = fmaxf(amax, fabsf(acc[i + 1]));
                }
                // the row's group max over the four warps of its 128 columns
                float* red = reinterpret_cast<float*>(smem + C::RED_OFF) + (tcount & 1) * 4 * BM;
                red[(ew >> 2) * BM + row_in_tile] = amax;
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars->red_full[tcount & 1]);
                if (!mbar_wait(&bars->red_full[tcount & 1], (uint32_t)(tcount >> 1) & 1u,
                               abort_flag, status, STATUS_GEMM_EPILOGUE)) {
                    ok = false;
                    break;
                }
                amax = fmaxf(fmaxf(red[row_in_tile], red[BM + row_in_tile]),
                             fmaxf(red[2 * BM + row_in_tile], red[3 * BM + row_in_tile]));
                const float scale = group_scale(amax);
                const GroupDivider dv(scale);
                const bool big = !(amax < 0x1p+100f);
                uint32_t pk[8];
#pragma unroll
                for (int i = 0; i < 32; i += 4) {
                    float a = acc[i], b = acc[i + 1], c = acc[i + 2], d = acc[i + 3];
                    bool rare = big;
                    dv.quant2_sat(a, b, rare);
                    dv.quant2_sat(c, d, rare);
                    if (rare) {  // a zero, tiny or non-finite value: the exact path
                        a = acc[i];
                        b = acc[i + 1];
                        c = acc[i + 2];
                        d = acc[i + 3];
                        dv.quant2(a, b);
                        dv.quant2(c, d);
                    }
                    pk[i >> 2] = (uint32_t)fp8x2(a, b) | ((uint32_t)fp8x2(c, d) << 16);
                }
                if (valid) {
                    const int j = tile % num_n;
                    uint8_t* dst = reinterpret_cast<uint8_t*>(out) + (int64_t)m * (N / 2) +
                                   j * 128 + col0;
                    *reinterpret_cast<uint4*>(dst) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                    *reinterpret_cast<uint4*>(dst + 16) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                    if (col0 == 0) q_scale[(int64_t)j * q_scale_ld + m] = scale;
                }
            } else if constexpr (TSTORE) {
                // this warp's 32 rows x 64 columns, row r's 16-byte chunk j at
                // r * 128 + (j ^ r % 8) * 16: the 128-byte swizzle of map_c,
                // and conflict-free for one row per lane
                uint8_t* stage = smem + STAGES * C::STAGE_BYTES + ew * 4096;
                if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
                __syncwarp();
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    *reinterpret_cast<uint4*>(stage + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                        float_to_bf16x8(acc + 8 * j);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                // rows past M are clipped by the tensor map's bounds
                if (lane == 0 && m0 + quarter * 32 < M) {
                    tma_store_2d(&map_c, smem_u32(stage), n0 + col0, m0 + quarter * 32);
                    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                }
            } else if (valid) {
                OutT* dst = out + (int64_t)m * N + n0 + col0;
                if constexpr (sizeof(OutT) == 2) {
#pragma unroll
                    for (int j = 0; j < C::SLICE; j += 8)
                        *reinterpret_cast<uint4*>(dst + j) = float_to_bf16x8(acc + j);
                } else {
#pragma unroll
                    for (int j = 0; j < C::SLICE; j += 4)
                        *reinterpret_cast<float4*>(dst + j) =
                            make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
                }
            }
        }
        // the global writes of the last stores complete before the block exits
        if (TSTORE && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                     "r"(C::TMEM_COLS)
                     : "memory");
    }
}

// 2-D K-major fp8 tensor map: rows x k bytes, box box_rows x 128, 128B swizzle.
int make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t k, int box_rows) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = get_encoder();
    if (!enc) {
        set_error("qb_gemm_fp8_bs: cuTensorMapEncodeTiled unavailable");
        return QB_ERR_CUDA;
    }
    cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)k};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("qb_gemm_fp8_bs: cuTensorMapEncodeTiled failed (%d)", (int)r);
        return QB_ERR_CUDA;
    }
    return QB_OK;
}

// bf16 output map: rows x n, box 32 rows x 64 columns, 128-byte swizzle
int make_out_map(CUtensorMap* map, void* base, int64_t rows, int64_t n) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = get_encoder();
    if (!enc) {
        set_error("qb_gemm_fp8_bs: cuTensorMapEncodeTiled unavailable");
        return QB_ERR_CUDA;
    }
    cuuint64_t dims[2] = {(cuuint64_t)n, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)n * 2};
    cuuint32_t box[2] = {64, 32};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("qb_gemm_fp8_bs: cuTensorMapEncodeTiled (out) failed (%d)", (int)r);
        return QB_ERR_CUDA;
    }
    return QB_OK;
}

// SILU: n = 2 * inter weight rows, out fp8 [m, inter], q_scale [inter / 128, q_scale_ld]
template <int BN, int NST = MAX_STAGES, bool TSTORE = false, bool SILU = false>
int launch(const void* a, const float* a_scale, int64_t a_scale_ld, const void* w,
           const float* w_scale, void* out, int64_t m, int64_t n, int64_t k, cudaStream_t stream,
           float* q_scale = nullptr, int64_t q_scale_ld = 0) {
    using C = Cfg<BN, NST, TSTORE, SILU>;
    using OutT = typename std::conditional<SILU, uint8_t, bf16>::type;
    CUtensorMap map_a, map_b, map_c;
    memset(&map_c, 0, sizeof(map_c));
    int st = make_map(&map_a, a, m, k, BM);
    if (st) return st;
    st = make_map(&map_b, w, n, k, SILU ? 128 : BN);
    if (st) return st;
    if (TSTORE) {
        st = make_out_map(&map_c, out, m, n);
        if (st) return st;
    }
    auto kernel = gemm_fp8_bs_kernel<BN, OutT, NST, TSTORE, SILU>;
    static bool attr[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             C::SMEM);
        if (e != cudaSuccess) return launch_status("qb_gemm_fp8_bs: smem attribute");
        attr[dev] = true;
    }
    uint32_t* status = device_status_ptr();
    if (!status) return launch_status("qb_gemm_fp8_bs: status word");
    const int64_t tiles = ((m + BM - 1) / BM) * (n / BN);
    const int grid = (int)(tiles < sm_count() ? tiles : sm_count());
    kernel<<<grid, NUM_THREADS, C::SMEM, stream>>>(map_a, map_b, map_c, a_scale, a_scale_ld,
                                                   w_scale, (OutT*)out, q_scale, q_scale_ld,
                                                   (int)m, (int)n, (int)k, status);
    return launch_status(SILU ? "qb_gemm_fp8_silu_quant" : "qb_gemm_fp8_bs");
}

}  // namespace

extern "C" int qb_gemm_fp8_bs(const void* a, const float* a_scale, int64_t a_scale_ld,
                              const void* w, const float* w_scale, void* out, int64_t m, int64_t n,
                              int64_t k, void* stream) {
    if (m < 0 || n <= 0 || k <= 0) return invalid("qb_gemm_fp8_bs: bad sizes");
    if (k % BK != 0) return invalid("qb_gemm_fp8_bs: k must be a multiple of 128");
    if (n % 128 != 0) return invalid("qb_gemm_fp8_bs: n must be a multiple of 128");
    if (m > 0x7fffffffLL || n > 0x7fffffffLL || k > 0x7fffffffLL)
        return invalid("qb_gemm_fp8_bs: sizes exceed int32");
    if (a_scale_ld < m) return invalid("qb_gemm_fp8_bs: a_scale_ld < m");
    if (!aligned(a, 16) || !aligned(w, 16) || !aligned(out, 16))
        return invalid("qb_gemm_fp8_bs: a, w and out must be 16-byte aligned");
    if (!a_scale || !w_scale) return invalid("qb_gemm_fp8_bs: NULL scales");
    if (m == 0) return QB_OK;
    cudaStream_t s = (cudaStream_t)stream;
    // The TMA-store epilogue (3 stages, the tile staged in shared memory)
    // beats 4 stages with per-thread row stores on every 4B shape (measured on
    // B200: qkv 2,144 vs 1,815, o 2,200 vs 1,989, gate_up 1,973 vs 1,694,
    // down 2,324 vs 2,011 TFLOP/s at 110k rows).
    if (n % 256 == 0)
        return launch<256, 3, true>(a, a_scale, a_scale_ld, w, w_scale, out, m, n, k, s);
    return launch<128, 4, false>(a, a_scale, a_scale_ld, w, w_scale, out, m, n, k, s);
}

extern "C" int qb_gemm_fp8_silu_quant(const void* a, const float* a_scale, int64_t a_scale_ld,
                                      const void* w, const float* w_scale, void* q_out,
                                      float* scale_out, int64_t scale_ld, int64_t m,
                                      int64_t inter, int64_t k, void* stream) {
    if (m < 0 || inter <= 0 || k <= 0) return invalid("qb_gemm_fp8_silu_quant: bad sizes");
    if (k % BK != 0) return invalid("qb_gemm_fp8_silu_quant: k must be a multiple of 128");
    if (inter % 128 != 0)
        return invalid("qb_gemm_fp8_silu_quant: inter must be a multiple of 128");
    if (m > 0x7fffffffLL || 2 * inter > 0x7fffffffLL || k > 0x7fffffffLL)
        return invalid("qb_gemm_fp8_silu_quant: sizes exceed int32");
    if (a_scale_ld < m) return invalid("qb_gemm_fp8_silu_quant: a_scale_ld < m");
    if (scale_ld < m) return invalid("qb_gemm_fp8_silu_quant: scale_ld < m");
    if (!aligned(a, 16) || !aligned(w, 16) || !aligned(q_out, 16))
        return invalid("qb_gemm_fp8_silu_quant: a, w and q_out must be 16-byte aligned");
    if (!a_scale || !w_scale || !scale_out)
        return invalid("qb_gemm_fp8_silu_quant: NULL scales");
    if (m == 0) return QB_OK;
    return launch<256, 4, false, true>(a, a_scale, a_scale_ld, w, w_scale, q_out, m, 2 * inter,
                                       k, (cudaStream_t)stream, scale_out, scale_ld);
}
