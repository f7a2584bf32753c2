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
template <int BN, int NST = MAX_STAGES, bool TSTORE = false, bool SILU = false,
          bool ROPE = false, bool MX = false>
struct Cfg {
    static constexpr int STAGES = NST;
    static_assert(NST >= 2 && NST <= MAX_STAGES, "stages");
    static_assert(!MX || BN == 256, "UE8M0 tiles are 256 wide");
    static constexpr int A_BYTES = BM * BK;
    static constexpr int B_BYTES = BN * BK;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    // accumulator buffers in TMEM: 512 / BN K-block partials; MX one
    // whole-K accumulator in columns 0-255 and the stages' scale factors
    // from column TM_SF (12 columns a stage: SFA 4, SFB 8)
    static constexpr int NBUF = MX ? 1 : 512 / BN;
    static constexpr int TMEM_COLS = 512;
    static constexpr int TM_SF = 256;
    static_assert(!MX || TM_SF + 12 * NST <= TMEM_COLS, "scale-factor columns");
    // MX: raw fp32 scales land by cp.async RAW_SLOTS - 1 K blocks ahead of
    // their conversion into the SF ring (tcgen05.cp source layout)
    static constexpr int RAW_SLOTS = MX ? (ROPE ? 4 : 8) : SCALE_SLOTS;
    // MX: one SF slot per stage, filled and released with the stage (its
    // full barrier takes the scale loader's arrival besides the TMA bytes,
    // its empty barrier frees both), so the MMA thread waits and commits
    // once per K block
    static constexpr int SF_SLOTS = MX ? NST : 1;  // (1: keeps the MX-only code well formed)
    static constexpr int SF_BYTES = 1536;  // SFA 32 x 16 B, SFB 2 x 32 x 16 B
    static constexpr int SLICE = BN / 4;      // columns per epilogue warp
    static_assert(!TSTORE || SLICE == 64, "TMA-store staging rows are 128 bytes");
    // TSTORE: one 32 x 64 bf16 staging box per epilogue warp; ROPE: the same
    // 4 KB per warp holds the pair's sum-of-squares partials, then the two
    // 32 x 32 output boxes (64-byte swizzle)
    // SILU: one 32 x 32 fp8 box (1 KB) per epilogue warp
    // TSTORE with MX: the bf16 tile leaves in 32 x 16 boxes (32-byte
    // swizzle) through 1 KB per warp, so four operand stages fit
    static constexpr bool SMALL_OUT = TSTORE && MX;
    static constexpr int OUT_BYTES = SMALL_OUT           ? EPI_WARPS * 1024
                                     : (TSTORE || ROPE) ? EPI_WARPS * 32 * SLICE * 2
                                     : SILU             ? EPI_WARPS * 32 * 32
                                                        : 0;
    static constexpr int SCALE_OFF = STAGES * STAGE_BYTES + OUT_BYTES;
    static_assert(!SILU || (BN == 256 && !TSTORE), "SILU tiles are 128 gate + 128 up columns");
    static_assert(!ROPE || (BN == 256 && !TSTORE && !SILU), "ROPE tiles are two heads");
    static constexpr int SF_OFF = SCALE_OFF + RAW_SLOTS * 528;
    // SILU: per-row group max partials, [2 tile parities][4 slices][BM rows];
    // ROPE: the q and k norm weights (2 x 128 bf16), then each epilogue
    // warp's 32 rows of (position, KV destination)
    static constexpr int RED_OFF = SF_OFF + (MX ? SF_SLOTS * SF_BYTES : 0);
    static constexpr int RED_BYTES = SILU ? 2 * 4 * BM * 4 : ROPE ? 512 + EPI_WARPS * 32 * 16 : 0;
    static constexpr int BAR_OFF = RED_OFF + RED_BYTES;
    static constexpr int BAR_BYTES = 512;
    static constexpr int SMEM = BAR_OFF + BAR_BYTES + 1024;
    // instruction descriptor: D f32, A/B e4m3, both K-major, N, M=128
    static constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(BN >> 3) << 17) |
                                      ((uint32_t)(BM >> 4) << 24);
    // block-scaled (kind::mxf8f6f4): A/B e4m3, both K-major, dense K=32,
    // N, UE8M0 scale factors (bit 23), M=128, scale-factor ids 0
    static constexpr uint32_t IDESC_MX = ((uint32_t)(BN >> 3) << 17) | (1u << 23) |
                                         ((uint32_t)(BM >> 4) << 24);
    static_assert(SMEM <= 232448, "shared memory per block");
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
    uint64_t red_full[2];  // SILU: a tile's partials are in shared memory
    // ROPE: per row quarter (its four warps: two heads x two column halves),
    // [0] the partials and rotary rows are staged, [1] all four have read them
    uint64_t quad[2][4];
    // ROPE: per warp pair (the two column halves of a head's rows): both
    // have read each other's partials
    uint64_t pair[8];
    uint32_t tmem_base;
    int abort;
};
static_assert(sizeof(Barriers) <= 512, "barrier block");

// ROPE: the q/k norm + rotary + KV append of qb_qknorm_rope, applied in the
// qkv GEMM's epilogue (arguments as that entry point takes them)
struct RopeArgs {
    // bf16 [rows, width] maps, box 32 x 32, 64-byte swizzle: q_out, k_out,
    // v_out, k_pool, v_pool (the pools only with row_dst)
    CUtensorMap map_q, map_k, map_v, map_kp, map_vp;
    const int64_t* positions;
    const bf16* cos_sin;
    int64_t max_pos;
    const bf16* q_w;
    const bf16* k_w;
    float eps;
    int n_q, n_kv;
    bf16* q_out;
    bf16* k_out;
    bf16* v_out;
    const int64_t* row_dst;
    bf16* k_pool;
    bf16* v_pool;
    int64_t pool_rows;
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

// D (+)= sum_k a[m,k] w[n,k] 2^(sfa[m] - 127) 2^(sfb[n] - 127) over K=32:
// the block-scaled MMA with UE8M0 scale factors read from TMEM (sfa: 4
// columns for the 128 rows, sfb: 8 columns for the 256 columns)
__device__ __forceinline__ void mma_mx(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t sfa, uint32_t sfb,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], "
        "p;\n\t}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
        : "memory");
}

// The UE8M0 byte of a power-of-two fp32 scale (its biased exponent; 0 for
// a zero scale, which only rows past M carry). bad: not a power of two.
__device__ __forceinline__ uint32_t ue8m0_byte(float s, bool& bad) {
    const uint32_t b = __float_as_uint(s);
    bad |= b != 0u && ((b & 0x807FFFFFu) != 0u || (b >> 23) == 255u);
    return (b >> 23) & 0xFFu;
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
// map_c is read only when TSTORE (bf16 out, box 64 x 32, 128-byte swizzle)
// or SILU (fp8 out, box 32 x 32, 32-byte swizzle).
// MX (the UE8M0 mode): power-of-two scales applied by the block-scaled MMA,
// one accumulator over the whole K, and UE8M0 quantisation in the SILU
// epilogue.
template <int BN, typename OutT = bf16, int NST = MAX_STAGES, bool TSTORE = false,
          bool SILU = false, bool ROPE = false, bool MX = false>
__global__ void __launch_bounds__(NUM_THREADS, 1)
gemm_fp8_bs_kernel(const __grid_constant__ CUtensorMap map_a,
                   const __grid_constant__ CUtensorMap map_b,
                   const __grid_constant__ CUtensorMap map_c, const float* __restrict__ a_scale,
                   int64_t a_scale_ld, const float* __restrict__ w_scale, OutT* __restrict__ out,
                   float* __restrict__ q_scale, int64_t q_scale_ld, int M, int N, int K,
                   uint32_t* status, const __grid_constant__ RopeArgs rope) {
    using C = Cfg<BN, NST, TSTORE, SILU, ROPE, MX>;
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
            mbar_init(&bars->full[s], MX ? 2 : 1);  // MX: + the scale loader's arrival
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
        for (int q = 0; q < 4; ++q) {
            // four warps' lane 0 and the 4 x 32 lanes' cp.async arrivals
            mbar_init(&bars->quad[0][q], 4 + 4 * 32);
            mbar_init(&bars->quad[1][q], 4);
        }
        for (int q = 0; q < 8; ++q) mbar_init(&bars->pair[q], 2);
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
    if constexpr (ROPE) {
        // the norm weights, 16 bytes a lane: q_w by lanes 0-15, k_w by 16-31
        if (warp == 2) {
            const bf16* src = lane < 16 ? rope.q_w + lane * 8 : rope.k_w + (lane - 16) * 8;
            reinterpret_cast<uint4*>(smem + C::RED_OFF)[lane] =
                *reinterpret_cast<const uint4*>(src);
        }
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
                mbar_drain(&bars->full[s], (uint32_t)(j / STAGES) & 1u, status, STATUS_GEMM_DRAIN);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int it = 0, acc_it = 0, tcount = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, ++tcount) {
                for (int kb = 0; kb < n_kb; ++kb, ++it, ++acc_it) {
                    const int s = it % STAGES;
                    if (!mbar_wait(&bars->full[s], (uint32_t)(it / STAGES) & 1u, abort_flag,
                                   status, STATUS_GEMM_MMA)) {
                        ok = false;
                        break;
                    }
                    if constexpr (MX) {
                        // the tile's accumulator is free once the epilogue
                        // has loaded the previous tile
                        if (kb == 0 && !mbar_wait(&bars->tmem_empty[0],
                                                  ((uint32_t)tcount & 1u) ^ 1u, abort_flag, status,
                                                  STATUS_GEMM_MMA)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        // stage s's scale-factor columns: the MMAs of the K
                        // block that used them last completed before this
                        // stage's operands could be loaded again
                        const uint32_t sfa = tmem_base + (uint32_t)(C::TM_SF + 12 * s);
                        const uint32_t sfb = sfa + 4u;
                        const uint32_t src = smem_u32(smem + C::SF_OFF + s * C::SF_BYTES);
                        tmem_cp_32x128b_x4(sfa, rows16_desc(src));
                        tmem_cp_32x128b_x4(sfb, rows16_desc(src + 512));
                        tmem_cp_32x128b_x4(sfb + 4u, rows16_desc(src + 1024));
                        const uint32_t sa = smem_u32(smem + s * C::STAGE_BYTES);
                        const uint64_t adesc = sw128_desc(sa);
                        const uint64_t bdesc = sw128_desc(sa + C::A_BYTES);
#pragma unroll
                        for (int k = 0; k < BK / 32; ++k)
                            mma_mx(tmem_base, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k),
                                   C::IDESC_MX, sfa, sfb, (kb > 0 || k > 0) ? 1u : 0u);
                        mma_commit(&bars->empty[s]);
                        if (kb == n_kb - 1) mma_commit(&bars->tmem_full[0]);
                        continue;
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
            mbar_drain(&bars->drain, 0, status, STATUS_GEMM_DRAIN);
        }
    } else if (warp == 2 && MX) {
        // ---------------- scale-factor loader (UE8M0) ----------------
        // A K block's 128 activation scales and the tile's two weight block
        // scales land by cp.async in the raw ring; LAG K blocks later their
        // exponent bytes are written in the layout tcgen05.cp 32x128b takes
        // (row r: the words of tile rows r, 32 + r, 64 + r, 96 + r; for the
        // weights columns likewise, one block scale in each 128) and handed
        // to the MMA thread.
        constexpr int LAG = C::RAW_SLOTS - 1;
        constexpr int NB = BN / 128;
        auto sf_convert = [&](int j) -> bool {
            // stage slot's SF area is free once its previous MMAs (and
            // their scale-factor copies) completed: the stage's empty phase
            const int slot = j % STAGES;
            if (!mbar_wait(&bars->empty[slot], ((uint32_t)(j / STAGES) & 1u) ^ 1u,
                           abort_flag, status, STATUS_GEMM_EPILOGUE))
                return false;
            __syncwarp();  // every lane's copies of block j have landed
            const ScaleSlot* raw = scales + j % C::RAW_SLOTS;
            bool bad = false;
            uint4 a4;
            a4.x = ue8m0_byte(raw->a[lane], bad);
            a4.y = ue8m0_byte(raw->a[32 + lane], bad);
            a4.z = ue8m0_byte(raw->a[64 + lane], bad);
            a4.w = ue8m0_byte(raw->a[96 + lane], bad);
            const uint32_t w0 = ue8m0_byte(raw->w[0], bad), w1 = ue8m0_byte(raw->w[1], bad);
            uint8_t* sf = smem + C::SF_OFF + slot * C::SF_BYTES;
            *reinterpret_cast<uint4*>(sf + lane * 16) = a4;
            *reinterpret_cast<uint4*>(sf + 512 + lane * 16) = make_uint4(w0, w0, w0, w0);
            *reinterpret_cast<uint4*>(sf + 1024 + lane * 16) = make_uint4(w1, w1, w1, w1);
            if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(status, STATUS_BAD_SCALE);
            // the copies read shared memory through the async proxy
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->full[slot]);
            return true;
        };
        int it = 0, done = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
            const int m0 = (tile / num_n) * BM, n0 = (tile % num_n) * BN;
            for (int kb = 0; kb < n_kb; ++kb) {
                ScaleSlot* sl = scales + it % C::RAW_SLOTS;
                const float* col = a_scale + (int64_t)kb * a_scale_ld;
#pragma unroll
                for (int j = 0; j < BM / 32; ++j) {
                    const int r = j * 32 + lane;
                    const bool valid = m0 + r < M;
                    cp_async4(smem_u32(&sl->a[r]), valid ? col + m0 + r : a_scale,
                              valid ? 4u : 0u);
                }
                if (lane < NB) {
                    const int wb = SILU ? (tile % num_n) + lane * (N / 256) : n0 / 128 + lane;
                    cp_async4(smem_u32(&sl->w[lane]), w_scale + (int64_t)wb * n_kb + kb, 4u);
                }
                asm volatile("cp.async.commit_group;" ::: "memory");
                ++it;
                if (it > LAG) {
                    asm volatile("cp.async.wait_group %0;" ::"n"(LAG) : "memory");
                    if (!sf_convert(done++)) {
                        ok = false;
                        break;
                    }
                }
            }
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
        while (ok && done < it) ok = sf_convert(done++);
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
        // its column slice (SILU: gate columns col0.., up columns 128 + col0..;
        // ROPE: head (ew / 4) / 2 of the tile, its columns 32 s.. and 64 + 32 s..
        // for s = (ew / 4) % 2: the rotary lanes 16 s .. 16 s + 15)
        const int col0 = SILU ? (ew >> 2) * 32
                              : ROPE ? ((ew >> 2) >> 1) * 128 + ((ew >> 2) & 1) * 32
                                     : (ew >> 2) * C::SLICE;
        const int row_in_tile = quarter * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
        int acc_it = 0, tcount = 0, gcount = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, ++tcount) {
            const int m0 = (tile / num_n) * BM, n0 = (tile % num_n) * BN;
            const int m = m0 + row_in_tile;
            const bool valid = m < M;
            const int wblk = col0 / 128;
            if constexpr (ROPE) {
                // the row's position and KV destination, landed by the tile's end
                if (valid) {
                    const uint32_t pd = smem_u32(smem + C::RED_OFF + 512 + (ew * 32 + lane) * 16);
                    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(pd),
                                 "l"(rope.positions + m)
                                 : "memory");
                    if (rope.row_dst)
                        asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(pd + 8),
                                     "l"(rope.row_dst + m)
                                     : "memory");
                }
            }
            float acc[C::SLICE];
            if constexpr (MX) {
                // the whole-K accumulator: load this warp's columns, hand
                // the buffer back to the MMA thread for the next tile
                if (!mbar_wait(&bars->tmem_full[0], (uint32_t)tcount & 1u, abort_flag, status,
                               STATUS_GEMM_EPILOGUE)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t taddr = tmem_base + lane_addr + (uint32_t)col0;
#pragma unroll
                for (int c = 0; c < C::SLICE; c += 32) {
                    uint32_t v[32];
                    const uint32_t cc = (SILU && c > 0) ? 128u : (ROPE && c > 0) ? 64u : (uint32_t)c;
                    tmem_ld16_nowait(taddr + cc, v);
                    tmem_ld16_nowait(taddr + cc + 16u, v + 16);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 32; ++j) acc[c + j] = __uint_as_float(v[j]);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars->tmem_empty[0]);
            }
#pragma unroll
            for (int j = 0; j < C::SLICE; ++j)
                if (!MX) acc[j] = 0.0f;
            for (int kb = 0; kb < (MX ? 0 : n_kb); ++kb, ++acc_it) {
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
                    // SILU: the second 32 columns are the up half's; ROPE: the
                    // head's second half
                    const uint32_t cc = (SILU && c > 0) ? 128u : (ROPE && c > 0) ? 64u : (uint32_t)c;
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
                const float scale = MX ? ue8m0_scale(amax) : group_scale(amax);
                const GroupDivider dv(scale);
                const bool big = !(amax < 0x1p+100f);
                uint32_t pk[8];
                if constexpr (MX) {
                    // q = y * 2^-e exactly, rounded once by the conversion
                    const float inv = ue8m0_inverse(scale);
                    const uint64_t inv2 = f2pack(inv, inv);
#pragma unroll
                    for (int i = 0; i < 32; i += 4) {
                        float a, b, c, d;
                        f2unpack(f2mul(f2pack(acc[i], acc[i + 1]), inv2), a, b);
                        f2unpack(f2mul(f2pack(acc[i + 2], acc[i + 3]), inv2), c, d);
                        pk[i >> 2] = (uint32_t)fp8x2(a, b) | ((uint32_t)fp8x2(c, d) << 16);
                    }
                }
#pragma unroll
                for (int i = 0; i < (MX ? 0 : 32); i += 4) {
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
                // the warp's 32 rows x 32 codes leave as one TMA box: row r at
                // r * 32, its 16-byte halves swapped when r % 8 >= 4 (the
                // 32-byte swizzle of map_c; conflict-free for a row a lane)
                const int j = tile % num_n;
                uint8_t* stage = smem + STAGES * C::STAGE_BYTES + ew * 1024;
                if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
                __syncwarp();
                const int sw = (lane >> 2) & 1;
                *reinterpret_cast<uint4*>(stage + lane * 32 + (sw << 4)) =
                    make_uint4(pk[0], pk[1], pk[2], pk[3]);
                *reinterpret_cast<uint4*>(stage + lane * 32 + ((sw ^ 1) << 4)) =
                    make_uint4(pk[4], pk[5], pk[6], pk[7]);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                // rows past M are clipped by the map's bounds
                if (lane == 0 && m0 + quarter * 32 < M) {
                    tma_store_2d(&map_c, smem_u32(stage), j * 128 + col0, m0 + quarter * 32);
                    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                }
                if (valid && col0 == 0) q_scale[(int64_t)j * q_scale_ld + m] = scale;
            } else if constexpr (ROPE) {
                // qb_qknorm_rope on this tile's two heads, bit for bit. Lane L
                // of that kernel's warp holds columns 2L, 2L + 1, 64 + 2L,
                // 65 + 2L of a head row; here warp sub (0 or 1) of a pair holds
                // lanes 16 sub .. 16 sub + 15 of every row. The four warps of
                // a row quarter share one staging exchange: each stages its
                // 16 sum-of-squares lane partials a row (for warp_sum's xor
                // tree 16, 8, 4, 2, 1 across the pair) and one rotary half
                // (head 0's warps the cos, head 1's the sin of their columns).
                const int sl = ew >> 2, hh = sl >> 1, sub = sl & 1;
                const int gh = n0 / 128 + hh;  // head in q | k | v
                const int n_qk = rope.n_q + rope.n_kv;
                const bool rot = gh < n_qk, kv = gh >= rope.n_q;
                const bool group = n0 / 128 < n_qk;  // the tile's first head rotates
                const int sw = (lane >> 1) & 3;      // 64-byte swizzle of row lane
                uint8_t* const stages = smem + STAGES * C::STAGE_BYTES;
                uint8_t* stage = stages + ew * 4096;
                // the bf16 GEMM output that kernel reads
#pragma unroll
                for (int j = 0; j < 64; ++j) acc[j] = bf16_round(acc[j]);
                asm volatile("cp.async.wait_all;" ::: "memory");
                const int64_t* pd =
                    reinterpret_cast<const int64_t*>(smem + C::RED_OFF + 512 + (ew * 32 + lane) * 16);
                int64_t pos = valid ? pd[0] : 0;
                if (pos < 0 || pos >= rope.max_pos) {
                    if (sl == 0) atomicOr(status, STATUS_BAD_INDEX);
                    pos = 0;
                }
                // the staging area is free once the last tile's stores read it
                if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
                __syncwarp();
                if (group) {
                    // [2 KB, 4 KB): this warp's rotary half of the row's table
                    // entry (head 0's warps cos, head 1's sin, columns 32 sub ..)
                    const bf16* tab = rope.cos_sin + pos * 128 + 64 * hh + 32 * sub;
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(
                                         stage + 2048 + lane * 64 + ((j ^ sw) << 4))),
                                     "l"(tab + 8 * j)
                                     : "memory");
                    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(
                                     smem_u32(&bars->quad[0][quarter]))
                                 : "memory");
                    // [0, 2 KB): the row's 16 lane partials
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        float ps[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int l = 4 * q + e;
                            float ss = __fmul_rn(acc[2 * l], acc[2 * l]);
                            ss = __fmaf_rn(acc[2 * l + 1], acc[2 * l + 1], ss);
                            ss = __fmaf_rn(acc[32 + 2 * l], acc[32 + 2 * l], ss);
                            ps[e] = __fmaf_rn(acc[33 + 2 * l], acc[33 + 2 * l], ss);
                        }
                        *reinterpret_cast<float4*>(stage + lane * 64 + ((q ^ sw) << 4)) =
                            make_float4(ps[0], ps[1], ps[2], ps[3]);
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&bars->quad[0][quarter]);
                }
                // columns 32 sub + 2l, + 1 in p[l], 64 + 32 sub + 2l, + 1 in
                // p[16 + l], exactly (the values are bf16 already)
                uint32_t p[32];
#pragma unroll
                for (int l = 0; l < 16; ++l) {
                    p[l] = bf16x2_bits(acc[2 * l], acc[2 * l + 1]);
                    p[16 + l] = bf16x2_bits(acc[32 + 2 * l], acc[33 + 2 * l]);
                }
                if (group) {
                    if (!mbar_wait(&bars->quad[0][quarter], (uint32_t)gcount & 1u, abort_flag, status,
                                   STATUS_GEMM_EPILOGUE)) {
                        ok = false;
                        break;
                    }
                    float rstd = 0.0f;
                    if (rot) {
                        const uint8_t* partner = stages + (ew ^ 4) * 4096;
                        // lane partials l of both warps added (the tree's first
                        // level), then l + 8, + 4, + 2, + 1
                        float t8[8];
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            float t[8];  // chunks h and h + 2: lanes 4h .. 4h + 3 and + 8
#pragma unroll
                            for (int k2 = 0; k2 < 2; ++k2) {
                                const int q = h + 2 * k2;
                                const int at = lane * 64 + ((q ^ sw) << 4);
                                const float4 mine = *reinterpret_cast<const float4*>(stage + at);
                                const float4 o = *reinterpret_cast<const float4*>(partner + at);
                                t[4 * k2] = __fadd_rn(mine.x, o.x);
                                t[4 * k2 + 1] = __fadd_rn(mine.y, o.y);
                                t[4 * k2 + 2] = __fadd_rn(mine.z, o.z);
                                t[4 * k2 + 3] = __fadd_rn(mine.w, o.w);
                            }
#pragma unroll
                            for (int e = 0; e < 4; ++e) t8[4 * h + e] = __fadd_rn(t[e], t[4 + e]);
                        }
#pragma unroll
                        for (int l = 0; l < 4; ++l) t8[l] = __fadd_rn(t8[l], t8[l + 4]);
                        t8[0] = __fadd_rn(t8[0], t8[2]);
                        t8[1] = __fadd_rn(t8[1], t8[3]);
                        const float ss = __fadd_rn(t8[0], t8[1]);
                        rstd = 1.0f / sqrtf(ss / 128.0f + rope.eps);
                    }
                    // [0, 2 KB) takes the lo outputs once the pair has read both
                    // partials (every pair of a rotating tile takes this step)
                    const int pair_id = hh * 4 + quarter;
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&bars->pair[pair_id]);
                    if (!mbar_wait(&bars->pair[pair_id], (uint32_t)gcount & 1u, abort_flag, status,
                                   STATUS_GEMM_EPILOGUE)) {
                        ok = false;
                        break;
                    }
                    if (rot) {
                        const uint4* wt = reinterpret_cast<const uint4*>(smem + C::RED_OFF) +
                                          (kv ? 16 : 0) + 4 * sub;
                        // the cos and sin halves staged by this quarter's head-0
                        // and head-1 warps of the same column half
                        const uint8_t* cos_at = stages + ((ew & 3) + 4 * sub) * 4096 + 2048;
                        const uint8_t* sin_at = stages + ((ew & 3) + 4 * (2 + sub)) * 4096 + 2048;
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const int at = lane * 64 + ((j ^ sw) << 4);
                            const uint4 c4 = *reinterpret_cast<const uint4*>(cos_at + at);
                            const uint4 s4 = *reinterpret_cast<const uint4*>(sin_at + at);
                            const uint4 wa4 = wt[j], wb4 = wt[8 + j];
                            const uint32_t c8[4] = {c4.x, c4.y, c4.z, c4.w};
                            const uint32_t s8[4] = {s4.x, s4.y, s4.z, s4.w};
                            const uint32_t wa8[4] = {wa4.x, wa4.y, wa4.z, wa4.w};
                            const uint32_t wb8[4] = {wb4.x, wb4.y, wb4.z, wb4.w};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const int l = 4 * j + e;
                                const float2 c = bf16x2_float2(c8[e]), sn = bf16x2_float2(s8[e]);
                                const float2 wa = bf16x2_float2(wa8[e]), wb = bf16x2_float2(wb8[e]);
                                const float2 a = bf16x2_float2(p[l]), b = bf16x2_float2(p[16 + l]);
                                const float ax = __fmul_rn(__fmul_rn(a.x, rstd), wa.x);
                                const float ay = __fmul_rn(__fmul_rn(a.y, rstd), wa.y);
                                const float bx = __fmul_rn(__fmul_rn(b.x, rstd), wb.x);
                                const float by = __fmul_rn(__fmul_rn(b.y, rstd), wb.y);
                                p[l] = bf16x2_bits(__fsub_rn(__fmul_rn(ax, c.x), __fmul_rn(bx, sn.x)),
                                                   __fsub_rn(__fmul_rn(ay, c.y), __fmul_rn(by, sn.y)));
                                p[16 + l] =
                                    bf16x2_bits(__fadd_rn(__fmul_rn(bx, c.x), __fmul_rn(ax, sn.x)),
                                                __fadd_rn(__fmul_rn(by, c.y), __fmul_rn(ay, sn.y)));
                            }
                            // stored before the next chunk's operands are loaded:
                            // one chunk's operands in registers at a time
                            *reinterpret_cast<uint4*>(stage + at) =
                                make_uint4(p[4 * j], p[4 * j + 1], p[4 * j + 2], p[4 * j + 3]);
                        }
                    }
                    // every staged partial and rotary half has been read
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&bars->quad[1][quarter]);
                    if (!mbar_wait(&bars->quad[1][quarter], (uint32_t)gcount & 1u, abort_flag, status,
                                   STATUS_GEMM_EPILOGUE)) {
                        ok = false;
                        break;
                    }
                    ++gcount;
                }
                // the row's two 32-column pieces: two 32 x 32 boxes (the lo
                // piece of a rotated head is in place already)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (!rot)
                        *reinterpret_cast<uint4*>(stage + lane * 64 + ((j ^ sw) << 4)) =
                            make_uint4(p[4 * j], p[4 * j + 1], p[4 * j + 2], p[4 * j + 3]);
                    *reinterpret_cast<uint4*>(stage + 2048 + lane * 64 + ((j ^ sw) << 4)) =
                        make_uint4(p[16 + 4 * j], p[17 + 4 * j], p[18 + 4 * j], p[19 + 4 * j]);
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                // KV append: one box store when the 32 rows land on 32
                // consecutive pool rows, else per-row stores
                int64_t dst = (valid && rope.row_dst) ? pd[1] : -1;
                if (dst >= rope.pool_rows) {
                    if (sl == 0) atomicOr(status, STATUS_BAD_INDEX);
                    dst = -1;
                }
                bool pool_box = false;
                int64_t d0 = 0;
                if (kv && __any_sync(0xffffffffu, dst >= 0)) {
                    d0 = __shfl_sync(0xffffffffu, dst, 0);
                    pool_box = __all_sync(0xffffffffu, dst == d0 + lane) && d0 >= 0 &&
                               d0 + 32 <= rope.pool_rows;
                    if (!pool_box && dst >= 0) {
                        const int kvw = rope.n_kv * 128;
                        bf16* pr = (rot ? rope.k_pool : rope.v_pool) + dst * kvw +
                                   (rot ? gh - rope.n_q : gh - n_qk) * 128 + 32 * sub;
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            *reinterpret_cast<uint4*>(pr + 8 * j) =
                                make_uint4(p[4 * j], p[4 * j + 1], p[4 * j + 2], p[4 * j + 3]);
                            *reinterpret_cast<uint4*>(pr + 64 + 8 * j) = make_uint4(
                                p[16 + 4 * j], p[17 + 4 * j], p[18 + 4 * j], p[19 + 4 * j]);
                        }
                    }
                }
                // rows past M are clipped by the maps' bounds
                if (lane == 0 && m0 + quarter * 32 < M) {
                    const CUtensorMap* mo = !kv ? &rope.map_q : rot ? &rope.map_k : &rope.map_v;
                    const int x = (!kv ? gh : rot ? gh - rope.n_q : gh - n_qk) * 128 + 32 * sub;
                    const int y = m0 + quarter * 32;
                    tma_store_2d(mo, smem_u32(stage), x, y);
                    tma_store_2d(mo, smem_u32(stage + 2048), x + 64, y);
                    if (pool_box) {
                        const CUtensorMap* mp = rot ? &rope.map_kp : &rope.map_vp;
                        tma_store_2d(mp, smem_u32(stage), x, (int)d0);
                        tma_store_2d(mp, smem_u32(stage + 2048), x + 64, (int)d0);
                    }
                    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                }
            } else if constexpr (C::SMALL_OUT) {
                // this warp's 32 rows x 64 columns as four 32 x 16 boxes
                // through one 1 KB area: row r's 16-byte half j at r * 32 +
                // (j ^ (r / 4) % 2) * 16 (the 32-byte swizzle of map_c)
                uint8_t* stage = smem + STAGES * C::STAGE_BYTES + ew * 1024;
                const int sw = (lane >> 2) & 1;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
                    __syncwarp();
                    *reinterpret_cast<uint4*>(stage + lane * 32 + (sw << 4)) =
                        float_to_bf16x8(acc + 16 * q);
                    *reinterpret_cast<uint4*>(stage + lane * 32 + ((sw ^ 1) << 4)) =
                        float_to_bf16x8(acc + 16 * q + 8);
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    __syncwarp();
                    // rows past M are clipped by the tensor map's bounds
                    if (lane == 0 && m0 + quarter * 32 < M) {
                        tma_store_2d(&map_c, smem_u32(stage), n0 + col0 + 16 * q,
                                     m0 + quarter * 32);
                        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                    }
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
        if ((TSTORE || ROPE || SILU) && lane == 0)
            asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        // ROPE: this thread's row and rotary copies land before the block
        // exits, also when a bounded wait gave up mid-tile
        if (ROPE) asm volatile("cp.async.wait_all;" ::: "memory");
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

// bf16 [rows, n] map, box 32 rows x 32 columns, 64-byte swizzle (the
// ROPE epilogue's output boxes)
int make_box32_map(CUtensorMap* map, void* base, int64_t rows, int64_t n) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = get_encoder();
    if (!enc) {
        set_error("qb_gemm_fp8_qknorm_rope: cuTensorMapEncodeTiled unavailable");
        return QB_ERR_CUDA;
    }
    cuuint64_t dims[2] = {(cuuint64_t)n, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)n * 2};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                     CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("qb_gemm_fp8_qknorm_rope: cuTensorMapEncodeTiled (out) failed (%d)", (int)r);
        return QB_ERR_CUDA;
    }
    return QB_OK;
}

// fp8 [rows, n] map, box 32 rows x 32 columns, 32-byte swizzle (the SILU
// epilogue's output boxes)
int make_fp8_box32_map(CUtensorMap* map, void* base, int64_t rows, int64_t n) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = get_encoder();
    if (!enc) {
        set_error("qb_gemm_fp8_silu_quant: cuTensorMapEncodeTiled unavailable");
        return QB_ERR_CUDA;
    }
    cuuint64_t dims[2] = {(cuuint64_t)n, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)n};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B,
                     CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("qb_gemm_fp8_silu_quant: cuTensorMapEncodeTiled (out) failed (%d)", (int)r);
        return QB_ERR_CUDA;
    }
    return QB_OK;
}

// bf16 output map: rows x n, box 32 rows x 64 columns, 128-byte swizzle
// (small: box 32 rows x 16 columns, 32-byte swizzle)
int make_out_map(CUtensorMap* map, void* base, int64_t rows, int64_t n, bool small = false) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = get_encoder();
    if (!enc) {
        set_error("qb_gemm_fp8_bs: cuTensorMapEncodeTiled unavailable");
        return QB_ERR_CUDA;
    }
    cuuint64_t dims[2] = {(cuuint64_t)n, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)n * 2};
    cuuint32_t box[2] = {small ? 16u : 64u, 32};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE,
                     small ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("qb_gemm_fp8_bs: cuTensorMapEncodeTiled (out) failed (%d)", (int)r);
        return QB_ERR_CUDA;
    }
    return QB_OK;
}

// SILU: n = 2 * inter weight rows, out fp8 [m, inter], q_scale [inter / 128, q_scale_ld]
template <int BN, int NST = MAX_STAGES, bool TSTORE = false, bool SILU = false,
          bool ROPE = false, bool MX = false>
int launch(const void* a, const float* a_scale, int64_t a_scale_ld, const void* w,
           const float* w_scale, void* out, int64_t m, int64_t n, int64_t k, cudaStream_t stream,
           float* q_scale = nullptr, int64_t q_scale_ld = 0, const RopeArgs* rope = nullptr) {
    using C = Cfg<BN, NST, TSTORE, SILU, ROPE, MX>;
    using OutT = typename std::conditional<SILU, uint8_t, bf16>::type;
    CUtensorMap map_a, map_b, map_c;
    memset(&map_c, 0, sizeof(map_c));
    int st = make_map(&map_a, a, m, k, BM);
    if (st) return st;
    st = make_map(&map_b, w, n, k, SILU ? 128 : BN);
    if (st) return st;
    if (TSTORE) {
        st = make_out_map(&map_c, out, m, n, C::SMALL_OUT);
        if (st) return st;
    }
    if (SILU) {
        st = make_fp8_box32_map(&map_c, out, m, n / 2);
        if (st) return st;
    }
    auto kernel = gemm_fp8_bs_kernel<BN, OutT, NST, TSTORE, SILU, ROPE, MX>;
    static std::atomic<bool> attr[MAX_DEVICES];
    if (!set_smem_once(attr, kernel, C::SMEM))
        return launch_status("qb_gemm_fp8_bs: smem attribute");
    uint32_t* status = device_status_ptr();
    if (!status) return launch_status("qb_gemm_fp8_bs: status word");
    const int64_t tiles = ((m + BM - 1) / BM) * (n / BN);
    const int grid = (int)(tiles < sm_count() ? tiles : sm_count());
    RopeArgs none;
    memset(&none, 0, sizeof(none));
    kernel<<<grid, NUM_THREADS, C::SMEM, stream>>>(map_a, map_b, map_c, a_scale, a_scale_ld,
                                                   w_scale, (OutT*)out, q_scale, q_scale_ld,
                                                   (int)m, (int)n, (int)k, status,
                                                   rope ? *rope : none);
    return launch_status(SILU   ? "qb_gemm_fp8_silu_quant"
                         : ROPE ? "qb_gemm_fp8_qknorm_rope"
                                : "qb_gemm_fp8_bs");
}

}  // namespace

extern "C" int qb_gemm_fp8_bs(const void* a, const float* a_scale, int64_t a_scale_ld,
                              const void* w, const float* w_scale, void* out, int64_t m, int64_t n,
                              int64_t k, int ue8m0, void* stream) {
    if (m < 0 || n <= 0 || k <= 0) return invalid("qb_gemm_fp8_bs: bad sizes");
    if (k % BK != 0) return invalid("qb_gemm_fp8_bs: k must be a multiple of 128");
    if (n % 128 != 0) return invalid("qb_gemm_fp8_bs: n must be a multiple of 128");
    if (ue8m0 && n % 256 != 0) return invalid("qb_gemm_fp8_bs: ue8m0 needs n a multiple of 256");
    if (m > 0x7fffffffLL || n > 0x7fffffffLL || k > 0x7fffffffLL)
        return invalid("qb_gemm_fp8_bs: sizes exceed int32");
    if (a_scale_ld < m) return invalid("qb_gemm_fp8_bs: a_scale_ld < m");
    if (!aligned(a, 16) || !aligned(w, 16) || !aligned(out, 16))
        return invalid("qb_gemm_fp8_bs: a, w and out must be 16-byte aligned");
    if (!a_scale || !w_scale) return invalid("qb_gemm_fp8_bs: NULL scales");
    if (m == 0) return QB_OK;
    cudaStream_t s = (cudaStream_t)stream;
    // UE8M0: the block-scaled MMA applies the power-of-two scales
    if (ue8m0)
        return launch<256, 4, true, false, false, true>(a, a_scale, a_scale_ld, w, w_scale, out, m,
                                                        n, k, s);
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
                                      int64_t inter, int64_t k, int ue8m0, void* stream) {
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
    if (ue8m0)
        return launch<256, 4, false, true, false, true>(a, a_scale, a_scale_ld, w, w_scale, q_out,
                                                        m, 2 * inter, k, (cudaStream_t)stream,
                                                        scale_out, scale_ld);
    return launch<256, 4, false, true>(a, a_scale, a_scale_ld, w, w_scale, q_out, m, 2 * inter,
                                       k, (cudaStream_t)stream, scale_out, scale_ld);
}

extern "C" int qb_gemm_fp8_qknorm_rope(
    const void* a, const float* a_scale, int64_t a_scale_ld, const void* w, const float* w_scale,
    int64_t m, int64_t k, const int64_t* positions, const void* cos_sin, int64_t max_pos,
    const void* q_w, const void* k_w, float eps, int n_q, int n_kv, int head_dim, void* q_out,
    void* k_out, void* v_out, const int64_t* row_dst, void* k_pool, void* v_pool,
    int64_t pool_rows, int ue8m0, void* stream) {
    if (head_dim != 128) return invalid("qb_gemm_fp8_qknorm_rope: head_dim must be 128");
    if (m < 0 || k <= 0 || n_q <= 0 || n_kv <= 0 || n_q % n_kv != 0)
        return invalid("qb_gemm_fp8_qknorm_rope: bad sizes or head counts");
    const int64_t n = (int64_t)(n_q + 2 * n_kv) * 128;
    if (n % 256 != 0)
        return invalid("qb_gemm_fp8_qknorm_rope: n_q + 2 n_kv must be even (two heads a tile)");
    if (k % BK != 0) return invalid("qb_gemm_fp8_qknorm_rope: k must be a multiple of 128");
    if (m > 0x7fffffffLL || k > 0x7fffffffLL)
        return invalid("qb_gemm_fp8_qknorm_rope: sizes exceed int32");
    if (a_scale_ld < m) return invalid("qb_gemm_fp8_qknorm_rope: a_scale_ld < m");
    if (!aligned(a, 16) || !aligned(w, 16) || !aligned(q_out, 16) || !aligned(k_out, 16) ||
        !aligned(v_out, 16) || !aligned(q_w, 16) || !aligned(k_w, 16) || !aligned(cos_sin, 16))
        return invalid(
            "qb_gemm_fp8_qknorm_rope: a, w, the outputs, weights and cos_sin must be 16-byte "
            "aligned");
    if (row_dst && (!k_pool || !v_pool || !aligned(k_pool, 16) || !aligned(v_pool, 16)))
        return invalid("qb_gemm_fp8_qknorm_rope: KV append needs 16-byte aligned pools");
    if (!a_scale || !w_scale || !positions || !cos_sin || !q_w || !k_w)
        return invalid("qb_gemm_fp8_qknorm_rope: NULL input");
    if (max_pos <= 0) return invalid("qb_gemm_fp8_qknorm_rope: empty rotary cache");
    if (pool_rows > 0x7fffffffLL) return invalid("qb_gemm_fp8_qknorm_rope: pool_rows exceeds int32");
    if (m == 0) return QB_OK;
    RopeArgs r;
    memset(&r, 0, sizeof(r));
    int st = make_box32_map(&r.map_q, q_out, m, (int64_t)n_q * 128);
    if (!st) st = make_box32_map(&r.map_k, k_out, m, (int64_t)n_kv * 128);
    if (!st) st = make_box32_map(&r.map_v, v_out, m, (int64_t)n_kv * 128);
    if (!st && row_dst && pool_rows > 0) {
        st = make_box32_map(&r.map_kp, k_pool, pool_rows, (int64_t)n_kv * 128);
        if (!st) st = make_box32_map(&r.map_vp, v_pool, pool_rows, (int64_t)n_kv * 128);
    }
    if (st) return st;
    r.positions = positions;
    r.cos_sin = (const bf16*)cos_sin;
    r.max_pos = max_pos;
    r.q_w = (const bf16*)q_w;
    r.k_w = (const bf16*)k_w;
    r.eps = eps;
    r.n_q = n_q;
    r.n_kv = n_kv;
    r.q_out = (bf16*)q_out;
    r.k_out = (bf16*)k_out;
    r.v_out = (bf16*)v_out;
    r.row_dst = row_dst;
    r.k_pool = (bf16*)k_pool;
    r.v_pool = (bf16*)v_pool;
    r.pool_rows = pool_rows;
    if (ue8m0)
        return launch<256, 3, false, false, true, true>(a, a_scale, a_scale_ld, w, w_scale, nullptr,
                                                        m, n, k, (cudaStream_t)stream, nullptr, 0,
                                                        &r);
    return launch<256, 3, false, false, true>(a, a_scale, a_scale_ld, w, w_scale, nullptr, m, n,
                                              k, (cudaStream_t)stream, nullptr, 0, &r);
}
