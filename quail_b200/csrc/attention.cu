// Tree attention, fused: for each query row, (A) causal attention over its
// own cu_a segment, (B) attention over the resident KV pages of its read
// group (the shared prefix it borrows), then the LSE merge with the
// reference's bf16 roundings and the per-head fp8 quantisation of the
// o_proj input.
//
// One block = 64 query rows of one segment x HP query heads of one KV head
// (the GQA group, HP <= 4): K/V tiles of 64 keys are staged once in shared
// memory (16-byte XOR swizzle, cp.async double buffering) and read by all
// HP heads. Warp w computes rows 16 (w % 4) .. +16 of head w / 4 with bf16
// mma.sync (fp32 accumulation); Q tiles and call B's results live in shared
// memory. P is rounded to bf16 before PV and the row sum uses the fp32 P, as
// FlashAttention does. Every rounding step is explicit (__f*_rn, the
// FMA-only exp2 / ln of common.cuh) and the row sums follow one fixed
// order: thread tq of a quad adds keys 8 nt + 2 tq + {0, 1} of each tile in
// (nt, e) order, and the quad combines its four sums with an xor butterfly
// - so a CPU restatement can reproduce every bit.
#include "common.cuh"

namespace qb {
// attention_tc.cu: the tcgen05 kernel for even GQA groups; -1 = not its shapes
int launch_attention_tc(bool unified, const char* who, const void* q, const void* k,
                        const void* v, int64_t rows, int n_q, int n_kv, const int32_t* cu,
                        const int32_t* tiles, int64_t n_tiles, const int32_t* read_cu_q,
                        const int32_t* read_used, const int32_t* table, int64_t n_reads,
                        int64_t table_width, const int32_t* source, const void* k_pool,
                        const void* v_pool, int64_t n_pages, int page_tokens,
                        float softmax_scale, void* q_out, float* scale_out, int64_t scale_ld,
                        void* stream);
}  // namespace qb

namespace {

using namespace qb;

constexpr int D = 128;       // head dim
constexpr int BM = 64;       // query rows per block
constexpr int BN = 64;       // keys per tile
constexpr int ROW_GROUPS = BM / 16;
constexpr int MAX_HP = 4;    // query heads per block
constexpr int TILE_ELEMS = BN * D;
constexpr int OB_LD = D + 8;  // padded row of call B's staged output

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src),
                 "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    bf162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// element offset of (row, 16-byte chunk) in a swizzled [64][D] tile
__device__ __forceinline__ int swz(int row, int chunk) { return row * D + ((chunk ^ (row & 7)) << 3); }

struct KeySource {
    const bf16* k;       // row-major [rows][n_kv][D]
    const bf16* v;
    int64_t n_rows;      // rows the source holds (bounds check)
    // paged source: key j lives at row table[j / page_tokens] * page_tokens +
    // j % page_tokens; contiguous source: row base + j
    const int32_t* table;
    int page_tokens;
    int64_t base;
};

__device__ __forceinline__ int64_t key_row(const KeySource& s, int j, uint32_t* status) {
    if (s.table == nullptr) return s.base + j;
    const int64_t page = s.table[j / s.page_tokens];
    const int64_t r = page * s.page_tokens + (j % s.page_tokens);
    if (page < 0 || r >= s.n_rows) {
        atomicOr(status, STATUS_BAD_INDEX);
        return -1;
    }
    return r;
}

// Stage keys [j0, j0 + BN) of KV head hk into one K and one V tile (zeros
// past n_keys); all threads of the block take part.
__device__ __forceinline__ void load_tile(const KeySource& s, int j0, int n_keys, int n_kv, int hk,
                                          bf16* sk, bf16* sv, uint32_t* status) {
    const uint32_t k_base = smem_u32(sk), v_base = smem_u32(sv);
    for (int idx = threadIdx.x; idx < BN * D / 8; idx += blockDim.x) {
        const int kr = idx >> 4, chunk = idx & 15;
        int64_t row = -1;
        if (j0 + kr < n_keys) row = key_row(s, j0 + kr, status);
        const int64_t off = (row < 0 ? 0 : (row * n_kv + hk) * D) + chunk * 8;
        const int bytes = row < 0 ? 0 : 16;
        const uint32_t so = (uint32_t)swz(kr, chunk) * 2u;
        cp_async16(k_base + so, s.k + off, bytes);
        cp_async16(v_base + so, s.v + off, bytes);
    }
}

struct Softmax {
    float m[2], l[2];
    float acc[16][4];  // 16 dim tiles of 8 x (rows gr, gr+8)
};

// Attend the warp's 16 query rows (Q tile in shared memory at q_tile, rows
// r16 .. r16+15) to keys [0, n_keys) of a source; causal masks key j >
// query position q_first + row. Leaves m, unnormalised l and acc in st.
__device__ __forceinline__ void attend(const KeySource& src, int n_keys, bool causal, int q_first,
                                       int n_kv, int hk, uint32_t q_tile, int r16, float sl2,
                                       Softmax& st, bf16* kv, uint32_t* status) {
    const int lane = threadIdx.x & 31;
    const int gr = lane >> 2, tq = lane & 3;
    const int qr0 = q_first + r16 + gr, qr1 = qr0 + 8;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        st.m[r] = -INFINITY;
        st.l[r] = 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) st.acc[i][j] = 0.0f;

    int key_end = n_keys;
    if (causal) key_end = min(n_keys, q_first + BM);  // the block's last row bounds its keys
    // keys past this bound are masked for all 16 rows of the warp
    const int warp_end = causal ? min(key_end, q_first + r16 + 16) : key_end;
    const int n_tiles = (key_end + BN - 1) / BN;
    bf16* bufk[2] = {kv, kv + 2 * TILE_ELEMS};
    bf16* bufv[2] = {kv + TILE_ELEMS, kv + 3 * TILE_ELEMS};

    __syncthreads();  // the buffers may still be read by a previous call
    if (n_tiles > 0) load_tile(src, 0, key_end, n_kv, hk, bufk[0], bufv[0], status);
    cp_async_commit();
    for (int t = 0; t < n_tiles; ++t) {
        if (t + 1 < n_tiles)
            load_tile(src, (t + 1) * BN, key_end, n_kv, hk, bufk[(t + 1) & 1], bufv[(t + 1) & 1],
                      status);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        const uint32_t kb = smem_u32(bufk[t & 1]), vb = smem_u32(bufv[t & 1]);
        const int j0 = t * BN;

        // 8-key groups of the tile visible to some row of the warp; the rest
        // have p = 0 exactly, so their QK^T, exp2 and PV steps are skipped
        // (an all-zero PV step leaves the accumulator unchanged)
        const int vis = warp_end - j0;
        const int n8 = vis >= BN ? 8 : (vis <= 0 ? 0 : (vis + 7) >> 3);

        // S = Q K^T for 64 keys: 8 key tiles of 8, dims in 8 steps of 16
        float s[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) s[i][j] = 0.0f;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            uint32_t qa[4];
            {
                const int mi = lane >> 3, i = lane & 7;
                const int row = r16 + (mi & 1) * 8 + i;
                ldsm_x4(q_tile + (uint32_t)swz(row, 2 * ks + (mi >> 1)) * 2u, qa[0], qa[1], qa[2],
                        qa[3]);
            }
#pragma unroll
            for (int nt = 0; nt < 8; nt += 2) {
                if (nt >= n8) break;
                const int mi = lane >> 3, i = lane & 7;
                const int key = (nt + (mi >> 1)) * 8 + i;
                const int chunk = 2 * ks + (mi & 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(kb + (uint32_t)swz(key, chunk) * 2u, b0, b1, b2, b3);
                mma_bf16(s[nt], qa, b0, b1);
                mma_bf16(s[nt + 1], qa, b2, b3);
            }
        }
        // mask (only tiles that reach past the keys or the warp's first row's
        // diagonal) and row max
        float mx[2] = {-INFINITY, -INFINITY};
        const bool edge = j0 + BN > key_end || (causal && j0 + BN - 1 > q_first + r16);
        if (edge) {
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                if (nt >= n8) break;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int key = j0 + nt * 8 + 2 * tq + (e & 1);
                    const int qr = (e < 2) ? qr0 : qr1;
                    const bool ok = key < key_end && (!causal || key <= qr);
                    if (!ok) s[nt][e] = -INFINITY;
                }
            }
        }
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            if (nt >= n8) break;
#pragma unroll
            for (int e = 0; e < 4; ++e) mx[e >> 1] = fmaxf(mx[e >> 1], s[nt][e]);
        }
        float alpha[2], msl[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
            const float m_new = fmaxf(st.m[r], mx[r]);
            if (m_new == -INFINITY) {  // nothing visible yet
                alpha[r] = 1.0f;
                msl[r] = 0.0f;
            } else {
                alpha[r] = qexp2f(__fmul_rn(__fsub_rn(st.m[r], m_new), sl2));
                msl[r] = __fmul_rn(m_new, sl2);
            }
            st.m[r] = m_new;
            st.l[r] = __fmul_rn(st.l[r], alpha[r]);
        }
        // a row whose max did not move has alpha == 1: its rescale is exact
        // and skipped (warp-uniform in the common case)
        if (alpha[0] != 1.0f || alpha[1] != 1.0f) {
            const uint64_t a0 = f2pack(alpha[0], alpha[0]), a1 = f2pack(alpha[1], alpha[1]);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                f2unpack(f2mul(f2pack(st.acc[i][0], st.acc[i][1]), a0), st.acc[i][0],
                         st.acc[i][1]);
                f2unpack(f2mul(f2pack(st.acc[i][2], st.acc[i][3]), a1), st.acc[i][2],
                         st.acc[i][3]);
            }
        }
        // P = exp2(s * sl2 - m * sl2); fp32 row sums; bf16 P for PV
        uint32_t pa[4][4];
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            float p[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            if (nt < n8) {
                // x = s * sl2 - m * sl2 and exp2, two lanes per instruction
                const uint64_t sl = f2pack(sl2, sl2);
                f2unpack(f2fma(f2pack(s[nt][0], s[nt][1]), sl, f2pack(-msl[0], -msl[0])), p[0],
                         p[1]);
                f2unpack(f2fma(f2pack(s[nt][2], s[nt][3]), sl, f2pack(-msl[1], -msl[1])), p[2],
                         p[3]);
                qexp2f_x2(p[0], p[1]);
                qexp2f_x2(p[2], p[3]);
#pragma unroll
                for (int e = 0; e < 4; ++e) st.l[e >> 1] = __fadd_rn(st.l[e >> 1], p[e]);
            }
            const int kk = nt >> 1, half = nt & 1;
            pa[kk][half * 2 + 0] = pack_bf16(p[0], p[1]);
            pa[kk][half * 2 + 1] = pack_bf16(p[2], p[3]);
        }
        // O += P V: 4 key steps of 16 x 16 dim tiles of 8
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            if (2 * kk >= n8) break;
#pragma unroll
            for (int nd = 0; nd < 16; nd += 2) {
                const int mi = lane >> 3, i = lane & 7;
                const int key = kk * 16 + (mi & 1) * 8 + i;
                const int chunk = nd + (mi >> 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(vb + (uint32_t)swz(key, chunk) * 2u, b0, b1, b2, b3);
                mma_bf16(st.acc[nd], pa[kk], b0, b1);
                mma_bf16(st.acc[nd + 1], pa[kk], b2, b3);
            }
        }
        __syncthreads();  // the buffer is refilled two tiles later
    }
    cp_async_wait<0>();
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        st.l[r] = __fadd_rn(st.l[r], __shfl_xor_sync(0xffffffffu, st.l[r], 1));
        st.l[r] = __fadd_rn(st.l[r], __shfl_xor_sync(0xffffffffu, st.l[r], 2));
    }
}

__device__ __forceinline__ int read_group(const int32_t* cu_q, int64_t n_reads, int idx) {
    // the group g with cu_q[g] <= idx < cu_q[g + 1]
    int lo = 0, hi = (int)n_reads;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (cu_q[mid] <= idx) lo = mid; else hi = mid;
    }
    return lo;
}

// Shared memory: Q [hp][64][128] | K/V tiles x2 | (tree) call B output
// [hp][64][OB_LD] bf16 | call B lse [hp][64] f32.
__host__ __device__ constexpr size_t smem_bytes(int hp, bool tree) {
    return (size_t)hp * BM * D * 2 + 4 * (size_t)TILE_ELEMS * 2 +
           (tree ? (size_t)hp * BM * OB_LD * 2 + (size_t)hp * BM * 4 : 0);
}

// UNIFIED = false: the tree path (cu_a segments, call B over read groups,
// merge). UNIFIED = true: the unified path, one causal paged call; cu_a is
// then the unified cu_q, sequence s reads read_used[s] keys through table
// row s, and its queries are the last cu_a[s+1] - cu_a[s] of those keys.
template <bool UNIFIED>
__global__ void __launch_bounds__(ROW_GROUPS * 32 * MAX_HP, 1)
tree_attention_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k,
                      const bf16* __restrict__ v, int64_t rows, int n_q, int n_kv, int hp,
                      const int32_t* __restrict__ cu_a, const int32_t* __restrict__ tiles,
                      const int32_t* __restrict__ read_cu_q, const int32_t* __restrict__ read_used,
                      const int32_t* __restrict__ read_table, int64_t n_reads,
                      int64_t table_width, const int32_t* __restrict__ source,
                      const bf16* __restrict__ k_pool, const bf16* __restrict__ v_pool,
                      int64_t pool_rows, int page_tokens, float scale,
                      uint8_t* __restrict__ q_out, float* __restrict__ scale_out,
                      int64_t scale_ld, uint32_t* status) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    bf16* qs = reinterpret_cast<bf16*>(smem_raw);
    bf16* kv = qs + hp * BM * D;
    bf16* ob = kv + 4 * TILE_ELEMS;
    float* lse_b_s = reinterpret_cast<float*>(ob + hp * BM * OB_LD);
    __shared__ int s_grp[BM];
    __shared__ int s_list[BM];  // the distinct read groups of the tile, ascending
    __shared__ int s_nlist;

    const int seg = tiles[2 * blockIdx.x];
    const int row0 = tiles[2 * blockIdx.x + 1];
    const int group = n_q / n_kv;
    const int hk = blockIdx.y / (group / hp);
    const int h_first = hk * group + (blockIdx.y % (group / hp)) * hp;
    const int seg_start = cu_a[seg], seg_end = cu_a[seg + 1];
    if (seg_start < 0 || seg_end > rows || row0 < seg_start || row0 >= seg_end) {
        if (threadIdx.x == 0) atomicOr(status, STATUS_BAD_INDEX);
        return;
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gr = lane >> 2, tq = lane & 3;
    const int r16 = (warp % ROW_GROUPS) * 16;
    const int g = warp / ROW_GROUPS;     // head within the block
    const int h = h_first + g;
    const float sl2 = __fmul_rn(scale, 1.44269504088896341f);
    const uint32_t q_tile = smem_u32(qs + g * BM * D);

    // Q tiles of the block's heads, zero past the segment end
    for (int idx = threadIdx.x; idx < hp * BM * (D / 8); idx += blockDim.x) {
        const int hh = idx / (BM * (D / 8)), rem = idx % (BM * (D / 8));
        const int r = rem >> 4, chunk = rem & 15;
        const int row = row0 + r;
        const bool ok = row < seg_end;
        const bf16* src = q + ((int64_t)(ok ? row : row0) * n_q + h_first + hh) * D + chunk * 8;
        cp_async16(smem_u32(qs + hh * BM * D + swz(r, chunk)), src, ok ? 16 : 0);
    }
    cp_async_commit();

    // read group per tile row (-1: reads nothing resident)
    if (threadIdx.x < BM) {
        const int r = row0 + threadIdx.x;
        int grp = -1;
        if (!UNIFIED && r < seg_end && n_reads > 0) {
            const int src = source[r];
            if (src >= 0) {
                if (src >= read_cu_q[n_reads]) atomicOr(status, STATUS_BAD_INDEX);
                else grp = read_group(read_cu_q, n_reads, src);
            }
        }
        s_grp[threadIdx.x] = grp;
    }
    cp_async_wait<0>();
    __syncthreads();
    if (!UNIFIED) {
        if (threadIdx.x == 0) {
            int n = 0, cur = -1;
            while (true) {
                int next = INT_MAX;
                for (int i = 0; i < BM; ++i) {
                    const int x = s_grp[i];
                    if (x > cur && x < next) next = x;
                }
                if (next == INT_MAX) break;
                s_list[n++] = next;
                cur = next;
            }
            s_nlist = n;
        }
        __syncthreads();
    }

    Softmax st;
    const int my_row[2] = {r16 + gr, r16 + gr + 8};
    bf16* ob_head = ob + g * BM * OB_LD;
    float* lse_head = lse_b_s + g * BM;

    if (!UNIFIED) {
        const int n_list = s_nlist;
        for (int li = 0; li < n_list; ++li) {
            const int cur = s_list[li];
            KeySource src{k_pool, v_pool, pool_rows, read_table + (int64_t)cur * table_width,
                          page_tokens, 0};
            int used = read_used[cur];
            if (used < 0 || (int64_t)((used + page_tokens - 1) / page_tokens) > table_width) {
                if (threadIdx.x == 0) atomicOr(status, STATUS_BAD_INDEX);
                used = 0;
            }
            attend(src, used, false, 0, n_kv, hk, q_tile, r16, sl2, st, kv, status);
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                if (s_grp[my_row[r]] != cur) continue;
                const float inv = __frcp_rn(st.l[r]);
#pragma unroll
                for (int nd = 0; nd < 16; ++nd)
                    *reinterpret_cast<uint32_t*>(ob_head + my_row[r] * OB_LD + nd * 8 + 2 * tq) =
                        pack_bf16(__fmul_rn(st.acc[nd][2 * r], inv),
                                  __fmul_rn(st.acc[nd][2 * r + 1], inv));
                if (tq == 0) lse_head[my_row[r]] = __fmaf_rn(st.m[r], scale, qlnf(st.l[r]));
            }
        }
        // call A: causal over the segment's own rows
        KeySource own{k, v, rows, nullptr, 1, seg_start};
        attend(own, seg_end - seg_start, true, row0 - seg_start, n_kv, hk, q_tile, r16, sl2, st,
               kv, status);
    } else {
        // one causal call over the sequence's pages: retained KV + current rows
        int used = read_used[seg];
        const int q_len = seg_end - seg_start;
        if (used < q_len || (int64_t)((used + page_tokens - 1) / page_tokens) > table_width) {
            if (threadIdx.x == 0) atomicOr(status, STATUS_BAD_INDEX);
            used = q_len;
        }
        KeySource paged{k_pool, v_pool, pool_rows, read_table + (int64_t)seg * table_width,
                        page_tokens, 0};
        attend(paged, used, true, used - q_len + (row0 - seg_start), n_kv, hk, q_tile, r16, sl2,
               st, kv, status);
    }
    __syncwarp();

    // merge + per-head fp8 quantisation; one head = one 128-column group
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int row = row0 + my_row[r];
        const bool has_b = !UNIFIED && s_grp[my_row[r]] >= 0;
        const float inv = __frcp_rn(st.l[r]);
        const float lse_a = __fmaf_rn(st.m[r], scale, qlnf(st.l[r]));
        float y[32];
        float amax = 0.0f;
        float w = 0.0f;
        if (has_b) w = bf16_round(sigmoidf_ref(__fsub_rn(lse_head[my_row[r]], lse_a)));
#pragma unroll
        for (int nd = 0; nd < 16; ++nd) {
            bf162 bb;
            if (has_b)
                bb = *reinterpret_cast<const bf162*>(ob_head + my_row[r] * OB_LD + nd * 8 + 2 * tq);
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const float a = bf16_round(__fmul_rn(st.acc[nd][2 * r + e], inv));
                float val = a;
                if (has_b) {
                    const float b = e == 0 ? __low2float(bb) : __high2float(bb);
                    val = bf16_round(__fadd_rn(a, __fmul_rn(__fsub_rn(b, a), w)));
                }
                y[2 * nd + e] = val;
                amax = fmaxf(amax, fabsf(val));
            }
        }
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        if (row >= seg_end) continue;
        const float sc = group_scale(amax);
        const GroupDivider dv(sc);
        uint8_t* out = q_out + ((int64_t)row * n_q + h) * D;
#pragma unroll
        for (int nd = 0; nd < 16; ++nd)
            *reinterpret_cast<uint16_t*>(out + nd * 8 + 2 * tq) =
                fp8x2(dv.quant(y[2 * nd]), dv.quant(y[2 * nd + 1]));
        if (tq == 0) scale_out[(int64_t)h * scale_ld + row] = sc;
    }
}

template <bool UNIFIED>
int launch_attention(const char* who, const void* q, const void* k, const void* v, int64_t rows,
                     int n_q, int n_kv, const int32_t* cu, const int32_t* tiles, int64_t n_tiles,
                     const int32_t* read_cu_q, const int32_t* read_used, const int32_t* table,
                     int64_t n_reads, int64_t table_width, const int32_t* source,
                     const void* k_pool, const void* v_pool, int64_t n_pages, int page_tokens,
                     float softmax_scale, void* q_out, float* scale_out, int64_t scale_ld,
                     void* stream) {
    if (n_tiles == 0 || rows == 0) return QB_OK;
    if (n_tiles > 0x7fffffffLL) {
        set_error("%s: too many tiles", who);
        return QB_ERR_INVALID;
    }
    const int group = n_q / n_kv;
    const int hp = group < MAX_HP ? group : MAX_HP;
    if (group % hp != 0) {
        set_error("%s: query heads per KV head must be 1, 2, 4 or a multiple of 4", who);
        return QB_ERR_INVALID;
    }
    uint32_t* status = device_status_ptr();
    if (!status) return launch_status(who);
    const size_t smem = smem_bytes(MAX_HP, !UNIFIED);
    static std::atomic<bool> attr_set[MAX_DEVICES];
    if (!set_smem_once(attr_set, tree_attention_kernel<UNIFIED>, (int)smem))
        return launch_status(who);
    dim3 grid((unsigned)n_tiles, (unsigned)(n_kv * (group / hp)));
    tree_attention_kernel<UNIFIED><<<grid, ROW_GROUPS * 32 * hp, smem_bytes(hp, !UNIFIED),
                                     (cudaStream_t)stream>>>(
        (const bf16*)q, (const bf16*)k, (const bf16*)v, rows, n_q, n_kv, hp, cu, tiles,
        read_cu_q, read_used, table, n_reads, table_width, source, (const bf16*)k_pool,
        (const bf16*)v_pool, n_pages * (int64_t)page_tokens, page_tokens, softmax_scale,
        (uint8_t*)q_out, scale_out, scale_ld, status);
    return launch_status(who);
}

int check_common(const char* who, int64_t rows, int n_q, int n_kv, int head_dim, int64_t n_seg,
                 int64_t n_tiles, int64_t scale_ld, const void* q_out, const float* scale_out) {
    if (head_dim != D) {
        set_error("%s: head_dim must be 128", who);
        return QB_ERR_INVALID;
    }
    if (n_q <= 0 || n_kv <= 0 || n_q % n_kv) {
        set_error("%s: n_q must be a positive multiple of n_kv", who);
        return QB_ERR_INVALID;
    }
    if (rows < 0 || rows > 0x7fffffffLL || n_seg < 0 || n_tiles < 0 || scale_ld < rows ||
        !q_out || !scale_out) {
        set_error("%s: bad sizes or outputs", who);
        return QB_ERR_INVALID;
    }
    return QB_OK;
}

}  // namespace

extern "C" int qb_tree_attention_tiles(const int32_t* cu_a_host, int64_t n_seg, int32_t* tiles_host,
                                       int64_t capacity, int64_t* n_tiles) {
    // Host helper: the (segment, first row) list of 64-row query tiles,
    // longest-work tiles first is left to the caller; here in segment order.
    if (!cu_a_host || !tiles_host || !n_tiles || n_seg < 0)
        return qb::invalid("qb_tree_attention_tiles: NULL argument");
    int64_t count = 0;
    for (int64_t s = 0; s < n_seg; ++s) {
        for (int32_t r = cu_a_host[s]; r < cu_a_host[s + 1]; r += BM) {
            if (count >= capacity) return qb::invalid("qb_tree_attention_tiles: capacity");
            tiles_host[2 * count] = (int32_t)s;
            tiles_host[2 * count + 1] = r;
            ++count;
        }
    }
    *n_tiles = count;
    return QB_OK;
}

extern "C" int qb_tree_attention(const void* q, const void* k, const void* v, int64_t rows,
                                 int n_q, int n_kv, int head_dim, const int32_t* cu_a,
                                 int64_t n_seg, const int32_t* tiles, int64_t n_tiles,
                                 const int32_t* read_cu_q, const int32_t* read_used,
                                 const int32_t* read_table, int64_t n_reads,
                                 int64_t table_width, const int32_t* source, const void* k_pool,
                                 const void* v_pool, int64_t n_pages, int page_tokens,
                                 float softmax_scale, void* q_out, float* scale_out,
                                 int64_t scale_ld, void* stream) {
    const char* who = "qb_tree_attention";
    int st = check_common(who, rows, n_q, n_kv, head_dim, n_seg, n_tiles, scale_ld, q_out,
                          scale_out);
    if (st) return st;
    if (n_reads > 0 && (!read_cu_q || !read_used || !read_table || !source || !k_pool ||
                        !v_pool || table_width <= 0))
        return invalid("qb_tree_attention: reads need cu_q, used, table, source and pools");
    if (n_reads > 0 && (page_tokens <= 0 || BN % page_tokens != 0))
        return invalid("qb_tree_attention: page_tokens must divide 64");
    if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) ||
        (n_reads > 0 && (!aligned(k_pool, 16) || !aligned(v_pool, 16))))
        return invalid("qb_tree_attention: q, k, v and pools must be 16-byte aligned");
    if (n_tiles == 0 || rows == 0) return QB_OK;
    st = qb::launch_attention_tc(false, who, q, k, v, rows, n_q, n_kv, cu_a, tiles, n_tiles,
                                 read_cu_q, read_used, read_table, n_reads, table_width, source,
                                 k_pool, v_pool, n_pages, page_tokens, softmax_scale, q_out,
                                 scale_out, scale_ld, stream);
    if (st != -1) return st;
    return launch_attention<false>(who, q, k, v, rows, n_q, n_kv, cu_a, tiles, n_tiles,
                                   read_cu_q, read_used, read_table, n_reads, table_width, source,
                                   k_pool, v_pool, n_pages, page_tokens, softmax_scale, q_out,
                                   scale_out, scale_ld, stream);
}

extern "C" int qb_unified_attention(const void* q, int64_t rows, int n_q, int n_kv, int head_dim,
                                    const int32_t* cu_q, int64_t n_seq, const int32_t* tiles,
                                    int64_t n_tiles, const int32_t* used, const int32_t* table,
                                    int64_t table_width, const void* k_pool, const void* v_pool,
                                    int64_t n_pages, int page_tokens, float softmax_scale,
                                    void* q_out, float* scale_out, int64_t scale_ld,
                                    void* stream) {
    const char* who = "qb_unified_attention";
    int st = check_common(who, rows, n_q, n_kv, head_dim, n_seq, n_tiles, scale_ld, q_out,
                          scale_out);
    if (st) return st;
    if (!cu_q || !used || !table || !k_pool || !v_pool || table_width <= 0)
        return invalid("qb_unified_attention: needs cu_q, used, table and pools");
    if (page_tokens <= 0 || BN % page_tokens != 0)
        return invalid("qb_unified_attention: page_tokens must divide 64");
    if (!aligned(q, 16) || !aligned(k_pool, 16) || !aligned(v_pool, 16))
        return invalid("qb_unified_attention: q and pools must be 16-byte aligned");
    if (n_tiles == 0 || rows == 0) return QB_OK;
    st = qb::launch_attention_tc(true, who, q, nullptr, nullptr, rows, n_q, n_kv, cu_q, tiles,
                                 n_tiles, nullptr, used, table, 0, table_width, nullptr, k_pool,
                                 v_pool, n_pages, page_tokens, softmax_scale, q_out, scale_out,
                                 scale_ld, stream);
    if (st != -1) return st;
    return launch_attention<true>(who, q, k_pool, v_pool, rows, n_q, n_kv, cu_q, tiles, n_tiles,
                                  nullptr, used, table, 0, table_width, nullptr, k_pool, v_pool,
                                  n_pages, page_tokens, softmax_scale, q_out, scale_out, scale_ld,
                                  stream);
}
