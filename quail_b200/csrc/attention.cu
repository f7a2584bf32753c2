// Entry points of the tree and unified attention paths: argument checks on
// the host, then the tcgen05 kernel of attention_tc.cu. That kernel takes
// even GQA groups (2, 4 or a multiple of 4 query heads per KV head: every
// Qwen3 shape) and page sizes dividing 64; other shapes are rejected with
// QB_ERR_INVALID.
#include "common.cuh"

namespace qb {
// attention_tc.cu: the tcgen05 kernel; -1 = not its shapes
int launch_attention_tc(bool unified, const char* who, const void* q, const void* k,
                        const void* v, int64_t rows, int n_q, int n_kv, const int32_t* cu,
                        const int32_t* tiles, int64_t n_tiles, const int32_t* read_cu_q,
                        const int32_t* read_used, const int32_t* table, int64_t n_reads,
                        int64_t table_width, const int32_t* source, const void* k_pool,
                        const void* v_pool, int64_t n_pages, int page_tokens,
                        float softmax_scale, void* q_out, float* scale_out, int64_t scale_ld,
                        bool ue8m0, void* stream);
}  // namespace qb

namespace {

using namespace qb;

constexpr int D = 128;   // head dim
constexpr int BM = 64;   // query rows per tile
constexpr int BN = 64;   // keys per tile

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
                                 int64_t scale_ld, int ue8m0, void* stream) {
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
                                 scale_out, scale_ld, ue8m0 != 0, stream);
    if (st == -1)
        return invalid("qb_tree_attention: query heads per KV head must be 2, 4 or a multiple "
                       "of 4, and page_tokens a divisor of 64 of at least 8");
    return st;
}

extern "C" int qb_unified_attention(const void* q, int64_t rows, int n_q, int n_kv, int head_dim,
                                    const int32_t* cu_q, int64_t n_seq, const int32_t* tiles,
                                    int64_t n_tiles, const int32_t* used, const int32_t* table,
                                    int64_t table_width, const void* k_pool, const void* v_pool,
                                    int64_t n_pages, int page_tokens, float softmax_scale,
                                    void* q_out, float* scale_out, int64_t scale_ld,
                                    int ue8m0, void* stream) {
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
                                 scale_ld, ue8m0 != 0, stream);
    if (st == -1)
        return invalid("qb_unified_attention: query heads per KV head must be 2, 4 or a "
                       "multiple of 4, and page_tokens a divisor of 64 of at least 8");
    return st;
}
