// gkv_kernels.cuh -- launch parameters shared by the host pool
// (gkv_pool.cpp) and the sm_100a kernels (gkv_kernels.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gkv {

// Device status word bits (pool->d_status), read by gkv_device_status().
enum : int {
    DEV_ERR_WAIT_TIMEOUT = 1,  // an mbarrier wait ran out of its time limit
    DEV_ERR_BAD_PAGE = 2,      // a block-table entry outside [0, num_pages)
};

// ---------------------------------------------------------------- append
// One batch entry of an append / seed.
struct AppendEntry {
    int32_t seq_id;
    int32_t len_before;  // positions already in the sequence
    int32_t n_new;       // rows appended
    int32_t src_row0;    // first source row of this entry
};

// One page the append touches.  src_pid:
//   PAGE_EXISTING -> write only the appended rows
//   PAGE_NEW      -> zero-fill the page, then the appended rows, set table
//   >= 0          -> copy page src_pid (copy-on-write / clone tail), then the
//                    appended rows, set table
struct TouchedPage {
    int32_t entry;
    int32_t pidx;  // logical page index in the sequence
    int32_t pid;   // physical page
    int32_t src_pid;
};
constexpr int32_t PAGE_EXISTING = -1;
constexpr int32_t PAGE_NEW = -2;

// An append touching at most kAppendInlinePages pages of at most
// kAppendInlineEntries sequences carries its descriptor in the kernel's
// parameter block (no upload before the launch).
constexpr int kAppendInlineEntries = 128;
constexpr int kAppendInlinePages = 256;
struct AppendInline {
    AppendEntry entries[kAppendInlineEntries];
    TouchedPage pages[kAppendInlinePages];
};

struct AppendParams {
    const AppendEntry *entries;  // null: AppendInline::entries
    const TouchedPage *pages;    // null: AppendInline::pages
    int32_t n_pages;
    const uint16_t *k_src;  // token-major [rows, KVH, dh], or head-major: per entry [KVH, n_new, dh]
    const uint16_t *v_src;
    int32_t head_major;     // 1: head-major (seed; the reference's verify k / v [KVH, S, dh])
    uint16_t *k_pool;       // [num_pages, KVH, P, dh]
    uint16_t *v_pool;
    int32_t *table;         // [max_seqs, table_stride]
    int32_t table_stride;
    int32_t kvh, dh, P;
};

// ---------------------------------------------------------------- attend
// Row (query token s of sequence b, query head kvh*G + g) of q and out, in
// units of head_dim: token-major [n, n_q, KVH*G] (the default), or the
// reference's verify / batched-flash layout [n, KVH, n_q, G] -- per sequence
// [KVH, S, G, dh] (Engine.verifyAttn, Engine.swift:2618-2646;
// pagedFlashBatched, PagedAttention.swift:370-376).
__host__ __device__ inline int64_t qo_row(bool head_major, int64_t b, int s, int kvh, int g, int n_q, int KVH,
                                          int G) {
    return head_major ? ((b * KVH + kvh) * n_q + s) * G + g : (b * n_q + s) * (int64_t)(KVH * G) + kvh * G + g;
}

struct AttendEntry {
    int32_t seq_id;
    int32_t len;        // keys in the sequence (query rows are the last n_q)
    int32_t unit_base;  // first work unit of this sequence (kvh-major inside)
    int32_t ntiles;     // key tiles per kv head = ceil(len / TK)
};

// Fused append: the pages sequence b's n_q new rows (positions len-n_q ..
// len-1, n_q <= P) land on, in position order -- at most two: the partly
// filled tail page and one fresh page.
struct FusedTail {
    int32_t pid[2];    // physical pages
    int32_t pidx[2];   // their logical indices in the sequence; pidx[1] < 0: one page
    int32_t fresh[2];  // 1: just allocated (zero-filled, table entry written here)
    int32_t pad[2];
};

// Producer fusion (gkv_attn_step; q_gate == nullptr turns it off): the
// attend kernel builds its fp16 q rows from the raw q|gate projections --
// RMSNorm with q_norm, then partial NEOX RoPE of the first n_rot elements
// with the token's cos/sin row -- and multiplies every output by sigmoid of
// the gate half; the fused append builds the new K row the same way from
// k_raw (k_norm) and rounds v_raw to fp16 (SIMD/Attention.swift:72-139).
struct ProducerArgs {
    const float *q_gate;               // [n_seqs, n_q, KVH*G, 2*dh]: q | gate per head
    const float *k_raw, *v_raw;        // [n_seqs, KVH, dh]
    const float *q_norm, *k_norm;      // [dh]
    const float *rope_cos, *rope_sin;  // [n_seqs, n_q, n_rot/2]
    int32_t n_rot;
    float eps;
};

// The descriptor of a call with at most kInlineSeqs sequences travels in the
// attend kernel's parameter block instead of a device buffer: no upload sits
// between two launches, so a launch follows the previous kernel directly and
// its start-up overlaps that kernel's tail (programmatic dependent launch).
constexpr int kInlineSeqs = 128;
struct InlineDesc {
    AttendEntry entries[kInlineSeqs];
    FusedTail tails[kInlineSeqs];
};

struct AttendParams {
    const AttendEntry *entries;  // null: InlineDesc::entries
    int32_t n_seqs;
    int32_t total_units;
    // fused append (fused = 1): k_new/v_new [n_seqs * n_q, KVH, dh] fp16
    // ([n_seqs, KVH, n_q, dh] when head_major), the n_q new rows of every
    // sequence, written into the pool before the key
    // tiles holding them are loaded; tails (null: InlineDesc::tails) say where
    int32_t fused;
    const FusedTail *tails;
    const uint16_t *k_new, *v_new;
    uint16_t *k_pool_w, *v_pool_w;
    int32_t *table_w;
    const int32_t *table;
    int32_t table_stride;
    const uint16_t *k_pool;  // used by the cp.async loader (P < 8)
    const uint16_t *v_pool;
    const uint16_t *q;       // [n_seqs, n_q, KVH*G, dh], head_major: [n_seqs, KVH, n_q, G, dh]
    void *out;               // q's layout; fp32, or fp16 when out_f16
    int32_t head_major;      // q / out (and the fused append's k_new / v_new) head-major
    int32_t out_f16;         // out values rounded to fp16 (nearest even)
    float *partials;         // [n_items + grid, 32 + 16*dh]
    int32_t *counters;       // [n_items], zero between launches
    int32_t *status;         // device status word
    int32_t n_q, G, kvh, P, num_pages;
    float scale_log2;        // scale * log2(e)
    ProducerArgs prod;
};

// K/V rows of a producer step built outside the attend kernel (when the
// append cannot be fused): k_out/v_out [n_seqs, KVH, dh] fp16.
struct ProduceParams {
    ProducerArgs prod;
    uint16_t *k_out, *v_out;
    int32_t n_seqs, kvh;
};

// Host-side launchers (gkv_kernels.cu).
// One bounded wait on an mbarrier nothing arrives on (gkv_check_bounded_wait).
cudaError_t launch_bounded_wait_probe(int *status, uint64_t limit_ns, cudaStream_t s);
// inl: the inline descriptor when p.entries / p.pages are null.
cudaError_t launch_append(const AppendParams &p, cudaStream_t s, const AppendInline *inl = nullptr);
// Number of CTAs the attend launch will use for `units` work units (at
// most sm_count times the CTAs one SM holds; INT32_MAX units: the maximum).
int attend_grid(int dh, int P, int units, int sm_count);
// Floats of partial-result scratch per slot.
__host__ __device__ inline int64_t attend_partial_floats(int dh) { return 32 + 16 * (int64_t)dh; }
// desc: the inline descriptor when p.entries is null (else may be null).
cudaError_t launch_attend(const AttendParams &p, const CUtensorMap *tmap_k,
                          const CUtensorMap *tmap_v, int dh, int grid,
                          cudaStream_t s, const InlineDesc *desc = nullptr);
// Key tile length used by the attend kernel for head_dim dh.
int attend_tile_keys(int dh);
// True when the attend kernel can run the producer fusion for head_dim dh.
bool producer_supported(int dh);
cudaError_t launch_produce_kv(const ProduceParams &p, int dh, cudaStream_t s);

// ---------------------------------------------------------------- chunk
// Causal attention for many query rows per (sequence, kv head): prefill
// chunks and wide verify batches (n_q * G > 16).  One CTA per block of
// `qtok` query tokens x G heads (<= 128 rows = one tcgen05 M tile).
struct ChunkParams {
    const AttendEntry *entries;  // seq_id, len (unit fields unused)
    int32_t n_seqs;
    const int32_t *table;
    int32_t table_stride;
    const uint16_t *q;  // [n_seqs, n_q, KVH*G, dh], head_major: [n_seqs, KVH, n_q, G, dh]
    void *out;          // q's layout; fp32, or fp16 when out_f16
    int32_t head_major;
    int32_t out_f16;
    int32_t p_f16;      // P rounded once to fp16 (GKV_ATTEND_P_F16), else P_hi + P_lo
    int32_t *status;
    int32_t n_q, G, kvh, P, num_pages;
    int32_t qtok;       // query tokens per CTA
    int32_t n_qblocks;  // ceil(n_q / qtok)
    float scale_log2;
};
// True when the chunk kernel handles (dh, P, G).
bool chunk_supported(int dh, int P, int G);
cudaError_t launch_chunk(const ChunkParams &p, const CUtensorMap *tmap_k,
                         const CUtensorMap *tmap_v, int dh, cudaStream_t s);

// A window of a sequence into head-major [KVH, rows, dh]: output row r < count
// is position start + r, rows count..rows-1 are zero.  compact() is the
// window (0, len, len); tileAt() is (start, count, tile_p).
struct CompactParams {
    const int32_t *table;  // row of the sequence
    const uint16_t *k_pool, *v_pool;
    uint16_t *K, *V;       // [KVH, rows, dh]
    int64_t start, count, rows;
    int32_t kvh, dh, P;
};
cudaError_t launch_compact(const CompactParams &p, cudaStream_t s);

// Host helpers for gkv_attend_noalloc (gkv_pool.cpp): record the calling
// thread's gkv_last_error() message and return `code`; encode the attend
// kernel's TMA view of a caller-owned K or V page array.
int report_error(int code, const char *fmt, ...);
// GKV_OK when a kernel may read or write ptr from GPU `device` (-1: the
// current one): device memory of that GPU, managed memory, or -- host_ok --
// page-locked host memory mapped at the same address.  Pageable host memory
// would fault the kernel; it is refused with GKV_ERR_INVALID.  Null passes.
int check_reachable(const void *ptr, int device, bool host_ok, const char *what);
int encode_page_tensor_map(CUtensorMap *map, const void *pages, int num_pages, int kv_heads,
                           int page_tokens, int head_dim);

}  // namespace gkv
