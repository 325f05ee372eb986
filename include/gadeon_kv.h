/*
 * gadeon_kv.h -- C ABI of the B200 paged KV cache (libgadeonkv.so).
 *
 * One gkv_pool is the physical page pool of ONE full-attention layer on ONE
 * GPU: K and V pages of [kv_heads, page_tokens, head_dim] fp16, a block table
 * per sequence, and a seeded LIFO free list.  A sequence inside a pool plays
 * the role of the reference's per-layer PagePool
 * (leok7v/gadeon LLM/src/CoreML/PagedAttention.swift:21-287); the attend
 * entry points replace hostFlashDecode (:317-366), the causal verify loop
 * (LLM/src/CoreML/Engine.swift:2620-2646) and the batched prefill flash
 * (PagedAttention.swift:376-495), and on the Metal side MetalKVPool
 * (LLM/src/Metal/MetalKVPool.swift:20-126) with the kernels kv_append,
 * kv_append_batch, attn_head, attn_batch, attn_batch_mm
 * (LLM/metal/Kernels.metal:1265-1457, :1721-2014).
 *
 * Conventions
 *   - Every call returns a status (GKV_OK == 0); gkv_last_error() gives the
 *     calling thread's message for its last failure.  A failing call leaves
 *     the pool unchanged (validation happens before any mutation).
 *   - K/V/Q and outputs of the pool calls are device memory of the pool's
 *     GPU, managed memory, page-locked host memory mapped at the same
 *     address (cudaHostAlloc / cudaMallocHost / cudaHostRegister), or plain
 *     pageable host memory.  The kernels read and write page-locked host
 *     buffers in place over the host link; such a buffer must stay valid
 *     and unchanged until the stream has finished the call.  A kernel cannot
 *     reach pageable memory, so the call stages it through a page-locked
 *     bounce buffer the pool owns (grown with cudaHostAlloc when a call needs
 *     more), which the kernels read and write in place: pageable inputs are
 *     copied into it before the launch, pageable outputs out of it after the
 *     launch has finished.  A call with a pageable output returns once that
 *     output is in place (it waits for the device); pageable inputs may be
 *     reused as soon as the call returns.  The GDN rollback and
 *     gkv_attend_noalloc take device memory only.  Id and length arrays are
 *     HOST pointers.  `stream` is a cudaStream_t (NULL = the legacy default
 *     stream).  Work is enqueued asynchronously.
 *   - Host bookkeeping (lengths, block tables, free list) is updated when the
 *     call returns; the device copy of the tables is updated in stream order.
 *   - A pool is not thread-safe: serialise calls on one pool (the reference
 *     serialises them inside one Swift actor, Engine.swift:41) and issue all
 *     of its work on one stream, or order the streams yourself.
 *   - fp16 values are IEEE binary16 bit patterns; attention accumulates in
 *     fp32 and writes fp32 (or fp16, GKV_ATTEND_OUT_F16).
 */
#ifndef GADEON_KV_H
#define GADEON_KV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct gkv_pool gkv_pool;

enum gkv_status {
    GKV_OK = 0,
    GKV_ERR_INVALID = 1,     /* bad argument, shape or geometry */
    GKV_ERR_NO_PAGES = 2,    /* free list exhausted (pool left unchanged) */
    GKV_ERR_CUDA = 3,        /* a CUDA runtime/driver call failed */
    GKV_ERR_BAD_SEQ = 4,     /* unknown/released sequence, or length out of range */
    GKV_ERR_UNSUPPORTED = 5, /* geometry with no kernel in this build */
    GKV_ERR_CAPACITY = 6     /* max_seqs or max_pages_per_seq exceeded */
};

/* Message for the calling thread's last failing call ("" if none).  No
 * reference counterpart: the Swift's thrown errors carry their message. */
const char *gkv_last_error(void);
/* Library version string.  No reference counterpart. */
const char *gkv_version(void);

typedef struct gkv_pool_config {
    int32_t device;            /* CUDA device ordinal */
    int32_t kv_heads;          /* KVH (2 or 4 for Qwen3.5 hybrids) */
    int32_t head_dim;          /* dh: 64, 128, 256 or 512 */
    int32_t page_tokens;       /* P: power of two, 1..16384 */
    int32_t num_pages;         /* physical pages in this pool */
    int32_t max_seqs;          /* block-table rows */
    int32_t max_pages_per_seq; /* block-table row length (context <= this * P) */
    uint64_t seed;             /* free-list permutation seed */
} gkv_pool_config;

/* Create a pool (PagePool.init(P:kvHeads:dh:), PagedAttention.swift:40;
 * MetalKVPool.init, MetalKVPool.swift:34).  The free list's pop order is the
 * splitmix64 Fisher-Yates permutation of 0..num_pages-1 for `seed`. */
int gkv_pool_create(const gkv_pool_config *cfg, gkv_pool **out);
int gkv_pool_destroy(gkv_pool *pool);

/* A new empty sequence (a new PagePool, PagedAttention.swift:40-42); ids
 * are the lowest unused id. */
int gkv_seq_create(gkv_pool *pool, int32_t *seq_id);
/* Drop every page of the sequence (last page first) and retire its id: the
 * end of a PagePool, whose pages Swift's ARC frees (PagedAttention.swift
 * :25-26). */
int gkv_seq_release(gkv_pool *pool, int32_t seq_id);
/* PagePool.length / pageCount (PagedAttention.swift:27, :79). */
int gkv_seq_length(const gkv_pool *pool, int32_t seq_id, int64_t *length);
int gkv_seq_page_count(const gkv_pool *pool, int32_t seq_id, int32_t *pages);
int gkv_free_page_count(const gkv_pool *pool, int32_t *pages);

/* Batched append (PagePool.append(k:v:), PagedAttention.swift:85-94, called
 * per row by Engine.stepHidden :1921, batchedAttn :1797-1800 and verifyAttn
 * :2629-2630; Metal kv_append / kv_append_batch, Kernels.metal:1446-1457,
 * :1726-1740).  Sequence seq_ids[i] takes n_new[i] rows; k and v are
 * token-major [sum(n_new), kv_heads, head_dim] fp16, rows in batch order.
 * A page is allocated (and zero-filled) whenever a row lands on slot 0. */
int gkv_append(gkv_pool *pool, int32_t n_seqs, const int32_t *seq_ids,
               const int32_t *n_new, const void *k, const void *v,
               void *stream);

/* PagePool.seed(K:V:count:) (PagedAttention.swift:99-112): bulk-load an
 * EMPTY sequence from head-major [kv_heads, count, head_dim] fp16. */
int gkv_seed(gkv_pool *pool, int32_t seq_id, const void *K, const void *V,
             int64_t count, void *stream);

/* Paged GQA attention over the block tables (hostFlashDecode,
 * PagedAttention.swift:317-366; causal verify Engine.swift:2620-2646; Metal
 * attn_head / attn_batch, Kernels.metal:1423-1439, :1767-1793).
 * Each sequence's n_q query rows are its LAST n_q positions (append them
 * first): row r sees keys [0, length - n_q + r].  n_q == 1 is single-token
 * decode (the newest query sees every key, like hostFlashDecode).
 * q: [n_seqs, n_q, kv_heads*group, head_dim] fp16 (head h = kvh*group + g,
 * PagedAttention.swift:331-332); out: same shape, fp32.
 * scale multiplies q.k (hostFlashDecode uses head_dim^-0.5, :321); it must
 * be finite and non-zero.  Up to 16 rows per kv head (n_q*group <= 16) run
 * the split-K decode/verify kernel; more rows (prefill chunks) run the
 * tensor-core chunk kernel, which needs head_dim <= 256 and page_tokens >= 8
 * (else GKV_ERR_UNSUPPORTED). */
int gkv_attend(gkv_pool *pool, int32_t n_seqs, const int32_t *seq_ids,
               int32_t n_q, int32_t group, const void *q, float *out,
               float scale, void *stream);

/* The two attention forms under their own names, for callers that bind
 * decode and causal attention separately: gkv_attend_decode is gkv_attend
 * with n_q = 1 (hostFlashDecode, PagedAttention.swift:317-366; Metal
 * attn_head, Kernels.metal:1423-1439); gkv_attend_causal is gkv_attend
 * (verifyAttn, Engine.swift:2620-2646; pagedFlashBatched,
 * PagedAttention.swift:376-416; Metal attn_batch, Kernels.metal:1767-1793). */
int gkv_attend_decode(gkv_pool *pool, int32_t n_seqs, const int32_t *seq_ids,
                      int32_t group, const void *q, float *out, float scale,
                      void *stream);
int gkv_attend_causal(gkv_pool *pool, int32_t n_seqs, const int32_t *seq_ids,
                      int32_t n_q, int32_t group, const void *q, float *out,
                      float scale, void *stream);

/* One decode / verify / chunk step in one call: gkv_append of n_q rows per
 * sequence followed by gkv_attend of those n_q rows (Engine.stepHidden's
 * append + hostFlashDecode, Engine.swift:1921-1927; verifyAttn, :2620-2646;
 * batchedAttn, :1797-1820). */
int gkv_append_attend(gkv_pool *pool, int32_t n_seqs, const int32_t *seq_ids,
                      int32_t n_q, int32_t group, const void *k,
                      const void *v, const void *q, float *out, float scale,
                      void *stream);

/* Layout and output options of gkv_attend_ex / gkv_append_attend_ex. */
enum gkv_attend_flags {
    /* q and out [n_seqs, kv_heads, n_q, group, head_dim] -- per sequence
     * the reference's [KVH, S, G, dh] (verifyAttn's q and attn_out,
     * Engine.swift:2618-2646; pagedFlashBatched's q and result,
     * PagedAttention.swift:370-376) -- and gkv_append_attend_ex's k and v
     * [n_seqs, kv_heads, n_q, head_dim] (verifyAttn's k/v rows, [KVH, S, dh]
     * per sequence, Engine.swift:2051-2072) */
    GKV_ATTEND_HEAD_MAJOR = 1,
    /* out holds fp16: each fp32 result rounded to nearest even (verifyAttn
     * stores Float16(flat[...]), Engine.swift:2637) */
    GKV_ATTEND_OUT_F16 = 2,
    /* The tensor-core chunk path (n_q * group > 16) multiplies V by the
     * softmax weights rounded once to fp16, as the reference's Metal
     * attn_batch_mm does (half P tile times half V into fp32,
     * Kernels.metal:1891-1912), instead of by an fp16 pair P_hi + P_lo: a
     * third fewer tensor-core operations, and each output element within
     * 2^-10 x sum_i w_i |V_i| (+ fp32 rounding) of the exact result rather
     * than within the element-wise tolerance of the fp32 host path.  The
     * decode / verify path (n_q * group <= 16) ignores it: its split costs no
     * MMA there. */
    GKV_ATTEND_P_F16 = 4
};

/* gkv_attend with `flags` (gkv_attend_flags) choosing the layout of q and
 * out and the type of out; written by the kernels directly, with no extra
 * pass (pagedFlashBatched, PagedAttention.swift:376-416, with flags =
 * GKV_ATTEND_HEAD_MAJOR).  flags == 0 is gkv_attend. */
int gkv_attend_ex(gkv_pool *pool, int32_t n_seqs, const int32_t *seq_ids,
                  int32_t n_q, int32_t group, const void *q, void *out,
                  float scale, uint32_t flags, void *stream);

/* gkv_append_attend with `flags`: Engine.verifyAttn (Engine.swift:2620-2646)
 * as one call with flags = GKV_ATTEND_HEAD_MAJOR | GKV_ATTEND_OUT_F16 --
 * k, v [n_seqs, KVH, S, dh], q [n_seqs, KVH, S, G, dh], out fp16
 * [n_seqs, KVH, S, G, dh].  flags == 0 is gkv_append_attend. */
int gkv_append_attend_ex(gkv_pool *pool, int32_t n_seqs,
                         const int32_t *seq_ids, int32_t n_q, int32_t group,
                         const void *k, const void *v, const void *q,
                         void *out, float scale, uint32_t flags,
                         void *stream);

/* One decode token of a Qwen3.5 full-attention layer from its raw
 * projections, with the producer and the output gate fused into the append
 * and attention (Attn.step, LLM/src/SIMD/Attention.swift:72-139; Metal
 * split_qgate / rope_neox / gated attn_head, LLM/metal/Kernels.metal
 * :1100-1117, :1250-1262, :1330-1332):
 *   q, gate = split of q_gate [n_seqs, kv_heads*group, 2*head_dim] per head
 *   q = rope(rmsnorm(q, q_norm)), k = rope(rmsnorm(k_raw, k_norm))
 *   append (k, v_raw) as fp16 rows; out = attend(q) * sigmoid(gate)
 * rmsnorm: x / sqrt(mean(x^2) + eps) * w (Kernels.swift:26-37); rope: NEOX
 * on the first n_rot elements, pair (i, i + n_rot/2) rotated by this token's
 * rope_cos / rope_sin row [n_seqs, n_rot/2] (Kernels.swift:66-84; the
 * CoreML engine feeds such tables to its programs, Engine.swift:2168-2181).
 * k_raw, v_raw [n_seqs, kv_heads, head_dim]; q_norm, k_norm [head_dim];
 * out [n_seqs, kv_heads*group, head_dim]; every buffer fp32 on the device.
 * head_dim 128 or 256, group <= 16, n_rot a multiple of 16 <= head_dim. */
int gkv_attn_step(gkv_pool *pool, int32_t n_seqs, const int32_t *seq_ids,
                  int32_t group, const float *q_gate, const float *k_raw,
                  const float *v_raw, const float *q_norm, const float *k_norm,
                  float eps, const float *rope_cos, const float *rope_sin,
                  int32_t n_rot, float scale, float *out, void *stream);

/* Host helper: rope tables for gkv_attn_step, row t for position
 * positions[t]: angle = pos * base^(-2i/n_rot) in fp32, cos/sin (the
 * formula of Kernels.swift:74-76).  cos_out, sin_out: HOST [n, n_rot/2]. */
int gkv_rope_table(int32_t n_rot, float base, int32_t n,
                   const int64_t *positions, float *cos_out, float *sin_out);

/* PagePool.truncate(to:) for a batch (PagedAttention.swift:181-189; the
 * rollback of Engine.decodeSpecStep :2787, :2792): lengths drop to
 * new_len[i]; whole pages past ceil(new_len/P) leave the table last-first and
 * return to the free list when no clone shares them.  The kept tail keeps
 * its stale rows.  Host bookkeeping only: no device work is enqueued. */
int gkv_truncate(gkv_pool *pool, int32_t n_seqs, const int32_t *seq_ids,
                 const int64_t *new_len);

/* The drafter-pool maintenance of an MTP cycle (Engine.decodeSpecStep,
 * LLM/src/CoreML/Engine.swift:2788-2797: mtpPool.truncate(to: mtpBase),
 * then the m committed positions re-appended) in one call: sequence i is
 * truncated to base_len[i] and then n_new[i] rows of k / v (layout of
 * gkv_append) are appended.  Page-for-page the same as gkv_truncate
 * followed by gkv_append; if the append cannot be placed the truncate is
 * undone too. */
int gkv_rewind_append(gkv_pool *pool, int32_t n_seqs, const int32_t *seq_ids,
                      const int64_t *base_len, const int32_t *n_new,
                      const void *k, const void *v, void *stream);

/* PagePool.clone() (PagedAttention.swift:199-210; MetalKVPool.snapshot,
 * MetalKVPool.swift:102-109): a new sequence sharing every page of `src`,
 * with a private copy of a partially filled tail page. */
int gkv_clone_seq(gkv_pool *pool, int32_t src, int32_t *dst, void *stream);

/* PagePool.compact() (PagedAttention.swift:225-252): K and V as head-major
 * [kv_heads, length, head_dim] fp16 device buffers. */
int gkv_compact_seq(gkv_pool *pool, int32_t seq_id, void *K, void *V,
                    void *stream);

/* PagePool.tileAt(_:_:_:) (PagedAttention.swift:151-161): positions
 * [start, start + count) of the sequence into head-major
 * [kv_heads, tile_p, head_dim] fp16 K and V tiles, rows count..tile_p-1
 * zero -- the key window of one carry tile of pagedFlashCarry, which calls
 * it with start = i*tile_p and count = min(tile_p, length - start)
 * (:466-481).  Needs 0 <= count <= tile_p and start + count <= length
 * (else GKV_ERR_INVALID / GKV_ERR_BAD_SEQ).  The window may span pages (the
 * reference's never does: its page size is a multiple of tile_p). */
int gkv_tile_at(gkv_pool *pool, int32_t seq_id, int64_t start, int64_t count,
                int32_t tile_p, void *K, void *V, void *stream);

/* PagePool.fromCompact (PagedAttention.swift:256-264): a new sequence seeded
 * from head-major [kv_heads, length, head_dim] fp16 device buffers. */
int gkv_from_compact(gkv_pool *pool, const void *K, const void *V,
                     int64_t length, int32_t *seq_id, void *stream);

/* The pool section of Engine.serialize (Engine.swift:1078-1087): into the
 * HOST buffer buf, little-endian Int64 framing --
 *   count, then per layer in ascending layer id:
 *   layer, length, n, K[n] fp16, n, V[n] fp16   (n = kv_heads*length*head_dim,
 *   K/V head-major as PagePool.compact)
 * -- for sequence seq_ids[i] of pools[i] under layer id layer_ids[i].
 * buf == NULL: only *size is set (the bytes needed).  Synchronizes stream. */
int gkv_serialize(int32_t n_layers, gkv_pool *const *pools,
                  const int32_t *layer_ids, const int32_t *seq_ids, void *buf,
                  int64_t cap, int64_t *size, void *stream);

/* Engine.deserialize's pool half (Engine.swift:1106-1116): reads that
 * section from the HOST buffer into pools[i] (given in the data's layer
 * order) through gkv_from_compact; returns the new sequence ids, the layer
 * ids read and the bytes consumed.  The whole section is checked against
 * the pools' geometry before any sequence is made; a failing call changes
 * nothing.  Synchronizes stream. */
int gkv_deserialize(int32_t n_layers, gkv_pool *const *pools, const void *buf,
                    int64_t size, int32_t *layer_ids_out,
                    int32_t *seq_ids_out, int64_t *consumed, void *stream);

/* StateBytes header (Shared/StateBytes.swift:12-40): "GDNS" then Int64
 * version 1, 12 bytes.  gkv_state_header writes it (buf == NULL: *size
 * only); gkv_state_read_header accepts it and sets *offset to the payload,
 * else returns GKV_ERR_INVALID.  Host only. */
int gkv_state_header(void *buf, int64_t cap, int64_t *size);
int gkv_state_read_header(const void *buf, int64_t size, int64_t *offset);

/* ---- the GDN state rollback that runs beside gkv_truncate in an MTP cycle
 * (Engine.rollbackGDN, LLM/src/CoreML/Engine.swift:2678-2716) ---- */

/* MtpRollback.stateAfter (LLM/src/CoreML/MtpRollback.swift:47-60) for a batch
 * of n_items (sequence x GDN layer) items, item i with accepted prefix m[i]
 * in 1..C (HOST array):
 *   S_m[h] = exp(g[h,m-1]) S0[h] + sum_{t<m} exp(g[h,m-1]-g[h,t]) k[h,t] x delta[h,t]
 * Device fp32 buffers: s0/out [n_items, H, DK, DV], delta [n_items, H, C, DV],
 * k [n_items, H, C, DK], gcum [n_items, H, C] (inclusive gate cumsum).
 * C <= 64; every m[i] in 1..C; buffers 4-byte aligned (rows stream as
 * float4 when DV is a multiple of 4 and s0/delta/out are 16-byte aligned). */
int gkv_mtp_rollback(int32_t n_items, const int32_t *m, int32_t H, int32_t DK,
                     int32_t DV, int32_t C, const float *s0,
                     const float *delta, const float *k, const float *gcum,
                     float *out, void *stream);

/* Engine.convFromProj (Engine.swift:2719-2740) for a batch: conv state
 * [conv_dim, taps] after m[i] committed tokens; tap t holds position
 * m - taps + t, from this chunk's conv-projection rows proj [n_items, C,
 * conv_dim] when >= 0, else from the pre-verify tail pre [n_items, conv_dim,
 * taps] (oldest..newest).  out [n_items, conv_dim, taps]; all fp32 device. */
int gkv_conv_rollback(int32_t n_items, const int32_t *m, int32_t conv_dim,
                      int32_t taps, int32_t C, const float *proj,
                      const float *pre, float *out, void *stream);

/* gkv_mtp_rollback with the state stored as the reference stores it: fp16
 * (Engine.rollbackGDN, Engine.swift:2697-2705, reads the fp16 gdnState rec
 * arrays through floats() and writes MtpRollback.stateAfter's result back
 * through fp16Array).  s0 / out: fp16 [n_items, H, DK, DV], 2-byte aligned;
 * delta, k, gcum fp32 as above.  Each element is widened exactly, computed
 * in fp32 in the same order as gkv_mtp_rollback, and rounded to nearest
 * even: out == fp16(gkv_mtp_rollback(fp32(s0))) bit for bit.  Half the
 * state bytes of the fp32 entry point. */
int gkv_mtp_rollback_f16(int32_t n_items, const int32_t *m, int32_t H,
                         int32_t DK, int32_t DV, int32_t C, const void *s0,
                         const float *delta, const float *k,
                         const float *gcum, void *out, void *stream);

/* gkv_conv_rollback with the fp16 conv tail of the reference
 * (convFromProj, Engine.swift:2719-2740, writes Float16(val)): pre / out
 * fp16 [n_items, conv_dim, taps]; proj fp32.  A proj value is rounded to
 * nearest even, a carried tap is copied unchanged. */
int gkv_conv_rollback_f16(int32_t n_items, const int32_t *m, int32_t conv_dim,
                          int32_t taps, int32_t C, const float *proj,
                          const void *pre, void *out, void *stream);

/* The whole of Engine.rollbackGDN (Engine.swift:2678-2716) for a batch with
 * fp16 storage: gkv_mtp_rollback_f16 of (s0, delta, k, gcum) -> state_out
 * and gkv_conv_rollback_f16 of (proj, pre) -> conv_out, the same items and
 * m, in one launch when both shapes take the vector kernels (DV % 8 == 0,
 * C <= 8, DK <= 256, conv_dim % 8 == 0, taps <= 4, 16-byte aligned arrays),
 * else as those two calls.  Results identical to the two calls. */
int gkv_gdn_rollback_f16(int32_t n_items, const int32_t *m, int32_t H,
                         int32_t DK, int32_t DV, int32_t C, const void *s0,
                         const float *delta, const float *k, const float *gcum,
                         void *state_out, int32_t conv_dim, int32_t taps,
                         const float *proj, const void *pre, void *conv_out,
                         void *stream);
/* The same with fp32 storage (Engine.swift:2678-2716 over fp32 arrays):
 * gkv_mtp_rollback + gkv_conv_rollback in one launch (DV % 4 == 0 for the
 * state's vector kernel). */
int gkv_gdn_rollback(int32_t n_items, const int32_t *m, int32_t H, int32_t DK,
                     int32_t DV, int32_t C, const float *s0,
                     const float *delta, const float *k, const float *gcum,
                     float *state_out, int32_t conv_dim, int32_t taps,
                     const float *proj, const float *pre, float *conv_out,
                     void *stream);

/* Size of the library's static scratch array used by gkv_attend_noalloc
 * (held on every GPU that loads the library until the process exits), and
 * the largest batch and kv-head count that entry point takes.  With at most
 * GKV_NOALLOC_MAX_KV_HEADS kv heads every head_dim fits the array: a larger
 * batch simply runs as more launches. */
#define GKV_NOALLOC_SCRATCH_BYTES 8388608u
#define GKV_NOALLOC_MAX_SEQS 1024
#define GKV_NOALLOC_MAX_KV_HEADS 64

/* Paged GQA decode / verify attention that allocates nothing.  No
 * counterpart in the reference.  For callers that own all device memory
 * and cannot call cudaMalloc while serving (an engine with one arena
 * reserved at start-up, or a language binding with its own allocator): the
 * K/V pages ([num_pages][kv_heads][page_tokens][head_dim] fp16 each), the
 * block table (device int32, row i = batch entry i, table_stride entries)
 * and q/out are the caller's; seq_lens is a HOST array of the n_seqs
 * lengths.  q, out, n_q, group and scale mean what they mean for
 * gkv_attend, and the results match it.  The kernel's scratch (merge
 * counters, split-K partials, a status word) lives in one static __device__
 * array of GKV_NOALLOC_SCRATCH_BYTES; nothing is copied from the host (the
 * work descriptor rides in the kernel's parameter block, a batch of more
 * than 128 sequences runs as several launches on `stream`).  More than
 * GKV_NOALLOC_MAX_SEQS sequences or GKV_NOALLOC_MAX_KV_HEADS kv heads fail
 * with GKV_ERR_CAPACITY.  A block-table entry outside [0, num_pages) is
 * read as page 0 and recorded in the status word, which gkv_noalloc_status
 * reports.  The first call on each device looks up that array's device
 * address (set-up), so make that first call before any stream capture.
 * Calls share the array: calls that overlap on the GPU (other streams,
 * other threads) race. */
int gkv_attend_noalloc(const void *k_pages, const void *v_pages,
                       int32_t num_pages, int32_t kv_heads, int32_t head_dim,
                       int32_t page_tokens, const int32_t *block_table,
                       int32_t table_stride, int32_t n_seqs,
                       const int32_t *seq_lens, int32_t n_q, int32_t group,
                       const void *q, float *out, float scale, void *stream);

/* The device status bits gkv_attend_noalloc calls on the CURRENT device
 * left since the last read (bit 1 = a bounded wait ran out, bit 2 = a
 * block-table entry was outside the pages), then cleared.  Waits for
 * `stream`.  No counterpart in the reference (its device errors surface
 * through Metal command buffers, MetalGolden.swift:384). */
int gkv_noalloc_status(void *stream, int32_t *status);

/* ---- state export, for parity checks and debugging (synchronous) ---- */

/* State export for parity checks (no reference counterpart: the reference
 * keeps no block table or free list).
 * The sequence's block table as held ON THE DEVICE (first `pages` entries;
 * waits for the device).  cap = room in `pages_out`. */
int gkv_export_table(gkv_pool *pool, int32_t seq_id, int32_t *pages_out,
                     int32_t cap, int32_t *n_pages);
/* The free list in pop order (head first); no reference counterpart. */
int gkv_export_free_list(const gkv_pool *pool, int32_t *out, int32_t cap,
                         int32_t *n);
/* Reference count of a physical page (0 = free); no reference counterpart
 * (PagePool.clone shares pages by ARC, PagedAttention.swift:199-210). */
int gkv_page_refcount(const gkv_pool *pool, int32_t page_id, int32_t *ref);
/* Copy one physical page's K and V ([kv_heads, P, head_dim] fp16 each) to
 * host memory (waits for the device): the bytes of PagePool.kPage(_:) /
 * vPage(_:) (PagedAttention.swift:80-81) by physical id. */
int gkv_export_page(gkv_pool *pool, int32_t page_id, void *k_host,
                    void *v_host);
/* Waits for the device and returns the pool's device status word: 0, or
 * bit 1 = a kernel's bounded wait ran out, bit 2 = a block-table entry was
 * outside the pool.  No reference counterpart (the reference's device
 * errors surface through Metal command buffers, MetalGolden.swift:384). */
int gkv_device_status(gkv_pool *pool, int32_t *status);

/* Failure-detection check (no reference counterpart): on `device`, one
 * thread waits -- through the bounded wait every kernel of this library
 * uses on its mbarriers -- on a barrier that nothing ever arrives on.  The
 * wait gives up after limit_ns (1 ms .. 10 s), records the timeout and
 * returns, so the context stays usable; *status receives the status bits
 * (1 = a bounded wait ran out, the expected result).  Synchronizes the
 * device. */
int gkv_check_bounded_wait(int32_t device, int64_t limit_ns, int32_t *status);

#ifdef __cplusplus
}
#endif

#endif /* GADEON_KV_H */
