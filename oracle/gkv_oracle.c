/*
 * gkv_oracle.c -- CPU oracle for the paged KV-cache hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py load this library, and
 * only as the checker (or the timed CPU baseline).  The product library
 * (gadeon_b200/libgadeonkv.so) never links or calls it.
 *
 * What it restates (reference = leok7v/gadeon, paths relative to the
 * project root):
 *
 *   PagePool (LLM/src/CoreML/PagedAttention.swift:21-287)
 *     - a page is [KVH, P, dh] fp16, head-major inside the page
 *       (writePosition :116-127, zeroPage :278-286)
 *     - append: a fresh ZEROED page when length % P == 0, then one row per
 *       kv head at slot length % P (:85-94)
 *     - seed: bulk [KVH, count, dh] into ceil(count/P) fresh pages, tail
 *       zero-padded (:99-112, copyPrefix :131-143)
 *     - truncate: length = n; pop pages from the END until
 *       pageCount == ceil(n/P); the kept tail keeps its stale rows (:181-189)
 *     - clone: share every page, duplicate only a partial tail (:199-210)
 *     - compact / fromCompact: page-strided <-> [KVH, len, dh] (:225-276)
 *
 *   hostFlashDecode (PagedAttention.swift:317-366)
 *     for each kv head h, group member g (head = h*G + g, :331-332):
 *       s_j = (K_j . q) * scale          (vDSP_mmul -> plain fp32 dot)
 *       m   = max_j s_j
 *       e_j = exp(s_j - m); sum += e_j   (sequential fp32)
 *       o   = (sum_j e_j V_j) * (1/sum)  (vDSP_mmul -> plain fp32 loop)
 *     No mask: the query sees every one of `length` keys.
 *     Transcribed Apple-framework lines: vDSP_mmul -> explicit fp32 loops;
 *     vImageConvert_Planar16FtoPlanarF -> exact binary16 -> binary32
 *     widening (f16_to_f32 below).  vDSP's own summation order is not
 *     specified, so outputs compare by tolerance, never bits.
 *
 *   Causal verify / chunk (Engine.swift:2620-2646 verifyAttn; the per-token
 *   CPU route Engine.swift:1220-1224): append row s, then hostFlashDecode of
 *   query row s -- row s of a batch that starts at p0 sees keys [0, p0+s].
 *
 *   GDN rollback after an accepted speculative prefix (MtpRollback.stateAfter,
 *   LLM/src/CoreML/MtpRollback.swift:20-60; Engine.convFromProj,
 *   Engine.swift:2719-2740), pinned by the reference's own known answers
 *   (LLM/tests/MtpRollbackTests.swift).
 *
 * The block pool, block tables and free list do NOT exist in the reference
 * (each PagePool is a private array of ARC'd pages).  The oracle defines the
 * one explicit model that the GPU library mirrors bit-for-bit:
 *   - one physical pool of num_pages page ids per layer;
 *   - the free list is a LIFO stack; its initial pop order is a seeded
 *     Fisher-Yates permutation of 0..num_pages-1 driven by splitmix64
 *     (j = next() % (i+1), i from n-1 down to 1, starting from identity);
 *   - allocation pops from the head, in the order appends cross page
 *     boundaries: batch order of the sequences, ascending slots;
 *   - an allocated page is zero-filled (zeroPage);
 *   - pages carry a reference count (clone shares pages); truncate drops
 *     table entries last-first and pushes a page back on the free list
 *     when its count reaches zero (mirrors the removeLast loop);
 *   - an append whose tail page is shared first copies it to a fresh page
 *     (copy-on-write).  The reference writes into the shared page in that
 *     case, which would corrupt the bookmark it shares it with; the model
 *     fixes that on purpose;
 *   - sequence ids are the lowest unused id.
 *
 * Parity status: the reference is Swift + Accelerate + CoreML and cannot be
 * built or run here, and its repository commits no golden vectors for this
 * path.  This oracle is therefore "parity unpinned" against reference
 * outputs; it is checked against analytic known-answer cases (tests) and
 * against the golden fixtures it generated itself (tests/golden).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_OK 0
#define ORC_ERR_INVALID 1
#define ORC_ERR_NO_PAGES 2
#define ORC_ERR_BAD_SEQ 4

/* ------------------------------------------------------------------ */
/* fp16 <-> fp32 (IEEE binary16, round to nearest even)               */
/* ------------------------------------------------------------------ */

float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1f;
    uint32_t man = h & 0x3ff;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: normalise */
            int e = -1;
            do { man <<= 1; e++; } while ((man & 0x400) == 0);
            man &= 0x3ff;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t orc_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000;
    uint32_t absx = x & 0x7fffffffu;
    if (absx >= 0x7f800000u) { /* inf / nan */
        return (uint16_t)(sign | 0x7c00 | (absx > 0x7f800000u ? 0x200 : 0));
    }
    if (absx >= 0x477ff000u) return (uint16_t)(sign | 0x7c00); /* overflow */
    int32_t e = (int32_t)(absx >> 23) - 127;
    uint32_t man = absx & 0x7fffff;
    if (e < -14) { /* subnormal or zero in fp16 */
        if (e < -25) return (uint16_t)sign;
        man |= 0x800000;
        int shift = -e - 14 + 13; /* 14..24 */
        uint32_t q = man >> shift;
        uint32_t rem = man & ((1u << shift) - 1);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t q = ((uint32_t)(e + 15) << 10) | (man >> 13);
    uint32_t rem = man & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (q & 1))) q++;
    return (uint16_t)(sign | q);
}

void orc_f16_to_f32_array(const uint16_t *src, float *dst, int64_t n) {
    for (int64_t i = 0; i < n; i++) dst[i] = orc_f16_to_f32(src[i]);
}

/* orc_f16_to_f32 tabulated for all 65,536 inputs (filled once, from the
 * function above, so the two agree bit for bit): widening the fp32 mirror
 * is a table lookup per element. */
static float f16_table[65536];
static pthread_once_t f16_table_once = PTHREAD_ONCE_INIT;

static void f16_table_fill(void) {
    for (uint32_t h = 0; h < 65536; h++) f16_table[h] = orc_f16_to_f32((uint16_t)h);
}

static const float *f16_lut(void) {
    pthread_once(&f16_table_once, f16_table_fill);
    return f16_table;
}

void orc_f32_to_f16_array(const float *src, uint16_t *dst, int64_t n) {
    for (int64_t i = 0; i < n; i++) dst[i] = orc_f32_to_f16(src[i]);
}

/* ------------------------------------------------------------------ */
/* seeded generators                                                   */
/* ------------------------------------------------------------------ */

static uint64_t splitmix64(uint64_t *s) {
    uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* N(0,1) draws: splitmix64 -> two uniforms in (0,1] (53-bit) -> Box-Muller
 * in double -> float -> fp16 RNE.  `stream` selects an independent
 * sequence for the same seed. */
void orc_fill_normal_f16(uint64_t seed, uint64_t stream, uint16_t *out,
                         int64_t n) {
    uint64_t s = seed ^ (stream * 0xD1B54A32D192ED03ull);
    const double two_pi = 6.283185307179586476925286766559;
    int64_t i = 0;
    while (i < n) {
        double u1 = ((double)(splitmix64(&s) >> 11) + 1.0) * (1.0 / 9007199254740992.0);
        double u2 = ((double)(splitmix64(&s) >> 11)) * (1.0 / 9007199254740992.0);
        double r = sqrt(-2.0 * log(u1));
        out[i++] = orc_f32_to_f16((float)(r * cos(two_pi * u2)));
        if (i < n) out[i++] = orc_f32_to_f16((float)(r * sin(two_pi * u2)));
    }
}

/* The free list's initial pop order. */
void orc_permutation(uint64_t seed, int32_t n, int32_t *out) {
    uint64_t s = seed;
    for (int32_t i = 0; i < n; i++) out[i] = i;
    for (int32_t i = n - 1; i > 0; i--) {
        int32_t j = (int32_t)(splitmix64(&s) % (uint64_t)(i + 1));
        int32_t t = out[i];
        out[i] = out[j];
        out[j] = t;
    }
}

/* ------------------------------------------------------------------ */
/* block pool model                                                    */
/* ------------------------------------------------------------------ */

typedef struct {
    int active;
    int64_t len;
    int32_t *pages;
    int32_t npages, cap;
    /* fp32 mirror (PagePool.kF32/vF32/f32Len, PagedAttention.swift:36-38):
     * per kv head [mcap, dh], valid up to the watermark f32len. */
    float *kf, *vf;
    int64_t mcap, f32len;
} OrcSeq;

typedef struct {
    int kvh, dh, P, num_pages;
    int64_t page_elems; /* KVH * P * dh halves */
    uint16_t *k, *v;    /* [num_pages][KVH][P][dh] */
    int32_t *stack;     /* free list, top = stack[top-1] is the head */
    int32_t top;
    int32_t *ref;
    OrcSeq *seqs;
    int32_t nseqs, seqcap;
} OrcPool;

OrcPool *orc_pool_create(int kv_heads, int head_dim, int page_tokens,
                         int num_pages, uint64_t seed) {
    if (kv_heads <= 0 || head_dim <= 0 || page_tokens <= 0 || num_pages <= 0)
        return NULL;
    OrcPool *p = (OrcPool *)calloc(1, sizeof(OrcPool));
    p->kvh = kv_heads;
    p->dh = head_dim;
    p->P = page_tokens;
    p->num_pages = num_pages;
    p->page_elems = (int64_t)kv_heads * page_tokens * head_dim;
    p->k = (uint16_t *)malloc((size_t)num_pages * p->page_elems * 2);
    p->v = (uint16_t *)malloc((size_t)num_pages * p->page_elems * 2);
    /* free pages hold garbage until allocated; mark it recognisably */
    memset(p->k, 0xAB, (size_t)num_pages * p->page_elems * 2);
    memset(p->v, 0xCD, (size_t)num_pages * p->page_elems * 2);
    int32_t *perm = (int32_t *)malloc(sizeof(int32_t) * num_pages);
    orc_permutation(seed, num_pages, perm);
    p->stack = (int32_t *)malloc(sizeof(int32_t) * num_pages);
    for (int i = 0; i < num_pages; i++) p->stack[i] = perm[num_pages - 1 - i];
    p->top = num_pages;
    free(perm);
    p->ref = (int32_t *)calloc(num_pages, sizeof(int32_t));
    return p;
}

void orc_pool_destroy(OrcPool *p) {
    if (!p) return;
    for (int i = 0; i < p->nseqs; i++) {
        free(p->seqs[i].pages);
        free(p->seqs[i].kf);
        free(p->seqs[i].vf);
    }
    free(p->seqs);
    free(p->k);
    free(p->v);
    free(p->stack);
    free(p->ref);
    free(p);
}

static OrcSeq *get_seq(OrcPool *p, int id) {
    if (id < 0 || id >= p->nseqs || !p->seqs[id].active) return NULL;
    return &p->seqs[id];
}

int orc_seq_create(OrcPool *p) {
    for (int i = 0; i < p->nseqs; i++)
        if (!p->seqs[i].active) {
            p->seqs[i].active = 1;
            p->seqs[i].len = 0;
            p->seqs[i].npages = 0;
            p->seqs[i].f32len = 0;
            return i;
        }
    if (p->nseqs == p->seqcap) {
        p->seqcap = p->seqcap ? 2 * p->seqcap : 16;
        p->seqs = (OrcSeq *)realloc(p->seqs, sizeof(OrcSeq) * p->seqcap);
    }
    OrcSeq *s = &p->seqs[p->nseqs];
    memset(s, 0, sizeof(*s));
    s->active = 1;
    return p->nseqs++;
}

static void seq_push_page(OrcSeq *s, int32_t pid) {
    if (s->npages == s->cap) {
        s->cap = s->cap ? 2 * s->cap : 16;
        s->pages = (int32_t *)realloc(s->pages, sizeof(int32_t) * s->cap);
    }
    s->pages[s->npages++] = pid;
}

static int32_t pop_page(OrcPool *p) { return p->stack[--p->top]; }

static void unref_page(OrcPool *p, int32_t pid) {
    if (--p->ref[pid] == 0) p->stack[p->top++] = pid;
}

static uint16_t *kpage(OrcPool *p, int32_t pid) { return p->k + (int64_t)pid * p->page_elems; }
static uint16_t *vpage(OrcPool *p, int32_t pid) { return p->v + (int64_t)pid * p->page_elems; }

static int32_t alloc_zero_page(OrcPool *p) {
    int32_t pid = pop_page(p);
    p->ref[pid] = 1;
    memset(kpage(p, pid), 0, p->page_elems * 2);
    memset(vpage(p, pid), 0, p->page_elems * 2);
    return pid;
}

/* pages an append of n rows onto s would pop (COW tail + new pages) */
static int64_t pages_needed(OrcPool *p, OrcSeq *s, int64_t n) {
    if (n <= 0) return 0;
    int64_t P = p->P;
    int64_t have = s->npages;
    int64_t need = (s->len + n + P - 1) / P;
    int64_t cow = (s->len % P != 0 && p->ref[s->pages[have - 1]] > 1) ? 1 : 0;
    return cow + (need - have);
}

/* Copy-on-write of a shared tail page before rows land in it. */
static void cow_tail(OrcPool *p, OrcSeq *s) {
    if (s->len % p->P == 0) return;
    int32_t old = s->pages[s->npages - 1];
    if (p->ref[old] <= 1) return;
    int32_t pid = pop_page(p);
    p->ref[pid] = 1;
    memcpy(kpage(p, pid), kpage(p, old), p->page_elems * 2);
    memcpy(vpage(p, pid), vpage(p, old), p->page_elems * 2);
    p->ref[old]--; /* still > 0: it stays with its other owner */
    s->pages[s->npages - 1] = pid;
}

/* One position's K/V rows ([KVH, dh] each, given by a row pointer and a
 * kv-head stride) at the tail: PagePool.append + writePosition. */
static void append_row(OrcPool *p, OrcSeq *s, const uint16_t *k,
                       const uint16_t *v, int64_t head_stride) {
    int P = p->P, dh = p->dh;
    if (s->len % P == 0) seq_push_page(s, alloc_zero_page(p));
    int64_t slot = s->len % P;
    int32_t pid = s->pages[s->npages - 1];
    for (int h = 0; h < p->kvh; h++) {
        memcpy(kpage(p, pid) + ((int64_t)h * P + slot) * dh, k + h * head_stride, dh * 2);
        memcpy(vpage(p, pid) + ((int64_t)h * P + slot) * dh, v + h * head_stride, dh * 2);
    }
    s->len++;
}

/* Batched append: sequence seq_ids[i] takes n_new[i] rows, read from the
 * token-major k/v [sum(n_new), KVH, dh] in batch order.  Validates the whole
 * batch (ids, page supply) before mutating anything. */
int orc_append(OrcPool *p, int n, const int32_t *seq_ids, const int32_t *n_new,
               const uint16_t *k, const uint16_t *v) {
    int64_t need = 0;
    for (int i = 0; i < n; i++) {
        OrcSeq *s = get_seq(p, seq_ids[i]);
        if (!s || n_new[i] < 0) return ORC_ERR_BAD_SEQ;
        for (int j = 0; j < i; j++)
            if (seq_ids[j] == seq_ids[i]) return ORC_ERR_INVALID;
        need += pages_needed(p, s, n_new[i]);
    }
    if (need > p->top) return ORC_ERR_NO_PAGES;
    int64_t row = 0, rs = (int64_t)p->kvh * p->dh;
    for (int i = 0; i < n; i++) {
        OrcSeq *s = get_seq(p, seq_ids[i]);
        if (n_new[i] > 0) cow_tail(p, s);
        for (int r = 0; r < n_new[i]; r++, row++)
            append_row(p, s, k + row * rs, v + row * rs, p->dh);
    }
    return ORC_OK;
}

/* PagePool.seed: the sequence must be empty; K/V are [KVH, count, dh]. */
int orc_seed(OrcPool *p, int seq, const uint16_t *K, const uint16_t *V,
             int64_t count) {
    OrcSeq *s = get_seq(p, seq);
    if (!s || s->len != 0 || count < 0) return ORC_ERR_BAD_SEQ;
    if ((count + p->P - 1) / p->P > p->top) return ORC_ERR_NO_PAGES;
    for (int64_t t = 0; t < count; t++)
        append_row(p, s, K + t * p->dh, V + t * p->dh, count * p->dh);
    return ORC_OK;
}

/* PagePool.truncate(to:) for a batch: validate all, then apply in order. */
int orc_truncate(OrcPool *p, int n, const int32_t *seq_ids,
                 const int64_t *new_len) {
    for (int i = 0; i < n; i++) {
        OrcSeq *s = get_seq(p, seq_ids[i]);
        if (!s || new_len[i] < 0 || new_len[i] > s->len) return ORC_ERR_BAD_SEQ;
    }
    for (int i = 0; i < n; i++) {
        OrcSeq *s = get_seq(p, seq_ids[i]);
        s->len = new_len[i];
        if (s->f32len > s->len) s->f32len = s->len;
        int64_t need = (s->len + p->P - 1) / p->P;
        while (s->npages > need) unref_page(p, s->pages[--s->npages]);
    }
    return ORC_OK;
}

int orc_seq_release(OrcPool *p, int seq) {
    OrcSeq *s = get_seq(p, seq);
    if (!s) return ORC_ERR_BAD_SEQ;
    int64_t zero = 0;
    orc_truncate(p, 1, &seq, &zero);
    s->active = 0;
    return ORC_OK;
}

/* PagePool.clone: share every page, duplicate a partial tail.  Returns the
 * new sequence id, or -ORC_ERR_* on failure. */
int orc_clone(OrcPool *p, int src) {
    OrcSeq *s = get_seq(p, src);
    if (!s) return -ORC_ERR_BAD_SEQ;
    int partial = s->len % p->P != 0;
    if (partial && p->top < 1) return -ORC_ERR_NO_PAGES;
    int id = orc_seq_create(p);
    s = get_seq(p, src); /* realloc may have moved it */
    OrcSeq *c = get_seq(p, id);
    for (int32_t i = 0; i < s->npages; i++) {
        seq_push_page(c, s->pages[i]);
        p->ref[s->pages[i]]++;
    }
    c->len = s->len;
    if (partial) {
        int32_t old = c->pages[c->npages - 1];
        int32_t pid = pop_page(p);
        p->ref[pid] = 1;
        memcpy(kpage(p, pid), kpage(p, old), p->page_elems * 2);
        memcpy(vpage(p, pid), vpage(p, old), p->page_elems * 2);
        p->ref[old]--;
        c->pages[c->npages - 1] = pid;
    }
    return id;
}

/* compact(): [KVH, len, dh] K and V. */
int orc_compact(OrcPool *p, int seq, uint16_t *K, uint16_t *V) {
    OrcSeq *s = get_seq(p, seq);
    if (!s) return ORC_ERR_BAD_SEQ;
    int P = p->P, dh = p->dh;
    for (int h = 0; h < p->kvh; h++)
        for (int64_t t = 0; t < s->len; t++) {
            int32_t pid = s->pages[t / P];
            int64_t src = ((int64_t)h * P + t % P) * dh;
            int64_t dst = ((int64_t)h * s->len + t) * dh;
            memcpy(K + dst, kpage(p, pid) + src, dh * 2);
            memcpy(V + dst, vpage(p, pid) + src, dh * 2);
        }
    return ORC_OK;
}

/* tileAt(start, count, tileP) (PagedAttention.swift:151-161, copyWindow
 * :164-176): positions [start, start+count) into [KVH, tileP, dh] K and V,
 * rows count..tileP-1 zero (zeroPage).  The reference reads the window from
 * one page (its P is a multiple of tileP); this reads each row from its own
 * page, the same bytes when the window lies in one page. */
int orc_tile_at(OrcPool *p, int seq, int64_t start, int64_t count, int tile_p,
                uint16_t *K, uint16_t *V) {
    OrcSeq *s = get_seq(p, seq);
    if (!s) return ORC_ERR_BAD_SEQ;
    if (tile_p < 1 || count < 0 || count > tile_p) return ORC_ERR_INVALID;
    if (start < 0 || start + count > s->len) return ORC_ERR_BAD_SEQ;
    int P = p->P, dh = p->dh;
    memset(K, 0, (size_t)p->kvh * tile_p * dh * 2);
    memset(V, 0, (size_t)p->kvh * tile_p * dh * 2);
    for (int h = 0; h < p->kvh; h++)
        for (int64_t r = 0; r < count; r++) {
            int64_t t = start + r;
            int32_t pid = s->pages[t / P];
            int64_t src = ((int64_t)h * P + t % P) * dh;
            int64_t dst = ((int64_t)h * tile_p + r) * dh;
            memcpy(K + dst, kpage(p, pid) + src, dh * 2);
            memcpy(V + dst, vpage(p, pid) + src, dh * 2);
        }
    return ORC_OK;
}

/* fromCompact: a new sequence seeded from [KVH, length, dh]. */
int orc_from_compact(OrcPool *p, const uint16_t *K, const uint16_t *V,
                     int64_t length) {
    if ((length + p->P - 1) / p->P > p->top) return -ORC_ERR_NO_PAGES;
    int id = orc_seq_create(p);
    int rc = orc_seed(p, id, K, V, length);
    if (rc) return -rc;
    return id;
}

/* ---- state export (for bit-exact comparison) ---- */
int64_t orc_seq_length(OrcPool *p, int seq) {
    OrcSeq *s = get_seq(p, seq);
    return s ? s->len : -1;
}
int32_t orc_seq_pages(OrcPool *p, int seq, int32_t *out) {
    OrcSeq *s = get_seq(p, seq);
    if (!s) return -1;
    if (out) memcpy(out, s->pages, sizeof(int32_t) * s->npages);
    return s->npages;
}
/* free list in pop order (head first) */
int32_t orc_free_list(OrcPool *p, int32_t *out) {
    if (out)
        for (int32_t i = 0; i < p->top; i++) out[i] = p->stack[p->top - 1 - i];
    return p->top;
}
int32_t orc_page_ref(OrcPool *p, int32_t pid) { return p->ref[pid]; }
const uint16_t *orc_page_k(OrcPool *p, int32_t pid) { return kpage(p, pid); }
const uint16_t *orc_page_v(OrcPool *p, int32_t pid) { return vpage(p, pid); }

/* ------------------------------------------------------------------ */
/* attention                                                           */
/* ------------------------------------------------------------------ */

/* floats32()/growF32 (PagedAttention.swift:46-77): widen rows
 * [f32len, n) of every kv head from the fp16 pages into the fp32 mirror. */
static void grow_mirror(OrcPool *p, OrcSeq *s, int64_t n) {
    int KVH = p->kvh, dh = p->dh, P = p->P;
    const float *lut = f16_lut();
    if (n > s->mcap) {
        int64_t cap = s->mcap ? s->mcap : 64;
        while (cap < n) cap *= 2;
        float *kf = (float *)malloc(sizeof(float) * KVH * cap * dh);
        float *vf = (float *)malloc(sizeof(float) * KVH * cap * dh);
        for (int h = 0; h < KVH && s->f32len > 0; h++) {
            memcpy(kf + (int64_t)h * cap * dh, s->kf + (int64_t)h * s->mcap * dh,
                   sizeof(float) * s->f32len * dh);
            memcpy(vf + (int64_t)h * cap * dh, s->vf + (int64_t)h * s->mcap * dh,
                   sizeof(float) * s->f32len * dh);
        }
        free(s->kf);
        free(s->vf);
        s->kf = kf;
        s->vf = vf;
        s->mcap = cap;
    }
    for (int h = 0; h < KVH; h++)
        for (int64_t t = s->f32len; t < n; t++) {
            int32_t pid = s->pages[t / P];
            int64_t off = ((int64_t)h * P + t % P) * dh;
            const uint16_t *kr = kpage(p, pid) + off, *vr = vpage(p, pid) + off;
            float *kd = s->kf + ((int64_t)h * s->mcap + t) * dh;
            float *vd = s->vf + ((int64_t)h * s->mcap + t) * dh;
            for (int d = 0; d < dh; d++) {
                kd[d] = lut[kr[d]];
                vd[d] = lut[vr[d]];
            }
        }
    if (n > s->f32len) s->f32len = n;
}

/* K_j . q: fp32, eight interleaved partial sums combined pairwise (the
 * shape of a vectorised GEMV row; vDSP's own order is unspecified). */
static float dot_f32(const float *a, const float *b, int n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int d = 0;
    for (; d + 8 <= n; d += 8)
        for (int u = 0; u < 8; u++) acc[u] += a[d + u] * b[d + u];
    for (; d < n; d++) acc[d & 7] += a[d] * b[d];
    return ((acc[0] + acc[4]) + (acc[1] + acc[5])) + ((acc[2] + acc[6]) + (acc[3] + acc[7]));
}

/* hostFlashDecode over the first n keys of one sequence whose mirror is
 * already grown to >= n.  q: [KVH, G, dh] fp16.  out: [KVH*G*dh] fp32.
 * scores: >= n floats of scratch. */
static void flash_decode_one(OrcPool *p, OrcSeq *s, const uint16_t *q, int G,
                             float scale, int64_t n, float *out, float *scores) {
    int KVH = p->kvh, dh = p->dh;
    for (int64_t i = 0; i < (int64_t)KVH * G * dh; i++) out[i] = 0.0f;
    if (n == 0) return;
    float qf[1024];
    for (int kvh = 0; kvh < KVH; kvh++) {
        const float *kf = s->kf + (int64_t)kvh * s->mcap * dh;
        const float *vf = s->vf + (int64_t)kvh * s->mcap * dh;
        for (int g = 0; g < G; g++) {
            int h = kvh * G + g;
            for (int d = 0; d < dh; d++) qf[d] = orc_f16_to_f32(q[(int64_t)h * dh + d]);
            for (int64_t j = 0; j < n; j++) scores[j] = dot_f32(kf + j * dh, qf, dh);
            float mx = -INFINITY;
            for (int64_t j = 0; j < n; j++) {
                float sc = scores[j] * scale;
                scores[j] = sc;
                if (sc > mx) mx = sc;
            }
            float sum = 0.0f;
            for (int64_t j = 0; j < n; j++) {
                float e = expf(scores[j] - mx);
                scores[j] = e;
                sum += e;
            }
            /* o[d] = sum_j e_j V[j][d], accumulated in key order */
            float *o = out + (int64_t)h * dh;
            for (int64_t j = 0; j < n; j++) {
                const float e = scores[j];
                const float *vr = vf + j * dh;
                for (int d = 0; d < dh; d++) o[d] += e * vr[d];
            }
            float inv = 1.0f / sum;
            for (int d = 0; d < dh; d++) o[d] *= inv;
        }
    }
}

/* hostFlashDecode(q:pool:G:) for one sequence over its whole length. */
int orc_flash_decode(OrcPool *p, int seq, const uint16_t *q, int G, float scale,
                     float *out) {
    OrcSeq *s = get_seq(p, seq);
    if (!s || p->dh > 1024) return ORC_ERR_BAD_SEQ;
    grow_mirror(p, s, s->len);
    float *scores = (float *)malloc(sizeof(float) * (s->len + 1));
    flash_decode_one(p, s, q, G, scale, s->len, out, scores);
    free(scores);
    return ORC_OK;
}

/* Causal attend for a batch, the per-token route: sequence b's n_q query
 * rows are its LAST n_q positions; row r (position len - n_q + r) sees
 * keys [0, len - n_q + r].  q: [n, n_q, KVH*G, dh] fp16; out same shape,
 * fp32.  The (sequence, row) jobs are spread over n_threads host threads
 * (each job is independent; each runs the serial reference loop). */
typedef struct {
    OrcPool *p;
    int n, n_q, G;
    const int32_t *ids;
    const int32_t *rows; /* NULL: every row 0..n_q-1; else the n_rows chosen rows */
    int n_rows;
    const uint16_t *q;
    float scale;
    float *out;
    int64_t next; /* shared job counter */
    pthread_mutex_t mu;
    int64_t max_len;
} CausalJob;

static void *causal_worker(void *arg) {
    CausalJob *J = (CausalJob *)arg;
    OrcPool *p = J->p;
    int64_t H = (int64_t)p->kvh * J->G;
    float *work = (float *)malloc(sizeof(float) * (J->max_len + 1));
    for (;;) {
        pthread_mutex_lock(&J->mu);
        int64_t job = J->next++;
        pthread_mutex_unlock(&J->mu);
        if (job >= (int64_t)J->n * J->n_rows) break;
        int b = (int)(job / J->n_rows), i = (int)(job % J->n_rows);
        int r = J->rows ? J->rows[i] : i;
        OrcSeq *s = get_seq(p, J->ids[b]);
        int64_t nk = s->len - J->n_q + r + 1;
        int64_t row = (int64_t)b * J->n_rows + i;
        flash_decode_one(p, s, J->q + row * H * p->dh, J->G, J->scale, nk,
                         J->out + row * H * p->dh, work);
    }
    free(work);
    return NULL;
}

/* Grows the mirror of batch entry b to its sequence's length; an id that
 * appears earlier in the batch is left to that entry's job. */
static void *grow_worker(void *arg) {
    CausalJob *J = (CausalJob *)arg;
    for (;;) {
        pthread_mutex_lock(&J->mu);
        int64_t b = J->next++;
        pthread_mutex_unlock(&J->mu);
        if (b >= J->n) break;
        int first = 1;
        for (int64_t e = 0; e < b && first; e++) first = J->ids[e] != J->ids[b];
        if (!first) continue;
        OrcSeq *s = get_seq(J->p, J->ids[b]);
        grow_mirror(J->p, s, s->len);
    }
    return NULL;
}

static int attend_jobs(OrcPool *p, int n, const int32_t *seq_ids, int n_q,
                       const int32_t *rows, int n_rows, const uint16_t *q, int G,
                       float scale, float *out, int n_threads) {
    int64_t max_len = 1;
    if (p->dh > 1024) return ORC_ERR_INVALID;
    for (int b = 0; b < n; b++) {
        OrcSeq *s = get_seq(p, seq_ids[b]);
        if (!s || s->len < n_q || n_q < 1) return ORC_ERR_BAD_SEQ;
        if (s->len > max_len) max_len = s->len;
    }
    for (int i = 0; rows && i < n_rows; i++)
        if (rows[i] < 0 || rows[i] >= n_q) return ORC_ERR_INVALID;
    CausalJob J = {p, n, n_q, G, seq_ids, rows, n_rows, q, scale, out, 0,
                   PTHREAD_MUTEX_INITIALIZER, max_len};
    if (n_threads < 1) n_threads = 1;
    if (n_threads == 1) {
        /* the mirror grows once per sequence before the rows fan out */
        for (int b = 0; b < n; b++) {
            OrcSeq *s = get_seq(p, seq_ids[b]);
            grow_mirror(p, s, s->len);
        }
        causal_worker(&J);
        return ORC_OK;
    }
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * n_threads);
    /* the same growth, one sequence per job over the threads, then the rows */
    for (int i = 0; i < n_threads; i++) pthread_create(&th[i], NULL, grow_worker, &J);
    for (int i = 0; i < n_threads; i++) pthread_join(th[i], NULL);
    J.next = 0;
    for (int i = 0; i < n_threads; i++) pthread_create(&th[i], NULL, causal_worker, &J);
    for (int i = 0; i < n_threads; i++) pthread_join(th[i], NULL);
    free(th);
    return ORC_OK;
}

int orc_attend_causal(OrcPool *p, int n, const int32_t *seq_ids, int n_q,
                      const uint16_t *q, int G, float scale, float *out,
                      int n_threads) {
    return attend_jobs(p, n, seq_ids, n_q, NULL, n_q, q, G, scale, out, n_threads);
}

/* The same causal attend for chosen query rows only (test helper, for
 * full-size chunks whose every row would take the CPU too long): for each
 * sequence b and each i < n_rows, query row rows[i] of b's last n_q
 * positions sees keys [0, len_b - n_q + rows[i]].  q holds those rows only,
 * [n, n_rows, KVH*G, dh] fp16; out the same shape, fp32. */
int orc_attend_rows(OrcPool *p, int n, const int32_t *seq_ids, int n_q,
                    const int32_t *rows, int n_rows, const uint16_t *q, int G,
                    float scale, float *out, int n_threads) {
    if (!rows || n_rows < 1) return ORC_ERR_INVALID;
    return attend_jobs(p, n, seq_ids, n_q, rows, n_rows, q, G, scale, out, n_threads);
}

/* Frees a sequence's fp32 mirror (test helper: bounds the host memory of
 * full-size checks over many long sequences); the next attend widens its
 * rows again, so results do not change. */
int orc_seq_drop_mirror(OrcPool *p, int seq) {
    OrcSeq *s = get_seq(p, seq);
    if (!s) return ORC_ERR_BAD_SEQ;
    free(s->kf);
    free(s->vf);
    s->kf = s->vf = NULL;
    s->mcap = s->f32len = 0;
    return ORC_OK;
}

/* ------------------------------------------------------------------ */
/* GDN rollback after an accepted speculative prefix                   */
/* ------------------------------------------------------------------ */

/* MtpRollback.stateAfter (LLM/src/CoreML/MtpRollback.swift:20-60) for a
 * batch of n items (sequence x GDN layer), each with its own accepted
 * prefix m[i] in 1..C:
 *   S_m[h] = exp(gcum[h,m-1]) * S0[h]
 *            + sum_{t<m} exp(gcum[h,m-1] - gcum[h,t]) * outer(k[h,t], delta[h,t])
 * in the reference's order: out = eM * s0, then for t ascending
 * out[i][j] += (w_t * k[t][i]) * delta[t][j].
 * s0/out [n,H,DK,DV], delta [n,H,C,DV], k [n,H,C,DK], gcum [n,H,C]; fp32. */
void orc_mtp_rollback(int n, const int32_t *m, int H, int DK, int DV, int C,
                      const float *s0, const float *delta, const float *k,
                      const float *gcum, float *out) {
    for (int it = 0; it < n; it++)
        for (int h = 0; h < H; h++) {
            const int64_t hs = (int64_t)it * H + h;
            const float *g = gcum + hs * C;
            const float *kk = k + hs * C * DK;
            const float *dd = delta + hs * C * DV;
            const float *s = s0 + hs * DK * DV;
            float *o = out + hs * DK * DV;
            const int mm = m[it];
            const float gLast = g[mm - 1];
            const float eM = expf(gLast);
            for (int i = 0; i < DK * DV; i++) o[i] = eM * s[i];
            for (int t = 0; t < mm; t++) {
                const float w = expf(gLast - g[t]);
                for (int i = 0; i < DK; i++) {
                    const float wk = w * kk[t * DK + i];
                    for (int j = 0; j < DV; j++) o[i * DV + j] += wk * dd[t * DV + j];
                }
            }
        }
}

/* Engine.convFromProj (LLM/src/CoreML/Engine.swift:2719-2740): conv state
 * [CD, taps] after m committed tokens; tap t holds position m - taps + t,
 * taken from this chunk's conv-projection rows proj [C, CD] when >= 0 and
 * from the pre-verify tail pre [CD, taps] (oldest..newest) otherwise.
 * Batched over n items; fp32 in and out (the engine then stores fp16). */
void orc_conv_rollback(int n, const int32_t *m, int CD, int taps, int C,
                       const float *proj, const float *pre, float *out) {
    for (int it = 0; it < n; it++) {
        const float *pr = proj + (int64_t)it * C * CD;
        const float *pc = pre + (int64_t)it * CD * taps;
        float *o = out + (int64_t)it * CD * taps;
        for (int t = 0; t < taps; t++) {
            const int pos = m[it] - taps + t;
            for (int c = 0; c < CD; c++)
                o[c * taps + t] = pos >= 0 ? pr[pos * CD + c] : pc[c * taps + (m[it] + t)];
        }
    }
}

/* ------------------------------------------------------------------------
 * Producer of a Qwen3.5 full-attention step (SIMD/Attention.swift:72-139),
 * restated for gkv_attn_step's parity tests.  Every product and sum is
 * rounded on its own, as the Swift source writes them (no contraction into
 * fused multiply-adds).
 */
#pragma GCC push_options
#pragma GCC optimize("fp-contract=off")

/* Kern.rmsnormRows (SIMD/Kernels.swift:26-37): each row of d floats becomes
 * x * (1 / sqrt(sum(x^2) / d + eps)) * w, in place. */
void orc_rmsnorm_rows(float *x, int d, int rows, const float *w, float eps) {
    for (int r = 0; r < rows; ++r) {
        float *p = x + (size_t)r * d;
        float ss = 0.f;
        for (int i = 0; i < d; ++i) ss += p[i] * p[i];
        const float s = 1.f / sqrtf(ss / (float)d + eps);
        for (int i = 0; i < d; ++i) p[i] = p[i] * s * w[i];
    }
}

/* Kern.ropeNeox (SIMD/Kernels.swift:66-84) with the angle's cos / sin given
 * per pair: for every head, pair (i, i + n_rot/2), i < n_rot/2, becomes
 * (a c - b s, a s + b c); elements past n_rot are untouched. */
void orc_rope_neox(float *x, int head_dim, int n_head, int n_rot, const float *cs, const float *sn) {
    const int half = n_rot / 2;
    for (int h = 0; h < n_head; ++h) {
        float *p = x + (size_t)h * head_dim;
        for (int i = 0; i < half; ++i) {
            const float a = p[i], b = p[i + half];
            p[i] = a * cs[i] - b * sn[i];
            p[i + half] = a * sn[i] + b * cs[i];
        }
    }
}

/* The angle of ropeNeox (Kernels.swift:74-76): freq = base^(-2i/n_rot),
 * angle = pos * freq, in fp32; tables [n, n_rot/2]. */
void orc_rope_table(int n_rot, float base, int n, const int64_t *pos, float *cs, float *sn) {
    const int half = n_rot / 2;
    for (int t = 0; t < n; ++t)
        for (int i = 0; i < half; ++i) {
            const float freq = powf(base, -2.f * (float)i / (float)n_rot);
            const float ang = (float)pos[t] * freq;
            cs[(size_t)t * half + i] = cosf(ang);
            sn[(size_t)t * half + i] = sinf(ang);
        }
}

/* attnOut[i] *= sigmoidf(gate[i]) (Attention.swift:133-135, sigmoidf =
 * 1 / (1 + expf(-x)), Kernels.swift:6). */
void orc_gate(float *x, const float *gate, int64_t n) {
    for (int64_t i = 0; i < n; ++i) x[i] *= 1.f / (1.f + expf(-gate[i]));
}

#pragma GCC pop_options
