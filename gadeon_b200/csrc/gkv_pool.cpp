// gkv_pool.cpp -- host side of libgadeonkv.so: the C ABI of include/gadeon_kv.h.
//
// The host owns the allocation decisions (free list, reference counts,
// lengths, block tables); the device owns the page bytes and a copy of the
// block tables that the kernels read.  Every mutating call validates the
// whole batch first, then updates the host state and enqueues the matching
// device work in stream order through a small descriptor upload.
//
// Allocation policy (the reference has no free list -- PagePool pages are
// ARC objects, LLM/src/CoreML/PagedAttention.swift:25-26 -- so this is the
// one explicit model, mirrored bit-for-bit by the CPU oracle):
//   * initial pop order = splitmix64 Fisher-Yates permutation of the page ids;
//   * pops happen in batch order, per sequence: copy-on-write of a shared
//     tail page first, then one fresh page per page boundary crossed;
//   * fresh pages are zero-filled (PagePool.zeroPage, :278-286);
//   * truncate drops table entries last-first (:185-188) and pushes a page
//     back when its reference count reaches zero (LIFO: next pop reuses it).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <initializer_list>
#include <string>
#include <vector>

#include "gadeon_kv.h"
#include "gkv_kernels.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char *what) {
    return fail(GKV_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

#define GKV_CUDA(call, what)                          \
    do {                                              \
        cudaError_t e_ = (call);                      \
        if (e_ != cudaSuccess) return cuda_fail(e_, what); \
    } while (0)

uint64_t splitmix64(uint64_t *s) {
    uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

bool is_pow2(int64_t x) { return x > 0 && (x & (x - 1)) == 0; }

// Restores the caller's current device on scope exit.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static const EncodeTiledFn fn = [] {  // looked up once, thread-safe
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return reinterpret_cast<EncodeTiledFn>(p);
        return static_cast<EncodeTiledFn>(nullptr);
    }();
    return fn;
}

// Pinned host slots + matching device slots for per-call descriptors.  A
// slot is reused only after the event recorded behind its last use fired.
struct Staging {
    static constexpr int kSlots = 64;
    size_t slot_bytes = 0;
    uint8_t *h = nullptr;
    uint8_t *d = nullptr;
    cudaEvent_t ev[kSlots] = {};
    bool used[kSlots] = {};
    int next = 0;

    void release() {
        for (int i = 0; i < kSlots; ++i)
            if (ev[i]) {
                cudaEventSynchronize(ev[i]);
                cudaEventDestroy(ev[i]);
                ev[i] = nullptr;
            }
        if (h) cudaFreeHost(h);
        if (d) cudaFree(d);
        h = d = nullptr;
        slot_bytes = 0;
    }

    // Returns the slot index, or -1 with the CUDA error in *err.
    int acquire(size_t bytes, cudaError_t *err) {
        *err = cudaSuccess;
        if (bytes > slot_bytes) {
            release();
            size_t sb = 64 * 1024;
            while (sb < bytes) sb *= 2;
            if ((*err = cudaMallocHost(&h, sb * kSlots)) != cudaSuccess) return -1;
            if ((*err = cudaMalloc(&d, sb * kSlots)) != cudaSuccess) return -1;
            for (int i = 0; i < kSlots; ++i) {
                if ((*err = cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming)) != cudaSuccess)
                    return -1;
                used[i] = false;
            }
            slot_bytes = sb;
        }
        const int s = next;
        next = (next + 1) % kSlots;
        if (used[s] && (*err = cudaEventSynchronize(ev[s])) != cudaSuccess) return -1;
        return s;
    }
    uint8_t *host(int s) { return h + (size_t)s * slot_bytes; }
    uint8_t *dev(int s) { return d + (size_t)s * slot_bytes; }
    cudaError_t upload(int s, size_t bytes, cudaStream_t st) {
        return cudaMemcpyAsync(dev(s), host(s), bytes, cudaMemcpyHostToDevice, st);
    }
    cudaError_t done(int s, cudaStream_t st) {
        used[s] = true;
        return cudaEventRecord(ev[s], st);
    }
};

struct Seq {
    bool active = false;
    int64_t len = 0;
    std::vector<int32_t> pages;
};

}  // namespace

struct gkv_pool {
    gkv_pool_config cfg{};
    int sm_count = 0;
    int tile_keys = 0;
    size_t page_elems = 0;  // KVH * P * dh halves
    uint16_t *d_k = nullptr, *d_v = nullptr;
    int32_t *d_table = nullptr;
    int32_t *d_status = nullptr;
    float *d_partials = nullptr;
    int32_t *d_counters = nullptr;
    uint16_t *d_prod = nullptr;  // [2][max_seqs * KVH * dh] fp16 K/V rows of gkv_attn_step's unfused route
    uint8_t *h_bounce = nullptr;  // page-locked copies of a call's pageable host buffers
    size_t bounce_bytes = 0;
    cudaEvent_t bounce_ev = nullptr;  // recorded behind the last launch that used h_bounce
    bool bounce_pending = false;
    CUtensorMap tmk{}, tmv{};  // chunk kernel: boxes of min(P, 64) rows
    CUtensorMap tak{}, tav{};  // attend kernel: boxes of min(P, tile_keys) rows
    std::vector<int32_t> stack;  // free list; back() is the head
    std::vector<int32_t> ref;
    std::vector<Seq> seqs;
    Staging staging;

    Seq *seq(int32_t id) {
        if (id < 0 || id >= (int32_t)seqs.size() || !seqs[id].active) return nullptr;
        return &seqs[id];
    }
    const Seq *seq(int32_t id) const {
        if (id < 0 || id >= (int32_t)seqs.size() || !seqs[id].active) return nullptr;
        return &seqs[id];
    }
    int32_t pop() {
        const int32_t pid = stack.back();
        stack.pop_back();
        ref[pid] = 1;
        return pid;
    }
    void unref(int32_t pid) {
        if (--ref[pid] == 0) stack.push_back(pid);
    }
    int64_t pages_for(int64_t len) const { return (len + cfg.page_tokens - 1) / cfg.page_tokens; }
    // Pages an append of n rows onto s pops (shared-tail copy + new pages).
    int64_t pages_needed(const Seq &s, int64_t n) const {
        if (n <= 0) return 0;
        const int64_t P = cfg.page_tokens;
        const int64_t cow = (s.len % P != 0 && ref[s.pages.back()] > 1) ? 1 : 0;
        return cow + pages_for(s.len + n) - (int64_t)s.pages.size();
    }
    int32_t new_seq_id() {
        for (size_t i = 0; i < seqs.size(); ++i)
            if (!seqs[i].active) return (int32_t)i;
        if ((int32_t)seqs.size() >= cfg.max_seqs) return -1;
        seqs.emplace_back();
        return (int32_t)seqs.size() - 1;
    }
};

namespace {

int check_batch(const gkv_pool *pool, int32_t n, const int32_t *ids) {
    if (n < 0 || (n > 0 && !ids)) return fail(GKV_ERR_INVALID, "bad batch (n=%d)", n);
    std::vector<char> seen(pool->seqs.size(), 0);
    for (int32_t i = 0; i < n; ++i) {
        if (!pool->seq(ids[i])) return fail(GKV_ERR_BAD_SEQ, "unknown sequence id %d", ids[i]);
        if (seen[ids[i]]++) return fail(GKV_ERR_INVALID, "sequence %d twice in one batch", ids[i]);
    }
    return GKV_OK;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Caller buffers a kernel reads or writes with plain loads and stores: device
// memory of the pool's GPU, managed memory, or page-locked host memory mapped
// at the same address (zero-copy: the kernel moves those bytes over the host
// link itself).  Pageable host memory would fault the kernel: refused.
int check_buffers(const gkv_pool *pool, std::initializer_list<std::pair<const void *, const char *>> bufs) {
    for (const auto &b : bufs) {
        const int rc = gkv::check_reachable(b.first, pool->cfg.device, true, b.second);
        if (rc) return rc;
    }
    return GKV_OK;
}

// Pageable host buffers (plain host arrays: malloc, a Swift [Float], numpy).
// A kernel cannot reach them, so a call given one copies it, on the CPU, into
// a page-locked bounce buffer the pool owns, which the kernels read and write
// in place over the host link as they do a caller's own page-locked buffers.
// After the launch the call records an event; when it has pageable outputs it
// waits for that event and copies them out of the bounce buffer, so it
// returns with its outputs in place.  Pageable inputs may be reused as soon
// as the call returns.  The next call that stages waits for the event before
// it writes the bounce buffer again, and the buffer grows (cudaHostAlloc)
// when a call needs more than it holds.
bool is_pageable(const void *ptr) {
    if (!ptr) return false;
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, ptr) != cudaSuccess) {
        cudaGetLastError();
        return false;  // check_buffers reports it
    }
    return a.type == cudaMemoryTypeUnregistered;
}

class HostStage {
public:
    explicit HostStage(gkv_pool *pool) : pool_(pool) {}
    // Registers a caller buffer of `bytes`; when it is pageable host memory,
    // reserve() points *ptr at the pool's bounce buffer.
    void in(const void **ptr, size_t bytes) { add(const_cast<void **>(ptr), bytes, false); }
    void out(void **ptr, size_t bytes) { add(ptr, bytes, true); }
    // Waits until the previous staged launch is done with the bounce buffer,
    // makes room (the one step that may allocate: call it with the pool's
    // device current and before any bookkeeping changes) and re-points the
    // registered pageable buffers.
    int reserve() {
        if (items_.empty()) return GKV_OK;
        if (pool_->bounce_pending) {
            GKV_CUDA(cudaEventSynchronize(pool_->bounce_ev), "waiting for the previous staged call");
            pool_->bounce_pending = false;
        }
        size_t total = 0;
        for (Item &it : items_) {
            it.off = total;
            total += (it.bytes + 255) & ~size_t(255);
        }
        if (total > pool_->bounce_bytes) {
            if (pool_->h_bounce) cudaFreeHost(pool_->h_bounce);
            pool_->h_bounce = nullptr;
            pool_->bounce_bytes = 0;
            size_t cap = size_t(1) << 20;
            while (cap < total) cap *= 2;
            void *h = nullptr;
            const cudaError_t e = cudaHostAlloc(&h, cap, cudaHostAllocDefault);
            if (e != cudaSuccess) return cuda_fail(e, "bounce buffer for pageable host buffers");
            pool_->h_bounce = static_cast<uint8_t *>(h);
            pool_->bounce_bytes = cap;
        }
        if (!pool_->bounce_ev)
            GKV_CUDA(cudaEventCreateWithFlags(&pool_->bounce_ev, cudaEventDisableTiming), "bounce event");
        for (Item &it : items_) *it.slot = pool_->h_bounce + it.off;
        return GKV_OK;
    }
    // The pageable inputs into the bounce buffer (before the launch).
    void copy_in() const {
        for (const Item &it : items_)
            if (!it.out) std::memcpy(*it.slot, it.host, it.bytes);
    }
    // After the launches: guards the bounce buffer with an event and, when
    // there are pageable outputs, waits for them and copies them out.
    int finish(cudaStream_t st) const {
        if (items_.empty()) return GKV_OK;
        GKV_CUDA(cudaEventRecord(pool_->bounce_ev, st), "bounce event record");
        pool_->bounce_pending = true;
        bool outs = false;
        for (const Item &it : items_) outs |= it.out;
        if (!outs) return GKV_OK;
        GKV_CUDA(cudaEventSynchronize(pool_->bounce_ev), "waiting for the staged outputs");
        pool_->bounce_pending = false;
        for (const Item &it : items_)
            if (it.out) std::memcpy(it.host, *it.slot, it.bytes);
        return GKV_OK;
    }

private:
    struct Item {
        void **slot;
        void *host;
        size_t bytes;
        bool out;
        size_t off;
    };
    void add(void **ptr, size_t bytes, bool out) {
        if (bytes > 0 && is_pageable(*ptr)) items_.push_back({ptr, *ptr, bytes, out, 0});
    }
    gkv_pool *pool_;
    std::vector<Item> items_;
};

// Host half of an append/seed: validates, mutates the bookkeeping, and fills
// the descriptor (entries + touched pages).  Nothing is mutated on failure.
int plan_append(gkv_pool *pool, int32_t n, const int32_t *ids, const int32_t *n_new,
                std::vector<gkv::AppendEntry> &entries, std::vector<gkv::TouchedPage> &pages) {
    const int64_t P = pool->cfg.page_tokens;
    int64_t need = 0;
    for (int32_t i = 0; i < n; ++i) {
        if (n_new[i] < 0) return fail(GKV_ERR_INVALID, "n_new[%d] = %d", i, n_new[i]);
        const Seq &s = *pool->seq(ids[i]);
        if (pool->pages_for(s.len + n_new[i]) > pool->cfg.max_pages_per_seq)
            return fail(GKV_ERR_CAPACITY, "sequence %d would exceed %d pages", ids[i],
                        pool->cfg.max_pages_per_seq);
        if (s.len + n_new[i] > INT32_MAX)
            return fail(GKV_ERR_CAPACITY, "sequence %d length overflow", ids[i]);
        need += pool->pages_needed(s, n_new[i]);
    }
    if (need > (int64_t)pool->stack.size())
        return fail(GKV_ERR_NO_PAGES, "append needs %lld pages, %zu free", (long long)need,
                    pool->stack.size());
    int32_t row0 = 0;
    entries.clear();
    pages.clear();
    for (int32_t i = 0; i < n; ++i) {
        Seq &s = *pool->seq(ids[i]);
        entries.push_back({ids[i], (int32_t)s.len, n_new[i], row0});
        row0 += n_new[i];
        if (n_new[i] == 0) continue;
        if (s.len % P != 0) {
            const int32_t tail = s.pages.back();
            const int32_t pidx = (int32_t)s.pages.size() - 1;
            if (pool->ref[tail] > 1) {  // copy-on-write of a shared tail
                const int32_t pid = pool->pop();
                pool->ref[tail]--;
                s.pages.back() = pid;
                pages.push_back({i, pidx, pid, tail});
            } else {
                pages.push_back({i, pidx, tail, gkv::PAGE_EXISTING});
            }
        }
        const int64_t want = pool->pages_for(s.len + n_new[i]);
        while ((int64_t)s.pages.size() < want) {
            const int32_t pid = pool->pop();
            pages.push_back({i, (int32_t)s.pages.size(), pid, gkv::PAGE_NEW});
            s.pages.push_back(pid);
        }
        s.len += n_new[i];
    }
    return GKV_OK;
}

// The fused append's pages per sequence, in position order: true when every
// sequence's new rows land on one or two pages none of which is a shared
// (copy-on-write) tail -- the rows can then ride in the attend kernel.
bool fused_tails(const std::vector<gkv::TouchedPage> &pages, int32_t n_seqs, std::vector<gkv::FusedTail> &tails) {
    tails.assign(n_seqs, gkv::FusedTail{{-1, -1}, {-1, -1}, {0, 0}, {0, 0}});
    std::vector<int> cnt(n_seqs, 0);
    for (const gkv::TouchedPage &tp : pages) {
        if (tp.src_pid >= 0) return false;
        int &c = cnt[tp.entry];
        if (c == 2) return false;
        tails[tp.entry].pid[c] = tp.pid;
        tails[tp.entry].pidx[c] = tp.pidx;
        tails[tp.entry].fresh[c] = tp.src_pid == gkv::PAGE_NEW ? 1 : 0;
        ++c;
    }
    for (int32_t i = 0; i < n_seqs; ++i)
        if (cnt[i] == 0) return false;
    return true;
}

// True when an entry writes in place into a page that an earlier entry of
// the same batch copies (two sequences sharing one partial tail page, both
// appending: the first takes a copy, the last writes the original).  One CTA
// per touched page would race the copy's reads against those writes.
bool copy_source_written(const std::vector<gkv::TouchedPage> &pages) {
    std::vector<int32_t> srcs;
    for (const gkv::TouchedPage &tp : pages)
        if (tp.src_pid >= 0) srcs.push_back(tp.src_pid);
    if (srcs.empty()) return false;
    std::sort(srcs.begin(), srcs.end());
    for (const gkv::TouchedPage &tp : pages)
        if (tp.src_pid < 0 && std::binary_search(srcs.begin(), srcs.end(), tp.pid)) return true;
    return false;
}

// Uploads entries+pages and launches the append kernel.
int enqueue_append(gkv_pool *pool, const std::vector<gkv::AppendEntry> &entries,
                   const std::vector<gkv::TouchedPage> &pages, const void *k, const void *v,
                   int head_major, cudaStream_t st) {
    if (pages.empty()) return GKV_OK;
    if (copy_source_written(pages)) {
        // the copies (and their entries' rows on the copies) first, the
        // in-place writes after them in stream order; every touched page is
        // independent of the others, so the split changes nothing else
        std::vector<gkv::TouchedPage> copies, rest;
        for (const gkv::TouchedPage &tp : pages) (tp.src_pid >= 0 ? copies : rest).push_back(tp);
        const int rc = enqueue_append(pool, entries, copies, k, v, head_major, st);
        return rc ? rc : enqueue_append(pool, entries, rest, k, v, head_major, st);
    }
    const size_t eb = entries.size() * sizeof(gkv::AppendEntry);
    const size_t pb = pages.size() * sizeof(gkv::TouchedPage);
    // small appends (decode rows, MTP drafts) carry the descriptor in the
    // kernel's parameter block; large ones (prefill chunks) upload it
    const bool inl = entries.size() <= (size_t)gkv::kAppendInlineEntries &&
                     pages.size() <= (size_t)gkv::kAppendInlinePages;
    gkv::AppendInline desc;
    gkv::AppendParams p{};
    int slot = -1;
    if (inl) {
        memcpy(desc.entries, entries.data(), eb);
        memcpy(desc.pages, pages.data(), pb);
    } else {
        cudaError_t err;
        slot = pool->staging.acquire(eb + pb, &err);
        if (slot < 0) return cuda_fail(err, "descriptor staging");
        memcpy(pool->staging.host(slot), entries.data(), eb);
        memcpy(pool->staging.host(slot) + eb, pages.data(), pb);
        GKV_CUDA(pool->staging.upload(slot, eb + pb, st), "descriptor upload");
        p.entries = reinterpret_cast<const gkv::AppendEntry *>(pool->staging.dev(slot));
        p.pages = reinterpret_cast<const gkv::TouchedPage *>(pool->staging.dev(slot) + eb);
    }
    p.n_pages = (int32_t)pages.size();
    p.k_src = static_cast<const uint16_t *>(k);
    p.v_src = static_cast<const uint16_t *>(v);
    p.head_major = head_major;
    p.k_pool = pool->d_k;
    p.v_pool = pool->d_v;
    p.table = pool->d_table;
    p.table_stride = pool->cfg.max_pages_per_seq;
    p.kvh = pool->cfg.kv_heads;
    p.dh = pool->cfg.head_dim;
    p.P = pool->cfg.page_tokens;
    GKV_CUDA(gkv::launch_append(p, st, inl ? &desc : nullptr), "append kernel launch");
    if (!inl) GKV_CUDA(pool->staging.done(slot, st), "descriptor event");
    return GKV_OK;
}

// Validation shared by gkv_attend / gkv_append_attend (after the append).
int check_attend(const gkv_pool *pool, int32_t n, const int32_t *ids, int32_t n_q, int32_t group,
                 const void *q, const void *out) {
    if (n_q < 1 || group < 1) return fail(GKV_ERR_INVALID, "n_q=%d group=%d", n_q, group);
    if ((int64_t)n_q * group > 16 &&
        !gkv::chunk_supported(pool->cfg.head_dim, pool->cfg.page_tokens, group))
        return fail(GKV_ERR_UNSUPPORTED,
                    "n_q*group = %lld rows per kv head needs the chunk kernel (head_dim <= 256, "
                    "page_tokens >= 8)",
                    (long long)n_q * group);
    if (n > 0 && (!q || !out)) return fail(GKV_ERR_INVALID, "null q/out");
    if (!aligned16(q) || !aligned16(out)) return fail(GKV_ERR_INVALID, "q/out not 16-byte aligned");
    for (int32_t i = 0; i < n; ++i)
        if (pool->seq(ids[i])->len < n_q)
            return fail(GKV_ERR_BAD_SEQ, "sequence %d has %lld < n_q=%d positions", ids[i],
                        (long long)pool->seq(ids[i])->len, n_q);
    return GKV_OK;
}

// tails != null: single-token decode with the append fused into the attend
// kernel (k_new / v_new hold each sequence's new row).
int enqueue_attend(gkv_pool *pool, int32_t n, const int32_t *ids, int32_t n_q, int32_t group,
                   const void *q, void *out, float scale, uint32_t flags, cudaStream_t st,
                   const gkv::FusedTail *tails = nullptr, const void *k_new = nullptr,
                   const void *v_new = nullptr, const gkv::ProducerArgs *prod = nullptr) {
    const int32_t head_major = (flags & GKV_ATTEND_HEAD_MAJOR) ? 1 : 0;
    const int32_t out_f16 = (flags & GKV_ATTEND_OUT_F16) ? 1 : 0;
    const int32_t p_f16 = (flags & GKV_ATTEND_P_F16) ? 1 : 0;
    if (n == 0) return GKV_OK;
    const int TK = pool->tile_keys, KVH = pool->cfg.kv_heads;
    const bool chunk = (int64_t)n_q * group > 16;  // many rows per kv head: tcgen05 chunk kernel
    // Up to kInlineSeqs sequences: the descriptor rides in the kernel's
    // parameter block (no upload between launches).
    const bool inl = !chunk && n <= gkv::kInlineSeqs;
    gkv::InlineDesc desc;
    int slot = -1;
    size_t ebytes = 0;
    size_t bytes = 0;
    gkv::AttendEntry *ent = desc.entries;
    if (!inl) {
        cudaError_t err;
        ebytes = ((size_t)n * sizeof(gkv::AttendEntry) + 255) & ~size_t(255);
        bytes = tails ? ebytes + (size_t)n * sizeof(gkv::FusedTail) : (size_t)n * sizeof(gkv::AttendEntry);
        slot = pool->staging.acquire(bytes, &err);
        if (slot < 0) return cuda_fail(err, "descriptor staging");
        ent = reinterpret_cast<gkv::AttendEntry *>(pool->staging.host(slot));
        if (tails) memcpy(pool->staging.host(slot) + ebytes, tails, (size_t)n * sizeof(gkv::FusedTail));
    } else if (tails) {
        memcpy(desc.tails, tails, (size_t)n * sizeof(gkv::FusedTail));
    }
    int64_t units = 0;
    for (int32_t i = 0; i < n; ++i) {
        const Seq &s = *pool->seq(ids[i]);
        const int32_t ntiles = (int32_t)((s.len + TK - 1) / TK);
        ent[i] = {ids[i], (int32_t)s.len, (int32_t)units, ntiles};
        units += (int64_t)KVH * ntiles;
    }
    if (!chunk && units > INT32_MAX) return fail(GKV_ERR_CAPACITY, "too many key tiles in one call");
    // the pinned slot is complete: the copy reads it when the stream gets there
    if (!inl) GKV_CUDA(pool->staging.upload(slot, bytes, st), "descriptor upload");
    if (chunk) {
        gkv::ChunkParams c{};
        c.entries = reinterpret_cast<const gkv::AttendEntry *>(pool->staging.dev(slot));
        c.n_seqs = n;
        c.table = pool->d_table;
        c.table_stride = pool->cfg.max_pages_per_seq;
        c.q = static_cast<const uint16_t *>(q);
        c.out = out;
        c.head_major = head_major;
        c.out_f16 = out_f16;
        c.p_f16 = p_f16;
        c.status = pool->d_status;
        c.n_q = n_q;
        c.G = group;
        c.kvh = KVH;
        c.P = pool->cfg.page_tokens;
        c.num_pages = pool->cfg.num_pages;
        c.qtok = 128 / group;
        c.n_qblocks = (n_q + c.qtok - 1) / c.qtok;
        c.scale_log2 = scale * 1.4426950408889634f;
        GKV_CUDA(gkv::launch_chunk(c, &pool->tmk, &pool->tmv, pool->cfg.head_dim, st),
                 "chunk kernel launch");
        GKV_CUDA(pool->staging.done(slot, st), "descriptor event");
        return GKV_OK;
    }
    gkv::AttendParams p{};
    if (!inl) {
        p.entries = reinterpret_cast<const gkv::AttendEntry *>(pool->staging.dev(slot));
        if (tails) p.tails = reinterpret_cast<const gkv::FusedTail *>(pool->staging.dev(slot) + ebytes);
    }
    if (tails) {
        p.fused = 1;
        p.k_new = static_cast<const uint16_t *>(k_new);
        p.v_new = static_cast<const uint16_t *>(v_new);
        p.k_pool_w = pool->d_k;
        p.v_pool_w = pool->d_v;
        p.table_w = pool->d_table;
    }
    p.n_seqs = n;
    p.total_units = (int32_t)units;
    p.table = pool->d_table;
    p.table_stride = pool->cfg.max_pages_per_seq;
    p.k_pool = pool->d_k;
    p.v_pool = pool->d_v;
    p.q = static_cast<const uint16_t *>(q);
    p.out = out;
    p.head_major = head_major;
    p.out_f16 = out_f16;
    p.partials = pool->d_partials;
    p.counters = pool->d_counters;
    p.status = pool->d_status;
    p.n_q = n_q;
    p.G = group;
    p.kvh = KVH;
    p.P = pool->cfg.page_tokens;
    p.num_pages = pool->cfg.num_pages;
    p.scale_log2 = scale * 1.4426950408889634f;
    if (prod) p.prod = *prod;
    const int grid = gkv::attend_grid(pool->cfg.head_dim, p.P, (int)units, pool->sm_count);
    GKV_CUDA(gkv::launch_attend(p, &pool->tak, &pool->tav, pool->cfg.head_dim, grid, st, inl ? &desc : nullptr),
             "attend kernel launch");
    if (!inl) GKV_CUDA(pool->staging.done(slot, st), "descriptor event");
    return GKV_OK;
}

void free_device(gkv_pool *p) {
    p->staging.release();
    cudaFree(p->d_k);
    cudaFree(p->d_v);
    cudaFree(p->d_table);
    cudaFree(p->d_status);
    cudaFree(p->d_partials);
    cudaFree(p->d_counters);
    cudaFree(p->d_prod);
    p->d_prod = nullptr;
    if (p->h_bounce) cudaFreeHost(p->h_bounce);
    if (p->bounce_ev) cudaEventDestroy(p->bounce_ev);
    p->h_bounce = nullptr;
    p->bounce_bytes = 0;
    p->bounce_ev = nullptr;
    p->bounce_pending = false;
    p->d_k = p->d_v = nullptr;
    p->d_table = p->d_status = p->d_counters = nullptr;
    p->d_partials = nullptr;
}

}  // namespace

namespace gkv {

int report_error(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int check_reachable(const void *ptr, int device, bool host_ok, const char *what) {
    if (!ptr) return GKV_OK;
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, ptr) != cudaSuccess) {
        cudaGetLastError();  // clear the sticky-free error of the query
        return report_error(GKV_ERR_INVALID, "%s: not an address the CUDA runtime knows", what);
    }
    if (device < 0 && cudaGetDevice(&device) != cudaSuccess) {
        cudaGetLastError();
        return report_error(GKV_ERR_CUDA, "%s: no current device", what);
    }
    switch (a.type) {
        case cudaMemoryTypeDevice:
            if (a.device != device)
                return report_error(GKV_ERR_INVALID, "%s is memory of GPU %d; the call runs on GPU %d", what,
                                    a.device, device);
            return GKV_OK;
        case cudaMemoryTypeManaged:
            return GKV_OK;
        case cudaMemoryTypeHost:
            if (!host_ok)
                return report_error(GKV_ERR_INVALID, "%s is host memory; this argument must be device memory",
                                    what);
            if (a.devicePointer != ptr)
                return report_error(GKV_ERR_INVALID,
                                    "%s: page-locked host memory not mapped at the same address on the GPU", what);
            return GKV_OK;
        default:
            return report_error(GKV_ERR_INVALID,
                                "%s is pageable host memory: pass device memory%s", what,
                                host_ok ? " or page-locked host memory (cudaHostAlloc / cudaHostRegister)" : "");
    }
}

int encode_page_tensor_map(CUtensorMap *map, const void *pages, int num_pages, int kv_heads,
                           int page_tokens, int head_dim) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return report_error(GKV_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    const int bh = std::min(page_tokens, attend_tile_keys(head_dim));
    const cuuint64_t dims[2] = {(cuuint64_t)head_dim,
                                (cuuint64_t)num_pages * kv_heads * page_tokens};
    const cuuint64_t strides[1] = {(cuuint64_t)head_dim * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)bh};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(pages), dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return report_error(GKV_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return GKV_OK;
}

}  // namespace gkv

// ------------------------------------------------------------ wire format
// The pool section of Engine.serialize / deserialize (Engine.swift:1078-1087,
// :1106-1116): little-endian Int64 framing, layers in ascending order, each
// `layer, length, count, K[count] fp16, count, V[count] fp16` with K/V the
// head-major compact [kv_heads, length, head_dim] (PagePool.compact).  And
// the StateBytes header, "GDNS" + Int64 version 1 (Shared/StateBytes.swift
// :12-40).

namespace {

void put_i64(uint8_t *&p, int64_t v) {
    for (int i = 0; i < 8; ++i) p[i] = (uint8_t)((uint64_t)v >> (8 * i));
    p += 8;
}

bool get_i64(const uint8_t *base, int64_t size, int64_t &off, int64_t *v) {
    if (off < 0 || size - off < 8) return false;
    uint64_t x = 0;
    for (int i = 0; i < 8; ++i) x |= (uint64_t)base[off + i] << (8 * i);
    *v = (int64_t)x;
    off += 8;
    return true;
}

int64_t compact_elems(const gkv_pool *pool, int64_t len) {
    return (int64_t)pool->cfg.kv_heads * len * pool->cfg.head_dim;
}

constexpr uint8_t kStateMagic[4] = {'G', 'D', 'N', 'S'};
constexpr int64_t kStateVersion = 1;

}  // namespace

extern "C" {

const char *gkv_last_error(void) { return g_last_error.c_str(); }

const char *gkv_version(void) { return "gadeon-kv-b200 0.1 (sm_100a)"; }

int gkv_pool_create(const gkv_pool_config *cfg, gkv_pool **out) {
    if (!cfg || !out) return fail(GKV_ERR_INVALID, "null argument");
    *out = nullptr;
    const gkv_pool_config c = *cfg;
    if (c.kv_heads < 1 || c.kv_heads > 64) return fail(GKV_ERR_INVALID, "kv_heads=%d", c.kv_heads);
    if (c.head_dim != 64 && c.head_dim != 128 && c.head_dim != 256 && c.head_dim != 512)
        return fail(GKV_ERR_UNSUPPORTED, "head_dim=%d (64/128/256/512)", c.head_dim);
    if (!is_pow2(c.page_tokens) || c.page_tokens > 16384)
        return fail(GKV_ERR_INVALID, "page_tokens=%d (power of two <= 16384)", c.page_tokens);
    if (c.num_pages < 1 || c.max_seqs < 1 || c.max_pages_per_seq < 1)
        return fail(GKV_ERR_INVALID, "num_pages/max_seqs/max_pages_per_seq must be >= 1");
    if ((int64_t)c.num_pages * c.kv_heads * c.page_tokens >= INT32_MAX)
        return fail(GKV_ERR_CAPACITY, "num_pages*kv_heads*page_tokens rows exceed 2^31");
    if ((int64_t)c.max_pages_per_seq * c.page_tokens > INT32_MAX)
        return fail(GKV_ERR_CAPACITY, "max context exceeds 2^31 positions");
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(GKV_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (no CUDA driver)");
    int ndev = 0;
    GKV_CUDA(cudaGetDeviceCount(&ndev), "cudaGetDeviceCount");
    if (c.device < 0 || c.device >= ndev) return fail(GKV_ERR_INVALID, "device %d", c.device);
    DeviceGuard guard(c.device);
    cudaDeviceProp prop;
    GKV_CUDA(cudaGetDeviceProperties(&prop, c.device), "cudaGetDeviceProperties");
    if (prop.major < 10)
        return fail(GKV_ERR_UNSUPPORTED, "device %d is sm_%d%d; this build targets sm_100a",
                    c.device, prop.major, prop.minor);

    gkv_pool *p = new gkv_pool();
    p->cfg = c;
    p->sm_count = prop.multiProcessorCount;
    p->tile_keys = gkv::attend_tile_keys(c.head_dim);
    p->page_elems = (size_t)c.kv_heads * c.page_tokens * c.head_dim;
    const size_t page_bytes = p->page_elems * 2;
    const size_t items = (size_t)c.max_seqs * c.kv_heads;
    cudaError_t e;
#define GKV_ALLOC(ptr, bytes)                                       \
    if ((e = cudaMalloc(&(ptr), (bytes))) != cudaSuccess) {         \
        free_device(p);                                             \
        delete p;                                                   \
        return cuda_fail(e, "cudaMalloc " #ptr);                    \
    }
    GKV_ALLOC(p->d_k, page_bytes * c.num_pages);
    GKV_ALLOC(p->d_v, page_bytes * c.num_pages);
    GKV_ALLOC(p->d_table, sizeof(int32_t) * (size_t)c.max_seqs * c.max_pages_per_seq);
    GKV_ALLOC(p->d_status, sizeof(int32_t));
    GKV_ALLOC(p->d_partials,
              sizeof(float) * (items + gkv::attend_grid(c.head_dim, c.page_tokens, INT32_MAX, p->sm_count)) *
                  gkv::attend_partial_floats(c.head_dim));
    GKV_ALLOC(p->d_counters, sizeof(int32_t) * items);
    if (gkv::producer_supported(c.head_dim)) GKV_ALLOC(p->d_prod, sizeof(uint16_t) * 2 * items * c.head_dim);
#undef GKV_ALLOC
    if ((e = cudaMemset(p->d_table, 0xff, sizeof(int32_t) * (size_t)c.max_seqs *
                                              c.max_pages_per_seq)) != cudaSuccess ||
        (e = cudaMemset(p->d_status, 0, sizeof(int32_t))) != cudaSuccess ||
        (e = cudaMemset(p->d_counters, 0, sizeof(int32_t) * items)) != cudaSuccess ||
        (e = cudaDeviceSynchronize()) != cudaSuccess) {
        free_device(p);
        delete p;
        return cuda_fail(e, "pool initialisation");
    }
    // TMA views of the pools: rows of head_dim halves, one row per
    // (page, kv head, slot); boxes of 64 columns x BH rows, 128B swizzle.
    // The chunk kernel loads page groups of min(P, 64) rows, the attend
    // kernel groups of min(P, its key tile).
    if (c.page_tokens >= 8) {
        const cuuint64_t dims[2] = {(cuuint64_t)c.head_dim,
                                    (cuuint64_t)c.num_pages * c.kv_heads * c.page_tokens};
        const cuuint64_t strides[1] = {(cuuint64_t)c.head_dim * 2};
        const cuuint32_t estr[2] = {1, 1};
        struct View {
            CUtensorMap *map;
            void *base;
            int bh;
        } views[4] = {{&p->tmk, p->d_k, std::min(c.page_tokens, 64)},
                      {&p->tmv, p->d_v, std::min(c.page_tokens, 64)},
                      {&p->tak, p->d_k, std::min(c.page_tokens, p->tile_keys)},
                      {&p->tav, p->d_v, std::min(c.page_tokens, p->tile_keys)}};
        for (const View &vw : views) {
            const cuuint32_t box[2] = {64, (cuuint32_t)vw.bh};
            CUresult r = enc(vw.map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, vw.base, dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
            if (r != CUDA_SUCCESS) {
                free_device(p);
                delete p;
                return fail(GKV_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
            }
        }
    }
    // Free list: pops yield the seeded permutation in order.
    std::vector<int32_t> perm(c.num_pages);
    for (int32_t i = 0; i < c.num_pages; ++i) perm[i] = i;
    uint64_t st = c.seed;
    for (int32_t i = c.num_pages - 1; i > 0; --i) {
        const int32_t j = (int32_t)(splitmix64(&st) % (uint64_t)(i + 1));
        std::swap(perm[i], perm[j]);
    }
    p->stack.assign(perm.rbegin(), perm.rend());
    p->ref.assign(c.num_pages, 0);
    *out = p;
    return GKV_OK;
}

int gkv_pool_destroy(gkv_pool *pool) {
    if (!pool) return GKV_OK;
    {
        DeviceGuard guard(pool->cfg.device);
        cudaDeviceSynchronize();
        free_device(pool);
    }
    delete pool;
    return GKV_OK;
}

int gkv_seq_create(gkv_pool *pool, int32_t *seq_id) {
    if (!pool || !seq_id) return fail(GKV_ERR_INVALID, "null argument");
    const int32_t id = pool->new_seq_id();
    if (id < 0) return fail(GKV_ERR_CAPACITY, "max_seqs=%d reached", pool->cfg.max_seqs);
    pool->seqs[id] = Seq();
    pool->seqs[id].active = true;
    *seq_id = id;
    return GKV_OK;
}

int gkv_seq_release(gkv_pool *pool, int32_t seq_id) {
    if (!pool) return fail(GKV_ERR_INVALID, "null pool");
    Seq *s = pool->seq(seq_id);
    if (!s) return fail(GKV_ERR_BAD_SEQ, "unknown sequence id %d", seq_id);
    while (!s->pages.empty()) {
        pool->unref(s->pages.back());
        s->pages.pop_back();
    }
    s->len = 0;
    s->active = false;
    return GKV_OK;
}

int gkv_seq_length(const gkv_pool *pool, int32_t seq_id, int64_t *length) {
    if (!pool || !length) return fail(GKV_ERR_INVALID, "null argument");
    const Seq *s = pool->seq(seq_id);
    if (!s) return fail(GKV_ERR_BAD_SEQ, "unknown sequence id %d", seq_id);
    *length = s->len;
    return GKV_OK;
}

int gkv_seq_page_count(const gkv_pool *pool, int32_t seq_id, int32_t *pages) {
    if (!pool || !pages) return fail(GKV_ERR_INVALID, "null argument");
    const Seq *s = pool->seq(seq_id);
    if (!s) return fail(GKV_ERR_BAD_SEQ, "unknown sequence id %d", seq_id);
    *pages = (int32_t)s->pages.size();
    return GKV_OK;
}

int gkv_free_page_count(const gkv_pool *pool, int32_t *pages) {
    if (!pool || !pages) return fail(GKV_ERR_INVALID, "null argument");
    *pages = (int32_t)pool->stack.size();
    return GKV_OK;
}

int gkv_append(gkv_pool *pool, int32_t n_seqs, const int32_t *seq_ids, const int32_t *n_new,
               const void *k, const void *v, void *stream) {
    if (!pool) return fail(GKV_ERR_INVALID, "null pool");
    int rc = check_batch(pool, n_seqs, seq_ids);
    if (rc) return rc;
    if (n_seqs > 0 && !n_new) return fail(GKV_ERR_INVALID, "null n_new");
    int64_t rows = 0;
    for (int32_t i = 0; i < n_seqs; ++i) rows += std::max(n_new[i], 0);
    if (rows > 0 && (!k || !v)) return fail(GKV_ERR_INVALID, "null k/v");
    DeviceGuard guard(pool->cfg.device);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    HostStage hs(pool);
    const size_t kb = (size_t)rows * pool->cfg.kv_heads * pool->cfg.head_dim * 2;
    hs.in(&k, kb);
    hs.in(&v, kb);
    if ((rc = hs.reserve())) return rc;
    if (!aligned16(k) || !aligned16(v)) return fail(GKV_ERR_INVALID, "k/v not 16-byte aligned");
    if (rows > 0 && (rc = check_buffers(pool, {{k, "k"}, {v, "v"}}))) return rc;
    std::vector<gkv::AppendEntry> entries;
    std::vector<gkv::TouchedPage> pages;
    rc = plan_append(pool, n_seqs, seq_ids, n_new, entries, pages);
    if (rc) return rc;
    hs.copy_in();
    rc = enqueue_append(pool, entries, pages, k, v, 0, st);
    return rc ? rc : hs.finish(st);
}

int gkv_seed(gkv_pool *pool, int32_t seq_id, const void *K, const void *V, int64_t count,
             void *stream) {
    if (!pool) return fail(GKV_ERR_INVALID, "null pool");
    Seq *s = pool->seq(seq_id);
    if (!s) return fail(GKV_ERR_BAD_SEQ, "unknown sequence id %d", seq_id);
    if (s->len != 0) return fail(GKV_ERR_BAD_SEQ, "seed needs an empty sequence (%d has %lld)",
                                 seq_id, (long long)s->len);
    if (count < 0 || count > INT32_MAX) return fail(GKV_ERR_INVALID, "count=%lld", (long long)count);
    if (count > 0 && (!K || !V)) return fail(GKV_ERR_INVALID, "null K/V");
    DeviceGuard guard(pool->cfg.device);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    HostStage hs(pool);
    const size_t kb = (size_t)count * pool->cfg.kv_heads * pool->cfg.head_dim * 2;
    hs.in(&K, kb);
    hs.in(&V, kb);
    int rc = hs.reserve();
    if (rc) return rc;
    if (!aligned16(K) || !aligned16(V)) return fail(GKV_ERR_INVALID, "K/V not 16-byte aligned");
    if (count > 0 && (rc = check_buffers(pool, {{K, "K"}, {V, "V"}}))) return rc;
    const int32_t n = (int32_t)count;
    std::vector<gkv::AppendEntry> entries;
    std::vector<gkv::TouchedPage> pages;
    rc = plan_append(pool, 1, &seq_id, &n, entries, pages);
    if (rc) return rc;
    hs.copy_in();
    rc = enqueue_append(pool, entries, pages, K, V, 1, st);
    return rc ? rc : hs.finish(st);
}

int gkv_attend_ex(gkv_pool *pool, int32_t n_seqs, const int32_t *seq_ids, int32_t n_q, int32_t group,
                  const void *q, void *out, float scale, uint32_t flags, void *stream) {
    if (!pool) return fail(GKV_ERR_INVALID, "null pool");
    if (flags & ~(uint32_t)(GKV_ATTEND_HEAD_MAJOR | GKV_ATTEND_OUT_F16 | GKV_ATTEND_P_F16))
        return fail(GKV_ERR_INVALID, "unknown flags 0x%x", flags);
    int rc = check_batch(pool, n_seqs, seq_ids);
    if (rc) return rc;
    if (!(std::isfinite(scale) && scale != 0.f)) return fail(GKV_ERR_INVALID, "scale must be finite and non-zero");
    if (n_q < 1 || group < 1) return fail(GKV_ERR_INVALID, "n_q=%d group=%d", n_q, group);
    DeviceGuard guard(pool->cfg.device);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    HostStage hs(pool);
    const size_t nqo = (size_t)n_seqs * n_q * pool->cfg.kv_heads * group * pool->cfg.head_dim;
    hs.in(&q, nqo * 2);
    hs.out(&out, nqo * ((flags & GKV_ATTEND_OUT_F16) ? 2 : 4));
    if ((rc = hs.reserve())) return rc;
    rc = check_attend(pool, n_seqs, seq_ids, n_q, group, q, out);
    if (rc) return rc;
    if (n_seqs > 0 && (rc = check_buffers(pool, {{q, "q"}, {out, "out"}}))) return rc;
    hs.copy_in();
    rc = enqueue_attend(pool, n_seqs, seq_ids, n_q, group, q, out, scale, flags, st);
    return rc ? rc : hs.finish(st);
}

int gkv_attend(gkv_pool *pool, int32_t n_seqs, const int32_t *seq_ids, int32_t n_q, int32_t group,
               const void *q, float *out, float scale, void *stream) {
    return gkv_attend_ex(pool, n_seqs, seq_ids, n_q, group, q, out, scale, 0u, stream);
}

int gkv_attend_decode(gkv_pool *pool, int32_t n_seqs, const int32_t *seq_ids, int32_t group, const void *q,
                      float *out, float scale, void *stream) {
    return gkv_attend_ex(pool, n_seqs, seq_ids, 1, group, q, out, scale, 0u, stream);
}

int gkv_attend_causal(gkv_pool *pool, int32_t n_seqs, const int32_t *seq_ids, int32_t n_q, int32_t group,
                      const void *q, float *out, float scale, void *stream) {
    return gkv_attend_ex(pool, n_seqs, seq_ids, n_q, group, q, out, scale, 0u, stream);
}

int gkv_append_attend_ex(gkv_pool *pool, int32_t n_seqs, const int32_t *seq_ids, int32_t n_q, int32_t group,
                         const void *k, const void *v, const void *q, void *out, float scale, uint32_t flags,
                         void *stream) {
    if (!pool) return fail(GKV_ERR_INVALID, "null pool");
    if (flags & ~(uint32_t)(GKV_ATTEND_HEAD_MAJOR | GKV_ATTEND_OUT_F16 | GKV_ATTEND_P_F16))
        return fail(GKV_ERR_INVALID, "unknown flags 0x%x", flags);
    int rc = check_batch(pool, n_seqs, seq_ids);
    if (rc) return rc;
    if (n_q < 1 || group < 1) return fail(GKV_ERR_INVALID, "n_q=%d group=%d", n_q, group);
    if ((int64_t)n_q * group > 16 &&
        !gkv::chunk_supported(pool->cfg.head_dim, pool->cfg.page_tokens, group))
        return fail(GKV_ERR_UNSUPPORTED,
                    "n_q*group = %lld rows per kv head needs the chunk kernel (head_dim <= 256, "
                    "page_tokens >= 8)",
                    (long long)n_q * group);
    if (n_seqs > 0 && (!k || !v || !q || !out)) return fail(GKV_ERR_INVALID, "null k/v/q/out");
    if (!(std::isfinite(scale) && scale != 0.f)) return fail(GKV_ERR_INVALID, "scale must be finite and non-zero");
    DeviceGuard guard(pool->cfg.device);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    HostStage hs(pool);
    const size_t nkv = (size_t)n_seqs * n_q * pool->cfg.kv_heads * pool->cfg.head_dim;
    const size_t nqo = nkv * group;
    hs.in(&k, nkv * 2);
    hs.in(&v, nkv * 2);
    hs.in(&q, nqo * 2);
    hs.out(&out, nqo * ((flags & GKV_ATTEND_OUT_F16) ? 2 : 4));
    if ((rc = hs.reserve())) return rc;
    if (!aligned16(k) || !aligned16(v) || !aligned16(q) || !aligned16(out))
        return fail(GKV_ERR_INVALID, "k/v/q/out not 16-byte aligned");
    if (n_seqs > 0 && (rc = check_buffers(pool, {{k, "k"}, {v, "v"}, {q, "q"}, {out, "out"}}))) return rc;
    std::vector<int32_t> n_new(n_seqs, n_q);
    std::vector<gkv::AppendEntry> entries;
    std::vector<gkv::TouchedPage> pages;
    rc = plan_append(pool, n_seqs, seq_ids, n_new.data(), entries, pages);
    if (rc) return rc;
    hs.copy_in();
    // Decode and verify steps of the split-K kernel (n_q*group <= 16, n_q <=
    // P) with TMA-staged pages and no shared tail page: the append rides
    // inside the attend kernel (one launch per layer).
    std::vector<gkv::FusedTail> tails;
    const bool fuse = (int64_t)n_q * group <= 16 && n_q <= pool->cfg.page_tokens && pool->cfg.page_tokens >= 8 &&
                      (pool->cfg.head_dim == 128 || pool->cfg.head_dim == 256) && fused_tails(pages, n_seqs, tails);
    if (fuse) {
        rc = enqueue_attend(pool, n_seqs, seq_ids, n_q, group, q, out, scale, flags, st, tails.data(), k, v);
    } else {
        rc = enqueue_append(pool, entries, pages, k, v, (flags & GKV_ATTEND_HEAD_MAJOR) ? 1 : 0, st);
        if (!rc) rc = enqueue_attend(pool, n_seqs, seq_ids, n_q, group, q, out, scale, flags, st);
    }
    return rc ? rc : hs.finish(st);
}

int gkv_append_attend(gkv_pool *pool, int32_t n_seqs, const int32_t *seq_ids, int32_t n_q, int32_t group,
                      const void *k, const void *v, const void *q, float *out, float scale, void *stream) {
    return gkv_append_attend_ex(pool, n_seqs, seq_ids, n_q, group, k, v, q, out, scale, 0u, stream);
}

int gkv_attn_step(gkv_pool *pool, int32_t n_seqs, const int32_t *seq_ids, int32_t group, const float *q_gate,
                  const float *k_raw, const float *v_raw, const float *q_norm, const float *k_norm, float eps,
                  const float *rope_cos, const float *rope_sin, int32_t n_rot, float scale, float *out,
                  void *stream) {
    if (!pool) return fail(GKV_ERR_INVALID, "null pool");
    int rc = check_batch(pool, n_seqs, seq_ids);
    if (rc) return rc;
    const int dh = pool->cfg.head_dim;
    if (!gkv::producer_supported(dh)) return fail(GKV_ERR_UNSUPPORTED, "gkv_attn_step needs head_dim 128 or 256");
    if (group < 1 || group > 16) return fail(GKV_ERR_INVALID, "group=%d (1..16 query heads per kv head)", group);
    if (n_rot < 16 || n_rot > dh || n_rot % 16)
        return fail(GKV_ERR_INVALID, "n_rot=%d (a multiple of 16 in 16..%d)", n_rot, dh);
    if (!(std::isfinite(eps) && eps >= 0.f)) return fail(GKV_ERR_INVALID, "eps must be finite and >= 0");
    if (!(std::isfinite(scale) && scale != 0.f)) return fail(GKV_ERR_INVALID, "scale must be finite and non-zero");
    if (n_seqs > 0 && (!q_gate || !k_raw || !v_raw || !q_norm || !k_norm || !rope_cos || !rope_sin || !out))
        return fail(GKV_ERR_INVALID, "null argument");
    DeviceGuard guard(pool->cfg.device);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    // the staging slots: they outlive every use of hs below
    const void *in[7] = {q_gate, k_raw, v_raw, q_norm, k_norm, rope_cos, rope_sin};
    void *o = out;
    HostStage hs(pool);
    {
        const size_t n = (size_t)n_seqs, KVH = (size_t)pool->cfg.kv_heads, D = (size_t)dh;
        const size_t nH = KVH * (size_t)group, hr = (size_t)(n_rot / 2);
        const size_t in_bytes[7] = {n * nH * 2 * D * 4, n * KVH * D * 4, n * KVH * D * 4, D * 4, D * 4,
                                    n * hr * 4, n * hr * 4};
        if (n_seqs > 0) {
            for (int i = 0; i < 7; ++i) hs.in(&in[i], in_bytes[i]);
            hs.out(&o, n * nH * D * 4);
            if ((rc = hs.reserve())) return rc;
        }
        q_gate = static_cast<const float *>(in[0]);
        k_raw = static_cast<const float *>(in[1]);
        v_raw = static_cast<const float *>(in[2]);
        q_norm = static_cast<const float *>(in[3]);
        k_norm = static_cast<const float *>(in[4]);
        rope_cos = static_cast<const float *>(in[5]);
        rope_sin = static_cast<const float *>(in[6]);
        out = static_cast<float *>(o);
    }
    if (!aligned16(q_gate) || !aligned16(k_raw) || !aligned16(v_raw) || !aligned16(out) ||
        ((reinterpret_cast<uintptr_t>(q_norm) | reinterpret_cast<uintptr_t>(k_norm) |
          reinterpret_cast<uintptr_t>(rope_cos) | reinterpret_cast<uintptr_t>(rope_sin)) & 3))
        return fail(GKV_ERR_INVALID, "q_gate/k_raw/v_raw/out must be 16-byte aligned, the rest 4-byte");
    if (n_seqs > 0 && (rc = check_buffers(pool, {{q_gate, "q_gate"}, {k_raw, "k_raw"}, {v_raw, "v_raw"},
                                                 {q_norm, "q_norm"}, {k_norm, "k_norm"}, {rope_cos, "rope_cos"},
                                                 {rope_sin, "rope_sin"}, {out, "out"}})))
        return rc;
    std::vector<int32_t> n_new(n_seqs, 1);
    std::vector<gkv::AppendEntry> entries;
    std::vector<gkv::TouchedPage> pages;
    rc = plan_append(pool, n_seqs, seq_ids, n_new.data(), entries, pages);
    if (rc) return rc;
    hs.copy_in();
    gkv::ProducerArgs prod{q_gate, k_raw, v_raw, q_norm, k_norm, rope_cos, rope_sin, n_rot, eps};
    // Same fusion rule as gkv_append_attend: TMA-staged pages and no shared
    // tail page -> the attend kernel's prologue builds and writes the rows.
    std::vector<gkv::FusedTail> tails;
    if (pool->cfg.page_tokens >= 8 && fused_tails(pages, n_seqs, tails)) {
        rc = enqueue_attend(pool, n_seqs, seq_ids, 1, group, nullptr, out, scale, 0u, st, tails.data(), nullptr,
                            nullptr, &prod);
        return rc ? rc : hs.finish(st);
    }
    // Otherwise the rows are built by a small kernel, appended (copy-on-write
    // of a shared tail included), then attended.
    const size_t rows = (size_t)n_seqs * pool->cfg.kv_heads;
    gkv::ProduceParams pp{prod, pool->d_prod, pool->d_prod + rows * dh, n_seqs, pool->cfg.kv_heads};
    GKV_CUDA(gkv::launch_produce_kv(pp, dh, st), "producer kernel launch");
    rc = enqueue_append(pool, entries, pages, pp.k_out, pp.v_out, 0, st);
    if (rc) return rc;
    rc = enqueue_attend(pool, n_seqs, seq_ids, 1, group, nullptr, out, scale, 0u, st, nullptr, nullptr, nullptr,
                        &prod);
    return rc ? rc : hs.finish(st);
}

int gkv_rope_table(int32_t n_rot, float base, int32_t n, const int64_t *positions, float *cos_out,
                   float *sin_out) {
    if (n_rot < 2 || n_rot % 2 || !(std::isfinite(base) && base > 0.f) || n < 0)
        return fail(GKV_ERR_INVALID, "n_rot=%d base=%g n=%d", n_rot, (double)base, n);
    if (n > 0 && (!positions || !cos_out || !sin_out)) return fail(GKV_ERR_INVALID, "null argument");
    const int half = n_rot / 2;
    for (int32_t t = 0; t < n; ++t)
        for (int i = 0; i < half; ++i) {
            // Kernels.swift:74-76: freq = base^(-2i/nRot), angle = pos * freq (fp32)
            const float freq = powf(base, -2.0f * (float)i / (float)n_rot);
            const float ang = (float)positions[t] * freq;
            cos_out[(size_t)t * half + i] = cosf(ang);
            sin_out[(size_t)t * half + i] = sinf(ang);
        }
    return GKV_OK;
}

int gkv_truncate(gkv_pool *pool, int32_t n_seqs, const int32_t *seq_ids, const int64_t *new_len) {
    if (!pool) return fail(GKV_ERR_INVALID, "null pool");
    int rc = check_batch(pool, n_seqs, seq_ids);
    if (rc) return rc;
    if (n_seqs > 0 && !new_len) return fail(GKV_ERR_INVALID, "null new_len");
    for (int32_t i = 0; i < n_seqs; ++i) {
        const Seq &s = *pool->seq(seq_ids[i]);
        if (new_len[i] < 0 || new_len[i] > s.len)
            return fail(GKV_ERR_BAD_SEQ, "truncate sequence %d to %lld (length %lld)", seq_ids[i],
                        (long long)new_len[i], (long long)s.len);
    }
    for (int32_t i = 0; i < n_seqs; ++i) {
        Seq &s = *pool->seq(seq_ids[i]);
        s.len = new_len[i];
        const int64_t need = pool->pages_for(s.len);
        while ((int64_t)s.pages.size() > need) {
            pool->unref(s.pages.back());
            s.pages.pop_back();
        }
    }
    return GKV_OK;
}

int gkv_rewind_append(gkv_pool *pool, int32_t n_seqs, const int32_t *seq_ids, const int64_t *base_len,
                      const int32_t *n_new, const void *k, const void *v, void *stream) {
    if (!pool) return fail(GKV_ERR_INVALID, "null pool");
    int rc = check_batch(pool, n_seqs, seq_ids);
    if (rc) return rc;
    if (n_seqs > 0 && (!base_len || !n_new)) return fail(GKV_ERR_INVALID, "null base_len/n_new");
    int64_t rows = 0;
    for (int32_t i = 0; i < n_seqs; ++i) {
        const Seq &s = *pool->seq(seq_ids[i]);
        if (base_len[i] < 0 || base_len[i] > s.len)
            return fail(GKV_ERR_BAD_SEQ, "rewind sequence %d to %lld (length %lld)", seq_ids[i],
                        (long long)base_len[i], (long long)s.len);
        if (n_new[i] < 0) return fail(GKV_ERR_INVALID, "n_new[%d] = %d", i, n_new[i]);
        rows += n_new[i];
    }
    if (rows > 0 && (!k || !v)) return fail(GKV_ERR_INVALID, "null k/v");
    DeviceGuard guard(pool->cfg.device);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    HostStage hs(pool);
    const size_t kb = (size_t)rows * pool->cfg.kv_heads * pool->cfg.head_dim * 2;
    hs.in(&k, kb);
    hs.in(&v, kb);
    if ((rc = hs.reserve())) return rc;
    if (!aligned16(k) || !aligned16(v)) return fail(GKV_ERR_INVALID, "k/v not 16-byte aligned");
    if (rows > 0 && (rc = check_buffers(pool, {{k, "k"}, {v, "v"}}))) return rc;
    // truncate (PagePool.truncate: pages pushed last-first), keeping an undo
    // log so that an append refused for lack of pages leaves no trace
    struct Undo {
        int32_t seq;
        int64_t len;
        std::vector<int32_t> pages;  // removed, in removal order
        std::vector<char> freed;     // pushed onto the free list
    };
    std::vector<Undo> undo(n_seqs);
    for (int32_t i = 0; i < n_seqs; ++i) {
        Seq &s = *pool->seq(seq_ids[i]);
        undo[i].seq = seq_ids[i];
        undo[i].len = s.len;
        s.len = base_len[i];
        const int64_t need = pool->pages_for(s.len);
        while ((int64_t)s.pages.size() > need) {
            const int32_t pid = s.pages.back();
            s.pages.pop_back();
            undo[i].pages.push_back(pid);
            undo[i].freed.push_back(pool->ref[pid] == 1);
            pool->unref(pid);
        }
    }
    std::vector<gkv::AppendEntry> entries;
    std::vector<gkv::TouchedPage> pages;
    rc = plan_append(pool, n_seqs, seq_ids, n_new, entries, pages);
    if (rc) {
        for (int32_t i = n_seqs - 1; i >= 0; --i) {
            Seq &s = *pool->seq(undo[i].seq);
            for (size_t j = undo[i].pages.size(); j-- > 0;) {
                const int32_t pid = undo[i].pages[j];
                if (undo[i].freed[j]) pool->stack.pop_back();  // the push of this page, undone
                pool->ref[pid]++;
                s.pages.push_back(pid);
            }
            s.len = undo[i].len;
        }
        return rc;
    }
    hs.copy_in();
    rc = enqueue_append(pool, entries, pages, k, v, 0, st);
    return rc ? rc : hs.finish(st);
}

int gkv_clone_seq(gkv_pool *pool, int32_t src, int32_t *dst, void *stream) {
    if (!pool || !dst) return fail(GKV_ERR_INVALID, "null argument");
    if (!pool->seq(src)) return fail(GKV_ERR_BAD_SEQ, "unknown sequence id %d", src);
    const bool partial = pool->seq(src)->len % pool->cfg.page_tokens != 0;
    if (partial && pool->stack.empty()) return fail(GKV_ERR_NO_PAGES, "clone needs 1 free page");
    const int32_t id = pool->new_seq_id();
    if (id < 0) return fail(GKV_ERR_CAPACITY, "max_seqs=%d reached", pool->cfg.max_seqs);
    DeviceGuard guard(pool->cfg.device);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const Seq &s = *pool->seq(src);
    Seq c;
    c.active = true;
    c.len = s.len;
    c.pages = s.pages;
    const size_t stride = pool->cfg.max_pages_per_seq;
    if (!c.pages.empty()) {
        cudaError_t e = cudaMemcpyAsync(pool->d_table + id * stride, pool->d_table + src * stride,
                                        sizeof(int32_t) * c.pages.size(),
                                        cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) return cuda_fail(e, "clone table copy");
    }
    for (int32_t pid : c.pages) pool->ref[pid]++;
    std::vector<gkv::AppendEntry> entries;
    std::vector<gkv::TouchedPage> pages;
    if (partial) {
        const int32_t old = c.pages.back();
        const int32_t pid = pool->pop();
        pool->ref[old]--;
        c.pages.back() = pid;
        entries.push_back({id, (int32_t)c.len, 0, 0});
        pages.push_back({0, (int32_t)c.pages.size() - 1, pid, old});
    }
    pool->seqs[id] = std::move(c);
    *dst = id;
    return enqueue_append(pool, entries, pages, nullptr, nullptr, 0, st);
}

int gkv_compact_seq(gkv_pool *pool, int32_t seq_id, void *K, void *V, void *stream) {
    if (!pool) return fail(GKV_ERR_INVALID, "null pool");
    const Seq *s = pool->seq(seq_id);
    if (!s) return fail(GKV_ERR_BAD_SEQ, "unknown sequence id %d", seq_id);
    if (s->len > 0 && (!K || !V)) return fail(GKV_ERR_INVALID, "null K/V");
    DeviceGuard guard(pool->cfg.device);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    HostStage hs(pool);
    const size_t kb = (size_t)pool->cfg.kv_heads * s->len * pool->cfg.head_dim * 2;
    hs.out(&K, kb);
    hs.out(&V, kb);
    int rc = hs.reserve();
    if (rc) return rc;
    if (!aligned16(K) || !aligned16(V)) return fail(GKV_ERR_INVALID, "K/V not 16-byte aligned");
    if (s->len > 0 && (rc = check_buffers(pool, {{K, "K"}, {V, "V"}}))) return rc;
    gkv::CompactParams p{};
    p.table = pool->d_table + (size_t)seq_id * pool->cfg.max_pages_per_seq;
    p.k_pool = pool->d_k;
    p.v_pool = pool->d_v;
    p.K = static_cast<uint16_t *>(K);
    p.V = static_cast<uint16_t *>(V);
    p.start = 0;
    p.count = p.rows = s->len;
    p.kvh = pool->cfg.kv_heads;
    p.dh = pool->cfg.head_dim;
    p.P = pool->cfg.page_tokens;
    GKV_CUDA(gkv::launch_compact(p, st), "compact kernel launch");
    return hs.finish(st);
}

int gkv_tile_at(gkv_pool *pool, int32_t seq_id, int64_t start, int64_t count, int32_t tile_p, void *K, void *V,
                void *stream) {
    if (!pool) return fail(GKV_ERR_INVALID, "null pool");
    const Seq *s = pool->seq(seq_id);
    if (!s) return fail(GKV_ERR_BAD_SEQ, "unknown sequence id %d", seq_id);
    if (tile_p < 1 || count < 0 || count > tile_p)
        return fail(GKV_ERR_INVALID, "count=%lld tile_p=%d (need 0 <= count <= tile_p, tile_p >= 1)",
                    (long long)count, tile_p);
    if (start < 0 || start + count > s->len)
        return fail(GKV_ERR_BAD_SEQ, "window [%lld, %lld) outside sequence %d of length %lld", (long long)start,
                    (long long)(start + count), seq_id, (long long)s->len);
    if (!K || !V) return fail(GKV_ERR_INVALID, "null K/V");
    DeviceGuard guard(pool->cfg.device);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    HostStage hs(pool);
    const size_t kb = (size_t)pool->cfg.kv_heads * tile_p * pool->cfg.head_dim * 2;
    hs.out(&K, kb);
    hs.out(&V, kb);
    int rc = hs.reserve();
    if (rc) return rc;
    if (!aligned16(K) || !aligned16(V)) return fail(GKV_ERR_INVALID, "K/V not 16-byte aligned");
    if ((rc = check_buffers(pool, {{K, "K"}, {V, "V"}}))) return rc;
    gkv::CompactParams p{};
    p.table = pool->d_table + (size_t)seq_id * pool->cfg.max_pages_per_seq;
    p.k_pool = pool->d_k;
    p.v_pool = pool->d_v;
    p.K = static_cast<uint16_t *>(K);
    p.V = static_cast<uint16_t *>(V);
    p.start = start;
    p.count = count;
    p.rows = tile_p;
    p.kvh = pool->cfg.kv_heads;
    p.dh = pool->cfg.head_dim;
    p.P = pool->cfg.page_tokens;
    GKV_CUDA(gkv::launch_compact(p, st), "tile kernel launch");
    return hs.finish(st);
}

int gkv_from_compact(gkv_pool *pool, const void *K, const void *V, int64_t length,
                     int32_t *seq_id, void *stream) {
    if (!pool || !seq_id) return fail(GKV_ERR_INVALID, "null argument");
    if (length < 0) return fail(GKV_ERR_INVALID, "length=%lld", (long long)length);
    if (length > 0) {  // before a sequence is made, so a refused buffer leaves nothing behind
        if (!K || !V) return fail(GKV_ERR_INVALID, "null K/V");
        for (const void *b : {K, V})  // pageable host memory: staged by gkv_seed below
            if (!is_pageable(b)) {
                const int rc = check_buffers(pool, {{b, b == K ? "K" : "V"}});
                if (rc) return rc;
            }
    }
    if (pool->pages_for(length) > (int64_t)pool->stack.size())
        return fail(GKV_ERR_NO_PAGES, "fromCompact needs %lld pages",
                    (long long)pool->pages_for(length));
    int32_t id;
    int rc = gkv_seq_create(pool, &id);
    if (rc) return rc;
    rc = gkv_seed(pool, id, K, V, length, stream);
    if (rc) {
        gkv_seq_release(pool, id);
        return rc;
    }
    *seq_id = id;
    return GKV_OK;
}

int gkv_export_table(gkv_pool *pool, int32_t seq_id, int32_t *pages_out, int32_t cap,
                     int32_t *n_pages) {
    if (!pool || !n_pages) return fail(GKV_ERR_INVALID, "null argument");
    const Seq *s = pool->seq(seq_id);
    if (!s) return fail(GKV_ERR_BAD_SEQ, "unknown sequence id %d", seq_id);
    const int32_t n = (int32_t)s->pages.size();
    *n_pages = n;
    if (!pages_out || n == 0) return GKV_OK;
    if (cap < n) return fail(GKV_ERR_INVALID, "cap %d < %d pages", cap, n);
    DeviceGuard guard(pool->cfg.device);
    GKV_CUDA(cudaDeviceSynchronize(), "synchronize");
    GKV_CUDA(cudaMemcpy(pages_out, pool->d_table + (size_t)seq_id * pool->cfg.max_pages_per_seq,
                        sizeof(int32_t) * n, cudaMemcpyDeviceToHost),
             "table copy");
    return GKV_OK;
}

int gkv_export_free_list(const gkv_pool *pool, int32_t *out, int32_t cap, int32_t *n) {
    if (!pool || !n) return fail(GKV_ERR_INVALID, "null argument");
    const int32_t m = (int32_t)pool->stack.size();
    *n = m;
    if (!out) return GKV_OK;
    if (cap < m) return fail(GKV_ERR_INVALID, "cap %d < %d free pages", cap, m);
    for (int32_t i = 0; i < m; ++i) out[i] = pool->stack[m - 1 - i];
    return GKV_OK;
}

int gkv_page_refcount(const gkv_pool *pool, int32_t page_id, int32_t *ref) {
    if (!pool || !ref) return fail(GKV_ERR_INVALID, "null argument");
    if (page_id < 0 || page_id >= pool->cfg.num_pages)
        return fail(GKV_ERR_INVALID, "page %d", page_id);
    *ref = pool->ref[page_id];
    return GKV_OK;
}

int gkv_export_page(gkv_pool *pool, int32_t page_id, void *k_host, void *v_host) {
    if (!pool || !k_host || !v_host) return fail(GKV_ERR_INVALID, "null argument");
    if (page_id < 0 || page_id >= pool->cfg.num_pages)
        return fail(GKV_ERR_INVALID, "page %d", page_id);
    DeviceGuard guard(pool->cfg.device);
    const size_t bytes = pool->page_elems * 2;
    GKV_CUDA(cudaDeviceSynchronize(), "synchronize");
    GKV_CUDA(cudaMemcpy(k_host, pool->d_k + page_id * pool->page_elems, bytes,
                        cudaMemcpyDeviceToHost),
             "page copy");
    GKV_CUDA(cudaMemcpy(v_host, pool->d_v + page_id * pool->page_elems, bytes,
                        cudaMemcpyDeviceToHost),
             "page copy");
    return GKV_OK;
}

int gkv_check_bounded_wait(int32_t device, int64_t limit_ns, int32_t *status) {
    if (!status) return fail(GKV_ERR_INVALID, "null status");
    if (limit_ns < 1000000 || limit_ns > 10000000000ll)
        return fail(GKV_ERR_INVALID, "limit_ns=%lld (1 ms .. 10 s)", (long long)limit_ns);
    int count = 0;
    GKV_CUDA(cudaGetDeviceCount(&count), "device count");
    if (device < 0 || device >= count) return fail(GKV_ERR_INVALID, "device %d of %d", device, count);
    DeviceGuard guard(device);
    int32_t *d = nullptr;
    GKV_CUDA(cudaMalloc(&d, sizeof(int32_t)), "probe status");
    cudaError_t e = cudaMemset(d, 0, sizeof(int32_t));
    if (e == cudaSuccess) e = gkv::launch_bounded_wait_probe(d, (uint64_t)limit_ns, 0);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(status, d, sizeof(int32_t), cudaMemcpyDeviceToHost);
    cudaFree(d);
    if (e != cudaSuccess) return cuda_fail(e, "bounded-wait probe");
    return GKV_OK;
}

int gkv_device_status(gkv_pool *pool, int32_t *status) {
    if (!pool || !status) return fail(GKV_ERR_INVALID, "null argument");
    DeviceGuard guard(pool->cfg.device);
    GKV_CUDA(cudaDeviceSynchronize(), "synchronize");
    GKV_CUDA(cudaMemcpy(status, pool->d_status, sizeof(int32_t), cudaMemcpyDeviceToHost),
             "status copy");
    return GKV_OK;
}


int gkv_serialize(int32_t n_layers, gkv_pool *const *pools, const int32_t *layer_ids, const int32_t *seq_ids,
                  void *buf, int64_t cap, int64_t *size, void *stream) {
    if (n_layers < 0 || !size || (n_layers > 0 && (!pools || !layer_ids || !seq_ids)))
        return fail(GKV_ERR_INVALID, "null argument");
    int64_t total = 8;
    std::vector<int32_t> order(n_layers);
    for (int32_t i = 0; i < n_layers; ++i) {
        if (!pools[i]) return fail(GKV_ERR_INVALID, "null pool %d", i);
        const Seq *s = pools[i]->seq(seq_ids[i]);
        if (!s) return fail(GKV_ERR_BAD_SEQ, "unknown sequence id %d in pool %d", seq_ids[i], i);
        total += 8 * 4 + 4 * compact_elems(pools[i], s->len);  // layer, length, n, n + K, V
        order[i] = i;
    }
    // Engine.serialize walks b.pools.keys.sorted()
    std::sort(order.begin(), order.end(), [&](int32_t a, int32_t b) { return layer_ids[a] < layer_ids[b]; });
    for (int32_t i = 1; i < n_layers; ++i)
        if (layer_ids[order[i]] == layer_ids[order[i - 1]])
            return fail(GKV_ERR_INVALID, "layer id %d given twice", layer_ids[order[i]]);
    *size = total;
    if (!buf) return GKV_OK;
    if (cap < total) return fail(GKV_ERR_CAPACITY, "buffer of %lld bytes < %lld", (long long)cap, (long long)total);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint8_t *p = static_cast<uint8_t *>(buf);
    put_i64(p, n_layers);
    for (int32_t oi = 0; oi < n_layers; ++oi) {
        gkv_pool *pool = pools[order[oi]];
        const int32_t sid = seq_ids[order[oi]];
        const int64_t len = pool->seq(sid)->len, n = compact_elems(pool, len);
        put_i64(p, layer_ids[order[oi]]);
        put_i64(p, len);
        uint16_t *dk = nullptr;
        if (n > 0) {
            DeviceGuard guard(pool->cfg.device);
            GKV_CUDA(cudaMalloc(&dk, sizeof(uint16_t) * 2 * n), "serialize scratch");
            int rc = gkv_compact_seq(pool, sid, dk, dk + n, stream);
            cudaError_t e = cudaSuccess;
            if (rc == GKV_OK) {
                put_i64(p, n);
                e = cudaMemcpyAsync(p, dk, sizeof(uint16_t) * n, cudaMemcpyDeviceToHost, st);
                p += 2 * n;
                put_i64(p, n);
                if (e == cudaSuccess) e = cudaMemcpyAsync(p, dk + n, sizeof(uint16_t) * n, cudaMemcpyDeviceToHost, st);
                p += 2 * n;
                if (e == cudaSuccess) e = cudaStreamSynchronize(st);
            }
            cudaFree(dk);
            if (rc) return rc;
            if (e != cudaSuccess) return cuda_fail(e, "serialize copy");
        } else {
            put_i64(p, 0);
            put_i64(p, 0);
        }
    }
    return GKV_OK;
}

int gkv_deserialize(int32_t n_layers, gkv_pool *const *pools, const void *buf, int64_t size, int32_t *layer_ids_out,
                    int32_t *seq_ids_out, int64_t *consumed, void *stream) {
    if (n_layers < 0 || !buf || size < 0 || (n_layers > 0 && (!pools || !layer_ids_out || !seq_ids_out)))
        return fail(GKV_ERR_INVALID, "null argument");
    const uint8_t *b = static_cast<const uint8_t *>(buf);
    // parse and check everything before any sequence is created
    struct Sec { int64_t layer, len, n, k_off, v_off; };
    std::vector<Sec> secs(n_layers);
    int64_t off = 0, count = 0;
    if (!get_i64(b, size, off, &count)) return fail(GKV_ERR_INVALID, "truncated: no layer count");
    if (count != n_layers) return fail(GKV_ERR_INVALID, "%lld layers in the data, %d pools", (long long)count, n_layers);
    for (int32_t i = 0; i < n_layers; ++i) {
        if (!pools[i]) return fail(GKV_ERR_INVALID, "null pool %d", i);
        Sec &s = secs[i];
        int64_t kn = 0, vn = 0;
        if (!get_i64(b, size, off, &s.layer) || !get_i64(b, size, off, &s.len) || !get_i64(b, size, off, &kn))
            return fail(GKV_ERR_INVALID, "truncated section %d", i);
        if (s.len < 0 || s.layer < INT32_MIN || s.layer > INT32_MAX)
            return fail(GKV_ERR_INVALID, "section %d: layer %lld length %lld", i, (long long)s.layer, (long long)s.len);
        s.n = compact_elems(pools[i], s.len);
        if (kn != s.n) return fail(GKV_ERR_INVALID, "section %d: %lld K values, pool geometry needs %lld", i,
                                   (long long)kn, (long long)s.n);
        s.k_off = off;
        if (size - off < 2 * kn) return fail(GKV_ERR_INVALID, "truncated K of section %d", i);
        off += 2 * kn;
        if (!get_i64(b, size, off, &vn) || vn != s.n) return fail(GKV_ERR_INVALID, "section %d: V count", i);
        s.v_off = off;
        if (size - off < 2 * vn) return fail(GKV_ERR_INVALID, "truncated V of section %d", i);
        off += 2 * vn;
        if (pools[i]->pages_for(s.len) > (int64_t)pools[i]->stack.size())
            return fail(GKV_ERR_NO_PAGES, "section %d needs %lld pages", i, (long long)pools[i]->pages_for(s.len));
    }
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    int32_t made = 0;
    int rc = GKV_OK;
    for (; made < n_layers && rc == GKV_OK; ++made) {
        gkv_pool *pool = pools[made];
        const Sec &s = secs[made];
        DeviceGuard guard(pool->cfg.device);
        uint16_t *dk = nullptr;
        cudaError_t e = cudaSuccess;
        if (s.n > 0) {
            e = cudaMalloc(&dk, sizeof(uint16_t) * 2 * s.n);
            if (e == cudaSuccess) e = cudaMemcpyAsync(dk, b + s.k_off, sizeof(uint16_t) * s.n, cudaMemcpyHostToDevice, st);
            if (e == cudaSuccess)
                e = cudaMemcpyAsync(dk + s.n, b + s.v_off, sizeof(uint16_t) * s.n, cudaMemcpyHostToDevice, st);
        }
        if (e != cudaSuccess) {
            rc = cuda_fail(e, "deserialize copy");
        } else {
            rc = gkv_from_compact(pool, dk, dk + s.n, s.len, &seq_ids_out[made], stream);
            const cudaError_t e2 = cudaStreamSynchronize(st);
            if (rc == GKV_OK && e2 != cudaSuccess) rc = cuda_fail(e2, "deserialize synchronize");
        }
        if (dk) cudaFree(dk);
        if (rc != GKV_OK) break;
        layer_ids_out[made] = (int32_t)s.layer;
    }
    if (rc != GKV_OK) {  // a failing call changes nothing: release what was made
        for (int32_t i = 0; i < made; ++i) gkv_seq_release(pools[i], seq_ids_out[i]);
        return rc;
    }
    if (consumed) *consumed = off;
    return GKV_OK;
}

int gkv_state_header(void *buf, int64_t cap, int64_t *size) {
    if (!size) return fail(GKV_ERR_INVALID, "null size");
    *size = 12;
    if (!buf) return GKV_OK;
    if (cap < 12) return fail(GKV_ERR_CAPACITY, "buffer of %lld bytes < 12", (long long)cap);
    uint8_t *p = static_cast<uint8_t *>(buf);
    memcpy(p, kStateMagic, 4);
    p += 4;
    put_i64(p, kStateVersion);
    return GKV_OK;
}

int gkv_state_read_header(const void *buf, int64_t size, int64_t *offset) {
    if (!buf || !offset) return fail(GKV_ERR_INVALID, "null argument");
    const uint8_t *b = static_cast<const uint8_t *>(buf);
    int64_t off = 4, version = 0;
    if (size < 12 || memcmp(b, kStateMagic, 4) != 0) return fail(GKV_ERR_INVALID, "not a GDNS state file");
    get_i64(b, size, off, &version);
    if (version != kStateVersion) return fail(GKV_ERR_INVALID, "GDNS version %lld", (long long)version);
    *offset = off;
    return GKV_OK;
}

}  // extern "C"
