/*
 * gadeon_kv.hpp -- header-only C++ layer over the gadeon_kv C ABI.
 *
 * It mirrors the reference's Swift interface for the paged KV path, so a
 * C++ host reads like the Swift call sites it replaces:
 *
 *   PagePool                 LLM/src/CoreML/PagedAttention.swift:21-287
 *     init(P:kvHeads:dh:)    :40      -> PagePool(BlockPool&)
 *     length, pageCount      :27, :79 -> length(), pageCount()
 *     append(k:v:)           :85-94   -> append(k, v)
 *     seed(K:V:count:)       :99-112  -> seed(K, V, count)
 *     truncate(to:)          :181-189 -> truncate(to)
 *     clone()                :199-210 -> clone()
 *     compact()              :225-252 -> compact() (host vectors)
 *     tileAt(_:_:_:)         :151-161 -> tileAt(start, count, tileP, K, V)
 *     kPage(_:), vPage(_:)   :80-81   -> kPage(i), vPage(i) (host vectors)
 *   MetalKVPool.snapshot() / restore(_:) (LLM/src/Metal/MetalKVPool.swift:102-120)
 *                                     -> snapshot(), restore(snap)
 *     floats32()             :46-62   -> floats32() (host vectors)
 *     fromCompact(k:v:length:P:kvHeads:dh:) :256-264
 *                                     -> PagePool::fromCompact(pool, k, v, length)
 *   hostFlashDecode(q:pool:G:)        :317-366 -> hostFlashDecode(q, pool, G, ...)
 *   Engine.rollbackGDN (LLM/src/CoreML/Engine.swift:2678-2716) for a batch
 *                                     -> rollbackGDN(...), fp16 state and conv tail
 *
 * The Swift PagePool owns its pages; here every PagePool is one sequence of
 * a BlockPool, the device-resident page store of one layer (the geometry
 * P / kvHeads / dh the Swift initializer takes is the BlockPool's).  Where
 * the Swift throws (page allocation, PagedAttention.swift:85, :99, :199,
 * :256) and wherever the C ABI returns a non-zero status, these wrappers
 * throw gadeon::Error carrying the status code and gkv_last_error().
 *
 * Buffers: fp16 values are passed as uint16_t bit patterns, like the
 * Swift's [UInt16] (compact / fromCompact).  Pointer arguments of append,
 * seed, hostFlashDecode and the batched BlockPool calls follow the C ABI:
 * device memory or page-locked host memory of the pool's device (read and
 * written in place), or plain host memory, which the library stages through
 * the pool's device memory.  compact() / fromCompact() and the
 * std::vector overload of hostFlashDecode take ordinary host memory.
 * Streams are cudaStream_t (nullptr = the legacy default stream).
 */
#ifndef GADEON_KV_HPP
#define GADEON_KV_HPP

#include <cuda_runtime_api.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "gadeon_kv.h"

namespace gadeon {

/* A failing C ABI call: code is its gkv_status, what() its message. */
struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string &msg) : std::runtime_error(msg), code(c) {}
};

inline void check(int rc) {
    if (rc != GKV_OK) throw Error(rc, gkv_last_error());
}

namespace detail {
/* IEEE binary16 bits -> binary32, exact (the widening floats32() does). */
inline float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu, bits;
    if (exp == 0x1fu) {
        bits = sign | 0x7f800000u | (man << 13);
    } else if (exp != 0) {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    } else if (man == 0) {
        bits = sign;
    } else {  // subnormal: normalise
        int e = -1;
        do {
            man <<= 1;
            ++e;
        } while (!(man & 0x400u));
        bits = sign | ((uint32_t)(112 - e) << 23) | ((man & 0x3ffu) << 13);
    }
    float f;
    std::memcpy(&f, &bits, sizeof f);
    return f;
}
}  // namespace detail

inline void check_cuda(cudaError_t e, const char *what) {
    if (e != cudaSuccess) throw Error(GKV_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

/* The page store of one layer: the physical K and V pages in HBM, the free
 * list and every sequence's block-table row (gkv_pool_create). */
class BlockPool {
public:
    explicit BlockPool(const gkv_pool_config &cfg) : cfg_(cfg) { check(gkv_pool_create(&cfg_, &h_)); }
    BlockPool(int kvHeads, int dh, int P, int numPages, int maxSeqs, int maxPagesPerSeq, int device = 0,
              uint64_t seed = 0)
        : BlockPool(gkv_pool_config{device, kvHeads, dh, P, numPages, maxSeqs, maxPagesPerSeq, seed}) {}
    ~BlockPool() {
        if (h_) gkv_pool_destroy(h_);
    }
    BlockPool(const BlockPool &) = delete;
    BlockPool &operator=(const BlockPool &) = delete;
    BlockPool(BlockPool &&o) noexcept : cfg_(o.cfg_), h_(o.h_) { o.h_ = nullptr; }
    BlockPool &operator=(BlockPool &&o) noexcept {
        if (this != &o) {
            if (h_) gkv_pool_destroy(h_);
            cfg_ = o.cfg_;
            h_ = o.h_;
            o.h_ = nullptr;
        }
        return *this;
    }

    gkv_pool *handle() const { return h_; }
    const gkv_pool_config &config() const { return cfg_; }
    int P() const { return cfg_.page_tokens; }
    int kvHeads() const { return cfg_.kv_heads; }
    int dh() const { return cfg_.head_dim; }
    int device() const { return cfg_.device; }
    int32_t freePageCount() const {
        int32_t n = 0;
        check(gkv_free_page_count(h_, &n));
        return n;
    }

    /* Batched forms of the per-sequence calls (one launch for the batch). */
    void append(const std::vector<int32_t> &ids, const std::vector<int32_t> &nNew, const void *k, const void *v,
                cudaStream_t s = nullptr) {
        same_size(ids.size(), nNew.size());
        check(gkv_append(h_, (int32_t)ids.size(), ids.data(), nNew.data(), k, v, s));
    }
    void attend(const std::vector<int32_t> &ids, int nQ, int G, const void *q, float *out, float scale,
                cudaStream_t s = nullptr) {
        check(gkv_attend(h_, (int32_t)ids.size(), ids.data(), nQ, G, q, out, scale, s));
    }
    void appendAttend(const std::vector<int32_t> &ids, int nQ, int G, const void *k, const void *v, const void *q,
                      float *out, float scale, cudaStream_t s = nullptr) {
        check(gkv_append_attend(h_, (int32_t)ids.size(), ids.data(), nQ, G, k, v, q, out, scale, s));
    }
    void truncate(const std::vector<int32_t> &ids, const std::vector<int64_t> &newLen) {
        same_size(ids.size(), newLen.size());
        check(gkv_truncate(h_, (int32_t)ids.size(), ids.data(), newLen.data()));
    }
    void rewindAppend(const std::vector<int32_t> &ids, const std::vector<int64_t> &baseLen,
                      const std::vector<int32_t> &nNew, const void *k, const void *v, cudaStream_t s = nullptr) {
        same_size(ids.size(), baseLen.size());
        same_size(ids.size(), nNew.size());
        check(gkv_rewind_append(h_, (int32_t)ids.size(), ids.data(), baseLen.data(), nNew.data(), k, v, s));
    }

private:
    static void same_size(size_t a, size_t b) {
        if (a != b) throw Error(GKV_ERR_INVALID, "batch arrays differ in length");
    }
    gkv_pool_config cfg_;
    gkv_pool *h_ = nullptr;
};

/* One sequence's cache in a BlockPool: the reference's PagePool.  The
 * sequence is released when the object is destroyed. */
class PagePool {
public:
    /* init(P:kvHeads:dh:) -- a new, empty sequence. */
    explicit PagePool(BlockPool &bp) : bp_(&bp) { check(gkv_seq_create(bp.handle(), &id_)); }
    /* Adopt an existing sequence id of bp (it is released with this object). */
    PagePool(BlockPool &bp, int32_t seqId) : bp_(&bp), id_(seqId) {}
    ~PagePool() {
        if (bp_ && id_ >= 0) gkv_seq_release(bp_->handle(), id_);
    }
    PagePool(const PagePool &) = delete;
    PagePool &operator=(const PagePool &) = delete;
    PagePool(PagePool &&o) noexcept : bp_(o.bp_), id_(o.id_) { o.id_ = -1; }
    PagePool &operator=(PagePool &&o) noexcept {
        if (this != &o) {
            if (bp_ && id_ >= 0) gkv_seq_release(bp_->handle(), id_);
            bp_ = o.bp_;
            id_ = o.id_;
            o.id_ = -1;
        }
        return *this;
    }

    BlockPool &blockPool() const { return *bp_; }
    int32_t seqId() const { return id_; }
    int P() const { return bp_->P(); }
    int kvHeads() const { return bp_->kvHeads(); }
    int dh() const { return bp_->dh(); }
    int64_t length() const {
        int64_t n = 0;
        check(gkv_seq_length(bp_->handle(), id_, &n));
        return n;
    }
    int32_t pageCount() const {
        int32_t n = 0;
        check(gkv_seq_page_count(bp_->handle(), id_, &n));
        return n;
    }

    /* append(k:v:) -- one position, k and v [kvHeads, dh] fp16. */
    void append(const void *k, const void *v, cudaStream_t s = nullptr) {
        const int32_t one = 1;
        check(gkv_append(bp_->handle(), 1, &id_, &one, k, v, s));
    }
    /* seed(K:V:count:) -- an empty sequence from [kvHeads, count, dh] fp16. */
    void seed(const void *K, const void *V, int64_t count, cudaStream_t s = nullptr) {
        check(gkv_seed(bp_->handle(), id_, K, V, count, s));
    }
    /* truncate(to:) -- host bookkeeping only; to > length() throws. */
    void truncate(int64_t to) {
        check(gkv_truncate(bp_->handle(), 1, &id_, &to));
    }
    /* clone() -- shares every full page, copies a partially filled tail. */
    PagePool clone(cudaStream_t s = nullptr) const {
        int32_t dst = -1;
        check(gkv_clone_seq(bp_->handle(), id_, &dst, s));
        return PagePool(*bp_, dst);
    }
    /* MetalKVPool.snapshot() (MetalKVPool.swift:102-109) -- clone(). */
    PagePool snapshot(cudaStream_t s = nullptr) const { return clone(s); }
    /* MetalKVPool.restore(_:) (:110-120) -- this sequence becomes a copy of
     * snap (shared full pages, its own tail copy); snap stays intact and may
     * be restored again.  The sequence id changes. */
    void restore(const PagePool &snap, cudaStream_t s = nullptr) {
        if (snap.bp_ != bp_) throw Error(GKV_ERR_INVALID, "restore: the snapshot belongs to another BlockPool");
        int32_t dst = -1;
        check(gkv_clone_seq(bp_->handle(), snap.id_, &dst, s));
        gkv_seq_release(bp_->handle(), id_);
        id_ = dst;
    }
    /* compact() -- (k, v) as [kvHeads, length, dh] fp16 in host vectors.
     * Reads the pool's pool section for this one sequence (gkv_serialize:
     * Int64 count, layer, length, n, K[n], n, V[n]) and unpacks it. */
    std::pair<std::vector<uint16_t>, std::vector<uint16_t>> compact(cudaStream_t s = nullptr) const {
        gkv_pool *h = bp_->handle();
        const int32_t layer = 0;
        int64_t size = 0;
        check(gkv_serialize(1, &h, &layer, &id_, nullptr, 0, &size, s));
        std::vector<uint8_t> buf((size_t)size);
        check(gkv_serialize(1, &h, &layer, &id_, buf.data(), size, &size, s));
        const int64_t n = get_i64(buf, 24);  // after count, layer, length
        std::vector<uint16_t> k((size_t)n), v((size_t)n);
        if (n > 0) {
            std::memcpy(k.data(), buf.data() + 32, (size_t)n * 2);
            std::memcpy(v.data(), buf.data() + 40 + n * 2, (size_t)n * 2);
        }
        return {std::move(k), std::move(v)};
    }
    /* tileAt(_:_:_:) -- positions [start, start + count) into head-major
     * [kvHeads, tileP, dh] fp16 tiles K and V (device or host memory),
     * rows count..tileP-1 zero. */
    void tileAt(int64_t start, int64_t count, int tileP, void *K, void *V, cudaStream_t s = nullptr) const {
        check(gkv_tile_at(bp_->handle(), id_, start, count, tileP, K, V, s));
    }
    /* kPage(_:) / vPage(_:) -- page i of the sequence as stored,
     * [kvHeads, P, dh] fp16 on the host (rows past length() included, as the
     * pool holds them).  Waits for the device. */
    std::vector<uint16_t> kPage(int i) const { return page(i).first; }
    std::vector<uint16_t> vPage(int i) const { return page(i).second; }
    /* floats32() -- per kv head, the sequence's rows widened to fp32:
     * k[h] and v[h] hold length() * dh values. */
    std::pair<std::vector<std::vector<float>>, std::vector<std::vector<float>>> floats32(
        cudaStream_t s = nullptr) const {
        const auto kv = compact(s);
        const size_t per = kv.first.size() / (size_t)kvHeads();
        std::vector<std::vector<float>> k((size_t)kvHeads()), v((size_t)kvHeads());
        for (int h = 0; h < kvHeads(); ++h) {
            k[h].resize(per);
            v[h].resize(per);
            for (size_t j = 0; j < per; ++j) {
                k[h][j] = detail::half_to_float(kv.first[h * per + j]);
                v[h][j] = detail::half_to_float(kv.second[h * per + j]);
            }
        }
        return {std::move(k), std::move(v)};
    }
    /* fromCompact(k:v:length:P:kvHeads:dh:) -- a new sequence of bp seeded
     * from host [kvHeads, length, dh] fp16 (through gkv_deserialize's pool
     * section reader, which takes host memory). */
    static PagePool fromCompact(BlockPool &bp, const std::vector<uint16_t> &k, const std::vector<uint16_t> &v,
                                int64_t length, cudaStream_t s = nullptr) {
        if (length < 0) throw Error(GKV_ERR_INVALID, "fromCompact: negative length");
        const int64_t n = (int64_t)bp.kvHeads() * length * bp.dh();
        if ((int64_t)k.size() != n || (int64_t)v.size() != n)
            throw Error(GKV_ERR_INVALID, "fromCompact: k/v hold " + std::to_string(k.size()) + "/" +
                                             std::to_string(v.size()) + " values, geometry needs " +
                                             std::to_string(n));
        std::vector<uint8_t> buf((size_t)(8 * 5 + 4 * n));
        uint8_t *p = buf.data();
        put_i64(p, 1);       // count
        put_i64(p, 0);       // layer
        put_i64(p, length);
        put_i64(p, n);
        if (n > 0) std::memcpy(p, k.data(), (size_t)n * 2);
        p += n * 2;
        put_i64(p, n);
        if (n > 0) std::memcpy(p, v.data(), (size_t)n * 2);
        gkv_pool *h = bp.handle();
        int32_t layer = 0, id = -1;
        int64_t used = 0;
        check(gkv_deserialize(1, &h, buf.data(), (int64_t)buf.size(), &layer, &id, &used, s));
        return PagePool(bp, id);
    }

private:
    std::pair<std::vector<uint16_t>, std::vector<uint16_t>> page(int i) const {
        const int32_t n = pageCount();
        if (i < 0 || i >= n)
            throw Error(GKV_ERR_INVALID, "page " + std::to_string(i) + " of a sequence with " + std::to_string(n) +
                                             " pages");
        std::vector<int32_t> table((size_t)n);
        int32_t got = 0;
        check(gkv_export_table(bp_->handle(), id_, table.data(), n, &got));
        const size_t elems = (size_t)kvHeads() * (size_t)P() * (size_t)dh();
        std::vector<uint16_t> k(elems), v(elems);
        check(gkv_export_page(bp_->handle(), table[(size_t)i], k.data(), v.data()));
        return {std::move(k), std::move(v)};
    }
    static void put_i64(uint8_t *&p, int64_t x) {
        for (int i = 0; i < 8; ++i) *p++ = (uint8_t)((uint64_t)x >> (8 * i));
    }
    static int64_t get_i64(const std::vector<uint8_t> &b, size_t off) {
        uint64_t x = 0;
        for (int i = 0; i < 8; ++i) x |= (uint64_t)b[off + i] << (8 * i);
        return (int64_t)x;
    }
    BlockPool *bp_;
    int32_t id_ = -1;
};

/* hostFlashDecode(q:pool:G:) -- the newest query, q [kvHeads, G, dh] fp16,
 * attending every one of the pool's length() keys with scale dh^-0.5;
 * out [kvHeads*G*dh] fp32 (head h = kvh*G + g).  q and out: device,
 * page-locked or plain host memory (plain host memory is staged by the
 * library, and the call then waits for the result).  An empty pool gives
 * zeros, as the Swift (:323). */
inline void hostFlashDecode(const void *q, const PagePool &pool, int G, float *out, cudaStream_t s = nullptr) {
    if (G <= 0) throw Error(GKV_ERR_INVALID, "hostFlashDecode: G must be positive");
    if (pool.length() == 0) {
        const size_t bytes = sizeof(float) * pool.kvHeads() * G * pool.dh();
        cudaPointerAttributes a{};
        if (cudaPointerGetAttributes(&a, out) == cudaSuccess && a.type == cudaMemoryTypeUnregistered) {
            std::memset(out, 0, bytes);
        } else {
            cudaGetLastError();
            check_cuda(cudaMemsetAsync(out, 0, bytes, s), "zero output");
        }
        return;
    }
    const int32_t id = pool.seqId();
    check(gkv_attend(pool.blockPool().handle(), 1, &id, 1, G, q, out, (float)std::pow((double)pool.dh(), -0.5), s));
}

/* The Swift's value-returning form: host q in, host [Float] out.  The
 * vectors are plain (pageable) host memory, which the library stages
 * through the pool's device memory; the call waits for the result. */
inline std::vector<float> hostFlashDecode(const std::vector<uint16_t> &q, const PagePool &pool, int G) {
    const size_t nq = (size_t)pool.kvHeads() * (size_t)G * (size_t)pool.dh();
    if (G <= 0 || q.size() != nq) throw Error(GKV_ERR_INVALID, "hostFlashDecode: q must hold kvHeads*G*dh values");
    std::vector<float> out(nq);  // zeros: an empty pool's result (PagedAttention.swift:323)
    if (pool.length() > 0) hostFlashDecode(q.data(), pool, G, out.data(), nullptr);
    return out;
}

/* Engine.rollbackGDN for a batch of (sequence, GDN layer) items with the
 * reference's fp16 storage: each item's recurrent state [H, DK, DV] rolled
 * back to its accepted prefix m[i] (MtpRollback.stateAfter) and its conv
 * tail [convDim, taps] rebuilt (convFromProj), in one launch where the
 * shapes allow (gkv_gdn_rollback_f16).  m is a host array of nItems values
 * in 1..C; every other pointer is device memory. */
inline void rollbackGDN(int32_t nItems, const int32_t *m, int32_t H, int32_t DK, int32_t DV, int32_t C,
                        const void *s0, const float *delta, const float *k, const float *gcum, void *stateOut,
                        int32_t convDim, int32_t taps, const float *proj, const void *pre, void *convOut,
                        cudaStream_t s = nullptr) {
    check(gkv_gdn_rollback_f16(nItems, m, H, DK, DV, C, s0, delta, k, gcum, stateOut, convDim, taps, proj, pre,
                               convOut, s));
}
/* The same for an engine that keeps fp32 state and conv tail (gkv_gdn_rollback). */
inline void rollbackGDN(int32_t nItems, const int32_t *m, int32_t H, int32_t DK, int32_t DV, int32_t C,
                        const float *s0, const float *delta, const float *k, const float *gcum, float *stateOut,
                        int32_t convDim, int32_t taps, const float *proj, const float *pre, float *convOut,
                        cudaStream_t s = nullptr) {
    check(gkv_gdn_rollback(nItems, m, H, DK, DV, C, s0, delta, k, gcum, stateOut, convDim, taps, proj, pre, convOut,
                           s));
}

}  // namespace gadeon

#endif /* GADEON_KV_HPP */
