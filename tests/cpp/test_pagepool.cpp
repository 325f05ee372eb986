// C++ parity test of include/gadeon_kv.hpp against the CPU oracle
// (oracle/gkv_oracle.c, the restatement of PagePool and hostFlashDecode,
// LLM/src/CoreML/PagedAttention.swift:21-366).  Built and run by
// tests/test_cpp_layer.py: compiled in the CPU suite, run on a B200 in the
// GPU suite.  Exits 0 when every check passes.
//
// The scenario follows the reference's own use of one layer's pool in a
// decode session (Engine.swift): seed from a prefill, per-token append +
// hostFlashDecode across page boundaries, a clone (snapshot) that grows
// while the original is truncated (speculative rollback), compact /
// fromCompact round trips, and the throwing paths.
#include "gadeon_kv.hpp"

#include <cuda_runtime_api.h>

#include <cmath>
#include <cstdio>
#include <algorithm>
#include <cstdlib>
#include <vector>

extern "C" {
typedef struct OrcPool OrcPool;
OrcPool *orc_pool_create(int kv_heads, int head_dim, int page_tokens, int num_pages, uint64_t seed);
void orc_pool_destroy(OrcPool *p);
int orc_seq_create(OrcPool *p);
int orc_seed(OrcPool *p, int seq, const uint16_t *K, const uint16_t *V, int64_t count);
int orc_append(OrcPool *p, int n, const int32_t *seq_ids, const int32_t *n_new, const uint16_t *k,
               const uint16_t *v);
int orc_truncate(OrcPool *p, int n, const int32_t *seq_ids, const int64_t *new_len);
int orc_clone(OrcPool *p, int src);
int orc_seq_release(OrcPool *p, int seq);
int orc_compact(OrcPool *p, int seq, uint16_t *K, uint16_t *V);
int orc_tile_at(OrcPool *p, int seq, int64_t start, int64_t count, int tile_p, uint16_t *K, uint16_t *V);
int orc_from_compact(OrcPool *p, const uint16_t *K, const uint16_t *V, int64_t length);
int64_t orc_seq_length(OrcPool *p, int seq);
int32_t orc_seq_pages(OrcPool *p, int seq, int32_t *out);
int32_t orc_free_list(OrcPool *p, int32_t *out);
const uint16_t *orc_page_k(OrcPool *p, int32_t pid);
const uint16_t *orc_page_v(OrcPool *p, int32_t pid);
int orc_flash_decode(OrcPool *p, int seq, const uint16_t *q, int G, float scale, float *out);
void orc_fill_normal_f16(uint64_t seed, uint64_t stream, uint16_t *out, int64_t n);
}

static int g_failures = 0;
#define CHECK(cond, ...)                                          \
    do {                                                          \
        if (!(cond)) {                                            \
            ++g_failures;                                         \
            std::fprintf(stderr, "FAIL %s:%d: ", __FILE__, __LINE__); \
            std::fprintf(stderr, __VA_ARGS__);                    \
            std::fprintf(stderr, "\n");                           \
        }                                                         \
    } while (0)

namespace {

const int KVH = 2, DH = 128, P = 16, PAGES = 96, G = 4;
const uint64_t SEED = 1234;

std::vector<uint16_t> normal(uint64_t stream, size_t n) {
    std::vector<uint16_t> x(n);
    orc_fill_normal_f16(SEED, stream, x.data(), (int64_t)n);
    return x;
}

// A device copy of a host vector.
template <class T>
struct Dev {
    T *p = nullptr;
    explicit Dev(const std::vector<T> &h) {
        gadeon::check_cuda(cudaMalloc((void **)&p, h.size() * sizeof(T) + 16), "cudaMalloc");
        gadeon::check_cuda(cudaMemcpy(p, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice), "copy");
    }
    explicit Dev(size_t n) { gadeon::check_cuda(cudaMalloc((void **)&p, n * sizeof(T) + 16), "cudaMalloc"); }
    ~Dev() { cudaFree(p); }
    std::vector<T> host(size_t n) const {
        std::vector<T> h(n);
        gadeon::check_cuda(cudaMemcpy(h.data(), p, n * sizeof(T), cudaMemcpyDeviceToHost), "copy");
        return h;
    }
};

// The attention tolerance of the path (fp16 storage, fp32 accumulation),
// element-wise against the oracle: |got - want| <= 2e-3 everywhere, and
// <= 1e-2 * |want| wherever |want| >= 2e-3.
void check_attn(const std::vector<float> &got, const std::vector<float> &want, const char *what) {
    double max_abs = 0, max_rel = 0;
    bool finite = true;
    for (size_t i = 0; i < want.size(); ++i) {
        if (!std::isfinite(got[i])) finite = false;
        const double d = std::fabs((double)got[i] - want[i]);
        max_abs = std::fmax(max_abs, d);
        if (std::fabs(want[i]) >= 2e-3) max_rel = std::fmax(max_rel, d / std::fabs((double)want[i]));
    }
    CHECK(finite && max_abs <= 2e-3 && max_rel <= 1e-2, "%s: max-abs %.3e max-rel %.3e", what, max_abs, max_rel);
}

std::vector<int32_t> gpu_table(const gadeon::PagePool &s) {
    std::vector<int32_t> t(64);
    int32_t n = 0;
    gadeon::check(gkv_export_table(s.blockPool().handle(), s.seqId(), t.data(), (int32_t)t.size(), &n));
    t.resize(n);
    return t;
}

std::vector<int32_t> orc_table(OrcPool *o, int seq) {
    std::vector<int32_t> t(64);
    t.resize(orc_seq_pages(o, seq, t.data()));
    return t;
}

void check_state(const gadeon::PagePool &s, OrcPool *o, int oseq, const char *what) {
    CHECK(s.length() == orc_seq_length(o, oseq), "%s: length %lld vs %lld", what, (long long)s.length(),
          (long long)orc_seq_length(o, oseq));
    CHECK(gpu_table(s) == orc_table(o, oseq), "%s: block tables differ", what);
    CHECK(s.pageCount() == (int32_t)orc_table(o, oseq).size(), "%s: page count", what);
    auto kv = s.compact();
    std::vector<uint16_t> ok(kv.first.size()), ov(kv.second.size());
    orc_compact(o, oseq, ok.data(), ov.data());
    CHECK(kv.first == ok && kv.second == ov, "%s: compact() not bit-exact", what);
}

void check_free_list(const gadeon::BlockPool &bp, OrcPool *o, const char *what) {
    std::vector<int32_t> g(PAGES), w(PAGES);
    int32_t n = 0;
    gadeon::check(gkv_export_free_list(bp.handle(), g.data(), PAGES, &n));
    g.resize(n);
    w.resize(orc_free_list(o, w.data()));
    CHECK(g == w, "%s: free lists differ (%zu vs %zu pages)", what, g.size(), w.size());
}

void check_decode(const gadeon::PagePool &s, OrcPool *o, int oseq, uint64_t stream, const char *what) {
    const size_t nq = (size_t)KVH * G * DH;
    auto q = normal(stream, nq);
    std::vector<float> want(nq);
    orc_flash_decode(o, oseq, q.data(), G, (float)std::pow((double)DH, -0.5), want.data());
    Dev<uint16_t> dq(q);
    Dev<float> dout(nq);
    gadeon::hostFlashDecode(dq.p, s, G, dout.p);
    check_attn(dout.host(nq), want, what);
    check_attn(gadeon::hostFlashDecode(q, s, G), want, what);  // the value-returning form
}

template <class F>
int thrown_code(F f) {
    try {
        f();
    } catch (const gadeon::Error &e) {
        return e.code;
    }
    return GKV_OK;
}

void run() {
    gadeon::BlockPool bp(KVH, DH, P, PAGES, 8, 64, 0, SEED);
    OrcPool *o = orc_pool_create(KVH, DH, P, PAGES, SEED);
    CHECK(bp.P() == P && bp.kvHeads() == KVH && bp.dh() == DH, "geometry");

    // an empty pool decodes to zeros (hostFlashDecode returns early on n == 0)
    {
        gadeon::PagePool e(bp);
        auto z = gadeon::hostFlashDecode(std::vector<uint16_t>((size_t)KVH * G * DH, 0x3c00), e, G);
        bool zero = true;
        for (float x : z) zero = zero && x == 0.0f;
        CHECK(zero, "empty pool: hostFlashDecode not all zeros");
    }

    // seed(K:V:count:) from a 37-token prefill, then decode 30 tokens
    gadeon::PagePool a(bp);
    const int oa = orc_seq_create(o);
    CHECK(a.seqId() == oa, "sequence ids %d vs %d", a.seqId(), oa);
    const int64_t prefill = 37;
    auto K = normal(1, (size_t)KVH * prefill * DH), V = normal(2, (size_t)KVH * prefill * DH);
    {
        Dev<uint16_t> dK(K), dV(V);
        a.seed(dK.p, dV.p, prefill);
        cudaDeviceSynchronize();
    }
    orc_seed(o, oa, K.data(), V.data(), prefill);
    check_state(a, o, oa, "after seed");
    check_decode(a, o, oa, 100, "decode after seed");
    for (int t = 0; t < 30; ++t) {
        auto k = normal(200 + t, (size_t)KVH * DH), v = normal(300 + t, (size_t)KVH * DH);
        Dev<uint16_t> dk(k), dv(v);
        a.append(dk.p, dv.p);
        const int32_t one = 1;
        orc_append(o, 1, &oa, &one, k.data(), v.data());
        if (t % 7 == 0 || t == 29) {
            char what[64];
            std::snprintf(what, sizeof what, "decode at length %lld", (long long)a.length());
            check_decode(a, o, oa, 400 + t, what);
        }
    }
    check_state(a, o, oa, "after appends");
    check_free_list(bp, o, "after appends");

    // clone() of a partial tail, the clone grows, the original rolls back
    gadeon::PagePool b = a.clone();
    int ob = orc_clone(o, oa);
    CHECK(b.seqId() == ob, "clone ids %d vs %d", b.seqId(), ob);
    for (int t = 0; t < 12; ++t) {
        auto k = normal(500 + t, (size_t)KVH * DH), v = normal(600 + t, (size_t)KVH * DH);
        Dev<uint16_t> dk(k), dv(v);
        b.append(dk.p, dv.p);
        const int32_t one = 1;
        orc_append(o, 1, &ob, &one, k.data(), v.data());
    }
    a.truncate(40);
    const int64_t to = 40;
    orc_truncate(o, 1, &oa, &to);
    check_state(a, o, oa, "original after truncate");
    check_state(b, o, ob, "clone after appends");
    check_decode(a, o, oa, 700, "decode after truncate");
    check_decode(b, o, ob, 701, "decode of the clone");
    check_free_list(bp, o, "after clone + truncate");

    // tileAt over the carry windows of pagedFlashCarry (start = i*tileP,
    // count = min(tileP, length - start)), bit for bit
    for (int tileP : {8, 32}) {
        const int64_t n = b.length();
        const size_t elems = (size_t)KVH * tileP * DH;
        Dev<uint16_t> tk(elems), tv(elems);
        std::vector<uint16_t> ok(elems), ov(elems);
        for (int64_t start = 0; start < n; start += tileP) {
            const int64_t count = std::min<int64_t>(tileP, n - start);
            b.tileAt(start, count, tileP, tk.p, tv.p);
            orc_tile_at(o, ob, start, count, tileP, ok.data(), ov.data());
            CHECK(tk.host(elems) == ok && tv.host(elems) == ov, "tileAt(%lld, %lld, %d) not bit-exact",
                  (long long)start, (long long)count, tileP);
        }
        CHECK(thrown_code([&] { b.tileAt(n - 1, 2, tileP, tk.p, tv.p); }) == GKV_ERR_BAD_SEQ,
              "tileAt past the end");
    }

    // kPage / vPage: the pages as stored; floats32: compact() widened
    {
        const auto table = orc_table(o, ob);
        for (int i = 0; i < b.pageCount(); i += 2) {
            const uint16_t *wk = orc_page_k(o, table[(size_t)i]), *wv = orc_page_v(o, table[(size_t)i]);
            const size_t elems = (size_t)KVH * P * DH;
            CHECK(b.kPage(i) == std::vector<uint16_t>(wk, wk + elems) &&
                      b.vPage(i) == std::vector<uint16_t>(wv, wv + elems),
                  "kPage/vPage(%d) not the stored page", i);
        }
        CHECK(thrown_code([&] { b.kPage(b.pageCount()); }) == GKV_ERR_INVALID, "kPage past the last page");
        const auto f = b.floats32();
        const auto c = b.compact();
        const size_t per = (size_t)b.length() * DH;
        bool same = f.first.size() == (size_t)KVH && f.first[1].size() == per;
        for (size_t j = 0; same && j < per; ++j)
            same = f.first[1][j] == gadeon::detail::half_to_float(c.first[per + j]) &&
                   f.second[0][j] == gadeon::detail::half_to_float(c.second[j]);
        CHECK(same, "floats32() is not compact() widened");
    }

    // MetalKVPool.snapshot / restore: a restore leaves the snapshot intact
    {
        gadeon::PagePool snap = b.snapshot();
        const int osnap = orc_clone(o, ob);
        CHECK(snap.seqId() == osnap, "snapshot ids %d vs %d", snap.seqId(), osnap);
        auto k = normal(900, (size_t)KVH * DH), v = normal(901, (size_t)KVH * DH);
        Dev<uint16_t> dk(k), dv(v);
        b.append(dk.p, dv.p);
        const int32_t one = 1;
        orc_append(o, 1, &ob, &one, k.data(), v.data());
        const int old = b.seqId();
        b.restore(snap);
        const int nb = orc_clone(o, osnap);
        orc_seq_release(o, old);
        CHECK(b.seqId() == nb, "restore ids %d vs %d", b.seqId(), nb);
        ob = nb;
        check_state(b, o, nb, "after restore");
        check_state(snap, o, osnap, "snapshot after restore");
        check_free_list(bp, o, "after restore");
        orc_seq_release(o, osnap);  // snap's destructor releases it on the GPU side
    }
    check_free_list(bp, o, "after the snapshot is released");

    // compact() -> fromCompact round trip
    auto kv = b.compact();
    gadeon::PagePool c = gadeon::PagePool::fromCompact(bp, kv.first, kv.second, b.length());
    const int oc = orc_from_compact(o, kv.first.data(), kv.second.data(), (int64_t)kv.first.size() / (KVH * DH));
    CHECK(c.seqId() == oc, "fromCompact ids %d vs %d", c.seqId(), oc);
    check_state(c, o, oc, "fromCompact");
    check_decode(c, o, oc, 800, "decode after fromCompact");
    gadeon::PagePool empty = gadeon::PagePool::fromCompact(bp, {}, {}, 0);
    CHECK(empty.length() == 0 && empty.pageCount() == 0, "fromCompact of length 0");

    // the throwing paths; each leaves the pool as it was
    const int32_t free_before = bp.freePageCount();
    CHECK(thrown_code([&] { a.truncate(a.length() + 1); }) == GKV_ERR_BAD_SEQ, "truncate past the end");
    CHECK(thrown_code([&] { gadeon::PagePool::fromCompact(bp, kv.first, kv.second, b.length() + 1); }) ==
              GKV_ERR_INVALID,
          "fromCompact with too few values");
    {
        Dev<uint16_t> dK(K), dV(V);
        CHECK(thrown_code([&] { a.seed(dK.p, dV.p, prefill); }) == GKV_ERR_BAD_SEQ, "seed of a non-empty sequence");
    }
    {
        const int64_t too_long = (int64_t)(PAGES + 1) * P;
        std::vector<uint16_t> big((size_t)KVH * too_long * DH, 0);
        CHECK(thrown_code([&] { gadeon::PagePool::fromCompact(bp, big, big, too_long); }) == GKV_ERR_NO_PAGES,
              "fromCompact beyond the free pages");
    }
    CHECK(bp.freePageCount() == free_before, "a refused call changed the free list");
    check_state(a, o, oa, "after refused calls");

    // plain (pageable) host arrays: the library stages them through device
    // memory, and the append lands as from device buffers
    {
        std::vector<uint16_t> kp = normal(901, (size_t)KVH * DH), vp = normal(902, (size_t)KVH * DH);
        a.append(kp.data(), vp.data());
        int32_t id = oa, one = 1;
        CHECK(orc_append(o, 1, &id, &one, kp.data(), vp.data()) == 0, "oracle append");
        check_state(a, o, oa, "after an append from pageable host memory");
        check_decode(a, o, oa, 903, "decode after an append from pageable host memory");
    }

    // release (destructors, last page first) returns every page
    {
        gadeon::PagePool moved = std::move(c);
        CHECK(c.seqId() == -1, "moved-from PagePool keeps its id");
    }
    orc_seq_release(o, oc);
    check_free_list(bp, o, "after releasing the fromCompact sequence");
    orc_pool_destroy(o);
}

}  // namespace

int main() {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        std::fprintf(stderr, "no CUDA device\n");
        return 2;
    }
    try {
        run();
    } catch (const gadeon::Error &e) {
        std::fprintf(stderr, "unexpected gadeon::Error %d: %s\n", e.code, e.what());
        return 1;
    }
    if (g_failures) {
        std::fprintf(stderr, "%d check(s) failed\n", g_failures);
        return 1;
    }
    std::printf("test_pagepool: all checks passed\n");
    return 0;
}
