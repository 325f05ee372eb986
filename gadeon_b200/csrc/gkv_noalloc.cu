// gkv_noalloc.cu -- gkv_attend_noalloc: paged GQA decode / verify attention
// over caller-owned device memory that allocates nothing.
//
// Who needs it: callers that own every device byte themselves and may not
// call cudaMalloc while serving -- an engine that reserves one arena at
// start-up (a cudaMalloc later can synchronise the whole device, or fail
// once the arena holds nearly all of HBM), or a host-language binding whose
// device memory comes from its own allocator.  They keep the K/V pages and
// block tables in their own buffers and still get this library's attention
// kernel.
//
// The kernel's scratch -- a status word, the split-K merge counters and the
// split-K partial results -- lives in one file-scope __device__ array of
// GKV_NOALLOC_SCRATCH_BYTES.  Every GPU that loads the library holds that
// array until the process exits.  All calls share it and it keeps the last
// call's contents: each call clears the merge counters (they must start at
// zero); the status word collects error bits until gkv_noalloc_status reads
// and clears it.  Calls whose work overlaps on the GPU (two streams, or two
// host threads) race on the array.
//
// The per-call work descriptor travels in the kernel's parameter block
// (InlineDesc), so a call copies nothing from the host: a batch of more
// than kInlineSeqs sequences, or one whose partial results would not fit
// the array, runs as several launches of at most kInlineSeqs sequences on
// the caller's stream, one after another, each reusing the whole array.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "gadeon_kv.h"
#include "gkv_kernels.cuh"

namespace {

__device__ __align__(256) unsigned char g_noalloc_scratch[GKV_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
// The launch grid is capped at what the attend kernel would use on a
// 148-SM B200, whatever the GPU, so which calls fit the array does not
// depend on the SM count.
constexpr int kGridSms = 148;
// Layout of the array: [status word][merge counters][partials].
constexpr size_t kOffStatus = 0;
constexpr size_t kOffCounters = 256;
constexpr size_t kCounterBytes = sizeof(int32_t) * gkv::kInlineSeqs * GKV_NOALLOC_MAX_KV_HEADS;
constexpr size_t kOffPartials = kOffCounters + ((kCounterBytes + 255) & ~size_t(255));

struct DeviceScratch {
    bool ready = false;
    unsigned char *ptr = nullptr;  // device address of g_noalloc_scratch
    int sm_count = 0;
};

DeviceScratch g_dev[kMaxDevices];
std::mutex g_mu;

// Host code may not hand g_noalloc_scratch itself to a kernel: in host code
// that name is a host-side stand-in, not a device address.  Resolve the real
// address once per device, with that device current.
int scratch_for_current_device(DeviceScratch **out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return gkv::report_error(GKV_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return gkv::report_error(GKV_ERR_INVALID, "device %d", dev);
    std::lock_guard<std::mutex> lock(g_mu);
    DeviceScratch &d = g_dev[dev];
    if (!d.ready) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess)
            return gkv::report_error(GKV_ERR_CUDA, "cudaGetSymbolAddress(noalloc scratch): %s",
                                     cudaGetErrorString(e));
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess)
            return gkv::report_error(GKV_ERR_CUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
        d.ptr = static_cast<unsigned char *>(p);
        d.sm_count = sms;
        d.ready = true;
    }
    *out = &d;
    return GKV_OK;
}

}  // namespace

extern "C" int gkv_attend_noalloc(const void *k_pages, const void *v_pages, int32_t num_pages,
                                  int32_t kv_heads, int32_t head_dim, int32_t page_tokens,
                                  const int32_t *block_table, int32_t table_stride, int32_t n_seqs,
                                  const int32_t *seq_lens, int32_t n_q, int32_t group,
                                  const void *q, float *out, float scale, void *stream) {
    using gkv::report_error;
    if (head_dim != 64 && head_dim != 128 && head_dim != 256 && head_dim != 512)
        return report_error(GKV_ERR_UNSUPPORTED, "head_dim=%d (64/128/256/512)", head_dim);
    if (page_tokens <= 0 || (page_tokens & (page_tokens - 1)) || page_tokens > 16384)
        return report_error(GKV_ERR_INVALID, "page_tokens=%d (power of two <= 16384)", page_tokens);
    if (kv_heads < 1 || num_pages < 1 || table_stride < 1)
        return report_error(GKV_ERR_INVALID, "kv_heads/num_pages/table_stride must be >= 1");
    if (kv_heads > GKV_NOALLOC_MAX_KV_HEADS)
        return report_error(GKV_ERR_CAPACITY, "kv_heads=%d exceeds the no-alloc limit of %d", kv_heads,
                            GKV_NOALLOC_MAX_KV_HEADS);
    if ((int64_t)num_pages * kv_heads * page_tokens >= INT32_MAX)
        return report_error(GKV_ERR_CAPACITY, "num_pages*kv_heads*page_tokens rows exceed 2^31");
    if (n_q < 1 || group < 1) return report_error(GKV_ERR_INVALID, "n_q=%d group=%d", n_q, group);
    if ((int64_t)n_q * group > 16)
        return report_error(GKV_ERR_UNSUPPORTED, "n_q*group = %d query rows per kv head (max 16)",
                            n_q * group);
    if (!(std::isfinite(scale) && scale != 0.f))
        return report_error(GKV_ERR_INVALID, "scale must be finite and non-zero");
    if (n_seqs < 0 || (n_seqs > 0 && !seq_lens))
        return report_error(GKV_ERR_INVALID, "bad batch (n_seqs=%d)", n_seqs);
    if (n_seqs > GKV_NOALLOC_MAX_SEQS)
        return report_error(GKV_ERR_CAPACITY, "n_seqs=%d exceeds the no-alloc limit of %d sequences",
                            n_seqs, GKV_NOALLOC_MAX_SEQS);
    if (n_seqs == 0) return GKV_OK;
    if (!k_pages || !v_pages || !block_table || !q || !out)
        return report_error(GKV_ERR_INVALID, "null device pointer");
    for (const void *ptr : {k_pages, v_pages, q, static_cast<const void *>(out)})
        if (reinterpret_cast<uintptr_t>(ptr) & 15)
            return report_error(GKV_ERR_INVALID, "k_pages/v_pages/q/out must be 16-byte aligned");
    {  // every buffer must be device (or managed) memory of the current GPU
        const void *bufs[5] = {k_pages, v_pages, block_table, q, out};
        const char *names[5] = {"k_pages", "v_pages", "block_table", "q", "out"};
        for (int i = 0; i < 5; ++i)
            if (const int rc = gkv::check_reachable(bufs[i], -1, false, names[i])) return rc;
    }
    for (int32_t i = 0; i < n_seqs; ++i) {
        const int64_t len = seq_lens[i];
        if (len < n_q || len > (int64_t)table_stride * page_tokens)
            return report_error(GKV_ERR_BAD_SEQ, "seq_lens[%d]=%lld (need n_q=%d <= len <= %lld)", i,
                                (long long)len, n_q, (long long)table_stride * page_tokens);
    }

    DeviceScratch *d = nullptr;
    int rc = scratch_for_current_device(&d);
    if (rc) return rc;
    // Sequences per launch: the descriptor fits the parameter block, and the
    // partials (one slot per (sequence, kv head) plus one per CTA) fit the
    // array.
    const int64_t pf_bytes = (int64_t)sizeof(float) * gkv::attend_partial_floats(head_dim);
    const int64_t slots = (int64_t)(GKV_NOALLOC_SCRATCH_BYTES - kOffPartials) / pf_bytes;
    const int grid_cap = gkv::attend_grid(head_dim, page_tokens, INT32_MAX, std::min(d->sm_count, kGridSms));
    const int64_t per_launch = std::min<int64_t>(gkv::kInlineSeqs, (slots - grid_cap) / kv_heads);
    if (per_launch < 1)
        return report_error(GKV_ERR_CAPACITY,
                            "kv_heads=%d at head_dim=%d needs more scratch than the static no-alloc array "
                            "holds (%u bytes)",
                            kv_heads, head_dim, (unsigned)GKV_NOALLOC_SCRATCH_BYTES);

    CUtensorMap tmk{}, tmv{};
    if (page_tokens >= 8) {
        rc = gkv::encode_page_tensor_map(&tmk, k_pages, num_pages, kv_heads, page_tokens, head_dim);
        if (rc) return rc;
        rc = gkv::encode_page_tensor_map(&tmv, v_pages, num_pages, kv_heads, page_tokens, head_dim);
        if (rc) return rc;
    }
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    // the merge counters start at zero (a launch cut short by a bounded
    // wait could leave some set); the status word is left as it is
    cudaError_t e = cudaMemsetAsync(d->ptr + kOffCounters, 0, kCounterBytes, st);
    if (e != cudaSuccess) return report_error(GKV_ERR_CUDA, "gkv_attend_noalloc: %s", cudaGetErrorString(e));

    const int TK = gkv::attend_tile_keys(head_dim);
    const int64_t nH = (int64_t)kv_heads * group;
    gkv::InlineDesc desc;
    for (int32_t b0 = 0; b0 < n_seqs; b0 += (int32_t)per_launch) {
        const int32_t nb = (int32_t)std::min<int64_t>(per_launch, n_seqs - b0);
        int64_t units = 0;
        for (int32_t i = 0; i < nb; ++i) {
            const int32_t len = seq_lens[b0 + i];
            const int32_t ntiles = (len + TK - 1) / TK;
            // seq_id = the row of the caller's block table
            desc.entries[i] = {b0 + i, len, (int32_t)units, ntiles};
            units += (int64_t)kv_heads * ntiles;
        }
        if (units > INT32_MAX) return report_error(GKV_ERR_CAPACITY, "too many key tiles in one launch");
        const int grid = std::min(gkv::attend_grid(head_dim, page_tokens, (int)units, d->sm_count), grid_cap);
        gkv::AttendParams p{};
        p.entries = nullptr;  // the inline descriptor
        p.n_seqs = nb;
        p.total_units = (int32_t)units;
        p.table = block_table;
        p.table_stride = table_stride;
        p.k_pool = static_cast<const uint16_t *>(k_pages);
        p.v_pool = static_cast<const uint16_t *>(v_pages);
        // the kernel indexes q and out by the batch entry within this launch
        p.q = static_cast<const uint16_t *>(q) + (int64_t)b0 * n_q * nH * head_dim;
        p.out = out + (int64_t)b0 * n_q * nH * head_dim;
        p.status = reinterpret_cast<int32_t *>(d->ptr + kOffStatus);
        p.counters = reinterpret_cast<int32_t *>(d->ptr + kOffCounters);
        p.partials = reinterpret_cast<float *>(d->ptr + kOffPartials);
        p.n_q = n_q;
        p.G = group;
        p.kvh = kv_heads;
        p.P = page_tokens;
        p.num_pages = num_pages;
        p.scale_log2 = scale * 1.4426950408889634f;
        e = gkv::launch_attend(p, &tmk, &tmv, head_dim, grid, st, &desc);
        if (e != cudaSuccess)
            return report_error(GKV_ERR_CUDA, "gkv_attend_noalloc: %s", cudaGetErrorString(e));
    }
    return GKV_OK;
}

extern "C" int gkv_noalloc_status(void *stream, int32_t *status) {
    using gkv::report_error;
    if (!status) return report_error(GKV_ERR_INVALID, "null status");
    DeviceScratch *d = nullptr;
    const int rc = scratch_for_current_device(&d);
    if (rc) return rc;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    int32_t word = 0;
    // in stream order after the caller's launches: read the word, clear it
    cudaError_t e = cudaMemcpyAsync(&word, d->ptr + kOffStatus, sizeof(word), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(d->ptr + kOffStatus, 0, sizeof(word), st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return report_error(GKV_ERR_CUDA, "gkv_noalloc_status: %s", cudaGetErrorString(e));
    *status = word;
    return GKV_OK;
}
