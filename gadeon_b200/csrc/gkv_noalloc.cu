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
// The kernel's scratch -- the per-call work descriptor, the split-K partial
// results, the merge counters and a status word -- lives in one file-scope
// __device__ array of GKV_NOALLOC_SCRATCH_BYTES.  Every GPU that loads the
// library holds that array until the process exits.  All calls share it and
// it keeps the last call's contents, so each call clears the parts that must
// start at zero (counters, status); calls whose work overlaps on the GPU
// (two streams, or two host threads) race on it.
#include <cuda_runtime.h>

#include <mutex>

#include "gadeon_kv.h"
#include "gkv_kernels.cuh"

namespace {

__device__ __align__(256) unsigned char g_noalloc_scratch[GKV_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;

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

size_t round256(size_t x) { return (x + 255) & ~size_t(255); }

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
    if ((int64_t)num_pages * kv_heads * page_tokens >= INT32_MAX)
        return report_error(GKV_ERR_CAPACITY, "num_pages*kv_heads*page_tokens rows exceed 2^31");
    if (n_q < 1 || group < 1) return report_error(GKV_ERR_INVALID, "n_q=%d group=%d", n_q, group);
    if ((int64_t)n_q * group > 16)
        return report_error(GKV_ERR_UNSUPPORTED, "n_q*group = %d query rows per kv head (max 16)",
                            n_q * group);
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

    // Work descriptor on the host stack: no heap, no device allocation.
    gkv::AttendEntry entries[GKV_NOALLOC_MAX_SEQS];
    const int TK = gkv::attend_tile_keys(head_dim);
    int64_t units = 0;
    for (int32_t i = 0; i < n_seqs; ++i) {
        const int64_t len = seq_lens[i];
        if (len < n_q || len > (int64_t)table_stride * page_tokens)
            return report_error(GKV_ERR_BAD_SEQ, "seq_lens[%d]=%lld (need n_q=%d <= len <= %lld)", i,
                                (long long)len, n_q, (long long)table_stride * page_tokens);
        const int32_t ntiles = (int32_t)((len + TK - 1) / TK);
        entries[i] = {i, (int32_t)len, (int32_t)units, ntiles};
        units += (int64_t)kv_heads * ntiles;
        if (units > INT32_MAX) return report_error(GKV_ERR_CAPACITY, "too many key tiles in one call");
    }

    DeviceScratch *d = nullptr;
    int rc = scratch_for_current_device(&d);
    if (rc) return rc;
    const int grid = gkv::attend_grid(head_dim, page_tokens, (int)units, d->sm_count);
    const size_t items = (size_t)n_seqs * kv_heads;
    const size_t off_status = round256(sizeof(gkv::AttendEntry) * n_seqs);
    const size_t off_counters = off_status + 256;
    const size_t off_partials = off_counters + round256(sizeof(int32_t) * items);
    const size_t need =
        off_partials + sizeof(float) * (items + grid) * gkv::attend_partial_floats(head_dim);
    if (need > GKV_NOALLOC_SCRATCH_BYTES)
        return report_error(GKV_ERR_CAPACITY,
                            "this call needs %zu bytes of scratch; the static no-alloc array holds %u "
                            "(fewer sequences, kv heads or a smaller head_dim fit)",
                            need, (unsigned)GKV_NOALLOC_SCRATCH_BYTES);

    gkv::AttendParams p{};
    p.entries = reinterpret_cast<const gkv::AttendEntry *>(d->ptr);
    p.n_seqs = n_seqs;
    p.total_units = (int32_t)units;
    p.table = block_table;
    p.table_stride = table_stride;
    p.k_pool = static_cast<const uint16_t *>(k_pages);
    p.v_pool = static_cast<const uint16_t *>(v_pages);
    p.q = static_cast<const uint16_t *>(q);
    p.out = out;
    p.status = reinterpret_cast<int32_t *>(d->ptr + off_status);
    p.counters = reinterpret_cast<int32_t *>(d->ptr + off_counters);
    p.partials = reinterpret_cast<float *>(d->ptr + off_partials);
    p.n_q = n_q;
    p.G = group;
    p.kvh = kv_heads;
    p.P = page_tokens;
    p.num_pages = num_pages;
    p.scale_log2 = scale * 1.4426950408889634f;

    CUtensorMap tmk{}, tmv{};
    if (page_tokens >= 8) {
        rc = gkv::encode_page_tensor_map(&tmk, k_pages, num_pages, kv_heads, page_tokens, head_dim);
        if (rc) return rc;
        rc = gkv::encode_page_tensor_map(&tmv, v_pages, num_pages, kv_heads, page_tokens, head_dim);
        if (rc) return rc;
    }
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(d->ptr, entries, sizeof(gkv::AttendEntry) * n_seqs,
                                    cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess)  // status word and merge counters start at zero
        e = cudaMemsetAsync(d->ptr + off_status, 0, off_partials - off_status, st);
    if (e == cudaSuccess) e = gkv::launch_attend(p, &tmk, &tmv, head_dim, grid, st);
    if (e != cudaSuccess)
        return report_error(GKV_ERR_CUDA, "gkv_attend_noalloc: %s", cudaGetErrorString(e));
    return GKV_OK;
}
