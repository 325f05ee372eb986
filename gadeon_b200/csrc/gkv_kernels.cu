// gkv_kernels.cu -- sm_100a kernels of the paged KV cache.
//
//   append_kernel   one CTA per touched page: appended rows, zero fill of a
//                   fresh page, copy-on-write / clone-tail copies, block-table
//                   entry.  Replaces PagePool.append/seed/clone's memcpys
//                   (LLM/src/CoreML/PagedAttention.swift:85-143, :199-220) and
//                   Metal kv_append / kv_append_batch
//                   (LLM/metal/Kernels.metal:1446-1457, :1726-1740).
//   attend_kernel   persistent split-K paged GQA attention for up to 16
//                   query rows per kv head (decode: G rows; MTP verify:
//                   n_q*G rows, causal among the drafts).  Replaces
//                   hostFlashDecode (PagedAttention.swift:317-366), the
//                   verify loop (LLM/src/CoreML/Engine.swift:2620-2646) and
//                   Metal attn_head / attn_batch
//                   (Kernels.metal:1339-1439, :1767-1793).
//   compact_kernel  page-strided window -> [KVH, rows, dh] (PagePool.compact,
//                   PagedAttention.swift:225-252, and tileAt, :151-161).
//
// attend_kernel design (B200):
//   * work unit = one TK-key tile of one (sequence, kv head); units are laid
//     out sequence-major, kv-head-major inside; CTA c of a persistent grid
//     takes the contiguous unit range [U*c/C, U*(c+1)/C), so every CTA moves
//     the same number of K/V bytes whatever the context lengths;
//   * a producer warp streams K and V page slabs with TMA
//     (cp.async.bulk.tensor.2d, 128B swizzle, no multicast) into an
//     NSTAGE-deep mbarrier ring; page ids come from the block table;
//   * four consumer warps: QK^T with mma.sync m16n8k16 (fp16 in, fp32
//     accumulate; the G (or n_q*G) query rows of the kv head form the M=16
//     side, so every K/V byte is read once per kv head), online softmax in
//     fp32 (exp2 domain) with the key range split across warps, P.V with the
//     head dim split across warps;
//   * an item split across CTAs writes (m, l, O) partials; the last CTA to
//     finish the item (atomic counter, no spinning) merges them with the
//     same online-softmax rule as pagedFlashBatched's host merge
//     (PagedAttention.swift:396-409).
#include <atomic>
#include <cuda_fp16.h>

#include "gkv_kernels.cuh"
#include "gkv_ptx.cuh"

namespace gkv {
namespace {

using namespace ptx;

// ------------------------------------------------------------ append
__global__ void __launch_bounds__(256)
    append_kernel(const __grid_constant__ AppendParams p, const __grid_constant__ AppendInline d) {
    // launched with programmatic stream serialization: everything below
    // waits for the previous kernel's memory; the next may start its set-up
    grid_dep_launch_dependents();
    grid_dep_wait();
    const TouchedPage tp = (p.pages ? p.pages : d.pages)[blockIdx.x];
    const AppendEntry e = (p.entries ? p.entries : d.entries)[tp.entry];
    const int P = p.P, dh = p.dh, KVH = p.kvh;
    const int CH = dh >> 3;  // 16-byte chunks per row
    const int64_t page_lo = (int64_t)tp.pidx * P;
    const int64_t row_lo = e.len_before, row_hi = (int64_t)e.len_before + e.n_new;
    const bool whole = tp.src_pid != PAGE_EXISTING;
    int s_lo, s_hi;
    if (whole) {
        s_lo = 0;
        s_hi = P;
    } else {
        s_lo = (int)(max(row_lo, page_lo) - page_lo);
        s_hi = (int)(min(row_hi, page_lo + P) - page_lo);
    }
    const int nslots = s_hi - s_lo;
    const int64_t page_elems = (int64_t)KVH * P * dh;
    const int64_t total = 2ll * KVH * nslots * CH;
    for (int64_t i = threadIdx.x; i < total; i += blockDim.x) {
        const int c = (int)(i % CH);
        int64_t rest = i / CH;
        const int slot = s_lo + (int)(rest % nslots);
        rest /= nslots;
        const int h = (int)(rest % KVH);
        const int kv = (int)(rest / KVH);
        const int64_t pos = page_lo + slot;
        const int64_t in_page = ((int64_t)h * P + slot) * dh;
        uint4 val;
        if (pos >= row_lo && pos < row_hi) {
            const int64_t r = pos - row_lo;
            const uint16_t *src = kv ? p.v_src : p.k_src;
            // head-major: entry e's block [KVH, n_new, dh] starts at row src_row0 * KVH
            const int64_t off = p.head_major ? ((int64_t)e.src_row0 * KVH + (int64_t)h * e.n_new + r) * dh
                                             : (((int64_t)e.src_row0 + r) * KVH + h) * dh;
            val = reinterpret_cast<const uint4 *>(src + off)[c];
        } else if (tp.src_pid >= 0) {
            const uint16_t *pool = kv ? p.v_pool : p.k_pool;
            val = reinterpret_cast<const uint4 *>(pool + tp.src_pid * page_elems + in_page)[c];
        } else {
            val = make_uint4(0u, 0u, 0u, 0u);
        }
        uint16_t *pool = kv ? p.v_pool : p.k_pool;
        reinterpret_cast<uint4 *>(pool + tp.pid * page_elems + in_page)[c] = val;
    }
    if (whole && threadIdx.x == 0)
        p.table[(int64_t)e.seq_id * p.table_stride + tp.pidx] = tp.pid;
}

// ------------------------------------------------------------ compact
__global__ void __launch_bounds__(256) compact_kernel(const CompactParams p) {
    const int CH = p.dh >> 3;
    const int64_t total = 2ll * p.kvh * p.rows * CH;
    const int64_t page_elems = (int64_t)p.kvh * p.P * p.dh;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % CH);
        int64_t rest = i / CH;
        const int64_t r = rest % p.rows;
        rest /= p.rows;
        const int h = (int)(rest % p.kvh);
        const int kv = (int)(rest / p.kvh);
        uint16_t *dst = (kv ? p.V : p.K) + ((int64_t)h * p.rows + r) * p.dh;
        uint4 x = make_uint4(0u, 0u, 0u, 0u);
        if (r < p.count) {
            const int64_t t = p.start + r;
            const int32_t pid = p.table[t / p.P];
            const uint16_t *src = (kv ? p.v_pool : p.k_pool) + pid * page_elems +
                                  ((int64_t)h * p.P + t % p.P) * p.dh;
            x = reinterpret_cast<const uint4 *>(src)[c];
        }
        reinterpret_cast<uint4 *>(dst)[c] = x;
    }
}

// ------------------------------------------------------------ attend
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kRows = 16;  // query rows per (sequence, kv head) item

// dh 256 runs two CTAs per SM (32-key tiles, Q read from shared memory,
// <= 204 registers): one consumer warp per SM sub-partition is latency-bound
// on its MMA / softmax chain, two independent ones keep HBM streaming.
template <int DH>
struct Cfg {
    static constexpr int CTAS = DH == 256 ? 2 : 1;         // resident CTAs per SM
    static constexpr int TK = DH >= 256 ? 32 : 64;        // keys per tile
    static constexpr int NCB = DH / 64;                    // 128-byte column blocks
    static constexpr int CH = DH / 8;                      // 16-byte chunks per row
    static constexpr int TILE_BYTES = TK * DH * 2;         // one K (or V) tile
    static constexpr int NSTAGE = DH <= 128 ? 6 : 3;
    static constexpr int KPW = TK / kConsumerWarps;        // keys per warp in QK
    static constexpr int NT_QK = KPW / 8;                  // n8 tiles per warp in QK
    static constexpr int DPW = DH / kConsumerWarps;        // head-dim columns per warp in PV
    static constexpr int NT_PV = DPW / 8;
    static constexpr bool Q_REGS = DH <= 128;              // keep Q fragments in registers
    static constexpr int TKP = TK + 8;                     // padded P row (halves)
    static constexpr int OFF_Q = NSTAGE * 2 * TILE_BYTES;
    static constexpr int OFF_P = OFF_Q + kRows * DH * 2;      // P_hi [16][TKP] fp16
    static constexpr int OFF_PL = OFF_P + kRows * TKP * 2;    // P_lo [16][TKP] fp16
    static constexpr int OFF_RED = OFF_PL + kRows * TKP * 2;
    static constexpr int OFF_BAR = OFF_RED + 2 * kConsumerWarps * kRows * 4;
    static constexpr int OFF_FLAG = OFF_BAR + (2 * NSTAGE + 1) * 8;  // full, empty, rows_done
    static constexpr int SMEM = OFF_FLAG + 16;
    static constexpr int SMEM_ALLOC = SMEM + 1024;
    static_assert(TILE_BYTES % 1024 == 0, "tiles keep 1024-byte alignment");
    static_assert(NT_PV % 2 == 0, "P.V loads n8 tiles in pairs");
    static_assert(SMEM_ALLOC <= 227 * 1024, "fits one CTA per SM");
    static_assert(CTAS * (SMEM_ALLOC + 1024) <= 228 * 1024, "CTAS CTAs fit one SM");
};

// Byte offset of (key t, 16-byte chunk c16) inside a K or V tile.  The tile
// is [group][column block][BH rows][128 B]; 128B swizzle XORs the chunk with
// the row's low three bits (every sub-tile starts 1024-byte aligned).
__device__ __forceinline__ uint32_t tile_off(int t, int c16, int lbh, int ncb) {
    const int g = t >> lbh, r = t & ((1 << lbh) - 1);
    return (uint32_t)((((g * ncb + (c16 >> 3)) << lbh) + r) * 128 + (((c16 & 7) ^ (r & 7)) << 4));
}

// Q tile: [column block][16 rows][128 B], same swizzle.
__device__ __forceinline__ uint32_t q_off(int row, int c16) {
    return (uint32_t)(((c16 >> 3) * kRows + row) * 128 + (((c16 & 7) ^ (row & 7)) << 4));
}

// ---- producer fusion helpers (SIMD/Attention.swift:72-139)
// One head row of a projection, held by a warp: lane owns elements
// [lane*E, lane*E + E), E = DH/32.  RMSNorm with weight w (Kernels.swift
// :26-37: x * (1 / sqrt(mean(x^2) + eps)) * w), then NEOX RoPE of the first
// n_rot elements with the token's cos/sin row (Kernels.swift:66-84: pair
// (i, i + n_rot/2) -> (a c - b s, a s + b c)).  Products and sums are rounded
// one at a time, as the reference writes them (no fused multiply-add).
// The sum of squares runs in the reference's order, element 0 first, one
// rounded add after another (rmsnormRows, Kernels.swift:31): the running sum
// visits the lanes in turn, each adding its E squares.  So a K row stored in
// a page matches the reference bit for bit, and so does every fp16 q row.
template <int DH>
__device__ __forceinline__ void produce_row(const float *x, const float *w, float eps, const float *cs,
                                            const float *sn, int n_rot, int lane, float (&v)[DH / 32]) {
    constexpr int E = DH / 32;
    const int half = n_rot >> 1, d0 = lane * E;  // half % E == 0 (host check)
    const bool lo = d0 < half, hi = !lo && d0 < n_rot;
    const int src = lo ? lane + half / E : (hi ? lane - half / E : lane);
    const int ti = lo ? d0 : (hi ? d0 - half : 0);
    // every global load first: one memory latency per row, not three
    float wv[E], cv[E], sv[E];
#pragma unroll
    for (int i = 0; i < E; i += 4) {
        const float4 t = __ldg(reinterpret_cast<const float4 *>(x + d0 + i));
        v[i] = t.x;
        v[i + 1] = t.y;
        v[i + 2] = t.z;
        v[i + 3] = t.w;
    }
#pragma unroll
    for (int i = 0; i < E; ++i) {
        wv[i] = __ldg(w + d0 + i);
        cv[i] = (lo || hi) ? __ldg(cs + ti + i) : 1.f;
        sv[i] = (lo || hi) ? __ldg(sn + ti + i) : 0.f;
    }
    float sq[E];
#pragma unroll
    for (int i = 0; i < E; ++i) sq[i] = __fmul_rn(v[i], v[i]);
    float ss = 0.f;
#pragma unroll 1
    for (int l = 0; l < 32; ++l) {
        if (lane == l) {
#pragma unroll
            for (int i = 0; i < E; ++i) ss = __fadd_rn(ss, sq[i]);
        }
        ss = __shfl_sync(0xffffffffu, ss, l);
    }
    const float inv = 1.f / sqrtf(ss / (float)DH + eps);
#pragma unroll
    for (int i = 0; i < E; ++i) v[i] = __fmul_rn(__fmul_rn(v[i], inv), wv[i]);
#pragma unroll
    for (int i = 0; i < E; ++i) {
        const float pv = __shfl_sync(0xffffffffu, v[i], src);
        if (lo)
            v[i] = __fsub_rn(__fmul_rn(v[i], cv[i]), __fmul_rn(pv, sv[i]));
        else if (hi)
            v[i] = __fadd_rn(__fmul_rn(pv, sv[i]), __fmul_rn(v[i], cv[i]));
    }
}

// This lane's E elements as fp16 (round to nearest even) at dst + lane*E.
template <int DH>
__device__ __forceinline__ void store_row_f16(uint16_t *dst, int lane, const float (&v)[DH / 32]) {
    constexpr int E = DH / 32;
    if constexpr (E == 8) {
        *reinterpret_cast<uint4 *>(dst + lane * E) = make_uint4(pack_half2(v[0], v[1]), pack_half2(v[2], v[3]),
                                                                pack_half2(v[4], v[5]), pack_half2(v[6], v[7]));
    } else {
        static_assert(E == 4, "producer rows of 128 or 256 elements");
        *reinterpret_cast<uint2 *>(dst + lane * E) = make_uint2(pack_half2(v[0], v[1]), pack_half2(v[2], v[3]));
    }
}

// A raw fp32 row rounded to fp16 (V of a producer step).
template <int DH>
__device__ __forceinline__ void copy_row_f16(uint16_t *dst, const float *x, int lane) {
    float v[DH / 32];
#pragma unroll
    for (int i = 0; i < DH / 32; i += 4) {
        const float4 t = __ldg(reinterpret_cast<const float4 *>(x + lane * (DH / 32) + i));
        v[i] = t.x;
        v[i + 1] = t.y;
        v[i + 2] = t.z;
        v[i + 3] = t.w;
    }
    store_row_f16<DH>(dst, lane, v);
}

// sigmoid(x) = 1 / (1 + exp(-x)) (Kernels.swift:6), the output gate.
__device__ __forceinline__ float sigmoid_gate(float x) { return 1.f / (1.f + expf(-x)); }

// Walks work units in order: unit -> (sequence b, kv head, tile j).
struct UnitWalker {
    const AttendEntry *entries;
    int n_seqs, kvh_count;
    int b, kvh, j;
    AttendEntry e;

    __device__ void seek(int u, int n_seqs) {
        int lo = 0, hi = n_seqs - 1;
        while (lo < hi) {  // last b with unit_base <= u
            const int mid = (lo + hi + 1) >> 1;
            if (entries[mid].unit_base <= u) lo = mid;
            else hi = mid - 1;
        }
        b = lo;
        e = entries[b];
        const int off = u - e.unit_base;
        kvh = off / e.ntiles;
        j = off - kvh * e.ntiles;
    }
    __device__ void next() {
        if (++j < e.ntiles) return;
        j = 0;
        if (++kvh < kvh_count) return;
        kvh = 0;
        if (++b < n_seqs) e = entries[b];
    }
};

__device__ __forceinline__ int cta_of_unit(int64_t u, int64_t units, int64_t ctas) {
    return (int)(((u + 1) * ctas - 1) / units);
}

template <int DH, bool TMA, bool FUSED, bool PROD>
__global__ void __launch_bounds__(kThreads, Cfg<DH>::CTAS)
    attend_kernel(const __grid_constant__ AttendParams p, const __grid_constant__ CUtensorMap tmk,
                  const __grid_constant__ CUtensorMap tmv, const __grid_constant__ InlineDesc d) {
    using C = Cfg<DH>;
    constexpr int TK = C::TK, NSTAGE = C::NSTAGE;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::OFF_BAR);
    uint64_t *empty = full + NSTAGE;
    uint64_t *rows_done = empty + NSTAGE;  // fused append rows stored (consumers -> producer)
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + C::OFF_FLAG);
    volatile int *merge_flag = abort_flag + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const int64_t U = p.total_units, NC = gridDim.x;
    const int u_begin = (int)(U * blockIdx.x / NC);
    const int u_end = (int)(U * (blockIdx.x + 1) / NC);

    // The next launch in the stream may place its CTAs on SMs this grid
    // leaves; it waits for this grid's memory before touching any of it.
    grid_dep_launch_dependents();
    if (threadIdx.x == 0) {
        for (int s = 0; s < NSTAGE; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        mbar_init(rows_done, kConsumerWarps * 32);
        *abort_flag = 0;
        *merge_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    // From here on the kernel reads and writes memory that earlier work in
    // the stream produced (descriptor, block table, pages, q, scratch).
    grid_dep_wait();
    if (u_begin >= u_end) return;
    // Stage buffers are not cleared: a key row the producer did not load
    // (past the sequence end) is masked to -inf in S, and its V row is
    // zeroed before P.V, so stale or uninitialised shared memory never
    // reaches the output.

    const AttendEntry *entries = p.entries ? p.entries : d.entries;
    const FusedTail *tails = p.tails ? p.tails : d.tails;
    const int lP = __ffs(p.P) - 1;
    const int lbh = TMA ? min(lP, __ffs(TK) - 1) : (__ffs(TK) - 1);  // log2 rows per tile group
    const int KVH = p.kvh;
    UnitWalker w{entries, p.n_seqs, KVH, 0, 0, 0, {}};
    w.seek(u_begin, p.n_seqs);

    if (warp == kConsumerWarps) {
        // ================================================= producer warp
        int stage = 0;
        uint32_t phase = 0;
        for (int u = u_begin; u < u_end; ++u, w.next()) {
            const int t0 = w.j * TK;
            const int nkeys = min(TK, w.e.len - t0);
            const int32_t *trow = p.table + (int64_t)w.e.seq_id * p.table_stride;
            uint8_t *sK = smem + stage * 2 * C::TILE_BYTES;
            uint8_t *sV = sK + C::TILE_BYTES;
            if constexpr (TMA) {
                const int ngroups = (nkeys + (1 << lbh) - 1) >> lbh;
                // fused append: a tile holding new rows (positions >= len -
                // n_q) takes their pages' ids from the descriptor, since the
                // table entry of a fresh page may be written by another CTA's
                // prologue
                const bool fuse_here = FUSED && t0 + TK > w.e.len - p.n_q;
                FusedTail ft{};
                if constexpr (FUSED) {
                    if (fuse_here) ft = tails[w.b];
                }
                int row0 = 0;
                if (lane < ngroups) {  // table read before the wait hides its latency
                    const int tg = t0 + (lane << lbh);
                    int pid;
                    if (fuse_here && (tg >> lP) == ft.pidx[0]) pid = ft.pid[0];
                    else if (fuse_here && (tg >> lP) == ft.pidx[1]) pid = ft.pid[1];
                    else pid = __ldg(trow + (tg >> lP));
                    if (pid < 0 || pid >= p.num_pages) {
                        atomicOr(p.status, DEV_ERR_BAD_PAGE);
                        pid = 0;
                    }
                    row0 = (pid * KVH + w.kvh) * p.P + (tg & (p.P - 1));
                }
                if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status)) break;
                // the consumers store this CTA's new rows (and zero fresh
                // pages) while the ring fills; only a tile holding new rows
                // waits for those stores
                if (fuse_here && !mbar_wait(rows_done, 0, abort_flag, p.status)) break;
                if (lane == 0)
                    mbar_expect_tx(&full[stage], (uint32_t)(ngroups << lbh) * DH * 2 * 2);
                __syncwarp();
                if (lane < ngroups) {
#pragma unroll
                    for (int cb = 0; cb < C::NCB; ++cb) {
                        const uint32_t off = (uint32_t)((lane * C::NCB + cb) << lbh) * 128;
                        tma_load_2d(smem_u32(sK) + off, &tmk, cb * 64, row0, &full[stage]);
                        tma_load_2d(smem_u32(sV) + off, &tmv, cb * 64, row0, &full[stage]);
                    }
                }
            } else {
                if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status)) break;
                const int64_t page_elems = (int64_t)KVH * p.P * DH;
                for (int i = lane; i < nkeys * C::CH; i += 32) {
                    const int t = i / C::CH, c16 = i - t * C::CH;
                    const int pos = t0 + t;
                    int pid = __ldg(trow + (pos >> lP));
                    if (pid < 0 || pid >= p.num_pages) {
                        atomicOr(p.status, DEV_ERR_BAD_PAGE);
                        pid = 0;
                    }
                    const int64_t src =
                        pid * page_elems + ((int64_t)w.kvh * p.P + (pos & (p.P - 1))) * DH + c16 * 8;
                    const uint32_t off = tile_off(t, c16, lbh, C::NCB);
                    cp_async16(smem_u32(sK) + off, p.k_pool + src);
                    cp_async16(smem_u32(sV) + off, p.v_pool + src);
                }
                cp_async_wait_all();
                __syncwarp();
                if (lane == 0) mbar_arrive(&full[stage]);
            }
            if (++stage == NSTAGE) {
                stage = 0;
                phase ^= 1;
            }
        }
        return;
    }

    // ===================================================== consumer warps
    const int tid = threadIdx.x;  // 0..127
    uint8_t *sQ = smem + C::OFF_Q;
    __half *sP = reinterpret_cast<__half *>(smem + C::OFF_P);
    __half *sPl = reinterpret_cast<__half *>(smem + C::OFF_PL);
    float *red_max = reinterpret_cast<float *>(smem + C::OFF_RED);
    float *red_sum = red_max + kConsumerWarps * kRows;
    const int G = p.G, R = p.n_q * p.G, nH = KVH * p.G;
    const int lr = lane >> 2;  // fragment row (and row + 8)
    const int lc = 2 * (lane & 3);
    const int64_t pf = attend_partial_floats(DH);

    float o[C::NT_PV][4];
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    uint32_t qa[C::Q_REGS ? DH / 16 : 1][4];
    int stage = 0;
    uint32_t phase = 0;
    bool item_start = true;
    // Causal limits of this thread's two fragment rows: key t is visible to
    // row r iff t <= len - n_q + r / G (padding rows use the last real row).
    const int rq0 = min(lr, R - 1) / G, rq1 = min(lr + 8, R - 1) / G;
    // Up to 8 query rows (decode: G rows): P_lo of row r rides in the unused
    // row r + 8 of the same MMA, so P_hi.V and P_lo.V cost one MMA; rows
    // r and r + 8 of O are added at the end.  16 rows (MTP verify) run a
    // second MMA over a P_lo tile.
    const bool stack = R <= 8;

    if constexpr (FUSED) {
        // Fused append, while the producer's first loads are in flight: for
        // every key tile of this CTA that holds new rows (positions len-n_q ..
        // len-1, the last one or two tiles of an item), write that kv head's
        // rows; for a fresh page whose first row lies in the tile, zero its
        // rows past the sequence end (PagePool.zeroPage) and record its
        // table entry.  Each row has exactly one writer.  Then fence the
        // stores against the TMA reads of those tiles.
        UnitWalker a = w;
        int u = u_begin, n_own = 0;
        while (u < u_end) {
            const int item_first = a.e.unit_base + a.kvh * a.e.ntiles;
            const int item_last = item_first + a.e.ntiles - 1;
            const int len = a.e.len, p0 = len - p.n_q;  // first new position
            const FusedTail ft = tails[a.b];
            for (int jj = p0 / TK; jj <= (len - 1) / TK; ++jj) {
                if (item_first + jj < u_begin || item_first + jj >= u_end) continue;  // another CTA's tile
                const int t_lo = max(p0, jj * TK), t_hi = min(len, jj * TK + TK);   // new rows here
#pragma unroll
                for (int s = 0; s < 2; ++s) {
                    if (ft.pidx[s] < 0) continue;
                    const int pg = ft.pidx[s] * p.P;  // the page's first position
                    const int64_t slab = ((int64_t)ft.pid[s] * KVH + a.kvh) * p.P * DH;
                    uint4 *kd = reinterpret_cast<uint4 *>(p.k_pool_w + slab);
                    uint4 *vd = reinterpret_cast<uint4 *>(p.v_pool_w + slab);
                    const int r_lo = max(t_lo, pg), r_hi = min(t_hi, pg + p.P);
                    if constexpr (PROD) {
                        // one warp builds each new K/V row from the raw
                        // projections (rows round-robin over the warps)
                        for (int pos = r_lo; pos < r_hi; ++pos, ++n_own) {
                            if (warp != n_own % kConsumerWarps) continue;
                            const int r = pos - p0;
                            const int64_t tok = (int64_t)a.b * p.n_q + r;
                            const int64_t row = tok * KVH + a.kvh;
                            const int hr = p.prod.n_rot >> 1;
                            float kv[DH / 32];
                            produce_row<DH>(p.prod.k_raw + row * DH, p.prod.k_norm, p.prod.eps,
                                            p.prod.rope_cos + tok * hr, p.prod.rope_sin + tok * hr, p.prod.n_rot,
                                            lane, kv);
                            store_row_f16<DH>(p.k_pool_w + slab + (int64_t)(pos - pg) * DH, lane, kv);
                            copy_row_f16<DH>(p.v_pool_w + slab + (int64_t)(pos - pg) * DH, p.prod.v_raw + row * DH,
                                             lane);
                        }
                    } else {
                        for (int i = tid; i < (r_hi - r_lo) * C::CH; i += 128) {
                            const int pos = r_lo + i / C::CH, c = i % C::CH;
                            const int64_t src =
                                (p.head_major ? ((int64_t)a.b * KVH + a.kvh) * p.n_q + (pos - p0)
                                              : ((int64_t)a.b * p.n_q + (pos - p0)) * KVH + a.kvh) * C::CH + c;
                            kd[(pos - pg) * C::CH + c] = reinterpret_cast<const uint4 *>(p.k_new)[src];
                            vd[(pos - pg) * C::CH + c] = reinterpret_cast<const uint4 *>(p.v_new)[src];
                        }
                    }
                    if (ft.fresh[s] && pg >= jj * TK && pg < jj * TK + TK) {
                        for (int i = tid; i < (pg + p.P - len) * C::CH; i += 128) {  // rows past the end
                            kd[(len - pg) * C::CH + i] = make_uint4(0u, 0u, 0u, 0u);
                            vd[(len - pg) * C::CH + i] = make_uint4(0u, 0u, 0u, 0u);
                        }
                        if (a.kvh == 0 && tid == 0)
                            p.table_w[(int64_t)a.e.seq_id * p.table_stride + ft.pidx[s]] = ft.pid[s];
                    }
                }
            }
            // next item
            u = item_last + 1;
            a.j = a.e.ntiles - 1;
            a.next();
        }
        fence_proxy_async_global();
        mbar_arrive(rows_done);
    }

    for (int u = u_begin; u < u_end; ++u) {
        const int b = w.b, kvh = w.kvh, j = w.j, len = w.e.len;
        if (item_start) {
            consumer_sync();  // earlier readers of sQ are done
            if constexpr (PROD) {
                // q rows from the raw q|gate projection: warp w builds rows
                // w, w+4, ... (RMSNorm + RoPE), lane l its DH/32 elements
                constexpr int E = DH / 32;
                const int hr = p.prod.n_rot >> 1;
                for (int row = warp; row < kRows; row += kConsumerWarps) {
                    float qv[E];
                    if (row < R) {
                        const int s = row / G, g = row - s * G;
                        const int64_t tok = (int64_t)b * p.n_q + s;
                        produce_row<DH>(p.prod.q_gate + (tok * nH + kvh * G + g) * (2 * DH), p.prod.q_norm,
                                        p.prod.eps, p.prod.rope_cos + tok * hr, p.prod.rope_sin + tok * hr,
                                        p.prod.n_rot, lane, qv);
                    } else {
#pragma unroll
                        for (int i = 0; i < E; ++i) qv[i] = 0.f;
                    }
                    uint8_t *dst = sQ + q_off(row, lane * E / 8) + (lane * E % 8) * 2;
                    if constexpr (E == 8)
                        *reinterpret_cast<uint4 *>(dst) = make_uint4(pack_half2(qv[0], qv[1]), pack_half2(qv[2], qv[3]),
                                                                     pack_half2(qv[4], qv[5]), pack_half2(qv[6], qv[7]));
                    else
                        *reinterpret_cast<uint2 *>(dst) = make_uint2(pack_half2(qv[0], qv[1]), pack_half2(qv[2], qv[3]));
                }
            } else {
                for (int i = tid; i < kRows * C::CH; i += 128) {
                    const int row = i / C::CH, c16 = i - row * C::CH;
                    uint4 val = make_uint4(0u, 0u, 0u, 0u);
                    if (row < R) {
                        const int s = row / G, g = row - s * G;
                        const uint16_t *src =
                            p.q + qo_row(p.head_major, b, s, kvh, g, p.n_q, KVH, G) * DH + c16 * 8;
                        val = *reinterpret_cast<const uint4 *>(src);
                    }
                    *reinterpret_cast<uint4 *>(sQ + q_off(row, c16)) = val;
                }
            }
            consumer_sync();
            if constexpr (C::Q_REGS) {
#pragma unroll
                for (int ks = 0; ks < DH / 16; ++ks) {
                    const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
                    const int c16 = 2 * ks + (lane >> 4);
                    ldsm_x4(smem_u32(sQ) + q_off(row, c16), qa[ks][0], qa[ks][1], qa[ks][2],
                            qa[ks][3]);
                }
            }
#pragma unroll
            for (int n = 0; n < C::NT_PV; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
            m0 = m1 = -INFINITY;
            l0 = l1 = 0.f;
        }
        const int t0 = j * TK;
        const int nkeys = min(TK, len - t0);
        uint8_t *sK = smem + stage * 2 * C::TILE_BYTES;
        uint8_t *sV = sK + C::TILE_BYTES;
        if (!mbar_wait(&full[stage], phase, abort_flag, p.status)) break;

        // Rows past the sequence end may hold stale or other sequences'
        // data; zero them in V so p = 0 never meets a non-finite value.
        const bool partial = nkeys < TK;
        if (partial) {
            for (int i = tid; i < (TK - nkeys) * C::CH; i += 128) {
                const int t = nkeys + i / C::CH, c16 = i % C::CH;
                *reinterpret_cast<uint4 *>(sV + tile_off(t, c16, lbh, C::NCB)) =
                    make_uint4(0u, 0u, 0u, 0u);
            }
        }

        // ---- S = Q K^T for this warp's KPW keys
        float s[C::NT_QK][4];
#pragma unroll
        for (int n = 0; n < C::NT_QK; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < DH / 16; ++ks) {
            uint32_t a0, a1, a2, a3;
            if constexpr (C::Q_REGS) {
                a0 = qa[ks][0];
                a1 = qa[ks][1];
                a2 = qa[ks][2];
                a3 = qa[ks][3];
            } else {
                const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
                ldsm_x4(smem_u32(sQ) + q_off(row, 2 * ks + (lane >> 4)), a0, a1, a2, a3);
            }
            if constexpr (C::NT_QK >= 2) {
#pragma unroll
                for (int np = 0; np < C::NT_QK / 2; ++np) {
                    const int key = warp * C::KPW + np * 16 + (lane & 7) + ((lane >> 4) << 3);
                    const int c16 = 2 * ks + ((lane >> 3) & 1);
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4(smem_u32(sK) + tile_off(key, c16, lbh, C::NCB), b0, b1, b2, b3);
                    mma16816(s[2 * np], a0, a1, a2, a3, b0, b1);
                    mma16816(s[2 * np + 1], a0, a1, a2, a3, b2, b3);
                }
            } else {
                const int key = warp * C::KPW + (lane & 7);
                const int c16 = 2 * ks + ((lane >> 3) & 1);
                uint32_t b0, b1;
                ldsm_x2(smem_u32(sK) + tile_off(key, c16, lbh, C::NCB), b0, b1);
                mma16816(s[0], a0, a1, a2, a3, b0, b1);
            }
        }

        // ---- scale, mask, online softmax (exp2 domain)
        const int lim = len - p.n_q;  // keys <= lim are visible to every row
        const bool masked = t0 + TK - 1 > lim;
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int n = 0; n < C::NT_QK; ++n) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                float v = s[n][e] * p.scale_log2;
                if (masked) {
                    const int key = t0 + warp * C::KPW + n * 8 + lc + (e & 1);
                    const int lmt = lim + ((e >> 1) ? rq1 : rq0);
                    v = key <= lmt ? v : -INFINITY;
                }
                s[n][e] = v;
            }
            mx0 = fmaxf(mx0, fmaxf(s[n][0], s[n][1]));
            mx1 = fmaxf(mx1, fmaxf(s[n][2], s[n][3]));
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        if ((lane & 3) == 0) {
            red_max[warp * kRows + lr] = mx0;
            red_max[warp * kRows + lr + 8] = mx1;
        }
        consumer_sync();
        float tm0 = red_max[lr], tm1 = red_max[lr + 8];
#pragma unroll
        for (int ww = 1; ww < kConsumerWarps; ++ww) {
            tm0 = fmaxf(tm0, red_max[ww * kRows + lr]);
            tm1 = fmaxf(tm1, red_max[ww * kRows + lr + 8]);
        }
        const float mn0 = fmaxf(m0, tm0), mn1 = fmaxf(m1, tm1);
        const float mu0 = mn0 == -INFINITY ? 0.f : mn0;
        const float mu1 = mn1 == -INFINITY ? 0.f : mn1;
        const float c0 = fast_exp2(m0 - mu0), c1 = fast_exp2(m1 - mu1);
        m0 = mn0;
        m1 = mn1;
        float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
        for (int n = 0; n < C::NT_QK; ++n) {
            const float p0 = fast_exp2(s[n][0] - mu0), p1 = fast_exp2(s[n][1] - mu0);
            // stacked: rows r + 8 are padding, their P slots take row r's P_lo
            const float p2 = stack ? 0.f : fast_exp2(s[n][2] - mu1);
            const float p3 = stack ? 0.f : fast_exp2(s[n][3] - mu1);
            ps0 += p0 + p1;
            ps1 += p2 + p3;
            const int kb = warp * C::KPW + n * 8 + lc;
            uint32_t h01, l01, h23, l23;
            split_half2(p0, p1, h01, l01);
            *reinterpret_cast<uint32_t *>(sP + lr * C::TKP + kb) = h01;
            if (stack) {
                *reinterpret_cast<uint32_t *>(sP + (lr + 8) * C::TKP + kb) = l01;
            } else {
                split_half2(p2, p3, h23, l23);
                *reinterpret_cast<uint32_t *>(sP + (lr + 8) * C::TKP + kb) = h23;
                *reinterpret_cast<uint32_t *>(sPl + lr * C::TKP + kb) = l01;
                *reinterpret_cast<uint32_t *>(sPl + (lr + 8) * C::TKP + kb) = l23;
            }
        }
        l0 = l0 * c0 + ps0;
        l1 = l1 * c1 + ps1;
        const float c1o = stack ? c0 : c1;  // stacked: rows r + 8 hold row r's P_lo.V
#pragma unroll
        for (int n = 0; n < C::NT_PV; ++n) {
            o[n][0] *= c0;
            o[n][1] *= c0;
            o[n][2] *= c1o;
            o[n][3] *= c1o;
        }
        consumer_sync();

        // ---- O += P V for this warp's DPW head-dim columns, as P_lo.V + P_hi.V
#pragma unroll
        for (int kk = 0; kk < TK / 16; ++kk) {
            uint32_t a0, a1, a2, a3, c0, c1, c2, c3;
            {
                const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
                const int key = kk * 16 + (lane >> 4) * 8;
                ldsm_x4(smem_u32(sP + row * C::TKP + key), a0, a1, a2, a3);
                if (!stack) ldsm_x4(smem_u32(sPl + row * C::TKP + key), c0, c1, c2, c3);
            }
            const int key = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
            for (int jp = 0; jp < C::NT_PV / 2; ++jp) {
                const int c16 = (warp * C::DPW) / 8 + jp * 2 + (lane >> 4);
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(smem_u32(sV) + tile_off(key, c16, lbh, C::NCB), b0, b1, b2, b3);
                if (!stack) {
                    mma16816(o[2 * jp], c0, c1, c2, c3, b0, b1);
                    mma16816(o[2 * jp + 1], c0, c1, c2, c3, b2, b3);
                }
                mma16816(o[2 * jp], a0, a1, a2, a3, b0, b1);
                mma16816(o[2 * jp + 1], a0, a1, a2, a3, b2, b3);
            }
        }
        if (partial) fence_proxy_async();  // generic zeroing vs the next TMA write
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
        if (++stage == NSTAGE) {
            stage = 0;
            phase ^= 1;
        }

        // ---- item end: final output, or a partial for the merge
        const bool last_of_item = (j == w.e.ntiles - 1) || (u == u_end - 1);
        if (last_of_item) {
            if (stack) {  // row r's O = its P_hi.V (row r) + its P_lo.V (row r + 8)
#pragma unroll
                for (int n = 0; n < C::NT_PV; ++n) {
                    o[n][0] += o[n][2];
                    o[n][1] += o[n][3];
                }
            }
            float ls0 = l0, ls1 = l1;
            ls0 += __shfl_xor_sync(0xffffffffu, ls0, 1);
            ls0 += __shfl_xor_sync(0xffffffffu, ls0, 2);
            ls1 += __shfl_xor_sync(0xffffffffu, ls1, 1);
            ls1 += __shfl_xor_sync(0xffffffffu, ls1, 2);
            if ((lane & 3) == 0) {
                red_sum[warp * kRows + lr] = ls0;
                red_sum[warp * kRows + lr + 8] = ls1;
            }
            consumer_sync();
            float L0 = 0.f, L1 = 0.f;
#pragma unroll
            for (int ww = 0; ww < kConsumerWarps; ++ww) {
                L0 += red_sum[ww * kRows + lr];
                L1 += red_sum[ww * kRows + lr + 8];
            }
            const int item_first = w.e.unit_base + kvh * w.e.ntiles;
            const int item_last = item_first + w.e.ntiles - 1;
            const int col0 = warp * C::DPW + lc;
            if (item_first >= u_begin && item_last < u_end) {
                const float i0 = 1.f / L0, i1 = 1.f / L1;
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const int row = lr + half * 8;
                    if (row < R) {
                        const int s_ = row / G, g = row - s_ * G;
                        const int64_t orow = qo_row(p.head_major, b, s_, kvh, g, p.n_q, KVH, G);
                        const float inv = half ? i1 : i0;
#pragma unroll
                        for (int n = 0; n < C::NT_PV; ++n) {
                            float2 r2 = make_float2(o[n][2 * half] * inv, o[n][2 * half + 1] * inv);
                            if constexpr (PROD) {  // attnOut *= sigmoid(gate) (Attention.swift:133-135)
                                const float *gt = p.prod.q_gate +
                                                  (((int64_t)b * p.n_q + s_) * nH + kvh * G + g) * (2 * DH) + DH;
                                r2.x *= sigmoid_gate(__ldg(gt + col0 + n * 8));
                                r2.y *= sigmoid_gate(__ldg(gt + col0 + n * 8 + 1));
                            }
                            const int64_t at = orow * DH + col0 + n * 8;
                            if (p.out_f16)
                                *reinterpret_cast<uint32_t *>(static_cast<uint16_t *>(p.out) + at) =
                                    pack_half2(r2.x, r2.y);
                            else
                                *reinterpret_cast<float2 *>(static_cast<float *>(p.out) + at) = r2;
                        }
                    }
                }
            } else {
                const int item = b * KVH + kvh;
                float *part = p.partials + (int64_t)(item + blockIdx.x) * pf;
                if (warp == 0 && (lane & 3) == 0) {
                    part[lr] = m0;
                    part[lr + 8] = m1;
                    part[16 + lr] = L0;
                    part[16 + lr + 8] = L1;
                }
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    if (lr + half * 8 >= R) continue;  // padding rows are never merged
                    float *dst = part + 32 + (int64_t)(lr + half * 8) * DH;
#pragma unroll
                    for (int n = 0; n < C::NT_PV; ++n)
                        *reinterpret_cast<float2 *>(dst + col0 + n * 8) =
                            make_float2(o[n][2 * half], o[n][2 * half + 1]);
                }
                __threadfence();
                consumer_sync();
                const int c_first = cta_of_unit(item_first, U, NC);
                const int c_last = cta_of_unit(item_last, U, NC);
                if (tid == 0) {
                    const int prev = atomicAdd(p.counters + item, 1);
                    const int last = prev == c_last - c_first;
                    if (last) {
                        p.counters[item] = 0;  // ready for the next launch
                        __threadfence();
                    }
                    *merge_flag = last;
                }
                consumer_sync();
                if (*merge_flag) {
                    const int nparts = c_last - c_first + 1;
                    const float *base = p.partials + (int64_t)(item + c_first) * pf;
                    for (int idx = tid; idx < R * DH; idx += 128) {
                        const int row = idx / DH, d = idx - row * DH;
                        float M = -INFINITY;
                        for (int k = 0; k < nparts; ++k) M = fmaxf(M, __ldcg(base + k * pf + row));
                        const float Mu = M == -INFINITY ? 0.f : M;
                        float Ls = 0.f, Os = 0.f;
                        for (int k = 0; k < nparts; ++k) {
                            const float *pk = base + k * pf;
                            const float wk = fast_exp2(__ldcg(pk + row) - Mu);
                            Ls += __ldcg(pk + 16 + row) * wk;
                            Os += __ldcg(pk + 32 + (int64_t)row * DH + d) * wk;
                        }
                        const int s_ = row / G, g = row - s_ * G;
                        float res = Os / Ls;
                        if constexpr (PROD) {
                            const int64_t grow = ((int64_t)b * p.n_q + s_) * nH + kvh * G + g;
                            res *= sigmoid_gate(__ldg(p.prod.q_gate + grow * (2 * DH) + DH + d));
                        }
                        const int64_t at = qo_row(p.head_major, b, s_, kvh, g, p.n_q, KVH, G) * DH + d;
                        if (p.out_f16)
                            static_cast<__half *>(p.out)[at] = __float2half_rn(res);
                        else
                            static_cast<float *>(p.out)[at] = res;
                    }
                }
            }
        }
        w.next();
        item_start = w.j == 0;
    }
}

template <int DH, bool TMA, bool FUSED = false, bool PROD = false>
cudaError_t launch_attend_t(const AttendParams &p, const CUtensorMap *tk, const CUtensorMap *tv,
                            int grid, cudaStream_t s, const InlineDesc *desc) {
    auto kern = attend_kernel<DH, TMA, FUSED, PROD>;
    static std::atomic<bool> configured[64];  // per device; setting the attribute twice is harmless
    static const InlineDesc empty_desc{};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || !configured[dev].load(std::memory_order_acquire)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             Cfg<DH>::SMEM_ALLOC);
        if (e != cudaSuccess) return e;
        if (dev < 64) configured[dev].store(true, std::memory_order_release);
    }
    // Programmatic stream serialization: the launch may begin while the
    // previous kernel of the stream drains; the kernel's grid_dep_wait()
    // precedes every access to memory that kernel could have written.
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = Cfg<DH>::SMEM_ALLOC;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p, *tk, *tv, desc ? *desc : empty_desc);
}

// Failure-detection probe: one thread waits, through the same bounded wait
// every kernel uses, on an mbarrier that nothing ever arrives on.  The wait
// gives up after limit_ns, records DEV_ERR_WAIT_TIMEOUT in *status and the
// kernel returns -- no fault, no trap, no hang.
__global__ void bounded_wait_probe_kernel(int *status, uint64_t limit_ns) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
    mbar_wait_for(&bar, 0, &abort_flag, status, limit_ns);
}

}  // namespace

cudaError_t launch_bounded_wait_probe(int *status, uint64_t limit_ns, cudaStream_t s) {
    bounded_wait_probe_kernel<<<1, 1, 0, s>>>(status, limit_ns);
    return cudaGetLastError();
}

cudaError_t launch_append(const AppendParams &p, cudaStream_t s, const AppendInline *inl) {
    if (p.n_pages <= 0) return cudaSuccess;
    static const AppendInline empty_desc{};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)p.n_pages);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, append_kernel, p, inl ? *inl : empty_desc);
}

cudaError_t launch_compact(const CompactParams &p, cudaStream_t s) {
    if (p.rows <= 0) return cudaSuccess;
    const int64_t total = 2ll * p.kvh * p.rows * (p.dh / 8);
    const int64_t blocks = (total + 255) / 256;
    compact_kernel<<<(unsigned)(blocks < 65535 * 16 ? blocks : 65535 * 16), 256, 0, s>>>(p);
    return cudaGetLastError();
}

int attend_tile_keys(int dh) {
    switch (dh) {
        case 64: return Cfg<64>::TK;
        case 128: return Cfg<128>::TK;
        case 256: return Cfg<256>::TK;
        case 512: return Cfg<512>::TK;
        default: return 0;
    }
}

int attend_grid(int dh, int P, int units, int sm_count) {
    (void)P;
    int per_sm = 1;
    switch (dh) {
        case 64: per_sm = Cfg<64>::CTAS; break;
        case 128: per_sm = Cfg<128>::CTAS; break;
        case 256: per_sm = Cfg<256>::CTAS; break;
        case 512: per_sm = Cfg<512>::CTAS; break;
    }
    const int cap = sm_count * per_sm;
    return units < cap ? units : cap;
}

// dh 128 / 256 with the producer fusion: TMA (fused append or not) or the
// cp.async loader (P < 8, append done beforehand).
template <int DH>
cudaError_t launch_attend_prod(const AttendParams &p, const CUtensorMap *tk, const CUtensorMap *tv, int grid,
                               cudaStream_t s, const InlineDesc *d) {
    if (p.P < 8) return launch_attend_t<DH, false, false, true>(p, tk, tv, grid, s, d);
    return p.fused ? launch_attend_t<DH, true, true, true>(p, tk, tv, grid, s, d)
                   : launch_attend_t<DH, true, false, true>(p, tk, tv, grid, s, d);
}

// grid: n_seqs * KVH rows, 4 warps per block, one warp per row.
template <int DH>
__global__ void __launch_bounds__(128) produce_kv_kernel(const __grid_constant__ ProduceParams p) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
    if (row >= (int64_t)p.n_seqs * p.kvh) return;
    const int64_t b = row / p.kvh;
    const int hr = p.prod.n_rot >> 1;
    float kv[DH / 32];
    produce_row<DH>(p.prod.k_raw + row * DH, p.prod.k_norm, p.prod.eps, p.prod.rope_cos + b * hr,
                    p.prod.rope_sin + b * hr, p.prod.n_rot, lane, kv);
    store_row_f16<DH>(p.k_out + row * DH, lane, kv);
    copy_row_f16<DH>(p.v_out + row * DH, p.prod.v_raw + row * DH, lane);
}

bool producer_supported(int dh) { return dh == 128 || dh == 256; }

cudaError_t launch_produce_kv(const ProduceParams &p, int dh, cudaStream_t s) {
    const int64_t rows = (int64_t)p.n_seqs * p.kvh;
    if (rows <= 0) return cudaSuccess;
    const unsigned blocks = (unsigned)((rows + 3) / 4);
    if (dh == 256)
        produce_kv_kernel<256><<<blocks, 128, 0, s>>>(p);
    else if (dh == 128)
        produce_kv_kernel<128><<<blocks, 128, 0, s>>>(p);
    else
        return cudaErrorInvalidValue;
    return cudaGetLastError();
}

cudaError_t launch_attend(const AttendParams &p, const CUtensorMap *tk, const CUtensorMap *tv,
                          int dh, int grid, cudaStream_t s, const InlineDesc *d) {
    const bool tma = p.P >= 8;
    if (p.prod.q_gate) {
        if (dh == 128) return launch_attend_prod<128>(p, tk, tv, grid, s, d);
        if (dh == 256) return launch_attend_prod<256>(p, tk, tv, grid, s, d);
        return cudaErrorInvalidValue;
    }
    switch (dh) {
        case 64: return tma ? launch_attend_t<64, true>(p, tk, tv, grid, s, d)
                            : launch_attend_t<64, false>(p, tk, tv, grid, s, d);
        case 128: return tma ? (p.fused ? launch_attend_t<128, true, true>(p, tk, tv, grid, s, d)
                                        : launch_attend_t<128, true>(p, tk, tv, grid, s, d))
                             : launch_attend_t<128, false>(p, tk, tv, grid, s, d);
        case 256: return tma ? (p.fused ? launch_attend_t<256, true, true>(p, tk, tv, grid, s, d)
                                        : launch_attend_t<256, true>(p, tk, tv, grid, s, d))
                             : launch_attend_t<256, false>(p, tk, tv, grid, s, d);
        case 512: return tma ? launch_attend_t<512, true>(p, tk, tv, grid, s, d)
                             : launch_attend_t<512, false>(p, tk, tv, grid, s, d);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace gkv
