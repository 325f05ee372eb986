// gkv_chunk.cu -- causal paged attention for prefill chunks on the 5th-gen
// tensor cores (tcgen05 + tensor memory).
//
// Replaces the prefill-chunk attention of the reference: the per-page /
// carry-chained ANE flash tiles merged on the host
// (pagedFlashBatched / pagedFlashCarry / pagedFlashCarrySingle,
// LLM/src/CoreML/PagedAttention.swift:376-495, band mask :512-529) and Metal
// attn_batch_mm (LLM/metal/Kernels.metal:1935-2012).  Row s of a chunk that
// starts at p0 sees keys [0, p0 + s]; the result equals appending the rows
// one by one and running hostFlashDecode after each (Engine.swift:1220-1224).
//
// One CTA owns one (sequence, kv head, block of qtok = 128/G query tokens):
// its M = 128 rows are the qtok tokens x G query heads of the kv head, so
// every K/V tile it stages feeds all G heads.  Keys are walked in tiles of
// 128 (two 64-key halves).  Warp roles:
//   warps 0-3  softmax: thread r owns row r.  It stages its Q row in tensor
//              memory (the A operand of Q K^T), reads its S row (128 keys)
//              from tensor memory, applies the causal mask and the online
//              softmax (exp2 domain), writes P (fp16) to shared memory for
//              the P.V MMA.  The running max is raised only when it grows by
//              more than 2^8; only then is that row of O rescaled in tensor
//              memory.
//   warp 4     TMA loads of K halves (one lane per page) into a 4-stage ring whose stages are
//              stacked per 64-column block, so the two halves of a tile form
//              one 128-row operand with a uniform stride.
//   warp 5     TMA loads of V halves into a 2-stage ring.
//   warp 6     owns tensor memory; one thread issues S = Q K^T
//              (tcgen05.mma M=128, N=128) and O += P V (N = dh, V read
//              MN-major, eight K=16 steps) into the fp32 O accumulator that
//              stays in tensor memory for the whole loop.
// Measured on B200: an N=64 tcgen05.mma costs as long as an N=128 one, so Q K^T
// runs with N=128.  S is single-buffered (softmax releases it as soon as it
// has read its row), so Q K^T of tile j+1 overlaps the softmax of tile j.
// Completion flows through mbarriers: tcgen05.commit for tensor-core work,
// TMA transaction counts for loads.  Every wait is bounded; a timeout raises
// the device status word.
#include <cuda_fp16.h>

#include "gkv_kernels.cuh"
#include "gkv_ptx.cuh"

namespace gkv {
namespace {

using namespace ptx;

constexpr int kSoftmaxWarps = 4;
constexpr int kChunkThreads = (kSoftmaxWarps + 3) * 32;
constexpr int kKWarp = 4, kVWarp = 5, kMmaWarp = 6;
constexpr int kChunkRows = 128;   // tcgen05 M
constexpr int kHalf = 64;         // keys per TMA stage
constexpr int kTile = 2 * kHalf;  // keys per tile (tcgen05 N of Q K^T)
constexpr int kKStages = 4;       // K ring: two tiles of two halves
constexpr int kVStages = 2;       // V ring: the two halves of one tile
constexpr uint32_t kTmemMaxCols = 512;  // tensor memory columns per SM

template <int DH>
struct ChunkCfg {
    static constexpr int NCB = DH / 64;
    static constexpr int HALF_BYTES = kHalf * DH * 2;               // one 64-key stage
    static constexpr int KCB_STRIDE = kKStages * kHalf * 128;       // K column-block stride
    static constexpr int P_BYTES = kChunkRows * kTile * 2;          // two 64-key atoms
    static constexpr int OFF_K = 0;
    static constexpr int OFF_V = OFF_K + kKStages * HALF_BYTES;
    static constexpr int OFF_P = OFF_V + kVStages * HALF_BYTES;
    static constexpr int OFF_BAR = OFF_P + P_BYTES;
    static constexpr int NBARS = 2 + 2 + 2 + 2 + 4;
    static constexpr int SMEM = OFF_BAR + NBARS * 8 + 16;
    // Tensor memory: S (128 fp32 columns), O (dh fp32 columns), Q (dh fp16 =
    // dh/2 columns, the A operand of Q K^T).
    static constexpr uint32_t O_COL = kTile;
    static constexpr uint32_t Q_COL = O_COL + DH;
    static constexpr uint32_t USED_COLS = Q_COL + DH / 2;
    static constexpr uint32_t TMEM_COLS = USED_COLS <= 256 ? 256 : 512;
    static_assert(USED_COLS <= TMEM_COLS, "S, O and Q fit tensor memory");
    // Co-resident CTAs must not ask for more than the SM's 512 columns,
    // else tcgen05.alloc would wait for a neighbour to finish: pad the
    // shared-memory request so at most 512 / TMEM_COLS CTAs fit on an SM.
    static constexpr int MIN_SMEM = (228 * 1024) / (int)(kTmemMaxCols / TMEM_COLS + 1) + 1024;
    static constexpr int SMEM_ALLOC = SMEM + 1024 > MIN_SMEM ? SMEM + 1024 : MIN_SMEM;
    static_assert(SMEM_ALLOC <= 227 * 1024, "fits the per-CTA shared memory limit");
};

template <int DH>
__global__ void __launch_bounds__(kChunkThreads, 1)
    chunk_kernel(const __grid_constant__ ChunkParams p, const __grid_constant__ CUtensorMap tmk,
                 const __grid_constant__ CUtensorMap tmv) {
    using C = ChunkCfg<DH>;
    constexpr int M = kChunkRows, TT = kTile, H = kHalf;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::OFF_BAR);
    uint64_t *k_full = bars;        // [2] per tile slot: TMA -> MMA
    uint64_t *k_empty = bars + 2;   // [2] MMA commit -> K loader
    uint64_t *v_full = bars + 4;    // [2] per V stage
    uint64_t *v_empty = bars + 6;   // [2]
    uint64_t *s_full = bars + 8;    // MMA commit -> softmax
    uint64_t *s_free = bars + 9;    // softmax warps -> MMA
    uint64_t *p_full = bars + 10;   // softmax warps -> MMA
    uint64_t *p_free = bars + 11;   // MMA commit (P.V done) -> softmax
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + C::NBARS);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int qb = p.n_qblocks - 1 - (int)blockIdx.x;  // longest key ranges first
    const int kvh = blockIdx.y, b = blockIdx.z;
    const AttendEntry e = p.entries[b];
    const int G = p.G, KVH = p.kvh, nH = KVH * G;
    const int p0 = e.len - p.n_q;
    const int t_lo = qb * p.qtok, t_hi = min(p.n_q, t_lo + p.qtok);
    const int kend = p0 + t_hi;  // keys [0, kend) feed this block
    const int nt = (kend + TT - 1) / TT;

    if (tid == 0) {
        for (int i = 0; i < 8; ++i) mbar_init(&bars[i], 1);
        mbar_init(s_full, 1);
        mbar_init(s_free, kSoftmaxWarps);
        mbar_init(p_full, kSoftmaxWarps);
        mbar_init(p_free, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    // K/V stages start zeroed so never-loaded slots hold finite values.
    for (int i = tid; i < (C::OFF_P - C::OFF_K) / 16; i += kChunkThreads)
        reinterpret_cast<uint4 *>(smem + C::OFF_K)[i] = make_uint4(0u, 0u, 0u, 0u);
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // Q into tensor memory: softmax thread r writes row r = token t_lo + r/G,
    // head kvh*G + r%G as dh/2 packed fp16 pairs (padding rows zero).
    if (warp < kSoftmaxWarps) {
        const int t = tid / G, g = tid - t * G, tok = t_lo + t;
        const bool valid = t < p.qtok && tok < t_hi;
        const uint4 *src = reinterpret_cast<const uint4 *>(
            p.q + (((int64_t)b * p.n_q + (valid ? tok : 0)) * nH + kvh * G + g) * DH);
        const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16) + C::Q_COL;
#pragma unroll 1
        for (int c0 = 0; c0 < DH / 2; c0 += 32) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint4 x = valid ? src[c0 / 4 + i] : make_uint4(0u, 0u, 0u, 0u);
                v[4 * i] = __uint_as_float(x.x);
                v[4 * i + 1] = __uint_as_float(x.y);
                v[4 * i + 2] = __uint_as_float(x.z);
                v[4 * i + 3] = __uint_as_float(x.w);
            }
            tmem_st32(trow + c0, v);
        }
        tmem_wait_st();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    if (warp == kKWarp || warp == kVWarp) {
        // ============================================ TMA producers
        // Lane i of the warp owns page group i of a 128-key tile (group =
        // min(P, 64) keys of one page; half h = i / gph).  Every lane reads its
        // block-table entry before the slot wait, in parallel, so the table
        // latency is paid once per tile instead of once per page; then each
        // lane issues its own group's boxes.
        const bool is_k = warp == kKWarp;
        const CUtensorMap *map = is_k ? &tmk : &tmv;
        const int lP = __ffs(p.P) - 1;
        const int bh = min(p.P, H);
        const int gph = H / bh;  // page groups per 64-key half (<= 8: P >= 8)
        const int32_t *trow = p.table + (int64_t)e.seq_id * p.table_stride;
        auto half_bytes = [&](int t0) { return ((max(0, min(H, kend - t0)) + bh - 1) / bh) * bh * DH * 2; };
        const int h_lane = lane / gph, g_lane = lane % gph;
        for (int j = 0; j < nt; ++j) {
            const int t0 = j * TT;
            const int tg = t0 + h_lane * H + g_lane * bh;
            const bool mine = lane < 2 * gph && tg < kend;
            int row0 = 0;
            if (mine) {
                int pid = __ldg(trow + (tg >> lP));
                if (pid < 0 || pid >= p.num_pages) {
                    atomicOr(p.status, DEV_ERR_BAD_PAGE);
                    pid = 0;
                }
                row0 = (pid * KVH + kvh) * p.P + (tg & (p.P - 1));
            }
            bool ok = true;
            if (lane == 0) {
                if (is_k) {
                    const int slot = j & 1;
                    if (j >= 2) ok = mbar_wait(&k_empty[slot], ((j >> 1) - 1) & 1, abort_flag, p.status);
                    if (ok) mbar_expect_tx(&k_full[slot], (uint32_t)(half_bytes(t0) + half_bytes(t0 + H)));
                } else {
                    for (int h = 0; h < 2 && ok; ++h) {
                        if (j >= 1) ok = mbar_wait(&v_empty[h], (j - 1) & 1, abort_flag, p.status);
                        if (ok) mbar_expect_tx(&v_full[h], (uint32_t)half_bytes(t0 + h * H));
                    }
                }
            }
            if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
            if (mine) {
                uint8_t *dst;
                int cb_stride;
                uint64_t *bar;
                if (is_k) {
                    dst = smem + C::OFF_K + ((j & 1) * 2 + h_lane) * H * 128;
                    cb_stride = C::KCB_STRIDE;
                    bar = &k_full[j & 1];
                } else {
                    dst = smem + C::OFF_V + h_lane * C::HALF_BYTES;
                    cb_stride = H * 128;
                    bar = &v_full[h_lane];
                }
#pragma unroll
                for (int cb = 0; cb < C::NCB; ++cb)
                    tma_load_2d(smem_u32(dst) + (uint32_t)(cb * cb_stride + g_lane * bh * 128), map, cb * 64,
                                row0, bar);
            }
            __syncwarp();
        }
    } else if (warp == kMmaWarp) {
        // ============================================ MMA issue (lane 0)
        if (lane == 0) {
            constexpr uint32_t IDESC_QK = umma_idesc_f16(M, TT, 0);
            constexpr uint32_t IDESC_PV = umma_idesc_f16(M, DH, 1);
            auto issue_pv = [&](int i) -> bool {
                if (!mbar_wait(p_full, i & 1, abort_flag, p.status)) return false;
                const int halves = min(2, (kend - i * TT + H - 1) / H);
                for (int h = 0; h < halves; ++h) {
                    if (!mbar_wait(&v_full[h], i & 1, abort_flag, p.status)) return false;
                    tc_fence_after();
                    const uint32_t sV = smem_u32(smem + C::OFF_V + h * C::HALF_BYTES);
                    const uint32_t sP = smem_u32(smem + C::OFF_P + h * M * 128);
#pragma unroll
                    for (int kk = 0; kk < H / 16; ++kk) {
                        const uint64_t a = umma_desc_sw128(sP + kk * 32, 16, 1024);
                        // V is MN-major: 64-column blocks H*128 bytes apart
                        // (LBO), 8-key groups 1024 bytes apart (SBO).
                        const uint64_t bd = umma_desc_sw128(sV + kk * 16 * 128, H * 128, 1024);
                        umma_f16(tmem + C::O_COL, a, bd, IDESC_PV, (i > 0 || h > 0 || kk > 0) ? 1u : 0u);
                    }
                    umma_commit(&v_empty[h]);
                }
                if (halves < 2) umma_commit(&v_empty[1]);  // the unloaded half's stage is free too
                umma_commit(p_free);
                return true;
            };
            bool ok = true;
            for (int j = 0; j < nt && ok; ++j) {
                ok = mbar_wait(&k_full[j & 1], (j >> 1) & 1, abort_flag, p.status) &&
                     (j < 1 || mbar_wait(s_free, (j - 1) & 1, abort_flag, p.status));
                if (!ok) break;
                tc_fence_after();
                const uint32_t sK = smem_u32(smem + C::OFF_K + (j & 1) * 2 * H * 128);
#pragma unroll
                for (int ks = 0; ks < DH / 16; ++ks) {  // A = Q from tensor memory, 8 columns per K=16
                    const uint64_t bd =
                        umma_desc_sw128(sK + (ks >> 2) * C::KCB_STRIDE + (ks & 3) * 32, 16, 1024);
                    umma_f16_ts(tmem, tmem + C::Q_COL + ks * 8, bd, IDESC_QK, ks > 0);
                }
                umma_commit(s_full);
                umma_commit(&k_empty[j & 1]);
                if (j >= 1) ok = issue_pv(j - 1);
            }
            if (ok) issue_pv(nt - 1);
        }
    } else {
        // ============================================ softmax warps
        const int r = tid;
        const uint32_t tmem_row = tmem + ((uint32_t)(warp * 32) << 16);
        const int tr = r / G, tok = t_lo + tr;
        const bool row_valid = tr < p.qtok && tok < t_hi;
        const int lim = row_valid ? p0 + tok : p0;  // last visible key
        const int all_visible = p0 + t_lo;           // keys <= this are visible to every row
        const float sl = p.scale_log2;
        const float sgn = sl >= 0.f ? 1.f : -1.f;
        float m_ref = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nt; ++j) {
            if (!mbar_wait(s_full, j & 1, abort_flag, p.status)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float s[TT];  // this row's 128 raw scores
#pragma unroll
            for (int q4 = 0; q4 < TT / 32; ++q4) {
                float (&part)[32] = *reinterpret_cast<float (*)[32]>(&s[q4 * 32]);
                tmem_ld32(tmem_row + (uint32_t)(q4 * 32), part);
            }
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_free);

            const int t0 = j * TT;
            if (t0 + TT - 1 > all_visible) {
                // masked keys become -inf * sign(scale) so scale * s = -inf
#pragma unroll
                for (int c = 0; c < TT; ++c)
                    if (t0 + c > lim) s[c] = -INFINITY * sgn;
            }
            // extreme of the raw scores (max for scale > 0), 8 chains
            float ex[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) ex[u] = s[u] * sgn;
#pragma unroll
            for (int c = 8; c < TT; ++c) ex[c & 7] = fmaxf(ex[c & 7], s[c] * sgn);
            const float e01 = fmaxf(ex[0], ex[1]), e23 = fmaxf(ex[2], ex[3]);
            const float e45 = fmaxf(ex[4], ex[5]), e67 = fmaxf(ex[6], ex[7]);
            const float ext = fmaxf(fmaxf(e01, e23), fmaxf(e45, e67)) * sgn;
            const float mt = ext == -INFINITY * sgn ? -INFINITY : ext * sl;
            const float m_new = fmaxf(m_ref, mt);
            const bool raise = m_new > m_ref + 8.f;  // lazy: keep m_ref unless it grew by > 2^8
            float factor = 1.f;
            if (raise) {
                factor = m_ref == -INFINITY ? 0.f : fast_exp2(m_ref - m_new);
                m_ref = m_new;
            }
            const float nmu = m_ref == -INFINITY ? 0.f : -m_ref;
            if (j >= 1) {
                // P.V of tile j-1 must be done before P is rewritten or O rescaled.
                if (!mbar_wait(p_free, (j - 1) & 1, abort_flag, p.status)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (__any_sync(0xffffffffu, raise)) {
#pragma unroll 1
                    for (int c0 = 0; c0 < DH; c0 += 32) {
                        float o[32];
                        tmem_ld32(tmem_row + C::O_COL + c0, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] *= factor;
                        tmem_st32(tmem_row + C::O_COL + c0, o);
                    }
                    tmem_wait_st();
                }
            }
            uint8_t *sP = smem + C::OFF_P;
            float ps[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int ch = 0; ch < TT / 8; ++ch) {  // 16-byte chunks of 8 keys
                uint32_t w4[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float a0 = fast_exp2(fmaf(s[ch * 8 + 2 * u], sl, nmu));
                    const float a1 = fast_exp2(fmaf(s[ch * 8 + 2 * u + 1], sl, nmu));
                    ps[(2 * u) & 7] += a0;
                    ps[(2 * u + 1) & 7] += a1;
                    w4[u] = pack_half2(a0, a1);
                }
                // P atom (ch / 8) holds keys 64*(ch/8) .. +63 of all rows
                *reinterpret_cast<uint4 *>(sP + (ch >> 3) * M * 128 + r * 128 + (((ch & 7) ^ (r & 7)) << 4)) =
                    make_uint4(w4[0], w4[1], w4[2], w4[3]);
            }
            l = l * factor + (((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7])));
            const int nkeys = min(TT, kend - t0);
            if (nkeys < TT) {
                // last tile: rows past the block's end may hold stale data;
                // P is 0 there, zero V too so 0 * V stays 0.
                for (int h = 0; h < 2; ++h) {
                    const int valid_h = nkeys - h * H;
                    if (valid_h <= 0 || valid_h >= H) continue;
                    if (!mbar_wait(&v_full[h], j & 1, abort_flag, p.status)) {
                        ok = false;
                        break;
                    }
                    uint8_t *sV = smem + C::OFF_V + h * C::HALF_BYTES;
                    for (int i = tid; i < (H - valid_h) * (DH / 8); i += kSoftmaxWarps * 32) {
                        const int key = valid_h + i / (DH / 8), c16 = i % (DH / 8);
                        *reinterpret_cast<uint4 *>(sV + ((c16 >> 3) * H + key) * 128 +
                                                   (((c16 & 7) ^ (key & 7)) << 4)) = make_uint4(0u, 0u, 0u, 0u);
                    }
                }
                if (!ok) break;
            }
            fence_proxy_async();  // P (and V zeroing) written by threads -> tensor core
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
        }
        // ---- epilogue: O / l for valid rows once the last P.V is done
        if (ok && mbar_wait(p_free, (nt - 1) & 1, abort_flag, p.status)) {
            tc_fence_after();
            const float inv = 1.f / l;
            float *dst =
                p.out + (((int64_t)b * p.n_q + (row_valid ? tok : 0)) * nH + kvh * G + (r - tr * G)) * DH;
#pragma unroll 1
            for (int c0 = 0; c0 < DH; c0 += 32) {
                float o[32];
                tmem_ld32(tmem_row + C::O_COL + c0, o);
                tmem_wait_ld();
                if (row_valid) {
#pragma unroll
                    for (int i = 0; i < 32; i += 4)
                        *reinterpret_cast<float4 *>(dst + c0 + i) =
                            make_float4(o[i] * inv, o[i + 1] * inv, o[i + 2] * inv, o[i + 3] * inv);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

template <int DH>
cudaError_t launch_chunk_t(const ChunkParams &p, const CUtensorMap *tk, const CUtensorMap *tv,
                           cudaStream_t s) {
    auto kern = chunk_kernel<DH>;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             ChunkCfg<DH>::SMEM_ALLOC);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    dim3 grid(p.n_qblocks, p.kvh, p.n_seqs);
    kern<<<grid, kChunkThreads, ChunkCfg<DH>::SMEM_ALLOC, s>>>(p, *tk, *tv);
    return cudaGetLastError();
}

}  // namespace

bool chunk_supported(int dh, int P, int G) {
    return (dh == 64 || dh == 128 || dh == 256) && P >= 8 && G >= 1 && G <= kChunkRows;
}

cudaError_t launch_chunk(const ChunkParams &p, const CUtensorMap *tk, const CUtensorMap *tv, int dh,
                         cudaStream_t s) {
    switch (dh) {
        case 64: return launch_chunk_t<64>(p, tk, tv, s);
        case 128: return launch_chunk_t<128>(p, tk, tv, s);
        case 256: return launch_chunk_t<256>(p, tk, tv, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace gkv
