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
// every K/V tile it stages feeds all G heads.  Warp roles:
//   warps 0-3  softmax: thread r owns row r.  It reads its S row from tensor
//              memory, applies the causal mask and the online softmax (exp2
//              domain), writes P (fp16) to shared memory for the P.V MMA.
//              The running max is raised only when it grows by more than
//              2^8; only then is that row of O rescaled in tensor memory.
//   warp 4     TMA loads of K tiles (64 keys; box = one page's rows) into an
//              NS-stage ring.
//   warp 5     TMA loads of V tiles into their own NS-stage ring.
//   warp 6     owns tensor memory; one thread issues S = Q K^T
//              (tcgen05.mma M=128, N=64) into a double-buffered S, and
//              O += P V (N = dh, V read MN-major) into the fp32 O
//              accumulator that stays in tensor memory for the whole loop.
// Q is staged once in shared memory (128B swizzle, K-major); P is double
// buffered, so the softmax of tile j overlaps P.V of tile j-1 and Q K^T of
// tile j+1 on the tensor core.  Completion flows through mbarriers:
// tcgen05.commit for tensor-core work, TMA transaction counts for loads.
// Every wait is bounded; a timeout raises the device status word.
#include <cuda_fp16.h>

#include "gkv_kernels.cuh"
#include "gkv_ptx.cuh"

namespace gkv {
namespace {

using namespace ptx;

constexpr int kSoftmaxWarps = 4;
constexpr int kChunkThreads = (kSoftmaxWarps + 3) * 32;
constexpr int kKWarp = 4, kVWarp = 5, kMmaWarp = 6;
constexpr int kChunkRows = 128;  // tcgen05 M
constexpr int kChunkKeys = 64;   // keys per tile (tcgen05 N of QK^T)
constexpr uint32_t kTmemMaxCols = 512;  // tensor memory columns per SM

template <int DH>
struct ChunkCfg {
    static constexpr int NCB = DH / 64;
    static constexpr int NS = DH >= 256 ? 2 : (DH >= 128 ? 3 : 4);  // K and V ring stages
    static constexpr int Q_BYTES = kChunkRows * DH * 2;
    static constexpr int KT_BYTES = kChunkKeys * DH * 2;
    static constexpr int P_BYTES = kChunkRows * kChunkKeys * 2;
    static constexpr int OFF_K = Q_BYTES;
    static constexpr int OFF_V = OFF_K + NS * KT_BYTES;
    static constexpr int OFF_P = OFF_V + NS * KT_BYTES;
    static constexpr int OFF_BAR = OFF_P + 2 * P_BYTES;
    static constexpr int NBARS = 4 * NS + 8;
    static constexpr int SMEM = OFF_BAR + NBARS * 8 + 16;
    static constexpr uint32_t O_COL = 2 * kChunkKeys;
    // S[2] + O columns, rounded up to the power of two tcgen05.alloc takes
    static constexpr uint32_t TMEM_COLS = O_COL + DH <= 256 ? 256 : 512;
    static_assert(O_COL + DH <= TMEM_COLS, "S and O fit tensor memory");
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
    constexpr int TK = kChunkKeys, M = kChunkRows, NS = C::NS;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sQ = smem;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::OFF_BAR);
    uint64_t *k_full = bars;              // [NS] TMA -> MMA
    uint64_t *k_empty = bars + NS;        // [NS] MMA commit -> K loader
    uint64_t *v_full = bars + 2 * NS;     // [NS]
    uint64_t *v_empty = bars + 3 * NS;    // [NS]
    uint64_t *s_full = bars + 4 * NS;     // [2] MMA commit -> softmax
    uint64_t *s_free = s_full + 2;        // [2] softmax warps -> MMA
    uint64_t *p_full = s_full + 4;        // [2] softmax warps -> MMA
    uint64_t *p_free = s_full + 6;        // [2] MMA commit (P.V done) -> softmax
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
    const int nt = (kend + TK - 1) / TK;

    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], kSoftmaxWarps);
            mbar_init(&p_full[i], kSoftmaxWarps);
            mbar_init(&p_free[i], 1);
        }
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
    // Q rows: row r = token t_lo + r / G, head kvh*G + r % G; padding rows zero.
    for (int i = tid; i < M * (DH / 8); i += kChunkThreads) {
        const int r = i / (DH / 8), c16 = i % (DH / 8);
        const int t = r / G, g = r - t * G, tok = t_lo + t;
        uint4 val = make_uint4(0u, 0u, 0u, 0u);
        if (t < p.qtok && tok < t_hi)
            val = *reinterpret_cast<const uint4 *>(
                p.q + (((int64_t)b * p.n_q + tok) * nH + kvh * G + g) * DH + c16 * 8);
        *reinterpret_cast<uint4 *>(sQ + ((c16 >> 3) * M + r) * 128 + (((c16 & 7) ^ (r & 7)) << 4)) =
            val;
    }
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == kKWarp || warp == kVWarp) {
        // ============================================ TMA producers (lane 0)
        if (lane == 0) {
            const bool is_k = warp == kKWarp;
            const CUtensorMap *map = is_k ? &tmk : &tmv;
            uint64_t *full = is_k ? k_full : v_full;
            uint64_t *empty = is_k ? k_empty : v_empty;
            uint8_t *ring = smem + (is_k ? C::OFF_K : C::OFF_V);
            const int lP = __ffs(p.P) - 1;
            const int bh = min(p.P, TK);
            const int32_t *trow = p.table + (int64_t)e.seq_id * p.table_stride;
            for (int j = 0; j < nt; ++j) {
                const int s = j % NS;
                if (j >= NS && !mbar_wait(&empty[s], ((j / NS) - 1) & 1, abort_flag, p.status)) break;
                const int t0 = j * TK;
                const int ngroups = (min(TK, kend - t0) + bh - 1) / bh;
                mbar_expect_tx(&full[s], (uint32_t)(ngroups * bh * DH * 2));
                for (int g = 0; g < ngroups; ++g) {
                    const int tg = t0 + g * bh;
                    int pid = __ldg(trow + (tg >> lP));
                    if (pid < 0 || pid >= p.num_pages) {
                        atomicOr(p.status, DEV_ERR_BAD_PAGE);
                        pid = 0;
                    }
                    const int row0 = (pid * KVH + kvh) * p.P + (tg & (p.P - 1));
#pragma unroll
                    for (int cb = 0; cb < C::NCB; ++cb)
                        tma_load_2d(smem_u32(ring + s * C::KT_BYTES) + (uint32_t)(cb * TK * 128 + g * bh * 128),
                                    map, cb * 64, row0, &full[s]);
                }
            }
        }
    } else if (warp == kMmaWarp) {
        // ============================================ MMA issue (lane 0)
        if (lane == 0) {
            constexpr uint32_t IDESC_QK = umma_idesc_f16(M, TK, 0);
            constexpr uint32_t IDESC_PV = umma_idesc_f16(M, DH, 1);
            auto issue_pv = [&](int i) -> bool {
                if (!mbar_wait(&p_full[i & 1], (i >> 1) & 1, abort_flag, p.status)) return false;
                if (!mbar_wait(&v_full[i % NS], (i / NS) & 1, abort_flag, p.status)) return false;
                tc_fence_after();
                const uint32_t sV = smem_u32(smem + C::OFF_V + (i % NS) * C::KT_BYTES);
                const uint32_t sP = smem_u32(smem + C::OFF_P + (i & 1) * C::P_BYTES);
#pragma unroll
                for (int kk = 0; kk < TK / 16; ++kk) {
                    const uint64_t a = umma_desc_sw128(sP + kk * 32, 16, 1024);
                    // V is MN-major: 64-column blocks TK*128 bytes apart (LBO),
                    // 8-key groups 1024 bytes apart (SBO).
                    const uint64_t bd = umma_desc_sw128(sV + kk * 16 * 128, TK * 128, 1024);
                    umma_f16(tmem + C::O_COL, a, bd, IDESC_PV, (i > 0 || kk > 0) ? 1u : 0u);
                }
                umma_commit(&p_free[i & 1]);
                umma_commit(&v_empty[i % NS]);
                return true;
            };
            bool ok = true;
            for (int j = 0; j < nt && ok; ++j) {
                ok = mbar_wait(&k_full[j % NS], (j / NS) & 1, abort_flag, p.status) &&
                     (j < 2 || mbar_wait(&s_free[j & 1], ((j - 2) >> 1) & 1, abort_flag, p.status));
                if (!ok) break;
                tc_fence_after();
                const uint32_t sK = smem_u32(smem + C::OFF_K + (j % NS) * C::KT_BYTES);
#pragma unroll
                for (int ks = 0; ks < DH / 16; ++ks) {
                    const uint64_t a =
                        umma_desc_sw128(smem_u32(sQ) + (ks >> 2) * M * 128 + (ks & 3) * 32, 16, 1024);
                    const uint64_t bd = umma_desc_sw128(sK + (ks >> 2) * TK * 128 + (ks & 3) * 32, 16, 1024);
                    umma_f16(tmem + (uint32_t)((j & 1) * TK), a, bd, IDESC_QK, ks > 0);
                }
                umma_commit(&s_full[j & 1]);
                umma_commit(&k_empty[j % NS]);
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
        float m_ref = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nt; ++j) {
            const int sb = j & 1;
            if (!mbar_wait(&s_full[sb], (j >> 1) & 1, abort_flag, p.status)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float sa[32], sc[32];  // keys t0..t0+31 and t0+32..t0+63
            tmem_ld32(tmem_row + (uint32_t)(sb * TK), sa);
            tmem_ld32(tmem_row + (uint32_t)(sb * TK + 32), sc);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_free[sb]);

            const int t0 = j * TK;
            const bool masked = t0 + TK - 1 > all_visible;
            float mt = -INFINITY;
#pragma unroll
            for (int c = 0; c < 32; ++c) {
                float va = sa[c] * p.scale_log2, vc = sc[c] * p.scale_log2;
                if (masked) {
                    if (t0 + c > lim) va = -INFINITY;
                    if (t0 + 32 + c > lim) vc = -INFINITY;
                }
                sa[c] = va;
                sc[c] = vc;
                mt = fmaxf(mt, fmaxf(va, vc));
            }
            const float m_new = fmaxf(m_ref, mt);
            const bool raise = m_new > m_ref + 8.f;  // lazy: keep m_ref unless it grew by > 2^8
            float factor = 1.f;
            if (raise) {
                factor = m_ref == -INFINITY ? 0.f : fast_exp2(m_ref - m_new);
                m_ref = m_new;
            }
            const float mu = m_ref == -INFINITY ? 0.f : m_ref;
            if (j >= 1 && __any_sync(0xffffffffu, raise)) {
                // O rows move to the new max: wait for P.V of tile j-1 first.
                if (!mbar_wait(&p_free[(j - 1) & 1], ((j - 1) >> 1) & 1, abort_flag, p.status)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
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
            // P buffer sb was read by P.V of tile j-2.
            if (j >= 2 && !mbar_wait(&p_free[sb], ((j - 2) >> 1) & 1, abort_flag, p.status)) {
                ok = false;
                break;
            }
            uint8_t *sP = smem + C::OFF_P + sb * C::P_BYTES;
            float ps = 0.f;
#pragma unroll
            for (int ch = 0; ch < TK / 8; ++ch) {
                uint32_t w4[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int c = (ch & 3) * 8 + 2 * u;
                    const float x0 = ch < 4 ? sa[c] : sc[c];
                    const float x1 = ch < 4 ? sa[c + 1] : sc[c + 1];
                    const float a0 = fast_exp2(x0 - mu), a1 = fast_exp2(x1 - mu);
                    ps += a0 + a1;
                    w4[u] = pack_half2(a0, a1);
                }
                *reinterpret_cast<uint4 *>(sP + r * 128 + ((ch ^ (r & 7)) << 4)) =
                    make_uint4(w4[0], w4[1], w4[2], w4[3]);
            }
            l = l * factor + ps;
            const int nkeys = min(TK, kend - t0);
            if (nkeys < TK) {
                // last tile: rows past the block's end may hold stale data;
                // P is 0 there, zero this warp's share of V too so 0*V stays 0.
                if (!mbar_wait(&v_full[j % NS], (j / NS) & 1, abort_flag, p.status)) {
                    ok = false;
                    break;
                }
                uint8_t *sV = smem + C::OFF_V + (j % NS) * C::KT_BYTES;
                for (int i = tid; i < (TK - nkeys) * (DH / 8); i += kSoftmaxWarps * 32) {
                    const int key = nkeys + i / (DH / 8), c16 = i % (DH / 8);
                    *reinterpret_cast<uint4 *>(sV + ((c16 >> 3) * TK + key) * 128 +
                                               (((c16 & 7) ^ (key & 7)) << 4)) = make_uint4(0u, 0u, 0u, 0u);
                }
            }
            fence_proxy_async();  // P (and V zeroing) written by threads -> tensor core
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[sb]);
        }
        // ---- epilogue: O / l for valid rows once the last P.V is done
        if (ok && mbar_wait(&p_free[(nt - 1) & 1], ((nt - 1) >> 1) & 1, abort_flag, p.status)) {
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
